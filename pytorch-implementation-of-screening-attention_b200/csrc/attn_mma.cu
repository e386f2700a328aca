// bf16 tensor-core screening attention, head dim 64 (warp-level mma.sync
// m16n8k16, fp32 accumulation, cp.async double-buffered K/V tiles in
// XOR-swizzled shared memory).
//
// Per (b, h) the math is multiscreen/attention.py:156-196:
//   S = q^ k^T,  a = relu(1 - r (1 - S)),  alpha = a^2 m,  o = alpha v^,
//   y = TanhNorm(o).
// The tensor cores see the RAW bf16 projections (exact); the unit
// normalisation enters as fp32 per-row / per-column scales on the scores
// (S = (q.k) / (|q| |k|), alpha v^ = (alpha / |v|) v), so no rounded copy of
// q^, k^, v^ exists anywhere.
// The softmask m(rel) = (1 + cos(pi rel / w)) / 2 is evaluated without a
// per-score cos: with rel = u - v (u = j - p0 for key j, v = p - p0 for a
// query at position p, p0 the tile's first query position),
//   cos(pi (u - v)/w) = cos(pi u/w) cos(pi v/w) + sin(pi u/w) sin(pi v/w),
// so per score m = fma(c_v, c_u, fma(s_v, s_u, 1/2)) from a per-row and a
// per-column (cos, sin) pair computed once per tile with sincospif.  The
// window/causal predicate is only evaluated on tiles that straddle the
// window edge.  A warp skips the alpha/PV work of a 16x64 score block when
// no score clears the trim threshold (t = 1 - r (1 - s) <= 0 everywhere),
// and skips the block entirely when it lies outside the window.
#include "rowops.cuh"

namespace screen {
namespace {

typedef __nv_bfloat16 bf16;
constexpr int kD = 64;           // head dim of this path
constexpr int kKS = kD / 16;     // k-steps over D
constexpr int kNTO = kD / 8;     // n-tiles over D
constexpr int kCH = kD / 8;      // 16-byte chunks per row

// Copy rows [t0, t0+ROWS) of one head of a (B,T,H,D) bf16 tensor (row
// stride `rowstride` elements) into a swizzled tile; rows outside [0, Tlim)
// are zero-filled.
template <int ROWS, int NT>
__device__ __forceinline__ void load_tile(uint32_t sbase, const bf16* head0, long long rowstride,
                                          long long t0, long long Tlim, int tid) {
#pragma unroll
  for (int c = tid; c < ROWS * kCH; c += NT) {
    const int row = c / kCH, ch = c % kCH;
    const long long t = t0 + row;
    const bool ok = (t >= 0) && (t < Tlim);
    const bf16* src = head0 + (ok ? t * rowstride : 0) + ch * 8;
    cp_async16(sbase + tile_off<kD>(row, ch), src, ok);
  }
}

__device__ __forceinline__ const bf16* head_ptr(const Rows& x, int b, int h) {
  return reinterpret_cast<const bf16*>(x.p) + (long long)b * x.sb + (long long)h * kD;
}

// Unpack the bf16 A fragments of a 16 x D row block into fp32 values in the
// C-fragment layout (the two layouts coincide element for element).
__device__ __forceinline__ void frags_to_c(const uint32_t (&f)[kKS][4], float (&x)[kNTO][4]) {
#pragma unroll
  for (int kk = 0; kk < kKS; ++kk) {
    float2 t0 = unpack_bf16(f[kk][0]), t1 = unpack_bf16(f[kk][1]);
    float2 t2 = unpack_bf16(f[kk][2]), t3 = unpack_bf16(f[kk][3]);
    x[2 * kk][0] = t0.x; x[2 * kk][1] = t0.y; x[2 * kk][2] = t1.x; x[2 * kk][3] = t1.y;
    x[2 * kk + 1][0] = t2.x; x[2 * kk + 1][1] = t2.y;
    x[2 * kk + 1][2] = t3.x; x[2 * kk + 1][3] = t3.y;
  }
}

// out = inv * (acc - inv^2 (x . acc) x) for the two rows of each thread: the
// unit-normalisation Jacobian applied to acc = dL/dx^ with x^ = x * inv
// (x the raw row); rows [row0, row0+16) of the warp, written with strides.
__device__ __forceinline__ void store_norm_jacobian(const float (&acc)[kNTO][4],
                                                    const uint32_t (&xf)[kKS][4],
                                                    const float (&inv)[2], const OutRows& out,
                                                    int b, int h, long long row0, long long T,
                                                    int g, int tq) {
  float xv[kNTO][4];
  frags_to_c(xf, xv);
  float d0 = 0.f, d1 = 0.f;
#pragma unroll
  for (int n = 0; n < kNTO; ++n) {
    d0 += xv[n][0] * acc[n][0] + xv[n][1] * acc[n][1];
    d1 += xv[n][2] * acc[n][2] + xv[n][3] * acc[n][3];
  }
  d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
  d0 += __shfl_xor_sync(0xffffffffu, d0, 2);
  d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
  d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const long long t = row0 + g + hr * 8;
    if (t < T) {
      const float iv = inv[hr];
      const float c = iv * iv * (hr ? d1 : d0);
      uint32_t* o = reinterpret_cast<uint32_t*>(reinterpret_cast<bf16*>(out.p) +
                                                (long long)b * out.sb + t * out.st +
                                                (long long)h * kD);
#pragma unroll
      for (int n = 0; n < kNTO; ++n)
        o[n * 4 + tq] = pack_bf16(iv * (acc[n][2 * hr] - c * xv[n][2 * hr]),
                                  iv * (acc[n][2 * hr + 1] - c * xv[n][2 * hr + 1]));
    }
  }
}

// A fragments (16 rows x D) of a swizzled tile, rows [row0, row0+16).
__device__ __forceinline__ void load_a_frags(uint32_t sbase, int row0, int lane,
                                             uint32_t (&f)[kKS][4]) {
  const int mat = lane >> 3;
  const int row = row0 + (lane & 7) + (mat & 1) * 8;
#pragma unroll
  for (int kk = 0; kk < kKS; ++kk) {
    const int ch = 2 * kk + (mat >> 1);
    ldsm_x4(sbase + tile_off<kD>(row, ch), f[kk][0], f[kk][1], f[kk][2], f[kk][3]);
  }
}

// acc[16 x 64] += A[16 x D] * T[64 rows x D]^T   (T row-major in smem)
__device__ __forceinline__ void gemm_abt(float (&acc)[8][4], const uint32_t (&a)[kKS][4],
                                         uint32_t sbase, int lane) {
  const int mat = lane >> 3;
#pragma unroll
  for (int kk = 0; kk < kKS; ++kk) {
#pragma unroll
    for (int ntp = 0; ntp < 4; ++ntp) {
      const int row = 16 * ntp + (mat >> 1) * 8 + (lane & 7);
      const int ch = 2 * kk + (mat & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sbase + tile_off<kD>(row, ch), b0, b1, b2, b3);
      mma_bf16(acc[2 * ntp], a[kk], b0, b1);
      mma_bf16(acc[2 * ntp + 1], a[kk], b2, b3);
    }
  }
}

// acc[16 x D] += P[16 x 64] * T[64 rows x D]   (P given as C-layout fp32
// fragments, converted to bf16 A fragments; T row-major in smem)
__device__ __forceinline__ void gemm_pt(float (&acc)[kNTO][4], const float (&pc)[8][4],
                                        uint32_t sbase, int lane) {
  const int mat = lane >> 3;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16(pc[2 * kk][0], pc[2 * kk][1]);
    a[1] = pack_bf16(pc[2 * kk][2], pc[2 * kk][3]);
    a[2] = pack_bf16(pc[2 * kk + 1][0], pc[2 * kk + 1][1]);
    a[3] = pack_bf16(pc[2 * kk + 1][2], pc[2 * kk + 1][3]);
#pragma unroll
    for (int ndp = 0; ndp < kNTO / 2; ++ndp) {
      const int row = 16 * kk + (mat & 1) * 8 + (lane & 7);
      const int ch = 2 * ndp + (mat >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sbase + tile_off<kD>(row, ch), b0, b1, b2, b3);
      mma_bf16(acc[2 * ndp], a, b0, b1);
      mma_bf16(acc[2 * ndp + 1], a, b2, b3);
    }
  }
}

__device__ __forceinline__ bool block_dead(long long dlo, long long dhi, int dmax, bool causal) {
  // d = p - j ranges over [dlo, dhi] in this block
  return causal ? (dhi < 0 || dlo > dmax) : (dhi < -(long long)dmax || dlo > dmax);
}
__device__ __forceinline__ bool block_inside(long long dlo, long long dhi, int dmax, bool causal) {
  return causal ? (dlo >= 0 && dhi <= dmax) : (dlo >= -(long long)dmax && dhi <= dmax);
}
__device__ __forceinline__ bool in_window(float rel, float dmaxf, bool causal) {
  // rel = j - p
  return causal ? (rel <= 0.f && rel >= -dmaxf) : (fabsf(rel) <= dmaxf);
}

// ===========================================================================
// Forward: CTA = 128 queries (8 warps x 16 rows), key tiles of 64.
//   x = (q.k) / |k| per score, t = 1 - r + (r / |q|) x = 1 - r (1 - S),
//   alpha' = a^2 m / |v| so that o = sum_j alpha'_ij v_j = sum_j alpha_ij v^_j.
// ===========================================================================
constexpr int kFwdBM = 128, kFwdBN = 64, kFwdThreads = 256;
constexpr size_t kFwdSmem = (size_t)kFwdBM * kD * 2 + 4 * (size_t)kFwdBN * kD * 2 +
                            2 * kFwdBN * sizeof(float4) + 2 * kFwdBN * sizeof(float);

__global__ void __launch_bounds__(kFwdThreads, 2) mma_fwd_kernel(AttnShape s, FwdPtrs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + kFwdBM * kD * 2;
  const uint32_t sV = sK + 2 * kFwdBN * kD * 2;
  float4* sCol = reinterpret_cast<float4*>(smem + kFwdBM * kD * 2 + 4 * kFwdBN * kD * 2);
  float* sIk = reinterpret_cast<float*>(sCol + 2 * kFwdBN);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const long long i0 = (long long)blockIdx.x * kFwdBM;
  const bool causal = s.causal != 0;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const float dmaxf = (float)dmax;
  const long long p0 = i0 + s.q_offset;
  long long ilast = i0 + kFwdBM - 1;
  if (ilast > s.Tq - 1) ilast = s.Tq - 1;
  long long lo, hi;
  key_range(p0, ilast + s.q_offset, dmax, causal, s.Tk, lo, hi);
  const bool any = dmax >= 0 && lo <= hi;

  const bf16* qh = head_ptr(p.q, b, h);
  const bf16* kh = head_ptr(p.k, b, h);
  const bf16* vh = head_ptr(p.v, b, h);
  const long long nkb = (long long)b * s.Tk * s.H + h;  // norms index of (b, 0, h)

  load_tile<kFwdBM, kFwdThreads>(sQ, qh, p.q.st, i0, s.Tq, tid);
  const int kt0 = any ? (int)(lo / kFwdBN) : 0;
  const int kt1 = any ? (int)(hi / kFwdBN) : -1;

  // per key column: (keep, cos, sin)(pi u / w) / |v|, u = j - p0; and 1/|k|
  auto col_info = [&](int kt, int buf) {
    if (tid < kFwdBN) {
      const long long j = (long long)kt * kFwdBN + tid;
      const bool keep = j < s.Tk && !(s.kpm && s.kpm[(long long)b * s.kpm_sb + j]);
      const float u = (float)(j - p0);
      float sn, cs;
      sincospif(u / w, &sn, &cs);
      const float iv = keep ? 1.0f / p.nv[nkb + j * s.H] : 0.f;
      sCol[buf * kFwdBN + tid] = make_float4(0.5f * iv, cs * iv, sn * iv, u);
      sIk[buf * kFwdBN + tid] = keep ? 1.0f / p.nk[nkb + j * s.H] : 0.f;
    }
  };
  if (any) {
    load_tile<kFwdBN, kFwdThreads>(sK, kh, p.k.st, (long long)kt0 * kFwdBN, s.Tk, tid);
    load_tile<kFwdBN, kFwdThreads>(sV, vh, p.v.st, (long long)kt0 * kFwdBN, s.Tk, tid);
    col_info(kt0, 0);
  }
  cp_async_commit();

  // per query row: (cos, sin)(pi v / w) / 2 of v = p - p0, and r / |q|
  float crow[2], srow[2], vrow[2], rq[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int vi = warp * 16 + g + hr * 8;
    const float v = (float)vi;
    float sn, cs;
    sincospif(v / w, &sn, &cs);
    crow[hr] = 0.5f * cs;
    srow[hr] = 0.5f * sn;
    vrow[hr] = v;
    const long long i = i0 + vi;
    rq[hr] = (i < s.Tq) ? r / p.nq[((long long)b * s.Tq + i) * s.H + h] : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  uint32_t qf[kKS][4];
  load_a_frags(sQ, warp * 16, lane, qf);

  float o[kNTO][4];
#pragma unroll
  for (int n = 0; n < kNTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  unsigned long long visited = 0, live_blocks = 0;
  const long long pw0 = p0 + warp * 16;  // first query position of this warp
  const float one_minus_r = 1.0f - r;

  for (int kt = kt0; kt <= kt1; ++kt) {
    const int buf = (kt - kt0) & 1;
    if (kt < kt1) {
      const uint32_t off = (buf ^ 1) * kFwdBN * kD * 2;
      load_tile<kFwdBN, kFwdThreads>(sK + off, kh, p.k.st, (long long)(kt + 1) * kFwdBN, s.Tk,
                                     tid);
      load_tile<kFwdBN, kFwdThreads>(sV + off, vh, p.v.st, (long long)(kt + 1) * kFwdBN, s.Tk,
                                     tid);
      cp_async_commit();
      col_info(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    const long long j0 = (long long)kt * kFwdBN;
    const long long dlo = pw0 - (j0 + kFwdBN - 1), dhi = pw0 + 15 - j0;
    if (!block_dead(dlo, dhi, dmax, causal)) {
      ++visited;
      const uint32_t kb = sK + buf * kFwdBN * kD * 2, vb = sV + buf * kFwdBN * kD * 2;
      const float4* ci = sCol + buf * kFwdBN;
      const float* ik = sIk + buf * kFwdBN;
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      gemm_abt(sc, qf, kb, lane);
      float mx0 = -3.0e38f, mx1 = -3.0e38f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float ik0 = ik[n * 8 + 2 * tq], ik1 = ik[n * 8 + 2 * tq + 1];
        sc[n][0] *= ik0; sc[n][1] *= ik1; sc[n][2] *= ik0; sc[n][3] *= ik1;
        mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
      }
      const bool live = fmaf(rq[0], mx0, one_minus_r) > 0.f ||
                        fmaf(rq[1], mx1, one_minus_r) > 0.f || r <= 0.f;
      if (__any_sync(0xffffffffu, live)) {
        ++live_blocks;
        const bool inside = block_inside(dlo, dhi, dmax, causal);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hr = e >> 1;
            const float4 c = ci[n * 8 + 2 * tq + (e & 1)];
            float a = fmaxf(fmaf(rq[hr], sc[n][e], one_minus_r), 0.f);
            if (!inside && !in_window(c.w - vrow[hr], dmaxf, causal)) a = 0.f;
            const float m = fmaf(crow[hr], c.y, fmaf(srow[hr], c.z, c.x));
            sc[n][e] = a * a * m;
          }
        }
        gemm_pt(o, sc, vb, lane);
      }
    }
    __syncthreads();
  }

  // TanhNorm epilogue
  float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int n = 0; n < kNTO; ++n) {
    ss0 += o[n][0] * o[n][0] + o[n][1] * o[n][1];
    ss1 += o[n][2] * o[n][2] + o[n][3] * o[n][3];
  }
  ss0 += __shfl_xor_sync(0xffffffffu, ss0, 1);
  ss0 += __shfl_xor_sync(0xffffffffu, ss0, 2);
  ss1 += __shfl_xor_sync(0xffffffffu, ss1, 1);
  ss1 += __shfl_xor_sync(0xffffffffu, ss1, 2);
  bf16* y = reinterpret_cast<bf16*>(p.y);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const long long i = i0 + warp * 16 + g + hr * 8;
    if (i < s.Tq) {
      const float nraw = sqrtf(hr ? ss1 : ss0);
      const float sc = tanhnorm_scale(nraw, s.eps);
      const long long row = ((long long)b * s.Tq + i) * s.H + h;
      uint32_t* yr = reinterpret_cast<uint32_t*>(y + row * kD);
#pragma unroll
      for (int n = 0; n < kNTO; ++n)
        yr[n * 4 + tq] = pack_bf16(o[n][2 * hr] * sc, o[n][2 * hr + 1] * sc);
      if (tq == 0) p.no[row] = nraw;
    }
  }
  if (p.tile_stats && lane == 0) {
    atomicAdd((unsigned long long*)&p.tile_stats[0], visited);
    atomicAdd((unsigned long long*)&p.tile_stats[1], live_blocks);
  }
}

// ===========================================================================
// Backward, query side: CTA = 128 queries (8 warps), key tiles of 64.
//   dP = G v^T, dS = dP m 2a r, dq^ = sum_j dS k^_j, then the Jacobian.
//   Column scales: 1/|k| on S; m/(|v||k|) so dS'' = dP_raw m'' 2a r pairs
//   with the raw k rows.
// ===========================================================================
constexpr int kDqBM = 128, kDqBN = 64, kDqThreads = 256;
constexpr size_t kDqSmem = 3 * (size_t)kDqBM * kD * 2 + 4 * (size_t)kDqBN * kD * 2 +
                           2 * kDqBN * sizeof(float4) + 2 * kDqBN * sizeof(float);

__global__ void __launch_bounds__(kDqThreads, 1) mma_bwd_dq_kernel(AttnShape s, BwdPtrs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sG = sQ + kDqBM * kD * 2;
  const uint32_t sGl = sG + kDqBM * kD * 2;
  const uint32_t sK = sGl + kDqBM * kD * 2;
  const uint32_t sV = sK + 2 * kDqBN * kD * 2;
  float4* sCol = reinterpret_cast<float4*>(smem + 3 * kDqBM * kD * 2 + 4 * kDqBN * kD * 2);
  float* sIk = reinterpret_cast<float*>(sCol + 2 * kDqBN);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const long long i0 = (long long)blockIdx.x * kDqBM;
  const bool causal = s.causal != 0;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const float dmaxf = (float)dmax;
  const long long p0 = i0 + s.q_offset;
  long long ilast = i0 + kDqBM - 1;
  if (ilast > s.Tq - 1) ilast = s.Tq - 1;
  long long lo, hi;
  key_range(p0, ilast + s.q_offset, dmax, causal, s.Tk, lo, hi);
  const bool any = dmax >= 0 && lo <= hi;

  const bf16* qh = head_ptr(p.q, b, h);
  const bf16* kh = head_ptr(p.k, b, h);
  const bf16* vh = head_ptr(p.v, b, h);
  const bf16* gh = reinterpret_cast<const bf16*>(p.G) + ((long long)b * s.Tq * s.H + h) * kD;
  const bf16* glh = gh + (long long)s.B * s.Tq * s.H * kD;  // G_lo plane
  const long long nkb = (long long)b * s.Tk * s.H + h;

  load_tile<kDqBM, kDqThreads>(sQ, qh, p.q.st, i0, s.Tq, tid);
  load_tile<kDqBM, kDqThreads>(sG, gh, (long long)s.H * kD, i0, s.Tq, tid);
  load_tile<kDqBM, kDqThreads>(sGl, glh, (long long)s.H * kD, i0, s.Tq, tid);
  const int kt0 = any ? (int)(lo / kDqBN) : 0;
  const int kt1 = any ? (int)(hi / kDqBN) : -1;
  auto col_info = [&](int kt, int buf) {
    if (tid < kDqBN) {
      const long long j = (long long)kt * kDqBN + tid;
      const bool keep = j < s.Tk && !(s.kpm && s.kpm[(long long)b * s.kpm_sb + j]);
      const float u = (float)(j - p0);
      float sn, cs;
      sincospif(u / w, &sn, &cs);
      const float ik = keep ? 1.0f / p.nk[nkb + j * s.H] : 0.f;
      const float sc = keep ? ik / p.nv[nkb + j * s.H] : 0.f;
      sCol[buf * kDqBN + tid] = make_float4(0.5f * sc, cs * sc, sn * sc, u);
      sIk[buf * kDqBN + tid] = ik;
    }
  };
  if (any) {
    load_tile<kDqBN, kDqThreads>(sK, kh, p.k.st, (long long)kt0 * kDqBN, s.Tk, tid);
    load_tile<kDqBN, kDqThreads>(sV, vh, p.v.st, (long long)kt0 * kDqBN, s.Tk, tid);
    col_info(kt0, 0);
  }
  cp_async_commit();
  float crow[2], srow[2], vrow[2], rq[2], iq[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int vi = warp * 16 + g + hr * 8;
    const float v = (float)vi;
    float sn, cs;
    sincospif(v / w, &sn, &cs);
    crow[hr] = 0.5f * cs;
    srow[hr] = 0.5f * sn;
    vrow[hr] = v;
    const long long i = i0 + vi;
    iq[hr] = (i < s.Tq) ? 1.0f / p.nq[((long long)b * s.Tq + i) * s.H + h] : 0.f;
    rq[hr] = r * iq[hr];
  }
  cp_async_wait<0>();
  __syncthreads();
  uint32_t qf[kKS][4], gf[kKS][4];
  load_a_frags(sQ, warp * 16, lane, qf);
  load_a_frags(sG, warp * 16, lane, gf);

  float dq[kNTO][4];
#pragma unroll
  for (int n = 0; n < kNTO; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
  const long long pw0 = p0 + warp * 16;
  const float one_minus_r = 1.0f - r;
  const float two_r = 2.0f * r;

  for (int kt = kt0; kt <= kt1; ++kt) {
    const int buf = (kt - kt0) & 1;
    if (kt < kt1) {
      const uint32_t off = (buf ^ 1) * kDqBN * kD * 2;
      load_tile<kDqBN, kDqThreads>(sK + off, kh, p.k.st, (long long)(kt + 1) * kDqBN, s.Tk, tid);
      load_tile<kDqBN, kDqThreads>(sV + off, vh, p.v.st, (long long)(kt + 1) * kDqBN, s.Tk, tid);
      cp_async_commit();
      col_info(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const long long j0 = (long long)kt * kDqBN;
    const long long dlo = pw0 - (j0 + kDqBN - 1), dhi = pw0 + 15 - j0;
    if (!block_dead(dlo, dhi, dmax, causal)) {
      const uint32_t kb = sK + buf * kDqBN * kD * 2, vb = sV + buf * kDqBN * kD * 2;
      const float4* ci = sCol + buf * kDqBN;
      const float* ik = sIk + buf * kDqBN;
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      gemm_abt(sc, qf, kb, lane);
      float mx0 = -3.0e38f, mx1 = -3.0e38f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float ik0 = ik[n * 8 + 2 * tq], ik1 = ik[n * 8 + 2 * tq + 1];
        sc[n][0] *= ik0; sc[n][1] *= ik1; sc[n][2] *= ik0; sc[n][3] *= ik1;
        mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
      }
      const bool live = fmaf(rq[0], mx0, one_minus_r) > 0.f ||
                        fmaf(rq[1], mx1, one_minus_r) > 0.f || r <= 0.f;
      if (__any_sync(0xffffffffu, live)) {
        float dp[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) dp[n][0] = dp[n][1] = dp[n][2] = dp[n][3] = 0.f;
        gemm_abt(dp, gf, vb, lane);
        {
          uint32_t gl[kKS][4];
          load_a_frags(sGl, warp * 16, lane, gl);
          gemm_abt(dp, gl, vb, lane);
        }
        const bool inside = block_inside(dlo, dhi, dmax, causal);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hr = e >> 1;
            const float4 c = ci[n * 8 + 2 * tq + (e & 1)];
            float a = fmaxf(fmaf(rq[hr], sc[n][e], one_minus_r), 0.f);
            if (!inside && !in_window(c.w - vrow[hr], dmaxf, causal)) a = 0.f;
            const float m = fmaf(crow[hr], c.y, fmaf(srow[hr], c.z, c.x));
            sc[n][e] = dp[n][e] * m * a * two_r;  // dS / |k|
          }
        }
        gemm_pt(dq, sc, kb, lane);
      }
    }
    __syncthreads();
  }
  store_norm_jacobian(dq, qf, iq, p.dq, b, h, i0 + warp * 16, s.Tq, g, tq);
}

// ===========================================================================
// Backward, key side: CTA = 128 keys (8 warps x 16), query tiles of 64.
//   S^T, dP^T = v G^T, alpha, dS; dv^ += alpha^T G, dk^ += dS^T q^;
//   dr, dw partials; Jacobians for dk, dv.
//   Column (query) scale 1/|q| on S and dS; row (key) scales 1/|k|, 1/|v|.
// ===========================================================================
constexpr int kKvBN = 128, kKvBQ = 64, kKvThreads = 256;
constexpr size_t kKvSmem = 2 * (size_t)kKvBN * kD * 2 + 6 * (size_t)kKvBQ * kD * 2 +
                           2 * kKvBQ * sizeof(float4);

__global__ void __launch_bounds__(kKvThreads, 1) mma_bwd_dkdv_kernel(AttnShape s, BwdPtrs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[2][8];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + kKvBN * kD * 2;
  const uint32_t sQ = sV + kKvBN * kD * 2;
  const uint32_t sG = sQ + 2 * kKvBQ * kD * 2;
  const uint32_t sGl = sG + 2 * kKvBQ * kD * 2;
  float4* sCol = reinterpret_cast<float4*>(smem + 2 * kKvBN * kD * 2 + 6 * kKvBQ * kD * 2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const long long j0 = (long long)blockIdx.x * kKvBN;
  const bool causal = s.causal != 0;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const float dmaxf = (float)dmax;
  long long jlast = j0 + kKvBN - 1;
  if (jlast > s.Tk - 1) jlast = s.Tk - 1;
  long long plo, phi;
  query_pos_range(j0, jlast, dmax, causal, plo, phi);
  long long ilo = plo - s.q_offset, ihi = phi - s.q_offset;
  if (ilo < 0) ilo = 0;
  if (ihi > s.Tq - 1) ihi = s.Tq - 1;
  const bool any = dmax >= 0 && ilo <= ihi;

  const bf16* qh = head_ptr(p.q, b, h);
  const bf16* kh = head_ptr(p.k, b, h);
  const bf16* vh = head_ptr(p.v, b, h);
  const bf16* gh = reinterpret_cast<const bf16*>(p.G) + ((long long)b * s.Tq * s.H + h) * kD;
  const bf16* glh = gh + (long long)s.B * s.Tq * s.H * kD;  // G_lo plane
  const long long gst = (long long)s.H * kD;

  load_tile<kKvBN, kKvThreads>(sK, kh, p.k.st, j0, s.Tk, tid);
  load_tile<kKvBN, kKvThreads>(sV, vh, p.v.st, j0, s.Tk, tid);
  const int qt0 = any ? (int)(ilo / kKvBQ) : 0;
  const int qt1 = any ? (int)(ihi / kKvBQ) : -1;
  auto col_info = [&](int qt, int buf) {
    if (tid < kKvBQ) {
      const long long i = (long long)qt * kKvBQ + tid;
      const float v = (float)(i + s.q_offset - j0);
      float sn, cs;
      sincospif(v / w, &sn, &cs);
      const float iqv = i < s.Tq ? 1.0f / p.nq[((long long)b * s.Tq + i) * s.H + h] : 0.f;
      sCol[buf * kKvBQ + tid] = make_float4(cs, sn, v, iqv);
    }
  };
  if (any) {
    load_tile<kKvBQ, kKvThreads>(sQ, qh, p.q.st, (long long)qt0 * kKvBQ, s.Tq, tid);
    load_tile<kKvBQ, kKvThreads>(sG, gh, gst, (long long)qt0 * kKvBQ, s.Tq, tid);
    load_tile<kKvBQ, kKvThreads>(sGl, glh, gst, (long long)qt0 * kKvBQ, s.Tq, tid);
    col_info(qt0, 0);
  }
  cp_async_commit();

  // per key row: u = j - j0, (cos, sin)(pi u / w) / 2, keep, 1/|k|, 1/|v|
  float crow[2], srow[2], urow[2], ikr[2], ivr[2], rk[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int u = warp * 16 + g + hr * 8;
    const long long j = j0 + u;
    float sn, cs;
    sincospif((float)u / w, &sn, &cs);
    crow[hr] = 0.5f * cs;
    srow[hr] = 0.5f * sn;
    urow[hr] = (float)u;
    const bool keep = j < s.Tk && !(s.kpm && s.kpm[(long long)b * s.kpm_sb + j]);
    const long long nidx = ((long long)b * s.Tk + (j < s.Tk ? j : 0)) * s.H + h;
    ikr[hr] = (j < s.Tk) ? 1.0f / p.nk[nidx] : 0.f;
    ivr[hr] = (j < s.Tk) ? 1.0f / p.nv[nidx] : 0.f;
    rk[hr] = keep ? r * ikr[hr] : 0.f;  // masked key: t = 1 - r <= 0 never live
  }
  // a masked key must contribute nothing even when r <= 1 (t = 1 - r > 0)
  float keepf[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const long long j = j0 + warp * 16 + g + hr * 8;
    keepf[hr] = (j < s.Tk && !(s.kpm && s.kpm[(long long)b * s.kpm_sb + j])) ? 1.f : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  uint32_t kf[kKS][4], vf[kKS][4];
  load_a_frags(sK, warp * 16, lane, kf);
  load_a_frags(sV, warp * 16, lane, vf);

  float dk[kNTO][4], dv[kNTO][4];
#pragma unroll
  for (int n = 0; n < kNTO; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;
  float acc_r = 0.f, acc_w = 0.f;
  const long long jw0 = j0 + warp * 16;
  const float one_minus_r = 1.0f - r;

  for (int qt = qt0; qt <= qt1; ++qt) {
    const int buf = (qt - qt0) & 1;
    if (qt < qt1) {
      const uint32_t off = (buf ^ 1) * kKvBQ * kD * 2;
      load_tile<kKvBQ, kKvThreads>(sQ + off, qh, p.q.st, (long long)(qt + 1) * kKvBQ, s.Tq, tid);
      load_tile<kKvBQ, kKvThreads>(sG + off, gh, gst, (long long)(qt + 1) * kKvBQ, s.Tq, tid);
      load_tile<kKvBQ, kKvThreads>(sGl + off, glh, gst, (long long)(qt + 1) * kKvBQ, s.Tq, tid);
      cp_async_commit();
      col_info(qt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const long long pq0 = (long long)qt * kKvBQ + s.q_offset;
    const long long dlo = pq0 - (jw0 + 15), dhi = pq0 + kKvBQ - 1 - jw0;
    if (!block_dead(dlo, dhi, dmax, causal)) {
      const uint32_t qb = sQ + buf * kKvBQ * kD * 2, gb = sG + buf * kKvBQ * kD * 2;
      const float4* ci = sCol + buf * kKvBQ;
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      gemm_abt(sc, kf, qb, lane);
      float mx0 = -3.0e38f, mx1 = -3.0e38f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float iq0 = ci[n * 8 + 2 * tq].w, iq1 = ci[n * 8 + 2 * tq + 1].w;
        sc[n][0] *= iq0; sc[n][1] *= iq1; sc[n][2] *= iq0; sc[n][3] *= iq1;
        mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
      }
      const bool live = fmaf(rk[0], mx0, one_minus_r) > 0.f ||
                        fmaf(rk[1], mx1, one_minus_r) > 0.f || r <= 0.f;
      if (__any_sync(0xffffffffu, live)) {
        float dp[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) dp[n][0] = dp[n][1] = dp[n][2] = dp[n][3] = 0.f;
        gemm_abt(dp, vf, gb, lane);
        gemm_abt(dp, vf, sGl + buf * kKvBQ * kD * 2, lane);
        const bool inside = block_inside(dlo, dhi, dmax, causal);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int hr = e >> 1;
            const float4 c = ci[n * 8 + 2 * tq + (e & 1)];
            const float x = sc[n][e];                 // (q.k) / |q|
            const float rel = urow[hr] - c.z;         // j - p
            float a = fmaxf(fmaf(rk[hr], x, one_minus_r), 0.f) * keepf[hr];
            if (!inside && !in_window(rel, dmaxf, causal)) a = 0.f;
            const float m = fmaf(crow[hr], c.x, fmaf(srow[hr], c.y, 0.5f));
            const float sinrel = 2.0f * (srow[hr] * c.x - crow[hr] * c.y);
            const float d_ = dp[n][e] * ivr[hr];      // G . v^
            const float a2 = a * a;
            const float q2 = d_ * m * 2.0f * a;
            acc_r = fmaf(q2, fmaf(x, ikr[hr], -1.0f), acc_r);
            acc_w = fmaf(d_ * a2, rel * sinrel, acc_w);
            sc[n][e] = a2 * m;                        // alpha
            dp[n][e] = q2 * r * c.w;                  // dS / |q|
          }
        }
        gemm_pt(dv, sc, gb, lane);
        gemm_pt(dk, dp, qb, lane);
      }
    }
    __syncthreads();
  }

  // dr / dw partial of this CTA
  acc_r = warp_sum(acc_r);
  acc_w = warp_sum(acc_w);
  if (lane == 0) {
    red[0][warp] = acc_r;
    red[1][warp] = acc_w;
  }
  store_norm_jacobian(dk, kf, ikr, p.dk, b, h, j0 + warp * 16, s.Tk, g, tq);
  store_norm_jacobian(dv, vf, ivr, p.dv, b, h, j0 + warp * 16, s.Tk, g, tq);
  __syncthreads();
  if (tid == 0) {
    float sr = 0.f, sw = 0.f;
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) {
      sr += red[0][k2];
      sw += red[1][k2];
    }
    const long long P = (long long)s.B * gridDim.x;
    const long long idx = (long long)h * P + (long long)b * gridDim.x + blockIdx.x;
    p.part_r[idx] = sr;
    p.part_w[idx] = sw;
  }
}

}  // namespace

bool mma_supported(int dtype, int D) { return dtype == SCREEN_BF16 && D == kD; }

long long mma_bwd_partials(int, const AttnShape& s) {
  return (long long)s.B * ((s.Tk + kKvBN - 1) / kKvBN);
}

// a failed opt-in stays in cudaGetLastError, which the entry point checks
static void ensure_attrs() {
  if (ensure_smem_optin((const void*)mma_fwd_kernel, (int)kFwdSmem) == cudaSuccess &&
      ensure_smem_optin((const void*)mma_bwd_dq_kernel, (int)kDqSmem) == cudaSuccess)
    ensure_smem_optin((const void*)mma_bwd_dkdv_kernel, (int)kKvSmem);
}

void mma_fwd(int, const AttnShape& s, const FwdPtrs& p, cudaStream_t st) {
  if (s.Tq == 0 || s.B == 0 || s.H == 0) return;
  ensure_attrs();
  dim3 grid((s.Tq + kFwdBM - 1) / kFwdBM, s.B * s.H);
  mma_fwd_kernel<<<grid, kFwdThreads, kFwdSmem, st>>>(s, p);
}

void mma_bwd(int, const AttnShape& s, const BwdPtrs& p, int stages, cudaStream_t st) {
  if (s.B == 0 || s.H == 0) return;
  ensure_attrs();
  if (s.Tq > 0 && (stages & 2)) {
    dim3 g1((s.Tq + kDqBM - 1) / kDqBM, s.B * s.H);
    mma_bwd_dq_kernel<<<g1, kDqThreads, kDqSmem, st>>>(s, p);
  }
  if (s.Tk > 0 && (stages & 4)) {
    dim3 g2((s.Tk + kKvBN - 1) / kKvBN, s.B * s.H);
    mma_bwd_dkdv_kernel<<<g2, kKvThreads, kKvSmem, st>>>(s, p);
  }
}

}  // namespace screen
