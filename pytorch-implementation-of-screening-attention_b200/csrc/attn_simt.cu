// Generic SIMT screening attention (fp32 math, one warp per row, lanes over
// D).  Serves fp32 I/O -- the tensor cores have no full-fp32 mode and the
// fp32 contract is 1e-4 relative -- and the small head dims 16/32 that the
// reference's own tests use.  The bf16 D=64/128 path runs on the tensor cores
// (attn_mma.cu).  Element math follows multiscreen/attention.py:75-119,161-196
// operation for operation: t = 1 - r (1 - s), a = relu(t), alpha = a^2 m,
// m = (cos(pi rel / w) + 1) / 2.
#include "rowops.cuh"

namespace screen {

namespace {
constexpr float kPi = 3.14159265358979323846f;
constexpr int kRowsPerBlock = 8;  // one warp per row, 8 warps

template <int D> struct Lanes { static constexpr int NE = (D + 31) / 32; };

template <typename T, int D>
__device__ __forceinline__ void load_row(const T* base, float (&x)[Lanes<D>::NE], int lane) {
#pragma unroll
  for (int e = 0; e < Lanes<D>::NE; ++e) {
    int d = lane + 32 * e;
    x[e] = (d < D) ? to_f(base[d]) : 0.f;
  }
}
template <typename T, int D>
__device__ __forceinline__ void store_row(T* base, const float (&x)[Lanes<D>::NE], int lane) {
#pragma unroll
  for (int e = 0; e < Lanes<D>::NE; ++e) {
    int d = lane + 32 * e;
    if (d < D) base[d] = from_f<T>(x[e]);
  }
}

// Unit row x / max(|x|, eps) of a raw (B,T,H,D) tensor (attention.py:156-158).
template <typename T, int D>
__device__ __forceinline__ void load_unit(const Rows& x, const float* norms, int b, long long t,
                                          int T_, int H, int h, float (&out)[Lanes<D>::NE],
                                          int lane) {
  load_row<T, D>(reinterpret_cast<const T*>(x.p) + b * x.sb + t * x.st + (long long)h * D, out,
                 lane);
  const float n = norms[((long long)b * T_ + t) * H + h];
#pragma unroll
  for (int e = 0; e < Lanes<D>::NE; ++e) out[e] = out[e] / n;
}

__device__ __forceinline__ bool key_masked(const AttnShape& s, int b, long long j) {
  return s.kpm != nullptr && s.kpm[(long long)b * s.kpm_sb + j] != 0;
}

// ---------------------------------------------------------------------------
// Forward: one warp per query row.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) simt_fwd_kernel(AttnShape s, FwdPtrs p) {
  constexpr int NE = Lanes<D>::NE;
  const int lane = threadIdx.x & 31;
  const long long i = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int b = bh / s.H, h = bh % s.H;
  if (i >= s.Tq) return;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const long long pos = i + s.q_offset;
  long long lo, hi;
  key_range(pos, pos, dmax, s.causal != 0, s.Tk, lo, hi);

  float q[NE], o[NE], kv[NE];
  load_unit<T, D>(p.q, p.nq, b, i, s.Tq, s.H, h, q, lane);
#pragma unroll
  for (int e = 0; e < NE; ++e) o[e] = 0.f;
  // attention dropout (attention.py:190): this query row's counter key
  const uint32_t drow = drop_row(drop_bh_key(s, (uint32_t)bh), (uint32_t)i);

  for (long long j = lo; j <= hi && dmax >= 0; ++j) {
    if (key_masked(s, b, j)) continue;
    load_unit<T, D>(p.k, p.nk, b, j, s.Tk, s.H, h, kv, lane);
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < NE; ++e) dot += q[e] * kv[e];
    const float sim = warp_sum(dot);
    const float t = 1.0f - r * (1.0f - sim);
    if (t > 0.f && drop_keep(drow, (uint32_t)j, s.drop_thr)) {
      const float rel = (float)(j - pos);
      const float m = 0.5f * (cosf(kPi * rel / w) + 1.0f);
      const float alpha = t * t * m;
      load_unit<T, D>(p.v, p.nv, b, j, s.Tk, s.H, h, kv, lane);
#pragma unroll
      for (int e = 0; e < NE; ++e) o[e] += alpha * kv[e];
    }
  }
  // kept scores carry the dropout scale 1 / (1 - p)
#pragma unroll
  for (int e = 0; e < NE; ++e) o[e] *= s.drop_scale;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < NE; ++e) ss += o[e] * o[e];
  ss = warp_sum(ss);
  const float nraw = sqrtf(ss);
  const float g = tanhnorm_scale(nraw, s.eps);
#pragma unroll
  for (int e = 0; e < NE; ++e) o[e] *= g;
  const long long orow = ((long long)b * s.Tq + i) * s.H + h;
  store_row<T, D>(reinterpret_cast<T*>(p.y) + orow * D, o, lane);
  if (lane == 0) p.no[orow] = nraw;
}

// ---------------------------------------------------------------------------
// Backward, query side: dq^ = sum_j dS_ij k^_j, then the normalisation
// Jacobian dq = (dq^ - q^ (q^.dq^)) / max(|q|, eps).
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) simt_bwd_dq_kernel(AttnShape s, BwdPtrs p) {
  constexpr int NE = Lanes<D>::NE;
  const int lane = threadIdx.x & 31;
  const long long i = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int bh = blockIdx.y;
  const int b = bh / s.H, h = bh % s.H;
  if (i >= s.Tq) return;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const long long pos = i + s.q_offset;
  long long lo, hi;
  key_range(pos, pos, dmax, s.causal != 0, s.Tk, lo, hi);
  const long long qrow = ((long long)b * s.Tq + i) * s.H + h;
  float q[NE], g[NE], dq[NE], kk[NE], vv[NE];
  load_unit<T, D>(p.q, p.nq, b, i, s.Tq, s.H, h, q, lane);
  load_row<float, D>(reinterpret_cast<const float*>(p.G) + qrow * D, g, lane);
#pragma unroll
  for (int e = 0; e < NE; ++e) dq[e] = 0.f;
  const uint32_t drow = drop_row(drop_bh_key(s, (uint32_t)bh), (uint32_t)i);
  for (long long j = lo; j <= hi && dmax >= 0; ++j) {
    if (key_masked(s, b, j) || !drop_keep(drow, (uint32_t)j, s.drop_thr)) continue;
    load_unit<T, D>(p.k, p.nk, b, j, s.Tk, s.H, h, kk, lane);
    load_unit<T, D>(p.v, p.nv, b, j, s.Tk, s.H, h, vv, lane);
    float d1 = 0.f, d2 = 0.f;
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      d1 += q[e] * kk[e];
      d2 += g[e] * vv[e];
    }
    const float sim = warp_sum(d1);
    const float dp = warp_sum(d2);
    const float t = 1.0f - r * (1.0f - sim);
    if (t > 0.f) {
      const float rel = (float)(j - pos);
      const float m = 0.5f * (cosf(kPi * rel / w) + 1.0f);
      const float dS = dp * m * 2.0f * t * r;
#pragma unroll
      for (int e = 0; e < NE; ++e) dq[e] += dS * kk[e];
    }
  }
#pragma unroll
  for (int e = 0; e < NE; ++e) dq[e] *= s.drop_scale;
  float dot = 0.f;
#pragma unroll
  for (int e = 0; e < NE; ++e) dot += q[e] * dq[e];
  dot = warp_sum(dot);
  const float inv = 1.0f / p.nq[qrow];
#pragma unroll
  for (int e = 0; e < NE; ++e) dq[e] = (dq[e] - q[e] * dot) * inv;
  store_row<T, D>(reinterpret_cast<T*>(p.dq.p) + b * p.dq.sb + i * p.dq.st + (long long)h * D,
                  dq, lane);
}

// ---------------------------------------------------------------------------
// Backward, key side: dv^_j = sum_i alpha_ij G_i, dk^_j = sum_i dS_ij q^_i,
// plus the dr / dw partial sums of this block's keys.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) simt_bwd_dkdv_kernel(AttnShape s, BwdPtrs p) {
  constexpr int NE = Lanes<D>::NE;
  __shared__ float red_r[kRowsPerBlock], red_w[kRowsPerBlock];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long j = (long long)blockIdx.x * kRowsPerBlock + warp;
  const int bh = blockIdx.y;
  const int b = bh / s.H, h = bh % s.H;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  float acc_r = 0.f, acc_w = 0.f;
  if (j < s.Tk) {
    const float* Gp = reinterpret_cast<const float*>(p.G);
    const long long krow = ((long long)b * s.Tk + j) * s.H + h;
    float k[NE], v[NE], dk[NE], dv[NE], qq[NE], gg[NE];
    load_unit<T, D>(p.k, p.nk, b, j, s.Tk, s.H, h, k, lane);
    load_unit<T, D>(p.v, p.nv, b, j, s.Tk, s.H, h, v, lane);
#pragma unroll
    for (int e = 0; e < NE; ++e) dk[e] = dv[e] = 0.f;
    if (!key_masked(s, b, j) && dmax >= 0) {
      long long plo, phi;
      query_pos_range(j, j, dmax, s.causal != 0, plo, phi);
      long long ilo = plo - s.q_offset, ihi = phi - s.q_offset;
      if (ilo < 0) ilo = 0;
      if (ihi > s.Tq - 1) ihi = s.Tq - 1;
      const uint32_t bhk = drop_bh_key(s, (uint32_t)bh);
      for (long long i = ilo; i <= ihi; ++i) {
        if (s.drop_thr && !drop_keep(drop_row(bhk, (uint32_t)i), (uint32_t)j, s.drop_thr)) continue;
        const long long qrow = ((long long)b * s.Tq + i) * s.H + h;
        load_unit<T, D>(p.q, p.nq, b, i, s.Tq, s.H, h, qq, lane);
        load_row<float, D>(Gp + qrow * D, gg, lane);
        float d1 = 0.f, d2 = 0.f;
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          d1 += qq[e] * k[e];
          d2 += gg[e] * v[e];
        }
        const float sim = warp_sum(d1);
        const float dp = warp_sum(d2);
        const float t = 1.0f - r * (1.0f - sim);
        if (t > 0.f) {
          const float rel = (float)(j - (i + s.q_offset));
          const float ang = kPi * rel / w;
          const float m = 0.5f * (cosf(ang) + 1.0f);
          const float alpha = t * t * m;
          const float q2 = dp * m * 2.0f * t;
          const float dS = q2 * r;
#pragma unroll
          for (int e = 0; e < NE; ++e) {
            dv[e] += alpha * gg[e];
            dk[e] += dS * qq[e];
          }
          acc_r += q2 * (sim - 1.0f);
          acc_w += dp * t * t * rel * sinf(ang);
        }
      }
    }
    // kept scores carry the dropout scale
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      dk[e] *= s.drop_scale;
      dv[e] *= s.drop_scale;
    }
    acc_r *= s.drop_scale;
    acc_w *= s.drop_scale;
    // normalisation Jacobians
    float d1 = 0.f, d2 = 0.f;
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      d1 += k[e] * dk[e];
      d2 += v[e] * dv[e];
    }
    d1 = warp_sum(d1);
    d2 = warp_sum(d2);
    const float ik = 1.0f / p.nk[krow], iv = 1.0f / p.nv[krow];
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      dk[e] = (dk[e] - k[e] * d1) * ik;
      dv[e] = (dv[e] - v[e] * d2) * iv;
    }
    store_row<T, D>(reinterpret_cast<T*>(p.dk.p) + b * p.dk.sb + j * p.dk.st + (long long)h * D,
                    dk, lane);
    store_row<T, D>(reinterpret_cast<T*>(p.dv.p) + b * p.dv.sb + j * p.dv.st + (long long)h * D,
                    dv, lane);
  }
  if (lane == 0) {
    red_r[warp] = acc_r;
    red_w[warp] = acc_w;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sr = 0.f, sw = 0.f;
    for (int k2 = 0; k2 < kRowsPerBlock; ++k2) {
      sr += red_r[k2];
      sw += red_w[k2];
    }
    const long long P = (long long)s.B * gridDim.x;
    const long long idx = (long long)h * P + (long long)b * gridDim.x + blockIdx.x;
    p.part_r[idx] = sr;
    p.part_w[idx] = sw;
  }
}

template <typename T, int D>
void launch_simt_fwd(const AttnShape& s, const FwdPtrs& p, cudaStream_t st) {
  if (s.Tq == 0 || s.B == 0 || s.H == 0) return;
  dim3 grid((s.Tq + kRowsPerBlock - 1) / kRowsPerBlock, s.B * s.H);
  simt_fwd_kernel<T, D><<<grid, 256, 0, st>>>(s, p);
}
template <typename T, int D>
void launch_simt_bwd(const AttnShape& s, const BwdPtrs& p, int stages, cudaStream_t st) {
  if (s.B == 0 || s.H == 0) return;
  if (s.Tq > 0 && (stages & 2)) {
    dim3 g1((s.Tq + kRowsPerBlock - 1) / kRowsPerBlock, s.B * s.H);
    simt_bwd_dq_kernel<T, D><<<g1, 256, 0, st>>>(s, p);
  }
  if (s.Tk > 0 && (stages & 4)) {
    dim3 g2((s.Tk + kRowsPerBlock - 1) / kRowsPerBlock, s.B * s.H);
    simt_bwd_dkdv_kernel<T, D><<<g2, 256, 0, st>>>(s, p);
  }
}
}  // namespace

long long simt_bwd_partials(const AttnShape& s) {
  return (long long)s.B * ((s.Tk + kRowsPerBlock - 1) / kRowsPerBlock);
}

#define SCREEN_DISPATCH(FN, ...)                                   \
  do {                                                             \
    if (dtype == SCREEN_F32) {                                     \
      switch (D) {                                                 \
        case 16: FN<float, 16>(__VA_ARGS__); break;                \
        case 32: FN<float, 32>(__VA_ARGS__); break;                \
        case 64: FN<float, 64>(__VA_ARGS__); break;                \
        case 128: FN<float, 128>(__VA_ARGS__); break;              \
      }                                                            \
    } else {                                                       \
      switch (D) {                                                 \
        case 16: FN<__nv_bfloat16, 16>(__VA_ARGS__); break;        \
        case 32: FN<__nv_bfloat16, 32>(__VA_ARGS__); break;        \
        case 64: FN<__nv_bfloat16, 64>(__VA_ARGS__); break;        \
        case 128: FN<__nv_bfloat16, 128>(__VA_ARGS__); break;      \
      }                                                            \
    }                                                              \
  } while (0)

void simt_fwd(int dtype, int D, const AttnShape& s, const FwdPtrs& p, cudaStream_t st) {
  SCREEN_DISPATCH(launch_simt_fwd, s, p, st);
}
void simt_bwd(int dtype, int D, const AttnShape& s, const BwdPtrs& p, int stages,
              cudaStream_t st) {
  SCREEN_DISPATCH(launch_simt_bwd, s, p, stages, st);
}

}  // namespace screen
