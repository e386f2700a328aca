// Paged K/V cache append and single-token screening decode.
//
// The cache holds UNIT rows k^, v^ (attention.py:157-158 applied once at
// append time) in pages of [H, page_size, D], so one head's rows inside a
// page are contiguous.  Decode for the newest token of sequence b (position
// t = seq_lens[b]-1) reads only keys j in [t - dmax, t] -- the causal window
// of attention.py:117-118 -- split across `num_splits` CTAs per (b, h).
// Because screening has no softmax normaliser (attention.py:193), the split
// partials combine by plain summation; TanhNorm (norm.py:23-25) is applied
// once after the sum.
#include "decode.cuh"

#include <cstdlib>

namespace screen {
namespace {

constexpr float kPi = 3.14159265358979323846f;

template <typename T> struct Vec16;  // 16 bytes of T <-> floats
template <> struct Vec16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float* p, float (&x)[4]) {
    float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
  static __device__ __forceinline__ void from_raw(uint4 u, float (&x)[4]) {
    x[0] = __uint_as_float(u.x); x[1] = __uint_as_float(u.y);
    x[2] = __uint_as_float(u.z); x[3] = __uint_as_float(u.w);
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y; x[4] = c.x; x[5] = c.y; x[6] = d.x; x[7] = d.y;
  }
  static __device__ __forceinline__ void from_raw(uint4 u, float (&x)[8]) {
    float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y; x[4] = c.x; x[5] = c.y; x[6] = d.x; x[7] = d.y;
  }
};

__device__ __forceinline__ long long page_row(const screen_kv_cache& c, int b, int H, int h,
                                              long long pos, int D) {
  const long long blk = pos / c.page_size;
  if (blk < 0 || blk >= c.max_blocks) return -1;
  const int page = c.block_table[(long long)b * c.max_blocks + blk];
  if (page < 0 || page >= c.num_pages) return -1;
  return (((long long)page * H + h) * c.page_size + pos % c.page_size) * D;
}

// ---------------------------------------------------------------------------
// Append: one group of D/4 lanes per (b, n, h) row; blockIdx.y selects K / V.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void kv_append_kernel(screen_kv_append_args a) {
  pdl_wait();      // reads the previous kernels' outputs from here on
  pdl_trigger();
  constexpr int G = D / 4;
  constexpr int RPB = 256 / G;
  const long long row = (long long)blockIdx.x * RPB + threadIdx.x / G;
  const int lane = threadIdx.x % G;
  const long long rows = (long long)a.B * a.n_new * a.H;
  const bool valid = row < rows;  // no early exit: the group shuffles below need every lane
  const long long rr = valid ? row : 0;
  const int h = (int)(rr % a.H);
  const long long n = (rr / a.H) % a.n_new;
  const int b = (int)(rr / ((long long)a.H * a.n_new));
  const bool isv = blockIdx.y == 1;
  const T* src = reinterpret_cast<const T*>(isv ? a.v : a.k) +
                 (long long)b * (isv ? a.v_sb : a.k_sb) + n * (isv ? a.v_st : a.k_st) +
                 (long long)h * D + lane * 4;
  float x[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = valid ? to_f(src[e]) : 0.f;
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, G);
  const float nrm = fmaxf(sqrtf(ss), a.eps);
  if (!valid) return;
  const long long dst = page_row(a.cache, b, a.H, h, (long long)a.positions[b] + n, D);
  if (dst < 0) return;
  T* out = reinterpret_cast<T*>(isv ? a.cache.v_pages : a.cache.k_pages) + dst + lane * 4;
#pragma unroll
  for (int e = 0; e < 4; ++e) out[e] = from_f<T>(x[e] / nrm);
}

// ---------------------------------------------------------------------------
// Decode split: CTA (split, b*H + h), 4 warps; LPK lanes read one 16-byte
// slice each of a key row, KPW keys per warp step.
// ---------------------------------------------------------------------------
// End of a decode CTA: with several splits, store this split's partial sum
// for decode_finish_kernel; with one split the CTA holds the whole
// alpha-weighted sum and applies TanhNorm itself (no finishing launch).
// red[k][d]: the per-warp sums.  Uniform over the CTA (it syncs).
template <typename T, int D, int NW>
__device__ __forceinline__ void store_split(const screen_decode_args& a, float* __restrict__ part,
                                            float (&red)[NW][D], int bh, int split) {
  const int tid = threadIdx.x;
  if (a.num_splits > 1) {
    for (int d = tid; d < D; d += blockDim.x) {
      float s2 = 0.f;
#pragma unroll
      for (int k = 0; k < NW; ++k) s2 += red[k][d];
      part[((long long)bh * a.num_splits + split) * D + d] = s2;
    }
    return;
  }
  for (int d = tid; d < D; d += blockDim.x) {
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NW; ++k) s2 += red[k][d];
    red[0][d] = s2;
  }
  __syncthreads();
  if (tid < 32) {
    float ss = 0.f;
    for (int d = tid; d < D; d += 32) ss = fmaf(red[0][d], red[0][d], ss);
    ss = warp_sum(ss);
    const float nraw = sqrtf(ss);
    const float g = tanhnorm_scale(nraw, a.eps);
    for (int d = tid; d < D; d += 32)
      reinterpret_cast<T*>(a.y)[(long long)bh * D + d] = from_f<T>(red[0][d] * g);
    if (tid == 0 && a.no) a.no[bh] = nraw;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) decode_split_kernel(screen_decode_args a,
                                                           float* __restrict__ part) {
  pdl_wait();      // reads the previous kernels' outputs from here on
  pdl_trigger();
  constexpr int VEC = Vec16<T>::N;
  constexpr int LPK = D / VEC;      // lanes per key row
  constexpr int KPW = 32 / LPK;     // keys per warp step
  constexpr int NW = 4;
  __shared__ float qs[D];
  __shared__ float red[NW][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int split = blockIdx.x;

  // unit query (attention.py:156)
  const T* qraw = reinterpret_cast<const T*>(a.q) + (long long)b * a.q_sb + (long long)h * D;
  for (int d = tid; d < D; d += 128) qs[d] = to_f(qraw[d]);
  __syncthreads();
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) ss += qs[d] * qs[d];
  ss = warp_sum(ss);
  const float qn = fmaxf(sqrtf(ss), a.eps);

  const float r = a.r[h], w = a.w[h];
  const int dmax = window_dmax(w);
  const long long t = (long long)a.seq_lens[b] - 1;
  long long lo = t - dmax, hi = t;
  if (lo < 0) lo = 0;
  const long long nkeys = (dmax >= 0 && t >= 0) ? hi - lo + 1 : 0;
  const long long chunk = (nkeys + a.num_splits - 1) / a.num_splits;
  const long long c0 = lo + (long long)split * chunk;
  long long c1 = c0 + chunk - 1;
  if (c1 > hi) c1 = hi;

  const int sub = lane % LPK, grp = lane / LPK;
  float qv[VEC], acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    qv[e] = qs[sub * VEC + e] / qn;
    acc[e] = 0.f;
  }
  const T* kp = reinterpret_cast<const T*>(a.cache.k_pages);
  const T* vp = reinterpret_cast<const T*>(a.cache.v_pages);
  // page ids of this CTA's key chunk, staged once in shared memory so that a
  // key's address needs no dependent block-table load
  constexpr int kPageCache = 256;
  __shared__ int spage[kPageCache];
  const int ps = a.cache.page_size;
  const int blk0 = nkeys > 0 ? (int)(c0 / ps) : 0;
  const int nblk = nkeys > 0 && c1 >= c0 ? (int)(c1 / ps) - blk0 + 1 : 0;
  for (int i = tid; i < nblk && i < kPageCache; i += 128) {
    const int blk = blk0 + i;
    int page = -1;
    if (blk < a.cache.max_blocks) {
      page = a.cache.block_table[(long long)b * a.cache.max_blocks + blk];
      if (page < 0 || page >= a.cache.num_pages) page = -1;
    }
    spage[i] = page;
  }
  __syncthreads();
  auto row_off = [&](long long j) -> long long {
    const int jj = (int)j, blk = jj / ps, idx = blk - blk0;
    if (idx >= kPageCache) return page_row(a.cache, b, a.H, h, j, D);
    const int page = spage[idx];
    if (page < 0) return -1;
    return (((long long)page * a.H + h) * ps + (jj - blk * ps)) * D;
  };
  if (nkeys > 0) {
    // kU key steps per iteration: their K rows are all in flight at once,
    // then the V rows of the keys that cleared the trim threshold
    constexpr int kU = 8;
    for (long long base = c0 + (long long)warp * KPW; base <= c1;
         base += (long long)NW * KPW * kU) {
      uint4 kraw[kU];
      long long off[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long long j = base + (long long)u * NW * KPW + grp;
        off[u] = j <= c1 ? row_off(j) : -1;
        kraw[u] = off[u] >= 0 ? *reinterpret_cast<const uint4*>(kp + off[u] + sub * VEC)
                              : make_uint4(0, 0, 0, 0);
      }
#ifdef SCREEN_DECODE_EAGER_V
      uint4 vraw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        vraw[u] = off[u] >= 0 ? *reinterpret_cast<const uint4*>(vp + off[u] + sub * VEC)
                              : make_uint4(0, 0, 0, 0);
#endif
      float alpha[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        float kx[VEC];
        Vec16<T>::from_raw(kraw[u], kx);
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) dot += qv[e] * kx[e];
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float tt = 1.0f - r * (1.0f - dot);
        alpha[u] = 0.f;
        if (off[u] >= 0 && tt > 0.f) {
          const long long j = base + (long long)u * NW * KPW + grp;
          const float rel = (float)(j - t);
          const float m = 0.5f * (cosf(kPi * rel / w) + 1.0f);
          alpha[u] = tt * tt * m;
        }
      }
#ifndef SCREEN_DECODE_EAGER_V
      uint4 vraw[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        vraw[u] = alpha[u] != 0.f ? *reinterpret_cast<const uint4*>(vp + off[u] + sub * VEC)
                                  : make_uint4(0, 0, 0, 0);
#endif
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        float vx[VEC];
        Vec16<T>::from_raw(vraw[u], vx);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = fmaf(alpha[u], vx[e], acc[e]);
      }
    }
  }
  // combine key groups of the warp, then the warps
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
  }
  if (grp == 0) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) red[warp][sub * VEC + e] = acc[e];
  }
  __syncthreads();
  store_split<T, D, NW>(a, part, red, bh, split);
}

// ---------------------------------------------------------------------------
// Decode split, bulk-copy form.  One head's rows inside a page are one
// contiguous run of page_size * D elements, so a producer thread streams
// sub-runs of SK <= 32 keys (K run + V run) into a ring of shared-memory
// stages with cp.async.bulk, completion counted in bytes on a per-stage
// mbarrier.  Stage s belongs to consumer warp s % NW, so the four consumer
// warps work on different sub-runs side by side:
//   * scores: lane l owns key l of the sub-run and reads its whole row in
//     16-byte chunks, chunk (c + l) mod C at step c -- eight lanes of a
//     quarter-warp then touch eight different bank groups although the rows
//     sit at a multiple of 128 bytes; the query is staged in the same chunk
//     order, products go through packed fp32 FMA;
//   * trim / mask: once per key, one key per lane (attention.py:160-171);
//   * alpha * v: only for the keys that cleared the trim (a ballot), each
//     lane owning a slice of d of the V row, alpha broadcast by shuffle.
// The bytes in flight per SM (stages x resident CTAs) keep HBM busy.  Every
// wait is bounded; on give-up the kernel raises g_decode_status, drains its
// own copies and returns.
// ---------------------------------------------------------------------------
__device__ int g_decode_status = 0;
constexpr uint64_t kDecWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr int kDecMaxStages = 16;
constexpr int kDecConsumers = 4;

__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

template <typename T, int D>
__global__ void __launch_bounds__(32 * (kDecConsumers + 1)) decode_bulk_kernel(
    screen_decode_args a, float* __restrict__ part, int nstages, int sk,
    screen_kv_append_args ap, int do_append) {
  pdl_wait();      // reads the previous kernels' outputs from here on
  pdl_trigger();
  using namespace sm100;
  constexpr int NW = kDecConsumers;
  constexpr int SZ = (int)sizeof(T);
  constexpr int C = D * SZ / 16;                  // 16-byte chunks per row
  constexpr int WORDS = D * SZ / 4;               // 32-bit words per row
  constexpr int WPL = WORDS >= 32 ? WORDS / 32 : 1;  // V words per lane
  constexpr int KPS = WORDS >= 32 ? 1 : 32 / WORDS;  // V keys per warp step
  constexpr int FPW = 4 / SZ;                     // floats per word
  constexpr int EPL = WPL * FPW;                  // accumulators per lane
  constexpr bool kBf16 = SZ == 2;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ __align__(8) uint64_t bars[2 * kDecMaxStages];
  __shared__ int stage_ok[kDecMaxStages];
  __shared__ int abort_s;
  // query in chunk order: qc[h][j] = floats 8j+4h .. 8j+4h+3 (bf16 rows) or
  // 4j .. 4j+3 (fp32 rows)
  __shared__ __align__(16) float4 qc[kBf16 ? 2 : 1][C];
  __shared__ float red[NW][D];
  __shared__ float qsum[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int split = blockIdx.x;
  const int ps = a.cache.page_size;
  const int subs = ps / sk;                       // sub-runs per page
  const uint32_t run_bytes = (uint32_t)sk * D * SZ;
  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[kDecMaxStages + s]); };
  volatile int* abort_flag = &abort_s;

  if (tid == 0) {
    for (int s = 0; s < nstages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    abort_s = 0;
    fence_proxy_async_smem();
  }
  // per-head parameters and the sequence length are requested together with
  // the query (independent loads, one memory round trip)
  const float r = a.r[h], w = a.w[h];
  const long long t = (long long)a.seq_lens[b] - 1;
  const T* qraw = reinterpret_cast<const T*>(a.q) + (long long)b * a.q_sb + (long long)h * D;
  float* qf = reinterpret_cast<float*>(&qc[0][0]);
  float ssq = 0.f;
  for (int d = tid; d < D; d += blockDim.x) {
    const float x = to_f(qraw[d]);
    ssq += x * x;
    int at = d;
    if (kBf16) at = ((d >> 2) & 1) * (C * 4) + (d >> 3) * 4 + (d & 3);
    qf[at] = x;
  }
  ssq = warp_sum(ssq);
  if (lane == 0) qsum[warp] = ssq;
  __syncthreads();

  const int dmax = window_dmax(w);
  long long lo = t - dmax;
  if (lo < 0) lo = 0;
  const bool any = dmax >= 0 && t >= 0;
  // page-aligned split of the window's blocks
  const long long blo = any ? lo / ps : 0, bhi = any ? t / ps : -1;
  const long long nb = bhi - blo + 1;
  const long long per = (nb + a.num_splits - 1) / a.num_splits;
  const long long b0 = blo + (long long)split * per;
  long long b1 = b0 + per - 1;
  if (b1 > bhi) b1 = bhi;
  const int npages = any && b1 >= b0 ? (int)(b1 - b0 + 1) : 0;
  const int nunits = npages * subs;

  if (do_append) {
    // the newest token's unit k / v rows (the one new row of ap) go into the
    // cache first, written by the split whose pages hold that position (the
    // first split when the window is empty), with the arithmetic of
    // kv_append_kernel: groups of D / 4 lanes, K rows then V rows
    const int wsplit = any ? (int)((bhi - blo) / per) : 0;
    constexpr int G = D / 4;
    constexpr int NT = 2 * G < 32 ? 32 : 2 * G;   // whole warps take part in the shuffles
    if (split == wsplit && tid < NT) {
      const bool valid = tid < 2 * G;
      const bool isv = tid >= G;
      const int gl = tid % G;
      const T* src = reinterpret_cast<const T*>(isv ? ap.v : ap.k) +
                     (long long)b * (isv ? ap.v_sb : ap.k_sb) + (long long)h * D + gl * 4;
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = valid ? to_f(src[e]) : 0.f;
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, G);
      const float nrm = fmaxf(sqrtf(ss), ap.eps);
      const long long dst = valid ? page_row(ap.cache, b, ap.H, h, (long long)ap.positions[b], D)
                                  : -1;
      if (dst >= 0) {
        T* out = reinterpret_cast<T*>(isv ? ap.cache.v_pages : ap.cache.k_pages) + dst + gl * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) out[e] = from_f<T>(x[e] / nrm);
      }
      // the rows are read back below by bulk copies (the async proxy)
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();
  }

  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;

  if (warp == NW) {
    // producer warp: page ids of 32 pages fetched at once (one per lane, the
    // next 32 while these are issued); lane 0 waits and issues, verdicts are
    // broadcast so the warp stays converged
    const T* kp = reinterpret_cast<const T*>(a.cache.k_pages);
    const T* vp = reinterpret_cast<const T*>(a.cache.v_pages);
    auto page_of = [&](int i) -> int {
      const long long blk = b0 + i;
      if (i >= npages || blk >= a.cache.max_blocks) return -1;
      const int page = a.cache.block_table[(long long)b * a.cache.max_blocks + blk];
      return (page < 0 || page >= a.cache.num_pages) ? -1 : page;
    };
    int next_ids = page_of(lane);
    int issued = 0;
    bool stop = false;
    for (int p0 = 0; p0 < npages && !stop; p0 += 32) {
      const int ids = next_ids;
      next_ids = page_of(p0 + 32 + lane);
      const int pn = npages - p0 < 32 ? npages - p0 : 32;
      for (int pu = 0; pu < pn && !stop; ++pu) {
        const int page = __shfl_sync(0xffffffffu, ids, pu);
        for (int sub = 0; sub < subs; ++sub) {
          const int u = (p0 + pu) * subs + sub, s = u % nstages;
          int okw = 1;
          if (lane == 0 && u >= nstages)
            okw = mbar_wait(empty(s), ((u / nstages) - 1) & 1, abort_flag, kDecWaitLimitNs);
          okw = __shfl_sync(0xffffffffu, okw, 0);
          if (!okw) {
            stop = true;
            break;
          }
          if (lane == 0) {
            stage_ok[s] = page >= 0;
            if (page >= 0) {
              const long long off = (((long long)page * a.H + h) * ps + (long long)sub * sk) * D;
              const uint32_t dst = smem_u32(dsm + (size_t)s * 2 * run_bytes);
              mbar_arrive_expect_tx(full(s), 2 * run_bytes);
              bulk_g2s(dst, kp + off, run_bytes, full(s));
              bulk_g2s(dst + run_bytes, vp + off, run_bytes, full(s));
            } else {
              mbar_arrive(full(s));
            }
          }
          issued = u + 1;
        }
      }
    }
    if (lane == 0 && *abort_flag) {
      // let the copies already issued land before the CTA's smem goes away
      const int first = issued > nstages ? issued - nstages : 0;
      const uint64_t t0 = globaltimer();
      for (int u = first; u < issued; ++u)
        while (!mbar_try_wait(full(u % nstages), (u / nstages) & 1) &&
               globaltimer() - t0 < kDecWaitLimitNs) {
        }
    }
    __syncwarp();
  } else {
    float ssum = 0.f;
    for (int i = 0; i < (int)((blockDim.x + 31) / 32); ++i) ssum += qsum[i];
    const float inv_qn = 1.0f / fmaxf(sqrtf(ssum), a.eps);
    const int vg = lane / (WORDS >= 32 ? 32 : WORDS);   // key slot of this lane in a V step
    const int vw = lane % (WORDS >= 32 ? 32 : WORDS);   // first word of this lane
    for (int u = warp; u < nunits; u += NW) {
      const int s = u % nstages;
      int okw = 0;
      if (lane == 0) okw = mbar_wait(full(s), (u / nstages) & 1, abort_flag, kDecWaitLimitNs);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      while (!mbar_try_wait(full(s), (u / nstages) & 1)) {
      }
      if (stage_ok[s]) {
        const unsigned char* ks = dsm + (size_t)s * 2 * run_bytes;
        const unsigned char* vs = ks + run_bytes;
        const long long j = (b0 + u / subs) * ps + (long long)(u % subs) * sk + lane;
        const bool in = lane < sk && j >= lo && j <= t;
        float alpha = 0.f;
        if (lane < sk) {
          const unsigned char* row = ks + (size_t)lane * D * SZ;
          float2 d2a = make_float2(0.f, 0.f), d2b = make_float2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const int cj = (c + lane) & (C - 1);
            const uint4 kr = *reinterpret_cast<const uint4*>(row + 16 * cj);
            if (kBf16) {
              const float4 qa = qc[0][cj], qb = qc[kBf16 ? 1 : 0][cj];
              // chunk element order: words x,y,z,w hold d (0,1) (2,3) (4,5) (6,7)
              d2a = __ffma2_rn(bf16x2_to_f2(kr.x), make_float2(qa.x, qa.y), d2a);
              d2b = __ffma2_rn(bf16x2_to_f2(kr.y), make_float2(qa.z, qa.w), d2b);
              d2a = __ffma2_rn(bf16x2_to_f2(kr.z), make_float2(qb.x, qb.y), d2a);
              d2b = __ffma2_rn(bf16x2_to_f2(kr.w), make_float2(qb.z, qb.w), d2b);
            } else {
              const float4 qa = qc[0][cj];
              d2a = __ffma2_rn(make_float2(__uint_as_float(kr.x), __uint_as_float(kr.y)),
                               make_float2(qa.x, qa.y), d2a);
              d2b = __ffma2_rn(make_float2(__uint_as_float(kr.z), __uint_as_float(kr.w)),
                               make_float2(qa.z, qa.w), d2b);
            }
          }
          const float dot = ((d2a.x + d2b.x) + (d2a.y + d2b.y)) * inv_qn;
          const float tt = 1.0f - r * (1.0f - dot);
          if (in && tt > 0.f) {
            const float rel = (float)(j - t);
            const float m = 0.5f * (cosf(kPi * rel / w) + 1.0f);
            alpha = tt * tt * m;
          }
        }
        unsigned live = __ballot_sync(0xffffffffu, alpha != 0.f);
        while (live) {
          const int k0 = __ffs(live) - 1;
          const int kk = k0 + vg;
          const float al = __shfl_sync(0xffffffffu, alpha, kk & 31);
          if (KPS == 1) {
            live &= live - 1;
          } else {
            live &= ~(((1u << KPS) - 1u) << k0);
          }
          if (kk < sk && al != 0.f) {
            const uint32_t* vrow = reinterpret_cast<const uint32_t*>(vs + (size_t)kk * D * SZ);
#pragma unroll
            for (int q = 0; q < WPL; ++q) {
              const uint32_t vw32 = vrow[vw + 32 * q];
              if (kBf16) {
                const float2 v2 = bf16x2_to_f2(vw32);
                acc[2 * q] = fmaf(al, v2.x, acc[2 * q]);
                acc[2 * q + 1] = fmaf(al, v2.y, acc[2 * q + 1]);
              } else {
                acc[q] = fmaf(al, __uint_as_float(vw32), acc[q]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(s));
    }
  }
  if (tid == 0 && *abort_flag) atomicExch(&g_decode_status, (int)SCREEN_ERR_TIMEOUT);
  if (warp < NW) {
    // lanes of different key slots (KPS > 1) hold the same words
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
#pragma unroll
      for (int o = WORDS; o < 32; o <<= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    }
    if (lane < (WORDS >= 32 ? 32 : WORDS)) {
#pragma unroll
      for (int q = 0; q < WPL; ++q) {
#pragma unroll
        for (int f = 0; f < FPW; ++f) red[warp][(lane + 32 * q) * FPW + f] = acc[q * FPW + f];
      }
    }
  }
  __syncthreads();
  store_split<T, D, NW>(a, part, red, bh, split);
}

// Sum the splits, TanhNorm, store y (B,H,D) and |o|.  256 threads: 256/D
// groups each sum a strided subset of the splits, then one pass combines.
template <typename T, int D>
__global__ void __launch_bounds__(256) decode_finish_kernel(screen_decode_args a,
                                                            const float* __restrict__ part) {
  pdl_wait();      // reads the previous kernels' outputs from here on
  pdl_trigger();
  constexpr int NG = 256 / D;
  __shared__ float acc[NG][D];
  __shared__ float red[D];
  const int bh = blockIdx.x, d = threadIdx.x % D, grp = threadIdx.x / D;
  float o = 0.f;
  for (int s = grp; s < a.num_splits; s += NG)
    o += part[((long long)bh * a.num_splits + s) * D + d];
  acc[grp][d] = o;
  __syncthreads();
  if (threadIdx.x < D) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) t += acc[g][d];
    acc[0][d] = t;
    red[d] = t * t;
  }
  __syncthreads();
  for (int st = D / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) red[threadIdx.x] += red[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x < D) {
    const float nraw = sqrtf(red[0]);
    const float g = tanhnorm_scale(nraw, a.eps);
    reinterpret_cast<T*>(a.y)[(long long)bh * D + d] = from_f<T>(acc[0][d] * g);
    if (d == 0 && a.no) a.no[bh] = nraw;
  }
}

template <typename T, int D>
void launch_append(const screen_kv_append_args& a, cudaStream_t s) {
  constexpr int RPB = 256 / (D / 4);
  const long long rows = (long long)a.B * a.n_new * a.H;
  if (rows == 0) return;
  dim3 grid((unsigned)((rows + RPB - 1) / RPB), 2);
  launch_pdl(kv_append_kernel<T, D>, grid, dim3(256), 0, s, a);
}
// ap: one new k / v row per (b, h) to append before the decode (nullptr:
// none).  The bulk-copy kernel writes it itself; the fallback path launches
// the append kernel first.
template <typename T, int D>
void launch_decode(const screen_decode_args& a, float* part, cudaStream_t s,
                   const screen_kv_append_args* ap = nullptr) {
  if (a.B == 0 || a.H == 0) {
    if (ap) launch_append<T, D>(*ap, s);
    return;
  }
  dim3 grid(a.num_splits, a.B * a.H);
  // sub-runs of sk keys: the largest power of two <= 32 dividing page_size
  int sk = 1;
  while (sk < 32 && a.cache.page_size % (2 * sk) == 0) sk *= 2;
  const size_t stage_bytes = 2 * (size_t)sk * D * sizeof(T);
  // shared-memory ring budget per CTA: 64 KB leaves 3 CTAs per SM (32 and
  // 48 KB rings measured slower at 32K and 100K keys)
  constexpr int ring_kb = 64;
  int nstages = (int)(((size_t)ring_kb << 10) / stage_bytes);
  nstages = nstages / kDecConsumers * kDecConsumers;
  if (nstages > kDecMaxStages) nstages = kDecMaxStages;
  if (nstages < kDecConsumers) nstages = kDecConsumers;
  const size_t smem = (size_t)nstages * stage_bytes;
  if (smem <= (200u << 10) && stage_bytes % 16 == 0) {
    // the opt-in is per device; on failure the error stays in
    // cudaGetLastError for the entry point's launch check
    if (ensure_smem_optin((const void*)decode_bulk_kernel<T, D>, 200 << 10) != cudaSuccess) return;
    launch_pdl(decode_bulk_kernel<T, D>, grid, dim3(32 * (kDecConsumers + 1)), smem, s, a, part,
               nstages, sk, ap ? *ap : screen_kv_append_args{}, ap ? 1 : 0);
  } else {
    if (ap) launch_append<T, D>(*ap, s);
    launch_pdl(decode_split_kernel<T, D>, grid, dim3(128), 0, s, a, part);
  }
  if (a.num_splits > 1)
    launch_pdl(decode_finish_kernel<T, D>, dim3(a.B * a.H), dim3(256), 0, s, a, part);
}

}  // namespace

#define DEC_DISPATCH(FN, ...)                                      \
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

void kv_append(const screen_kv_append_args& a, cudaStream_t s) {
  const int dtype = a.dtype, D = a.D;
  DEC_DISPATCH(launch_append, a, s);
}
int decode_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(int)) != cudaSuccess) return SCREEN_ERR_CUDA;
  if (clear && v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_decode_status, &z, sizeof(int));
  }
  return v;
}
void decode(const screen_decode_args& a, float* part, cudaStream_t s) {
  const int dtype = a.dtype, D = a.D;
  DEC_DISPATCH(launch_decode, a, part, s);
}
void decode_append(const screen_kv_append_args& ap, const screen_decode_args& a, float* part,
                   cudaStream_t s) {
  const int dtype = a.dtype, D = a.D;
  DEC_DISPATCH(launch_decode, a, part, s, &ap);
}

}  // namespace screen
