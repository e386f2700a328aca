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
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
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
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_split_kernel(screen_decode_args a,
                                                           float* __restrict__ part) {
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
  for (int d = 0; d < D; ++d) ss += qs[d] * qs[d];
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
  if (nkeys > 0) {
    for (long long base = c0 + (long long)warp * KPW; base <= c1; base += (long long)NW * KPW) {
      const long long j = base + grp;
      const bool valid = j <= c1;
      const long long off = valid ? page_row(a.cache, b, a.H, h, j, D) : -1;
      float kx[VEC];
      float dot = 0.f;
      if (off >= 0) {
        Vec16<T>::load(kp + off + sub * VEC, kx);
#pragma unroll
        for (int e = 0; e < VEC; ++e) dot += qv[e] * kx[e];
      }
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const float tt = 1.0f - r * (1.0f - dot);
      if (off >= 0 && tt > 0.f) {
        const float rel = (float)(j - t);
        const float m = 0.5f * (cosf(kPi * rel / w) + 1.0f);
        const float alpha = tt * tt * m;
        float vx[VEC];
        Vec16<T>::load(vp + off + sub * VEC, vx);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] += alpha * vx[e];
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
  for (int d = tid; d < D; d += 128) {
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NW; ++k) s2 += red[k][d];
    part[((long long)bh * a.num_splits + split) * D + d] = s2;
  }
}

// Sum the splits, TanhNorm, store y (B,H,D) and |o|.
template <typename T, int D>
__global__ void decode_finish_kernel(screen_decode_args a, const float* __restrict__ part) {
  __shared__ float red[D];
  const int bh = blockIdx.x, d = threadIdx.x;
  float o = 0.f;
  for (int s = 0; s < a.num_splits; ++s) o += part[((long long)bh * a.num_splits + s) * D + d];
  red[d] = o * o;
  __syncthreads();
  for (int st = D / 2; st > 0; st >>= 1) {
    if (d < st) red[d] += red[d + st];
    __syncthreads();
  }
  const float nraw = sqrtf(red[0]);
  const float g = tanhnorm_scale(nraw, a.eps);
  reinterpret_cast<T*>(a.y)[(long long)bh * D + d] = from_f<T>(o * g);
  if (d == 0 && a.no) a.no[bh] = nraw;
}

template <typename T, int D>
void launch_append(const screen_kv_append_args& a, cudaStream_t s) {
  constexpr int RPB = 256 / (D / 4);
  const long long rows = (long long)a.B * a.n_new * a.H;
  if (rows == 0) return;
  dim3 grid((unsigned)((rows + RPB - 1) / RPB), 2);
  kv_append_kernel<T, D><<<grid, 256, 0, s>>>(a);
}
template <typename T, int D>
void launch_decode(const screen_decode_args& a, float* part, cudaStream_t s) {
  if (a.B == 0 || a.H == 0) return;
  dim3 grid(a.num_splits, a.B * a.H);
  decode_split_kernel<T, D><<<grid, 128, 0, s>>>(a, part);
  decode_finish_kernel<T, D><<<a.B * a.H, D, 0, s>>>(a, part);
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
void decode(const screen_decode_args& a, float* part, cudaStream_t s) {
  const int dtype = a.dtype, D = a.D;
  DEC_DISPATCH(launch_decode, a, part, s);
}

}  // namespace screen
