// Row-wise kernels: the clamped row norms of q/k/v that the unit-normalisation
// of attention.py:156-158 divides by,
// stand-alone TanhNorm forward/backward (norm.py:23-25), the TanhNorm
// backward prologue of the attention backward, and the deterministic
// per-head reduction of the dr / dw partials.
#include "rowops.cuh"

namespace screen {

// 4 consecutive elements <-> float4
template <typename T> struct Vec4;
template <> struct Vec4<float> {
  static __device__ __forceinline__ float4 load(const float* p) {
    return *reinterpret_cast<const float4*>(p);
  }
  static __device__ __forceinline__ void store(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
  }
};
template <> struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ float4 load(const __nv_bfloat16* p) {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float4 v) {
    uint2 u;
    u.x = pack_bf16(v.x, v.y);
    u.y = pack_bf16(v.z, v.w);
    *reinterpret_cast<uint2*>(p) = u;
  }
};

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Clamped row norms max(|x|, eps) of up to three (B,T,H,D) tensors; one group
// of G = D/4 lanes per row, blockIdx.y selects the tensor.
template <typename T, int D>
__global__ void row_norms_kernel(NormJob job0, NormJob job1, NormJob job2, int njobs, float eps) {
  constexpr int G = D / 4;
  constexpr int RPB = 256 / G;  // rows per block
  if ((int)blockIdx.y >= njobs) return;
  const NormJob& job = blockIdx.y == 0 ? job0 : (blockIdx.y == 1 ? job1 : job2);
  long long row = (long long)blockIdx.x * RPB + threadIdx.x / G;
  int lane = threadIdx.x % G;
  long long nrows = (long long)job.B * job.T * job.H;
  bool valid = row < nrows;
  long long rr = valid ? row : 0;
  long long h = rr % job.H;
  long long t = (rr / job.H) % job.T;
  long long b = rr / ((long long)job.H * job.T);
  const T* src = reinterpret_cast<const T*>(job.x.p) + b * job.x.sb + t * job.x.st + h * D +
                 lane * 4;
  float4 v = valid ? Vec4<T>::load(src) : make_float4(0.f, 0.f, 0.f, 0.f);
  float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  ss = group_sum<G>(ss);
  if (valid && lane == 0) job.norms[rr] = fmaxf(sqrtf(ss), eps);
}

template <typename T, int D>
static void launch_row_norms(const NormJob* jobs, int njobs, float eps, cudaStream_t s) {
  constexpr int G = D / 4;
  constexpr int RPB = 256 / G;
  long long maxrows = 0;
  for (int i = 0; i < njobs; ++i) {
    long long n = (long long)jobs[i].B * jobs[i].T * jobs[i].H;
    if (n > maxrows) maxrows = n;
  }
  if (maxrows == 0) return;
  dim3 grid((unsigned)((maxrows + RPB - 1) / RPB), njobs);
  NormJob j1 = njobs > 1 ? jobs[1] : jobs[0];
  NormJob j2 = njobs > 2 ? jobs[2] : jobs[0];
  row_norms_kernel<T, D><<<grid, 256, 0, s>>>(jobs[0], j1, j2, njobs, eps);
}

void row_norms(int dtype, int D, const NormJob* jobs, int njobs, float eps, cudaStream_t s) {
#define NORM_CASE(TT, DD) launch_row_norms<TT, DD>(jobs, njobs, eps, s)
  if (dtype == SCREEN_F32) {
    switch (D) {
      case 16: NORM_CASE(float, 16); break;
      case 32: NORM_CASE(float, 32); break;
      case 64: NORM_CASE(float, 64); break;
      case 128: NORM_CASE(float, 128); break;
    }
  } else {
    switch (D) {
      case 16: NORM_CASE(__nv_bfloat16, 16); break;
      case 32: NORM_CASE(__nv_bfloat16, 32); break;
      case 64: NORM_CASE(__nv_bfloat16, 64); break;
      case 128: NORM_CASE(__nv_bfloat16, 128); break;
    }
  }
#undef NORM_CASE
}

// ---------------------------------------------------------------------------
// Stand-alone TanhNorm over contiguous rows of any length D (norm.py:23-25):
// one warp per row, two passes over the row.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void tanhnorm_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, long long rows,
                                    int D, float eps) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps exit together
  const T* xr = x + row * D;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = to_f(xr[d]);
    ss += v * v;
  }
  const float g = tanhnorm_scale(sqrtf(warp_sum(ss)), eps);
  for (int d = lane; d < D; d += 32) y[row * D + d] = from_f<T>(to_f(xr[d]) * g);
}

// dx = g dy + [|x| > eps] g'(n)/n (x.dy) x
template <typename T>
__global__ void tanhnorm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                    T* __restrict__ dx, long long rows, int D, float eps) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * D;
  const T* dr = dy + row * D;
  float ss = 0.f, xd = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = to_f(xr[d]), g = to_f(dr[d]);
    ss += v * v;
    xd += v * g;
  }
  ss = warp_sum(ss);
  xd = warp_sum(xd);
  const float nraw = sqrtf(ss);
  const float g = tanhnorm_scale(nraw, eps);
  const float k = (nraw > eps) ? tanhnorm_bwd_coef(nraw) * g * g * xd : 0.f;
  for (int d = lane; d < D; d += 32)
    dx[row * D + d] = from_f<T>(g * to_f(dr[d]) + k * to_f(xr[d]));
}

void tanhnorm(int dtype, int D, bool bwd, const void* x, const void* dy, void* out,
              long long rows, float eps, cudaStream_t s) {
  if (rows == 0) return;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (dtype == SCREEN_F32) {
    if (!bwd)
      tanhnorm_fwd_kernel<float><<<grid, 256, 0, s>>>((const float*)x, (float*)out, rows, D, eps);
    else
      tanhnorm_bwd_kernel<float><<<grid, 256, 0, s>>>((const float*)x, (const float*)dy,
                                                      (float*)out, rows, D, eps);
  } else {
    typedef __nv_bfloat16 bf;
    if (!bwd)
      tanhnorm_fwd_kernel<bf><<<grid, 256, 0, s>>>((const bf*)x, (bf*)out, rows, D, eps);
    else
      tanhnorm_bwd_kernel<bf><<<grid, 256, 0, s>>>((const bf*)x, (const bf*)dy, (bf*)out, rows,
                                                   D, eps);
  }
}

// ---------------------------------------------------------------------------
// Attention-backward prologue: G = dL/do from dL/dy through TanhNorm, using
// the saved output y = g o and the saved |o|, contiguous (B,Tq,H,D).
// split = false: G in fp32.  split = true (tensor-core path): two bf16
// planes G_hi = bf16(G) and G_lo = bf16(G - G_hi), rows*D elements apart, so
// G_hi + G_lo carries ~16 mantissa bits into the dP = G v^T GEMM.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void tanhnorm_grad_from_y_kernel(const T* __restrict__ y, const float* __restrict__ no,
                                            const T* __restrict__ dy, long long dy_sb,
                                            long long dy_st, void* __restrict__ G, bool split,
                                            int B, int T_, int H, float eps) {
  constexpr int Gl = D / 4;
  constexpr int RPB = 256 / Gl;
  long long row = (long long)blockIdx.x * RPB + threadIdx.x / Gl;
  int lane = threadIdx.x % Gl;
  long long rows = (long long)B * T_ * H;
  bool valid = row < rows;
  long long rr = valid ? row : 0;
  // dy row offset: rr * D when dy is contiguous (the usual case), else
  // (b, t, h) from rr -- in 32-bit when the row count allows (a 64-bit
  // division per thread costs more than the row's memory traffic)
  long long doff;
  if (dy_st == (long long)H * D && dy_sb == (long long)T_ * H * D) {
    doff = rr * D;
  } else if (rows < (1ll << 31)) {
    const unsigned r32 = (unsigned)rr, hh = r32 % (unsigned)H, bt = r32 / (unsigned)H;
    doff = (long long)(bt / (unsigned)T_) * dy_sb + (long long)(bt % (unsigned)T_) * dy_st +
           (long long)hh * D;
  } else {
    const long long h = rr % H, t = (rr / H) % T_, b = rr / ((long long)H * T_);
    doff = b * dy_sb + t * dy_st + h * D;
  }
  float4 yv = valid ? Vec4<T>::load(y + rr * D + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 d = valid ? Vec4<T>::load(dy + doff + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
  float yd = group_sum<Gl>(yv.x * d.x + yv.y * d.y + yv.z * d.z + yv.w * d.w);
  float nraw = valid ? no[rr] : 0.f;
  float g = tanhnorm_scale(nraw, eps);
  float k = (nraw > eps) ? tanhnorm_bwd_coef(nraw) * yd : 0.f;
  if (!valid) return;
  const float4 gv = make_float4(g * d.x + k * yv.x, g * d.y + k * yv.y, g * d.z + k * yv.z,
                                g * d.w + k * yv.w);
  if (!split) {
    Vec4<float>::store(reinterpret_cast<float*>(G) + rr * D + lane * 4, gv);
  } else {
    __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(G);
    const float4 h4 = make_float4(__bfloat162float(__float2bfloat16_rn(gv.x)),
                                  __bfloat162float(__float2bfloat16_rn(gv.y)),
                                  __bfloat162float(__float2bfloat16_rn(gv.z)),
                                  __bfloat162float(__float2bfloat16_rn(gv.w)));
    Vec4<__nv_bfloat16>::store(hi + rr * D + lane * 4, h4);
    Vec4<__nv_bfloat16>::store(hi + rows * D + rr * D + lane * 4,
                               make_float4(gv.x - h4.x, gv.y - h4.y, gv.z - h4.z, gv.w - h4.w));
  }
}

// bf16 rows split into hi / lo planes (the tensor-core path): 16-byte
// accesses, D / 8 lanes per row, contiguous dy; each thread handles kRows rows
// (a block's row range, kRows apart) with all loads issued before any math
template <int D>
__global__ void __launch_bounds__(256) tanhnorm_grad_split_bf16_kernel(
    const __nv_bfloat16* __restrict__ y, const float* __restrict__ no,
    const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ G, long long rows,
    float eps) {
  constexpr int L = D / 8;
  constexpr int RPB = 256 / L;
  constexpr int kRows = 2;
  const int lane = threadIdx.x % L;
  const long long row0 = (long long)blockIdx.x * RPB * kRows + threadIdx.x / L;
  uint4 yu[kRows], du[kRows];
  float nr[kRows];
#pragma unroll
  for (int u = 0; u < kRows; ++u) {
    const long long row = row0 + (long long)u * RPB;
    const bool valid = row < rows;
    const long long off = (valid ? row : 0) * D + lane * 8;
    yu[u] = valid ? *reinterpret_cast<const uint4*>(y + off) : make_uint4(0, 0, 0, 0);
    du[u] = valid ? *reinterpret_cast<const uint4*>(dy + off) : make_uint4(0, 0, 0, 0);
    nr[u] = valid ? no[row] : 0.f;
  }
#pragma unroll
  for (int u = 0; u < kRows; ++u) {
    const long long row = row0 + (long long)u * RPB;
    const bool valid = row < rows;
    const uint32_t yw[4] = {yu[u].x, yu[u].y, yu[u].z, yu[u].w};
    const uint32_t dw[4] = {du[u].x, du[u].y, du[u].z, du[u].w};
    float yf[8], df[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a2 = unpack_bf16(yw[e]), b2 = unpack_bf16(dw[e]);
      yf[2 * e] = a2.x; yf[2 * e + 1] = a2.y;
      df[2 * e] = b2.x; df[2 * e + 1] = b2.y;
    }
    float yd = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) yd = fmaf(yf[e], df[e], yd);
    yd = group_sum<L>(yd);
    const float g = tanhnorm_scale(nr[u], eps);
    const float k = (nr[u] > eps) ? tanhnorm_bwd_coef(nr[u]) * yd : 0.f;
    if (!valid) continue;
    const long long off = row * D + lane * 8;
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float g0 = fmaf(g, df[2 * e], k * yf[2 * e]);
      const float g1 = fmaf(g, df[2 * e + 1], k * yf[2 * e + 1]);
      hw[e] = pack_bf16(g0, g1);
      const float2 hf = unpack_bf16(hw[e]);
      lw[e] = pack_bf16(g0 - hf.x, g1 - hf.y);
    }
    *reinterpret_cast<uint4*>(G + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(G + rows * D + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

template <typename T, int D>
static void launch_grad_from_y(const void* y, const float* no, const void* dy, long long sb,
                               long long st, void* G, bool split, int B, int T_, int H, float eps,
                               cudaStream_t s) {
  constexpr int RPB = 256 / (D / 4);
  long long rows = (long long)B * T_ * H;
  if (rows == 0) return;
  if constexpr (sizeof(T) == 2 && D % 8 == 0 && D <= 256) {
    if (split && st == (long long)H * D && sb == (long long)T_ * H * D &&
        (reinterpret_cast<uintptr_t>(dy) & 15) == 0) {
      constexpr int RPB8 = 256 / (D / 8) * 2;   // rows per block: 2 per thread
      tanhnorm_grad_split_bf16_kernel<D><<<(unsigned)((rows + RPB8 - 1) / RPB8), 256, 0, s>>>(
          (const __nv_bfloat16*)y, no, (const __nv_bfloat16*)dy, (__nv_bfloat16*)G, rows, eps);
      return;
    }
  }
  tanhnorm_grad_from_y_kernel<T, D><<<(unsigned)((rows + RPB - 1) / RPB), 256, 0, s>>>(
      (const T*)y, no, (const T*)dy, sb, st, G, split, B, T_, H, eps);
}

void tanhnorm_grad_from_y(int dtype, int D, const void* y, const float* no, const void* dy,
                          long long dy_sb, long long dy_st, void* G, bool split, int B, int T_,
                          int H, float eps, cudaStream_t s) {
#define GY_CASE(TT, DD) \
  launch_grad_from_y<TT, DD>(y, no, dy, dy_sb, dy_st, G, split, B, T_, H, eps, s)
  if (dtype == SCREEN_F32) {
    switch (D) {
      case 16: GY_CASE(float, 16); break;
      case 32: GY_CASE(float, 32); break;
      case 64: GY_CASE(float, 64); break;
      case 128: GY_CASE(float, 128); break;
    }
  } else {
    switch (D) {
      case 16: GY_CASE(__nv_bfloat16, 16); break;
      case 32: GY_CASE(__nv_bfloat16, 32); break;
      case 64: GY_CASE(__nv_bfloat16, 64); break;
      case 128: GY_CASE(__nv_bfloat16, 128); break;
    }
  }
#undef GY_CASE
}

// ---------------------------------------------------------------------------
// dr[h] = sum_p part_r[h][p];  dw[h] = pi / (2 w^2) * sum_p part_w[h][p].
// Fixed summation order => deterministic.
// ---------------------------------------------------------------------------
__global__ void reduce_param_grads_kernel(const float* __restrict__ part_r,
                                          const float* __restrict__ part_w, long long P,
                                          const float* __restrict__ w, float* __restrict__ dr,
                                          float* __restrict__ dw) {
  int h = blockIdx.x;
  __shared__ float sr[256], sw[256];
  float ar = 0.f, aw = 0.f;
  for (long long p = threadIdx.x; p < P; p += 256) {
    ar += part_r[(long long)h * P + p];
    aw += part_w[(long long)h * P + p];
  }
  sr[threadIdx.x] = ar;
  sw[threadIdx.x] = aw;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      sr[threadIdx.x] += sr[threadIdx.x + s];
      sw[threadIdx.x] += sw[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float wh = w[h];
    dr[h] = sr[0];
    dw[h] = sw[0] * (3.14159265358979323846f / (2.0f * wh * wh));
  }
}

void reduce_param_grads(const float* part_r, const float* part_w, long long P, int H,
                        const float* w, float* dr, float* dw, cudaStream_t s) {
  reduce_param_grads_kernel<<<H, 256, 0, s>>>(part_r, part_w, P, w, dr, dw);
}

// ---------------------------------------------------------------------------
// The module's parameter transforms r = exp(s_r) + 1, w = exp(s_v) + 1
// (attention.py:164-165) for all heads in one launch, and their backward
// ds = d exp(s) in the parameters' dtype (one thread per head and parameter).
// ---------------------------------------------------------------------------
namespace {
__device__ __forceinline__ float load_param(const void* p, int dtype, int i) {
  return dtype == SCREEN_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                              : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_param(void* p, int dtype, int i, float v) {
  if (dtype == SCREEN_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}
__global__ void head_params_fwd_kernel(int dtype, int H, const void* s_r, const void* s_v,
                                       float* r, float* w) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < H) r[i] = expf(load_param(s_r, dtype, i)) + 1.0f;
  else if (i < 2 * H) w[i - H] = expf(load_param(s_v, dtype, i - H)) + 1.0f;
}
__global__ void head_params_bwd_kernel(int dtype, int H, const void* s_r, const void* s_v,
                                       const float* dr, const float* dw, void* ds_r, void* ds_v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < H) {
    if (dr) store_param(ds_r, dtype, i, dr[i] * expf(load_param(s_r, dtype, i)));
  } else if (i < 2 * H) {
    if (dw) store_param(ds_v, dtype, i - H, dw[i - H] * expf(load_param(s_v, dtype, i - H)));
  }
}
}  // namespace

void head_params_fwd(int dtype, int H, const void* s_r, const void* s_v, float* r, float* w,
                     cudaStream_t s) {
  const int n = 2 * H, th = n < 256 ? ((n + 31) / 32) * 32 : 256;
  head_params_fwd_kernel<<<(n + th - 1) / th, th, 0, s>>>(dtype, H, s_r, s_v, r, w);
}

// ---------------------------------------------------------------------------
// Backward of Y = W diag(g) (a norm weight g folded into the columns of a
// projection W of `rows` x D): dW = dY diag(g), dg[c] = sum_o dY[o, c] W[o, c].
// CTA = 32 columns x 8 row slices, slices added in a fixed order.
// ---------------------------------------------------------------------------
namespace {
template <typename T>
__global__ void __launch_bounds__(256) col_scale_bwd_kernel(long long rows, int D, const T* dy,
                                                            const T* w, const T* g, T* dw, T* dg) {
  __shared__ float red[8][33];
  const int c = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + c;
  float acc = 0.f;
  if (d < D) {
    const float gc = to_f(g[d]);
    for (long long o = sl; o < rows; o += 8) {
      const long long at = o * D + d;
      const float v = to_f(dy[at]);
      if (dg) acc = fmaf(v, to_f(w[at]), acc);
      if (dw) dw[at] = from_f<T>(v * gc);
    }
  }
  red[sl][c] = acc;
  __syncthreads();
  if (dg && sl == 0 && d < D) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][c];
    dg[d] = from_f<T>(t);
  }
}
}  // namespace

void col_scale_bwd(int dtype, long long rows, int D, const void* dy, const void* w,
                   const void* g, void* dw, void* dg, cudaStream_t s) {
  const unsigned grid = (unsigned)((D + 31) / 32);
  if (dtype == SCREEN_BF16) {
    typedef __nv_bfloat16 bf;
    col_scale_bwd_kernel<bf><<<grid, 256, 0, s>>>(
        rows, D, static_cast<const bf*>(dy), static_cast<const bf*>(w), static_cast<const bf*>(g),
        static_cast<bf*>(dw), static_cast<bf*>(dg));
  } else {
    col_scale_bwd_kernel<float><<<grid, 256, 0, s>>>(
        rows, D, static_cast<const float*>(dy), static_cast<const float*>(w),
        static_cast<const float*>(g), static_cast<float*>(dw), static_cast<float*>(dg));
  }
}

void head_params_bwd(int dtype, int H, const void* s_r, const void* s_v, const float* dr,
                     const float* dw, void* ds_r, void* ds_v, cudaStream_t s) {
  const int n = 2 * H, th = n < 256 ? ((n + 31) / 32) * 32 : 256;
  head_params_bwd_kernel<<<(n + th - 1) / th, th, 0, s>>>(dtype, H, s_r, s_v, dr, dw, ds_r, ds_v);
}

// ---------------------------------------------------------------------------
// Longest-processing-time-first CTA order.  Under a causal window the CTAs of
// one launch carry very different numbers of tiles (a head with w = 4096 at
// the end of the sequence: 66 tiles; a head with w = 256: 6); launched in
// index order the longest ones can start last and leave the GPU idle at the
// tail.  The hardware dispatches CTAs roughly in blockIdx order, so a launch
// through perm runs the longest first.
// ---------------------------------------------------------------------------
namespace {
constexpr int kOrderBuckets = 1024;
__device__ __forceinline__ int item_tiles(const AttnShape& s, int kind, int ntiles, long long id) {
  const long long bh = id / ntiles;
  const int x = (int)(id % ntiles), h = (int)(bh % s.H);
  const int dmax = window_dmax(s.w[h]);
  if (dmax < 0) return 0;
  const bool causal = s.causal != 0;
  long long lo, hi;
  if (kind == 0) {
    const long long i0 = (long long)x * 128;
    long long il = i0 + 127;
    if (il > s.Tq - 1) il = s.Tq - 1;
    key_range(i0 + s.q_offset, il + s.q_offset, dmax, causal, s.Tk, lo, hi);
  } else {
    const long long j0 = (long long)x * 128;
    long long jl = j0 + 127;
    if (jl > s.Tk - 1) jl = s.Tk - 1;
    query_pos_range(j0, jl, dmax, causal, lo, hi);
    lo -= s.q_offset;
    hi -= s.q_offset;
    if (lo < 0) lo = 0;
    if (hi > s.Tq - 1) hi = s.Tq - 1;
  }
  if (lo > hi) return 0;
  const long long n = hi / 64 - lo / 64 + 1;
  return n > kOrderBuckets - 1 ? kOrderBuckets - 1 : (int)n;
}
// Sort key of a CTA.  Forward (kind 0): its own tile count.  Backward
// (kind 1): the count of its head's first key tile, so all key tiles of one
// head (every batch) sit together in the order, longest heads first.  The
// heads' windows differ by up to 16x, so the balance is that of
// longest-first; but the backward's live working set becomes the q, G and dq
// rows of about one head instead of every head: at cfg3 (B=8) the fused
// backward's DRAM traffic fell from 2.43 GB to 0.84 GB per launch (ncu) at
// the same duration.
__device__ __forceinline__ int order_key(const AttnShape& s, int kind, int ntiles, long long id) {
  return item_tiles(s, kind, ntiles, kind == 1 ? (id / ntiles) * ntiles : id);
}

__global__ void __launch_bounds__(1024) tile_order_kernel(AttnShape s, int kind, int ntiles,
                                                          long long N, int* perm) {
  __shared__ int cnt[kOrderBuckets];
  __shared__ int wsum[32];
  const int t = threadIdx.x;
  cnt[t] = 0;
  __syncthreads();
  for (long long id = t; id < N; id += blockDim.x)
    atomicAdd(&cnt[kOrderBuckets - 1 - order_key(s, kind, ntiles, id)], 1);
  __syncthreads();
  // exclusive prefix sum over the buckets (bucket 0 = most tiles)
  const int v = cnt[t];
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if ((t & 31) >= o) incl += u;
  }
  if ((t & 31) == 31) wsum[t >> 5] = incl;
  __syncthreads();
  if (t < 32) {
    int x = wsum[t];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, x, o);
      if (t >= o) x += u;
    }
    wsum[t] = x;   // inclusive over warps
  }
  __syncthreads();
  const int base = (t >> 5) ? wsum[(t >> 5) - 1] : 0;
  __syncthreads();
  cnt[t] = base + incl - v;
  __syncthreads();
  for (long long id = t; id < N; id += blockDim.x) {
    const int pos = atomicAdd(&cnt[kOrderBuckets - 1 - order_key(s, kind, ntiles, id)], 1);
    perm[pos] = (int)id;
  }
}
}  // namespace

void tile_order(const AttnShape& s, int kind, int ntiles, int* perm, cudaStream_t st) {
  const long long N = (long long)s.B * s.H * ntiles;
  if (N <= 0) return;
  tile_order_kernel<<<1, kOrderBuckets, 0, st>>>(s, kind, ntiles, N, perm);
}

}  // namespace screen
