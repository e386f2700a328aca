// RMSNorm of the blocks' pre-norms (torch.nn.RMSNorm as used at
// multiscreen/layers.py:60-76 and model.py:98), forward and backward.
//
// Under bf16 autocast the residual stream is fp32, the norm computes in fp32
// and the Linear after it casts the result to bf16; the forward here writes
// that bf16 row directly (the same rounding, done once).  The backward's
// weight gradient is a column sum over every row; PyTorch's kernel for it
// was a tenth of the cfg2 training step.  Here each warp keeps its lanes'
// column sums in registers over the rows it handles, the CTA combines its
// warps in shared memory and writes one partial row, and a second pass sums
// the partial rows in a fixed order (deterministic).
//
// Layout: a warp per row; lane l owns the 8-element chunks l, l + 32, ...
// (16-byte loads for bf16, two for fp32).
#include <cuda_bf16.h>
#include "rowops.cuh"

namespace screen {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxBlocks = 148 * 4;

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack_bf16(w4[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
                                            pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

// NCH: 8-element chunks per lane (D <= 256 * NCH)
template <typename TX, typename TW, typename TY, int NCH>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(screen_rmsnorm_args a) {
  const int lane = threadIdx.x & 31;
  const int nch = a.D / 8;
  const TX* x = reinterpret_cast<const TX*>(a.x);
  const TW* w = reinterpret_cast<const TW*>(a.w);
  TY* y = reinterpret_cast<TY*>(a.y);
  for (long long row = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5); row < a.rows;
       row += (long long)gridDim.x * kWarps) {
    float v[NCH][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        load8<TX>(x + row * a.D + 8 * c, v[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)a.D + a.eps);
    if (lane == 0) a.rstd[row] = rs;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        float g[8], o[8];
        load8<TW>(w + 8 * c, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = v[i][e] * rs * g[e];
        store8<TY>(y + row * a.D + 8 * c, o);
      }
    }
  }
}

// rows of CTA blk: blk, blk + G, ... in steps of kWarps rows (fixed order)
template <typename TX, typename TW, typename TY, int NCH>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_kernel(screen_rmsnorm_args a) {
  extern __shared__ float wsum[];   // [kWarps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nch = a.D / 8;
  const TX* x = reinterpret_cast<const TX*>(a.x);
  const TW* w = reinterpret_cast<const TW*>(a.w);
  const TY* dy = reinterpret_cast<const TY*>(a.dy);
  TX* dx = reinterpret_cast<TX*>(a.dx);
  float gw[NCH][8], acc[NCH][8];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
    if (c < nch) load8<TW>(w + 8 * c, gw[i]);
  }
  for (long long row = (long long)blockIdx.x * kWarps + warp; row < a.rows;
       row += (long long)gridDim.x * kWarps) {
    const float rs = a.rstd[row];
    float xh[NCH][8], g[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        float xv[8], dv[8];
        load8<TX>(x + row * a.D + 8 * c, xv);
        load8<TY>(dy + row * a.D + 8 * c, dv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[i][e] = xv[e] * rs;
          g[i][e] = dv[e] * gw[i][e];
          acc[i][e] = fmaf(dv[e], xh[i][e], acc[i][e]);
          dot = fmaf(g[i][e], xh[i][e], dot);
        }
      }
    }
    dot = warp_sum(dot) / (float)a.D;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rs * (g[i][e] - xh[i][e] * dot);
        store8<TX>(dx + row * a.D + 8 * c, o);
      }
    }
  }
  // the CTA's column partial: its warps' sums in a fixed order
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
#pragma unroll
      for (int e = 0; e < 8; ++e) wsum[warp * a.D + 8 * c + e] = acc[i][e];
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) t += wsum[k * a.D + d];
    a.partials[(long long)blockIdx.x * a.D + d] = t;
  }
}

// dw[d] = sum of the nblk partial rows: CTA = 32 columns x 8 row slices
// (slice s sums partial rows s, s + 8, ...), the slices added in order, so
// the result is deterministic and the 600-odd partial rows are read by 8
// independent streams per column instead of one
template <typename TW>
__global__ void __launch_bounds__(256) rmsnorm_dw_kernel(screen_rmsnorm_args a, int nblk) {
  __shared__ float red[8][33];
  const int c = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + c;
  float t0 = 0.f, t1 = 0.f;
  if (d < a.D) {
    int b = sl;
    for (; b + 8 < nblk; b += 16) {
      t0 += a.partials[(long long)b * a.D + d];
      t1 += a.partials[(long long)(b + 8) * a.D + d];
    }
    if (b < nblk) t0 += a.partials[(long long)b * a.D + d];
  }
  red[sl][c] = t0 + t1;
  __syncthreads();
  if (sl == 0 && d < a.D) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][c];
    reinterpret_cast<TW*>(a.dw)[d] = from_f<TW>(t);
  }
}

int grid_for(long long rows) {
  const long long g = (rows + kWarps - 1) / kWarps;
  return (int)(g < kMaxBlocks ? g : kMaxBlocks);
}

int check_args(const screen_rmsnorm_args* a, bool bwd) {
  if (!a || a->rows < 0 || a->D <= 0 || a->D % 8 != 0) return SCREEN_ERR_INVALID_ARG;
  if (a->D > 256 * 8) return SCREEN_ERR_UNSUPPORTED;
  auto dt_ok = [](int t) { return t == SCREEN_F32 || t == SCREEN_BF16; };
  if (!dt_ok(a->x_dtype) || !dt_ok(a->w_dtype) || !dt_ok(a->y_dtype)) return SCREEN_ERR_DTYPE;
  if (a->y_dtype != SCREEN_BF16 && a->y_dtype != a->x_dtype) return SCREEN_ERR_DTYPE;
  if (a->rows == 0) return SCREEN_OK;
  if (!a->x || !a->w || !a->rstd || (!bwd && !a->y) ||
      (bwd && (!a->dy || !a->dx || !a->dw || !a->partials)))
    return SCREEN_ERR_INVALID_ARG;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a->x) || !al16(a->w) || (!bwd && !al16(a->y)) ||
      (bwd && (!al16(a->dy) || !al16(a->dx))))
    return SCREEN_ERR_ALIGNMENT;
  return 1;
}

template <typename TX, typename TW, typename TY, int NCH>
int run(const screen_rmsnorm_args& a, bool bwd, cudaStream_t st) {
  const int grid = grid_for(a.rows);
  if (!bwd) {
    rmsnorm_fwd_kernel<TX, TW, TY, NCH><<<grid, kWarps * 32, 0, st>>>(a);
    return check_launch();
  }
  const int smem = kWarps * a.D * 4;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        ensure_smem_optin((const void*)rmsnorm_bwd_kernel<TX, TW, TY, NCH>, kWarps * 2048 * 4);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  rmsnorm_bwd_kernel<TX, TW, TY, NCH><<<grid, kWarps * 32, smem, st>>>(a);
  rmsnorm_dw_kernel<TW><<<(a.D + 31) / 32, 256, 0, st>>>(a, grid);
  return check_launch();
}

template <typename TX, typename TW, typename TY>
int run_nch(const screen_rmsnorm_args& a, bool bwd, cudaStream_t st) {
  const int nch = (a.D / 8 + 31) / 32;
  if (nch <= 1) return run<TX, TW, TY, 1>(a, bwd, st);
  if (nch <= 2) return run<TX, TW, TY, 2>(a, bwd, st);
  if (nch <= 4) return run<TX, TW, TY, 4>(a, bwd, st);
  return run<TX, TW, TY, 8>(a, bwd, st);
}

int dispatch(const screen_rmsnorm_args* a, bool bwd, cudaStream_t st) {
  const int v = check_args(a, bwd);
  if (v != 1) return v;
  typedef __nv_bfloat16 bf;
  const bool xf = a->x_dtype == SCREEN_F32, wf = a->w_dtype == SCREEN_F32,
             yb = a->y_dtype == SCREEN_BF16;
  if (xf && wf) return yb ? run_nch<float, float, bf>(*a, bwd, st) : run_nch<float, float, float>(*a, bwd, st);
  if (xf && !wf) return yb ? run_nch<float, bf, bf>(*a, bwd, st) : run_nch<float, bf, float>(*a, bwd, st);
  if (!xf && wf) return run_nch<bf, float, bf>(*a, bwd, st);
  return run_nch<bf, bf, bf>(*a, bwd, st);
}

}  // namespace
}  // namespace screen

extern "C" int64_t screen_rmsnorm_partials(int64_t rows) {
  return rows <= 0 ? 1 : screen::grid_for(rows);
}
extern "C" int screen_rmsnorm_fwd(const screen_rmsnorm_args* a, screen_stream_t stream) {
  return screen::dispatch(a, false, (cudaStream_t)stream);
}
extern "C" int screen_rmsnorm_bwd(const screen_rmsnorm_args* a, screen_stream_t stream) {
  return screen::dispatch(a, true, (cudaStream_t)stream);
}
