// Few-row linear layer for the decode step: y = act(xin W^T) (+ res) with
// M <= 8 rows, bf16 weights streamed once from HBM (the step reads every
// weight of the model for a handful of tokens, so it is bandwidth-bound; a
// GEMM tile with M = B wastes most of its work and picks small-N kernels).
//
// CTA = 8 warps, one output feature n per warp: the CTA first stages the M
// input rows in shared memory as bf16 (optionally RMSNorm'ed: the CTA sums
// each row's squares itself -- M x K values from L2, tiny next to W), then
// each lane streams 16-byte chunks of its warp's weight row (K / 256 chunks
// per lane, all loads issued before the FMAs) against the staged rows, the
// warp sums the M dot products with shuffles, and lane m writes y[m, n]
// after GELU / residual.  Replaces nn.RMSNorm -> nn.Linear -> nn.GELU ->
// residual add of multiscreen/layers.py:60-76 for the decode step.
#include <cuda_bf16.h>
#include "rowops.cuh"

namespace screen {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ float gelu_erf(float v) {
  return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}

constexpr int kUnroll = 4;   // 16-byte weight chunks per lane in flight per row

// R: output features per warp (rows of W); R > 1 amortises the CTA's input
// staging over more weight rows for very wide layers (the lm_head)
template <int M, int R>
__global__ void __launch_bounds__(kWarps * 32) rows_linear_kernel(screen_rows_linear_args a) {
  extern __shared__ __align__(16) __nv_bfloat16 xs[];   // [M][K]
  __shared__ float red[M][kWarps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K;
  const long long nb = ((long long)blockIdx.x * kWarps + warp) * R;
  // the first weight chunks of this warp's rows are requested before the
  // input staging, so their HBM latency overlaps it
  uint4 wpre[R][kUnroll];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const bool rowok = nb + i < a.N;
    const __nv_bfloat16* wr = reinterpret_cast<const __nv_bfloat16*>(a.W) + (nb + i) * (long long)K;
#pragma unroll
    for (int uu = 0; uu < kUnroll; ++uu) {
      const int k = 8 * lane + 256 * uu;
      wpre[i][uu] = rowok && k < K ? __ldg(reinterpret_cast<const uint4*>(wr + k))
                                    : make_uint4(0, 0, 0, 0);
    }
  }
  // the weights are not written by the kernels before this one; the input
  // rows and the residual are
  pdl_wait();
  pdl_trigger();
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x);
  const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
  // ---- stage the input rows (RMSNorm'ed when norm_w is given)
  float inv[M];
#pragma unroll
  for (int m = 0; m < M; ++m) inv[m] = 1.0f;
  if (nw) {
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = 0.f;
    for (int k8 = tid; k8 < K / 8; k8 += blockDim.x) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + m * a.x_stride + 8 * k8);
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(w4[e]);
          ss[m] = fmaf(f.x, f.x, fmaf(f.y, f.y, ss[m]));
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(ss[m]);
      if (lane == 0) red[m][warp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float t = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kWarps; ++w2) t += red[m][w2];
      inv[m] = rsqrtf(t / (float)K + a.norm_eps);
    }
  }
  for (int k8 = tid; k8 < K / 8; k8 += blockDim.x) {
    uint4 g = make_uint4(0, 0, 0, 0);
    if (nw) g = *reinterpret_cast<const uint4*>(nw + 8 * k8);
    const uint32_t g4[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int m = 0; m < M; ++m) {
      uint4 u = *reinterpret_cast<const uint4*>(x + m * a.x_stride + 8 * k8);
      if (nw) {
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // torch's fused RMSNorm: x * rsqrt(mean(x^2) + eps) * weight in
          // fp32, rounded once
          const float2 f = unpack_bf16(w4[e]), gf = unpack_bf16(g4[e]);
          o4[e] = pack_bf16(f.x * inv[m] * gf.x, f.y * inv[m] * gf.y);
        }
        u = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      *reinterpret_cast<uint4*>(xs + m * K + 8 * k8) = u;
    }
  }
  __syncthreads();
  // ---- R weight rows per warp
  if (nb >= a.N) return;
  float acc[R][M];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[i][m] = 0.f;
  for (int k0 = 8 * lane; k0 < K; k0 += 256 * kUnroll) {
    uint4 wv[R][kUnroll];
    if (k0 == 8 * lane) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int uu = 0; uu < kUnroll; ++uu) wv[i][uu] = wpre[i][uu];
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const bool rowok = nb + i < a.N;
        const __nv_bfloat16* wr =
            reinterpret_cast<const __nv_bfloat16*>(a.W) + (nb + i) * (long long)K;
#pragma unroll
        for (int uu = 0; uu < kUnroll; ++uu) {
          const int k = k0 + 256 * uu;
          wv[i][uu] = rowok && k < K ? __ldg(reinterpret_cast<const uint4*>(wr + k))
                                     : make_uint4(0, 0, 0, 0);
        }
      }
    }
#pragma unroll
    for (int uu = 0; uu < kUnroll; ++uu) {
      const int k = k0 + 256 * uu;
      if (k >= K) break;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * K + k);
        const uint32_t x4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const uint32_t w4[4] = {wv[i][uu].x, wv[i][uu].y, wv[i][uu].z, wv[i][uu].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 wf = unpack_bf16(w4[e]), xf = unpack_bf16(x4[e]);
            acc[i][m] = fmaf(wf.x, xf.x, fmaf(wf.y, xf.y, acc[i][m]));
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const long long n = nb + i;
#pragma unroll
    for (int m = 0; m < M; ++m) acc[i][m] = warp_sum(acc[i][m]);
    if (n < a.N && lane < M) {
      float v = acc[i][0];
#pragma unroll
      for (int m = 1; m < M; ++m)
        if (lane == m) v = acc[i][m];
      if (a.act == 1) v = __bfloat162float(__float2bfloat16_rn(v)), v = gelu_erf(v);
      __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(a.y) + lane * a.y_stride + n;
      if (a.res) {
        // torch: bf16(linear) + bf16(res), rounded once more
        v = __bfloat162float(__float2bfloat16_rn(v)) +
            __bfloat162float(
                reinterpret_cast<const __nv_bfloat16*>(a.res)[lane * a.res_stride + n]);
      }
      *yp = __float2bfloat16_rn(v);
    }
  }
}

template <int M, int R>
int launch_rows_linear_r(const screen_rows_linear_args& a, cudaStream_t st) {
  const size_t smem = (size_t)M * a.K * 2;
  // one opt-in per device at the 200 KB maximum covers every K
  if (smem > 48 * 1024) {
    const cudaError_t e = ensure_smem_optin((const void*)rows_linear_kernel<M, R>, 200 * 1024);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  const long long per_cta = (long long)kWarps * R;
  const unsigned grid = (unsigned)((a.N + per_cta - 1) / per_cta);
  // a failed launch leaves its error for check_launch
  launch_pdl(rows_linear_kernel<M, R>, dim3(grid), dim3(kWarps * 32), smem, st, a);
  return check_launch();
}

// wide layers (the vocabulary projection) take 4 rows per warp
template <int M>
int launch_rows_linear(const screen_rows_linear_args& a, cudaStream_t st) {
  return a.N >= 16384 ? launch_rows_linear_r<M, 4>(a, st) : launch_rows_linear_r<M, 1>(a, st);
}

}  // namespace
}  // namespace screen

extern "C" int screen_rows_linear(const screen_rows_linear_args* a, screen_stream_t stream) {
  using namespace screen;
  if (!a) return SCREEN_ERR_INVALID_ARG;
  if (a->M < 0 || a->M > 8 || a->N < 0 || a->K <= 0 || (a->K % 8) != 0 ||
      (a->act != 0 && a->act != 1))
    return SCREEN_ERR_INVALID_ARG;
  if (a->M == 0 || a->N == 0) return SCREEN_OK;
  if (!a->x || !a->W || !a->y) return SCREEN_ERR_INVALID_ARG;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a->x) || !al16(a->W) || (a->norm_w && !al16(a->norm_w)) || (a->x_stride % 8) != 0)
    return SCREEN_ERR_ALIGNMENT;
  if ((size_t)a->M * a->K * 2 > 200 * 1024) return SCREEN_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->M) {
    case 1: return launch_rows_linear<1>(*a, st);
    case 2: return launch_rows_linear<2>(*a, st);
    case 3: return launch_rows_linear<3>(*a, st);
    case 4: return launch_rows_linear<4>(*a, st);
    case 5: return launch_rows_linear<5>(*a, st);
    case 6: return launch_rows_linear<6>(*a, st);
    case 7: return launch_rows_linear<7>(*a, st);
    default: return launch_rows_linear<8>(*a, st);
  }
}
