// Shared device helpers for the Screening Attention kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "../../include/screening_b200.h"

namespace screen {

// ---------------------------------------------------------------------------
// Element access
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Window arithmetic.  The softmask of attention.py:117-118 keeps key j for the
// query at key-axis position p iff  -w < (j - p) <= 0  (causal) or
// |j - p| < w (non-causal, attention.py:182).  With d = p - j an integer this
// is  0 <= d <= dmax  (resp. |d| <= dmax)  for dmax = ceil(w) - 1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int window_dmax(float w) {
  float c = ceilf(w) - 1.0f;
  if (!(c >= 0.0f)) return -1;           // w <= 0 or NaN: empty window
  if (c > 1.0e9f) return 1000000000;     // effectively unbounded
  return (int)c;
}

// Key index range [lo, hi] (inclusive, clipped to [0,Tk)) any query with
// key-axis position in [p0, p1] can see.
__device__ __forceinline__ void key_range(long long p0, long long p1, int dmax, bool causal,
                                          int Tk, long long& lo, long long& hi) {
  lo = p0 - dmax;
  hi = causal ? p1 : p1 + dmax;
  if (lo < 0) lo = 0;
  if (hi > Tk - 1) hi = Tk - 1;
}
// Query-position range [lo, hi] (key-axis positions) that can see any key in [j0, j1].
__device__ __forceinline__ void query_pos_range(long long j0, long long j1, int dmax, bool causal,
                                                long long& lo, long long& hi) {
  lo = causal ? j0 : j0 - dmax;
  hi = j1 + dmax;
}

// ---------------------------------------------------------------------------
// Tensor-core primitives (mma.sync m16n8k16 bf16 -> fp32, ldmatrix, cp.async)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  int n = pred ? 16 : 0;  // src-size 0 => zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// Swizzled shared-memory tile of ROWS x D bf16 (rows of 2*D bytes, 16-byte
// chunks XOR-permuted by row so that ldmatrix row fetches hit distinct banks).
template <int D>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return (uint32_t)(row * (D * 2) + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------------------
// TanhNorm scalar pieces (norm.py:24-25): g(n) = tanh(n)/n with n clamped at
// eps, and  (g'(n)/n) / g(n)^2  for the backward (series near 0 avoids the
// cancellation of (1 - tanh^2)/n - tanh/n^2).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tanhnorm_scale(float nraw, float eps) {
  float n = fmaxf(nraw, eps);
  return tanhf(n) / n;
}
// Returns c such that dO = g*dY + c * (Y.dY) * Y, where Y = g*O, for |O| > eps.
__device__ __forceinline__ float tanhnorm_bwd_coef(float n) {
  float g, gp_over_n;
  if (n < 0.05f) {
    float n2 = n * n;
    g = 1.0f + n2 * (-1.0f / 3.0f + n2 * (2.0f / 15.0f - n2 * (17.0f / 315.0f)));
    gp_over_n = -2.0f / 3.0f + n2 * (8.0f / 15.0f - n2 * (102.0f / 315.0f));
  } else {
    float t = tanhf(n);
    g = t / n;
    gp_over_n = ((1.0f - t * t) / n - t / (n * n)) / n;
  }
  return gp_over_n / (g * g);
}

}  // namespace screen
