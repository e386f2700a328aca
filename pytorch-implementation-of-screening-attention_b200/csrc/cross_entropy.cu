// Cross-entropy of the LM loss (multiscreen/model.py:103-107) straight from
// the bf16 logits: one pass for the forward (online max / sum of exp per
// row, fp32) and one for the backward (softmax - onehot, scaled, written as
// bf16).  The unfused PyTorch path first copies the (tokens x vocabulary)
// logits to fp32 and runs log-softmax and NLL over them in several passes.
// CTA = one row, 256 threads, 16-byte loads.
#include <cuda_bf16.h>
#include "rowops.cuh"

namespace screen {
namespace {

constexpr int kT = 256;

// Raised (SCREEN_ERR_INVALID_ARG) by the forward when a label is neither
// ignore_index nor in [0, V).  F.cross_entropy stops with a device assert
// there; this kernel gives such a row loss 0 and gradient 0 (the Python
// caller leaves it out of the mean's denominator) and reports it through
// screen_device_status().
__device__ int g_xent_status = 0;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;   // both empty
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

__global__ void __launch_bounds__(kT) xent_fwd_kernel(screen_xent_args a) {
  const long long row = blockIdx.x;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.logits) + row * a.ld;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < a.V / 8; c += kT) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + 8 * c);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(w4[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
    float cm = v[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) cm = fmaxf(cm, v[e]);
    float cs = 0.f;
    if (cm != -INFINITY) {
#pragma unroll
      for (int e = 0; e < 8; ++e) cs += expf(v[e] - cm);
    }
    online_merge(m, s, cm, cs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[kT / 32], ss[kT / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < kT / 32; ++w) online_merge(M, S, sm[w], ss[w]);
    const float lse = M + logf(S);
    a.lse[row] = lse;
    const long long lab = a.labels[row];
    const bool out_of_range = lab < 0 || lab >= a.V;
    if (out_of_range && lab != a.ignore_index) atomicExch(&g_xent_status, (int)SCREEN_ERR_INVALID_ARG);
    a.loss[row] = (lab == a.ignore_index || out_of_range) ? 0.f : lse - __bfloat162float(x[lab]);
  }
}

__global__ void __launch_bounds__(kT) xent_bwd_kernel(screen_xent_args a) {
  const long long row = blockIdx.x;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.logits) + row * a.ld;
  __nv_bfloat16* dx = reinterpret_cast<__nv_bfloat16*>(a.dlogits) + row * a.dld;
  const long long lab = a.labels[row];
  const bool ign = lab == a.ignore_index || lab < 0 || lab >= a.V;
  const float sc = ign ? 0.f : *a.dscale, lse = a.lse[row];
  for (int c = threadIdx.x; c < a.V / 8; c += kT) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + 8 * c);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(w4[e]);
      const long long j = 8LL * c + 2 * e;
      const float g0 = (expf(f.x - lse) - (j == lab ? 1.f : 0.f)) * sc;
      const float g1 = (expf(f.y - lse) - (j + 1 == lab ? 1.f : 0.f)) * sc;
      o4[e] = pack_bf16(g0, g1);
    }
    *reinterpret_cast<uint4*>(dx + 8 * c) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

int xent_check(const screen_xent_args* a, bool bwd) {
  if (!a || a->rows < 0 || a->V <= 0 || (a->V % 8) != 0) return SCREEN_ERR_INVALID_ARG;
  if (a->rows == 0) return SCREEN_OK;
  if (!a->logits || !a->labels || !a->lse || (!bwd && !a->loss) ||
      (bwd && (!a->dlogits || !a->dscale)))
    return SCREEN_ERR_INVALID_ARG;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a->logits) || (a->ld % 8) != 0 || (bwd && (!al16(a->dlogits) || (a->dld % 8) != 0)))
    return SCREEN_ERR_ALIGNMENT;
  if (a->rows > 0x7fffffffLL) return SCREEN_ERR_UNSUPPORTED;
  return 1;
}

}  // namespace

int xent_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_xent_status, sizeof(int)) != cudaSuccess) return SCREEN_ERR_CUDA;
  if (clear && v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_xent_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace screen

extern "C" int screen_cross_entropy_fwd(const screen_xent_args* a, screen_stream_t stream) {
  using namespace screen;
  const int st = xent_check(a, false);
  if (st != 1) return st;
  xent_fwd_kernel<<<(unsigned)a->rows, kT, 0, (cudaStream_t)stream>>>(*a);
  return check_launch();
}

extern "C" int screen_cross_entropy_bwd(const screen_xent_args* a, screen_stream_t stream) {
  using namespace screen;
  const int st = xent_check(a, true);
  if (st != 1) return st;
  xent_bwd_kernel<<<(unsigned)a->rows, kT, 0, (cudaStream_t)stream>>>(*a);
  return check_launch();
}
