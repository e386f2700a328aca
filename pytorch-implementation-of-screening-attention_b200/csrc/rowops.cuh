// Host-side declarations of the row-wise kernels (rowops.cu) and of the
// attention kernel launchers (attn_simt.cu, attn_mma.cu).
#pragma once
#include "common.cuh"

namespace screen {

// A (B,T,H,D) tensor with unit stride over D, stride D over H and free
// batch / time strides (elements).
struct Rows {
  const void* p;
  long long sb, st;
};
struct OutRows {
  void* p;
  long long sb, st;
};

struct NormJob {
  Rows x;
  int B, T, H;
  float* norms;        // contiguous (B,T,H): max(|x|, eps)
};

void row_norms(int dtype, int D, const NormJob* jobs, int njobs, float eps, cudaStream_t s);
void tanhnorm(int dtype, int D, bool bwd, const void* x, const void* dy, void* out,
              long long rows, float eps, cudaStream_t s);
void tanhnorm_grad_from_y(int dtype, int D, const void* y, const float* no, const void* dy,
                          long long dy_sb, long long dy_st, void* G, bool split, int B, int T_,
                          int H, float eps, cudaStream_t s);
void reduce_param_grads(const float* part_r, const float* part_w, long long P, int H,
                        const float* w, float* dr, float* dw, cudaStream_t s);
// backward of W diag(g): dW = dY diag(g) and dg = column sums of dY * W
// (dw or dg null: not written); rows x D row-major, all of one dtype
void col_scale_bwd(int dtype, long long rows, int D, const void* dy, const void* w,
                   const void* g, void* dw, void* dg, cudaStream_t s);
// r = exp(s_r) + 1, w = exp(s_v) + 1 per head; backward ds = d exp(s) (dr or
// dw null: that gradient is not written)
void head_params_fwd(int dtype, int H, const void* s_r, const void* s_v, float* r, float* w,
                     cudaStream_t s);
void head_params_bwd(int dtype, int H, const void* s_r, const void* s_v, const float* dr,
                     const float* dw, void* ds_r, void* ds_v, cudaStream_t s);

struct AttnShape {
  int B, H, Tq, Tk;
  int causal;
  long long q_offset;
  float eps;
  const float* r;
  const float* w;
  const uint8_t* kpm;   // (B,Tk) or null
  long long kpm_sb;
  // attention dropout: score (bh, i, j) dropped iff drop_bits(...) < drop_thr;
  // drop_thr = 0: none.  drop_scale = 2^32 / (2^32 - drop_thr) multiplies
  // every output that is linear in alpha (o before TanhNorm, dq, dk, dv, dr, dw)
  uint32_t drop_thr;
  float drop_scale;
  uint32_t seed_lo, seed_hi;
};

// Counter-based dropout bits (lowbias32 finalizer as the mixing function):
// key of (seed, bh), row key of query i, bits of score (i, j).  The same
// values on the host (screen_dropout_bits) and in every kernel family.
__host__ __device__ __forceinline__ uint32_t drop_mix(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
__host__ __device__ __forceinline__ uint32_t drop_bh_key(const AttnShape& s, uint32_t bh) {
  return drop_mix(s.seed_lo ^ drop_mix(s.seed_hi ^ (bh * 0x9E3779B1u)));
}
__host__ __device__ __forceinline__ uint32_t drop_row(uint32_t bhk, uint32_t i) {
  return drop_mix(bhk ^ (i * 0x85EBCA77u));
}
constexpr uint32_t kDropColMul = 0xC2B2AE3Du;   // bits = drop_mix(row ^ j * kDropColMul)
__host__ __device__ __forceinline__ bool drop_keep(uint32_t row, uint32_t j, uint32_t thr) {
  return drop_mix(row ^ (j * kDropColMul)) >= thr;
}

struct FwdPtrs {
  Rows q, k, v;
  const float* nq; const float* nk; const float* nv;
  void* y; float* no;   // contiguous
  int64_t* tile_stats;
};

struct BwdPtrs {
  Rows q, k, v;
  const float* nq; const float* nk; const float* nv;
  const void* G;          // dL/do, contiguous (B,Tq,H,D): fp32 (SIMT path) or
                          // bf16 hi plane followed by bf16 lo plane (tensor cores)
  OutRows dq, dk, dv;
  float* part_r; float* part_w;   // [H][P] partials
  float* dq_acc = nullptr;        // fp32 (B,Tq,H,D) dq^ accumulator (fused tensor-core path)
};

// Generic SIMT kernels (fp32 math; any dtype, any supported D).
void simt_fwd(int dtype, int D, const AttnShape& s, const FwdPtrs& p, cudaStream_t st);
long long simt_bwd_partials(const AttnShape& s);
void simt_bwd(int dtype, int D, const AttnShape& s, const BwdPtrs& p, int stages,
              cudaStream_t st);

// tcgen05 / TMEM forward (bf16, D = 64 or 128).
bool tc_supported(int dtype, int D);
size_t tc_fwd_workspace(const AttnShape& s, int D);
int tc_fwd(const AttnShape& s, const FwdPtrs& p, void* workspace, bool norms_given, int D,
           cudaStream_t st);
int tc_device_status(bool clear);
// tcgen05 / TMEM backward (bf16, D = 64 or 128); aux_ws holds
// tc_bwd_aux_bytes()
bool tc_bwd_supported(int dtype, int D);
size_t tc_bwd_aux_bytes(const AttnShape& s);
long long tc_bwd_partials(const AttnShape& s);
// Longest-first launch order of the tcgen05 kernels' CTAs: perm[i] is the
// work item (bh * ntiles + tile) that CTA i runs, sorted by decreasing tile
// count.  kind 0: query tiles of 128 (forward), kind 1: key tiles of 128
// (key-major backward).  One CTA, counting sort; perm holds B*H*ntiles ints.
void tile_order(const AttnShape& s, int kind, int ntiles, int* perm, cudaStream_t st);
int tc_bwd(const AttnShape& s, const BwdPtrs& p, void* aux_ws, int stages, int D, cudaStream_t st);
int tc_bwd_device_status(bool clear);

// bf16 warp-level mma.sync kernels (D = 64).
bool mma_supported(int dtype, int D);
void mma_fwd(int D, const AttnShape& s, const FwdPtrs& p, cudaStream_t st);
long long mma_bwd_partials(int D, const AttnShape& s);
void mma_bwd(int D, const AttnShape& s, const BwdPtrs& p, int stages, cudaStream_t st);

}  // namespace screen
