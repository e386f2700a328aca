// extern "C" entry points of libscreening_b200.so (declared in
// include/screening_b200.h).  Validation, workspace carving and kernel
// dispatch; no allocation, no exceptions across the boundary.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "rowops.cuh"
#include "decode.cuh"

using namespace screen;

namespace {
thread_local char g_last_err[256] = "";
}  // namespace

namespace screen {
int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_last_err, sizeof(g_last_err), "%s", cudaGetErrorString(e));
    return SCREEN_ERR_LAUNCH;
  }
  return SCREEN_OK;
}
int record_cuda_error(cudaError_t e) {
  if (e == cudaSuccess) return SCREEN_OK;
  snprintf(g_last_err, sizeof(g_last_err), "%s", cudaGetErrorString(e));
  return SCREEN_ERR_CUDA;
}
}  // namespace screen

namespace {

bool dim_ok(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }
bool dtype_ok(int t) { return t == SCREEN_F32 || t == SCREEN_BF16; }
size_t elem_size(int t) { return t == SCREEN_F32 ? 4 : 2; }
bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
// raw (B,T,H,D) rows are read in 16-byte pieces
bool strides_ok(long long sb, long long st) { return sb % 4 == 0 && st % 4 == 0; }
bool raw_ok(int dtype, const void* p, long long sb, long long st) {
  const long long vec = 16 / (long long)elem_size(dtype);
  return al16(p) && sb % vec == 0 && st % vec == 0;
}
size_t round_up(size_t x) { return (x + 255) & ~(size_t)255; }

// Kernel family for bf16 D=64: the tcgen05 forward by default.  The
// environment variable SCREEN_KERNELS=mma|simt selects the warp-level mma.sync
// or the SIMT kernels instead -- a debugging aid for comparing implementations
// on identical inputs.
enum Family { FAM_TC, FAM_MMA, FAM_SIMT };
Family family_choice() {
  static const Family f = [] {
    const char* e = getenv("SCREEN_KERNELS");
    if (e && e[0] == 's') return FAM_SIMT;
    if (e && e[0] == 'm') return FAM_MMA;
    return FAM_TC;
  }();
  return f;
}
bool use_tc_fwd(int dtype, int D) { return family_choice() == FAM_TC && tc_supported(dtype, D); }
bool use_tc_bwd(int dtype, int D) { return family_choice() == FAM_TC && tc_bwd_supported(dtype, D); }
bool use_mma(int dtype, int D) { return family_choice() != FAM_SIMT && mma_supported(dtype, D); }
// the warp-level mma.sync kernels have no dropout; with dropout the SIMT family serves
bool use_mma_drop(int dtype, int D, uint32_t drop_thr) { return drop_thr == 0 && use_mma(dtype, D); }

int common_checks(int dtype, int B, int H, int Tq, int Tk, int D) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (!dim_ok(D)) return SCREEN_ERR_HEAD_DIM;
  if (B < 0 || H < 0 || Tq < 0 || Tk < 0) return SCREEN_ERR_INVALID_ARG;
  return SCREEN_OK;
}

AttnShape make_shape(int B, int H, int Tq, int Tk, int causal, long long q_offset, float eps,
                     const float* r, const float* w, const uint8_t* kpm, long long kpm_sb,
                     uint32_t drop_thr = 0, uint64_t seed = 0) {
  AttnShape s;
  s.B = B; s.H = H; s.Tq = Tq; s.Tk = Tk; s.causal = causal; s.q_offset = q_offset;
  s.eps = eps; s.r = r; s.w = w; s.kpm = kpm; s.kpm_sb = kpm_sb;
  s.drop_thr = drop_thr;
  s.drop_scale = drop_thr ? (float)(4294967296.0 / (4294967296.0 - (double)drop_thr)) : 1.0f;
  s.seed_lo = (uint32_t)seed;
  s.seed_hi = (uint32_t)(seed >> 32);
  return s;
}

struct BwdLayout {
  size_t g_off, pr_off, pw_off, aux_off, total;
  long long P;
};
BwdLayout bwd_layout(const screen_bwd_args* a) {
  BwdLayout L;
  AttnShape s = make_shape(a->B, a->H, a->Tq, a->Tk, a->causal, a->q_offset, a->eps, a->r, a->w,
                           a->key_padding_mask, a->kpm_sb, a->dropout_threshold,
                           a->dropout_seed);
  const bool tc = use_tc_bwd(a->dtype, a->D);
  L.P = tc ? tc_bwd_partials(s)
           : (use_mma_drop(a->dtype, a->D, a->dropout_threshold) ? mma_bwd_partials(a->D, s) : simt_bwd_partials(s));
  L.g_off = 0;
  // G: fp32, or two bf16 planes (hi, lo) on the tensor-core path -- 4 bytes/elem either way
  L.pr_off = round_up((size_t)a->B * a->Tq * a->H * a->D * 4);
  L.pw_off = L.pr_off + round_up((size_t)a->H * L.P * sizeof(float));
  L.aux_off = L.pw_off + round_up((size_t)a->H * L.P * sizeof(float));
  L.total = L.aux_off + (tc ? round_up(tc_bwd_aux_bytes(s)) : 0);
  return L;
}

}  // namespace

extern "C" {

int screen_version(void) { return SCREEN_ABI_VERSION; }

const char* screen_last_cuda_error(void) { return g_last_err; }

const char* screen_strerror(int status) {
  switch (status) {
    case SCREEN_OK: return "success";
    case SCREEN_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or bad flag)";
    case SCREEN_ERR_HEAD_DIM: return "unsupported head dim (supported: 16, 32, 64, 128)";
    case SCREEN_ERR_DTYPE: return "unsupported dtype (supported: float32, bfloat16)";
    case SCREEN_ERR_ALIGNMENT: return "pointer not 16-byte aligned or stride not a multiple of 4 elements";
    case SCREEN_ERR_WORKSPACE: return "workspace missing or smaller than the size query returned";
    case SCREEN_ERR_LAUNCH: return "kernel launch failed (see screen_last_cuda_error)";
    case SCREEN_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case SCREEN_ERR_CUDA: return "CUDA runtime error (see screen_last_cuda_error)";
    case SCREEN_ERR_UNSUPPORTED: return "request not supported by this build";
    case SCREEN_ERR_SCRATCH_LIMIT:
      return "request needs more than the static scratch of screen_decode_noalloc "
             "(B * H * num_splits * D * 4 bytes must be <= SCREEN_DECODE_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown status";
  }
}

int64_t screen_sizeof_args(int which) {
  switch (which) {
    case 0: return (int64_t)sizeof(screen_fwd_args);
    case 1: return (int64_t)sizeof(screen_bwd_args);
    case 2: return (int64_t)sizeof(screen_kv_cache);
    case 3: return (int64_t)sizeof(screen_kv_append_args);
    case 4: return (int64_t)sizeof(screen_decode_args);
    case 5: return (int64_t)sizeof(screen_rows_linear_args);
    case 6: return (int64_t)sizeof(screen_xent_args);
    case 7: return (int64_t)sizeof(screen_rmsnorm_args);
    default: return -1;
  }
}

int screen_fwd(const screen_fwd_args* a, screen_stream_t stream) {
  if (!a) return SCREEN_ERR_INVALID_ARG;
  int st = common_checks(a->dtype, a->B, a->H, a->Tq, a->Tk, a->D);
  if (st) return st;
  const int stages = a->stages ? a->stages : 3;
  cudaStream_t s = (cudaStream_t)stream;
  const bool nq = (long long)a->B * a->H * a->Tq > 0, nk = (long long)a->B * a->H * a->Tk > 0;
  if (nq && (!a->q || !a->nq || !a->y || !a->no || !a->r || !a->w)) return SCREEN_ERR_INVALID_ARG;
  if (nk && (!a->k || !a->v || !a->nk || !a->nv)) return SCREEN_ERR_INVALID_ARG;
  if (!raw_ok(a->dtype, a->q, a->q_sb, a->q_st) || !raw_ok(a->dtype, a->k, a->k_sb, a->k_st) ||
      !raw_ok(a->dtype, a->v, a->v_sb, a->v_st) || !al16(a->y))
    return SCREEN_ERR_ALIGNMENT;
  // the tensor-core forward computes the norms in its own prep pass
  const bool tc = use_tc_fwd(a->dtype, a->D) && nq && (stages & 2);
  if (!tc && !a->norms_given && (stages & 1)) {
    NormJob jobs[3];
    int n = 0;
    if (nq) jobs[n++] = NormJob{Rows{a->q, a->q_sb, a->q_st}, a->B, a->Tq, a->H, a->nq};
    if (nk) {
      jobs[n++] = NormJob{Rows{a->k, a->k_sb, a->k_st}, a->B, a->Tk, a->H, a->nk};
      jobs[n++] = NormJob{Rows{a->v, a->v_sb, a->v_st}, a->B, a->Tk, a->H, a->nv};
    }
    if (n) row_norms(a->dtype, a->D, jobs, n, a->eps, s);
    if ((st = check_launch())) return st;
  }
  if (!nq || !(stages & 2)) return SCREEN_OK;
  AttnShape sh = make_shape(a->B, a->H, a->Tq, a->Tk, a->causal, a->q_offset, a->eps, a->r, a->w,
                            a->key_padding_mask, a->kpm_sb, a->dropout_threshold,
                           a->dropout_seed);
  FwdPtrs p{Rows{a->q, a->q_sb, a->q_st}, Rows{a->k, a->k_sb, a->k_st},
            Rows{a->v, a->v_sb, a->v_st}, a->nq, a->nk, a->nv, a->y, a->no, a->tile_stats};
  if (tc) {
    const size_t need = tc_fwd_workspace(sh, a->D);
    if (need > 0 && (!a->workspace || a->workspace_bytes < need || !al16(a->workspace)))
      return SCREEN_ERR_WORKSPACE;
    if ((st = tc_fwd(sh, p, a->workspace, a->norms_given || !(stages & 1), a->D, s))) return st;
  } else if (use_mma_drop(a->dtype, a->D, a->dropout_threshold))
    mma_fwd(a->D, sh, p, s);
  else
    simt_fwd(a->dtype, a->D, sh, p, s);
  return check_launch();
}

uint32_t screen_dropout_bits(uint64_t seed, uint32_t bh, uint32_t i, uint32_t j) {
  AttnShape sh{};
  sh.seed_lo = (uint32_t)seed;
  sh.seed_hi = (uint32_t)(seed >> 32);
  return drop_mix(drop_row(drop_bh_key(sh, bh), i) ^ (j * kDropColMul));
}

size_t screen_fwd_workspace_size(const screen_fwd_args* a) {
  if (!a || common_checks(a->dtype, a->B, a->H, a->Tq, a->Tk, a->D)) return 0;
  if (!use_tc_fwd(a->dtype, a->D)) return 0;
  AttnShape sh = make_shape(a->B, a->H, a->Tq, a->Tk, a->causal, a->q_offset, a->eps, a->r, a->w,
                            a->key_padding_mask, a->kpm_sb, a->dropout_threshold,
                           a->dropout_seed);
  return round_up(tc_fwd_workspace(sh, a->D));
}

int screen_device_status(int clear) {
  const int a = tc_device_status(clear != 0), b = tc_bwd_device_status(clear != 0);
  const int c = decode_device_status(clear != 0), d = xent_device_status(clear != 0);
  return a != 0 ? a : (b != 0 ? b : (c != 0 ? c : d));
}

size_t screen_bwd_workspace_size(const screen_bwd_args* a) {
  if (!a || common_checks(a->dtype, a->B, a->H, a->Tq, a->Tk, a->D)) return 0;
  return bwd_layout(a).total;
}

int screen_bwd(const screen_bwd_args* a, screen_stream_t stream) {
  if (!a) return SCREEN_ERR_INVALID_ARG;
  int st = common_checks(a->dtype, a->B, a->H, a->Tq, a->Tk, a->D);
  if (st) return st;
  int stages = a->stages & 15;
  if (!stages) stages = 15;
  stages |= a->stages & SCREEN_BWD_DETERMINISTIC;
  if (a->H > 0 && (!a->r || !a->w || !a->dr || !a->dw)) return SCREEN_ERR_INVALID_ARG;
  const bool nq = (long long)a->B * a->H * a->Tq > 0, nk = (long long)a->B * a->H * a->Tk > 0;
  if (nq && (!a->q || !a->nq || !a->y || !a->no || !a->dy || !a->dq)) return SCREEN_ERR_INVALID_ARG;
  if (nk && (!a->k || !a->v || !a->nk || !a->nv || !a->dk || !a->dv)) return SCREEN_ERR_INVALID_ARG;
  if (!raw_ok(a->dtype, a->q, a->q_sb, a->q_st) || !raw_ok(a->dtype, a->k, a->k_sb, a->k_st) ||
      !raw_ok(a->dtype, a->v, a->v_sb, a->v_st) || !raw_ok(a->dtype, a->dy, a->dy_sb, a->dy_st) ||
      !raw_ok(a->dtype, a->dq, a->dq_sb, a->dq_st) || !raw_ok(a->dtype, a->dk, a->dk_sb, a->dk_st) ||
      !raw_ok(a->dtype, a->dv, a->dv_sb, a->dv_st) || !al16(a->y) || !al16(a->workspace))
    return SCREEN_ERR_ALIGNMENT;
  BwdLayout L = bwd_layout(a);
  if (L.total > 0 && (!a->workspace || a->workspace_bytes < L.total)) return SCREEN_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  void* G = ws + L.g_off;
  float* pr = reinterpret_cast<float*>(ws + L.pr_off);
  float* pw = reinterpret_cast<float*>(ws + L.pw_off);
  if (nq && (stages & 1))
    tanhnorm_grad_from_y(a->dtype, a->D, a->y, a->no, a->dy, a->dy_sb, a->dy_st, G,
                         // G as bf16 hi/lo planes for the tensor-core families
                         use_tc_bwd(a->dtype, a->D) ||
                             use_mma_drop(a->dtype, a->D, a->dropout_threshold),
                         a->B, a->Tq, a->H, a->eps, s);
  if ((st = check_launch())) return st;
  AttnShape sh = make_shape(a->B, a->H, a->Tq, a->Tk, a->causal, a->q_offset, a->eps, a->r, a->w,
                            a->key_padding_mask, a->kpm_sb, a->dropout_threshold,
                           a->dropout_seed);
  BwdPtrs p{Rows{a->q, a->q_sb, a->q_st}, Rows{a->k, a->k_sb, a->k_st},
            Rows{a->v, a->v_sb, a->v_st}, a->nq, a->nk, a->nv, G,
            OutRows{a->dq, a->dq_sb, a->dq_st}, OutRows{a->dk, a->dk_sb, a->dk_st},
            OutRows{a->dv, a->dv_sb, a->dv_st}, pr, pw};
  if (use_tc_bwd(a->dtype, a->D)) {
    if ((st = tc_bwd(sh, p, ws + L.aux_off, stages, a->D, s))) return st;
  } else if (use_mma_drop(a->dtype, a->D, a->dropout_threshold))
    mma_bwd(a->D, sh, p, stages, s);
  else
    simt_bwd(a->dtype, a->D, sh, p, stages, s);
  if ((st = check_launch())) return st;
  if (a->H > 0 && (stages & 8)) reduce_param_grads(pr, pw, L.P, a->H, a->w, a->dr, a->dw, s);
  return check_launch();
}

int screen_kv_append(const screen_kv_append_args* a, screen_stream_t stream) {
  if (!a) return SCREEN_ERR_INVALID_ARG;
  int st = common_checks(a->dtype, a->B, a->H, a->n_new, 0, a->D);
  if (st) return st;
  if ((long long)a->B * a->H * a->n_new == 0) return SCREEN_OK;
  if (!a->k || !a->v || !a->positions || !a->cache.k_pages || !a->cache.v_pages ||
      !a->cache.block_table || a->cache.page_size <= 0 || a->cache.max_blocks <= 0)
    return SCREEN_ERR_INVALID_ARG;
  if (!al16(a->k) || !al16(a->v) || !al16(a->cache.k_pages) || !al16(a->cache.v_pages))
    return SCREEN_ERR_ALIGNMENT;
  if (!strides_ok(a->k_sb, a->k_st) || !strides_ok(a->v_sb, a->v_st)) return SCREEN_ERR_ALIGNMENT;
  kv_append(*a, (cudaStream_t)stream);
  return check_launch();
}

size_t screen_decode_workspace_size(const screen_decode_args* a) {
  if (!a || a->num_splits < 1 || a->B < 0 || a->H < 0 || !dim_ok(a->D)) return 0;
  return round_up((size_t)a->B * a->H * a->num_splits * a->D * sizeof(float));
}

int screen_decode(const screen_decode_args* a, screen_stream_t stream) {
  if (!a) return SCREEN_ERR_INVALID_ARG;
  int st = common_checks(a->dtype, a->B, a->H, 0, 0, a->D);
  if (st) return st;
  if (a->num_splits < 1) return SCREEN_ERR_INVALID_ARG;
  if ((long long)a->B * a->H == 0) return SCREEN_OK;
  if (!a->q || !a->seq_lens || !a->r || !a->w || !a->y || !a->cache.k_pages ||
      !a->cache.v_pages || !a->cache.block_table || a->cache.page_size <= 0 ||
      a->cache.max_blocks <= 0)
    return SCREEN_ERR_INVALID_ARG;
  if (!al16(a->q) || !al16(a->cache.k_pages) || !al16(a->cache.v_pages) || !al16(a->workspace))
    return SCREEN_ERR_ALIGNMENT;
  if (a->q_sb % 4 != 0) return SCREEN_ERR_ALIGNMENT;
  const size_t need = screen_decode_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need) return SCREEN_ERR_WORKSPACE;
  decode(*a, reinterpret_cast<float*>(a->workspace), (cudaStream_t)stream);
  return check_launch();
}

int screen_decode_append(const screen_kv_append_args* ap, const screen_decode_args* a,
                         screen_stream_t stream) {
  if (!ap || !a) return SCREEN_ERR_INVALID_ARG;
  int st = common_checks(a->dtype, a->B, a->H, 0, 0, a->D);
  if (st) return st;
  if (ap->n_new != 1 || ap->dtype != a->dtype || ap->B != a->B || ap->H != a->H ||
      ap->D != a->D || a->num_splits < 1)
    return SCREEN_ERR_INVALID_ARG;
  // one cache: the rows are appended where the decode reads them
  if (memcmp(&ap->cache, &a->cache, sizeof(screen_kv_cache)) != 0) return SCREEN_ERR_INVALID_ARG;
  if ((long long)a->B * a->H == 0) return SCREEN_OK;
  if (!a->q || !a->seq_lens || !a->r || !a->w || !a->y || !a->cache.k_pages ||
      !a->cache.v_pages || !a->cache.block_table || a->cache.page_size <= 0 ||
      a->cache.max_blocks <= 0 || !ap->k || !ap->v || !ap->positions)
    return SCREEN_ERR_INVALID_ARG;
  if (!al16(a->q) || !al16(a->cache.k_pages) || !al16(a->cache.v_pages) || !al16(a->workspace) ||
      !al16(ap->k) || !al16(ap->v))
    return SCREEN_ERR_ALIGNMENT;
  if (a->q_sb % 4 != 0) return SCREEN_ERR_ALIGNMENT;
  if (!strides_ok(ap->k_sb, ap->k_st) || !strides_ok(ap->v_sb, ap->v_st)) return SCREEN_ERR_ALIGNMENT;
  const size_t need = screen_decode_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need) return SCREEN_ERR_WORKSPACE;
  decode_append(*ap, *a, reinterpret_cast<float*>(a->workspace), (cudaStream_t)stream);
  return check_launch();
}

int screen_tanhnorm_fwd(int32_t dtype, int64_t rows, int32_t D, float eps, const void* x,
                        void* y, screen_stream_t stream) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (D < 1) return SCREEN_ERR_INVALID_ARG;
  if (rows < 0) return SCREEN_ERR_INVALID_ARG;
  if (rows == 0) return SCREEN_OK;
  if (!x || !y) return SCREEN_ERR_INVALID_ARG;
  tanhnorm(dtype, D, false, x, nullptr, y, rows, eps, (cudaStream_t)stream);
  return check_launch();
}

int screen_tanhnorm_bwd(int32_t dtype, int64_t rows, int32_t D, float eps, const void* x,
                        const void* dy, void* dx, screen_stream_t stream) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (D < 1) return SCREEN_ERR_INVALID_ARG;
  if (rows < 0) return SCREEN_ERR_INVALID_ARG;
  if (rows == 0) return SCREEN_OK;
  if (!x || !dy || !dx) return SCREEN_ERR_INVALID_ARG;
  tanhnorm(dtype, D, true, x, dy, dx, rows, eps, (cudaStream_t)stream);
  return check_launch();
}

int screen_col_scale_bwd(int32_t dtype, int64_t rows, int32_t D, const void* dy, const void* w,
                         const void* g, void* dw, void* dg, screen_stream_t stream) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (rows < 0 || D <= 0) return SCREEN_ERR_INVALID_ARG;
  if ((!dw && !dg) || (rows == 0 && !dg)) return SCREEN_OK;
  if (!dy || !g || (dg && !w)) return SCREEN_ERR_INVALID_ARG;
  col_scale_bwd(dtype, rows, D, dy, w, g, dw, dg, (cudaStream_t)stream);
  return check_launch();
}

int screen_head_params_fwd(int32_t dtype, int32_t H, const void* s_r, const void* s_v,
                           float* r, float* w, screen_stream_t stream) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (H < 0) return SCREEN_ERR_INVALID_ARG;
  if (H == 0) return SCREEN_OK;
  if (!s_r || !s_v || !r || !w) return SCREEN_ERR_INVALID_ARG;
  head_params_fwd(dtype, H, s_r, s_v, r, w, (cudaStream_t)stream);
  return check_launch();
}

int screen_head_params_bwd(int32_t dtype, int32_t H, const void* s_r, const void* s_v,
                           const float* dr, const float* dw, void* ds_r, void* ds_v,
                           screen_stream_t stream) {
  if (!dtype_ok(dtype)) return SCREEN_ERR_DTYPE;
  if (H < 0) return SCREEN_ERR_INVALID_ARG;
  if (H == 0 || (!dr && !dw)) return SCREEN_OK;
  if (!s_r || !s_v || (dr && !ds_r) || (dw && !ds_v)) return SCREEN_ERR_INVALID_ARG;
  head_params_bwd(dtype, H, s_r, s_v, dr, dw, ds_r, ds_v, (cudaStream_t)stream);
  return check_launch();
}

}  // extern "C"
