/*
 * screening_b200.h -- C ABI of the B200 (sm_100a) Screening Attention kernels.
 *
 * Screening Attention ("Screening Is Enough", arXiv:2604.01178) as computed by
 * multiscreen/attention.py:151-196 and multiscreen/norm.py:23-25 of the
 * reference package `multiscreen`:
 *
 *   q^ = q / max(|q|, eps)    k^, v^ likewise              (attention.py:156-158)
 *   S  = q^ k^T                                           (attention.py:161)
 *   a  = relu(1 - r (1 - S)),  alpha = a^2                 (attention.py:75-90)
 *   m  = (cos(pi rel / w) + 1) / 2 inside the window       (attention.py:92-119,174-183)
 *        causal:     -w < rel <= 0      non-causal: |rel| < w,   rel = j - i
 *   alpha *= m;  alpha[:, :, :, j] = 0 for padded keys j   (attention.py:186-188)
 *   o  = alpha v^  (no normaliser)                         (attention.py:193)
 *   y  = tanh(|o|) / max(|o|, eps) * o                     (norm.py:23-25)
 *
 * Layout: every (B, T, H, D) tensor is row-major with unit stride over D and
 * stride D over H; the batch and time strides of the raw inputs are free
 * (given in elements).  All buffers are device memory owned by the caller; the
 * library never allocates or frees device memory and keeps no mutable global
 * state besides a per-device attribute cache.  Every entry point returns 0 on
 * success or a negative screen_status; nothing aborts and no C++ exception
 * crosses this boundary.  Launches go to `stream` (a cudaStream_t).
 *
 * Supported: D in {16, 32, 64, 128}; dtype SCREEN_F32 (fp32 I/O, fp32 math) or
 * SCREEN_BF16 (bf16 I/O, fp32 accumulation); any T_q, T_k >= 0.  Raw inputs
 * need 16-byte aligned base pointers and strides that are multiples of 8
 * elements (bf16) / 4 elements (fp32).
 */
#ifndef SCREENING_B200_H
#define SCREENING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SCREEN_ABI_VERSION 5

#if defined(__GNUC__)
#define SCREEN_API __attribute__((visibility("default")))
#else
#define SCREEN_API
#endif

typedef void* screen_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum screen_dtype { SCREEN_F32 = 0, SCREEN_BF16 = 1 };

enum screen_status {
  SCREEN_OK = 0,
  SCREEN_ERR_INVALID_ARG = -1,     /* null pointer, negative size, bad enum   */
  SCREEN_ERR_HEAD_DIM = -2,        /* D not in {16, 32, 64, 128}              */
  SCREEN_ERR_DTYPE = -3,           /* dtype not SCREEN_F32 / SCREEN_BF16      */
  SCREEN_ERR_ALIGNMENT = -4,       /* pointer or stride not 16-byte aligned   */
  SCREEN_ERR_WORKSPACE = -5,       /* workspace missing or too small          */
  SCREEN_ERR_LAUNCH = -6,          /* cudaGetLastError after a launch         */
  SCREEN_ERR_TIMEOUT = -7,         /* a bounded device-side wait gave up      */
  SCREEN_ERR_CUDA = -8,            /* other CUDA runtime error                */
  SCREEN_ERR_UNSUPPORTED = -9,     /* valid request this build does not do    */
  SCREEN_ERR_SCRATCH_LIMIT = -10   /* needs more than the static scratch      */
};

/* ------------------------------------------------------------------------ */
/* Forward.                                                                  */
/* The kernels read the RAW projections and apply the unit-normalisation as  */
/* fp32 per-row / per-column scales (S = (q.k) / (|q| |k|)), so bf16 inputs   */
/* enter the tensor cores exactly and no normalised copy is written.         */
/* ------------------------------------------------------------------------ */
typedef struct screen_fwd_args {
  int32_t dtype;                 /* enum screen_dtype of q, k, v, y           */
  int32_t B, H, Tq, Tk, D;
  int32_t causal;                /* nonzero: causal softmask                  */
  int32_t norms_given;           /* nonzero: nq, nk, nv are inputs            */
  int64_t q_offset;              /* key-axis position of query row 0; rel =   */
                                 /*   j - (i + q_offset).  0 for self-attn    */
  float eps;                     /* F.normalize / TanhNorm eps (1e-8)         */
  int32_t stages;                /* 0 = all; else bitmask: 1 norms,           */
                                 /*   2 attention (profiling)                 */
  /* raw projections (B,T,H,D), strides in elements                          */
  const void* q; int64_t q_sb, q_st;
  const void* k; int64_t k_sb, k_st;
  const void* v; int64_t v_sb, v_st;
  const float* r;                /* (H,) acceptance sharpness r = exp(s_r)+1 */
  const float* w;                /* (H,) window w = exp(s_v)+1               */
  const uint8_t* key_padding_mask; /* (B,Tk), nonzero = ignore key; or NULL  */
  int64_t kpm_sb;                /* batch stride of key_padding_mask          */
  float* nq; float* nk; float* nv; /* (B,T,H) max(|x|, eps), contiguous      */
  void* y;                       /* (B,Tq,H,D) TanhNorm(alpha v^), contiguous */
  float* no;                     /* (B,Tq,H) |alpha v^| before TanhNorm       */
  int64_t* tile_stats;           /* optional [2]: += 16x64 score blocks in    */
                                 /*   the window, += blocks with live scores  */
  void* workspace;               /* screen_fwd_workspace_size() bytes         */
  size_t workspace_bytes;
  /* attention dropout on alpha (attention.py:68,190): each (b, h, query i,  */
  /* key j) is dropped iff screen_dropout_bits(seed, b*H+h, i, j) <          */
  /* dropout_threshold, kept ones scaled by 2^32 / (2^32 - threshold).  0 =  */
  /* no dropout.  screen_bwd must get the same seed and threshold.           */
  uint32_t dropout_threshold;
  uint32_t _pad1;
  uint64_t dropout_seed;
} screen_fwd_args;

/* The dropout bits of score (bh, i, j) for a seed (host-side mirror of the
 * kernels' counter-based hash, for tests and for callers that need the mask):
 *   k  = mix(seed_lo ^ mix(seed_hi ^ bh * 0x9E3779B1))
 *   ri = mix(k ^ i * 0x85EBCA77),  bits = mix(ri ^ j * 0xC2B2AE3D)
 * with 32-bit wrap-around and mix(x) = the lowbias32 finalizer
 * (x ^= x>>16; x *= 0x7feb352d; x ^= x>>15; x *= 0x846ca68b; x ^= x>>16).
 * i is the query index (0..Tq-1) and j the key index (0..Tk-1) of the call.
 * No counterpart in the reference, whose dropout draws from torch's
 * generator (attention.py:190); bit parity with it is not possible. */
SCREEN_API uint32_t screen_dropout_bits(uint64_t seed, uint32_t bh, uint32_t i, uint32_t j);

/* Bytes of device workspace screen_fwd needs (bf16 D=64 tensor-core path: the
 * unit-V operand, 1/|k| per key and per-tile bounds; 0 otherwise). */
SCREEN_API size_t screen_fwd_workspace_size(const screen_fwd_args* a);

/* Fused screening forward (unit-normalisation, S, trim-and-square, softmask,
 * key padding, alpha v^, TanhNorm).
 * Replaces multiscreen/attention.py:156-196 and the op-level
 * screening_attention_fwd (multiscreen/kernels/screening_fwd.py:216-270),
 * whose inputs are pre-normalised (B,H,T,D) and whose output is pre-TanhNorm;
 * here the unit-normalisation and TanhNorm are fused in. */
SCREEN_API int screen_fwd(const screen_fwd_args* a, screen_stream_t stream);

/* screen_bwd stage flag: fixed-order (bitwise reproducible) dq */
#define SCREEN_BWD_DETERMINISTIC 16

/* ------------------------------------------------------------------------ */
/* Backward.                                                                 */
/* ------------------------------------------------------------------------ */
typedef struct screen_bwd_args {
  int32_t dtype;
  int32_t B, H, Tq, Tk, D;
  int32_t causal;
  int32_t stages;                /* 0 = all; else bitmask: 1 TanhNorm grad,   */
                                 /*   2 dq, 4 dk/dv, 8 dr/dw reduce; with    */
                                 /*   SCREEN_BWD_DETERMINISTIC (16) set, dq  */
                                 /*   is summed in a fixed order (else the   */
                                 /*   bf16 D=64 path forms dq inside the     */
                                 /*   dk/dv kernel with fp32 reductions, run */
                                 /*   by stage 4; stage 2 then adds nothing) */
  int64_t q_offset;
  float eps;
  int32_t _pad0;
  /* forward inputs and what screen_fwd returned                             */
  const void* q; int64_t q_sb, q_st;
  const void* k; int64_t k_sb, k_st;
  const void* v; int64_t v_sb, v_st;
  const float* nq; const float* nk; const float* nv;
  const void* y; const float* no;
  /* incoming gradient dL/dy (B,Tq,H,D), strides in elements                 */
  const void* dy; int64_t dy_sb, dy_st;
  const float* r; const float* w;
  const uint8_t* key_padding_mask; int64_t kpm_sb;
  /* outputs: gradients of the RAW projections (B,T,H,D), strides in elements*/
  void* dq; int64_t dq_sb, dq_st;
  void* dk; int64_t dk_sb, dk_st;
  void* dv; int64_t dv_sb, dv_st;
  float* dr; float* dw;          /* (H,) dL/dr, dL/dw                         */
  void* workspace; size_t workspace_bytes;
  uint32_t dropout_threshold;    /* as screen_fwd_args: the forward's values  */
  uint32_t _pad1;
  uint64_t dropout_seed;
} screen_bwd_args;

/* Bytes of device workspace screen_bwd needs for these shapes. */
SCREEN_API size_t screen_bwd_workspace_size(const screen_bwd_args* a);

/* Gradients dq, dk, dv (through the unit-normalisation and TanhNorm
 * Jacobians) and the per-head dr, dw.  Replaces autograd of
 * multiscreen/attention.py:156-196 and screening_attention_bwd
 * (multiscreen/kernels/screening_bwd.py:229-287), which returns no dr/dw. */
SCREEN_API int screen_bwd(const screen_bwd_args* a, screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Paged K/V cache and single-token decode (serves MultiscreenLM.generate,    */
/* replacing the full-prefix recompute at multiscreen/model.py:131-133).     */
/* ------------------------------------------------------------------------ */
typedef struct screen_kv_cache {
  void* k_pages;                 /* [num_pages, H, page_size, D] unit rows    */
  void* v_pages;                 /* same                                      */
  const int32_t* block_table;    /* [B, max_blocks] page ids                  */
  int32_t num_pages, page_size, max_blocks, _pad0;
} screen_kv_cache;

typedef struct screen_kv_append_args {
  int32_t dtype;                 /* of k, v and the pages                     */
  int32_t B, H, D, n_new;
  float eps;
  const void* k; int64_t k_sb, k_st;   /* raw (B,n_new,H,D)                   */
  const void* v; int64_t v_sb, v_st;
  const int32_t* positions;      /* (B,) position of token 0 of k, v         */
  screen_kv_cache cache;
} screen_kv_append_args;

/* Unit-normalise n_new new key/value rows per sequence and write them into
 * the paged cache at positions[b] .. positions[b]+n_new-1. */
SCREEN_API int screen_kv_append(const screen_kv_append_args* a, screen_stream_t stream);

typedef struct screen_decode_args {
  int32_t dtype;
  int32_t B, H, D;
  int32_t num_splits;            /* key-axis splits per (b,h); >= 1           */
  float eps;
  const void* q; int64_t q_sb;   /* raw (B,H,D) query of the newest token     */
  const int32_t* seq_lens;       /* (B,) tokens in cache incl. the newest one */
  const float* r; const float* w;
  screen_kv_cache cache;
  void* y;                       /* (B,H,D) TanhNorm output                   */
  float* no;                     /* (B,H) or NULL                             */
  void* workspace; size_t workspace_bytes;
} screen_decode_args;

SCREEN_API size_t screen_decode_workspace_size(const screen_decode_args* a);

/* One causal query per (b,h) at position seq_lens[b]-1 against the cached
 * keys inside its window.  Equals the last row of screen_fwd over the whole
 * prefix (the logits row generate() keeps at multiscreen/model.py:133).
 * With num_splits > 1 each (b,h) window is cut into that many runs of pages
 * whose partial sums go through the workspace and a finishing pass; with
 * num_splits == 1 one CTA per (b,h) applies TanhNorm itself (the workspace is
 * then not read). */
SCREEN_API int screen_decode(const screen_decode_args* a, screen_stream_t stream);

/* screen_kv_append of one new row per sequence (ap->n_new == 1) followed by
 * screen_decode over the same cache, as one launch where the decode kernel
 * streams the cache pages by bulk copies: the CTA whose pages hold
 * positions[b] writes the unit k / v rows (the same arithmetic as
 * screen_kv_append) before it reads the page.  The per-token step of
 * generate() (multiscreen/model.py:131-133 recomputes the whole prefix
 * instead).  ap->cache and a->cache must be the same descriptor; the new
 * token is normally at positions[b] == seq_lens[b] - 1. */
SCREEN_API int screen_decode_append(const screen_kv_append_args* ap, const screen_decode_args* a,
                                    screen_stream_t stream);

/* Bytes of the static device scratch array used by screen_decode_noalloc. */
#define SCREEN_DECODE_NOALLOC_SCRATCH_BYTES (4u << 20)

/* screen_decode without a workspace.  No counterpart in the reference.
 * For callers that cannot allocate device memory on their serving path (a
 * process whose device footprint is fixed after start-up, or a C / FFI caller
 * with no device allocator to provide a workspace).  The split-K partials go
 * to a static 4 MiB device array (SCREEN_DECODE_NOALLOC_SCRATCH_BYTES) that
 * every GPU loading this library keeps until exit; requests needing more
 * (B * H * num_splits * D * 4 bytes) return SCREEN_ERR_SCRATCH_LIMIT.  The
 * array's device address is looked up on the first call on each device, so
 * make that first call before any stream capture.  All calls share the
 * array: calls that overlap on the GPU race and must be serialised by the
 * caller.  `workspace` / `workspace_bytes` are ignored.  Allocates nothing. */
SCREEN_API int screen_decode_noalloc(const screen_decode_args* a, screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Few-row linear layer for the decode step of generate() (B <= 8 tokens):   */
/* y[m, n] = act(sum_k xin[m, k] W[n, k]) (+ res[m, n]), bf16 in and out,    */
/* fp32 accumulation.  xin = x, or RMSNorm(x) * norm_w when norm_w is given  */
/* (torch.nn.RMSNorm: x / sqrt(mean(x^2) + eps), the normalised row rounded  */
/* to bf16 as the unfused module does).  act: 0 none, 1 exact GELU           */
/* (nn.GELU()).  Replaces the nn.RMSNorm -> nn.Linear -> nn.GELU -> residual */
/* chain of the decode step (multiscreen/layers.py:60-76, model.py:97) that  */
/* the reference runs as separate PyTorch ops on its full-prefix recompute   */
/* (model.py:133): a bandwidth-bound pass over W instead of a GEMM with M=B. */
/* ------------------------------------------------------------------------ */
typedef struct screen_rows_linear_args {
  int32_t M, N, K;               /* M <= 8 rows, K % 8 == 0                   */
  int32_t act;                   /* 0 none, 1 GELU (erf)                      */
  float norm_eps;
  int32_t _pad0;
  const void* x; int64_t x_stride;     /* (M, K) bf16, row stride in elements  */
  const void* norm_w;            /* (K,) bf16 RMSNorm weight, or NULL         */
  const void* W;                 /* (N, K) bf16, contiguous                   */
  const void* res; int64_t res_stride; /* (M, N) bf16 added after act, or NULL*/
  void* y; int64_t y_stride;     /* (M, N) bf16                               */
} screen_rows_linear_args;

SCREEN_API int screen_rows_linear(const screen_rows_linear_args* a, screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Cross-entropy over bf16 logits rows (the LM loss, multiscreen/model.py:   */
/* 103-107: F.cross_entropy(logits, labels, ignore_index=-100), mean).       */
/* fwd: per row lse = log sum exp(x) and loss = lse - x[label] (0 for an     */
/* ignored label), one pass (online max / sum), fp32 math.  bwd: dlogits =   */
/* (softmax(x) - onehot(label)) * (*dscale), 0 for ignored rows, one pass.   */
/* The caller forms the mean (sum(loss) / count) and dscale = dmean / count  */
/* on the device.  V % 8 == 0 (pad the vocabulary with -inf logits);         */
/* logits rows 16-byte aligned.                                              */
/* ------------------------------------------------------------------------ */
typedef struct screen_xent_args {
  int64_t rows;
  int32_t V;                     /* row length (the padded vocabulary)        */
  int32_t ignore_index;
  const void* logits; int64_t ld;      /* (rows, V) bf16, row stride          */
  const int64_t* labels;         /* (rows,)                                   */
  float* lse;                    /* (rows,) fwd output, bwd input             */
  float* loss;                   /* (rows,) fwd output                        */
  void* dlogits; int64_t dld;    /* (rows, V) bf16, bwd output                */
  const float* dscale;           /* device scalar: dL/d(mean) / count          */
} screen_xent_args;

SCREEN_API int screen_cross_entropy_fwd(const screen_xent_args* a, screen_stream_t stream);
SCREEN_API int screen_cross_entropy_bwd(const screen_xent_args* a, screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* RMSNorm of the blocks' pre-norms (torch.nn.RMSNorm in multiscreen/        */
/* layers.py:35-36,60-76 and model.py:57,98): y = x / sqrt(mean(x^2) + eps)  */
/* * w over contiguous rows of length D (D % 8 == 0, rows 16-byte aligned),  */
/* fp32 math.  x and dx: fp32 or bf16; w and dw: fp32 or bf16; y and dy:     */
/* bf16 or x's dtype (bf16 is what autocast's next Linear would cast the     */
/* fp32 output to, rounded once).  fwd also writes rstd (rows,) fp32 for the */
/* backward.  bwd: dx = rstd (g - xh mean(g xh)) with g = dy w, xh = x rstd, */
/* and dw = sum over rows of dy xh in a fixed order: per-CTA column partials */
/* in `partials` (screen_rmsnorm_partials(rows) rows of D floats), summed by  */
/* a second pass.                                                            */
/* ------------------------------------------------------------------------ */
typedef struct screen_rmsnorm_args {
  int64_t rows;
  int32_t D;
  int32_t x_dtype, w_dtype, y_dtype;   /* SCREEN_F32 / SCREEN_BF16           */
  float eps;
  const void* x;                 /* (rows, D)                                 */
  const void* w;                 /* (D,)                                      */
  void* y;                       /* (rows, D) fwd output                      */
  float* rstd;                   /* (rows,) fwd output, bwd input             */
  const void* dy;                /* (rows, D) bwd input, y_dtype              */
  void* dx;                      /* (rows, D) bwd output, x_dtype             */
  void* dw;                      /* (D,) bwd output, w_dtype                  */
  float* partials;               /* bwd workspace                             */
} screen_rmsnorm_args;

SCREEN_API int64_t screen_rmsnorm_partials(int64_t rows);
SCREEN_API int screen_rmsnorm_fwd(const screen_rmsnorm_args* a, screen_stream_t stream);
SCREEN_API int screen_rmsnorm_bwd(const screen_rmsnorm_args* a, screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Stand-alone TanhNorm (multiscreen/norm.py:8-25) over contiguous rows of   */
/* length D (any D >= 1).                                                    */
/* ------------------------------------------------------------------------ */
SCREEN_API int screen_tanhnorm_fwd(int32_t dtype, int64_t rows, int32_t D, float eps,
                        const void* x, void* y, screen_stream_t stream);
SCREEN_API int screen_tanhnorm_bwd(int32_t dtype, int64_t rows, int32_t D, float eps,
                        const void* x, const void* dy, void* dx,
                        screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Per-head parameter transforms of ScreeningAttention, all heads in one     */
/* launch: r = exp(s_r) + 1 and w = exp(s_v) + 1 (multiscreen/attention.py:   */
/* 164-165; there they are four PyTorch ops per step, plus the casts of a     */
/* bf16 module).  s_r, s_v: H values of `dtype`; r, w: H fp32.  The backward  */
/* writes ds_r = dr exp(s_r), ds_v = dw exp(s_v) in `dtype`; a null dr (dw)   */
/* leaves ds_r (ds_v) unwritten.                                             */
/* ------------------------------------------------------------------------ */
SCREEN_API int screen_head_params_fwd(int32_t dtype, int32_t H, const void* s_r, const void* s_v,
                                      float* r, float* w, screen_stream_t stream);
SCREEN_API int screen_head_params_bwd(int32_t dtype, int32_t H, const void* s_r, const void* s_v,
                                      const float* dr, const float* dw, void* ds_r, void* ds_v,
                                      screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Backward of Y = W diag(g): a pre-attention RMSNorm weight g folded into    */
/* the columns of the QKV projection W (rows x D, row-major).  The RMSNorm    */
/* in front of self-attention (multiscreen/layers.py:73-74) needs no pass of  */
/* its own: its per-token scale cancels in the unit normalisation of q, k, v  */
/* (attention.py:156-158), so q, k, v = x (W diag(g))^T.  Writes              */
/* dW = dY diag(g) and dg[c] = sum_o dY[o, c] W[o, c] (fixed order); a null   */
/* dw or dg is not written.  dy, w, g, dw, dg all of `dtype`.                 */
/* ------------------------------------------------------------------------ */
SCREEN_API int screen_col_scale_bwd(int32_t dtype, int64_t rows, int32_t D, const void* dy,
                                    const void* w, const void* g, void* dw, void* dg,
                                    screen_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Misc.                                                                     */
/* ------------------------------------------------------------------------ */
SCREEN_API const char* screen_strerror(int status);
SCREEN_API int screen_version(void);                  /* SCREEN_ABI_VERSION             */
/* sizeof of the argument structs, for binding checks: 0 fwd, 1 bwd,
 * 2 kv_cache, 3 kv_append, 4 decode, 5 rows_linear, 6 xent; -1 for an unknown id. */
SCREEN_API int64_t screen_sizeof_args(int which);
/* Last CUDA error string seen by this thread inside the library. */
SCREEN_API const char* screen_last_cuda_error(void);
/* SCREEN_OK, or SCREEN_ERR_TIMEOUT if a kernel since the last clear gave up
 * a bounded device-side wait (the kernel then drained and returned).  Reads a
 * device status word (synchronising copy); `clear` resets it. */
SCREEN_API int screen_device_status(int clear);

#ifdef __cplusplus
}
#endif
#endif /* SCREENING_B200_H */
