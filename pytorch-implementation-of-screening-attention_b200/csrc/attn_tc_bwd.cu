// Screening attention backward on tcgen05 / TMEM (bf16, head dim 64 or 128;
// at 128 without the fused dQ, see KvCfg / DqCfg).
//
// Autograd of multiscreen/attention.py:156-196 (the reference leaves it to
// PyTorch; its Triton backward, kernels/screening_bwd.py, has no dr / dw):
//   dP = G v^T (G = dL/do through TanhNorm, as bf16 hi + lo planes),
//   dS = dP m 2a r [a > 0],  dv^ = alpha^T G,  dq^ = dS k^,  dk^ = dS^T q^,
//   dr = sum dP m 2a (S - 1),  dw = pi/(2 w^2) sum dP a^2 rel sin(pi rel / w),
// then the unit-normalisation Jacobians.  As in the forward the tensor cores
// see raw bf16 q / k / v; 1/|q|, 1/|k|, 1/|v| are fp32 row / column scales.
//
// Two kernels, both warp specialised (10 warps: 8 compute = two warpgroups
// splitting every 64-column tile in halves, 1 TMA producer, 1 MMA
// issuer), 512 TMEM columns, one CTA per SM:
//   tc_bwd_dq_kernel  (query-major, 128 queries, key tiles of 64):
//       S = Q K^T, dP = G_hi V^T + G_lo V^T, dQ += dS K
//   tc_bwd_kv_kernel  (key-major, 128 keys, query tiles of 64):
//       S^T = K Q^T, dP^T = V G_hi^T + V G_lo^T, dV += alpha G_hi, dK += dS Q,
//       plus the per-CTA dr / dw partials (summed in a fixed order later).
// Every wait is bounded (global timer); on expiry the CTA drains and records
// SCREEN_ERR_TIMEOUT in the device status word.
#include <type_traits>
#include "rowops.cuh"

namespace screen {
namespace {

using namespace sm100;
typedef __nv_bfloat16 bf16;

constexpr int kD = 64, kBM = 128, kBN = 64, kNS = 4, kThreads = 320;
constexpr int kCompute = 256;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t TILE_A = kBM * kD * 2;  // 128-row operand tile, 16 KB
constexpr uint32_t TILE_B = kBN * kD * 2;  // 64-row tile, 8 KB
constexpr uint32_t TM_COLS = 512;

struct Aux {
  const float* iqT;   // [B*H][Tqp] 1/|q| (0 past Tq)
  const float* ikT;   // [B*H][Tkp] 1/|k| (0 past Tk)
  const float* ivT;   // [B*H][Tkp] 1/(|v| |k|) (0 past Tk and for padded keys)
  const float4* mq;   // [B*H][Tqp/64] (max 1/|q| of the tile, -, -, -)
  const float4* mk;   // [B*H][Tkp/64] (max 1/|k| of the tile, -, -, -)
  const int* order;   // [B*H*ceil(Tk/128)] key-major CTA order (longest first)
  int Tqp, Tkp;
};

__device__ int g_bwd_status = 0;

__device__ __forceinline__ int* status_word() { return &g_bwd_status; }

__device__ __forceinline__ void store_unit_jacobian(const float (&acc)[64], const bf16* xrow,
                                                    float inv, bf16* out) {
  // out = inv * (acc - inv^2 (x . acc) x), x the raw row (the Jacobian of
  // x / |x| applied to acc = dL/dx^)
  float xv[64];
#pragma unroll
  for (int c8 = 0; c8 < 8; ++c8) {
    const uint4 u = reinterpret_cast<const uint4*>(xrow)[c8];
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16(w4[e]);
      xv[8 * c8 + 2 * e] = f.x;
      xv[8 * c8 + 2 * e + 1] = f.y;
    }
  }
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < 64; ++c) dot = fmaf(xv[c], acc[c], dot);
  const float cf = inv * inv * dot;
#pragma unroll
  for (int c8 = 0; c8 < 8; ++c8) {
    uint4 v;
    v.x = pack_bf16(inv * (acc[8 * c8 + 0] - cf * xv[8 * c8 + 0]),
                    inv * (acc[8 * c8 + 1] - cf * xv[8 * c8 + 1]));
    v.y = pack_bf16(inv * (acc[8 * c8 + 2] - cf * xv[8 * c8 + 2]),
                    inv * (acc[8 * c8 + 3] - cf * xv[8 * c8 + 3]));
    v.z = pack_bf16(inv * (acc[8 * c8 + 4] - cf * xv[8 * c8 + 4]),
                    inv * (acc[8 * c8 + 5] - cf * xv[8 * c8 + 5]));
    v.w = pack_bf16(inv * (acc[8 * c8 + 6] - cf * xv[8 * c8 + 6]),
                    inv * (acc[8 * c8 + 7] - cf * xv[8 * c8 + 7]));
    reinterpret_cast<uint4*>(out)[c8] = v;
  }
}

// store_unit_jacobian with the accumulator row read from TMEM 32 columns at a
// time (scaled by `scale`), in two passes (x . acc, then the output), so at
// most 32 accumulators and 8 raw values are live.  `ok` false: acc = 0.
// Warp-collective (tcgen05.ld): call it with the whole warp.
template <int D = 64>
__device__ __forceinline__ void store_unit_jacobian_tmem(uint32_t taddr, bool ok, float scale,
                                                         const bf16* xrow, float inv, bf16* out,
                                                         bool store) {
  float dot = 0.f;
#pragma unroll
  for (int h = 0; h < D / 32; ++h) {
    uint32_t u[32];
    if (ok) {
      tmem_ld32(taddr + 32 * h, u);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) u[c] = 0u;
    }
    if (store) {
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint4 xv = reinterpret_cast<const uint4*>(xrow)[4 * h + c8];
        const uint32_t w4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(w4[e]);
          dot = fmaf(f.x, __uint_as_float(u[8 * c8 + 2 * e]), dot);
          dot = fmaf(f.y, __uint_as_float(u[8 * c8 + 2 * e + 1]), dot);
        }
      }
    }
  }
  const float cf = inv * inv * dot * scale;
#pragma unroll
  for (int h = 0; h < D / 32; ++h) {
    uint32_t u[32];
    if (ok) {
      tmem_ld32(taddr + 32 * h, u);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) u[c] = 0u;
    }
    if (store) {
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint4 xv = reinterpret_cast<const uint4*>(xrow)[4 * h + c8];
        const uint32_t w4[4] = {xv.x, xv.y, xv.z, xv.w};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16(w4[e]);
          const float a0 = __uint_as_float(u[8 * c8 + 2 * e]) * scale;
          const float a1 = __uint_as_float(u[8 * c8 + 2 * e + 1]) * scale;
          o4[e] = pack_bf16(inv * (a0 - cf * f.x), inv * (a1 - cf * f.y));
        }
        reinterpret_cast<uint4*>(out)[4 * h + c8] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    }
  }
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&o)[64]) {
  uint32_t u[64];
  uint32_t (&a0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&u[0]);
  uint32_t (&a1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&u[32]);
  tmem_ld32(taddr, a0);
  tmem_ld32(taddr + 32, a1);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 64; ++c) o[c] = __uint_as_float(u[c]);
}

// ===========================================================================
// dq kernel
// ===========================================================================
// Per head dim D (64 or 128): operand tiles are D / 64 column halves of 64
// elements (128-byte rows, SW128), each one TMA box and one run of 4 K-steps.
template <int D>
struct DqCfg {
  // D = 64: two CTAs per SM; D = 128: one (the 128-row Q / G_hi / G_lo tiles
  // alone take 96 KB)
  static constexpr int kNSq = 3, kMinBlocks = D == 64 ? 2 : 1;
  static constexpr uint32_t TILE_A = kBM * D * 2, TILE_B = kBN * D * 2;
  static constexpr uint32_t HALF_A = kBM * 128, HALF_B = kBN * 128;
  // single S / dP buffers with dS written over the dP columns it came from,
  // dQ accumulator -> 128 + D of 256 TMEM columns
  static constexpr uint32_t TMq_S = 0, TMq_DP = 64, TMq_ACC = 128, TMq_COLS = 256;
  static constexpr uint32_t OFF_Q = 0, OFF_GH = TILE_A, OFF_GL = 2 * TILE_A;
  static constexpr uint32_t OFF_K = 3 * TILE_A;
  static constexpr uint32_t OFF_V = OFF_K + kNSq * TILE_B;
  static constexpr uint32_t OFF_COL = OFF_V + kNSq * TILE_B;  // ik | iv | cos | sin [64] + meta
  static constexpr uint32_t COLB = 4 * kBN * 4 + 16;
  static constexpr uint32_t OFF_TAB = OFF_COL + kNSq * COLB;
  static constexpr uint32_t OFF_BAR = OFF_TAB + 2 * kBN * 4;
  static constexpr int BAR_A = 0, BAR_FULL = 1, BAR_EMPTY = BAR_FULL + kNSq,
                       BAR_SD = BAR_EMPTY + kNSq, BAR_P = BAR_SD + 1, BAR_DONE = BAR_P + 1;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 8 * 16;
  static constexpr uint32_t SMEM = OFF_MISC + 64 + 1024;
  static_assert(kMinBlocks * (SMEM + 1024) <= 228 * 1024, "CTAs per SM");
  static_assert(TMq_ACC + D <= TMq_COLS, "TMEM budget");
};

// kDrop: attention dropout on alpha (counter-based bits, AttnShape::drop_thr)
template <bool kDrop, int D>
__global__ void __launch_bounds__(kThreads, DqCfg<D>::kMinBlocks)
    tc_bwd_dq_kernel(AttnShape s, BwdPtrs p, Aux ax, const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV) {
  using C = DqCfg<D>;
  constexpr int kD = D, kNSq = C::kNSq;
  constexpr uint32_t TILE_A = C::TILE_A, TILE_B = C::TILE_B, HALF_A = C::HALF_A,
                     HALF_B = C::HALF_B;
  constexpr uint32_t TMq_S = C::TMq_S, TMq_DP = C::TMq_DP, TMq_ACC = C::TMq_ACC,
                     TMq_COLS = C::TMq_COLS;
  constexpr uint32_t OFF_Q = C::OFF_Q, OFF_GH = C::OFF_GH, OFF_GL = C::OFF_GL, OFF_K = C::OFF_K,
                     OFF_V = C::OFF_V, OFF_COL = C::OFF_COL, COLB = C::COLB, OFF_TAB = C::OFF_TAB,
                     OFF_BAR = C::OFF_BAR, OFF_MISC = C::OFF_MISC;
  constexpr int BAR_A = C::BAR_A, BAR_FULL = C::BAR_FULL, BAR_EMPTY = C::BAR_EMPTY,
                BAR_SD = C::BAR_SD, BAR_P = C::BAR_P, BAR_DONE = C::BAR_DONE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_addr);
  float* colp = reinterpret_cast<float*>(gbase + OFF_COL);
  float* tab = reinterpret_cast<float*>(gbase + OFF_TAB);
  uint32_t* misc = reinterpret_cast<uint32_t*>(gbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
  const uint32_t bars = base + OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / s.H, h = bh % s.H;
  const long long i0 = (long long)blockIdx.x * kBM;
  const bool causal = s.causal != 0;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  const long long p0 = i0 + s.q_offset;
  long long ilast = i0 + kBM - 1;
  if (ilast > s.Tq - 1) ilast = s.Tq - 1;
  long long lo, hi;
  key_range(p0, ilast + s.q_offset, dmax, causal, s.Tk, lo, hi);
  const bool any = dmax >= 0 && lo <= hi;
  const int kt0 = any ? (int)(lo / kBN) : 0;
  const int n = any ? (int)(hi / kBN) - kt0 + 1 : 0;

  if (tid == 0) {
    mbar_init(bar(BAR_A), 1);
    for (int i = 0; i < kNSq; ++i) {
      // one arrival with the TMA byte count, one after the column factors
      mbar_init(bar(BAR_FULL + i), 2);
      mbar_init(bar(BAR_EMPTY + i), 1);
    }
    mbar_init(bar(BAR_SD), 1);
    mbar_init(bar(BAR_P), kCompute);
    mbar_init(bar(BAR_DONE), 2);
    misc[1] = misc[2] = misc[3] = misc[4] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(base + OFF_MISC, TMq_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == 8) {
    // ---------------------------------------------------------- producer
    // lane 0 issues the TMA copies: Q, G_hi, G_lo once (128 rows; G_lo is
    // batch b + B of the two-plane G map), then per key tile K, V and the
    // 1/|k|, 1/|v| runs with the tile's maxima; the warp fills the column
    // (cos, sin) by rotation
    if (lane == 0) {
      mbar_arrive_expect_tx(bar(BAR_A), 3 * TILE_A);
#pragma unroll
      for (int hf = 0; hf < kD / 64; ++hf) {
        tma_load_4d(base + OFF_Q + hf * HALF_A, &tmQ, 64 * hf, h, (int)i0, b, bar(BAR_A));
        tma_load_4d(base + OFF_GH + hf * HALF_A, &tmG, 64 * hf, h, (int)i0, b, bar(BAR_A));
        tma_load_4d(base + OFF_GL + hf * HALF_A, &tmG, 64 * hf, h, (int)i0, b + s.B,
                    bar(BAR_A));
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int c = lane + 32 * hh;
      float sn, cs;
      sincospif((float)c / w, &sn, &cs);
      tab[c] = cs;
      tab[kBN + c] = sn;
    }
    __syncwarp();
    const float cphi0 = tab[lane], sphi0 = tab[kBN + lane];
    const float cphi1 = tab[lane + 32], sphi1 = tab[kBN + lane + 32];
    const float* ikh = ax.ikT + (long long)bh * ax.Tkp;
    const float* ivh = ax.ivT + (long long)bh * ax.Tkp;
    const float4* mh = ax.mk + (long long)bh * (ax.Tkp / kBN);
    int issued = 0;
    for (int j = 0; j < n; ++j) {
      const int st = j % kNSq;
      if (j >= kNSq) {
        int okw = 1;
        if (lane == 0) okw = mbar_wait(bar(BAR_EMPTY + st), ((j / kNSq) - 1) & 1, abort_flag, kWaitLimitNs);
        if (!__shfl_sync(0xffffffffu, okw, 0)) break;
      }
      const int kt = kt0 + j;
      const long long j0 = (long long)kt * kBN;
      const uint32_t kb = base + OFF_K + st * TILE_B, vb = base + OFF_V + st * TILE_B;
      const uint32_t colb = base + OFF_COL + st * COLB;
      float* col = colp + st * (COLB / 4);
      if (lane == 0) {
        const uint32_t fb = bar(BAR_FULL + st);
        mbar_arrive_expect_tx(fb, 2 * TILE_B + 2 * kBN * 4 + 16);
#pragma unroll
        for (int hf = 0; hf < kD / 64; ++hf) {
          tma_load_4d(kb + hf * HALF_B, &tmK, 64 * hf, h, (int)j0, b, fb);
          tma_load_4d(vb + hf * HALF_B, &tmV, 64 * hf, h, (int)j0, b, fb);
        }
        bulk_g2s(colb, ikh + j0, kBN * 4, fb);
        bulk_g2s(colb + kBN * 4, ivh + j0, kBN * 4, fb);
        bulk_g2s(colb + 4 * kBN * 4, mh + kt, 16, fb);
      }
      issued = j + 1;
      float sb = 0.f, cb = 0.f;
      if (lane == 0) sincospif((float)(j0 - p0) / w, &sb, &cb);
      sb = __shfl_sync(0xffffffffu, sb, 0);
      cb = __shfl_sync(0xffffffffu, cb, 0);
      col[2 * kBN + lane] = cb * cphi0 - sb * sphi0;
      col[3 * kBN + lane] = sb * cphi0 + cb * sphi0;
      col[2 * kBN + lane + 32] = cb * cphi1 - sb * sphi1;
      col[3 * kBN + lane + 32] = sb * cphi1 + cb * sphi1;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_FULL + st));
    }
    if (lane == 0 && *abort_flag) {
      // let the copies already issued land before the CTA's smem goes away
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(bar(BAR_A), 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
      for (int j = issued > kNSq ? issued - kNSq : 0; j < issued; ++j)
        while (!mbar_try_wait(bar(BAR_FULL + j % kNSq), (j / kNSq) & 1) &&
               globaltimer() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(kBM, kBN, 0, 0);
      constexpr uint32_t idQ = idesc_bf16(kBM, kD, 0, 1);
      bool started = false, ok = mbar_wait(bar(BAR_A), 0, abort_flag, kWaitLimitNs);
      // S_j, dP_j into the single S / dP buffers; the next pair is issued
      // after dQ_j, which reads dS_j from the dP columns (in-order execution)
      auto issue_sd = [&](int jj) -> bool {
        const int st = jj % kNSq;
        if (!mbar_wait(bar(BAR_FULL + st), (jj / kNSq) & 1, abort_flag, kWaitLimitNs)) return false;
        tc_fence_after();
        const uint32_t kb = base + OFF_K + st * TILE_B, vb = base + OFF_V + st * TILE_B;
        // K-steps of 16 over the D / 64 column halves (four per half)
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * HALF_A + (kk & 3) * 32, ob = (kk >> 2) * HALF_B + (kk & 3) * 32;
          mma_ss(tmem + TMq_S, desc_sw128(base + OFF_Q + oa, 16, 1024),
                 desc_sw128(kb + ob, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * HALF_A + (kk & 3) * 32, ob = (kk >> 2) * HALF_B + (kk & 3) * 32;
          mma_ss(tmem + TMq_DP, desc_sw128(base + OFF_GH + oa, 16, 1024),
                 desc_sw128(vb + ob, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * HALF_A + (kk & 3) * 32, ob = (kk >> 2) * HALF_B + (kk & 3) * 32;
          mma_ss(tmem + TMq_DP, desc_sw128(base + OFF_GL + oa, 16, 1024),
                 desc_sw128(vb + ob, 16, 1024), idS, 1u);
        }
        mma_commit(bar(BAR_SD));
        return true;
      };
      if (n > 0) ok = issue_sd(0);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kNSq;
        ok = mbar_wait(bar(BAR_P), j & 1, abort_flag, kWaitLimitNs);
        if (!ok) break;
        tc_fence_after();
        // dS_j (bf16) sits in the first 16 columns of each compute group's
        // 32-column half of the dP buffer
        const uint32_t kb = base + OFF_K + st * TILE_B;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts(tmem + TMq_ACC, tmem + TMq_DP + (kk >> 1) * 32 + (kk & 1) * 8,
                 desc_sw128(kb + kk * 16 * 128, HALF_B, 1024), idQ,
                 (started || kk > 0) ? 1u : 0u);
        started = true;
        mma_commit(bar(BAR_EMPTY + st));
        if (j + 1 < n) ok = issue_sd(j + 1);
      }
      misc[3] = started ? 1u : 0u;
      mma_commit(bar(BAR_DONE));
      mbar_arrive(bar(BAR_DONE));
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- compute
    const int g = warp >> 2;                 // warpgroup: columns [32g, 32g+32)
    const int t = tid & 127;                 // query row = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int cb = 32 * g;
    const long long i = i0 + t;
    const float iq = (i < s.Tq) ? ax.iqT[(long long)bh * ax.Tqp + i] : 0.f;
    const float rq = r * iq;
    // attention dropout: this query row's counter key
    const uint32_t drow = kDrop ? drop_row(drop_bh_key(s, (uint32_t)bh), (uint32_t)i) : 0u;
    float crow, srow;
    {
      float sn, cs;
      sincospif((float)t / w, &sn, &cs);
      crow = 0.5f * cs;
      srow = 0.5f * sn;
    }
    const float omr = 1.0f - r;
    const long long pos = i + s.q_offset;
    const float2 rq2 = make_float2(rq, rq), omr2 = make_float2(omr, omr);
    const float2 cr2 = make_float2(crow, crow), sr2 = make_float2(srow, srow);
    const float2 half2 = make_float2(0.5f, 0.5f), twor2 = make_float2(2.f * r, 2.f * r);
    bool ok = true;
    // stage / phase kept incrementally; positions in 32-bit
    int st = 0, st_ph = 0;
    const int p0i = (int)p0, posi = (int)pos;
    const int in_lo = p0i + kBM - 1 - dmax, in_hi = causal ? p0i : p0i + dmax;
    int j0i = kt0 * kBN;
    for (int j = 0; j < n; ++j, j0i += kBN) {
      ok = mbar_wait(bar(BAR_FULL + st), st_ph, abort_flag, kWaitLimitNs) &&
           mbar_wait(bar(BAR_SD), j & 1, abort_flag, kWaitLimitNs);
      // warp-uniform verdict (the TMEM accesses below are warp-collective);
      // a warp that gives up leaves the loop alone -- every other wait on its
      // arrivals is bounded and sees the abort flag
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld32(tmem + TMq_S + cb + lane_off, sv);
      tmem_ld32(tmem + TMq_DP + cb + lane_off, dv);
      tmem_wait_ld();
      const float* col = colp + st * (COLB / 4);
      int imax = (int)sv[0];
#pragma unroll
      for (int c = 1; c + 1 < 32; c += 2) imax = __vimax3_s32(imax, (int)sv[c], (int)sv[c + 1]);
      imax = max(imax, (int)sv[31]);
      const bool mine = r < 1.0f ||
                        (imax > 0 && fmaf(rq, __int_as_float(imax) * col[4 * kBN], omr) > 0.f);
      // liveness per warp block (32 rows x 32 columns): a dead block stores
      // zeros, so the warps never wait on one another within a tile
      const bool live = __any_sync(0xffffffffu, mine);
      if (live) {
        const bool inside = j0i >= in_lo && j0i + kBN - 1 <= in_hi;
        const int clo_ = posi - dmax - j0i - cb, chi_ = (causal ? posi : posi + dmax) - j0i - cb;
        const int iclo = inside ? 0 : (clo_ < 0 ? 0 : (clo_ > 32 ? 32 : clo_));
        const int ichi = inside ? 31 : (chi_ < -1 ? -1 : (chi_ > 31 ? 31 : chi_));
        const float4* ik4 = reinterpret_cast<const float4*>(col + cb);
        const float4* iv4 = reinterpret_cast<const float4*>(col + kBN + cb);
        const float4* cc4 = reinterpret_cast<const float4*>(col + 2 * kBN + cb);
        const float4* sc4 = reinterpret_cast<const float4*>(col + 3 * kBN + cb);
        uint32_t pk[16];
        // interior tiles run without the window-edge selects
        auto run = [&](auto edge) {
          constexpr bool EDGE = decltype(edge)::value;
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 ikv = ik4[q4], ivv = iv4[q4], ccv = cc4[q4], scv = sc4[q4];
#pragma unroll
            for (int hp = 0; hp < 2; ++hp) {
              const int c = 4 * q4 + 2 * hp;
              const float2 ik2 = hp ? make_float2(ikv.z, ikv.w) : make_float2(ikv.x, ikv.y);
              const float2 iv2 = hp ? make_float2(ivv.z, ivv.w) : make_float2(ivv.x, ivv.y);
              const float2 cc2 = hp ? make_float2(ccv.z, ccv.w) : make_float2(ccv.x, ccv.y);
              const float2 sc2 = hp ? make_float2(scv.z, scv.w) : make_float2(scv.x, scv.y);
              const float2 x = __fmul2_rn(make_float2(__uint_as_float(sv[c]),
                                                      __uint_as_float(sv[c + 1])), ik2);
              // relu(t) = saturate(t): t = 1 - r (1 - S) <= 1, so the clamp is free
              float a0 = __saturatef(fmaf(rq, x.x, omr)), a1 = __saturatef(fmaf(rq, x.y, omr));
              if (EDGE) {
                a0 = (c >= iclo && c <= ichi) ? a0 : 0.f;
                a1 = (c + 1 >= iclo && c + 1 <= ichi) ? a1 : 0.f;
              }
              if (kDrop) {
                const uint32_t jk = (uint32_t)(j0i + cb + c);
                a0 = drop_keep(drow, jk, s.drop_thr) ? a0 : 0.f;
                a1 = drop_keep(drow, jk + 1u, s.drop_thr) ? a1 : 0.f;
              }
              const float2 a2 = make_float2(a0, a1);
              const float2 m2 = __ffma2_rn(cr2, cc2, __ffma2_rn(sr2, sc2, half2));
              // dS / (2 r) = (G v) (1/|v| 1/|k|) m a; the 2 r goes to the epilogue
              const float2 am = __fmul2_rn(a2, m2);
              const float2 ds = __fmul2_rn(__fmul2_rn(make_float2(__uint_as_float(dv[c]),
                                                                  __uint_as_float(dv[c + 1])),
                                                      iv2),
                                           am);
              pk[2 * q4 + hp] = pack_bf16(ds.x, ds.y);
            }
          }
        };
        if (inside)
          run(std::false_type{});
        else
          run(std::true_type{});
        tmem_st16(tmem + TMq_DP + cb + lane_off, pk);   // over this group's dP
      } else {
        const uint32_t zero[16] = {};
        tmem_st16(tmem + TMq_DP + cb + lane_off, zero);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(BAR_P));
      if (++st == kNSq) { st = 0; st_ph ^= 1; }
    }
    // epilogue (warpgroup 0): dQ -> normalisation Jacobian -> dq
    if (g == 0) {
      ok = ok && mbar_wait(bar(BAR_DONE), 0, abort_flag, kWaitLimitNs);
      // tcgen05.ld is warp-collective: every lane takes the same branch
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const bool st_row = ok && i < s.Tq;
      const long long ii = st_row ? i : 0;
      const bf16* qrow = reinterpret_cast<const bf16*>(p.q.p) + (long long)b * p.q.sb +
                         ii * p.q.st + (long long)h * kD;
      bf16* orow = reinterpret_cast<bf16*>(p.dq.p) + (long long)b * p.dq.sb + ii * p.dq.st +
                   (long long)h * kD;
      // dS was stored without its 2 r
      store_unit_jacobian_tmem<kD>(tmem + TMq_ACC + lane_off, ok && misc[3],
                               2.0f * r * (kDrop ? s.drop_scale : 1.0f), qrow, iq,
                               orow, st_row);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TMq_COLS);
  if (tid == 0 && *abort_flag) atomicExch(status_word(), (int)SCREEN_ERR_TIMEOUT);
}

// ===========================================================================
// dk / dv kernel
// ===========================================================================
// D = 64: the fused kernel (dQ here too) with a 4-stage ring; D = 128 (and
// the fixed-order path) without dQ: 3 stages, no dS^T staging, and the dV /
// dK accumulators take D columns each.
template <int D, bool kFuse>
struct KvCfg {
  static constexpr int kNS = D == 64 ? 4 : 3;
  static constexpr uint32_t TILE_A = kBM * D * 2, TILE_B = kBN * D * 2;
  static constexpr uint32_t HALF_A = kBM * 128, HALF_B = kBN * 128;
  static constexpr uint32_t OFF_K = 0, OFF_V = TILE_A;
  static constexpr uint32_t OFF_Q = 2 * TILE_A;          // per stage: Q | G_hi | G_lo
  static constexpr uint32_t STAGE = 3 * TILE_B;
  // dS^T staging for the fused dQ MMA: two buffers, each a pair of query tiles
  // [128 keys][64 queries] bf16 (SW128), 16 KB apart (the operand's LBO)
  static constexpr uint32_t OFF_STG = OFF_Q + kNS * STAGE;
  static constexpr uint32_t STG_PAIR = 2 * kBM * 64 * 2;
  // per stage: iq | cos | sin [64] + meta (16 B) + dropout row keys of the 64 queries
  static constexpr uint32_t OFF_COL = OFF_STG + (kFuse ? 2 * STG_PAIR : 0);
  static constexpr uint32_t COLB = 3 * kBN * 4 + 16 + kBN * 4;
  static constexpr uint32_t OFF_TAB = OFF_COL + kNS * COLB;
  static constexpr uint32_t OFF_RED = OFF_TAB + 2 * kBN * 4;   // [2][8] dr / dw warp sums
  static constexpr uint32_t OFF_BAR = OFF_RED + 64 * 4;
  static constexpr int BAR_A = 0, BAR_FULL = 1, BAR_EMPTY = BAR_FULL + kNS,
                       BAR_SD = BAR_EMPTY + kNS, BAR_P = BAR_SD + 2, BAR_DONE = BAR_P + 2,
                       BAR_DQF = BAR_DONE + 1, BAR_DQE = BAR_DQF + 2, BAR_SF = BAR_DQE + 2,
                       BAR_COUNT = BAR_SF + 2;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 8 * 24;
  static constexpr uint32_t SMEM = OFF_MISC + 64 + 1024;
  // TMEM: S and dP double-buffered; alpha / dS (bf16) written over the S / dP
  // columns they came from; dV, dK (and with kFuse two dQ accumulators)
  static constexpr uint32_t TK_S = 0, TK_DP = 128, TK_ACCV = 256, TK_ACCK = 256 + D,
                            TK_ACCQ = 384;
  static_assert(BAR_COUNT <= 24, "barrier space");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(OFF_STG % 1024 == 0 && STG_PAIR == 8 * 4096, "dQ drain regions");
  static_assert(TK_ACCK + D <= TM_COLS && (!kFuse || (D == 64 && TK_ACCQ + 128 <= TM_COLS)),
                "TMEM budget");
};

// kFuse: dQ is computed here too (dQ += dS K on the tensor cores per pair of
// query tiles, added into an fp32 accumulator with vector reductions);
// otherwise tc_bwd_dq_kernel computes it (deterministic order)
// kDrop: attention dropout on alpha (counter-based bits, AttnShape::drop_thr)
template <bool kFuse, bool kDrop, int D = 64>
__global__ void __launch_bounds__(kThreads, 1)
    tc_bwd_kv_kernel(AttnShape s, BwdPtrs p, Aux ax, const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmG, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmDQ) {
  using C = KvCfg<D, kFuse>;
  constexpr int kD = D, kNS = C::kNS;
  constexpr uint32_t TILE_A = C::TILE_A, TILE_B = C::TILE_B, HALF_A = C::HALF_A,
                     HALF_B = C::HALF_B;
  constexpr uint32_t OFF_K = C::OFF_K, OFF_V = C::OFF_V, OFF_Q = C::OFF_Q, STAGE = C::STAGE,
                     OFF_STG = C::OFF_STG, STG_PAIR = C::STG_PAIR, OFF_COL = C::OFF_COL,
                     COLB = C::COLB, OFF_TAB = C::OFF_TAB, OFF_RED = C::OFF_RED,
                     OFF_BAR = C::OFF_BAR, OFF_MISC = C::OFF_MISC;
  constexpr int BAR_A = C::BAR_A, BAR_FULL = C::BAR_FULL, BAR_EMPTY = C::BAR_EMPTY,
                BAR_SD = C::BAR_SD, BAR_P = C::BAR_P, BAR_DONE = C::BAR_DONE,
                BAR_DQF = C::BAR_DQF, BAR_DQE = C::BAR_DQE, BAR_SF = C::BAR_SF;
  constexpr uint32_t TK_S = C::TK_S, TK_DP = C::TK_DP, TK_ACCV = C::TK_ACCV,
                     TK_ACCK = C::TK_ACCK, TK_ACCQ = C::TK_ACCQ;
  static_assert(!kFuse || D == 64, "the fused dQ path is built for D = 64");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_addr);
  float* colp = reinterpret_cast<float*>(gbase + OFF_COL);
  float* tab = reinterpret_cast<float*>(gbase + OFF_TAB);
  float* red = reinterpret_cast<float*>(gbase + OFF_RED);
  uint32_t* misc = reinterpret_cast<uint32_t*>(gbase + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
  const uint32_t bars = base + OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA -> (b, h, key tile) through the longest-first order
  const int nkt = (s.Tk + kBM - 1) / kBM;
  const long long item = ax.order[blockIdx.x];
  const int bh = (int)(item / nkt), b = bh / s.H, h = bh % s.H;
  const int kx = (int)(item % nkt);
  const long long j0 = (long long)kx * kBM;
  const bool causal = s.causal != 0;
  const float r = s.r[h], w = s.w[h];
  const int dmax = window_dmax(w);
  long long jlast = j0 + kBM - 1;
  if (jlast > s.Tk - 1) jlast = s.Tk - 1;
  long long plo, phi;
  query_pos_range(j0, jlast, dmax, causal, plo, phi);
  long long ilo = plo - s.q_offset, ihi = phi - s.q_offset;
  if (ilo < 0) ilo = 0;
  if (ihi > s.Tq - 1) ihi = s.Tq - 1;
  const bool any = dmax >= 0 && ilo <= ihi;
  const int qt0 = any ? (int)(ilo / kBN) : 0;
  const int n = any ? (int)(ihi / kBN) - qt0 + 1 : 0;

  if (tid == 0) {
    mbar_init(bar(BAR_A), 1);
    for (int i = 0; i < kNS; ++i) {
      // one arrival with the TMA byte count, one after the column factors
      mbar_init(bar(BAR_FULL + i), 2);
      mbar_init(bar(BAR_EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(BAR_SD + i), 1);
      mbar_init(bar(BAR_P + i), kCompute);
      mbar_init(bar(BAR_DQF + i), 1);
      mbar_init(bar(BAR_DQE + i), kCompute);
      mbar_init(bar(BAR_SF + i), kCompute / 32);
    }
    mbar_init(bar(BAR_DONE), 2);
    misc[1] = misc[2] = misc[3] = misc[4] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(base + OFF_MISC, TM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  const bf16* kh = reinterpret_cast<const bf16*>(p.k.p) + (long long)b * p.k.sb + (long long)h * kD;
  const bf16* vh = reinterpret_cast<const bf16*>(p.v.p) + (long long)b * p.v.sb + (long long)h * kD;
  float acc_r = 0.f, acc_w = 0.f;

  if (warp == 8) {
    // ---------------------------------------------------------- producer
    // lane 0 issues the TMA copies: K, V once (128 rows), then per query
    // tile Q, G_hi, G_lo and the 1/|q| run with its maximum; the warp fills
    // the column (cos, sin) by rotation
    if (lane == 0) {
      mbar_arrive_expect_tx(bar(BAR_A), 2 * TILE_A);
#pragma unroll
      for (int hf = 0; hf < kD / 64; ++hf) {
        tma_load_4d(base + OFF_K + hf * HALF_A, &tmK, 64 * hf, h, (int)j0, b, bar(BAR_A));
        tma_load_4d(base + OFF_V + hf * HALF_A, &tmV, 64 * hf, h, (int)j0, b, bar(BAR_A));
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int c = lane + 32 * hh;
      float sn, cs;
      sincospif((float)c / w, &sn, &cs);
      tab[c] = cs;
      tab[kBN + c] = sn;
    }
    __syncwarp();
    const float cphi0 = tab[lane], sphi0 = tab[kBN + lane];
    const float cphi1 = tab[lane + 32], sphi1 = tab[kBN + lane + 32];
    const uint32_t dbhk = kDrop ? drop_bh_key(s, (uint32_t)bh) : 0u;
    const float* iqh = ax.iqT + (long long)bh * ax.Tqp;
    const float4* mh = ax.mq + (long long)bh * (ax.Tqp / kBN);
    int issued = 0;
    for (int j = 0; j < n; ++j) {
      const int st = j % kNS;
      if (j >= kNS) {
        int okw = 1;
        if (lane == 0) okw = mbar_wait(bar(BAR_EMPTY + st), ((j / kNS) - 1) & 1, abort_flag, kWaitLimitNs);
        if (!__shfl_sync(0xffffffffu, okw, 0)) break;
      }
      const int qt = qt0 + j;
      const long long iq0 = (long long)qt * kBN;
      const uint32_t sb_ = base + OFF_Q + st * STAGE;
      const uint32_t colb = base + OFF_COL + st * COLB;
      float* col = colp + st * (COLB / 4);
      if (lane == 0) {
        const uint32_t fb = bar(BAR_FULL + st);
        mbar_arrive_expect_tx(fb, 3 * TILE_B + kBN * 4 + 16);
#pragma unroll
        for (int hf = 0; hf < kD / 64; ++hf) {
          tma_load_4d(sb_ + hf * HALF_B, &tmQ, 64 * hf, h, (int)iq0, b, fb);
          tma_load_4d(sb_ + TILE_B + hf * HALF_B, &tmG, 64 * hf, h, (int)iq0, b, fb);
          tma_load_4d(sb_ + 2 * TILE_B + hf * HALF_B, &tmG, 64 * hf, h, (int)iq0, b + s.B, fb);
        }
        bulk_g2s(colb, iqh + iq0, kBN * 4, fb);
        bulk_g2s(colb + 3 * kBN * 4, mh + qt, 16, fb);
      }
      issued = j + 1;
      // column angle pi (iq0 + c + q_offset - j0) / w by rotation
      float sb = 0.f, cbv = 0.f;
      if (lane == 0) sincospif((float)(iq0 + s.q_offset - j0) / w, &sb, &cbv);
      sb = __shfl_sync(0xffffffffu, sb, 0);
      cbv = __shfl_sync(0xffffffffu, cbv, 0);
      col[kBN + lane] = cbv * cphi0 - sb * sphi0;
      col[2 * kBN + lane] = sb * cphi0 + cbv * sphi0;
      col[kBN + lane + 32] = cbv * cphi1 - sb * sphi1;
      col[2 * kBN + lane + 32] = sb * cphi1 + cbv * sphi1;
      if constexpr (kDrop) {
        // dropout row keys of this tile's query indices
        uint32_t* dk = reinterpret_cast<uint32_t*>(col + 3 * kBN + 4);
        dk[lane] = drop_row(dbhk, (uint32_t)(iq0 + lane));
        dk[lane + 32] = drop_row(dbhk, (uint32_t)(iq0 + lane + 32));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_FULL + st));
    }
    if (lane == 0 && *abort_flag) {
      // let the copies already issued land before the CTA's smem goes away
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(bar(BAR_A), 0) && globaltimer() - t0 < kWaitLimitNs) {
      }
      for (int j = issued > kNS ? issued - kNS : 0; j < issued; ++j)
        while (!mbar_try_wait(bar(BAR_FULL + j % kNS), (j / kNS) & 1) &&
               globaltimer() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(kBM, kBN, 0, 0);
      constexpr uint32_t idMN = idesc_bf16(kBM, kD, 0, 1);
      constexpr uint32_t idQ = idesc_bf16(kBM, kD, 1, 1);   // A = dS^T staging, MN-major
      bool started = false, ok = mbar_wait(bar(BAR_A), 0, abort_flag, kWaitLimitNs);
      // shared-memory descriptors built once: an operand at byte offset x
      // from a base is base_desc + x / 16 (the start-address field holds
      // address / 16 in 14 bits; every address here is below 256 KB)
      const uint64_t dK_k = desc_sw128(base + OFF_K, 16, 1024);       // K-major (S: A = K)
      const uint64_t dV_k = desc_sw128(base + OFF_V, 16, 1024);       // K-major (dP: A = V)
      const uint64_t dQ_k = desc_sw128(base + OFF_Q, 16, 1024);       // stage 0 Q, K-major
      const uint64_t dQ_mn = desc_sw128(base + OFF_Q, HALF_B, 1024);  // stage 0 Q, MN-major
      const uint64_t dStg = desc_sw128(base + OFF_STG, TILE_A, 1024); // dS^T staging, MN-major
      const uint64_t dK_mn = desc_sw128(base + OFF_K, TILE_A, 1024);  // K, MN-major (dQ: B)
      int pair_i = 0;   // pairs of query tiles whose dQ has been issued
      auto issue_kv = [&](int jj) -> bool {
        const int bb = jj & 1, st = jj % kNS;
        if (!mbar_wait(bar(BAR_P + bb), (jj >> 1) & 1, abort_flag, kWaitLimitNs)) return false;
        tc_fence_after();
        // alpha_j / dS_j sit in the first 16 columns of each compute group's
        // 32-column half of the S / dP buffer
        const uint64_t qd = dQ_mn + (uint64_t)((st * STAGE) >> 4), gd = qd + (TILE_B >> 4);
        const uint32_t s0 = started ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t pcol = 64 * bb + (kk >> 1) * 32 + (kk & 1) * 8;
          mma_ts(tmem + TK_ACCV, tmem + TK_S + pcol, gd + kk * (16 * 128 / 16), idMN,
                 kk > 0 ? 1u : s0);
          mma_ts(tmem + TK_ACCK, tmem + TK_DP + pcol, qd + kk * (16 * 128 / 16), idMN,
                 kk > 0 ? 1u : s0);
        }
        started = true;
        if constexpr (kFuse) {
          const int qt = qt0 + jj;
          if ((qt & 1) || jj == n - 1) {
            // the pair of query tiles (qt & ~1, qt | 1) is complete:
            // dQ[128 q][64 d] = dS (A: [key][q] staging, MN-major, M = 128) x K
            const int buf = pair_i & 1;
            if (pair_i >= 2 &&
                !mbar_wait(bar(BAR_DQE + buf), ((pair_i >> 1) - 1) & 1, abort_flag, kWaitLimitNs))
              return false;
            tc_fence_after();
            const uint64_t sd = dStg + (uint64_t)(buf * (STG_PAIR >> 4));
#pragma unroll
            for (int kk = 0; kk < kBM / 16; ++kk)
              mma_ss(tmem + TK_ACCQ + 64 * buf, sd + kk * (16 * 128 / 16),
                     dK_mn + kk * (16 * 128 / 16), idQ, kk > 0 ? 1u : 0u);
            mma_commit(bar(BAR_DQF + buf));
            ++pair_i;
          }
        }
        mma_commit(bar(BAR_EMPTY + st));
        return true;
      };
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kNS, bb = j & 1;
        // buffer bb held alpha / dS of tile j - 2, read by MMAs issued
        // before these (in-order execution)
        ok = mbar_wait(bar(BAR_FULL + st), (j / kNS) & 1, abort_flag, kWaitLimitNs);
        if (!ok) break;
        tc_fence_after();
        fence_proxy_async_smem();
        const uint64_t qd = dQ_k + (uint64_t)((st * STAGE) >> 4), ghd = qd + (TILE_B >> 4),
                       gld = qd + (2 * TILE_B >> 4);
        // S and dP (hi) interleaved, then dP (lo); K-steps of 16 over the
        // D / 64 column halves (descriptor units of 16 bytes)
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t oa = ((kk >> 2) * HALF_A + (kk & 3) * 32) >> 4,
                         ob = ((kk >> 2) * HALF_B + (kk & 3) * 32) >> 4;
          mma_ss(tmem + TK_S + kBN * bb, dK_k + oa, qd + ob, idS, kk > 0 ? 1u : 0u);
          mma_ss(tmem + TK_DP + kBN * bb, dV_k + oa, ghd + ob, idS, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t oa = ((kk >> 2) * HALF_A + (kk & 3) * 32) >> 4,
                         ob = ((kk >> 2) * HALF_B + (kk & 3) * 32) >> 4;
          mma_ss(tmem + TK_DP + kBN * bb, dV_k + oa, gld + ob, idS, 1u);
        }
        mma_commit(bar(BAR_SD + bb));
        if (j >= 1) ok = issue_kv(j - 1);
      }
      if (ok && n >= 1) ok = issue_kv(n - 1);
      misc[3] = started ? 1u : 0u;
      mma_commit(bar(BAR_DONE));
      mbar_arrive(bar(BAR_DONE));
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- compute
    const int g = warp >> 2;
    const int t = tid & 127;                   // key row = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int cb = 32 * g;
    const long long jrow = j0 + t;
    const bool valid = jrow < s.Tk;
    const bool keep = valid && !(s.kpm && s.kpm[(long long)b * s.kpm_sb + jrow]);
    const long long nidx = ((long long)b * s.Tk + (valid ? jrow : 0)) * s.H + h;
    const float ik = valid ? 1.0f / p.nk[nidx] : 0.f;
    const float iv = valid ? 1.0f / p.nv[nidx] : 0.f;
    const float rk = keep ? r * ik : 0.f;
    const float omr = keep ? 1.0f - r : -1.0f;  // masked key rows: t <= 0, a = 0
    float crow, srow;
    {
      float sn, cs;
      sincospif((float)t / w, &sn, &cs);
      crow = 0.5f * cs;
      srow = 0.5f * sn;
    }
    const float2 rk2 = make_float2(rk, rk), omr2 = make_float2(omr, omr);
    const float2 cr2 = make_float2(crow, crow), sr2 = make_float2(srow, srow);
    const float2 sr2x2 = make_float2(2.f * srow, 2.f * srow);
    const float2 ncr2x2 = make_float2(-2.f * crow, -2.f * crow);
    const float2 half2 = make_float2(0.5f, 0.5f), twor2 = make_float2(2.f * r, 2.f * r);
    const float2 iv2 = make_float2(iv, iv), ik2 = make_float2(ik, ik);
    const float2 m1 = make_float2(-1.f, -1.f);
    // dS for the dQ MMA: dq^ = sum_j dS k^ = sum_j dS (1/|k|) K, dS = (G v)(1/|v|) m 2 a r
    const float rq_f = 2.0f * r * iv * ik * (kDrop ? s.drop_scale : 1.0f);
    const float2 rqf2 = make_float2(rq_f, rq_f);
    float2 accr2 = make_float2(0.f, 0.f), accw2 = make_float2(0.f, 0.f);
    bool ok = true;
    int pair_c = -1;    // pair of query tiles this tile belongs to (CTA-local count)
    int todo = -1;      // a complete pair whose dQ is yet to be drained
    int todo_qt = 0;
    uint32_t* stg_words = reinterpret_cast<uint32_t*>(gbase + OFF_STG);
    // drain pair pp: the dQ accumulator block of this warp (query rows
    // 32 (warp % 4) .. + 32 of the pair, columns [32 g, 32 g + 32)) goes through
    // its 4 KB region of the pair's staging buffer -- free once the dQ MMA that
    // read it has completed -- into one TMA tensor reduce-add (fp32, SW128)
    // onto the accumulator.  The region is written again for pair pp + 2 only
    // after every warp has seen its reduce finish reading (BAR_SF).
    int sf_pending = -1;   // staging buffer whose reduce this warp has not yet released
    auto drain = [&](int pp, int pqt) -> bool {
      const int buf = pp & 1;
      bool okd = mbar_wait(bar(BAR_DQF + buf), (pp >> 1) & 1, abort_flag, kWaitLimitNs);
      okd = __all_sync(0xffffffffu, okd);
      if (!okd) return false;
      tc_fence_after();
      uint32_t dqv[32];
      tmem_ld32(tmem + TK_ACCQ + 64 * buf + cb + lane_off, dqv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar(BAR_DQE + buf));
      const uint32_t region = OFF_STG + buf * STG_PAIR + warp * 4096;
      uint8_t* rrow = gbase + region + lane * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(rrow + ((c ^ (lane & 7)) << 4)) =
            make_uint4(dqv[4 * c], dqv[4 * c + 1], dqv[4 * c + 2], dqv[4 * c + 3]);
      fence_proxy_async_smem();   // generic-proxy writes -> TMA reads
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_4d(&tmDQ, base + region, cb, h, (pqt & ~1) * kBN + 32 * (warp & 3), b);
        bulk_commit();
      }
      sf_pending = buf;
      return true;
    };
    // release the staging region of the last reduce once it has been read
    auto release = [&]() {
      if (sf_pending >= 0) {
        if (lane == 0) {
          bulk_wait_read<0>();
          mbar_arrive(bar(BAR_SF + sf_pending));
        }
        sf_pending = -1;
      }
    };
    // this thread's 4 chunks (16 B each) of row t in half `hf` of staging buffer `buf`
    auto stg_row = [&](int buf, int hf) -> uint4* {
      return reinterpret_cast<uint4*>(gbase + OFF_STG + buf * STG_PAIR + hf * TILE_A + t * 128);
    };
    (void)stg_words;
    for (int j = 0; j < n; ++j) {
      const int st = j % kNS, bb = j & 1;
      const int qt = qt0 + j;
      if (kFuse && (j == 0 || (qt & 1) == 0)) ++pair_c;
      ok = mbar_wait(bar(BAR_FULL + st), (j / kNS) & 1, abort_flag, kWaitLimitNs) &&
           mbar_wait(bar(BAR_SD + bb), (j >> 1) & 1, abort_flag, kWaitLimitNs);
      // warp-uniform verdict (the TMEM accesses below are warp-collective);
      // a warp that gives up leaves the loop alone -- every other wait on its
      // arrivals is bounded and sees the abort flag
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      if constexpr (kFuse) release();
      uint32_t sv[32], dv[32];
      tmem_ld32(tmem + TK_S + kBN * bb + cb + lane_off, sv);
      tmem_ld32(tmem + TK_DP + kBN * bb + cb + lane_off, dv);
      tmem_wait_ld();
      const float* col = colp + st * (COLB / 4);
      int imax = (int)sv[0];
#pragma unroll
      for (int c = 1; c + 1 < 32; c += 2) imax = __vimax3_s32(imax, (int)sv[c], (int)sv[c + 1]);
      imax = max(imax, (int)sv[31]);
      const bool mine = (r < 1.0f && keep) ||
                        (imax > 0 && fmaf(rk, __int_as_float(imax) * col[3 * kBN], omr) > 0.f);
      // liveness per warp block (32 rows x 32 columns): a dead block stores
      // zeros, so the warps never wait on one another within a tile
      const bool live = __any_sync(0xffffffffu, mine);
      uint32_t pq[16];   // dS for the dQ MMA (bf16 pairs), zero for a dead block
      if (live) {
        // positions in 32-bit (key / query indices and offsets are < 2^31)
        const int pq0 = (qt0 + j) * kBN + (int)s.q_offset, j0i = (int)j0, jr = (int)jrow;
        // d = p - j over the tile: [pq0 - (j0 + 127), pq0 + 63 - j0]
        const int dlo = pq0 - (j0i + kBM - 1), dhi = pq0 + kBN - 1 - j0i;
        const bool inside = causal ? (dlo >= 0 && dhi <= dmax) : (dlo >= -dmax && dhi <= dmax);
        // this row's valid query columns: p - j in [0, dmax] (causal) or [-dmax, dmax]
        const int clo_ = (causal ? jr : jr - dmax) - pq0 - cb;
        const int chi_ = jr + dmax - pq0 - cb;
        const int iclo = inside ? 0 : (clo_ < 0 ? 0 : (clo_ > 32 ? 32 : clo_));
        const int ichi = inside ? 31 : (chi_ < -1 ? -1 : (chi_ > 31 ? 31 : chi_));
        const float relb = (float)(jr - pq0 - cb);   // rel = j - p = relb - c
        const float2 relb2 = make_float2(relb, relb);
        const float4* iq4 = reinterpret_cast<const float4*>(col + cb);
        const float4* cv4 = reinterpret_cast<const float4*>(col + kBN + cb);
        const float4* sv4 = reinterpret_cast<const float4*>(col + 2 * kBN + cb);
        const uint32_t* dkey = reinterpret_cast<const uint32_t*>(col + 3 * kBN + 4) + cb;
        uint32_t pa[16], pd[16];
        // interior tiles run without the window-edge selects
        auto run = [&](auto edge) {
          constexpr bool EDGE = decltype(edge)::value;
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 iqv = iq4[q4], cvv = cv4[q4], svv = sv4[q4];
#pragma unroll
            for (int hp = 0; hp < 2; ++hp) {
              const int c = 4 * q4 + 2 * hp;
              const float2 iq2 = hp ? make_float2(iqv.z, iqv.w) : make_float2(iqv.x, iqv.y);
              const float2 cv2 = hp ? make_float2(cvv.z, cvv.w) : make_float2(cvv.x, cvv.y);
              const float2 sn2 = hp ? make_float2(svv.z, svv.w) : make_float2(svv.x, svv.y);
              const float2 x = __fmul2_rn(make_float2(__uint_as_float(sv[c]),
                                                      __uint_as_float(sv[c + 1])), iq2);
              // relu(t) = saturate(t): t = 1 - r (1 - S) <= 1, so the clamp is free
              float a0 = __saturatef(fmaf(rk, x.x, omr)), a1 = __saturatef(fmaf(rk, x.y, omr));
              if (EDGE) {
                a0 = (c >= iclo && c <= ichi) ? a0 : 0.f;
                a1 = (c + 1 >= iclo && c + 1 <= ichi) ? a1 : 0.f;
              }
              if (kDrop) {
                a0 = drop_keep(dkey[c], (uint32_t)jr, s.drop_thr) ? a0 : 0.f;
                a1 = drop_keep(dkey[c + 1], (uint32_t)jr, s.drop_thr) ? a1 : 0.f;
              }
              const float2 a2 = make_float2(a0, a1);
              const float2 m2 = __ffma2_rn(cr2, cv2, __ffma2_rn(sr2, sn2, half2));
              const float2 sinrel = __ffma2_rn(ncr2x2, sn2, __fmul2_rn(sr2x2, cv2));
              // G v without this row's 1/|v|: it and the 2 r of dS are row
              // constants applied in the epilogue and to the dr / dw sums
              const float2 dp2 = make_float2(__uint_as_float(dv[c]), __uint_as_float(dv[c + 1]));
              const float2 asq = __fmul2_rn(a2, a2);
              const float2 al = __fmul2_rn(asq, m2);
              const float2 q2 = __fmul2_rn(dp2, __fmul2_rn(a2, m2));  // dP m a / (1/|v|)
              const float2 ds = __fmul2_rn(q2, iq2);
              pa[2 * q4 + hp] = pack_bf16(al.x, al.y);
              pd[2 * q4 + hp] = pack_bf16(ds.x, ds.y);
              if constexpr (kFuse) {
                const float2 dq2 = __fmul2_rn(q2, rqf2);
                pq[2 * q4 + hp] = pack_bf16(dq2.x, dq2.y);
              }
              accr2 = __ffma2_rn(q2, __ffma2_rn(x, ik2, m1), accr2);
              const float2 rel = __fadd2_rn(relb2, make_float2(-(float)c, -(float)(c + 1)));
              accw2 = __ffma2_rn(__fmul2_rn(dp2, asq), __fmul2_rn(rel, sinrel), accw2);
            }
          }
        };
        if (inside)
          run(std::false_type{});
        else
          run(std::true_type{});
        // alpha / dS over this group's own S / dP columns (already loaded)
        tmem_st16(tmem + TK_S + kBN * bb + cb + lane_off, pa);
        tmem_st16(tmem + TK_DP + kBN * bb + cb + lane_off, pd);
      } else {
        const uint32_t zero[16] = {};
        tmem_st16(tmem + TK_S + kBN * bb + cb + lane_off, zero);
        tmem_st16(tmem + TK_DP + kBN * bb + cb + lane_off, zero);
#pragma unroll
        for (int c = 0; c < 16; ++c) pq[c] = 0u;
      }
      if constexpr (kFuse) {
        // dS^T row t (this group's 32 queries) into half (qt & 1) of the
        // pair's staging buffer, SW128 (16-byte chunk c of the row at c ^ (t % 8));
        // a pair this CTA only half covers gets zeros in the other half
        const int buf = pair_c & 1, hf = qt & 1;
        if (pair_c >= 2 && (j == 0 || hf == 0)) {
          // first write of this pair: the reduce of pair pair_c - 2 must have
          // finished reading the buffer in every warp
          const int pv = pair_c - 2;
          const bool okf = __all_sync(
              0xffffffffu, mbar_wait(bar(BAR_SF + buf), (pv >> 1) & 1, abort_flag, kWaitLimitNs));
          if (!okf) { ok = false; break; }
        }
        uint4* row = stg_row(buf, hf);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          row[(4 * g + c) ^ (t & 7)] =
              make_uint4(pq[4 * c], pq[4 * c + 1], pq[4 * c + 2], pq[4 * c + 3]);
        if ((j == 0 && hf == 1) || (j == n - 1 && hf == 0)) {
          uint4* other = stg_row(buf, hf ^ 1);
#pragma unroll
          for (int c = 0; c < 4; ++c) other[(4 * g + c) ^ (t & 7)] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();   // generic-proxy writes -> tensor-core reads
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(BAR_P + bb));
      if constexpr (kFuse) {
        // drain the pair completed one tile ago (its dQ MMA has had a tile's
        // time), then remember this one if it completes a pair
        if (todo >= 0) {
          if (!drain(todo, todo_qt)) { ok = false; break; }
          todo = -1;
        }
        if ((qt & 1) || j == n - 1) {
          todo = pair_c;
          todo_qt = qt;
        }
      }
    }
    if (kFuse && ok && todo >= 0) ok = drain(todo, todo_qt);
    // every reduce this warp issued completes before the CTA's shared memory goes away
    if (kFuse && lane == 0) bulk_wait<0>();
    // dr = sum dP m 2a (S - 1); kept scores carry the dropout scale
    const float dsc = kDrop ? s.drop_scale : 1.0f;
    acc_r = 2.f * iv * dsc * (accr2.x + accr2.y);
    acc_w = iv * dsc * (accw2.x + accw2.y);
    // epilogue: warpgroup 0 -> dk, warpgroup 1 -> dv (normalisation Jacobians)
    ok = ok && mbar_wait(bar(BAR_DONE), 0, abort_flag, kWaitLimitNs);
    // tcgen05.ld is warp-collective: every lane takes the same branch
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if constexpr (kD == 64) {
      float acc[64];
      if (ok && misc[3]) {
        tmem_ld64(tmem + (g == 0 ? TK_ACCK : TK_ACCV) + lane_off, acc);
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) acc[c] = 0.f;
      }
      if (ok && valid) {
        if (g == 0) {
          // dS was stored without this key's 2 r / |v|
#pragma unroll
          for (int c = 0; c < 64; ++c) acc[c] *= 2.0f * r * iv * dsc;
          store_unit_jacobian(acc, kh + jrow * p.k.st, ik,
                              reinterpret_cast<bf16*>(p.dk.p) + (long long)b * p.dk.sb +
                                  jrow * p.dk.st + (long long)h * kD);
        } else {
          if (kDrop) {
#pragma unroll
            for (int c = 0; c < 64; ++c) acc[c] *= dsc;
          }
          store_unit_jacobian(acc, vh + jrow * p.v.st, iv,
                              reinterpret_cast<bf16*>(p.dv.p) + (long long)b * p.dv.sb +
                                  jrow * p.dv.st + (long long)h * kD);
        }
      }
    } else {
      // D = 128: the accumulator rows are streamed from TMEM 32 columns at
      // a time through the normalisation Jacobian
      const bool okacc = ok && misc[3] != 0;
      const long long jr = valid ? jrow : 0;
      if (g == 0) {
        // dS was stored without this key's 2 r / |v|
        store_unit_jacobian_tmem<kD>(tmem + TK_ACCK + lane_off, okacc, 2.0f * r * iv * dsc,
                                     kh + jr * p.k.st, ik,
                                     reinterpret_cast<bf16*>(p.dk.p) + (long long)b * p.dk.sb +
                                         jr * p.dk.st + (long long)h * kD,
                                     ok && valid);
      } else {
        store_unit_jacobian_tmem<kD>(tmem + TK_ACCV + lane_off, okacc, dsc, vh + jr * p.v.st, iv,
                                     reinterpret_cast<bf16*>(p.dv.p) + (long long)b * p.dv.sb +
                                         jr * p.dv.st + (long long)h * kD,
                                     ok && valid);
      }
    }
  }
  // dr / dw partial of this CTA, fixed summation order
  acc_r = warp_sum(acc_r);
  acc_w = warp_sum(acc_w);
  if (lane == 0 && warp < 8) {
    red[warp] = acc_r;
    red[8 + warp] = acc_w;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    float sr = 0.f, sw = 0.f;
    for (int k2 = 0; k2 < 8; ++k2) {
      sr += red[k2];
      sw += red[8 + k2];
    }
    const long long P = (long long)s.B * nkt;
    const long long idx = (long long)h * P + (long long)b * nkt + kx;
    p.part_r[idx] = sr;
    p.part_w[idx] = sw;
    if (*abort_flag) atomicExch(status_word(), (int)SCREEN_ERR_TIMEOUT);
  }
  if (warp == 0) tmem_dealloc(tmem, TM_COLS);
}

// transposed inverse norms per (b, h) and per-64-tile maxima; grid
// (B*H*tiles, 2): y = 0 for q, y = 1 for k (and v)
__global__ void tc_bwd_aux_kernel(const float* __restrict__ nq, const float* __restrict__ nk,
                                  const float* __restrict__ nv, const uint8_t* kpm,
                                  long long kpm_sb, int B, int H, int Tq, int Tk, int Tqp,
                                  int Tkp, float* iqT, float* ikT, float* ivT, float4* mq,
                                  float4* mk) {
  const bool isk = blockIdx.y == 1;
  const int Tp = isk ? Tkp : Tqp, T = isk ? Tk : Tq;
  const int ntiles = Tp / kBN;
  const long long blk = blockIdx.x;
  if (blk >= (long long)B * H * ntiles) return;
  const long long bhh = blk / ntiles;
  const int tile = (int)(blk % ntiles);
  const int bb = (int)(bhh / H), hh = (int)(bhh % H);
  const int c = threadIdx.x;  // 64 threads
  const long long t = (long long)tile * kBN + c;
  float x = 0.f;
  if (t < T) {
    const long long idx = ((long long)bb * T + t) * H + hh;
    if (!isk) {
      x = 1.0f / nq[idx];
      iqT[bhh * Tp + t] = x;
    } else {
      x = 1.0f / nk[idx];
      ikT[bhh * Tp + t] = x;
      const bool masked = kpm && kpm[(long long)bb * kpm_sb + t];
      ivT[bhh * Tp + t] = masked ? 0.f : x / nv[idx];   // 1/|v| * 1/|k|
    }
  } else {
    if (!isk) iqT[bhh * Tp + t] = 0.f;
    else {
      ikT[bhh * Tp + t] = 0.f;
      ivT[bhh * Tp + t] = 0.f;
    }
  }
  __shared__ float sm[2];
  float m = x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((c & 31) == 0) sm[c >> 5] = m;
  __syncthreads();
  if (c == 0) (isk ? mk : mq)[blk] = make_float4(fmaxf(sm[0], sm[1]), 0.f, 0.f, 0.f);
}

long long padT(int T) { return ((long long)T + kBN - 1) / kBN * kBN; }
size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// dq = (1/|q|) (dq^ - (1/|q|)^2 (q . dq^) q) from the fp32 accumulator of the
// fused kernel; 16 lanes per row, 4 elements each
__global__ void __launch_bounds__(256) tc_bwd_dq_finalize_kernel(
    const float* __restrict__ acc, Rows q, const float* __restrict__ nq, OutRows dq, int B, int Tq,
    int H) {
  const long long rows = (long long)B * Tq * H;
  const long long row = (long long)blockIdx.x * 16 + (threadIdx.x >> 4);
  const int l = threadIdx.x & 15;
  const bool valid = row < rows;
  const long long rr = valid ? row : 0;
  const unsigned r32 = (unsigned)rr, bt = r32 / (unsigned)H;
  const unsigned hh = r32 - bt * (unsigned)H, t = bt % (unsigned)Tq, bb = bt / (unsigned)Tq;
  const float4 a = *reinterpret_cast<const float4*>(acc + rr * kD + 4 * l);
  const uint2 qu = *reinterpret_cast<const uint2*>(reinterpret_cast<const bf16*>(q.p) +
                                                   bb * q.sb + t * q.st + hh * kD + 4 * l);
  const float2 q0 = unpack_bf16(qu.x), q1 = unpack_bf16(qu.y);
  float dot = a.x * q0.x + a.y * q0.y + a.z * q1.x + a.w * q1.y;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o, 16);
  if (!valid) return;
  const float inv = 1.0f / nq[rr];
  const float cf = inv * inv * dot;
  uint2 o;
  o.x = pack_bf16(inv * (a.x - cf * q0.x), inv * (a.y - cf * q0.y));
  o.y = pack_bf16(inv * (a.z - cf * q1.x), inv * (a.w - cf * q1.y));
  *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(dq.p) + bb * dq.sb + t * dq.st + hh * kD +
                            4 * l) = o;
}

bool tc_bwd_supported(int dtype, int D) { return dtype == SCREEN_BF16 && (D == 64 || D == 128); }

size_t tc_bwd_aux_bytes(const AttnShape& s) {
  const long long BH = (long long)s.B * s.H, Tqp = padT(s.Tq), Tkp = padT(s.Tk);
  return al256(BH * Tqp * 4) + 2 * al256(BH * Tkp * 4) + al256(BH * (Tqp / kBN) * 16) +
         al256(BH * (Tkp / kBN) * 16) + al256((size_t)BH * s.Tq * kD * 4) +
         al256((size_t)BH * ((s.Tk + kBM - 1) / kBM) * 4);
}

long long tc_bwd_partials(const AttnShape& s) {
  return (long long)s.B * ((s.Tk + kBM - 1) / kBM);
}

namespace {
template <int D>
int tc_bwd_d(const AttnShape& s, const BwdPtrs& p, void* aux_ws, int stages, cudaStream_t st) {
  {
    // D = 128 has no fused kernel: dq comes from the query-major kernel
    const void* fns[6] = {(const void*)tc_bwd_dq_kernel<false, D>,
                          (const void*)tc_bwd_dq_kernel<true, D>,
                          (const void*)tc_bwd_kv_kernel<false, false, D>,
                          (const void*)tc_bwd_kv_kernel<false, true, D>,
                          D == 64 ? (const void*)tc_bwd_kv_kernel<true, false, 64> : nullptr,
                          D == 64 ? (const void*)tc_bwd_kv_kernel<true, true, 64> : nullptr};
    const int sm[6] = {(int)DqCfg<D>::SMEM, (int)DqCfg<D>::SMEM, (int)KvCfg<D, false>::SMEM,
                       (int)KvCfg<D, false>::SMEM, (int)KvCfg<64, true>::SMEM,
                       (int)KvCfg<64, true>::SMEM};
    for (int i = 0; i < 6; ++i) {
      if (!fns[i]) continue;
      const cudaError_t e = ensure_smem_optin(fns[i], sm[i]);
      if (e != cudaSuccess) return record_cuda_error(e);
    }
  }
  const long long BH = (long long)s.B * s.H, Tqp = padT(s.Tq), Tkp = padT(s.Tk);
  uint8_t* w8 = reinterpret_cast<uint8_t*>(aux_ws);
  Aux ax;
  float* iqT = reinterpret_cast<float*>(w8);
  w8 += al256(BH * Tqp * 4);
  float* ikT = reinterpret_cast<float*>(w8);
  w8 += al256(BH * Tkp * 4);
  float* ivT = reinterpret_cast<float*>(w8);
  w8 += al256(BH * Tkp * 4);
  float4* mq = reinterpret_cast<float4*>(w8);
  w8 += al256(BH * (Tqp / kBN) * 16);
  float4* mk = reinterpret_cast<float4*>(w8);
  w8 += al256(BH * (Tkp / kBN) * 16);
  float* dq_acc = reinterpret_cast<float*>(w8);
  w8 += al256((size_t)BH * s.Tq * kD * 4);
  int* order = reinterpret_cast<int*>(w8);
  ax.iqT = iqT; ax.ikT = ikT; ax.ivT = ivT; ax.mq = mq; ax.mk = mk; ax.order = order;
  ax.Tqp = (int)Tqp; ax.Tkp = (int)Tkp;
  const long long nblk = BH * ((Tqp > Tkp ? Tqp : Tkp) / kBN);
  if (nblk > 0)
    tc_bwd_aux_kernel<<<dim3((unsigned)nblk, 2), 64, 0, st>>>(
        p.nq, p.nk, p.nv, s.kpm, s.kpm_sb, s.B, s.H, s.Tq, s.Tk, (int)Tqp, (int)Tkp, iqT, ikT,
        ivT, mq, mk);
  // TMA descriptors: q, k, v as given (raw, strided); G as two stacked
  // planes [2][B][Tq][H][D] (batch b + B is the low plane)
  CUtensorMap tq128, tq64, tg128, tg64, tk128, tk64, tv128, tv64;
  const long long gsb = (long long)s.Tq * s.H * D, gst = (long long)s.H * D;
  if (!make_tmap_bthd(&tq128, p.q.p, s.B, s.Tq, s.H, p.q.sb, p.q.st, kBM, D) ||
      !make_tmap_bthd(&tq64, p.q.p, s.B, s.Tq, s.H, p.q.sb, p.q.st, kBN, D) ||
      !make_tmap_bthd(&tg128, p.G, 2LL * s.B, s.Tq, s.H, gsb, gst, kBM, D) ||
      !make_tmap_bthd(&tg64, p.G, 2LL * s.B, s.Tq, s.H, gsb, gst, kBN, D) ||
      !make_tmap_bthd(&tk128, p.k.p, s.B, s.Tk, s.H, p.k.sb, p.k.st, kBM, D) ||
      !make_tmap_bthd(&tk64, p.k.p, s.B, s.Tk, s.H, p.k.sb, p.k.st, kBN, D) ||
      !make_tmap_bthd(&tv128, p.v.p, s.B, s.Tk, s.H, p.v.sb, p.v.st, kBM, D) ||
      !make_tmap_bthd(&tv64, p.v.p, s.B, s.Tk, s.H, p.v.sb, p.v.st, kBN, D))
    return SCREEN_ERR_CUDA;
  const bool deterministic = (stages & SCREEN_BWD_DETERMINISTIC) != 0;
  if (deterministic || D != 64) {
    // dq by its own query-major kernel: every sum in a fixed order.  Stage
    // 2 runs it, stage 4 the key-major kernel; at D = 128 (no fused kernel)
    // stage 4 outside the fixed-order mode runs both
    const bool run_dq = (stages & 2) || (!deterministic && (stages & 4));
    if (s.Tq > 0 && run_dq) {
      dim3 g1((s.Tq + kBM - 1) / kBM, s.B * s.H);
      if (s.drop_thr)
        tc_bwd_dq_kernel<true, D><<<g1, kThreads, DqCfg<D>::SMEM, st>>>(s, p, ax, tq128, tg128,
                                                                        tk64, tv64);
      else
        tc_bwd_dq_kernel<false, D><<<g1, kThreads, DqCfg<D>::SMEM, st>>>(s, p, ax, tq128, tg128,
                                                                         tk64, tv64);
    }
    if (s.Tk > 0 && (stages & 4)) {
      const int nkt = (s.Tk + kBM - 1) / kBM;
      tile_order(s, 1, nkt, order, st);
      if (s.drop_thr)
        tc_bwd_kv_kernel<false, true, D><<<(unsigned)(BH * nkt), kThreads,
                                           KvCfg<D, false>::SMEM, st>>>(s, p, ax, tq64, tg64,
                                                                         tk128, tv128, tq64);
      else
        tc_bwd_kv_kernel<false, false, D><<<(unsigned)(BH * nkt), kThreads,
                                            KvCfg<D, false>::SMEM, st>>>(s, p, ax, tq64, tg64,
                                                                          tk128, tv128, tq64);
    }
    return SCREEN_OK;
  }
  if constexpr (D == 64) {
    // fused: the key-major kernel also forms dq^ (TMA reduce-adds into
    // dq_acc), the finalize pass applies the 1/|q| Jacobian; stage 4 runs
    // both (dq with dk, dv), stage 2 alone runs nothing
    if (stages & 4) {
      const size_t acc_bytes = (size_t)BH * s.Tq * kD * 4;
      if (acc_bytes && cudaMemsetAsync(dq_acc, 0, acc_bytes, st) != cudaSuccess)
        return SCREEN_ERR_CUDA;
      BwdPtrs pf = p;
      pf.dq_acc = dq_acc;
      if (s.Tk > 0) {
        const int nkt = (s.Tk + kBM - 1) / kBM;
        tile_order(s, 1, nkt, order, st);
        CUtensorMap tdq;
        if (!make_tmap_dq(&tdq, dq_acc, s.B, s.Tq, s.H)) return SCREEN_ERR_CUDA;
        if (s.drop_thr)
          tc_bwd_kv_kernel<true, true><<<(unsigned)(BH * nkt), kThreads, KvCfg<64, true>::SMEM,
                                         st>>>(s, pf, ax, tq64, tg64, tk128, tv128, tdq);
        else
          tc_bwd_kv_kernel<true, false><<<(unsigned)(BH * nkt), kThreads, KvCfg<64, true>::SMEM,
                                          st>>>(s, pf, ax, tq64, tg64, tk128, tv128, tdq);
      }
      const long long rows = BH * s.Tq;
      if (rows > 0)
        tc_bwd_dq_finalize_kernel<<<(unsigned)((rows + 15) / 16), 256, 0, st>>>(
            dq_acc, p.q, p.nq, p.dq, s.B, s.Tq, s.H);
    }
  }
  return SCREEN_OK;
}
}  // namespace

int tc_bwd(const AttnShape& s, const BwdPtrs& p, void* aux_ws, int stages, int D,
           cudaStream_t st) {
  if (s.B == 0 || s.H == 0) return SCREEN_OK;
  return D == 128 ? tc_bwd_d<128>(s, p, aux_ws, stages, st) : tc_bwd_d<64>(s, p, aux_ws, stages, st);
}


int tc_bwd_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bwd_status, sizeof(int)) != cudaSuccess) return SCREEN_ERR_CUDA;
  if (clear && v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_bwd_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace screen
