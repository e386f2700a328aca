// Screening attention forward on the 5th-generation tensor cores (tcgen05,
// TMEM accumulators), bf16, head dim 64 or 128 (FwdCfg below).
//
// Math: multiscreen/attention.py:156-196 -- S = q^ k^T, a = relu(1-r(1-S)),
// alpha = a^2 m(rel), o = alpha v^, y = TanhNorm(o) (norm.py:23-25).
//
// A prep pass reads q, k, v once: clamped norms (kept for the backward), the
// unit rows V^ (bf16, padded keys zeroed) and 1/|k| transposed per (b, h)
// plus its per-64-key-tile (min, max).  K itself enters the tensor cores raw
// (exact bf16) with 1/|k| applied in fp32 per column, because r amplifies any
// error of S near the trim threshold; rounding V^ is harmless (alpha is
// rounded to bf16 anyway).
//
// CTA = 128 queries of one (b, h), six warps:
//   warps 0-3  "compute": thread t owns query row t = TMEM lane t.  Reads the
//              S tile from TMEM, applies 1/|k|, the trim, the softmask (rank-2
//              cos identity against per-row and per-column (cos, sin) pairs)
//              with packed f32x2 math, and writes P = alpha (bf16) back to
//              TMEM as the A operand of the PV MMA; TanhNorm epilogue.
//   warp 4     producer: cp.async Q once, then per 64-key tile K, V^, 1/|k|
//              and the tile's (min, max) through a 3-stage ring; the column
//              (cos, sin) come from one sincospif per tile and a rotation.
//   warp 5     MMA issuer (one thread): S_j = Q K_j^T (M=128, N=64, K=64) into
//              a double-buffered TMEM S, then O += P_{j-1} V^_{j-1} (A from
//              TMEM, V^ MN-major from shared memory) into the TMEM O.
// TMEM (D = 64): a ring of three 64-column S buffers with P written over
// them, O [192,256) -> 256 columns, so two CTAs share an SM (D = 128: two S
// buffers and O [128,256)).  Key tiles outside the window are never
// loaded; a tile whose scores provably all fall under the trim threshold
// skips the alpha/PV work.  Every wait is bounded by a global-timer limit; on
// expiry the CTA drains, frees its TMEM and records SCREEN_ERR_TIMEOUT in a
// device status word (screen_device_status).
#include "rowops.cuh"

namespace screen {
namespace {

using namespace sm100;
typedef __nv_bfloat16 bf16;

// kCG compute warpgroups split each key tile's 64 columns (32 / kCG each)
constexpr int kCG = 2;
constexpr int kBM = 128, kBN = 64;
constexpr int kCW = 4 * kCG;                 // compute warps
constexpr int kNC = kBN / kCG;               // columns per compute thread per tile
constexpr int kCT = 32 * kCW;                // compute threads
constexpr int kProdWarp = kCW, kMmaWarp = kCW + 1;
constexpr int kThreads = 32 * (kCW + 2);
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr uint32_t TM_S = 0, TM_COLS = 256;

// Per head dim D (64 or 128).  Operand tiles are stored as D / 64 column
// halves of 64 elements (128-byte rows, SW128), each half a separate TMA box
// and a separate run of K-steps for the MMA.
//   kNS: K / V^ ring stages; kSB: S / P buffers in TMEM (P, bf16, is written
//   over the S columns it came from), then O: kSB * 64 + D <= 256 columns,
//   so two CTAs share an SM at either D.
template <int D>
struct FwdCfg {
  static constexpr int kD = D, kHalves = D / 64;
  static constexpr int kNS = D == 64 ? 5 : 2;
  static constexpr int kSB = D == 64 ? 3 : 2;
  static constexpr uint32_t TILE_Q = kBM * D * 2, TILE_KV = kBN * D * 2;
  static constexpr uint32_t HALF_Q = kBM * 128, HALF_KV = kBN * 128;   // one 64-column half
  // shared-memory layout (offsets from a 1024-byte aligned base)
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + TILE_Q;
  static constexpr uint32_t OFF_V = OFF_K + kNS * TILE_KV;
  static constexpr uint32_t OFF_COL = OFF_V + kNS * TILE_KV;  // per stage ik|cos|sin [64] + meta
  static constexpr uint32_t COL_BYTES = 3 * kBN * 4 + 16;      // meta = (ik min, ik max, -, -)
  static constexpr uint32_t OFF_TAB = OFF_COL + kNS * COL_BYTES;  // (cos, sin)(pi c / w), c < 64
  static constexpr uint32_t OFF_BAR = OFF_TAB + 2 * kBN * 4;
  static constexpr int BAR_Q = 0, BAR_KV_FULL = 1, BAR_KV_EMPTY = BAR_KV_FULL + kNS,
                       BAR_S_FULL = BAR_KV_EMPTY + kNS, BAR_P_FULL = BAR_S_FULL + kSB,
                       BAR_O_FULL = BAR_P_FULL + kSB, BAR_COUNT = BAR_O_FULL + 1;
  static constexpr uint32_t OFF_MISC = OFF_BAR + 8 * 24;
  static constexpr uint32_t OFF_RED = OFF_MISC + 64;           // [kCG][kBM] epilogue sums
  static constexpr uint32_t SMEM_USED = OFF_RED + kCG * kBM * 4;
  // at least 80 KB per CTA: at most two CTAs (2 x 256 TMEM columns) per SM
  static constexpr uint32_t kSmemBytes =
      (SMEM_USED + 1024 > 80 * 1024) ? SMEM_USED + 1024 : 80 * 1024;
  static constexpr uint32_t TM_O = kSB * kBN;
  static_assert(BAR_COUNT <= 24, "barrier space");
  static_assert(TM_O + D <= TM_COLS, "TMEM budget");
  static_assert(2 * kSmemBytes <= 228 * 1024, "two CTAs per SM");
};

__device__ int g_device_status = 0;


// kDrop: attention dropout on alpha (counter-based bits, AttnShape::drop_thr)
template <bool kDrop, int D>
__global__ void __launch_bounds__(kThreads, 2)
    tc_fwd_kernel(AttnShape s, FwdPtrs p, const float* __restrict__ ikT,
                  const float4* __restrict__ ikmeta, int Tkp, const int* __restrict__ order,
                  const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV) {
  using C = FwdCfg<D>;
  constexpr int kD = D, kNS = C::kNS, kSB = C::kSB, kHalves = C::kHalves;
  constexpr uint32_t OFF_Q = C::OFF_Q, OFF_K = C::OFF_K, OFF_V = C::OFF_V, OFF_COL = C::OFF_COL,
                     COL_BYTES = C::COL_BYTES, OFF_TAB = C::OFF_TAB, OFF_BAR = C::OFF_BAR,
                     OFF_MISC = C::OFF_MISC, OFF_RED = C::OFF_RED, TM_O = C::TM_O;
  constexpr int BAR_Q = C::BAR_Q, BAR_KV_FULL = C::BAR_KV_FULL, BAR_KV_EMPTY = C::BAR_KV_EMPTY,
                BAR_S_FULL = C::BAR_S_FULL, BAR_P_FULL = C::BAR_P_FULL, BAR_O_FULL = C::BAR_O_FULL;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_addr);
  const uint32_t sQ = base + OFF_Q, sK = base + OFF_K, sV = base + OFF_V;
  float* colp = reinterpret_cast<float*>(gbase + OFF_COL);
  float* tab = reinterpret_cast<float*>(gbase + OFF_TAB);
  const uint32_t bars = base + OFF_BAR;
  uint32_t* misc = reinterpret_cast<uint32_t*>(gbase + OFF_MISC);
  // misc[0] tmem base, misc[4] abort, misc[5] O valid
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA -> (b, h, query tile) through the longest-first order
  const int nqt = (s.Tq + kBM - 1) / kBM;
  const long long item = order[blockIdx.x];
  const int bh = (int)(item / nqt), b = bh / s.H, h = bh % s.H;
  const long long i0 = (item % nqt) * kBM;
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
    mbar_init(bar(BAR_Q), 1);
    for (int i = 0; i < kNS; ++i) {
      // one arrival with the TMA byte count, one after the column factors
      mbar_init(bar(BAR_KV_FULL + i), 2);
      mbar_init(bar(BAR_KV_EMPTY + i), 1);
    }
    for (int i = 0; i < kSB; ++i) {
      mbar_init(bar(BAR_S_FULL + i), 1);
      mbar_init(bar(BAR_P_FULL + i), kCT);
    }
    mbar_init(bar(BAR_O_FULL), 2);
    misc[4] = 0;
    misc[5] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(base + OFF_MISC, TM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp == kProdWarp) {
    // ------------------------------------------------------------ producer
    // lane 0 issues the TMA copies (Q once; per 64-key tile K, V^ and the
    // 1/|k| run with its (min, max)); the warp computes the column (cos, sin)
    // of the tile from one sincospif and a rotation of the per-CTA table
    if (lane == 0) {
      mbar_arrive_expect_tx(bar(BAR_Q), kBM * kD * 2);
#pragma unroll
      for (int hf = 0; hf < kHalves; ++hf)
        tma_load_4d(sQ + hf * C::HALF_Q, &tmQ, 64 * hf, h, (int)i0, b, bar(BAR_Q));
    }
    // (cos, sin)(pi c / w) for the 64 column offsets of a tile
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
    const float* ikh = ikT + (long long)bh * Tkp;          // 1/|k| of (b, h), padded to 64
    const float4* mh = ikmeta + (long long)bh * (Tkp / kBN);
    for (int j = 0; j < n; ++j) {
      const int st = j % kNS;
      if (j >= kNS) {
        // lane 0 waits, the whole warp follows its verdict (no divergent exit)
        int okw = 1;
        if (lane == 0) {
          okw = mbar_wait(bar(BAR_KV_EMPTY + st), ((j / kNS) - 1) & 1, abort_flag, kWaitLimitNs);
        }
        if (!__shfl_sync(0xffffffffu, okw, 0)) break;
      }
      const int kt = kt0 + j;
      const long long j0 = (long long)kt * kBN;
      const uint32_t kb = sK + st * kBN * kD * 2, vb = sV + st * kBN * kD * 2;
      const uint32_t colb = base + OFF_COL + st * COL_BYTES;
      float* col = colp + st * (COL_BYTES / 4);
      if (lane == 0) {
        const uint32_t fb = bar(BAR_KV_FULL + st);
        mbar_arrive_expect_tx(fb, 2 * kBN * kD * 2 + kBN * 4 + 16);
#pragma unroll
        for (int hf = 0; hf < kHalves; ++hf) {
          tma_load_4d(kb + hf * C::HALF_KV, &tmK, 64 * hf, h, (int)j0, b, fb);
          tma_load_4d(vb + hf * C::HALF_KV, &tmV, 64 * hf, h, (int)j0, b, fb);
        }
        bulk_g2s(colb, ikh + j0, kBN * 4, fb);
        bulk_g2s(colb + 3 * kBN * 4, mh + kt, 16, fb);
      }
      // column angle pi (j0 + c - p0) / w = base + pi c / w, by rotation
      float sb = 0.f, cb = 0.f;
      if (lane == 0) sincospif((float)(j0 - p0) / w, &sb, &cb);
      sb = __shfl_sync(0xffffffffu, sb, 0);
      cb = __shfl_sync(0xffffffffu, cb, 0);
      col[kBN + lane] = cb * cphi0 - sb * sphi0;
      col[2 * kBN + lane] = sb * cphi0 + cb * sphi0;
      col[kBN + lane + 32] = cb * cphi1 - sb * sphi1;
      col[2 * kBN + lane + 32] = sb * cphi1 + cb * sphi1;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_KV_FULL + st));
    }
    if (lane == 0 && *abort_flag) {
      // let the copies already issued land before the CTA's smem goes away
      const uint64_t t0 = globaltimer();
      for (int j = n > kNS ? n - kNS : 0; j < n; ++j)
        while (!mbar_try_wait(bar(BAR_KV_FULL + j % kNS), (j / kNS) & 1) &&
               globaltimer() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(kBM, kBN, 0, 0);
      constexpr uint32_t idPV = idesc_bf16(kBM, kD, 0, 1);
      bool o_started = false, ok = mbar_wait(bar(BAR_Q), 0, abort_flag, kWaitLimitNs);
      // S_j = Q K_j^T into ring buffer j % kSB, kept kSB tiles ahead of the
      // compute warps; buffer reuse is ordered by the tensor core's in-order
      // execution (S_{j+kSB} is issued after PV_j, which read P_j there)
      auto issue_s = [&](int jj) -> bool {
        const int st = jj % kNS, bb = jj % kSB;
        {
          const bool okk = mbar_wait(bar(BAR_KV_FULL + st), (jj / kNS) & 1, abort_flag, kWaitLimitNs);
          if (!okk) return false;
        }
        tc_fence_after();
        const uint32_t kb = sK + st * kBN * kD * 2;
        // K-steps of 16: four per 64-column half of Q and K
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + TM_S + kBN * bb,
                 desc_sw128(sQ + (kk >> 2) * C::HALF_Q + (kk & 3) * 32, 16, 1024),
                 desc_sw128(kb + (kk >> 2) * C::HALF_KV + (kk & 3) * 32, 16, 1024), idS,
                 kk > 0 ? 1u : 0u);
        mma_commit(bar(BAR_S_FULL + bb));
        return true;
      };
      for (int j = 0; j < n && j < kSB && ok; ++j) ok = issue_s(j);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j % kNS, bb = j % kSB;
        {
          ok = mbar_wait(bar(BAR_P_FULL + bb), (j / kSB) & 1, abort_flag, kWaitLimitNs);
        }
        if (!ok) break;
        tc_fence_after();
        {
          // P_j sits in the first 16 columns of each compute group's half of
          // the buffer: keys [32 g, 32 g + 32) at columns [32 g, 32 g + 16)
          const uint32_t vb = sV + st * kBN * kD * 2;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t pcol = kCG == 2 ? (kk >> 1) * 32 + (kk & 1) * 8 : 8 * kk;
            // V^ MN-major: D / 64 chunks of 64 output columns, C::HALF_KV apart
            mma_ts(tmem + TM_O, tmem + TM_S + kBN * bb + pcol,
                   desc_sw128(vb + kk * 16 * 128, C::HALF_KV, 1024), idPV,
                   (o_started || kk > 0) ? 1u : 0u);
          }
          o_started = true;
        }
        mma_commit(bar(BAR_KV_EMPTY + st));
        if (j + kSB < n) ok = issue_s(j + kSB);
      }
      misc[5] = o_started ? 1u : 0u;
      mma_commit(bar(BAR_O_FULL));
      mbar_arrive(bar(BAR_O_FULL));
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ compute
    const int t = tid & (kBM - 1);  // query row in tile = TMEM lane
    const int g = tid / kBM;        // column group: columns [g * kNC, (g + 1) * kNC)
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const long long i = i0 + t;
    const float rq = (i < s.Tq) ? r / p.nq[((long long)b * s.Tq + i) * s.H + h] : 0.f;
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
    const float2 half2 = make_float2(0.5f, 0.5f);
    // attention dropout: this query row's counter key
    const uint32_t drow = kDrop ? drop_row(drop_bh_key(s, (uint32_t)bh), (uint32_t)i) : 0u;
    // alpha of columns (c, c+1) from the pair's S, 1/|k|, cos, sin
    auto pair_alpha = [&](float s0, float s1, float ik0, float ik1, float c0, float c1, float n0,
                          float n1, bool k0, bool k1) -> uint32_t {
      const float2 x = __fmul2_rn(make_float2(s0, s1), make_float2(ik0, ik1));
      // relu(t) = saturate(t): t = 1 - r (1 - S) <= 1, so the clamp is free
      const float a0 = __saturatef(fmaf(rq, x.x, omr)), a1 = __saturatef(fmaf(rq, x.y, omr));
      const float2 a2 = make_float2(k0 ? a0 : 0.f, k1 ? a1 : 0.f);
      const float2 m2 =
          __ffma2_rn(cr2, make_float2(c0, c1), __ffma2_rn(sr2, make_float2(n0, n1), half2));
      const float2 al = __fmul2_rn(__fmul2_rn(a2, m2), a2);
      return pack_bf16(al.x, al.y);
    };
    bool ok = true;
    unsigned long long live_tiles = 0;
    // ring positions kept incrementally (no per-tile division); positions
    // in 32-bit (key / query indices and offsets are < 2^31)
    int st = 0, st_ph = 0, bb = 0, bb_ph = 0;
    const int p0i = (int)p0, posi = (int)pos;
    int j0i = kt0 * kBN;
    // a tile is inside the window for every row iff its keys all lie in
    // [p0 + kBM - 1 - dmax, p0] (causal) / [.. , p0 + dmax] (non-causal)
    const int in_lo = p0i + kBM - 1 - dmax;
    for (int j = 0; j < n; ++j, j0i += kBN) {
      {
        ok = mbar_wait(bar(BAR_KV_FULL + st), st_ph, abort_flag, kWaitLimitNs) &&
             mbar_wait(bar(BAR_S_FULL + bb), bb_ph, abort_flag, kWaitLimitNs);
      }
      // warp-uniform verdict (the TMEM accesses below are warp-collective);
      // a warp that gives up leaves the loop alone -- every other wait on its
      // arrivals is bounded and sees the abort flag
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      static_assert(kNC == 32 || kNC == 64, "column split");
      uint32_t sv[kNC];
#pragma unroll
      for (int h32 = 0; h32 < kNC / 32; ++h32)
        tmem_ld32(tmem + TM_S + kBN * bb + kNC * g + 32 * h32 + lane_off,
                  *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * h32]));
      tmem_wait_ld();

      const float* colt = colp + st * (COL_BYTES / 4);   // whole-tile columns
      const float* col = colt + kNC * g;                  // this group's columns
      // trim pre-test.  For r >= 1 the threshold (r-1)/r on S is >= 0, so
      // only positive scores can be live; positive floats order like their
      // int bit patterns and negative ones are negative ints, so an integer
      // max over the raw bits finds the largest score when it is positive.
      int imax = (int)sv[0];
#pragma unroll
      for (int c = 1; c + 1 < kNC; c += 2) imax = __vimax3_s32(imax, (int)sv[c], (int)sv[c + 1]);
      imax = max(imax, (int)sv[kNC - 1]);
      const float smax = __int_as_float(imax);
      const float ikmax = colt[3 * kBN + 1];
      const bool mine = r < 1.0f || (imax > 0 && fmaf(rq, smax * ikmax, omr) > 0.f);
      // liveness per warp block (32 rows x kNC columns): a dead block stores
      // P = 0, so the warps never wait on one another within a tile
      const bool live = __any_sync(0xffffffffu, mine);
      uint32_t pk[kNC / 2];
      if (live) {
        const bool inside = j0i >= in_lo && j0i + kBN - 1 <= (causal ? p0i : p0i + dmax);
        const float4* ik4 = reinterpret_cast<const float4*>(col);
        const float4* cc4 = reinterpret_cast<const float4*>(col + kBN);
        const float4* sc4 = reinterpret_cast<const float4*>(col + 2 * kBN);
        // dropout: key j of column c is kept iff its counter bits clear the threshold
        const uint32_t jgk = (uint32_t)(j0i + kNC * g);
        auto kp = [&](int c) -> bool {
          return !kDrop || drop_keep(drow, jgk + (uint32_t)c, s.drop_thr);
        };
        if (inside) {
#pragma unroll
          for (int q4 = 0; q4 < kNC / 4; ++q4) {
            const float4 ikv = ik4[q4], ccv = cc4[q4], scv = sc4[q4];
            const int c = 4 * q4;
            pk[2 * q4] = pair_alpha(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1]), ikv.x,
                                    ikv.y, ccv.x, ccv.y, scv.x, scv.y, kp(c), kp(c + 1));
            pk[2 * q4 + 1] = pair_alpha(__uint_as_float(sv[c + 2]), __uint_as_float(sv[c + 3]),
                                        ikv.z, ikv.w, ccv.z, ccv.w, scv.z, scv.w, kp(c + 2),
                                        kp(c + 3));
          }
        } else {
          // window edge: this row's valid columns are the interval [clo, chi]
          const int jg = j0i + kNC * g;   // first key of this group's columns
          const int clo = posi - dmax - jg, chi = causal ? posi - jg : posi + dmax - jg;
          const int iclo = clo < 0 ? 0 : (clo > kNC ? kNC : clo);
          const int ichi = chi < -1 ? -1 : (chi > kNC - 1 ? kNC - 1 : chi);
#pragma unroll
          for (int q4 = 0; q4 < kNC / 4; ++q4) {
            const float4 ikv = ik4[q4], ccv = cc4[q4], scv = sc4[q4];
            const int c = 4 * q4;
            pk[2 * q4] = pair_alpha(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1]), ikv.x,
                                    ikv.y, ccv.x, ccv.y, scv.x, scv.y,
                                    c >= iclo && c <= ichi && kp(c),
                                    c + 1 >= iclo && c + 1 <= ichi && kp(c + 1));
            pk[2 * q4 + 1] = pair_alpha(__uint_as_float(sv[c + 2]), __uint_as_float(sv[c + 3]),
                                        ikv.z, ikv.w, ccv.z, ccv.w, scv.z, scv.w,
                                        c + 2 >= iclo && c + 2 <= ichi && kp(c + 2),
                                        c + 3 >= iclo && c + 3 <= ichi && kp(c + 3));
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < kNC / 2; ++c) pk[c] = 0u;
      }
      // P over this group's own S columns (already in registers)
      if constexpr (kNC == 64) {
        tmem_st32(tmem + TM_S + kBN * bb + lane_off, *reinterpret_cast<uint32_t(*)[32]>(pk));
      } else {
        tmem_st16(tmem + TM_S + kBN * bb + kNC * g + lane_off, pk);
      }
      tmem_wait_st();
      if (lane == 0) live_tiles += live ? 1 : 0;
      tc_fence_before();
      mbar_arrive(bar(BAR_P_FULL + bb));
      if (++st == kNS) { st = 0; st_ph ^= 1; }
      if (++bb == kSB) { bb = 0; bb_ph ^= 1; }
    }
    if (p.tile_stats && lane == 0) {
      // in 16x64 score blocks (the unit of the warp-level kernels): a tile is
      // 8 of them, a warp block of 32 rows x kNC columns kNC / 32
      if (tid == 0)
        atomicAdd((unsigned long long*)&p.tile_stats[0], 8ull * (unsigned long long)n);
      atomicAdd((unsigned long long*)&p.tile_stats[1], (unsigned long long)(kNC / 32) * live_tiles);
    }
    // epilogue: O -> TanhNorm -> y
    {
      ok = ok && mbar_wait(bar(BAR_O_FULL), 0, abort_flag, kWaitLimitNs);
    }
    // tcgen05.ld below is warp-collective: every lane takes the same branch
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    // each column group loads and stores its kD / kCG output columns; the
    // row's |o|^2 is summed over the groups through shared memory
    constexpr int kOC = kD / kCG;
    float o[kOC];
    if (ok && misc[5]) {
      uint32_t ov[kOC];
#pragma unroll
      for (int h32 = 0; h32 < kOC / 32; ++h32)
        tmem_ld32(tmem + TM_O + kOC * g + 32 * h32 + lane_off,
                  *reinterpret_cast<uint32_t(*)[32]>(&ov[32 * h32]));
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kOC; ++c) o[c] = __uint_as_float(ov[c]) * (kDrop ? s.drop_scale : 1.0f);
    } else {
#pragma unroll
      for (int c = 0; c < kOC; ++c) o[c] = 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kOC; ++c) ss = fmaf(o[c], o[c], ss);
    float* red = reinterpret_cast<float*>(gbase + OFF_RED);
    red[g * kBM + t] = ss;
    asm volatile("bar.sync 2, %0;" ::"r"(kCT) : "memory");
    if (ok) {
      float tot = 0.f;
#pragma unroll
      for (int gg = 0; gg < kCG; ++gg) tot += red[gg * kBM + t];
      const float nraw = sqrtf(tot);
      const float gsc = tanhnorm_scale(nraw, s.eps);
      if (i < s.Tq) {
        const long long row = ((long long)b * s.Tq + i) * s.H + h;
        uint4* yr = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(p.y) + row * kD + kOC * g);
#pragma unroll
        for (int c8 = 0; c8 < kOC / 8; ++c8) {
          uint4 v;
          v.x = pack_bf16(o[8 * c8 + 0] * gsc, o[8 * c8 + 1] * gsc);
          v.y = pack_bf16(o[8 * c8 + 2] * gsc, o[8 * c8 + 3] * gsc);
          v.z = pack_bf16(o[8 * c8 + 4] * gsc, o[8 * c8 + 5] * gsc);
          v.w = pack_bf16(o[8 * c8 + 6] * gsc, o[8 * c8 + 7] * gsc);
          yr[c8] = v;
        }
        if (g == 0) p.no[row] = nraw;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TM_COLS);
  if (tid == 0 && *abort_flag) atomicExch(&g_device_status, (int)SCREEN_ERR_TIMEOUT);
}

// One pass over q, k, v (bf16, D / 8 lanes x 16 B per row): the clamped
// row norms (written unless the caller gave them), the unit rows
// V^ = v / |v| (zero for padded keys) that the forward multiplies by alpha,
// and 1/|k| transposed to [B][H][Tk padded to 64] so a key tile's factors are
// one contiguous 256-byte run.
template <int kD>
__global__ void tc_prep_kernel(Rows q, Rows k, Rows v, int B, int Tq, int Tk, int H, float eps,
                               int norms_given, const uint8_t* kpm, long long kpm_sb,
                               float* __restrict__ nq, float* __restrict__ nk,
                               float* __restrict__ nv, bf16* __restrict__ vhat,
                               float* __restrict__ ikT, int Tkp) {
  constexpr int LPR = kD / 8;          // lanes per row (16 bytes each)
  constexpr int RPS = 256 / LPR;       // rows per block step
  const int sub = threadIdx.x % LPR;
  const long long rows_q = norms_given ? 0 : (long long)B * Tq * H;
  const long long rows_k = (long long)B * Tk * H;
  const long long total = rows_q + rows_k;
  // every lane of a warp runs the same number of iterations (RPS rows per
  // block step), so the LPR-lane shuffles below always see full groups
  for (long long base_row = (long long)blockIdx.x * RPS; base_row < total;
       base_row += (long long)gridDim.x * RPS) {
    const long long row = base_row + (threadIdx.x / LPR);
    const bool valid = row < total;
    const bool isq = row < rows_q;
    const long long rr = !valid ? 0 : (isq ? row : row - rows_q);
    const int T = isq ? Tq : Tk;
    long long hh, t, bb;
    if (total < (1ll << 31)) {
      // 32-bit division: a 64-bit one per row costs more than the row's bytes
      const unsigned r32 = (unsigned)rr, bt = r32 / (unsigned)H;
      hh = r32 - bt * (unsigned)H;
      t = bt % (unsigned)T;
      bb = bt / (unsigned)T;
    } else {
      hh = rr % H;
      t = (rr / H) % T;
      bb = rr / ((long long)H * T);
    }
    // a = the q row (q part) or the k row; c = the v row (k part) or zeros
    uint4 ua = make_uint4(0, 0, 0, 0), uc = make_uint4(0, 0, 0, 0);
    if (valid && isq) {
      ua = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(q.p) + bb * q.sb +
                                           t * q.st + hh * kD + sub * 8);
    } else if (valid) {
      ua = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(k.p) + bb * k.sb +
                                           t * k.st + hh * kD + sub * 8);
      uc = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(v.p) + bb * v.sb +
                                           t * v.st + hh * kD + sub * 8);
    }
    float sa = 0.f, sc = 0.f;
    const uint32_t a4[4] = {ua.x, ua.y, ua.z, ua.w};
    const uint32_t c4[4] = {uc.x, uc.y, uc.z, uc.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = unpack_bf16(a4[e]), fc = unpack_bf16(c4[e]);
      sa = fmaf(fa.x, fa.x, fmaf(fa.y, fa.y, sa));
      sc = fmaf(fc.x, fc.x, fmaf(fc.y, fc.y, sc));
    }
#pragma unroll
    for (int o = 1; o < LPR; o <<= 1) {
      sa += __shfl_xor_sync(0xffffffffu, sa, o);
      sc += __shfl_xor_sync(0xffffffffu, sc, o);
    }
    if (!valid) continue;
    if (isq) {
      if (sub == 0) nq[rr] = fmaxf(sqrtf(sa), eps);
      continue;
    }
    const float nkr = norms_given ? nk[rr] : fmaxf(sqrtf(sa), eps);
    const float nvr = norms_given ? nv[rr] : fmaxf(sqrtf(sc), eps);
    const bool masked = kpm && kpm[bb * kpm_sb + t];
    const float inv = masked ? 0.f : 1.0f / nvr;
    uint4 o;
    float2 f;
    f = unpack_bf16(uc.x); o.x = pack_bf16(f.x * inv, f.y * inv);
    f = unpack_bf16(uc.y); o.y = pack_bf16(f.x * inv, f.y * inv);
    f = unpack_bf16(uc.z); o.z = pack_bf16(f.x * inv, f.y * inv);
    f = unpack_bf16(uc.w); o.w = pack_bf16(f.x * inv, f.y * inv);
    *reinterpret_cast<uint4*>(vhat + rr * kD + sub * 8) = o;
    if (sub == 0) {
      if (!norms_given) {
        nk[rr] = nkr;
        nv[rr] = nvr;
      }
      ikT[(bb * H + hh) * Tkp + t] = 1.0f / nkr;
    }
  }
}

// per-64-key-tile (min, max) of 1/|k| (zero past Tk, and the padding zeroed):
// one warp per tile, two keys per lane
__global__ void tc_ik_meta_kernel(float* __restrict__ ikT, float4* __restrict__ meta, int BH,
                                  int Tk, int Tkp) {
  const int ntiles = Tkp / kBN;
  const long long idx = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (idx >= (long long)BH * ntiles) return;
  const long long bhh = idx / ntiles;
  const int tile = (int)(idx % ntiles);
  float* x = ikT + bhh * Tkp + (long long)tile * kBN;
  float mn = 3.0e38f, mx = 0.f;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int c = lane + 32 * hh;
    const long long t = (long long)tile * kBN + c;
    float vv = 0.f;
    if (t < Tk) vv = x[c]; else x[c] = 0.f;
    mn = fminf(mn, vv);
    mx = fmaxf(mx, vv);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) meta[idx] = make_float4(mn, mx, 0.f, 0.f);
}

long long tk_pad(int Tk) { return ((long long)Tk + kBN - 1) / kBN * kBN; }
size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

bool tc_supported(int dtype, int D) { return dtype == SCREEN_BF16 && (D == 64 || D == 128); }

size_t tc_fwd_workspace(const AttnShape& s, int D) {
  const long long BH = (long long)s.B * s.H, Tkp = tk_pad(s.Tk);
  return al256((size_t)s.B * s.Tk * s.H * D * 2) + al256((size_t)BH * Tkp * 4) +
         al256((size_t)BH * (Tkp / kBN) * 16) + al256((size_t)BH * ((s.Tq + kBM - 1) / kBM) * 4);
}

namespace {
template <int D>
int tc_fwd_d(const AttnShape& s, const FwdPtrs& p, void* workspace, bool norms_given,
             cudaStream_t st) {
  using C = FwdCfg<D>;
  {
    cudaError_t e = ensure_smem_optin((const void*)tc_fwd_kernel<false, D>, (int)C::kSmemBytes);
    if (e == cudaSuccess)
      e = ensure_smem_optin((const void*)tc_fwd_kernel<true, D>, (int)C::kSmemBytes);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  const long long BH = (long long)s.B * s.H, Tkp = tk_pad(s.Tk);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  bf16* vhat = reinterpret_cast<bf16*>(ws);
  float* ikT = reinterpret_cast<float*>(ws + al256((size_t)s.B * s.Tk * s.H * D * 2));
  float4* meta = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(ikT) +
                                           al256((size_t)BH * Tkp * 4));
  int* order = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(meta) +
                                      al256((size_t)BH * (Tkp / kBN) * 16));
  const long long rows = (long long)s.B * ((norms_given ? 0 : s.Tq) + s.Tk) * s.H;
  if (rows > 0) {
    constexpr int RPS = 256 / (D / 8);
    long long blocks = (rows + RPS - 1) / RPS;
    if (blocks > 148 * 16) blocks = 148 * 16;
    tc_prep_kernel<D><<<(unsigned)blocks, 256, 0, st>>>(
        p.q, p.k, p.v, s.B, s.Tq, s.Tk, s.H, s.eps, norms_given ? 1 : 0, s.kpm, s.kpm_sb,
        const_cast<float*>(p.nq), const_cast<float*>(p.nk), const_cast<float*>(p.nv), vhat, ikT,
        (int)Tkp);
  }
  const long long mt = BH * (Tkp / kBN);
  if (mt > 0)
    tc_ik_meta_kernel<<<(unsigned)((mt * 32 + 255) / 256), 256, 0, st>>>(ikT, meta, (int)BH, s.Tk,
                                                                   (int)Tkp);
  if (s.Tq == 0) return SCREEN_OK;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_bthd(&tq, p.q.p, s.B, s.Tq, s.H, p.q.sb, p.q.st, kBM, D) ||
      !make_tmap_bthd(&tk, p.k.p, s.B, s.Tk, s.H, p.k.sb, p.k.st, kBN, D) ||
      !make_tmap_bthd(&tv, vhat, s.B, s.Tk, s.H, (long long)s.Tk * s.H * D, (long long)s.H * D,
                      kBN, D))
    return SCREEN_ERR_CUDA;
  const int nqt = (s.Tq + kBM - 1) / kBM;
  tile_order(s, 0, nqt, order, st);
  if (s.drop_thr)
    tc_fwd_kernel<true, D><<<(unsigned)(BH * nqt), kThreads, C::kSmemBytes, st>>>(
        s, p, ikT, meta, (int)Tkp, order, tq, tk, tv);
  else
    tc_fwd_kernel<false, D><<<(unsigned)(BH * nqt), kThreads, C::kSmemBytes, st>>>(
        s, p, ikT, meta, (int)Tkp, order, tq, tk, tv);
  return SCREEN_OK;
}
}  // namespace

int tc_fwd(const AttnShape& s, const FwdPtrs& p, void* workspace, bool norms_given, int D,
           cudaStream_t st) {
  if (s.B == 0 || s.H == 0) return SCREEN_OK;
  return D == 128 ? tc_fwd_d<128>(s, p, workspace, norms_given, st)
                  : tc_fwd_d<64>(s, p, workspace, norms_given, st);
}


int tc_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return SCREEN_ERR_CUDA;
  if (clear && v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_device_status, &z, sizeof(int));
  }
  return v;
}

}  // namespace screen
