// K1: fused flash-style attention prefill for sm_100a.
//
// Replaces the score/softmax/context math of the reference's attention
// forward: nn/forward.py:525-551 (plain MHA), nn/flash_attention.py:42-80
// (streaming softmax, the algorithmic spec followed here), nn/forward.py:578-586
// (cross-attention) and the key-padding rule of graph/sequence.py:159-183.
//
// One CTA (three warpgroups, 384 threads) owns two 128-row query tiles (A, B)
// of one (batch, head) and streams 128-key tiles of K and V through shared
// memory:
//   warp 8      TMA producer: Q tiles once, then K/V tiles into a ring of stages
//   warp 9      MMA issuer: S = Q K^T (smem x smem) and O += P V (P from TMEM)
//   warps 10-11 idle members of the producer warpgroup
//   warps 0-3   softmax for tile A, warps 4-7 softmax for tile B: each thread
//               owns one query row == one TMEM lane, so row max / row sum need
//               no shuffles; P is written back into TMEM over the S columns.
// Tensor memory per CTA: S_A | S_B | O_A | O_B (128 + 128 + D + D columns).
// The online softmax rescales O lazily: only when a row max grows by more
// than 2^8 does the thread pull O out of TMEM, scale and store it back.
//
// Masking semantics (see PrefillParams): causal / sliding window / per-batch
// key-valid length / ALiBi, either with -inf exclusion (nn/ path) or with the
// graph path's additive -1e9 rule, which is applied exactly by tracking the
// number of -1e9 terms ("tier") per score when a row has no unmasked key.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

template <int D>
struct PrefillCfg {
  static constexpr int kThreads = 384;
  // Register split (setmaxnreg): the launch holds kLaunchRegs * 384 registers;
  // the producer warpgroup gives some up so the two softmax warpgroups can
  // keep a full 128-score row in registers. 2*128*216 + 128*56 <= 168*384.
  static constexpr int kLaunchRegs = 168;
  static constexpr int kSoftmaxRegs = 216;
  static constexpr int kProducerRegs = 56;
  static_assert(2 * 128 * kSoftmaxRegs + 128 * kProducerRegs <= kLaunchRegs * kThreads,
                "register split exceeds the launch allocation");
  static constexpr int kBlockM = 128;
  static constexpr int kBlockN = 128;
  static constexpr int kStages = (D == 128) ? 2 : 4;
  static constexpr int kAtoms = D / 64;  // 128-byte swizzle atoms along the head dim
  static constexpr int kTileBytes = kBlockN * D * 2;
  static constexpr int kAtomBytes = 128 * 128;  // 128 rows x 128 bytes
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + 2 * kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kStages * kTileBytes;
  static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 2 + 1;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // +align slack
  static constexpr uint32_t kTmemCols = 512;
  // Tensor-memory columns: S/P of tile x at 128*x, O of tile x at 256 + D*x.
  __host__ __device__ static constexpr uint32_t col_s(int x) { return 128u * x; }
  __host__ __device__ static constexpr uint32_t col_o(int x) { return 256u + D * x; }
};

struct RowBounds {
  long long jlo;  // smallest key index allowed by causal/window (may be < 0)
  long long jhi;  // largest key index allowed by causal/window
};

__device__ __forceinline__ RowBounds row_bounds(const PrefillParams& p, long long row) {
  const long long d = p.q_pos0 + row - p.k_pos0;  // key index at the same position
  RowBounds rb;
  const long long kBig = (1ll << 40);
  rb.jlo = (p.window >= 0) ? d - p.window : -kBig;
  rb.jhi = p.causal ? d : ((p.window >= 0) ? d + p.window : kBig);
  return rb;
}

// Key-tile range [lo, hi) a query tile must visit, and whether every row of it
// has at least one unmasked key (then -1e9 and -inf masking agree exactly).
__device__ __forceinline__ void tile_range(const PrefillParams& p, int r0, int lkey, int n_ktiles,
                                           int& lo, int& hi, bool& safe) {
  if (r0 >= p.Sq) {
    lo = hi = 0;
    safe = true;
    return;
  }
  const int r1 = min(r0 + 128, p.Sq) - 1;
  const RowBounds first = row_bounds(p, r0), last = row_bounds(p, r1);
  safe = (lkey > 0) && (first.jhi >= 0) && (last.jlo <= lkey - 1);
  if (p.additive && !safe) {
    lo = 0;
    hi = n_ktiles;
    return;
  }
  const long long klo = max(first.jlo, 0ll);
  const long long khi = min(last.jhi, (long long)lkey - 1);
  if (khi < klo || lkey <= 0) {
    lo = hi = 0;
    return;
  }
  lo = (int)(klo / 128);
  hi = (int)(khi / 128) + 1;
}

template <int D>
__global__ void __launch_bounds__(384, 1)
    attn_prefill_sm100(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using Cfg = PrefillCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_k_full = bars + 1;
  uint64_t* bar_k_empty = bar_k_full + Cfg::kStages;
  uint64_t* bar_v_full = bar_k_empty + Cfg::kStages;
  uint64_t* bar_v_empty = bar_v_full + Cfg::kStages;
  uint64_t* bar_s_full = bar_v_empty + Cfg::kStages;  // [2]
  uint64_t* bar_p_ready = bar_s_full + 2;             // [2]
  uint64_t* bar_o_done = bar_p_ready + 2;             // [2]
  uint64_t* bar_drain = bar_o_done + 2;               // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int bh = blockIdx.x;
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int hkv = h / (p.H / p.Hkv);
  const int pair = (int)gridDim.y - 1 - (int)blockIdx.y;  // heaviest causal pairs first
  const int r0_tile[2] = {pair * 256, pair * 256 + 128};

  const int n_ktiles = (p.Skv + 127) / 128;
  int lkey = p.Skv;
  if (p.kv_len != nullptr) lkey = max(0, min(p.kv_len[b], p.Skv));
  int lo_x[2], hi_x[2];
  bool safe_x[2];
  tile_range(p, r0_tile[0], lkey, n_ktiles, lo_x[0], hi_x[0], safe_x[0]);
  tile_range(p, r0_tile[1], lkey, n_ktiles, lo_x[1], hi_x[1], safe_x[1]);
  int lo = n_ktiles, hi = 0;
  for (int x = 0; x < 2; ++x) {
    if (lo_x[x] < hi_x[x]) {
      lo = min(lo, lo_x[x]);
      hi = max(hi, hi_x[x]);
    }
  }
  const bool any_work = lo < hi;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kNumBars; ++i) {
      uint32_t count = 1;
      if (bars + i == bar_p_ready || bars + i == bar_p_ready + 1) count = 4;
      mbar_init(bars + i, count);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc<Cfg::kTmemCols>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::kProducerRegs));
   if (warp == 8) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0 && any_work) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar_q, 2 * Cfg::kTileBytes);
      for (int x = 0; x < 2; ++x)
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_4d(smem + Cfg::kOffQ + x * Cfg::kTileBytes + a * Cfg::kAtomBytes, &tm_q, bar_q,
                      a * 64, r0_tile[x], h, b);
      int issued = 0, issued_v = 0;
      bool ok = true;
      for (int j = lo; j < hi && ok; ++j, ++issued) {
        const int st = issued % Cfg::kStages;
        const uint32_t use = issued / Cfg::kStages;
        if (use > 0) ok = mbar_wait(bar_k_empty + st, (use - 1) & 1, abort_flag, 10);
        if (!ok) break;
        mbar_arrive_expect_tx(bar_k_full + st, Cfg::kTileBytes);
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_4d(smem + Cfg::kOffK + st * Cfg::kTileBytes + a * Cfg::kAtomBytes, &tm_k,
                      bar_k_full + st, a * 64, j * 128, hkv, b);
        if (use > 0) ok = mbar_wait(bar_v_empty + st, (use - 1) & 1, abort_flag, 11);
        if (!ok) {
          ++issued;  // the K load of this iteration is in flight
          break;
        }
        mbar_arrive_expect_tx(bar_v_full + st, Cfg::kTileBytes);
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_load_4d(smem + Cfg::kOffV + st * Cfg::kTileBytes + a * Cfg::kAtomBytes, &tm_v,
                      bar_v_full + st, a * 64, j * 128, hkv, b);
        ++issued_v;
      }
      if (*abort_flag) {
        // Drain: every load issued lands before the CTA may exit. Loads land
        // on their own, so these bounded waits end unless the GPU is broken.
        volatile int no_abort = 0;
        mbar_wait(bar_q, 0, &no_abort, 12);
        for (int n = max(0, issued - Cfg::kStages); n < issued; ++n)
          mbar_wait(bar_k_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 13);
        for (int n = max(0, issued_v - Cfg::kStages); n < issued_v; ++n)
          mbar_wait(bar_v_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 14);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0 && any_work) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, false);
      const uint32_t idesc_o = idesc_bf16_f32(128, D, true);
      const uint32_t sQ = smem_u32(smem + Cfg::kOffQ);
      const uint32_t sK = smem_u32(smem + Cfg::kOffK);
      const uint32_t sV = smem_u32(smem + Cfg::kOffV);
      auto active = [&](int x, int j) { return j >= lo_x[x] && j < hi_x[x]; };
      auto issue_s = [&](int x, int st) {
        const uint32_t qa = sQ + x * Cfg::kTileBytes;
        const uint32_t ka = sK + st * Cfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * Cfg::kAtomBytes + (kk % 4) * 32;
          umma_ss(tmem_base + Cfg::col_s(x), smem_desc_sw128(qa + off, 16, 1024),
                  smem_desc_sw128(ka + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int x, int st, bool acc) {
        const uint32_t va = sV + st * Cfg::kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          umma_ts(tmem_base + Cfg::col_o(x), tmem_base + Cfg::col_s(x) + kk * 8,
                  smem_desc_sw128(va + kk * 2048, Cfg::kAtomBytes, 1024), idesc_o,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(bar_q, 0, abort_flag, 20);
      if (ok) ok = mbar_wait(bar_k_full + 0, 0, abort_flag, 21);
      if (ok) {
        tc_fence_after();
        for (int x = 0; x < 2; ++x)
          if (active(x, lo)) {
            issue_s(x, 0);
            umma_commit(bar_s_full + x);
          }
        umma_commit(bar_k_empty + 0);
      }
      uint32_t p_cnt[2] = {0, 0};
      for (int n = 0; ok && lo + n < hi; ++n) {
        const int j = lo + n;
        const int st = n % Cfg::kStages;
        const uint32_t ph = (n / Cfg::kStages) & 1;
        const bool has_next = j + 1 < hi;
        const int stn = (n + 1) % Cfg::kStages;
        const uint32_t phn = ((n + 1) / Cfg::kStages) & 1;
        ok = mbar_wait(bar_v_full + st, ph, abort_flag, 22);
        if (!ok) break;
        if (active(0, j)) {
          ok = mbar_wait(bar_p_ready + 0, p_cnt[0]++ & 1, abort_flag, 23);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, st, j > lo_x[0]);
        }
        if (has_next) {
          ok = mbar_wait(bar_k_full + stn, phn, abort_flag, 24);
          if (!ok) break;
          tc_fence_after();
          if (active(0, j + 1)) {
            issue_s(0, stn);
            umma_commit(bar_s_full + 0);
          }
        }
        if (active(1, j)) {
          ok = mbar_wait(bar_p_ready + 1, p_cnt[1]++ & 1, abort_flag, 25);
          if (!ok) break;
          tc_fence_after();
          issue_pv(1, st, j > lo_x[1]);
        }
        umma_commit(bar_v_empty + st);
        if (has_next) {
          if (active(1, j + 1)) {
            issue_s(1, stn);
            umma_commit(bar_s_full + 1);
          }
          umma_commit(bar_k_empty + stn);
        }
      }
      umma_commit(bar_o_done + 0);
      umma_commit(bar_o_done + 1);
      // Drain: TMEM may only be released once every issued MMA has finished.
      umma_commit(bar_drain);
      volatile int no_abort = 0;
      mbar_wait(bar_drain, 0, &no_abort, 26);
    }
    __syncwarp();
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::kSoftmaxRegs));
    // -------------------------------------------------------------- softmax
    const int x = warp / 4;  // query tile 0 (A) or 1 (B)
    const int quarter = warp % 4;
    const int row = r0_tile[x] + quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_s = Cfg::col_s(x);
    const uint32_t col_o = Cfg::col_o(x);
    const float sl2 = p.scale_log2;
    const float slope2 = (p.alibi != nullptr) ? p.alibi[h] * 1.4426950408889634f : 0.0f;
    const RowBounds rb = row_bounds(p, row);
    const long long row_lo = max(rb.jlo, 0ll);
    const long long row_hi = min(rb.jhi, (long long)lkey - 1);
    const long long diag = p.q_pos0 + row - p.k_pos0;
    const bool tiers = p.additive && !safe_x[x];

    float m_run = -INFINITY;
    float l_run = 0.0f;
    int tier = 3;
    bool ok = true;
    const int lo_t = lo_x[x], hi_t = hi_x[x];
    // Key tiles wholly inside [row_lo, row_hi] for every row of this tile.
    const int r_first = r0_tile[x], r_last = min(r0_tile[x] + 127, p.Sq - 1);
    const RowBounds rb_first = row_bounds(p, r_first), rb_last = row_bounds(p, r_last);
    const long long in_lo = max(rb_last.jlo, 0ll);
    const long long in_hi = min(rb_first.jhi, (long long)lkey - 1);

    for (int j = lo_t; j < hi_t; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full + x, (j - lo_t) & 1, abort_flag, 30 + x));
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      ENL_TMEM_LD128(lane_addr + col_s, sr);
      float s[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c]);
      const long long j0 = (long long)j * 128;
      const bool full_tile = (j0 >= in_lo) && (j0 + 127 <= in_hi) && !tiers && slope2 == 0.0f;
      bool reset = false;
      float m_tile = -INFINITY;
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < 128; ++c) m_tile = fmaxf(m_tile, s[c]);
        m_tile *= sl2;
      } else {
        // Per-tile bounds relative to the tile start, clamped into int range:
        // column c is key j0 + c.
        auto rel = [&](long long v) { return (int)max(-1ll, min(129ll, v - j0)); };
        const int c_lo = rel(row_lo), c_hi = rel(row_hi);  // unmasked columns [c_lo, c_hi]
        const float dbase = (float)(diag - j0);
        const bool alibi_abs = !p.causal;
        if (!tiers) {
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            float dist = dbase - (float)c;
            if (alibi_abs) dist = fabsf(dist);
            const float v = fmaf(s[c], sl2, -slope2 * dist);
            s[c] = (c >= c_lo && c <= c_hi) ? v : -INFINITY;
            m_tile = fmaxf(m_tile, s[c]);
          }
        } else {
          // -1e9 rule on rows without any unmasked key: only the scores with
          // the fewest -1e9 terms survive (exp(-1e9) underflows to 0 in float64).
          const int c_wlo = rel(rb.jlo), c_whi = rel(rb.jhi);  // causal/window bounds
          const int c_pad = rel(lkey);                          // first padded column
          const int cend = min(128, rel(p.Skv));                // columns [0, cend) exist
          // Smallest tier present in this tile, from interval arithmetic:
          // tier(c) = [c >= c_pad] + [c < c_wlo or c > c_whi].
          int tmin;
          if (max(0, c_wlo) <= min(min(c_whi, c_pad - 1), cend - 1)) {
            tmin = 0;
          } else {
            const int real_hi = min(c_pad, cend) - 1;  // real columns [0, real_hi]
            const bool real_blocked = real_hi >= 0 && (c_wlo > 0 || real_hi > c_whi);
            const bool pad_open =
                max(max(c_pad, 0), c_wlo) <= min(cend - 1, c_whi);  // padded, unblocked
            tmin = (real_blocked || pad_open) ? 1 : (cend > 0 ? 2 : 3);
          }
          const int new_tier = min(tier, tmin);
          reset = new_tier < tier;
          tier = new_tier;
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const int t = (int)(c >= c_pad) + (int)(c < c_wlo || c > c_whi);
            float dist = dbase - (float)c;
            if (alibi_abs) dist = fabsf(dist);
            const float v = fmaf(s[c], sl2, -slope2 * dist);
            s[c] = (c < cend && t == new_tier) ? v : -INFINITY;
            m_tile = fmaxf(m_tile, s[c]);
          }
        }
      }
      // Lazy rescale: keep the old reference max unless it grew by > 8 (log2).
      float factor = 1.0f;
      if (reset) {
        factor = 0.0f;
        m_run = m_tile;
        l_run = 0.0f;
      } else if (m_tile > m_run + 8.0f) {
        factor = exp2f(m_run - m_tile);  // 0 when m_run == -inf
        m_run = m_tile;
      }
      const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
      float rowsum = 0.0f;
      uint32_t pk[64];
      if (full_tile) {
        // Unmasked tile: s is still the raw dot product; fold the scale in.
        const float neg_m = -m_use;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p0 = fast_exp2(fmaf(s[2 * c], sl2, neg_m));
          const float p1 = fast_exp2(fmaf(s[2 * c + 1], sl2, neg_m));
          rowsum += p0 + p1;
          pk[c] = pack_bf16x2(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p0 = fast_exp2(s[2 * c] - m_use);
          const float p1 = fast_exp2(s[2 * c + 1] - m_use);
          rowsum += p0 + p1;
          pk[c] = pack_bf16x2(p0, p1);
        }
      }
      l_run = l_run * factor + rowsum;
      // O correction (warp-collective): only once O holds earlier tiles.
      const bool need_corr = (j > lo_t) && (factor != 1.0f);
      if (__any_sync(0xffffffffu, need_corr)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          ENL_TMEM_LD32(lane_addr + col_o + c * 32, o, 0);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          ENL_TMEM_ST32(lane_addr + col_o + c * 32, o, 0);
        }
      }
      ENL_TMEM_ST32(lane_addr + col_s, pk, 0);
      ENL_TMEM_ST32(lane_addr + col_s + 32, pk, 32);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_ready + x);
    }

    // ------------------------------------------------------------- epilogue
    const bool row_valid = row < p.Sq;
    ok = __all_sync(0xffffffffu, ok && !*abort_flag);
    const bool warp_has_rows = __any_sync(0xffffffffu, row_valid);
    if (ok && warp_has_rows) {
      const bool have_o = lo_t < hi_t;
      if (have_o)
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o_done + x, 0, abort_flag, 35 + x));
      if (ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l_run;  // 0/0 -> NaN for rows with no key
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                        ((long long)b * p.o_sb + (long long)row * p.o_ss + (long long)h * p.o_sh) *
                            (p.out_fp32 ? 4 : 2);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          __syncwarp();  // the stores below diverge by row; reconverge for tcgen05.ld
          if (have_o) {
            ENL_TMEM_LD32(lane_addr + col_o + c * 32, o, 0);
          }
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = have_o ? __uint_as_float(o[i]) * inv_l : NAN;
          if (row_valid && p.out_fp32) {
            float4* dst = reinterpret_cast<float4*>(orow + c * 32 * 4);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else if (row_valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32 * 2);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]),
                                  pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                  pack_bf16x2(v[8 * i + 4], v[8 * i + 5]),
                                  pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
          }
        }
        if (p.lse != nullptr && row_valid) {
          float lse = have_o ? (m_run + log2f(l_run)) * 0.6931471805599453f : NAN;
          if (tiers && tier > 0) lse -= 1e9f * (float)tier;
          p.lse[((long long)b * p.H + h) * p.Sq + row] = lse;
        }
      }
    }
    // Every tcgen05.ld/st above sits under warp-uniform control flow; rows
    // past Sq only skip their global stores.
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem_base);
  }
}

template <int D>
int prefill_smem_bytes() {
  return PrefillCfg<D>::kSmemBytes;
}

template <int D>
cudaError_t launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const PrefillParams& p, cudaStream_t stream) {
  using Cfg = PrefillCfg<D>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_sm100<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int q_tiles = (p.Sq + 127) / 128;
  const int pairs = (q_tiles + 1) / 2;
  dim3 grid(p.B * p.H, pairs);
  attn_prefill_sm100<D><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

template cudaError_t launch_prefill<64>(const CUtensorMap&, const CUtensorMap&,
                                        const CUtensorMap&, const PrefillParams&, cudaStream_t);
template cudaError_t launch_prefill<128>(const CUtensorMap&, const CUtensorMap&,
                                         const CUtensorMap&, const PrefillParams&, cudaStream_t);

}  // namespace enl
