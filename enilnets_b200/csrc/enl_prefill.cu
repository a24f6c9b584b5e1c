// K1: fused flash-style attention prefill for sm_100a.
//
// Replaces the score/softmax/context math of the reference's attention
// forward: nn/forward.py:525-551 (plain MHA), nn/flash_attention.py:42-80
// (streaming softmax, the algorithmic spec followed here), nn/forward.py:578-586
// (cross-attention) and the key-padding rule of graph/sequence.py:159-183.
//
// Persistent kernel: one CTA per SM (three warpgroups, 384 threads) walks a
// static list of work items, each one 128-row query tile of one
// (batch, head), and streams 128-key tiles of K and V through shared memory:
//   warp 8      TMA producer: each item's Q tile into one of two Q buffers,
//               then its K/V tiles into a ring shared by all items
//   warp 9      S issuer: S = Q K^T (smem x smem) into a double-buffered S
//               in tensor memory
//   warp 10     P V issuer: O += P V with P read from tensor memory
//   warp 11     output stores: for bf16 output the epilogue stages O in the
//               finished item's Q buffer (the Q tile's swizzled layout) and
//               this warp writes it with TMA bulk-tensor stores, then
//               releases the buffer to the next Q load
// The two issuers run independently (warp-uniform loops, elect.sync issue),
// so a P V never queues behind the issue of an S that the tensor pipe is
// still busy with; S(g + 2) waits only for P V(g) to finish with its buffer.
//   warps 0-3   softmax, key columns 0-63 of every key tile
//   warps 4-7   softmax, key columns 64-127
// Thread (warp w, lane l) owns query row 32*(w%4) + l == TMEM lane. The two
// softmax warpgroups are independent online-softmax streams over the two
// halves of every key tile, each with its own running max, sum and output
// accumulator (O0 over keys 64t..64t+63, O1 over keys 64t+64..64t+127 of
// tile t); the epilogue merges them by log-sum-exp.
//
// The MMA and TMA warps run ahead across item boundaries: while the softmax
// warps finish one item (last tiles, then the epilogue), the next item's Q,
// K/V and first two S tiles are already loaded and computed, so an item
// costs its tiles plus the epilogue instead of a full pipeline fill and
// drain. Only the first P V of the next item waits for the epilogue to have
// read the O accumulators.
//
// Tensor memory: S0 | S1 | O0 | O1 (128 + 128 + D + D columns). S is double
// buffered; each softmax half writes its bf16 P back over the first 32
// columns of its own half of S(j), and O_h += P_h V_h runs as soon as that
// half is published. The online softmax rescales O lazily: only when a row
// max grows by more than 2^8 does a thread pull its accumulator out of
// tensor memory, scale and store it back.
//
// Masking semantics (see PrefillParams): causal / sliding window / per-batch
// key-valid length / ALiBi, either with -inf exclusion (nn/ path) or with the
// graph path's additive -1e9 rule, which is applied exactly by tracking the
// number of -1e9 terms ("tier") per score when a row has no unmasked key.
#include <climits>

#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

// One in kEmuEvery score pairs of an unmasked tile takes its exponentials
// from exp2_poly (FMA pipe) instead of MUFU ex2; 0 disables the split.
#ifndef ENL_EXP_EMU_EVERY
#define ENL_EXP_EMU_EVERY 4
#endif
#ifndef ENL_EXP_EMU_EVERY_D64
#define ENL_EXP_EMU_EVERY_D64 4
#endif
constexpr int kEmuEvery = ENL_EXP_EMU_EVERY;
constexpr int kEmuEvery64 = ENL_EXP_EMU_EVERY_D64;  // head dim 64: half the tensor work per tile

// kSplit: fp32 inputs arrive as two bf16 planes, hi = bf16(x) and
// lo = bf16(x - hi), and each product is formed from three bf16 MMAs
// (hi*hi + hi*lo + lo*hi, fp32 accumulate), about 2^-16 relative error:
// better than tf32 on the same tensor cores. P is split the same way in
// tensor memory, its lo half over the second 32 columns of each key half.
template <int D, bool kSplit>
struct PrefillCfg {
  static constexpr int kThreads = 384;
  static constexpr int kPlanes = kSplit ? 2 : 1;  // bf16 planes per operand tile
  static constexpr int kStages = kSplit ? ((D == 128) ? 1 : 2) : ((D == 128) ? 2 : 4);
  static constexpr int kQBufs = (kSplit && D == 128) ? 1 : 2;
  static constexpr int kAtoms = D / 64;  // 128-byte swizzle atoms along the head dim
  static constexpr int kTileBytes = 128 * D * 2;          // one plane of a 128-row tile
  static constexpr int kOpBytes = kPlanes * kTileBytes;   // all planes of one tile
  static constexpr int kAtomBytes = 128 * 128;  // 128 rows x 128 bytes
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBufs * kOpBytes;
  static constexpr int kOffV = kOffK + kStages * kOpBytes;
  static constexpr int kOffX = kOffV + kStages * kOpBytes;  // epilogue exchange
  static constexpr int kXBytes = 3 * 2 * 128 * 4;            // m, l, tier [2 halves][128]
  static constexpr int kOffItems = kOffX + kXBytes;  // decoded items [8 softmax warps][2]
  static constexpr int kOffBar = kOffItems + 8 * 2 * 32;
  // q_full/empty[kQBufs], k_full/empty, v_full/empty, s_full[2],
  // p_ready[2 buf][2 half], o_prog[2], o_done, o_free, pv_done[2], drain[2],
  // stage_full
  static constexpr int kNumBars = 2 * kQBufs + 4 * kStages + 2 + 4 + 2 + 1 + 1 + 2 + 2 + 1;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // +align slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static constexpr uint32_t kTmemCols = 512;
  // Exponentials from the FMA-pipe polynomial are too coarse for the split path.
  static constexpr int kEmu = kSplit ? 0 : (D == 64 ? kEmuEvery64 : kEmuEvery);
  __host__ __device__ static constexpr uint32_t col_s(int buf) { return 128u * buf; }
  __host__ __device__ static constexpr uint32_t col_o(int half) { return 256u + D * half; }
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

// Work item t -> (batch, head, query tile) and its key-tile range. Items come
// in sections of p.sec_bh consecutive (batch, head) pairs; inside a section
// the last (heaviest under a causal mask) query tiles come first. CTA c takes
// items c, c + gridDim.x, ...: the CTAs running at one time share a few
// heads' K/V in L2, and the lightest items run last.
struct WorkItem {
  int b, h, hkv, r0;
  int lo, hi;  // key tiles [lo, hi)
  int lkey;    // valid keys of this batch row
  int safe;    // every row of the tile has an unmasked key
};
static_assert(sizeof(WorkItem) == 32, "softmax warps keep items in 32-byte slots");

// Template modes of K1: dense masks, block-sparse layouts, and dense masks
// with an arbitrary per-key mask.
constexpr int kModeDense = 0, kModeSparse = 1, kModeKeyMask = 2;

template <int kMode>
__device__ __forceinline__ WorkItem work_item(const PrefillParams& p, int t) {
  constexpr bool kSparse = kMode == kModeSparse;
  const int n_qt = (p.Sq + 127) / 128;
  const int n_bh = p.n_bh;
  const int per_sec = p.sec_bh * n_qt;
  const int s = t / per_sec;
  const int r = t - s * per_sec;
  const int sb = min(p.sec_bh, n_bh - s * p.sec_bh);
  const int qt = n_qt - 1 - r / sb;
  int bh = s * p.sec_bh + r % sb;
  if (p.units != nullptr) {  // this call's (batch, head) units, b * H + h each
    bh = p.units[bh];
    if (bh < 0 || bh >= p.B * p.H) {
      report_error(kDevBadIndex, bh);
      bh = 0;
    }
  }
  WorkItem w;
  w.b = bh / p.H;
  w.h = bh % p.H;
  w.hkv = w.h / (p.H / p.Hkv);
  w.r0 = qt * 128;
  w.lkey = p.Skv;
  if (p.kv_len != nullptr) w.lkey = max(0, min(p.kv_len[w.b], p.Skv));
  if constexpr (kSparse) {
    // Entries [sp_ptr[qt], sp_ptr[qt + 1]) of the layout; every row of a
    // sparse tile sees at least its own key, so -inf exclusion is exact.
    w.lo = p.sp_ptr[qt];
    w.hi = p.sp_ptr[qt + 1];
    if (w.lo < 0 || w.hi > p.sp_entries || w.lo > w.hi) {
      report_error(kDevBadIndex, qt);
      w.lo = w.hi = 0;
    }
    w.safe = 1;
  } else if constexpr (kMode == kModeKeyMask) {
    // Ranges computed per (batch row, query tile) by mask_tiles_kernel.
    const int4 mt = p.mask_tiles[(long long)w.b * n_qt + qt];
    w.lo = mt.x;
    w.hi = mt.y;
    w.safe = mt.z;
  } else {
    bool safe;
    tile_range(p, w.r0, w.lkey, (p.Skv + 127) / 128, w.lo, w.hi, safe);
    w.safe = safe;
  }
  return w;
}

// Key tile of the n-th visit of an item: the layout's entry in sparse mode,
// otherwise the visit index itself.
template <bool kSparse>
__device__ __forceinline__ int key_tile(const PrefillParams& p, int j) {
  if constexpr (kSparse) return p.sp_kt[j];
  return j;
}

// Walks this CTA's (item, key tile) sequence, skipping items without keys.
template <int kMode>
struct TileCursor {
  int t;       // item id (>= n_items: done)
  int j, lo, hi;
  int wi;      // ordinal of the item among this CTA's items with work
  __device__ __forceinline__ void seek(const PrefillParams& p) {
    while (t < p.n_items) {
      const WorkItem w = work_item<kMode>(p, t);
      if (w.lo < w.hi) {
        j = lo = w.lo;
        hi = w.hi;
        return;
      }
      t += gridDim.x;
    }
  }
  __device__ __forceinline__ void start(const PrefillParams& p) {
    t = blockIdx.x;
    wi = 0;
    seek(p);
  }
  __device__ __forceinline__ void next(const PrefillParams& p) {
    if (++j >= hi) {
      t += gridDim.x;
      ++wi;
      seek(p);
    }
  }
  __device__ __forceinline__ bool valid(const PrefillParams& p) const { return t < p.n_items; }
};

template <int D, bool kSplit, int kMode>
__global__ void __launch_bounds__(384, 1)
    attn_prefill_sm100(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const PrefillParams p) {
  using Cfg = PrefillCfg<D, kSplit>;
  constexpr bool kSparse = kMode == kModeSparse;
  constexpr bool kKeyMask = kMode == kModeKeyMask;
  // bf16 output of the bf16 path leaves through TMA stores: the epilogue
  // stages O in the finished item's Q buffer and warp 11 stores it, then
  // releases the buffer. Otherwise the epilogue stores rows directly and the
  // last S of an item releases its Q buffer.
  const bool tma_st = !kSplit && Cfg::kQBufs == 2 && !p.out_fp32;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* x_m = reinterpret_cast<float*>(smem + Cfg::kOffX);  // [2 half][128]
  float* x_l = x_m + 2 * 128;                                    // [2 half][128]
  int* x_t = reinterpret_cast<int*>(x_l + 2 * 128);              // [2 half][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* bar_q_full = bars + 0;                       // [kQBufs]
  uint64_t* bar_q_empty = bar_q_full + Cfg::kQBufs;      // [kQBufs]
  uint64_t* bar_k_full = bar_q_empty + Cfg::kQBufs;
  uint64_t* bar_k_empty = bar_k_full + Cfg::kStages;
  uint64_t* bar_v_full = bar_k_empty + Cfg::kStages;
  uint64_t* bar_v_empty = bar_v_full + Cfg::kStages;
  uint64_t* bar_s_full = bar_v_empty + Cfg::kStages;  // [2 buffers]
  uint64_t* bar_p_ready = bar_s_full + 2;             // [2 buffers][2 halves]
  uint64_t* bar_o_prog = bar_p_ready + 4;             // [2 halves] one phase per P V
  uint64_t* bar_o_done = bar_o_prog + 2;              // one phase per item
  uint64_t* bar_o_free = bar_o_done + 1;              // epilogue has read O; per item
  uint64_t* bar_pv_done = bar_o_free + 1;             // [2 buffers] P V of a tile complete
  uint64_t* bar_drain = bar_pv_done + 2;              // [2 issuing warps]
  uint64_t* bar_stage_full = bar_drain + 2;           // O staged for the TMA store; per item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kNumBars; ++i) {
      uint32_t count = 1;
      if (bars + i >= bar_p_ready && bars + i < bar_p_ready + 4) count = 4;  // one per warp
      if (bars + i == bar_o_free || bars + i == bar_stage_full) count = 8;  // every softmax warp
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

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int q_issued = 0, issued = 0, issued_v = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.n_items && ok; t += gridDim.x) {
        const WorkItem w = work_item<kMode>(p, t);
        if (w.lo >= w.hi) continue;
        // Split mode: the plane tensors interleave (hi, lo) per head, so
        // plane pl of head h is "head" kPlanes * h + pl of the tensor map.
        const int qb = q_issued % Cfg::kQBufs;
        const uint32_t quse = q_issued / Cfg::kQBufs;
        if (quse > 0) ok = mbar_wait(bar_q_empty + qb, (quse - 1) & 1, abort_flag, 9);
        if (!ok) break;
        mbar_arrive_expect_tx(bar_q_full + qb, Cfg::kOpBytes);
        for (int pl = 0; pl < Cfg::kPlanes; ++pl)
          for (int a = 0; a < Cfg::kAtoms; ++a)
            tma_load_4d(smem + Cfg::kOffQ + qb * Cfg::kOpBytes + pl * Cfg::kTileBytes +
                            a * Cfg::kAtomBytes,
                        &tm_q, bar_q_full + qb, a * 64, w.r0, Cfg::kPlanes * w.h + pl, w.b);
        ++q_issued;
        for (int j = w.lo; j < w.hi && ok; ++j, ++issued) {
          const int kt = key_tile<kSparse>(p, j);
          const int st = issued % Cfg::kStages;
          const uint32_t use = issued / Cfg::kStages;
          if (use > 0) ok = mbar_wait(bar_k_empty + st, (use - 1) & 1, abort_flag, 10);
          if (!ok) break;
          mbar_arrive_expect_tx(bar_k_full + st, Cfg::kOpBytes);
          for (int pl = 0; pl < Cfg::kPlanes; ++pl)
            for (int a = 0; a < Cfg::kAtoms; ++a)
              tma_load_4d(smem + Cfg::kOffK + st * Cfg::kOpBytes + pl * Cfg::kTileBytes +
                              a * Cfg::kAtomBytes,
                          &tm_k, bar_k_full + st, a * 64, kt * 128, Cfg::kPlanes * w.hkv + pl,
                          w.b);
          if (use > 0) ok = mbar_wait(bar_v_empty + st, (use - 1) & 1, abort_flag, 11);
          if (!ok) {
            ++issued;  // the K load of this iteration is in flight
            break;
          }
          mbar_arrive_expect_tx(bar_v_full + st, Cfg::kOpBytes);
          for (int pl = 0; pl < Cfg::kPlanes; ++pl)
            for (int a = 0; a < Cfg::kAtoms; ++a)
              tma_load_4d(smem + Cfg::kOffV + st * Cfg::kOpBytes + pl * Cfg::kTileBytes +
                              a * Cfg::kAtomBytes,
                          &tm_v, bar_v_full + st, a * 64, kt * 128, Cfg::kPlanes * w.hkv + pl,
                          w.b);
          ++issued_v;
        }
      }
      if (*abort_flag) {
        // Drain: every load issued lands before the CTA may exit. Loads land
        // on their own, so these bounded waits end unless the GPU is broken.
        volatile int no_abort = 0;
        for (int n = max(0, q_issued - Cfg::kQBufs); n < q_issued; ++n)
          mbar_wait(bar_q_full + n % Cfg::kQBufs, (n / Cfg::kQBufs) & 1, &no_abort, 12);
        for (int n = max(0, issued - Cfg::kStages); n < issued; ++n)
          mbar_wait(bar_k_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 13);
        for (int n = max(0, issued_v - Cfg::kStages); n < issued_v; ++n)
          mbar_wait(bar_v_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 14);
      }
    }
    __syncwarp();
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------- MMA (S, P V)
    // Each issuing warp runs its loop with warp-uniform values; elect.sync
    // inside the issue helpers picks the single lane that issues.
    const uint32_t idesc_s = idesc_bf16_f32(128, 128, false);
    const uint32_t idesc_o = idesc_bf16_f32(128, D, true);
    // Descriptor low words, computed once; each MMA adds an immediate
    // (16-byte units) for its buffer and K step.
    const uint32_t q_lo = desc_lo(smem_u32(smem + Cfg::kOffQ), 16);
    const uint32_t k_lo = desc_lo(smem_u32(smem + Cfg::kOffK), 16);
    const uint32_t v_lo = desc_lo(smem_u32(smem + Cfg::kOffV), Cfg::kAtomBytes);
    constexpr uint32_t kTileLo = Cfg::kTileBytes >> 4;  // one plane, 16-byte units
    constexpr uint32_t kOpLo = Cfg::kOpBytes >> 4;
    auto wait = [&](uint64_t* bar, uint32_t parity, int site) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site));
    };
    TileCursor<kMode> cur;
    cur.start(p);
    uint32_t g = 0;  // tiles of this CTA issued so far
    bool ok = true;
    if (warp == 9) {
      // S(g) overwrites the buffer that held P(g - 2): it waits for that
      // tile's P V to complete (pv_done), then for Q and K(g).
      for (; ok && cur.valid(p); ++g, cur.next(p)) {
        const int buf = g & 1;
        const int qb = cur.wi % Cfg::kQBufs;
        const int st = g % Cfg::kStages;
        if (g >= 2) ok = wait(bar_pv_done + buf, ((g - 2) >> 1) & 1, 24);
        if (ok && cur.j == cur.lo) ok = wait(bar_q_full + qb, (cur.wi / Cfg::kQBufs) & 1, 20);
        if (ok) ok = wait(bar_k_full + st, (g / Cfg::kStages) & 1, 21);
        if (!ok) break;
        tc_fence_after();
        const uint32_t qa = q_lo + qb * kOpLo;
        const uint32_t ka = k_lo + st * kOpLo;
        const uint32_t d = tmem_base + Cfg::col_s(buf);
        umma_ss_elect<false>(d, qa, ka, kDescHiSw128, idesc_s);
        if constexpr (kSplit) {
          umma_ss_elect<true>(d, qa, ka + kTileLo, kDescHiSw128, idesc_s);  // Qhi Klo
          umma_ss_elect<true>(d, qa + kTileLo, ka, kDescHiSw128, idesc_s);  // Qlo Khi
        }
#pragma unroll
        for (int kk = 1; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * (Cfg::kAtomBytes >> 4) + (kk % 4) * 2;
          umma_ss_elect<true>(d, qa + off, ka + off, kDescHiSw128, idesc_s);
          if constexpr (kSplit) {
            umma_ss_elect<true>(d, qa + off, ka + kTileLo + off, kDescHiSw128, idesc_s);
            umma_ss_elect<true>(d, qa + kTileLo + off, ka + off, kDescHiSw128, idesc_s);
          }
        }
        umma_commit_elect(bar_s_full + buf);
        umma_commit_elect(bar_k_empty + st);
        // The item's last S: its Q buffer is free once this MMA completes
        // (unless the epilogue stages O there).
        if (cur.j == cur.hi - 1 && !tma_st) umma_commit_elect(bar_q_empty + qb);
      }
    } else {
      // O_hf += P_hf V_hf over one key half: P of half hf sits in columns
      // [64*hf, 64*hf + 32) of the S buffer (two bf16 per column), V_hf is
      // key rows [64*hf, 64*hf + 64) of the V tile. Split mode adds Phi Vlo
      // and Plo Vhi, Plo in columns [32, 64) of the half.
      for (; ok && cur.valid(p); ++g, cur.next(p)) {
        const int buf = g & 1;
        const int st = g % Cfg::kStages;
        ok = wait(bar_v_full + st, (g / Cfg::kStages) & 1, 22);
        if (!ok) break;
        const bool first = cur.j == cur.lo;
        // The first P V of an item overwrites O: the previous item's
        // epilogue must have read it.
        if (first && cur.wi > 0) {
          ok = wait(bar_o_free, (cur.wi - 1) & 1, 25);
          if (!ok) break;
        }
        for (int hf = 0; hf < 2 && ok; ++hf) {
          ok = wait(bar_p_ready + 2 * buf + hf, (g >> 1) & 1, 23);
          if (!ok) break;
          tc_fence_after();
          const uint32_t va = v_lo + st * kOpLo + hf * 4 * (2048 >> 4);
          const uint32_t a = tmem_base + Cfg::col_s(buf) + hf * 64;
          const uint32_t d = tmem_base + Cfg::col_o(hf);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t vk = va + kk * (2048 >> 4);
            umma_ts_elect(d, a + kk * 8, vk, kDescHiSw128, idesc_o, (!first || kk > 0) ? 1u : 0u);
            if constexpr (kSplit) {
              umma_ts_elect(d, a + kk * 8, vk + kTileLo, kDescHiSw128, idesc_o, 1u);
              umma_ts_elect(d, a + 32 + kk * 8, vk, kDescHiSw128, idesc_o, 1u);
            }
          }
          umma_commit_elect(bar_o_prog + hf);
        }
        if (!ok) break;
        umma_commit_elect(bar_v_empty + st);
        umma_commit_elect(bar_pv_done + buf);
        if (cur.j == cur.hi - 1) umma_commit_elect(bar_o_done);
      }
    }
    // Drain: TMEM may only be released once every MMA this warp issued has
    // finished.
    uint64_t* drain = bar_drain + (warp - 9);
    umma_commit_elect(drain);
    volatile int no_abort = 0;
    mbar_wait(drain, 0, &no_abort, 26);
  } else if (warp == 11) {
    // ------------------------------------------------------------- O stores
    if (tma_st && lane == 0) {
      tma_prefetch_desc(&tm_o);
      int wi = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.n_items && ok; t += gridDim.x) {
        const WorkItem w = work_item<kMode>(p, t);
        if (w.lo >= w.hi) continue;
        const int qb = wi % Cfg::kQBufs;
        ok = mbar_wait(bar_stage_full, wi & 1, abort_flag, 40);
        if (!ok) break;
        const uint8_t* stage = smem + Cfg::kOffQ + qb * Cfg::kOpBytes;
        for (int a = 0; a < Cfg::kAtoms; ++a)
          tma_store_4d(&tm_o, stage + a * Cfg::kAtomBytes, a * 64, w.r0, w.h, w.b);
        bulk_commit_group();
        bulk_wait_read_all();  // the buffer may now take the next Q tile
        mbar_arrive(bar_q_empty + qb);
        ++wi;
      }
      bulk_wait_all();  // the output is in global memory before the CTA exits
    }
    __syncwarp();
  } else if (warp < 8) {
    // -------------------------------------------------------------- softmax
    const int half = warp / 4;  // key columns [64*half, 64*half + 64)
    const int quarter = warp % 4;
    const int rloc = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_h = 64 * half;
    const float sl2 = p.scale_log2;
    uint32_t g = 0;   // tiles of this CTA seen so far (S buffer and phase)
    int wi = 0;       // items with work seen so far (o_done / o_free phase)
    bool failed = false;  // a wait ran out of time; skip the remaining work
    // Each warp decodes the next item during the current one's epilogue
    // (where the decode's latency overlaps the waits) and keeps it in its
    // own shared-memory slot: nothing of it stays live in registers across
    // the tile loop, which runs at the register limit.
    WorkItem* slots = reinterpret_cast<WorkItem*>(smem + Cfg::kOffItems) + 2 * warp;
    if (lane == 0) slots[0] = work_item<kMode>(p, blockIdx.x);
    int k = 0;  // this CTA's item ordinal
    for (int t = blockIdx.x; t < p.n_items; t += gridDim.x, ++k) {
      __syncwarp();
      const WorkItem w = slots[k & 1];
      const int lo = w.lo, hi = w.hi, lkey = w.lkey;
      const int h = w.h;
      const int row = w.r0 + rloc;
      const float slope2 = (p.alibi != nullptr) ? p.alibi[h] * 1.4426950408889634f : 0.0f;
      // Mask bounds as key indices clamped to [-2, Skv + 2]: every index
      // outside [0, Skv) acts the same, and 32-bit values keep the loop
      // below within the register budget.
      auto clampk = [&](long long v) {
        return (int)max(-2ll, min((long long)p.Skv + 2, v));
      };
      const RowBounds rb = row_bounds(p, row);
      const int jlo_c = clampk(rb.jlo), jhi_c = clampk(rb.jhi);
      const int row_lo = max(jlo_c, 0);
      const int row_hi = min(jhi_c, lkey - 1);
      const long long diag = p.q_pos0 + row - p.k_pos0;
      const bool tiers = p.additive && !w.safe;
      // Key tiles wholly inside [row_lo, row_hi] for every row of the tile.
      const int r_last = min(w.r0 + 127, p.Sq - 1);
      const int in_lo = max(clampk(row_bounds(p, r_last).jlo), 0);
      const int in_hi = min(clampk(row_bounds(p, w.r0).jhi), lkey - 1);

      float m_run = -INFINITY;  // this half's running max (log2 domain)
      float l_run = 0.0f;       // this half's running sum
      int tier = 3;             // fewest -1e9 terms seen by this half (tier mode)

      for (int n = 0; lo + n < hi && !failed; ++n, ++g) {
        const int j = lo + n;
        const int buf = g & 1;
        // Sparse mode: this row's allowed columns of this half, loaded before
        // the wait so the load's latency hides behind it.
        unsigned long long allow = ~0ull;
        int kt = j;
        if constexpr (kSparse) {
          kt = p.sp_kt[j];
          allow = p.sp_mask[((long long)j * 2 + half) * 128 + rloc];
        }
        // Key-mask mode: which of this half's 64 keys are real (the same word
        // for every row of the batch row; columns past Skv read as padding).
        unsigned long long real = ~0ull;
        if constexpr (kKeyMask) {
          const int widx = kt * 2 + half;
          real = (widx * 64 < p.Skv) ? p.kv_mask[(long long)w.b * p.kv_mask_sb + widx] : 0ull;
        }
        failed = !__all_sync(0xffffffffu,
                             mbar_wait(bar_s_full + buf, (g >> 1) & 1, abort_flag, 30 + half));
        if (failed) break;
        tc_fence_after();
        const uint32_t s_addr = lane_addr + Cfg::col_s(buf) + col_h;
        if constexpr (kSparse) {
          if (__all_sync(0xffffffffu, allow == 0ull)) {
            // No key of this half is visible to any of the warp's rows (a
            // half-tile between selected blocks): publish P = 0 without
            // reading S or taking exponentials. The row statistics are
            // unchanged, as a tile of -inf scores would leave them.
            uint32_t z[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) z[c] = 0u;
            ENL_TMEM_ST32(s_addr, z, 0);
            if constexpr (kSplit) ENL_TMEM_ST32(s_addr + 32, z, 0);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_p_ready + 2 * buf + half);
            continue;
          }
        }
        float s[64];
        {
          uint32_t sr[64];
          ENL_TMEM_LD32X2(s_addr, sr, s_addr + 32, (sr + 32));  // both loads under one wait
#pragma unroll
          for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sr[c]);
        }
        const int j0 = kt * 128 + (int)col_h;  // key index of this half's column 0
        bool full_tile;
        if constexpr (kSparse)  // rows past Sq are never stored: they do not force masking
          full_tile = __all_sync(0xffffffffu, allow == ~0ull || row >= p.Sq) && slope2 == 0.0f;
        else
          full_tile = (j0 >= in_lo) && (j0 + 63 <= in_hi) && !tiers && slope2 == 0.0f &&
                      (!kKeyMask || real == ~0ull);
        bool reset = false;
        float m_tile = -INFINITY;
        if (full_tile) {
          float mx[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = fmax3(s[k], s[8 + k], s[16 + k]);
#pragma unroll
          for (int c = 24; c < 56; c += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = fmax3(mx[k], s[c + k], s[c + 8 + k]);
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], s[56 + k]);
          m_tile = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]),
                         fmaxf(mx[6], mx[7])) * sl2;
        } else {
          // Bounds relative to this half's first column, clamped into int
          // range: column c is key j0 + c.
          auto rel = [&](int v) { return max(-1, min(65, v - j0)); };
          const float dbase = (float)(diag - j0);
          const bool alibi_abs = !p.causal;
          if constexpr (kSparse) {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              float dist = dbase - (float)c;
              if (alibi_abs) dist = fabsf(dist);
              const float v = fmaf(s[c], sl2, -slope2 * dist);
              s[c] = ((allow >> c) & 1ull) ? v : -INFINITY;
              m_tile = fmaxf(m_tile, s[c]);
            }
          } else if (!tiers) {
            const int c_lo = rel(row_lo), c_hi = rel(row_hi);  // unmasked columns [c_lo, c_hi]
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              float dist = dbase - (float)c;
              if (alibi_abs) dist = fabsf(dist);
              const float v = fmaf(s[c], sl2, -slope2 * dist);
              const bool key_ok = !kKeyMask || ((real >> c) & 1ull);
              s[c] = (c >= c_lo && c <= c_hi && key_ok) ? v : -INFINITY;
              m_tile = fmaxf(m_tile, s[c]);
            }
          } else {
            // -1e9 rule on rows without any unmasked key: only the scores
            // with the fewest -1e9 terms survive (exp(-1e9) underflows to 0
            // in float64). tier(key) = [key >= lkey] + [key < jlo or key > jhi];
            // the smallest tier of this half's 64 columns comes from interval
            // arithmetic, the epilogue keeps the half with the smaller tier.
            const int c_wlo = rel(jlo_c), c_whi = rel(jhi_c), c_pad = rel(lkey);
            const int cend = min(64, rel(p.Skv));  // columns [0, cend) exist
            int tmin;
            unsigned long long realb = 0ull;  // key-mask mode: real columns
            if constexpr (kKeyMask) {
              // Same tiers from bit sets: real = mask word, below the valid
              // length and inside the sequence; win = columns [c_wlo, c_whi].
              auto below = [](int n) {  // bits [0, n)
                return n >= 64 ? ~0ull : (n <= 0 ? 0ull : ((1ull << n) - 1ull));
              };
              const unsigned long long exist = below(cend);
              realb = real & below(c_pad) & exist;
              const int wa = max(0, c_wlo), wb = min(63, c_whi);
              const unsigned long long win = wa > wb ? 0ull : (below(wb + 1) & ~below(wa));
              if (realb & win)
                tmin = 0;
              else if ((realb & ~win) | (~realb & win & exist))
                tmin = 1;
              else
                tmin = exist ? 2 : 3;
            } else if (max(0, c_wlo) <= min(min(c_whi, c_pad - 1), cend - 1)) {
              tmin = 0;
            } else {
              const int real_hi = min(c_pad, cend) - 1;  // real columns [0, real_hi]
              const bool real_blocked = real_hi >= 0 && (c_wlo > 0 || real_hi > c_whi);
              const bool pad_open = max(max(c_pad, 0), c_wlo) <= min(cend - 1, c_whi);
              tmin = (real_blocked || pad_open) ? 1 : (cend > 0 ? 2 : 3);
            }
            const int new_tier = min(tier, tmin);
            reset = new_tier < tier;
            tier = new_tier;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              const bool padded = kKeyMask ? !((realb >> c) & 1ull) : (c >= c_pad);
              const int tt = (int)padded + (int)(c < c_wlo || c > c_whi);
              float dist = dbase - (float)c;
              if (alibi_abs) dist = fabsf(dist);
              const float v = fmaf(s[c], sl2, -slope2 * dist);
              s[c] = (c < cend && tt == new_tier) ? v : -INFINITY;
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
        uint32_t pk[32];
        uint32_t pl[kSplit ? 32 : 1];  // split mode: bf16(p - bf16(p)) pairs
        if (full_tile) {
          // Unmasked tile: s is still the raw dot product; fold the scale in
          // with packed FMAs, accumulate the row sum in 4 packed lanes.
          const uint64_t scale2 = f2_pack(sl2, sl2);
          const uint64_t negm2 = f2_pack(-m_use, -m_use);
          uint64_t acc[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) acc[k] = f2_pack(0.0f, 0.0f);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(s[2 * c], s[2 * c + 1]), scale2, negm2), x0, x1);
            float p0, p1;
            if (Cfg::kEmu > 0 && (c % (Cfg::kEmu > 0 ? Cfg::kEmu : 1)) == Cfg::kEmu - 1) {
              exp2_poly2(x0, x1, p0, p1);
            } else {
              p0 = fast_exp2(x0);
              p1 = fast_exp2(x1);
            }
            acc[c % 4] = f2_add(acc[c % 4], f2_pack(p0, p1));
            pk[c] = pack_bf16x2(p0, p1);
            if constexpr (kSplit)
              pl[c] = pack_bf16x2(p0 - bf16lo_to_f32(pk[c]), p1 - bf16hi_to_f32(pk[c]));
          }
          float a0, a1, a2, a3, a4, a5, a6, a7;
          f2_unpack(acc[0], a0, a1);
          f2_unpack(acc[1], a2, a3);
          f2_unpack(acc[2], a4, a5);
          f2_unpack(acc[3], a6, a7);
          rowsum = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p0 = fast_exp2(s[2 * c] - m_use);
            const float p1 = fast_exp2(s[2 * c + 1] - m_use);
            rowsum += p0 + p1;
            pk[c] = pack_bf16x2(p0, p1);
            if constexpr (kSplit)
              pl[c] = pack_bf16x2(p0 - bf16lo_to_f32(pk[c]), p1 - bf16hi_to_f32(pk[c]));
          }
        }
        l_run = l_run * factor + rowsum;
        // O_half correction, after this half's P V of the previous tile has
        // finished (warp-collective; rare with the lazy threshold).
        const bool need_corr = (n > 0) && (factor != 1.0f);
        if (__any_sync(0xffffffffu, need_corr)) {
          failed = !__all_sync(0xffffffffu, mbar_wait(bar_o_prog + half, (g - 1) & 1,
                                                      abort_flag, 32 + half));
          if (failed) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o[16];
            const uint32_t oa = lane_addr + Cfg::col_o(half) + c * 16;
            ENL_TMEM_LD16(oa, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
            ENL_TMEM_ST16(oa, o);
          }
        }
        // Publish this half of P over its own first 32 S columns.
        ENL_TMEM_ST32(s_addr, pk, 0);
        if constexpr (kSplit) ENL_TMEM_ST32(s_addr + 32, pl, 0);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_p_ready + 2 * buf + half);
      }

      // ----------------------------------------------------------- epilogue
      if (lane == 0 && t + (int)gridDim.x < p.n_items)
        slots[(k + 1) & 1] = work_item<kMode>(p, t + gridDim.x);
      const WorkItem we = slots[k & 1];
      const int erow = we.r0 + rloc;
      // Merge the two halves by log-sum-exp: only the half(s) with the
      // fewest -1e9 terms count (tier mode), scaled to a common maximum.
      // Each thread then writes D/2 output columns of its row from both
      // accumulators. Every softmax thread passes both barriers once per
      // item, failed or not, so the named barriers always match up.
      x_m[half * 128 + rloc] = m_run;
      x_l[half * 128 + rloc] = l_run;
      x_t[half * 128 + rloc] = tier;
      named_bar_sync(1, 256);
      const float m0 = x_m[rloc], m1 = x_m[128 + rloc];
      const float l0 = x_l[rloc], l1 = x_l[128 + rloc];
      const bool etiers = p.additive && !we.safe;
      const int t0 = etiers ? x_t[rloc] : 0, t1 = etiers ? x_t[128 + rloc] : 0;
      named_bar_sync(1, 256);  // the exchange may be rewritten by the next item
      const int tfin = min(t0, t1);
      const bool use0 = (t0 == tfin) && (m0 != -INFINITY);
      const bool use1 = (t1 == tfin) && (m1 != -INFINITY);
      const float mfin = fmaxf(use0 ? m0 : -INFINITY, use1 ? m1 : -INFINITY);
      const float w0 = use0 ? exp2f(m0 - mfin) : 0.0f;
      const float w1 = use1 ? exp2f(m1 - mfin) : 0.0f;
      const float l_tot = w0 * l0 + w1 * l1;
      const bool row_valid = erow < p.Sq;
      const bool have_o = we.lo < we.hi;
      bool ok = __all_sync(0xffffffffu, !failed && !*abort_flag);
      const bool warp_has_rows = __any_sync(0xffffffffu, row_valid);
      if (ok && have_o)
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o_done, wi & 1, abort_flag, 35 + half));
      const bool staged = tma_st && have_o;
      if (ok && warp_has_rows) {
        if (have_o) tc_fence_after();
        const float inv_l = 1.0f / l_tot;  // 0/0 -> NaN for rows with no key
        const float s0 = w0 * inv_l, s1 = w1 * inv_l;
        const int c0 = half * (D / 2);  // this thread's output columns [c0, c0 + D/2)
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                        ((long long)we.b * p.o_sb + (long long)erow * p.o_ss +
                         (long long)we.h * p.o_sh + c0) *
                            (p.out_fp32 ? 4 : 2);
        // Staging: the item's Q buffer in the Q tile's own 128-byte swizzled
        // layout, which the O tensor map stores from.
        uint8_t* stage = smem + Cfg::kOffQ + (wi % Cfg::kQBufs) * Cfg::kOpBytes;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {  // 16-column chunks of this thread's D/2
          uint32_t o0[16], o1[16];
          __syncwarp();  // the stores below diverge by row; reconverge for tcgen05.ld
          if (have_o)
            ENL_TMEM_LD16X2(lane_addr + Cfg::col_o(0) + c0 + c * 16, o0,
                            lane_addr + Cfg::col_o(1) + c0 + c * 16, o1);
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            v[i] = (have_o && l_tot != 0.0f)
                       ? fmaf(__uint_as_float(o0[i]), s0, __uint_as_float(o1[i]) * s1)
                       : NAN;
          const int col0 = c0 + c * 16;
          if (staged) {
            const int atom = col0 / 64;
            const int chunk = (col0 % 64) / 8;  // 16-byte chunk within the 128-byte row
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              uint4* dst = reinterpret_cast<uint4*>(
                  stage + atom * Cfg::kAtomBytes + rloc * 128 + (((chunk + i) ^ (rloc & 7)) << 4));
              *dst = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]),
                                pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                pack_bf16x2(v[8 * i + 4], v[8 * i + 5]),
                                pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
            }
          } else if (row_valid && p.out_fp32) {
            // Columns past the tensors' head dim are TMA zero fill: not stored.
            float4* dst = reinterpret_cast<float4*>(orow + c * 16 * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (col0 + 4 * i + 4 <= p.d_real)
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else if (row_valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 16 * 2);
#pragma unroll
            for (int i = 0; i < 2; ++i)
              if (col0 + 8 * i + 8 <= p.d_real)
                dst[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]),
                                    pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                    pack_bf16x2(v[8 * i + 4], v[8 * i + 5]),
                                    pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
          }
        }
        if (p.lse != nullptr && row_valid && half == 0) {
          float lse = have_o ? (mfin + log2f(l_tot)) * 0.6931471805599453f : NAN;
          if (etiers && tfin > 0) lse -= 1e9f * (float)tfin;
          p.lse[((long long)we.b * p.H + we.h) * p.Sq + erow] = lse;
        }
      }
      if (staged) {
        // Every softmax warp reports once per item, whether or not it had
        // rows to write, so the store warp's count always completes.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_stage_full);
      }
      if (have_o) {
        // O has been read (or will not be): the next item's first P V may
        // overwrite it.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_o_free);
        ++wi;
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

template <int D, bool kSplit>
cudaError_t launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const CUtensorMap& to, const PrefillParams& p, cudaStream_t stream) {
  using Cfg = PrefillCfg<D, kSplit>;
  static bool configured[64] = {};  // per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    e = cudaFuncSetAttribute(attn_prefill_sm100<D, kSplit, kModeDense>, a, Cfg::kSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_prefill_sm100<D, kSplit, kModeSparse>, a, Cfg::kSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_prefill_sm100<D, kSplit, kModeKeyMask>, a, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  if (p.n_items <= 0) return cudaSuccess;
  const int grid = min(p.n_items, p.n_ctas);
  if (p.sp_ptr != nullptr)
    attn_prefill_sm100<D, kSplit, kModeSparse>
        <<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tq, tk, tv, to, p);
  else if (p.kv_mask != nullptr)
    attn_prefill_sm100<D, kSplit, kModeKeyMask>
        <<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tq, tk, tv, to, p);
  else
    attn_prefill_sm100<D, kSplit, kModeDense>
        <<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tq, tk, tv, to, p);
  return cudaGetLastError();
}

// Per (batch row, query tile) key-tile range under an arbitrary key mask.
// One thread per query row finds the first and last real key inside its
// causal/window interval; the block reduces them to the tile's range
// [lo, hi) and to `safe` (every row of the tile has an unmasked key). A tile
// with a fully masked row under the additive rule visits every key tile: its
// surviving scores (those with the fewest -1e9 terms) may lie anywhere.
__global__ void __launch_bounds__(128) mask_tiles_kernel(const PrefillParams p, int4* tiles) {
  const int qt = blockIdx.x, b = blockIdx.y;
  const int row = qt * 128 + threadIdx.x;
  const int lkey = p.kv_len != nullptr ? max(0, min(p.kv_len[b], p.Skv)) : p.Skv;
  int first = INT_MAX, last = -1;
  bool has = true;  // rows past Sq are never stored and do not count
  if (row < p.Sq) {
    const RowBounds rb = row_bounds(p, row);
    const long long klo = max(rb.jlo, 0ll), khi = min(rb.jhi, (long long)lkey - 1);
    has = false;
    if (klo <= khi) {
      const unsigned long long* m = p.kv_mask + (long long)b * p.kv_mask_sb;
      const int w0 = (int)(klo / 64), w1 = (int)(khi / 64);
      const unsigned long long lo_bits = ~0ull << (int)(klo % 64);
      const unsigned long long hi_bits = (khi % 64 == 63) ? ~0ull : ((1ull << (khi % 64 + 1)) - 1);
      for (int wd = w0; wd <= w1; ++wd) {
        unsigned long long x = m[wd];
        if (wd == w0) x &= lo_bits;
        if (wd == w1) x &= hi_bits;
        if (x) {
          first = wd * 64 + __ffsll((long long)x) - 1;
          break;
        }
      }
      if (first != INT_MAX) {
        has = true;
        for (int wd = w1; wd >= w0; --wd) {
          unsigned long long x = m[wd];
          if (wd == w0) x &= lo_bits;
          if (wd == w1) x &= hi_bits;
          if (x) {
            last = wd * 64 + 63 - __clzll((long long)x);
            break;
          }
        }
      }
    }
  }
  __shared__ int s_first[4], s_last[4];
  const int safe = __syncthreads_and(has);
  first = __reduce_min_sync(0xffffffffu, first);
  last = __reduce_max_sync(0xffffffffu, last);
  if (threadIdx.x % 32 == 0) {
    s_first[threadIdx.x / 32] = first;
    s_last[threadIdx.x / 32] = last;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    first = min(min(s_first[0], s_first[1]), min(s_first[2], s_first[3]));
    last = max(max(s_last[0], s_last[1]), max(s_last[2], s_last[3]));
    int4 t;
    if (!safe && p.additive) {
      t.x = 0;
      t.y = (p.Skv + 127) / 128;
    } else if (last >= 0) {
      t.x = first / 128;
      t.y = last / 128 + 1;
    } else {
      t.x = t.y = 0;
    }
    t.z = safe;
    t.w = 0;
    tiles[(long long)b * gridDim.x + qt] = t;
  }
}

cudaError_t launch_mask_tiles(const PrefillParams& p, int4* tiles, cudaStream_t stream) {
  const int n_qt = (p.Sq + 127) / 128;
  mask_tiles_kernel<<<dim3(n_qt, p.B), 128, 0, stream>>>(p, tiles);
  return cudaGetLastError();
}

#define ENL_INST_PREFILL(D, S)                                                              \
  template cudaError_t launch_prefill<D, S>(const CUtensorMap&, const CUtensorMap&,          \
                                            const CUtensorMap&, const CUtensorMap&,          \
                                            const PrefillParams&, cudaStream_t);
ENL_INST_PREFILL(64, false)
ENL_INST_PREFILL(128, false)
ENL_INST_PREFILL(64, true)
ENL_INST_PREFILL(128, true)
#undef ENL_INST_PREFILL

// fp32 -> (hi, lo) bf16 planes for the split path: dst[b][s][h][plane][d],
// hi = bf16(x), lo = bf16(x - hi). Four elements per thread (16-byte load,
// two 8-byte stores).
__global__ void split_planes_kernel(const float* __restrict__ src, long long sb, long long ss,
                                    long long sh, int B, int S, int H, int D,
                                    uint16_t* __restrict__ dst) {
  const int q4 = D / 4;
  const long long total = (long long)B * S * H * q4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % q4);
    long long r = i / q4;
    const int h = (int)(r % H);
    r /= H;
    const int s = (int)(r % S);
    const int b = (int)(r / S);
    const float4 x = *reinterpret_cast<const float4*>(src + b * sb + s * ss + h * sh + 4 * c);
    const uint32_t h01 = pack_bf16x2(x.x, x.y), h23 = pack_bf16x2(x.z, x.w);
    const uint32_t l01 = pack_bf16x2(x.x - bf16lo_to_f32(h01), x.y - bf16hi_to_f32(h01));
    const uint32_t l23 = pack_bf16x2(x.z - bf16lo_to_f32(h23), x.w - bf16hi_to_f32(h23));
    uint16_t* row = dst + (((long long)b * S + s) * H + h) * 2 * D + 4 * c;
    *reinterpret_cast<uint2*>(row) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(row + D) = make_uint2(l01, l23);
  }
}

cudaError_t launch_split_planes(const float* src, long long sb, long long ss, long long sh, int B,
                                int S, int H, int D, void* dst, cudaStream_t stream) {
  const long long total = (long long)B * S * H * (D / 4);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = min((total + threads - 1) / threads, 148ll * 16);
  split_planes_kernel<<<(int)blocks, threads, 0, stream>>>(src, sb, ss, sh, B, S, H, D,
                                                           reinterpret_cast<uint16_t*>(dst));
  return cudaGetLastError();
}

}  // namespace enl
