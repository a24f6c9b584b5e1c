// K5: attention backward on tcgen05 (nn/flash_attention.py:83-114).
//
// The reference recomputes each score block from Q and K, turns it into the
// forward's probabilities with the saved row statistics, and accumulates
//   dV += P^T dO,  dP = dO V^T,  dS = P * (dP - D) * scale,
//   dQ += dS K,    dK += dS^T Q,  with D = rowsum(dO * O).
// Here that is three launches:
//   bwd_prep_kernel       D per query row and LSE in log2 units, padded to
//                         whole 128-row tiles (pad rows: LSE +inf, so P = 0);
//   attn_bwd_dkdv_sm100   one CTA per (batch, kv head, 128-key tile): K and V
//                         stay in shared memory while the query tiles of
//                         every query head of the group stream through;
//                         S^T = K Q^T and dP^T = V dO^T in tensor memory,
//                         P^T and dS^T written back over dP^T as bf16, then
//                         dV += P^T dO and dK += dS^T Q accumulate in tensor
//                         memory (GQA sums the group's heads exactly there);
//   attn_bwd_dq_sm100     one CTA per (batch, head, 128-query tile): Q and dO
//                         stay, K and V stream; S and dP again, dS over dP,
//                         dQ += dS K in tensor memory.
// Both kernels end by staging the accumulator rows in shared memory and
// storing whole rows.
// Tensor memory per CTA: S (128 columns) + dP (128) + two D-column
// accumulators, 512 columns at D = 128: no room for a second S. Instead each
// tile is split into two 64-column halves with their own barriers. The
// elementwise warps read a half's dP whole, then write the packed bf16 P and
// dS of the half over its dP columns, so its S columns are free as soon as
// they are done: the next tile's S of that half is issued right behind this
// tile's accumulation, and only its dP waits for the accumulation to have
// read P and dS. The tensor pipe works while the other half's elementwise
// warps run. Recomputing S and dP in the dQ pass costs two GEMMs of seven but
// needs no atomics and no dQ staging.
//
// fp32 inputs (split mode, head dim <= 64): every operand arrives as bf16
// hi and lo planes (x = hi + lo, lo = bf16(x - hi)) and every product takes
// three MMAs, hi*hi + hi*lo + lo*hi, as K1's split mode does. P^T, dS^T (dS
// in the dQ pass) are split the same way: their hi halves go over dP as in
// the bf16 path, their lo halves into the 128 tensor-memory columns that a
// 64-wide head leaves free. Shared memory holds twice the tiles (195 KB).
//
// Warp roles (320 threads): 0-7 elementwise (warps w and w + 4 share TMEM
// lanes 32 (w % 4) .. + 31 and split the 128 columns in halves), 8 TMA, 9 MMA.
// Every wait is bounded (mbar_wait): on timeout a device error is recorded
// and every role stops issuing and drains.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

// 1-D bulk copy global -> shared (no multicast), completing on an mbarrier.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int D, bool kSplit>
struct BwdCfg {
  static constexpr int kThreads = 320;
  static constexpr int kPlanes = kSplit ? 2 : 1;
  static constexpr int kAtoms = D / 64;
  static constexpr int kAtomBytes = 128 * 128;
  static constexpr int kTileBytes = 128 * D * 2;          // one plane of one operand tile
  static constexpr int kOpBytes = kPlanes * kTileBytes;  // all planes of one operand tile
  static constexpr int kStages = 2;
  static constexpr int kOffRes = 0;                        // resident pair of operand tiles
  static constexpr int kOffStr = 2 * kOpBytes;             // streamed pairs [kStages][2]
  static constexpr int kOffRow = kOffStr + kStages * 2 * kOpBytes;  // [kStages][2][128] f32
  static constexpr int kOffBar = kOffRow + kStages * 2 * 128 * 4;
  // res_full, full[kStages], empty[kStages], s_full[2], p_ready[2], done[2], drain
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static constexpr uint32_t kColS = 0, kColDP = 128, kColAcc0 = 256, kColAcc1 = 256 + D;
  // Split mode: lo halves of the packed P^T / dS^T (dS) of half h at kColLo + 64 h.
  static constexpr uint32_t kColLo = 256 + 2 * D;
  static_assert(!kSplit || kColLo + 128 <= 512, "split mode needs 128 free TMEM columns");
  static constexpr uint32_t kLoPlane = kTileBytes >> 4;  // lo plane, descriptor units
};

// bf16 pair (a0, a1) into hi[i]; split mode adds the remainders' pair to lo[i].
template <bool kSplit>
__device__ __forceinline__ void put_pair(uint32_t* hi, uint32_t* lo, int i, float a0, float a1) {
  hi[i] = pack_bf16x2(a0, a1);
  if constexpr (kSplit)
    lo[i] = pack_bf16x2(a0 - bf16lo_to_f32(hi[i]), a1 - bf16hi_to_f32(hi[i]));
}

// Query-tile range [lo, hi) that can see key tile kt, and key-tile range that
// query tile qt can see (causal: key <= query; window: |query - key| <= w).
__device__ __forceinline__ void q_range_for_key_tile(const BwdParams& p, int kt, int& lo,
                                                     int& hi) {
  const int n_qt = (p.Sq + 127) / 128;
  const long long j0 = (long long)kt * 128, j1 = min((long long)p.Skv, j0 + 128) - 1;
  long long ilo = 0, ihi = (long long)p.Sq - 1;
  if (p.causal) ilo = max(ilo, j0);
  if (p.window >= 0) {
    ilo = max(ilo, j0 - p.window);
    ihi = min(ihi, j1 + p.window);
  }
  lo = (int)(ilo / 128);
  hi = (ihi < ilo) ? lo : (int)min((long long)n_qt, ihi / 128 + 1);
}

__device__ __forceinline__ void k_range_for_query_tile(const BwdParams& p, int qt, int& lo,
                                                       int& hi) {
  const int n_kt = (p.Skv + 127) / 128;
  const long long i0 = (long long)qt * 128, i1 = min((long long)p.Sq, i0 + 128) - 1;
  long long jlo = 0, jhi = (long long)p.Skv - 1;
  if (p.causal) jhi = min(jhi, i1);
  if (p.window >= 0) {
    jlo = max(jlo, i0 - p.window);
    jhi = min(jhi, i1 + p.window);
  }
  lo = (int)(jlo / 128);
  hi = (jhi < jlo) ? lo : (int)min((long long)n_kt, jhi / 128 + 1);
}

// P and dS of one (query i, key j) score, from the raw dot product s and the
// raw dO.v product dp. lse2 and dsum belong to the query row.
__device__ __forceinline__ void bwd_elem(const BwdParams& p, float s, float dp, long long i,
                                         long long j, float slope2, float lse2, float dsum,
                                         float& pr, float& ds) {
  const long long diff = i - j;
  bool ok = j < p.Skv && (!p.causal || diff >= 0);
  if (p.window >= 0) ok = ok && (diff <= p.window && -diff <= p.window);
  const float dist = p.causal ? (float)diff : fabsf((float)diff);
  const float x = fmaf(s, p.scale_log2, -slope2 * dist) - lse2;
  pr = ok ? fast_exp2(x) : 0.0f;
  ds = pr * (dp - dsum);
}

// One 16-lane group per query row. With bf16 O, 16-byte aligned rows and a
// head dim that is a multiple of 8, each lane reads 8 elements of O and dO
// per 16-byte load; otherwise one element at a time.
__global__ void bwd_prep_kernel(BwdPrepParams q) {
  const int sub = threadIdx.x % 16;
  const long long groups = (long long)gridDim.x * (blockDim.x / 16);
  const long long total = (long long)q.B * q.H * q.s_pad;
  const __nv_bfloat16* dob = reinterpret_cast<const __nv_bfloat16*>(q.dout);
  const float* dof = reinterpret_cast<const float*>(q.dout);
  const bool vec = !q.o_f32 && !q.do_f32 && q.d_real % 8 == 0 && q.o_sb % 8 == 0 && q.o_ss % 8 == 0 &&
                   q.o_sh % 8 == 0 && (reinterpret_cast<uintptr_t>(q.o) & 15u) == 0;
  for (long long idx = blockIdx.x * (long long)(blockDim.x / 16) + threadIdx.x / 16; idx < total;
       idx += groups) {
    const long long bh = idx / q.s_pad;
    const int i = (int)(idx % q.s_pad);
    const int b = (int)(bh / q.H), h = (int)(bh % q.H);
    float acc = 0.0f;
    if (i < q.Sq) {
      const long long oo = b * q.o_sb + (long long)i * q.o_ss + h * q.o_sh;
      const long long od = b * q.do_sb + (long long)i * q.do_ss + h * q.do_sh;
      if (vec) {
        const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(q.o);
        for (int d = 8 * sub; d < q.d_real; d += 128) {
          const uint4 x = *reinterpret_cast<const uint4*>(ob + oo + d);
          const uint4 y = *reinterpret_cast<const uint4*>(dob + od + d);
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            acc = fmaf(bf16lo_to_f32(xs[k]), bf16lo_to_f32(ys[k]), acc);
            acc = fmaf(bf16hi_to_f32(xs[k]), bf16hi_to_f32(ys[k]), acc);
          }
        }
      } else {
        for (int d = sub; d < q.d_real; d += 16) {
          const float o = q.o_f32 ? reinterpret_cast<const float*>(q.o)[oo + d]
                                  : __bfloat162float(
                                        reinterpret_cast<const __nv_bfloat16*>(q.o)[oo + d]);
          acc = fmaf(o, q.do_f32 ? dof[od + d] : __bfloat162float(dob[od + d]), acc);
        }
      }
    }
    const unsigned group = 0xffffu << (16 * ((threadIdx.x % 32) / 16));  // this 16-lane half
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) acc += __shfl_xor_sync(group, acc, m);
    if (sub == 0) {
      q.dsum[idx] = i < q.Sq ? acc : 0.0f;
      q.lse2[idx] = i < q.Sq ? q.lse[bh * q.Sq + i] * 1.4426950408889634f : INFINITY;
    }
  }
}

// Epilogue staging: accumulator rows in shared memory at a stride of D + 4
// floats, so rows stay 16-byte aligned and a warp's float4 writes (one row
// per lane) are conflict-free per quarter warp.
template <int D>
__device__ __forceinline__ void stage_row16(float* stg, int rloc, int col0,
                                            const uint32_t (&a)[16], float mul, bool have) {
  float4* dst = reinterpret_cast<float4*>(stg + rloc * (D + 4) + col0);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    dst[k] = have ? make_float4(__uint_as_float(a[4 * k]) * mul, __uint_as_float(a[4 * k + 1]) * mul,
                                __uint_as_float(a[4 * k + 2]) * mul,
                                __uint_as_float(a[4 * k + 3]) * mul)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
}

// Staged rows [0, nrows) to base + r * ss, d_real columns each, one row per
// warp step: float4 per lane when the outputs are 16-byte aligned (vec4),
// else one float per lane.
template <int D>
__device__ __forceinline__ void store_rows(const float* stg, float* base, long long ss, int nrows,
                                           int d_real, bool vec4, int warp, int lane) {
  if (vec4) {
#pragma unroll 4
    for (int r = warp; r < nrows; r += 8)
      for (int c4 = lane; c4 < d_real / 4; c4 += 32)
        *reinterpret_cast<float4*>(base + r * ss + 4 * c4) =
            *reinterpret_cast<const float4*>(stg + r * (D + 4) + 4 * c4);
  } else {
    for (int r = warp; r < nrows; r += 8)
      for (int c = lane; c < d_real; c += 32) base[r * ss + c] = stg[r * (D + 4) + c];
  }
}

// ---------------------------------------------------------------------------
// dK, dV. CTA c -> key tile c / (B * Hkv) (small tiles first: under a causal
// mask they see the most query tiles), (b, kv head) c % (B * Hkv).
// ---------------------------------------------------------------------------
template <int D, bool kSplit>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dkdv_sm100(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_do, const BwdParams p) {
  using Cfg = BwdCfg<D, kSplit>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* rows = reinterpret_cast<float*>(smem + Cfg::kOffRow);  // [stage][lse2 | dsum][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* bar_res = bars;
  uint64_t* bar_full = bar_res + 1;
  uint64_t* bar_empty = bar_full + Cfg::kStages;
  uint64_t* bar_s_full = bar_empty + Cfg::kStages;  // [2 halves]
  uint64_t* bar_p_ready = bar_s_full + 2;           // [2 halves], 4 warps each
  uint64_t* bar_done = bar_p_ready + 2;             // [2 halves] accumulation read P, dS
  uint64_t* bar_drain = bar_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_bk = p.B * p.Hkv;
  const int kt = blockIdx.x / n_bk;
  const int bk = blockIdx.x % n_bk;
  const int b = bk / p.Hkv, hkv = bk % p.Hkv;
  const int G = p.H / p.Hkv;
  int qlo, qhi;
  q_range_for_key_tile(p, kt, qlo, qhi);
  const int nq = max(0, qhi - qlo);
  const int n_units = G * nq;  // unit u: head hkv * G + u / nq, query tile qlo + u % nq

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kNumBars; ++i)
      mbar_init(bars + i, (bars + i == bar_p_ready || bars + i == bar_p_ready + 1) ? 4u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc<512>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0 && n_units > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      // Split mode: plane pl of head h is "head" kPlanes * h + pl of the maps.
      mbar_arrive_expect_tx(bar_res, 2 * Cfg::kOpBytes);
      for (int pl = 0; pl < Cfg::kPlanes; ++pl)
        for (int a = 0; a < Cfg::kAtoms; ++a) {
          uint8_t* dst = smem + Cfg::kOffRes + pl * Cfg::kTileBytes + a * Cfg::kAtomBytes;
          const int hp = Cfg::kPlanes * hkv + pl;
          tma_load_4d(dst, &tm_k, bar_res, a * 64, kt * 128, hp, b);
          tma_load_4d(dst + Cfg::kOpBytes, &tm_v, bar_res, a * 64, kt * 128, hp, b);
        }
      int issued = 0;
      bool ok = true;
      for (int u = 0; u < n_units; ++u) {
        const int st = u % Cfg::kStages;
        const int h = hkv * G + u / nq, qt = qlo + u % nq;
        if (u >= Cfg::kStages) ok = mbar_wait(bar_empty + st, (u / Cfg::kStages - 1) & 1,
                                              abort_flag, 80);
        if (!ok) break;
        uint8_t* dst = smem + Cfg::kOffStr + st * 2 * Cfg::kOpBytes;
        mbar_arrive_expect_tx(bar_full + st, 2 * Cfg::kOpBytes + 2 * 512);
        for (int pl = 0; pl < Cfg::kPlanes; ++pl)
          for (int a = 0; a < Cfg::kAtoms; ++a) {
            uint8_t* d2 = dst + pl * Cfg::kTileBytes + a * Cfg::kAtomBytes;
            const int hp = Cfg::kPlanes * h + pl;
            tma_load_4d(d2, &tm_q, bar_full + st, a * 64, qt * 128, hp, b);
            tma_load_4d(d2 + Cfg::kOpBytes, &tm_do, bar_full + st, a * 64, qt * 128, hp, b);
          }
        const long long roff = ((long long)b * p.H + h) * p.s_pad + (long long)qt * 128;
        bulk_load_1d(rows + st * 256, p.lse2 + roff, 512, bar_full + st);
        bulk_load_1d(rows + st * 256 + 128, p.dsum + roff, 512, bar_full + st);
        ++issued;
      }
      // Every issued load lands before the CTA may exit (bounded waits).
      volatile int no_abort = 0;
      mbar_wait(bar_res, 0, &no_abort, 81);
      for (int n = max(0, issued - Cfg::kStages); n < issued; ++n)
        mbar_wait(bar_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 82);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA
    const uint32_t idesc_s = idesc_bf16_f32(128, 64, false);  // one 64-query half
    const uint32_t idesc_o = idesc_bf16_f32(128, D, true);
    const uint32_t k_lo = desc_lo(smem_u32(smem + Cfg::kOffRes), 16);
    const uint32_t v_lo = k_lo + (Cfg::kOpBytes >> 4);
    constexpr uint32_t kLo = Cfg::kLoPlane;
    auto wait = [&](uint64_t* bar, uint32_t parity, int site) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site));
    };
    auto stage = [&](int u) {
      return smem_u32(smem + Cfg::kOffStr + (u % Cfg::kStages) * 2 * Cfg::kOpBytes);
    };
    // S^T and dP^T of query half h of unit u: K Q_h^T and V dO_h^T, where
    // Q_h / dO_h are rows 64h.. of the streamed tiles (64 rows x 128 bytes
    // into each swizzle atom).
    auto issue_s = [&](int u, int h) {
      const uint32_t q_k = desc_lo(stage(u), 16) + h * (8192 >> 4);
      const uint32_t ds = tmem + Cfg::kColS + 64 * h;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk / 4) * (Cfg::kAtomBytes >> 4) + (kk % 4) * 2;
        if (kk == 0)
          umma_ss_elect<false>(ds, k_lo + off, q_k + off, kDescHiSw128, idesc_s);
        else
          umma_ss_elect<true>(ds, k_lo + off, q_k + off, kDescHiSw128, idesc_s);
        if constexpr (kSplit) {
          umma_ss_elect<true>(ds, k_lo + off, q_k + kLo + off, kDescHiSw128, idesc_s);
          umma_ss_elect<true>(ds, k_lo + kLo + off, q_k + off, kDescHiSw128, idesc_s);
        }
      }
    };
    auto issue_dp = [&](int u, int h) {
      const uint32_t o_k = desc_lo(stage(u), 16) + h * (8192 >> 4) + (Cfg::kOpBytes >> 4);
      const uint32_t dp = tmem + Cfg::kColDP + 64 * h;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk / 4) * (Cfg::kAtomBytes >> 4) + (kk % 4) * 2;
        if (kk == 0)
          umma_ss_elect<false>(dp, v_lo + off, o_k + off, kDescHiSw128, idesc_s);
        else
          umma_ss_elect<true>(dp, v_lo + off, o_k + off, kDescHiSw128, idesc_s);
        if constexpr (kSplit) {
          umma_ss_elect<true>(dp, v_lo + off, o_k + kLo + off, kDescHiSw128, idesc_s);
          umma_ss_elect<true>(dp, v_lo + kLo + off, o_k + off, kDescHiSw128, idesc_s);
        }
      }
      umma_commit_elect(bar_s_full + h);  // S and dP of the half
    };
    // dV += P^T_h dO_h, dK += dS^T_h Q_h (K = the half's 64 queries); P^T_h and
    // dS^T_h are packed over the half's dP columns (first and second 32).
    auto issue_acc = [&](int u, int h) {
      const uint32_t q_mn = desc_lo(stage(u), Cfg::kAtomBytes);
      const uint32_t o_mn = q_mn + (Cfg::kOpBytes >> 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t boff = (h * 4 + kk) * (2048 >> 4);  // 16 query rows per step
        const uint32_t acc = (u > 0 || h > 0 || kk > 0) ? 1u : 0u;
        const uint32_t p_hi = tmem + Cfg::kColDP + h * 64 + kk * 8;
        const uint32_t s_hi = p_hi + 32;
        umma_ts_elect(tmem + Cfg::kColAcc0, p_hi, o_mn + boff, kDescHiSw128, idesc_o, acc);
        umma_ts_elect(tmem + Cfg::kColAcc1, s_hi, q_mn + boff, kDescHiSw128, idesc_o, acc);
        if constexpr (kSplit) {
          const uint32_t p_lo = tmem + Cfg::kColLo + h * 64 + kk * 8;
          const uint32_t s_lo = p_lo + 32;
          umma_ts_elect(tmem + Cfg::kColAcc0, p_hi, o_mn + kLo + boff, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(tmem + Cfg::kColAcc0, p_lo, o_mn + boff, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(tmem + Cfg::kColAcc1, s_hi, q_mn + kLo + boff, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(tmem + Cfg::kColAcc1, s_lo, q_mn + boff, kDescHiSw128, idesc_o, 1u);
        }
      }
      umma_commit_elect(bar_done + h);
      if (h == 1) umma_commit_elect(bar_empty + u % Cfg::kStages);  // Q, dO of u read
    };
    bool ok = n_units == 0 || wait(bar_res, 0, 83);
    if (ok && n_units > 0) {
      ok = wait(bar_full, 0, 84);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          issue_s(0, h);
          issue_dp(0, h);
        }
      }
    }
    for (int u = 0; ok && u < n_units; ++u) {
      for (int h = 0; h < 2 && ok; ++h) {
        ok = wait(bar_p_ready + h, u & 1, 86 + h);
        if (!ok) break;
        tc_fence_after();
        issue_acc(u, h);
        if (u + 1 < n_units) {
          if (h == 0) ok = wait(bar_full + (u + 1) % Cfg::kStages,
                                ((u + 1) / Cfg::kStages) & 1, 84);
          if (!ok) break;
          issue_s(u + 1, h);  // the half's S columns were read by the elementwise warps
          ok = wait(bar_done + h, u & 1, 85);  // packed P^T_h, dS^T_h read
          if (!ok) break;
          tc_fence_after();
          issue_dp(u + 1, h);
        }
      }
    }
    umma_commit_elect(bar_drain);
    volatile int no_abort = 0;
    mbar_wait(bar_drain, 0, &no_abort, 88);
  } else {
    // ---------------------------------------------------------- elementwise
    const int half = warp / 4, quarter = warp % 4;
    const int rloc = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const long long j = (long long)kt * 128 + rloc;  // this row's key
    bool failed = false;
    for (int u = 0; u < n_units && !failed; ++u) {
      const int st = u % Cfg::kStages;
      const int h = hkv * G + u / nq, qt = qlo + u % nq;
      const float slope2 = p.alibi ? p.alibi[h] * 1.4426950408889634f : 0.0f;
      failed = !__all_sync(0xffffffffu, mbar_wait(bar_full + st, (u / Cfg::kStages) & 1,
                                                  abort_flag, 89));
      if (!failed)
        failed = !__all_sync(0xffffffffu,
                             mbar_wait(bar_s_full + half, u & 1, abort_flag, 90 + half));
      if (failed) break;
      tc_fence_after();
      const float* lse2 = rows + st * 256;
      const float* dsum = lse2 + 128;
      // The half's dP first (all 64 columns, so the packed P and dS can go
      // over them), then S 32 columns at a time.
      uint32_t dph[64];
      ENL_TMEM_LD32X2(lane_addr + Cfg::kColDP + 64 * half, dph,
                      lane_addr + Cfg::kColDP + 64 * half + 32, (dph + 32));
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        const int c0 = 64 * half + 32 * ch;  // first query column of the chunk
        uint32_t sr[32], pk[16], dk[16];
        uint32_t pl[kSplit ? 16 : 1], dl[kSplit ? 16 : 1];  // split mode: lo halves
        const uint32_t* dr = dph + 32 * ch;
        ENL_TMEM_LD32(lane_addr + Cfg::kColS + c0, sr, 0);
        const long long i0 = (long long)qt * 128 + c0;
        // Every (query, key) of the chunk visible and no bias: P needs only
        // the column's LSE (queries past Sq carry +inf there, so P = 0).
        const bool open = slope2 == 0.0f && j < p.Skv && (!p.causal || j <= i0) &&
                          (p.window < 0 || (i0 + 31 - j <= p.window && j - i0 <= p.window));
        if (open) {
          const float4* l4 = reinterpret_cast<const float4*>(lse2 + c0);
          const float4* d4 = reinterpret_cast<const float4*>(dsum + c0);
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            const float4 L = l4[c / 4], Dd = d4[c / 4];
            const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c]), p.scale_log2, -L.x));
            const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c + 1]), p.scale_log2, -L.y));
            const float p2 = fast_exp2(fmaf(__uint_as_float(sr[c + 2]), p.scale_log2, -L.z));
            const float p3 = fast_exp2(fmaf(__uint_as_float(sr[c + 3]), p.scale_log2, -L.w));
            put_pair<kSplit>(pk, pl, c / 2, p0, p1);
            put_pair<kSplit>(pk, pl, c / 2 + 1, p2, p3);
            put_pair<kSplit>(dk, dl, c / 2, p0 * (__uint_as_float(dr[c]) - Dd.x),
                             p1 * (__uint_as_float(dr[c + 1]) - Dd.y));
            put_pair<kSplit>(dk, dl, c / 2 + 1, p2 * (__uint_as_float(dr[c + 2]) - Dd.z),
                             p3 * (__uint_as_float(dr[c + 3]) - Dd.w));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float p0, p1, d0, d1;
            bwd_elem(p, __uint_as_float(sr[c]), __uint_as_float(dr[c]), i0 + c, j, slope2,
                     lse2[c0 + c], dsum[c0 + c], p0, d0);
            bwd_elem(p, __uint_as_float(sr[c + 1]), __uint_as_float(dr[c + 1]), i0 + c + 1, j,
                     slope2, lse2[c0 + c + 1], dsum[c0 + c + 1], p1, d1);
            put_pair<kSplit>(pk, pl, c / 2, p0, p1);
            put_pair<kSplit>(dk, dl, c / 2, d0, d1);
          }
        }
        // packed P^T over the half's first 32 dP columns, dS^T over the last 32
        ENL_TMEM_ST16(lane_addr + Cfg::kColDP + 64 * half + 16 * ch, pk);
        ENL_TMEM_ST16(lane_addr + Cfg::kColDP + 64 * half + 32 + 16 * ch, dk);
        if constexpr (kSplit) {
          ENL_TMEM_ST16(lane_addr + Cfg::kColLo + 64 * half + 16 * ch, pl);
          ENL_TMEM_ST16(lane_addr + Cfg::kColLo + 64 * half + 32 + 16 * ch, dl);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_ready + half);
    }
    // Epilogue: dV, then dK (times the softmax scale). Each thread moves its
    // row's half of the accumulator into shared memory (the streamed stages
    // are free once the last accumulation completed; rows padded to D + 1
    // floats, so the row-per-lane writes hit distinct banks), then each warp
    // stores whole rows, 128 contiguous bytes per instruction. Every
    // elementwise thread passes both barriers of both passes, failed or not.
    bool ok = __all_sync(0xffffffffu, !failed && !*abort_flag);
    if (ok && n_units > 0)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar_done, (n_units - 1) & 1, abort_flag, 92) &&
                          mbar_wait(bar_done + 1, (n_units - 1) & 1, abort_flag, 93));
    float* stg = reinterpret_cast<float*>(smem + Cfg::kOffStr);  // [128][D + 4]
#pragma unroll 1
    for (int arr = 0; arr < 2; ++arr) {
      if (ok) {
        tc_fence_after();
        const uint32_t col_acc = arr ? Cfg::kColAcc1 : Cfg::kColAcc0;
        const float mul = arr ? p.scale : 1.0f;
#pragma unroll 1
        for (int c = 0; c < D / 2; c += 16) {
          const int col0 = half * (D / 2) + c;
          uint32_t av[16];
          __syncwarp();
          if (n_units > 0) ENL_TMEM_LD16(lane_addr + col_acc + col0, av);
          stage_row16<D>(stg, rloc, col0, av, mul, n_units > 0);
        }
      }
      named_bar_sync(1, 256);
      if (ok) {
        const long long ss = arr ? p.dk_ss : p.dv_ss;
        float* base = arr ? p.dk + b * p.dk_sb + hkv * p.dk_sh : p.dv + b * p.dv_sb + hkv * p.dv_sh;
        store_rows<D>(stg, base + (long long)kt * 128 * ss, ss, min(128, p.Skv - kt * 128),
                      p.d_real, p.out_vec4 != 0, warp, lane);
      }
      named_bar_sync(1, 256);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ---------------------------------------------------------------------------
// dQ. CTA c -> query tile (last first: under a causal mask it sees the most
// key tiles), (b, head) c % (B * H).
// ---------------------------------------------------------------------------
template <int D, bool kSplit>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dq_sm100(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_do, const BwdParams p) {
  using Cfg = BwdCfg<D, kSplit>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* bar_res = bars;
  uint64_t* bar_full = bar_res + 1;
  uint64_t* bar_empty = bar_full + Cfg::kStages;
  uint64_t* bar_s_full = bar_empty + Cfg::kStages;  // [2 halves]
  uint64_t* bar_p_ready = bar_s_full + 2;
  uint64_t* bar_done = bar_p_ready + 2;
  uint64_t* bar_drain = bar_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_bh = p.B * p.H;
  const int n_qt = (p.Sq + 127) / 128;
  const int qt = n_qt - 1 - (int)(blockIdx.x / n_bh);
  const int bh = blockIdx.x % n_bh;
  const int b = bh / p.H, h = bh % p.H;
  const int hkv = h / (p.H / p.Hkv);
  int klo, khi;
  k_range_for_query_tile(p, qt, klo, khi);
  const int n_units = max(0, khi - klo);  // unit u: key tile klo + u

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kNumBars; ++i)
      mbar_init(bars + i, (bars + i == bar_p_ready || bars + i == bar_p_ready + 1) ? 4u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc<512>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0 && n_units > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(bar_res, 2 * Cfg::kOpBytes);
      for (int pl = 0; pl < Cfg::kPlanes; ++pl)
        for (int a = 0; a < Cfg::kAtoms; ++a) {
          uint8_t* dst = smem + Cfg::kOffRes + pl * Cfg::kTileBytes + a * Cfg::kAtomBytes;
          const int hp = Cfg::kPlanes * h + pl;
          tma_load_4d(dst, &tm_q, bar_res, a * 64, qt * 128, hp, b);
          tma_load_4d(dst + Cfg::kOpBytes, &tm_do, bar_res, a * 64, qt * 128, hp, b);
        }
      int issued = 0;
      bool ok = true;
      for (int u = 0; u < n_units; ++u) {
        const int st = u % Cfg::kStages;
        const int kt = klo + u;
        if (u >= Cfg::kStages) ok = mbar_wait(bar_empty + st, (u / Cfg::kStages - 1) & 1,
                                              abort_flag, 100);
        if (!ok) break;
        uint8_t* dst = smem + Cfg::kOffStr + st * 2 * Cfg::kOpBytes;
        mbar_arrive_expect_tx(bar_full + st, 2 * Cfg::kOpBytes);
        for (int pl = 0; pl < Cfg::kPlanes; ++pl)
          for (int a = 0; a < Cfg::kAtoms; ++a) {
            uint8_t* d2 = dst + pl * Cfg::kTileBytes + a * Cfg::kAtomBytes;
            const int hp = Cfg::kPlanes * hkv + pl;
            tma_load_4d(d2, &tm_k, bar_full + st, a * 64, kt * 128, hp, b);
            tma_load_4d(d2 + Cfg::kOpBytes, &tm_v, bar_full + st, a * 64, kt * 128, hp, b);
          }
        ++issued;
      }
      volatile int no_abort = 0;
      mbar_wait(bar_res, 0, &no_abort, 101);
      for (int n = max(0, issued - Cfg::kStages); n < issued; ++n)
        mbar_wait(bar_full + n % Cfg::kStages, (n / Cfg::kStages) & 1, &no_abort, 102);
    }
    __syncwarp();
  } else if (warp == 9) {
    const uint32_t idesc_s = idesc_bf16_f32(128, 64, false);  // one 64-key half
    const uint32_t idesc_o = idesc_bf16_f32(128, D, true);
    const uint32_t q_lo = desc_lo(smem_u32(smem + Cfg::kOffRes), 16);
    const uint32_t o_lo = q_lo + (Cfg::kOpBytes >> 4);
    constexpr uint32_t kLo = Cfg::kLoPlane;
    auto wait = [&](uint64_t* bar, uint32_t parity, int site) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site));
    };
    auto stage = [&](int u) {
      return smem_u32(smem + Cfg::kOffStr + (u % Cfg::kStages) * 2 * Cfg::kOpBytes);
    };
    // S and dP of key half h of unit u: Q K_h^T and dO V_h^T.
    auto issue_s = [&](int u, int h) {
      const uint32_t k_k = desc_lo(stage(u), 16) + h * (8192 >> 4);
      const uint32_t ds = tmem + Cfg::kColS + 64 * h;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk / 4) * (Cfg::kAtomBytes >> 4) + (kk % 4) * 2;
        if (kk == 0)
          umma_ss_elect<false>(ds, q_lo + off, k_k + off, kDescHiSw128, idesc_s);
        else
          umma_ss_elect<true>(ds, q_lo + off, k_k + off, kDescHiSw128, idesc_s);
        if constexpr (kSplit) {
          umma_ss_elect<true>(ds, q_lo + off, k_k + kLo + off, kDescHiSw128, idesc_s);
          umma_ss_elect<true>(ds, q_lo + kLo + off, k_k + off, kDescHiSw128, idesc_s);
        }
      }
    };
    auto issue_dp = [&](int u, int h) {
      const uint32_t v_k = desc_lo(stage(u), 16) + h * (8192 >> 4) + (Cfg::kOpBytes >> 4);
      const uint32_t dp = tmem + Cfg::kColDP + 64 * h;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk / 4) * (Cfg::kAtomBytes >> 4) + (kk % 4) * 2;
        if (kk == 0)
          umma_ss_elect<false>(dp, o_lo + off, v_k + off, kDescHiSw128, idesc_s);
        else
          umma_ss_elect<true>(dp, o_lo + off, v_k + off, kDescHiSw128, idesc_s);
        if constexpr (kSplit) {
          umma_ss_elect<true>(dp, o_lo + off, v_k + kLo + off, kDescHiSw128, idesc_s);
          umma_ss_elect<true>(dp, o_lo + kLo + off, v_k + off, kDescHiSw128, idesc_s);
        }
      }
      umma_commit_elect(bar_s_full + h);
    };
    // dQ += dS_h K_h (K = the half's 64 keys); dS_h is packed over the half's
    // first 32 dP columns.
    auto issue_acc = [&](int u, int h) {
      const uint32_t k_mn = desc_lo(stage(u), Cfg::kAtomBytes);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t boff = (h * 4 + kk) * (2048 >> 4);  // 16 key rows per step
        const uint32_t acc = (u > 0 || h > 0 || kk > 0) ? 1u : 0u;
        const uint32_t s_hi = tmem + Cfg::kColDP + h * 64 + kk * 8;
        umma_ts_elect(tmem + Cfg::kColAcc0, s_hi, k_mn + boff, kDescHiSw128, idesc_o, acc);
        if constexpr (kSplit) {
          const uint32_t s_lo = tmem + Cfg::kColLo + h * 64 + kk * 8;
          umma_ts_elect(tmem + Cfg::kColAcc0, s_hi, k_mn + kLo + boff, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(tmem + Cfg::kColAcc0, s_lo, k_mn + boff, kDescHiSw128, idesc_o, 1u);
        }
      }
      umma_commit_elect(bar_done + h);
      if (h == 1) umma_commit_elect(bar_empty + u % Cfg::kStages);  // K, V of u read
    };
    bool ok = n_units == 0 || wait(bar_res, 0, 103);
    if (ok && n_units > 0) {
      ok = wait(bar_full, 0, 104);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          issue_s(0, h);
          issue_dp(0, h);
        }
      }
    }
    for (int u = 0; ok && u < n_units; ++u) {
      for (int h = 0; h < 2 && ok; ++h) {
        ok = wait(bar_p_ready + h, u & 1, 106 + h);
        if (!ok) break;
        tc_fence_after();
        issue_acc(u, h);
        if (u + 1 < n_units) {
          if (h == 0) ok = wait(bar_full + (u + 1) % Cfg::kStages,
                                ((u + 1) / Cfg::kStages) & 1, 104);
          if (!ok) break;
          issue_s(u + 1, h);  // the half's S columns were read by the elementwise warps
          ok = wait(bar_done + h, u & 1, 105);  // packed dS_h read
          if (!ok) break;
          tc_fence_after();
          issue_dp(u + 1, h);
        }
      }
    }
    umma_commit_elect(bar_drain);
    volatile int no_abort = 0;
    mbar_wait(bar_drain, 0, &no_abort, 108);
  } else {
    const int half = warp / 4, quarter = warp % 4;
    const int rloc = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const long long i = (long long)qt * 128 + rloc;  // this row's query
    const long long roff = (long long)bh * p.s_pad + i;
    const float lse2 = p.lse2[roff], dsum = p.dsum[roff];
    const float slope2 = p.alibi ? p.alibi[h] * 1.4426950408889634f : 0.0f;
    bool failed = false;
    for (int u = 0; u < n_units && !failed; ++u) {
      const int kt = klo + u;
      failed = !__all_sync(0xffffffffu,
                           mbar_wait(bar_s_full + half, u & 1, abort_flag, 110 + half));
      if (failed) break;
      tc_fence_after();
      uint32_t dph[64];  // the half's dP first, so the packed dS can go over it
      ENL_TMEM_LD32X2(lane_addr + Cfg::kColDP + 64 * half, dph,
                      lane_addr + Cfg::kColDP + 64 * half + 32, (dph + 32));
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        const int c0 = 64 * half + 32 * ch;  // first key column of the chunk
        uint32_t sr[32], dk[16];
        uint32_t dl[kSplit ? 16 : 1];  // split mode: lo halves
        const uint32_t* dr = dph + 32 * ch;
        ENL_TMEM_LD32(lane_addr + Cfg::kColS + c0, sr, 0);
        const long long j0 = (long long)kt * 128 + c0;
        const bool open = slope2 == 0.0f && j0 + 31 < p.Skv && (!p.causal || j0 + 31 <= i) &&
                          (p.window < 0 || (i - j0 <= p.window && j0 + 31 - i <= p.window));
        if (open) {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c]), p.scale_log2, -lse2));
            const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c + 1]), p.scale_log2, -lse2));
            put_pair<kSplit>(dk, dl, c / 2, p0 * (__uint_as_float(dr[c]) - dsum),
                             p1 * (__uint_as_float(dr[c + 1]) - dsum));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float p0, p1, d0, d1;
            bwd_elem(p, __uint_as_float(sr[c]), __uint_as_float(dr[c]), i, j0 + c, slope2, lse2,
                     dsum, p0, d0);
            bwd_elem(p, __uint_as_float(sr[c + 1]), __uint_as_float(dr[c + 1]), i, j0 + c + 1,
                     slope2, lse2, dsum, p1, d1);
            put_pair<kSplit>(dk, dl, c / 2, d0, d1);
          }
        }
        ENL_TMEM_ST16(lane_addr + Cfg::kColDP + 64 * half + 16 * ch, dk);
        if constexpr (kSplit) ENL_TMEM_ST16(lane_addr + Cfg::kColLo + 64 * half + 16 * ch, dl);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_ready + half);
    }
    // Epilogue through shared memory, as in the dK/dV kernel.
    bool ok = __all_sync(0xffffffffu, !failed && !*abort_flag);
    if (ok && n_units > 0)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar_done, (n_units - 1) & 1, abort_flag, 112) &&
                          mbar_wait(bar_done + 1, (n_units - 1) & 1, abort_flag, 113));
    float* stg = reinterpret_cast<float*>(smem + Cfg::kOffStr);  // [128][D + 4]
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < D / 2; c += 16) {
        const int col0 = half * (D / 2) + c;
        uint32_t aq[16];
        __syncwarp();
        if (n_units > 0) ENL_TMEM_LD16(lane_addr + Cfg::kColAcc0 + col0, aq);
        stage_row16<D>(stg, rloc, col0, aq, p.scale, n_units > 0);
      }
    }
    named_bar_sync(1, 256);
    if (ok) {
      float* base = p.dq + b * p.dq_sb + h * p.dq_sh + (long long)qt * 128 * p.dq_ss;
      store_rows<D>(stg, base, p.dq_ss, min(128, p.Sq - qt * 128), p.d_real, p.out_vec4 != 0,
                    warp, lane);
    }
    named_bar_sync(1, 256);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

template <int D, bool kSplit>
cudaError_t launch_bwd_main(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const CUtensorMap& tdo, const BwdParams& p, cudaStream_t stream) {
  using Cfg = BwdCfg<D, kSplit>;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    e = cudaFuncSetAttribute(attn_bwd_dkdv_sm100<D, kSplit>, a, Cfg::kSmemBytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_bwd_dq_sm100<D, kSplit>, a, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const long long n_kt = (p.Skv + 127) / 128, n_qt = (p.Sq + 127) / 128;
  attn_bwd_dkdv_sm100<D, kSplit><<<(unsigned)(n_kt * p.B * p.Hkv), Cfg::kThreads, Cfg::kSmemBytes,
                           stream>>>(tq, tk, tv, tdo, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_bwd_dq_sm100<D, kSplit><<<(unsigned)(n_qt * p.B * p.H), Cfg::kThreads, Cfg::kSmemBytes, stream>>>(
      tq, tk, tv, tdo, p);
  return cudaGetLastError();
}

cudaError_t launch_backward(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const CUtensorMap& tdo, const BwdPrepParams& prep, const BwdParams& p,
                            int D, bool split, cudaStream_t stream) {
  const long long rows = (long long)prep.B * prep.H * prep.s_pad;
  const long long blocks = min((rows + 15) / 16, 148ll * 32);  // 16 rows per 256-thread block
  bwd_prep_kernel<<<(int)blocks, 256, 0, stream>>>(prep);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (split)  // the ABI admits split mode only at head dims <= 64
    return launch_bwd_main<64, true>(tq, tk, tv, tdo, p, stream);
  return D == 128 ? launch_bwd_main<128, false>(tq, tk, tv, tdo, p, stream)
                  : launch_bwd_main<64, false>(tq, tk, tv, tdo, p, stream);
}

}  // namespace enl
