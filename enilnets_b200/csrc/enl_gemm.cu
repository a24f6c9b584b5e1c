// K6: the attention layers' projections, Y = X W^T + b, on tcgen05 CTA pairs.
//
// Replaces the reference's projection GEMMs (nn/forward.py:428-430 for
// Q/K/V, :551 for the output, the same in nn/forward.py:567-586 for cross
// attention and in nn/kvcache.py:148-154 for a cached step) and fuses the
// RoPE rotation of Q and K (nn/forward.py:80-88) into the epilogue.
//
// Persistent kernel over 256 x 256 output tiles. Two CTAs of a cluster work
// as one pair (tcgen05 cta_group::2): CTA r of the pair loads rows
// [128 r, 128 r + 128) of the tile's X rows and rows [128 r, 128 r + 128) of
// its W rows (output columns), each CTA with its own non-multicast TMA loads.
// The even CTA issues one M=256 x N=256 x K=16 MMA per 16-wide K step, which
// reads both CTAs' shared memory, and each CTA's tensor memory receives its
// 128 output rows x 256 columns. Per SM that is the same tensor work as an
// M=128 x N=256 MMA for half the W bytes of a one-CTA tile.
//
// Roles (192 threads per CTA):
//   warp 0      TMA producer (both CTAs): X and W tiles of 64 K columns into
//               a ring of stages; both CTAs' loads complete on the even
//               CTA's `full` barrier, which its producer arms with the
//               pair's bytes
//   warp 1      MMA issuer (even CTA only); allocates the pair's tensor
//               memory in both CTAs
//   warps 2-5   epilogue (both CTAs): each warp owns 32 rows (its TMEM lane
//               quarter); reads the fp32 accumulator, adds the bias, rotates
//               the RoPE columns, converts and stages 128-byte-wide chunks in
//               shared memory that the warp stores with TMA
// Tensor memory holds two 256-column accumulators, so the epilogue of one
// tile overlaps the K loop of the next. Stage release (`empty`) and
// accumulator hand-off (`acc_full`) are tcgen05.commit arrivals on both
// CTAs' barriers; the epilogue warps of both CTAs hand an accumulator back
// with remote arrivals on the even CTA's `acc_empty` barrier.
//
// fp32 inputs (the reference's default float32 models): X and W arrive as
// bf16 planes hi = bf16(x), lo = bf16(x - hi) and every product is
// hi*hi + hi*lo + lo*hi (three MMAs per K step), about 2^-16 relative error.
//
// Every wait is bounded (about 1 s). A wait that runs out records the error
// in the device error word, raises the CTA's abort flag and the CTA skips
// its remaining work; both CTAs always meet at the final cluster barrier
// before tensor memory is freed.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {
namespace gemm {

constexpr int kThreads = 192;
constexpr int kTileM = 256;  // output rows per CTA pair
constexpr int kTileN = 256;  // output columns per tile
constexpr int kBlockK = 64;  // K columns per stage: one 128-byte swizzle atom of bf16
constexpr int kHalfBytes = 128 * kBlockK * 2;  // one CTA's 128 x 64 bf16 operand tile
constexpr int kEpiWarps = 4;
constexpr int kStageBufBytes = 32 * 128;  // one warp's 32 rows x 128 bytes of output

template <bool kSplit>
struct Cfg {
  static constexpr int kPlanes = kSplit ? 2 : 1;
  static constexpr int kStages = kSplit ? 3 : 6;
  static constexpr int kStageBytes = 2 * kPlanes * kHalfBytes;  // X planes + W planes
  static constexpr int kOffStage = 0;
  static constexpr int kOffOut = kStages * kStageBytes;       // epilogue staging
  static constexpr int kOutBytes = kEpiWarps * 2 * kStageBufBytes;
  static constexpr int kOffBar = kOffOut + kOutBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  // Operand tile p of stage s: X plane p at 2p, W plane p at 2p + 1.
  __host__ __device__ static constexpr int off_x(int s, int plane) {
    return kOffStage + s * kStageBytes + (2 * plane) * kHalfBytes;
  }
  __host__ __device__ static constexpr int off_w(int s, int plane) {
    return kOffStage + s * kStageBytes + (2 * plane + 1) * kHalfBytes;
  }
};

// --------------------------------------------------------------- cluster PTX
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t n_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Shared::cluster address of the variable at `p` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Wait with cluster-scope acquire: the phase was completed by arrivals or
// MMA commits from the other CTA of the pair.
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_cl(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int site) {
  if (mbar_try_wait_cl(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) {
      report_error(kDevWaitTimeout, site);
      *abort_flag = 1;
      return false;
    }
  }
}
// 2-D tile load into this CTA's shared memory whose completion is counted on
// the even CTA's barrier (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
// Wait until at most one committed bulk store still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                   smem_u32(smem_result))
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(taddr) : "memory");
}
// One pair MMA (M=256, N=256, K=16) from an elected lane of the issuing warp.
__device__ __forceinline__ void umma_pair_elect(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                                uint32_t desc_hi, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, acc;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 acc, %5, 0;\n\t"
      "@p tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %4, acc;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in both CTAs of the pair once every
// pair MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ epilogue
// Rotate-half RoPE (nn/forward.py:80-88) on the 128 columns of v that hold
// whole heads of kD columns: column c of a head pairs with c + kD/2.
// cos/sin are this row's table rows (kD / 2 floats each, 16-byte aligned),
// read four at a time as the rotation needs them.
template <int kD>
__device__ __forceinline__ void rope_group(float (&v)[128], const float* __restrict__ cs,
                                           const float* __restrict__ sn, uint32_t head_mask) {
  constexpr int kH = kD / 2;
#pragma unroll
  for (int i4 = 0; i4 < kH; i4 += 4) {
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + i4));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + i4));
    const float c[4] = {c4.x, c4.y, c4.z, c4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int j = 0; j < 128 / kD; ++j) {
      if (!((head_mask >> j) & 1u)) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = i4 + e;
        const float x1 = v[j * kD + i], x2 = v[j * kD + i + kH];
        v[j * kD + i] = x1 * c[e] - x2 * sv[e];
        v[j * kD + i + kH] = x2 * c[e] + x1 * sv[e];
      }
    }
  }
}

template <bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
    proj_gemm_sm100(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_xlo,
                    const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_wlo,
                    const __grid_constant__ CUtensorMap tm_y, const ProjParams p) {
  using C = Cfg<kSplit>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The alignment fix-up is the same in both CTAs, so equal offsets name the
  // same buffers in either (the pair MMA relies on that).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* bar_full = bars;
  uint64_t* bar_empty = bar_full + C::kStages;
  uint64_t* bar_acc_full = bar_empty + C::kStages;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_drain = bar_acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int n_tiles_n = (p.N + kTileN - 1) / kTileN;
  const int n_tiles = ((p.M + kTileM - 1) / kTileM) * n_tiles_n;
  const int n_k = (p.K + kBlockK - 1) / kBlockK;
  const int first_tile = (int)cluster_id_x(), tile_step = (int)n_clusters_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + s, 1);
      mbar_init(bar_empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_acc_full + a, 1);
      mbar_init(bar_acc_empty + a, 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      if constexpr (kSplit) {
        tma_prefetch_desc(&tm_xlo);
        tma_prefetch_desc(&tm_wlo);
      }
      uint32_t it = 0;
      bool ok = true;
      for (int t = first_tile; t < n_tiles && ok; t += tile_step) {
        const int m0 = (t / n_tiles_n) * kTileM + 128 * (int)rank;
        const int n0 = (t % n_tiles_n) * kTileN + 128 * (int)rank;
        for (int kb = 0; kb < n_k && ok; ++kb, ++it) {
          const int s = it % C::kStages;
          const uint32_t use = it / C::kStages;
          if (use > 0) ok = wait_cl(bar_empty + s, (use - 1) & 1, abort_flag, 60);
          if (!ok) break;
          if (leader) mbar_arrive_expect_tx(bar_full + s, 2 * C::kStageBytes);
          const uint32_t full = map_to_rank(bar_full + s, 0);
          tma_load_2d_pair(smem + C::off_x(s, 0), &tm_x, full, kb * kBlockK, m0);
          tma_load_2d_pair(smem + C::off_w(s, 0), &tm_w, full, kb * kBlockK, n0);
          if constexpr (kSplit) {
            tma_load_2d_pair(smem + C::off_x(s, 1), &tm_xlo, full, kb * kBlockK, m0);
            tma_load_2d_pair(smem + C::off_w(s, 1), &tm_wlo, full, kb * kBlockK, n0);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (leader) {
      const uint32_t idesc = idesc_bf16_f32(256, 256, false);
      const uint32_t st_lo = desc_lo(smem_u32(smem + C::kOffStage), 16);
      auto wait = [&](uint64_t* bar, uint32_t parity, int site) {
        return __all_sync(0xffffffffu, wait_cl(bar, parity, abort_flag, site));
      };
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = first_tile; t < n_tiles && ok; t += tile_step, ++tc) {
        const int a = tc & 1;
        if (tc >= 2) ok = wait(bar_acc_empty + a, ((tc >> 1) - 1) & 1, 61);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem_base + 256u * a;
        for (int kb = 0; kb < n_k && ok; ++kb, ++it) {
          const int s = it % C::kStages;
          ok = wait(bar_full + s, (it / C::kStages) & 1, 62);
          if (!ok) break;
          tc_fence_after();
          const uint32_t xs = st_lo + (uint32_t)(s * C::kStageBytes) / 16;
          constexpr uint32_t kPlaneLo = 2 * kHalfBytes / 16;  // hi plane -> lo plane
          constexpr uint32_t kW = kHalfBytes / 16;            // X tile -> W tile
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint32_t off = kk * 2;  // 32 bytes per K16 step, in 16-byte units
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            umma_pair_elect(d, xs + off, xs + kW + off, kDescHiSw128, idesc, acc);
            if constexpr (kSplit) {
              umma_pair_elect(d, xs + off, xs + kW + kPlaneLo + off, kDescHiSw128, idesc, 1u);
              umma_pair_elect(d, xs + kPlaneLo + off, xs + kW + off, kDescHiSw128, idesc, 1u);
            }
          }
          umma_commit_pair_elect(bar_empty + s);
        }
        if (!ok) break;
        umma_commit_pair_elect(bar_acc_full + a);
      }
      // Tensor memory is freed only after every MMA issued here has completed
      // (on the normal path the epilogues have waited for them already).
      umma_commit_pair_elect(bar_drain);
      volatile int no_abort = 0;
      wait_cl(bar_drain, 0, &no_abort, 64);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp % 4;  // TMEM lane quarter of this warp
    const uint32_t lane_addr = tmem_base + ((uint32_t)(32 * q) << 16);
    uint8_t* stage_buf = smem + C::kOffOut + (warp - 2) * 2 * kStageBufBytes;
    const uint32_t acc_empty_leader[2] = {map_to_rank(bar_acc_empty + 0, 0),
                                          map_to_rank(bar_acc_empty + 1, 0)};
    const int cw = p.out_fp32 ? 32 : 64;  // columns per 128-byte chunk
    uint32_t tc = 0, nstore = 0;
    bool ok = true;
    for (int t = first_tile; t < n_tiles && ok; t += tile_step, ++tc) {
      const int a = tc & 1;
      ok = __all_sync(0xffffffffu, wait_cl(bar_acc_full + a, (tc >> 1) & 1, abort_flag, 63));
      if (!ok) break;
      tc_fence_after();
      const int mt = t / n_tiles_n, nt = t % n_tiles_n;
      const int row0 = mt * kTileM + 128 * (int)rank + 32 * q;  // first row of this warp
      const int m = row0 + lane;
      const bool rows_in = row0 < p.M;  // stores start inside the tensor
      const long long pos = p.rope_seq > 0 ? p.rope_pos0 + (m % p.rope_seq) : 0;
      for (int g = 0; g < kTileN / 128; ++g) {
        const int c0 = nt * kTileN + g * 128;  // first output column of the group
        float v[128];
        {
          uint32_t r[128];
          ENL_TMEM_LD128(lane_addr + 256u * a + 128u * g, r);
#pragma unroll
          for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
        }
        if (g == kTileN / 128 - 1) {
          // The accumulator is in registers: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty_leader[a]);
        }
        if (p.bias != nullptr) {
#pragma unroll
          for (int i = 0; i < 128; i += 4) {
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + i + 4 <= p.N) b4 = *reinterpret_cast<const float4*>(p.bias + c0 + i);
            v[i] += b4.x;
            v[i + 1] += b4.y;
            v[i + 2] += b4.z;
            v[i + 3] += b4.w;
          }
        }
        if (p.rope_cols > c0 && m < p.M) {
          // Heads of this group inside the rotated columns, one bit per head.
          const int D = p.rope_d;
          const int n_heads = 128 / D;
          uint32_t mask = 0;
          for (int j = 0; j < n_heads; ++j)
            if (c0 + (j + 1) * D <= p.rope_cols) mask |= 1u << j;
          const int h = D / 2;
          const float* cs = p.rope_cos + pos * h;
          const float* sn = p.rope_sin + pos * h;
          switch (D) {
            case 128: rope_group<128>(v, cs, sn, mask); break;
            case 64: rope_group<64>(v, cs, sn, mask); break;
            case 32: rope_group<32>(v, cs, sn, mask); break;
            case 16: rope_group<16>(v, cs, sn, mask); break;
            case 8: rope_group<8>(v, cs, sn, mask); break;
            default: break;
          }
        }
        // Stage and store 128-byte-wide chunks of this warp's 32 rows.
        for (int ch = 0; ch < 128 / cw && rows_in; ++ch) {
          const int col = c0 + ch * cw;
          if (col >= p.N) break;
          uint8_t* buf = stage_buf + (nstore & 1) * kStageBufBytes;
          if (lane == 0) bulk_wait_read_1();  // the buffer's previous store has read it
          __syncwarp();
          uint8_t* row = buf + lane * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u) {  // 16-byte units of the 128-byte row
            uint4 w;
            if (p.out_fp32) {
              const float* src = v + (ch * 32 + u * 4);
              w = make_uint4(__float_as_uint(src[0]), __float_as_uint(src[1]),
                             __float_as_uint(src[2]), __float_as_uint(src[3]));
            } else {
              const float* src = v + (ch * 64 + u * 8);
              w = make_uint4(pack_bf16x2(src[0], src[1]), pack_bf16x2(src[2], src[3]),
                             pack_bf16x2(src[4], src[5]), pack_bf16x2(src[6], src[7]));
            }
            *reinterpret_cast<uint4*>(row + ((u ^ (lane & 7)) << 4)) = w;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_y, buf, col, row0);
            bulk_commit_group();
          }
          ++nstore;
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  // Both CTAs finish their roles before the pair's tensor memory is freed:
  // the even CTA's MMAs write the odd CTA's tensor memory.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base);
  }
}

}  // namespace gemm

template <bool kSplit>
cudaError_t launch_proj_gemm(const CUtensorMap& tx, const CUtensorMap& txlo,
                             const CUtensorMap& tw, const CUtensorMap& twlo,
                             const CUtensorMap& ty, const ProjParams& p, int n_sms,
                             cudaStream_t stream) {
  using C = gemm::Cfg<kSplit>;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm::proj_gemm_sm100<kSplit>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const long long n_tiles = (long long)((p.M + gemm::kTileM - 1) / gemm::kTileM) *
                            ((p.N + gemm::kTileN - 1) / gemm::kTileN);
  if (n_tiles <= 0) return cudaSuccess;
  const long long pairs = std::min<long long>(n_tiles, std::max(1, n_sms / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(gemm::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm::proj_gemm_sm100<kSplit>, tx, txlo, tw, twlo, ty, p);
}

template cudaError_t launch_proj_gemm<false>(const CUtensorMap&, const CUtensorMap&,
                                             const CUtensorMap&, const CUtensorMap&,
                                             const CUtensorMap&, const ProjParams&, int,
                                             cudaStream_t);
template cudaError_t launch_proj_gemm<true>(const CUtensorMap&, const CUtensorMap&,
                                            const CUtensorMap&, const CUtensorMap&,
                                            const CUtensorMap&, const ProjParams&, int,
                                            cudaStream_t);

// fp32 -> bf16 planes hi = bf16(x), lo = bf16(x - hi) of a row-major (rows,
// cols) matrix with row stride `ld` elements, into two contiguous
// (rows, cols) planes. Four elements per thread.
__global__ void split_matrix_kernel(const float* __restrict__ src, long long ld, long long rows,
                                    int cols, uint16_t* __restrict__ hi,
                                    uint16_t* __restrict__ lo) {
  const int q4 = cols / 4;
  const long long total = rows * q4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / q4;
    const int c = (int)(i % q4) * 4;
    const float4 x = *reinterpret_cast<const float4*>(src + r * ld + c);
    const uint32_t h01 = pack_bf16x2(x.x, x.y), h23 = pack_bf16x2(x.z, x.w);
    const uint32_t l01 = pack_bf16x2(x.x - bf16lo_to_f32(h01), x.y - bf16hi_to_f32(h01));
    const uint32_t l23 = pack_bf16x2(x.z - bf16lo_to_f32(h23), x.w - bf16hi_to_f32(h23));
    *reinterpret_cast<uint2*>(hi + r * cols + c) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(lo + r * cols + c) = make_uint2(l01, l23);
  }
}

cudaError_t launch_split_matrix(const float* src, long long ld, long long rows, int cols,
                                void* hi, void* lo, cudaStream_t stream) {
  const long long total = rows * (cols / 4);
  if (total == 0) return cudaSuccess;
  const long long blocks = std::min<long long>((total + 255) / 256, 148ll * 16);
  split_matrix_kernel<<<(int)blocks, 256, 0, stream>>>(
      src, ld, rows, cols, reinterpret_cast<uint16_t*>(hi), reinterpret_cast<uint16_t*>(lo));
  return cudaGetLastError();
}

}  // namespace enl
