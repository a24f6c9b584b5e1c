// K4 on the tensor pipe: linearized attention (attention_kernel "linear" and
// "performer", nn/attention_kernels.py:119-143, the cached step of
// nn/kvcache.py:217-260) as chunked tcgen05 contractions.
//
// With phi >= 0 features, causal linear attention is
//   out_i = sum_{j <= i} (phi(q_i).phi(k_j)) v_j / (sum_{j <= i} phi(q_i).phi(k_j) + eps).
// Appending a ones column to V (V' = [V | 1 | 0 ...], Dp columns) makes the
// denominator column D of the same product. Over 128-row chunks c:
//   U_c     = phi(K_c)^T V'_c  (stored transposed, Dp x Df) [lin_state_chunk]
//   S_{c-1} = S_in + sum_{c' < c} U_c'            (exclusive) [lin_scan_chunks]
//   O'_c    = (phi(Q_c) phi(K_c)^T o mask) V'_c + phi(Q_c) S_{c-1}   [lin_out_chunk]
//   out     = O'_c[:, :D] / (O'_c[:, D] + eps)
// Non-causal calls use the total S for every chunk and no intra-chunk term.
// The carried state of a cached step is S_in (scaled); the returned state is
// the scan's total.
//
// Every operand is staged K-major as bf16 planes hi = bf16(x), lo = bf16(x - hi)
// and every product is hi*hi + hi*lo + lo*hi on kind::f16 MMAs with fp32
// accumulation (about 2^-16 relative error, inside the fp32 bar). A prep pass
// writes the planes: phi(Q) and phi(K) row-major (rows x features), V'
// transposed (columns x rows); the scan writes S^T.
#include <climits>

#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {
namespace lintc {

constexpr int kC = 128;       // rows per chunk
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 elementwise / epilogue

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// SS MMA from an elected lane with a runtime accumulate flag.
__device__ __forceinline__ void umma_ss_elect_acc(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                                  uint32_t desc_hi, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, acc;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 acc, %5, 0;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, acc;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf16_val(uint16_t b) {
  return __bfloat162float(__ushort_as_bfloat16(b));
}
__device__ __forceinline__ void split2(float x, uint16_t& hi, uint16_t& lo) {
  hi = bf16_bits(x);
  lo = bf16_bits(x - bf16_val(hi));
}

// ---------------------------------------------------------------- prep
// Four fp32 values -> bf16 hi at dst[0..3] and lo at dst[plane + 0..3].
__device__ __forceinline__ void store_split_quad(float4 x, uint16_t* dst, long long plane) {
  const uint32_t h01 = pack_bf16x2(x.x, x.y), h23 = pack_bf16x2(x.z, x.w);
  const uint32_t l01 = pack_bf16x2(x.x - bf16lo_to_f32(h01), x.y - bf16hi_to_f32(h01));
  const uint32_t l23 = pack_bf16x2(x.z - bf16lo_to_f32(h23), x.w - bf16hi_to_f32(h23));
  *reinterpret_cast<uint2*>(dst) = make_uint2(h01, h23);
  *reinterpret_cast<uint2*>(dst + plane) = make_uint2(l01, l23);
}

// Row-major planes: src (R, Df) fp32 -> dst[plane][R][Dfp] bf16.
__device__ __forceinline__ void prep_rows_quad(const float* __restrict__ src, long long r, int f,
                                               int Df, int Dfp, long long plane,
                                               uint16_t* __restrict__ dst) {
  store_split_quad(__ldg(reinterpret_cast<const float4*>(src + r * Df + f)), dst + r * Dfp + f,
                   plane);
}

__global__ void lin_prep_rows(const float* __restrict__ src, long long R, int Df, int Dfp,
                              DivU32 dq4, uint16_t* __restrict__ dst) {
  const long long plane = R * Dfp;
  if ((Df & 3) == 0) {
    // Four features per thread: one 16-byte load, two 8-byte stores.
    const long long n = R * dq4.d;
    if (n <= (1ll << 31)) {
      // Four loads in flight per thread before the first store.
      const uint32_t stride = gridDim.x * blockDim.x;
      for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < (uint32_t)n;
           i0 += 4 * stride) {
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t i = i0 + u * stride;
          if (i >= (uint32_t)n) break;
          const uint32_t r = dq4.div(i);
          x[u] = __ldg(reinterpret_cast<const float4*>(src + (long long)r * Df) +
                       (i - r * dq4.d));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t i = i0 + u * stride;
          if (i >= (uint32_t)n) break;
          const uint32_t r = dq4.div(i);
          store_split_quad(x[u], dst + (long long)r * Dfp + (i - r * dq4.d) * 4, plane);
        }
      }
      return;
    }
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
      const long long r = i / dq4.d;
      prep_rows_quad(src, r, (int)(i - r * dq4.d) * 4, Df, Dfp, plane, dst);
    }
    return;
  }
  const long long n = R * Df;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Df;
    const int f = (int)(i - r * Df);
    uint16_t hi, lo;
    split2(src[i], hi, lo);
    dst[r * Dfp + f] = hi;
    dst[plane + r * Dfp + f] = lo;
  }
}

// Transposed planes of V' = [V | 1 | 0...]: v[b, s, hkv, d] (element strides,
// bf16 or fp32) -> dst[plane][B * Hkv][Dp][Sp]; row D is 1 for s < S. One CTA
// per (b * Hkv + hkv, 64 positions): the 64 rows of V go into shared memory
// (an odd row stride, so that the column reads below are free of bank
// conflicts), then every 16 threads write one 128-byte run of a row of V'^T,
// four positions per thread, in both planes. D <= kVtMaxD, Sp a multiple of 4.
constexpr int kVtRows = 64, kVtMaxD = 128;

__global__ void __launch_bounds__(256)
    lin_prep_vt(const void* __restrict__ v, long long sb, long long ss, long long sh, int f32,
                int Hkv, int S, int D, int Dp, int Sp, long long BH, int vec, DivU32 dq4,
                uint16_t* __restrict__ dst) {
  __shared__ float tile[kVtRows * (kVtMaxD + 1)];
  const int ld = D | 1;
  const int bh = blockIdx.x;
  const int b = bh / Hkv, hkv = bh - b * Hkv;
  const int s0 = blockIdx.y * kVtRows;
  const int t = threadIdx.x;
  const long long base = (long long)b * sb + (long long)hkv * sh;
  if (vec) {  // D % 4 == 0, 16-byte (fp32) or 8-byte (bf16) aligned rows
    for (uint32_t k = t; k < kVtRows * dq4.d; k += 256) {
      const uint32_t r = dq4.div(k);
      const int c = (int)(k - r * dq4.d) * 4, s = s0 + (int)r;
      float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (s < S) {
        const long long off = base + (long long)s * ss + c;
        if (f32) {
          const float4 q = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(v) + off));
          x[0] = q.x, x[1] = q.y, x[2] = q.z, x[3] = q.w;
        } else {
          const uint2 q = __ldg(reinterpret_cast<const uint2*>(
              reinterpret_cast<const __nv_bfloat16*>(v) + off));
          x[0] = bf16lo_to_f32(q.x), x[1] = bf16hi_to_f32(q.x);
          x[2] = bf16lo_to_f32(q.y), x[3] = bf16hi_to_f32(q.y);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[r * ld + c + e] = x[e];
    }
  } else {
    for (int k = t; k < kVtRows * D; k += 256) {
      const int r = k / D, c = k - r * D, s = s0 + r;
      float x = 0.0f;
      if (s < S) {
        const long long off = base + (long long)s * ss + c;
        x = f32 ? reinterpret_cast<const float*>(v)[off]
                : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v)[off]);
      }
      tile[r * ld + c] = x;
    }
  }
  __syncthreads();
  const long long plane = BH * Dp * Sp;
  for (int k = t; k < Dp * (kVtRows / 4); k += 256) {
    const int d = k >> 4, j = (k & 15) * 4;
    if (s0 + j >= Sp) continue;
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int s = s0 + j + e;
      x[e] = s >= S ? 0.0f : d < D ? tile[(j + e) * ld + d] : d == D ? 1.0f : 0.0f;
    }
    const uint32_t h01 = pack_bf16x2(x[0], x[1]), h23 = pack_bf16x2(x[2], x[3]);
    const uint32_t l01 = pack_bf16x2(x[0] - bf16lo_to_f32(h01), x[1] - bf16hi_to_f32(h01));
    const uint32_t l23 = pack_bf16x2(x[2] - bf16lo_to_f32(h23), x[3] - bf16hi_to_f32(h23));
    const long long o = ((long long)bh * Dp + d) * Sp + s0 + j;
    *reinterpret_cast<uint2*>(dst + o) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(dst + plane + o) = make_uint2(l01, l23);
  }
}

// ------------------------------------------------------------- helpers
// A bounded wait by one warp's lanes, then tcgen05 ordering.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, site));
}

// Loads `n` consecutive TMEM columns (n a multiple of 16) of this warp's
// lanes into v, 16 at a time.
template <int kMax>
__device__ __forceinline__ void tmem_ld_cols(uint32_t addr, int n, float (&v)[kMax]) {
#pragma unroll
  for (int c = 0; c < kMax; c += 16) {
    if (c < n) {
      uint32_t r[16];
      ENL_TMEM_LD16(addr + c, r);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[c + i] = __uint_as_float(r[i]);
    }
  }
}

// ---------------------------------------------------- A: chunk states
// CTA (bh * n_chunks + c, m-tile): U[bh][c][f][d] for f in [128 mt, 128 mt + 128).
// Operands: A = phi(K)^T, M = features, K = the chunk's keys, read from the
// row-major phi(K) planes as an MN-major operand (two 64-feature atoms of 128
// keys per plane, 16 KB apart); B = V'^T rows d, chunk keys (K-major).
// M = 128, N = Dp, K = 128 keys.
struct StateSmem {
  __host__ __device__ static int a_bytes() { return 2 * 2 * 128 * 128; }  // [plane][atom] 128 x 128 B
  __host__ __device__ static int b_bytes(int Dp) { return 2 * 2 * Dp * 128; }
  __host__ __device__ static int total(int Dp) { return a_bytes() + b_bytes(Dp) + 64 + 1024; }
};

__global__ void __launch_bounds__(kThreads, 1)
    lin_state_chunk(const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_vt, LinTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int Dp = p.Dp;
  uint8_t* sa = smem;                       // [plane][atom][128][128 B]
  uint8_t* sb = smem + StateSmem::a_bytes();  // [plane][atom][Dp][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sb + StateSmem::b_bytes(Dp));
  uint64_t* bar_full = bars;
  uint64_t* bar_done = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x / p.n_chunks, c = blockIdx.x % p.n_chunks;
  const int f0 = blockIdx.y * 128, s0 = c * kC;
  const long long BH = (long long)p.B * p.Hkv;

  if (threadIdx.x == 0) {
    mbar_init(bar_full, 1);
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<256>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int a_atom = 128 * 128, b_atom = Dp * 128;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar_full, 2 * 2 * (a_atom + b_atom));
      for (int pl = 0; pl < 2; ++pl)
        for (int a = 0; a < 2; ++a) {
          tma_load_3d(sa + (pl * 2 + a) * a_atom, &tm_k, bar_full, f0 + 64 * a, s0,
                      (int)(pl * BH + bh));
          tma_load_3d(sb + (pl * 2 + a) * b_atom, &tm_vt, bar_full, s0 + 64 * a, 0,
                      (int)(pl * BH + bh));
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    bool ok = warp_wait(bar_full, 0, abort_flag, 70);
    if (ok) {
      tc_fence_after();
      // A MN-major (bit 15 of the instruction descriptor): its 64-feature
      // atoms lie a_atom bytes apart (leading byte offset), 16 keys are 2 KB.
      const uint32_t idesc = idesc_bf16_f32(128, Dp, false) | (1u << 15);
      const uint32_t a_lo = desc_lo(smem_u32(sa), a_atom), b_lo = desc_lo(smem_u32(sb), 16);
      const uint32_t a_pl = (2 * a_atom) >> 4, b_pl = (2 * b_atom) >> 4;
#pragma unroll 1
      for (int kk = 0; kk < kC / 16; ++kk) {
        const uint32_t ao = kk * (2048 >> 4);
        const uint32_t bo = (kk / 4) * (b_atom >> 4) + (kk % 4) * 2;
        const uint32_t acc = kk > 0 ? 1u : 0u;
        // hi*hi, hi*lo, lo*hi
        umma_ss_elect_acc(tmem, a_lo + ao, b_lo + bo, kDescHiSw128, idesc, acc);
        umma_ss_elect_acc(tmem, a_lo + ao, b_lo + b_pl + bo, kDescHiSw128, idesc, 1u);
        umma_ss_elect_acc(tmem, a_lo + a_pl + ao, b_lo + bo, kDescHiSw128, idesc, 1u);
      }
    }
    umma_commit_elect(bar_done);
  } else {
    // epilogue: row f = f0 + 32 q + lane of U[bh][c]
    const int q = warp % 4;
    const bool ok = warp_wait(bar_done, 0, abort_flag, 71);
    if (ok) {
      tc_fence_after();
      // U^T[bh][c][d][f]: for each column d the warp's 32 lanes (consecutive
      // features) store 128 contiguous bytes.
      const int f = f0 + 32 * q + lane;
      float* ut = p.u + ((long long)bh * p.n_chunks + c) * Dp * p.Df + f;
      const uint32_t addr = tmem + ((uint32_t)(32 * q) << 16);
      for (int c0 = 0; c0 < Dp; c0 += 16) {
        uint32_t r[16];
        ENL_TMEM_LD16(addr + c0, r);
        if (f < p.Df) {
#pragma unroll
          for (int i = 0; i < 16; ++i) ut[(long long)(c0 + i) * p.Df] = __uint_as_float(r[i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<256>(tmem);
  }
}

// ------------------------------------------------------ B: chunk scan
// One thread per (b * kv head, column d, feature pair f, f + 1), f fastest:
// the running sum over the chunks of U^T, written before each chunk's own sum
// is added (exclusive) as S^T planes st[plane][bh * n_chunks + c][d][f],
// starting from the carried state (times its scale). Non-causal calls write
// only the total, at c = 0. The total also goes to kv_out (d < D) / ks_out
// (d == D). Chunk sums are loaded four chunks at a time (8 bytes per thread
// and chunk) so their loads overlap; the planes take 4-byte stores. An odd
// feature count leaves the last pair's second feature out.
__global__ void __launch_bounds__(256) lin_scan_chunks(LinTcParams p, DivU32 dpair, DivU32 dcol) {
  const int Dp = p.Dp, Df = p.Df, D = p.D;
  const int n_pair = (int)dpair.d;  // (Df + 1) / 2
  const long long per_bh = (long long)Dp * Df;
  const uint32_t n = (uint32_t)((long long)p.B * p.Hkv * Dp * n_pair);
  const long long plane = (long long)p.B * p.Hkv * p.n_chunks * Dp * p.Dfp;
  const long long st_chunk = (long long)Dp * p.Dfp;
  const bool even = (Df & 1) == 0;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t row = dpair.div(i);  // bh * Dp + d
    const int f = (int)(i - row * dpair.d) * 2;
    const uint32_t bh = dcol.div(row);
    const int d = (int)(row - bh * dcol.d);
    const bool two = f + 1 < Df;
    const float scale = p.state_scale ? p.state_scale[bh] : 1.0f;
    float run0 = 0.0f, run1 = 0.0f;
    if (d < D && p.kv_in) {
      run0 = p.kv_in[((long long)bh * Df + f) * D + d] * scale;
      if (two) run1 = p.kv_in[((long long)bh * Df + f + 1) * D + d] * scale;
    }
    if (d == D && p.ks_in) {
      run0 = p.ks_in[(long long)bh * Df + f] * scale;
      if (two) run1 = p.ks_in[(long long)bh * Df + f + 1] * scale;
    }
    const float* u = p.u + (long long)bh * p.n_chunks * per_bh + (long long)d * Df + f;
    uint16_t* st = p.st + ((long long)bh * p.n_chunks * Dp + d) * p.Dfp + f;
    for (int cb = 0; cb < p.n_chunks; cb += 4) {
      float x0[4], x1[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x0[j] = x1[j] = 0.0f;
        if (cb + j < p.n_chunks) {
          const float* uj = u + (cb + j) * per_bh;
          if (even) {
            const float2 t = __ldg(reinterpret_cast<const float2*>(uj));
            x0[j] = t.x, x1[j] = t.y;
          } else {
            x0[j] = uj[0];
            if (two) x1[j] = uj[1];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (cb + j >= p.n_chunks) break;
        if (p.causal) {
          const uint32_t hi = pack_bf16x2(run0, run1);
          const uint32_t lo = pack_bf16x2(run0 - bf16lo_to_f32(hi), run1 - bf16hi_to_f32(hi));
          *reinterpret_cast<uint32_t*>(st + (cb + j) * st_chunk) = hi;
          *reinterpret_cast<uint32_t*>(st + plane + (cb + j) * st_chunk) = lo;
        }
        run0 += x0[j];
        run1 += x1[j];
      }
    }
    if (!p.causal) {
      const uint32_t hi = pack_bf16x2(run0, run1);
      const uint32_t lo = pack_bf16x2(run0 - bf16lo_to_f32(hi), run1 - bf16hi_to_f32(hi));
      *reinterpret_cast<uint32_t*>(st) = hi;
      *reinterpret_cast<uint32_t*>(st + plane) = lo;
    }
    if (d < D && p.kv_out) {
      p.kv_out[((long long)bh * Df + f) * D + d] = run0;
      if (two) p.kv_out[((long long)bh * Df + f + 1) * D + d] = run1;
    }
    if (d == D && p.ks_out) {
      p.ks_out[(long long)bh * Df + f] = run0;
      if (two) p.ks_out[(long long)bh * Df + f + 1] = run1;
    }
  }
}

// ---------------------------------------------------- C: chunk outputs
// CTA (b * H + h) x chunk. Per 64-feature step: phi(Q) and phi(K) tiles of
// the chunk (hi, lo) and the chunk's S^T tile (hi, lo) arrive in one stage;
// P += phi(Q) phi(K)^T and O' += phi(Q) S (three MMAs each per 16-wide step).
// Then the elementwise warps mask P causally, split it into bf16 hi/lo over
// its own tensor-memory columns, and O' += P V' runs as a TS MMA (P from
// tensor memory) against the chunk's V'^T tile, loaded into the same stage.
struct OutSmem {
  __host__ __device__ static int stage_bytes(int Dp) {
    const int qk = 2 * 2 * 128 * 128;  // Q, K tiles, both planes (64 features, 128 rows)
    const int s = 2 * Dp * 128;        // S^T tile, both planes
    const int v = 2 * 2 * Dp * 128;    // V'^T tile, both planes, two 64-key atoms
    return qk + s > v ? qk + s : v;
  }
  __host__ __device__ static int total(int Dp) { return stage_bytes(Dp) + 128 + 1024; }
};

__global__ void __launch_bounds__(kThreads, 2)
    lin_out_chunk(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_st,
                  const __grid_constant__ CUtensorMap tm_vt, LinTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int Dp = p.Dp;
  const int qk_atom = 128 * 128, s_atom = Dp * 128;
  uint8_t* sq = smem;                      // [plane][128 rows][128 B]
  uint8_t* sk = smem + 2 * qk_atom;        // [plane][128 rows][128 B]
  uint8_t* ss = smem + 4 * qk_atom;        // [plane][Dp rows][128 B]
  uint8_t* sv = smem;                      // [plane][atom][Dp rows][128 B] (after the loop)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OutSmem::stage_bytes(Dp));
  uint64_t* bar_full = bars;       // one phase per feature step, then one for V'
  uint64_t* bar_empty = bars + 1;  // stage consumed by the MMAs
  uint64_t* bar_p = bars + 2;      // P and the state term complete
  uint64_t* bar_pw = bars + 3;     // P masked and split (4 warps)
  uint64_t* bar_o = bars + 4;      // O' complete
  uint64_t* bar_drain = bars + 5;  // every MMA of the CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int hkv = h / (p.H / p.Hkv);
  const int bhk = b * p.Hkv + hkv;
  const int c = blockIdx.y, s0 = c * kC;
  const int n_f = (p.Df + 63) / 64;
  const long long BHq = (long long)p.B * p.H, BHk = (long long)p.B * p.Hkv;
  const long long st_idx = (long long)bhk * p.n_chunks + (p.causal ? c : 0);
  const long long ST_N = BHk * p.n_chunks;

  if (threadIdx.x == 0) {
    mbar_init(bar_full, 1);
    mbar_init(bar_empty, 1);
    mbar_init(bar_p, 1);
    mbar_init(bar_pw, 4);
    mbar_init(bar_o, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if (p.tmem_cols == 512)
      tmem_alloc<512>(tmem_slot);
    else
      tmem_alloc<256>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_p = tmem, t_o = tmem + 128;  // P: 128 columns, O': Dp columns

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int kf = 0; kf < n_f && ok; ++kf) {
        if (kf > 0) ok = mbar_wait(bar_empty, (kf - 1) & 1, abort_flag, 80);
        if (!ok) break;
        const int bytes = (p.causal ? 4 * qk_atom : 2 * qk_atom) + 2 * s_atom;
        mbar_arrive_expect_tx(bar_full, bytes);
        for (int pl = 0; pl < 2; ++pl) {
          tma_load_3d(sq + pl * qk_atom, &tm_q, bar_full, 64 * kf, s0, (int)(pl * BHq + bh));
          if (p.causal)
            tma_load_3d(sk + pl * qk_atom, &tm_k, bar_full, 64 * kf, s0, (int)(pl * BHk + bhk));
          tma_load_3d(ss + pl * s_atom, &tm_st, bar_full, 64 * kf, 0, (int)(pl * ST_N + st_idx));
        }
      }
      if (ok && p.causal) {
        ok = mbar_wait(bar_empty, (n_f - 1) & 1, abort_flag, 81);
        if (ok) {
          mbar_arrive_expect_tx(bar_full, 4 * s_atom);
          for (int pl = 0; pl < 2; ++pl)
            for (int a = 0; a < 2; ++a)
              tma_load_3d(sv + (pl * 2 + a) * s_atom, &tm_vt, bar_full, s0 + 64 * a, 0,
                          (int)(pl * BHk + bhk));
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    const uint32_t idesc_p = idesc_bf16_f32(128, 128, false);
    const uint32_t idesc_o = idesc_bf16_f32(128, Dp, false);
    const uint32_t q_lo = desc_lo(smem_u32(sq), 16), k_lo = desc_lo(smem_u32(sk), 16);
    const uint32_t s_lo = desc_lo(smem_u32(ss), 16), v_lo = desc_lo(smem_u32(sv), 16);
    const uint32_t qk_pl = qk_atom >> 4, s_pl = s_atom >> 4;
    bool ok = true;
    for (int kf = 0; kf < n_f && ok; ++kf) {
      ok = warp_wait(bar_full, kf & 1, abort_flag, 82);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t off = kk * 2;
        const uint32_t acc = (kf > 0 || kk > 0) ? 1u : 0u;
        if (p.causal) {
          umma_ss_elect_acc(t_p, q_lo + off, k_lo + off, kDescHiSw128, idesc_p, acc);
          umma_ss_elect_acc(t_p, q_lo + off, k_lo + qk_pl + off, kDescHiSw128, idesc_p, 1u);
          umma_ss_elect_acc(t_p, q_lo + qk_pl + off, k_lo + off, kDescHiSw128, idesc_p, 1u);
        }
        umma_ss_elect_acc(t_o, q_lo + off, s_lo + off, kDescHiSw128, idesc_o, acc);
        umma_ss_elect_acc(t_o, q_lo + off, s_lo + s_pl + off, kDescHiSw128, idesc_o, 1u);
        umma_ss_elect_acc(t_o, q_lo + qk_pl + off, s_lo + off, kDescHiSw128, idesc_o, 1u);
      }
      umma_commit_elect(bar_empty);
    }
    if (ok) umma_commit_elect(p.causal ? bar_p : bar_o);
    if (ok && p.causal) {
      // O' += P V': P hi in TMEM columns [0, 64), lo in [64, 128); V'^T in the stage.
      ok = warp_wait(bar_pw, 0, abort_flag, 83);
      if (ok) ok = warp_wait(bar_full, n_f & 1, abort_flag, 84);
      if (ok) {
        tc_fence_after();
        const uint32_t v_pl = (2 * s_atom) >> 4;
#pragma unroll 1
        for (int kk = 0; kk < kC / 16; ++kk) {
          const uint32_t vo = (kk / 4) * (s_atom >> 4) + (kk % 4) * 2;
          umma_ts_elect(t_o, t_p + kk * 8, v_lo + vo, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(t_o, t_p + kk * 8, v_lo + v_pl + vo, kDescHiSw128, idesc_o, 1u);
          umma_ts_elect(t_o, t_p + 64 + kk * 8, v_lo + vo, kDescHiSw128, idesc_o, 1u);
        }
        umma_commit_elect(bar_o);
      }
    }
    // Drain before tensor memory is freed.
    umma_commit_elect(bar_drain);
    volatile int no_abort = 0;
    mbar_wait(bar_drain, 0, &no_abort, 85);
  } else {
    const int q = warp % 4;
    const int row = 32 * q + lane;  // query row of the chunk == TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    bool ok = true;
    if (p.causal) {
      ok = warp_wait(bar_p, 0, abort_flag, 86);
      if (ok) {
        tc_fence_after();
        uint32_t r[128];
        ENL_TMEM_LD128(t_p + lane_off, r);
        uint32_t hi[64], lo[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float x0 = (2 * j <= row) ? __uint_as_float(r[2 * j]) : 0.0f;
          const float x1 = (2 * j + 1 <= row) ? __uint_as_float(r[2 * j + 1]) : 0.0f;
          hi[j] = pack_bf16x2(x0, x1);
          lo[j] = pack_bf16x2(x0 - bf16lo_to_f32(hi[j]), x1 - bf16hi_to_f32(hi[j]));
        }
        ENL_TMEM_ST32(t_p + lane_off, hi, 0);
        ENL_TMEM_ST32(t_p + lane_off + 32, hi, 32);
        ENL_TMEM_ST32(t_p + lane_off + 64, lo, 0);
        ENL_TMEM_ST32(t_p + lane_off + 96, lo, 32);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pw);
    }
    if (ok) ok = warp_wait(bar_o, 0, abort_flag, 87);
    if (ok) {
      tc_fence_after();
      // The denominator (column D) first, then the D output columns 16 at a time.
      float den = 0.0f;
      {
        uint32_t r[16];
        ENL_TMEM_LD16(t_o + lane_off + (uint32_t)(p.D & ~15), r);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i == (p.D & 15)) den = __uint_as_float(r[i]);
      }
      const float inv = 1.0f / (den + p.eps);
      const int s = s0 + row;
      const long long off = (long long)b * p.o_sb + (long long)s * p.o_ss + (long long)h * p.o_sh;
      const bool vec = p.o_f32 ? ((p.o_sh | p.o_ss | p.o_sb) & 3) == 0 &&
                                     (reinterpret_cast<uintptr_t>(p.o) & 15) == 0
                               : ((p.o_sh | p.o_ss | p.o_sb) & 7) == 0 &&
                                     (reinterpret_cast<uintptr_t>(p.o) & 15) == 0;
      for (int c0 = 0; c0 < p.D; c0 += 16) {
        uint32_t r[16];
        ENL_TMEM_LD16(t_o + lane_off + c0, r);
        if (s >= p.S) continue;
        float y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = __uint_as_float(r[i]) * inv;
        const int n = min(16, p.D - c0);
        if (p.o_f32) {
          float* dst = reinterpret_cast<float*>(p.o) + off + c0;
          if (vec && n == 16) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(dst + i) = make_float4(y[i], y[i + 1], y[i + 2], y[i + 3]);
          } else {
            for (int i = 0; i < n; ++i) dst[i] = y[i];
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.o) + off + c0;
          if (vec && n == 16) {
#pragma unroll
            for (int i = 0; i < 16; i += 8)
              *reinterpret_cast<uint4*>(dst + i) =
                  make_uint4(pack_bf16x2(y[i], y[i + 1]), pack_bf16x2(y[i + 2], y[i + 3]),
                             pack_bf16x2(y[i + 4], y[i + 5]), pack_bf16x2(y[i + 6], y[i + 7]));
          } else {
            for (int i = 0; i < n; ++i) dst[i] = __float2bfloat16(y[i]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (p.tmem_cols == 512)
      tmem_dealloc<512>(tmem);
    else
      tmem_dealloc<256>(tmem);
  }
}

// ------------------------------------------- Performer feature map (tcgen05)
// phi(x) = exp(x'.w - |x'|^2 / 2 - stab) / sqrt(Df), x' = x / Dh^(1/4)
// (nn/attention_kernels.py:38-74), for Df <= 256: one CTA per (b * H + h,
// 128-row block). The projections x.w run as split-bf16 MMAs (M = 128 rows,
// N = Df, K = Dh in 64-wide steps through a two-stage ring) into tensor
// memory; the epilogue threads (one row each) scale by Dh^(-1/4) and apply the
// stabilizer. kMode 0: the tile's maximum into stab[b * H + h] (ordered-int
// atomic max); 1: each row's own maximum (queries); 2: stab[b * H + h] (keys).
// Operands: xp[plane][B * H][S][Dhp] (row planes of the head view), wp[plane][Df][Dhp].
// One tile's epilogue for one warp: rows 32q..32q+31 of the 128-row tile at
// s0 of head bh, accumulator columns at addr (this warp's lane quarter).
// xs: the staged x tile (hi plane at 0, lo plane at kPerfX, one 64-wide K
// step per xs_step bytes), or null to read the planes from global memory.
// buf: the warp's 32-row x 128-byte staging buffer. xs_release (nullable):
// a barrier the warp's lane 0 arrives on once the row norms are read.
constexpr int kPerfX = 128 * 128;  // bytes of one plane of a 64-wide K step of x

template <int kMode>
__device__ __forceinline__ void perf_tile_epilogue(const PerfTcParams& p, uint32_t addr,
                                                   const uint8_t* xs, int xs_step, int bh,
                                                   int s0, int q, int lane, uint8_t* buf,
                                                   uint64_t* xs_release = nullptr) {
  const int row = 32 * q + lane, s = s0 + row;
  const long long BH = (long long)p.B * p.H;
  const int n_k = (p.Dh + 63) / 64;
  const int Dfn = (p.Df + 15) / 16 * 16;
  const float inv4 = rsqrtf(sqrtf((float)p.Dh));  // Dh^(-1/4)
  // |x'|^2 / 2 from the row's own planes (hi + lo recovers x to 2^-16):
  // 128 bytes per plane and K step, 16-byte units at (unit ^ row % 8) under
  // the 128-byte swizzle.
  float sq = 0.0f;
  if (s < p.S && kMode != 0) {
    if (xs) {
      for (int kb = 0; kb < n_k; ++kb) {
        const uint8_t* xr = xs + kb * xs_step + row * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (64 * kb + 8 * j >= p.Dh) break;
          const uint4 h = *reinterpret_cast<const uint4*>(xr + ((j ^ (row & 7)) << 4));
          const uint4 l = *reinterpret_cast<const uint4*>(xr + kPerfX + ((j ^ (row & 7)) << 4));
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (64 * kb + 8 * j + e < p.Dh) {
              const float hv = e & 1 ? bf16hi_to_f32(hw[e / 2]) : bf16lo_to_f32(hw[e / 2]);
              const float lv = e & 1 ? bf16hi_to_f32(lw[e / 2]) : bf16lo_to_f32(lw[e / 2]);
              const float x = (hv + lv) * inv4;
              sq = fmaf(x, x, sq);
            }
          }
        }
      }
    } else {
      const uint16_t* xh = p.xp + ((long long)bh * p.S + s) * p.Dhp;
      const uint16_t* xl = xh + BH * p.S * p.Dhp;
      for (int d = 0; d < p.Dh; ++d) {
        const float x = (bf16_val(xh[d]) + bf16_val(xl[d])) * inv4;
        sq = fmaf(x, x, sq);
      }
    }
    sq *= 0.5f;
  }
  if (xs_release) {
    __syncwarp();
    if (lane == 0) mbar_arrive(xs_release);
  }
  // The row maximum (mode 0 and 1): one pass over the accumulator.
  float m = -INFINITY;
  if (kMode != 2) {
    int c0 = 0;
    // 64 columns per wait while they last (two loads in flight), four
    // independent maxima per pass.
    for (; c0 + 64 <= Dfn; c0 += 64) {
      uint32_t r[64];
      ENL_TMEM_LD32X2(addr + c0, r, addr + c0 + 32, (r + 32));
      const int n_valid = p.Df - c0;
      float mx[4] = {m, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (i < n_valid) mx[i % 4] = fmaxf(mx[i % 4], __uint_as_float(r[i]));
      m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
    }
    for (; c0 < Dfn; c0 += 32) {
      uint32_t r[32];
      if (c0 + 32 <= Dfn) {
        ENL_TMEM_LD32(addr + c0, r, 0);
      } else {
        ENL_TMEM_LD16(addr + c0, r);
#pragma unroll
        for (int i = 16; i < 32; ++i) r[i] = __float_as_uint(-INFINITY);
      }
      const int n_valid = p.Df - c0;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n_valid) m = fmaxf(m, __uint_as_float(r[i]));
    }
    m *= inv4;
    if (s >= p.S) m = -INFINITY;
  }
  if (kMode == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && m > -INFINITY) atomicMax(reinterpret_cast<int*>(p.stab) + bh, ord_enc(m));
    return;
  }
  // 32 features at a time: each lane puts its row's 32 values in the warp's
  // 32-row x 128-byte buffer (16-byte units XOR-swizzled by row against bank
  // conflicts), then the warp stores 4 whole 128-byte row segments per
  // instruction. With p.planes a row's 128 bytes are its 32 bf16 hi values,
  // then the 32 lo values, and go to the two planes as 64-byte runs.
  // exp(a inv4 - sq - stab) / sqrt(Df) = 2^(a c1 - c2): one FMA and one ex2 per
  // feature, c1 = inv4 log2(e), c2 = (sq + stab) log2(e) + log2(Df) / 2.
  const float stab = kMode == 1 ? m : p.stab[bh];
  constexpr float kLog2e = 1.4426950408889634f;
  const float c1 = inv4 * kLog2e;
  const float c2 = (sq + stab) * kLog2e + 0.5f * __log2f((float)p.Df);
  const long long plane_elems = BH * p.S * p.Dfp;
  const int row0 = s0 + 32 * q;
  for (int c0 = 0; c0 < Dfn && row0 < p.S; c0 += 32) {
    uint32_t r[32];
    if (c0 + 32 <= Dfn) {
      ENL_TMEM_LD32(addr + c0, r, 0);
    } else {
      ENL_TMEM_LD16(addr + c0, r);
#pragma unroll
      for (int i = 16; i < 32; ++i) r[i] = 0u;
    }
    // All 32 exponentials independent (no branch between them), then the
    // columns past Df are zeroed by a select.
    const int n_valid = p.Df - c0;
    float y[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float e = fast_exp2(fmaf(__uint_as_float(r[i]), c1, -c2));
      y[i] = i < n_valid ? e : 0.0f;
    }
    __syncwarp();  // the previous chunk's reads of the buffer are done
    if (p.planes) {
      uint32_t hw[16], lw[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        hw[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
        lw[i] = pack_bf16x2(y[2 * i] - bf16lo_to_f32(hw[i]), y[2 * i + 1] - bf16hi_to_f32(hw[i]));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        *reinterpret_cast<uint4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(hw[4 * u], hw[4 * u + 1], hw[4 * u + 2], hw[4 * u + 3]);
        *reinterpret_cast<uint4*>(buf + lane * 128 + (((u + 4) ^ (lane & 7)) << 4)) =
            make_uint4(lw[4 * u], lw[4 * u + 1], lw[4 * u + 2], lw[4 * u + 3]);
      }
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_float4(y[4 * u], y[4 * u + 1], y[4 * u + 2], y[4 * u + 3]);
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int piece = 32 * k + lane, rr = piece / 8, u = piece % 8;
      if (row0 + rr >= p.S) continue;
      const uint4 v4 = *reinterpret_cast<const uint4*>(buf + rr * 128 + ((u ^ (rr & 7)) << 4));
      const long long grow = (long long)bh * p.S + row0 + rr;
      if (p.planes) {
        const int col = c0 + 8 * (u & 3);  // 8 features per 16-byte unit
        if (col < p.Df)
          *reinterpret_cast<uint4*>(p.planes + (u >> 2) * plane_elems + grow * p.Dfp + col) = v4;
      } else {
        const int col = c0 + 4 * u;
        if (col < p.Df) *reinterpret_cast<uint4*>(p.phi + grow * p.Df + col) = v4;
      }
    }
  }
  __syncwarp();  // the buffer is free for the warp's next tile
}

struct PerfSmem {
  __host__ __device__ static int stage_bytes() { return 2 * 128 * 128 + 2 * 256 * 128; }
  // Head dims up to 64 are one K step: one stage, so that two CTAs fit per SM.
  // The epilogue stages its output in stage 0, free once the MMAs are done.
  __host__ __device__ static int stages(int Dh) { return Dh > 64 ? 2 : 1; }
  __host__ __device__ static int total(int Dh) { return stages(Dh) * stage_bytes() + 128 + 1024; }
};

template <int kMode>
__global__ void __launch_bounds__(kThreads)
    phi_perf_tc(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                PerfTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  constexpr int kX = kPerfX;
  const int n_st = PerfSmem::stages(p.Dh);
  uint8_t* out_stage = smem;  // stage 0, after the MMAs have read it
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + n_st * PerfSmem::stage_bytes());
  uint64_t* bar_full = bars;       // [2]
  uint64_t* bar_empty = bars + 2;  // [2]
  uint64_t* bar_acc = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.y, s0 = blockIdx.x * 128;
  const int n_k = (p.Dh + 63) / 64;
  const long long BH = (long long)p.B * p.H;
  const int Dfn = (p.Df + 15) / 16 * 16;  // MMA N

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_full + i, 1);
      mbar_init(bar_empty + i, 1);
    }
    mbar_init(bar_acc, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<256>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < n_k && ok; ++kb) {
        const int st = kb % n_st;
        if (kb >= n_st) ok = mbar_wait(bar_empty + st, ((kb - n_st) / n_st) & 1, abort_flag, 90);
        if (!ok) break;
        uint8_t* base = smem + st * PerfSmem::stage_bytes();
        mbar_arrive_expect_tx(bar_full + st, 2 * kX + 2 * Dfn * 128);
        for (int pl = 0; pl < 2; ++pl) {
          tma_load_3d(base + pl * kX, &tm_x, bar_full + st, 64 * kb, s0, (int)(pl * BH + bh));
          tma_load_3d(base + 2 * kX + pl * Dfn * 128, &tm_w, bar_full + st, 64 * kb, 0, pl);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    const uint32_t idesc = idesc_bf16_f32(128, Dfn, false);
    bool ok = true;
    for (int kb = 0; kb < n_k && ok; ++kb) {
      const int st = kb % n_st;
      ok = warp_wait(bar_full + st, (kb / n_st) & 1, abort_flag, 91);
      if (!ok) break;
      tc_fence_after();
      uint8_t* base = smem + st * PerfSmem::stage_bytes();
      const uint32_t x_lo = desc_lo(smem_u32(base), 16);
      const uint32_t w_lo = desc_lo(smem_u32(base + 2 * kX), 16);
      const uint32_t x_pl = kX >> 4, w_pl = (Dfn * 128) >> 4;
#pragma unroll 1
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t off = kk * 2;
        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
        umma_ss_elect_acc(tmem, x_lo + off, w_lo + off, kDescHiSw128, idesc, acc);
        umma_ss_elect_acc(tmem, x_lo + off, w_lo + w_pl + off, kDescHiSw128, idesc, 1u);
        umma_ss_elect_acc(tmem, x_lo + x_pl + off, w_lo + off, kDescHiSw128, idesc, 1u);
      }
      umma_commit_elect(bar_empty + st);
    }
    umma_commit_elect(bar_acc);
  } else {
    const int q = warp % 4;
    const bool ok = warp_wait(bar_acc, 0, abort_flag, 92);
    if (ok) {
      tc_fence_after();
      // While every K step still has its own stage (head dims up to 128), the
      // row norms are read from the staged tiles; the stage's full barrier (one
      // completed phase) orders the TMA's writes before the reads.
      bool staged = kMode != 0 && n_k <= n_st;
      for (int kb = 0; kb < n_k && staged; ++kb)
        staged = warp_wait(bar_full + kb, 0, abort_flag, 93);
      perf_tile_epilogue<kMode>(p, tmem + ((uint32_t)(32 * q) << 16), staged ? smem : nullptr,
                                PerfSmem::stage_bytes(), bh, s0, q, lane,
                                out_stage + q * 32 * 128);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<256>(tmem);
  }
}

// Persistent form of the Performer map for head dims up to 64 (one K step):
// one CTA per SM walks the (b * H + h, 128-row block) tiles c, c + grid, ...
// The omega planes are loaded once and stay in shared memory; x tiles stream
// through a 3-stage ring; the projections of a tile go to one of two 256-column
// accumulators in tensor memory, so that a tile's MMAs and loads overlap the
// epilogue of the one before. Two groups of four epilogue warps take
// alternate tiles (group g always uses accumulator g). A ring stage is free
// once the MMAs that read it completed and the group's four warps read its
// row norms (five arrivals).
constexpr int kPersistThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 two epilogue groups
constexpr int kPersistStages = 3;
struct PersistSmem {
  static constexpr int kW = 2 * 256 * 128;      // omega, both planes, up to 256 features
  static constexpr int kXStage = 2 * kPerfX;    // x tile, both planes
  static constexpr int kOut = 8 * 32 * 128;     // eight warps' staging buffers
  static constexpr int kBars = 256;
  static constexpr int total() { return kW + kPersistStages * kXStage + kOut + kBars + 1024; }
};

template <int kMode>
__global__ void __launch_bounds__(kPersistThreads, 1)
    phi_perf_persist(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     PerfTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* w_s = smem;
  uint8_t* x_s = smem + PersistSmem::kW;
  uint8_t* out_s = x_s + kPersistStages * PersistSmem::kXStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_s + PersistSmem::kOut);
  uint64_t* w_full = bars;                            // [1]
  uint64_t* x_full = bars + 1;                        // [kPersistStages]
  uint64_t* x_empty = x_full + kPersistStages;        // [kPersistStages]
  uint64_t* acc_full = x_empty + kPersistStages;      // [2]
  uint64_t* acc_empty = acc_full + 2;                 // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long BH = (long long)p.B * p.H;
  const int n_rb = (p.S + 127) / 128;
  const long long n_tiles = BH * n_rb;
  const int n_local =
      blockIdx.x < n_tiles ? (int)((n_tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
  const int Dfn = (p.Df + 15) / 16 * 16;  // MMA N

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int i = 0; i < kPersistStages; ++i) {
      mbar_init(x_full + i, 1);
      mbar_init(x_empty + i, 5);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<512>(tmem_slot);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tile_of = [&](int j, int& bh, int& s0) {
    const long long t = blockIdx.x + (long long)j * gridDim.x;
    bh = (int)(t / n_rb);
    s0 = (int)(t - (long long)bh * n_rb) * 128;
  };

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(w_full, 2 * Dfn * 128);
      for (int pl = 0; pl < 2; ++pl) tma_load_3d(w_s + pl * 256 * 128, &tm_w, w_full, 0, 0, pl);
      for (int j = 0; j < n_local && ok; ++j) {
        const int st = j % kPersistStages;
        if (j >= kPersistStages)
          ok = mbar_wait(x_empty + st, ((j / kPersistStages) - 1) & 1, abort_flag, 94);
        if (!ok) break;
        int bh, s0;
        tile_of(j, bh, s0);
        uint8_t* xb = x_s + st * PersistSmem::kXStage;
        mbar_arrive_expect_tx(x_full + st, 2 * kPerfX);
        for (int pl = 0; pl < 2; ++pl)
          tma_load_3d(xb + pl * kPerfX, &tm_x, x_full + st, 0, s0, (int)(pl * BH + bh));
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    const uint32_t idesc = idesc_bf16_f32(128, Dfn, false);
    bool ok = warp_wait(w_full, 0, abort_flag, 95);
    const uint32_t w_lo = desc_lo(smem_u32(w_s), 16), w_pl = (256 * 128) >> 4;
    for (int j = 0; j < n_local && ok; ++j) {
      const int st = j % kPersistStages, a = j & 1;
      if (j >= 2) ok = warp_wait(acc_empty + a, ((j >> 1) - 1) & 1, abort_flag, 96);
      if (ok) ok = warp_wait(x_full + st, (j / kPersistStages) & 1, abort_flag, 97);
      if (!ok) break;
      tc_fence_after();
      const uint32_t x_lo = desc_lo(smem_u32(x_s + st * PersistSmem::kXStage), 16);
      const uint32_t x_pl = kPerfX >> 4, d = tmem + (uint32_t)(a * 256);
#pragma unroll 1
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t off = kk * 2;
        umma_ss_elect_acc(d, x_lo + off, w_lo + off, kDescHiSw128, idesc, kk > 0 ? 1u : 0u);
        umma_ss_elect_acc(d, x_lo + off, w_lo + w_pl + off, kDescHiSw128, idesc, 1u);
        umma_ss_elect_acc(d, x_lo + x_pl + off, w_lo + off, kDescHiSw128, idesc, 1u);
      }
      umma_commit_elect(x_empty + st);
      umma_commit_elect(acc_full + a);
    }
  } else {
    const int g = (warp - 2) / 4, q = warp % 4;
    uint8_t* buf = out_s + (warp - 2) * 32 * 128;
    bool ok = true;
    for (int j = g; j < n_local && ok; j += 2) {
      const int st = j % kPersistStages;
      ok = warp_wait(acc_full + g, (j >> 1) & 1, abort_flag, 98);
      if (ok) ok = warp_wait(x_full + st, (j / kPersistStages) & 1, abort_flag, 99);
      if (!ok) break;
      tc_fence_after();
      int bh, s0;
      tile_of(j, bh, s0);
      // Row norms from the staged tile, then the stage goes back to the ring
      // before the (longer) exponential and store pass.
      const uint8_t* xb = x_s + st * PersistSmem::kXStage;
      perf_tile_epilogue<kMode>(p, tmem + (uint32_t)(g * 256) + ((uint32_t)(32 * q) << 16), xb,
                                0, bh, s0, q, lane, buf, x_empty + st);
      tc_fence_before();
      if (lane == 0) mbar_arrive(acc_empty + g);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// x[b, s, h, :] (strided, bf16 or fp32) -> planes [plane][B * H][S][Dhp],
// four elements per thread (Dh % 4 == 0, 8- or 16-byte aligned rows, at most
// 2^31 groups of four: the flat index splits by multiply-high divisions),
// four loads in flight per thread before the first store.
__global__ void perf_prep_x4(const void* __restrict__ x, long long sb, long long ss,
                             long long sh, int f32, DivU32 dq4, DivU32 ds, DivU32 dh, int B,
                             int Dhp, uint16_t* __restrict__ dst) {
  const int S = (int)ds.d, H = (int)dh.d;
  const uint32_t n = (uint32_t)((long long)B * H * S * dq4.d);
  const long long plane = (long long)B * H * S * Dhp;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += 4 * stride) {
    float4 v[4];
    long long o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * stride;
      if (i >= n) break;
      const uint32_t r = dq4.div(i);
      const int d = (int)(i - r * dq4.d) * 4;
      const uint32_t bh = ds.div(r);
      const int s = (int)(r - bh * ds.d);
      const uint32_t b = dh.div(bh);
      const int h = (int)(bh - b * dh.d);
      const long long off = (long long)b * sb + (long long)s * ss + (long long)h * sh + d;
      o[u] = ((long long)bh * S + s) * Dhp + d;
      if (f32) {
        v[u] = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off));
      } else {
        const uint2 t = __ldg(reinterpret_cast<const uint2*>(
            reinterpret_cast<const __nv_bfloat16*>(x) + off));
        v[u] = make_float4(bf16lo_to_f32(t.x), bf16hi_to_f32(t.x), bf16lo_to_f32(t.y),
                           bf16hi_to_f32(t.y));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i0 + u * stride >= n) break;
      store_split_quad(v[u], dst + o[u], plane);
    }
  }
}

// Any alignment: one element per thread.
__global__ void perf_prep_x(const void* __restrict__ x, long long sb, long long ss, long long sh,
                            int f32, int B, int S, int H, int Dh, int Dhp,
                            uint16_t* __restrict__ dst) {
  const long long n = (long long)B * H * S * Dh;
  const long long plane = (long long)B * H * S * Dhp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % Dh);
    long long r = i / Dh;
    const int s = (int)(r % S);
    r /= S;
    const int h = (int)(r % H), b = (int)(r / H);
    const long long off = b * sb + (long long)s * ss + (long long)h * sh + d;
    const float v = f32 ? reinterpret_cast<const float*>(x)[off]
                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[off]);
    uint16_t hi, lo;
    split2(v, hi, lo);
    const long long o = (((long long)b * H + h) * S + s) * Dhp + d;
    dst[o] = hi;
    dst[plane + o] = lo;
  }
}

// omega (Df, Dh) fp32 -> planes [plane][Df][Dhp].
__global__ void perf_prep_w(const float* __restrict__ w, int Df, int Dh, int Dhp,
                            uint16_t* __restrict__ dst) {
  const int n = Df * Dh;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int f = i / Dh, d = i % Dh;
    uint16_t hi, lo;
    split2(w[i], hi, lo);
    dst[(long long)f * Dhp + d] = hi;
    dst[(long long)Df * Dhp + (long long)f * Dhp + d] = lo;
  }
}

}  // namespace lintc

bool perf_tc_supported(int Dh, int Df) { return Df <= 256 && Dh <= 256; }

cudaError_t launch_perf_prep(const void* x, long long sb, long long ss, long long sh, int f32,
                             const float* omega, const PerfTcParams& p, uint16_t* wp,
                             cudaStream_t stream) {
  using namespace lintc;
  const long long n = (long long)p.B * p.H * p.S * p.Dh;
  const bool vec = p.Dh % 4 == 0 && ((sb | ss | sh) % 4) == 0 &&
                   (reinterpret_cast<uintptr_t>(x) % (f32 ? 16 : 8)) == 0;
  if (n > 0 && vec && n / 4 <= (1ll << 31))
    perf_prep_x4<<<(int)std::min<long long>((n / 4 + 255) / 256, 148ll * 16), 256, 0, stream>>>(
        x, sb, ss, sh, f32, DivU32::make((uint32_t)(p.Dh / 4)), DivU32::make((uint32_t)p.S),
        DivU32::make((uint32_t)p.H), p.B, p.Dhp, p.xp);
  else if (n > 0)
    perf_prep_x<<<(int)std::min<long long>((n + 255) / 256, 148ll * 16), 256, 0, stream>>>(
        x, sb, ss, sh, f32, p.B, p.S, p.H, p.Dh, p.Dhp, p.xp);
  const int nw = p.Df * p.Dh;
  perf_prep_w<<<std::max(1, std::min((nw + 255) / 256, 1024)), 256, 0, stream>>>(
      omega, p.Df, p.Dh, p.Dhp, wp);
  return cudaGetLastError();
}

cudaError_t launch_perf_tc(const CUtensorMap& tx, const CUtensorMap& tw, const PerfTcParams& p,
                           int mode, cudaStream_t stream) {
  using namespace lintc;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    e = cudaFuncSetAttribute(phi_perf_tc<0>, a, PerfSmem::total(256));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(phi_perf_tc<1>, a, PerfSmem::total(256));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(phi_perf_tc<2>, a, PerfSmem::total(256));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(phi_perf_persist<0>, a, PersistSmem::total());
    if (e == cudaSuccess) e = cudaFuncSetAttribute(phi_perf_persist<1>, a, PersistSmem::total());
    if (e == cudaSuccess) e = cudaFuncSetAttribute(phi_perf_persist<2>, a, PersistSmem::total());
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  if (p.B * p.H == 0 || p.S == 0) return cudaSuccess;
  if (p.Dh <= 64 && p.Df <= 256) {
    const long long n_tiles = (long long)p.B * p.H * ((p.S + 127) / 128);
    const int grid = (int)std::min<long long>(n_tiles, p.n_sm > 0 ? p.n_sm : 148);
    const int smem = PersistSmem::total();
    switch (mode) {
      case 0: phi_perf_persist<0><<<grid, kPersistThreads, smem, stream>>>(tx, tw, p); break;
      case 1: phi_perf_persist<1><<<grid, kPersistThreads, smem, stream>>>(tx, tw, p); break;
      default: phi_perf_persist<2><<<grid, kPersistThreads, smem, stream>>>(tx, tw, p); break;
    }
    return cudaGetLastError();
  }
  const dim3 grid((p.S + 127) / 128, p.B * p.H);
  const int smem = PerfSmem::total(p.Dh);
  switch (mode) {
    case 0: phi_perf_tc<0><<<grid, kThreads, smem, stream>>>(tx, tw, p); break;
    case 1: phi_perf_tc<1><<<grid, kThreads, smem, stream>>>(tx, tw, p); break;
    default: phi_perf_tc<2><<<grid, kThreads, smem, stream>>>(tx, tw, p); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_perf_tc_maps(const CUtensorMap& tx, const CUtensorMap& tw,
                                const PerfTcParams& p, int global_stab, const float* stab_floor,
                                cudaStream_t stream) {
  if (!global_stab) return launch_perf_tc(tx, tw, p, 1, stream);
  // The CUDA-core kernels' stabilizer helpers: ordered-int init from the
  // floor, and the conversion back to floats after the atomic-max pass.
  PhiParams q{};
  q.B = p.B;
  q.H = p.H;
  q.stab = p.stab;
  q.stab_floor = stab_floor;
  const int nb = std::max(1, (p.B * p.H + 255) / 256);
  phi_init_kernel<<<nb, 256, 0, stream>>>(q);
  cudaError_t e = launch_perf_tc(tx, tw, p, 0, stream);
  if (e != cudaSuccess) return e;
  phi_decode_kernel<<<nb, 256, 0, stream>>>(q);
  return launch_perf_tc(tx, tw, p, 2, stream);
}

cudaError_t launch_rows_planes(const float* src, long long R, int Df, int Dfp, uint16_t* dst,
                               cudaStream_t stream) {
  using namespace lintc;
  const long long n = (R * Df + 3) / 4;
  if (n <= 0) return cudaSuccess;
  lin_prep_rows<<<(int)std::min<long long>((n + 255) / 256, 148ll * 16), 256, 0, stream>>>(
      src, R, Df, Dfp, DivU32::make((uint32_t)std::max(1, Df / 4)), dst);
  return cudaGetLastError();
}

cudaError_t launch_lin_prep(const float* phi_q, const float* phi_k, const void* v, long long v_sb,
                            long long v_ss, long long v_sh, int v_f32, const LinTcParams& p,
                            uint16_t* qp, uint16_t* kp, uint16_t* vt, cudaStream_t stream) {
  using namespace lintc;
  const long long BHk = (long long)p.B * p.Hkv;
  // phi_q / phi_k are null when the caller passed planes already.
  cudaError_t e = cudaSuccess;
  if (phi_q) e = launch_rows_planes(phi_q, (long long)p.B * p.H * p.S, p.Df, p.Dfp, qp, stream);
  if (e == cudaSuccess && phi_k) e = launch_rows_planes(phi_k, BHk * p.S, p.Df, p.Dfp, kp, stream);
  if (e != cudaSuccess) return e;
  if (BHk > 0 && p.S > 0) {
    const int n_sb = (p.Sp + kVtRows - 1) / kVtRows;
    if (p.D > kVtMaxD || p.Sp % 4 != 0 || n_sb > 65535) return cudaErrorInvalidValue;
    const int esz = v_f32 ? 4 : 2;
    const int vec = p.D % 4 == 0 && ((v_sb | v_ss | v_sh) % 4) == 0 &&
                    (reinterpret_cast<uintptr_t>(v) % (4 * esz)) == 0;
    const dim3 gv((unsigned)BHk, n_sb);
    lin_prep_vt<<<gv, 256, 0, stream>>>(v, v_sb, v_ss, v_sh, v_f32, p.Hkv, p.S, p.D, p.Dp, p.Sp,
                                       BHk, vec, DivU32::make((uint32_t)std::max(1, p.D / 4)),
                                       vt);
  }
  return cudaGetLastError();
}

cudaError_t launch_lin_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tvt,
                          const CUtensorMap& tst, const LinTcParams& p, cudaStream_t stream) {
  using namespace lintc;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    e = cudaFuncSetAttribute(lin_state_chunk, a, StateSmem::total(144));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(lin_out_chunk, a, OutSmem::total(144));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const long long BHk = (long long)p.B * p.Hkv, BHq = (long long)p.B * p.H;
  if (p.n_chunks > 0 && BHk > 0) {
    const dim3 ga((unsigned)(BHk * p.n_chunks), (p.Df + 127) / 128);
    lin_state_chunk<<<ga, kThreads, StateSmem::total(p.Dp), stream>>>(tk, tvt, p);
  }
  if (BHk > 0) {
    const int n_pair = (p.Df + 1) / 2;
    const long long n = BHk * p.Dp * n_pair;
    if (n > (1ll << 31)) return cudaErrorInvalidValue;
    lin_scan_chunks<<<(int)std::min<long long>((n + 255) / 256, 148ll * 32), 256, 0, stream>>>(
        p, DivU32::make((uint32_t)n_pair), DivU32::make((uint32_t)p.Dp));
  }
  if (p.n_chunks > 0 && BHq > 0) {
    const dim3 gc((unsigned)BHq, p.n_chunks);
    lin_out_chunk<<<gc, kThreads, OutSmem::total(p.Dp), stream>>>(tq, tk, tst, tvt, p);
  }
  return cudaGetLastError();
}

}  // namespace enl
