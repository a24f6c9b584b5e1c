// K4 on the tensor pipe: linearized attention (attention_kernel "linear" and
// "performer", nn/attention_kernels.py:119-143, the cached step of
// nn/kvcache.py:217-260) as chunked tcgen05 contractions.
//
// With phi >= 0 features, causal linear attention is
//   out_i = sum_{j <= i} (phi(q_i).phi(k_j)) v_j / (sum_{j <= i} phi(q_i).phi(k_j) + eps).
// Appending a ones column to V (V' = [V | 1 | 0 ...], Dp columns) makes the
// denominator column D of the same product. Over 128-row chunks c:
//   U_c     = phi(K_c)^T V'_c                     (Df x Dp)  [lin_state_chunk]
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
// writes the planes: phi(Q) and phi(K) row-major (rows x features), phi(K)
// and V' transposed (features / columns x rows), S^T by the scan.
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
// Row-major planes: src (R, Df) fp32 -> dst[plane][R][Dfp] bf16.
__global__ void lin_prep_rows(const float* __restrict__ src, long long R, int Df, int Dfp,
                              uint16_t* __restrict__ dst) {
  const long long n = R * Df;
  const long long plane = R * Dfp;
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

// Transposed planes of phi(K): src (BH, S, Df) -> dst[plane][BH][Dfp][Sp],
// through 32 x 32 shared-memory tiles.
__global__ void lin_prep_kt(const float* __restrict__ src, int S, int Df, int Sp, int Dfp,
                            long long BH, uint16_t* __restrict__ dst) {
  __shared__ float tile[32][33];
  const long long bh = blockIdx.z;
  const int s0 = blockIdx.x * 32, f0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const int s = s0 + r, f = f0 + tx;
    tile[r][tx] = (s < S && f < Df) ? src[(bh * S + s) * Df + f] : 0.0f;
  }
  __syncthreads();
  const long long plane = BH * Dfp * Sp;
  for (int r = ty; r < 32; r += 8) {
    const int f = f0 + r, s = s0 + tx;
    if (f < Df && s < Sp) {
      uint16_t hi, lo;
      split2(tile[tx][r], hi, lo);
      const long long o = (bh * Dfp + f) * Sp + s;
      dst[o] = hi;
      dst[plane + o] = lo;
    }
  }
}

// Transposed planes of V' = [V | 1 | 0...]: v[b, s, hkv, d] (element strides,
// bf16 or fp32) -> dst[plane][B * Hkv][Dp][Sp]; row D is 1 for s < S.
__global__ void lin_prep_vt(const void* __restrict__ v, long long sb, long long ss, long long sh,
                            int f32, int Hkv, int S, int D, int Dp, int Sp, long long BH,
                            uint16_t* __restrict__ dst) {
  __shared__ float tile[32][33];
  const long long bh = blockIdx.z;
  const int b = (int)(bh / Hkv), hkv = (int)(bh % Hkv);
  const int s0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int r = ty; r < 32; r += 8) {
    const int s = s0 + r, d = d0 + tx;
    float x = 0.0f;
    if (s < S) {
      if (d < D) {
        const long long off = b * sb + (long long)s * ss + hkv * sh + d;
        x = f32 ? reinterpret_cast<const float*>(v)[off]
                : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v)[off]);
      } else if (d == D) {
        x = 1.0f;
      }
    }
    tile[r][tx] = x;
  }
  __syncthreads();
  const long long plane = BH * Dp * Sp;
  for (int r = ty; r < 32; r += 8) {
    const int d = d0 + r, s = s0 + tx;
    if (d < Dp && s < Sp) {
      uint16_t hi, lo;
      split2(tile[tx][r], hi, lo);
      const long long o = (bh * Dp + d) * Sp + s;
      dst[o] = hi;
      dst[plane + o] = lo;
    }
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
// Operands: A = phi(K)^T rows f, chunk keys (two 64-key atoms per plane);
// B = V'^T rows d, chunk keys. M = 128, N = Dp, K = 128 keys.
struct StateSmem {
  __host__ __device__ static int a_bytes() { return 2 * 2 * 128 * 128; }  // [plane][atom] 128 x 128 B
  __host__ __device__ static int b_bytes(int Dp) { return 2 * 2 * Dp * 128; }
  __host__ __device__ static int total(int Dp) { return a_bytes() + b_bytes(Dp) + 64 + 1024; }
};

__global__ void __launch_bounds__(kThreads, 1)
    lin_state_chunk(const __grid_constant__ CUtensorMap tm_kt,
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
          tma_load_3d(sa + (pl * 2 + a) * a_atom, &tm_kt, bar_full, s0 + 64 * a, f0,
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
      const uint32_t idesc = idesc_bf16_f32(128, Dp, false);
      const uint32_t a_lo = desc_lo(smem_u32(sa), 16), b_lo = desc_lo(smem_u32(sb), 16);
      const uint32_t a_pl = (2 * a_atom) >> 4, b_pl = (2 * b_atom) >> 4;
#pragma unroll 1
      for (int kk = 0; kk < kC / 16; ++kk) {
        const uint32_t ao = (kk / 4) * (a_atom >> 4) + (kk % 4) * 2;
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
      const int f = f0 + 32 * q + lane;
      float* urow = p.u + (((long long)bh * p.n_chunks + c) * p.Df + f) * Dp;
      const uint32_t addr = tmem + ((uint32_t)(32 * q) << 16);
      for (int c0 = 0; c0 < Dp; c0 += 16) {
        uint32_t r[16];
        ENL_TMEM_LD16(addr + c0, r);
        if (f < p.Df) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(urow + c0 + i) =
                make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                            __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
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
// Per (b, kv head) and 32 x 32 tile of (feature, column): running sums over
// the chunks, written before each chunk's own sum is added (exclusive) as
// S^T planes st[plane][bh * n_chunks + c][d][f], starting from the carried
// state (times its scale). Non-causal calls write only the total, at c = 0.
// The total also goes to kv_out (d < D) / ks_out (d == D).
__global__ void __launch_bounds__(256) lin_scan_chunks(LinTcParams p) {
  __shared__ float tile[32][33];
  const int bh = blockIdx.z;
  const int f0 = blockIdx.y * 32, d0 = blockIdx.x * 32;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8
  const int Dp = p.Dp, Df = p.Df, D = p.D;
  const float scale = p.state_scale ? p.state_scale[bh] : 1.0f;
  // Thread (tx, ty) accumulates (f0 + ty + 8 j, d0 + tx), j < 4.
  float run[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int f = f0 + ty + 8 * j, d = d0 + tx;
    float x = 0.0f;
    if (f < Df && d < D && p.kv_in) x = p.kv_in[((long long)bh * Df + f) * D + d] * scale;
    if (f < Df && d == D && p.ks_in) x = p.ks_in[(long long)bh * Df + f] * scale;
    run[j] = x;
  }
  const long long plane = (long long)p.B * p.Hkv * p.n_chunks * Dp * p.Dfp;
  auto emit = [&](int c) {
    __syncthreads();  // previous readers of the tile are done
#pragma unroll
    for (int j = 0; j < 4; ++j) tile[tx][ty + 8 * j] = run[j];  // tile[d][f]
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = d0 + ty + 8 * j, f = f0 + tx;
      if (d < Dp && f < Df) {
        uint16_t hi, lo;
        split2(tile[ty + 8 * j][tx], hi, lo);
        const long long o = (((long long)bh * p.n_chunks + c) * Dp + d) * p.Dfp + f;
        p.st[o] = hi;
        p.st[plane + o] = lo;
      }
    }
  };
  for (int c = 0; c < p.n_chunks; ++c) {
    if (p.causal) emit(c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int f = f0 + ty + 8 * j, d = d0 + tx;
      if (f < Df && d < Dp) run[j] += p.u[(((long long)bh * p.n_chunks + c) * Df + f) * Dp + d];
    }
  }
  if (!p.causal) emit(0);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int f = f0 + ty + 8 * j, d = d0 + tx;
    if (f < Df && d < D && p.kv_out) p.kv_out[((long long)bh * Df + f) * D + d] = run[j];
    if (f < Df && d == D && p.ks_out) p.ks_out[(long long)bh * Df + f] = run[j];
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

__global__ void __launch_bounds__(kThreads)
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
      float v[160];
      tmem_ld_cols<160>(t_o + lane_off, Dp, v);
      const int s = s0 + row;
      if (s < p.S) {
        float den = 0.0f;
#pragma unroll
        for (int i = 0; i < 160; ++i)
          if (i == p.D) den = v[i];
        const float inv = 1.0f / (den + p.eps);
        const long long off = (long long)b * p.o_sb + (long long)s * p.o_ss + (long long)h * p.o_sh;
#pragma unroll
        for (int i = 0; i < 160; ++i) {
          if (i < p.D) {
            const float y = v[i] * inv;
            if (p.o_f32)
              reinterpret_cast<float*>(p.o)[off + i] = y;
            else
              reinterpret_cast<__nv_bfloat16*>(p.o)[off + i] = __float2bfloat16(y);
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

}  // namespace lintc

cudaError_t launch_lin_prep(const float* phi_q, const float* phi_k, const void* v, long long v_sb,
                            long long v_ss, long long v_sh, int v_f32, const LinTcParams& p,
                            uint16_t* qp, uint16_t* kp, uint16_t* kt, uint16_t* vt,
                            cudaStream_t stream) {
  using namespace lintc;
  const long long BHq = (long long)p.B * p.H, BHk = (long long)p.B * p.Hkv;
  const long long rq = BHq * p.S, rk = BHk * p.S;
  auto blocks = [](long long n) { return (int)std::min<long long>((n + 255) / 256, 148ll * 16); };
  if (rq * p.Df > 0) lin_prep_rows<<<blocks(rq * p.Df), 256, 0, stream>>>(phi_q, rq, p.Df, p.Dfp, qp);
  if (p.causal && rk * p.Df > 0)
    lin_prep_rows<<<blocks(rk * p.Df), 256, 0, stream>>>(phi_k, rk, p.Df, p.Dfp, kp);
  const dim3 tb(32, 8);
  if (BHk > 0 && p.S > 0) {
    const dim3 gk((p.Sp + 31) / 32, (p.Df + 31) / 32, (unsigned)BHk);
    lin_prep_kt<<<gk, tb, 0, stream>>>(phi_k, p.S, p.Df, p.Sp, p.Dfp, BHk, kt);
    const dim3 gv((p.Sp + 31) / 32, (p.Dp + 31) / 32, (unsigned)BHk);
    lin_prep_vt<<<gv, tb, 0, stream>>>(v, v_sb, v_ss, v_sh, v_f32, p.Hkv, p.S, p.D, p.Dp, p.Sp,
                                      BHk, vt);
  }
  return cudaGetLastError();
}

cudaError_t launch_lin_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tkt,
                          const CUtensorMap& tvt, const CUtensorMap& tst, const LinTcParams& p,
                          cudaStream_t stream) {
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
    lin_state_chunk<<<ga, kThreads, StateSmem::total(p.Dp), stream>>>(tkt, tvt, p);
  }
  if (BHk > 0) {
    const dim3 gs((p.Dp + 31) / 32, (p.Df + 31) / 32, (unsigned)BHk);
    lin_scan_chunks<<<gs, 256, 0, stream>>>(p);
  }
  if (p.n_chunks > 0 && BHq > 0) {
    const dim3 gc((unsigned)BHq, p.n_chunks);
    lin_out_chunk<<<gc, kThreads, OutSmem::total(p.Dp), stream>>>(tq, tk, tst, tvt, p);
  }
  return cudaGetLastError();
}

}  // namespace enl
