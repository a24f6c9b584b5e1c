// K4: linearized attention (the reference's attention_kernel="linear" and
// "performer" options), nn/attention_kernels.py:58-143 and the cached step of
// nn/kvcache.py:217-260.
//
// Both kernels replace softmax(q.k) by phi(q).phi(k), so attention
// reassociates into phi(Q) (phi(K)^T V) / (phi(Q) . sum phi(K)) and never
// forms a score matrix. The kernels, fp32 arithmetic throughout:
//   phi_linear_kernel   elu(x) + 1 of one head view into (B, H, S, Dh) fp32;
//   phi_perf_kernel     exp(w.x' - |x'|^2/2 - stab)/sqrt(Df) with
//                       x' = x / Dh^(1/4): the projections w.x' as a tiled
//                       GEMM (64 rows x 64 features per step), with a row
//                       stabilizer (queries) or one per (b, h) reduced by an
//                       ordered-int atomic max over the rows (keys);
//   linear_attn_kernel  per (b, query head, 32-column slice of V): causal
//                       prefix sums over 16-row chunks (intra-chunk scores
//                       phi(q_i).phi(k_j), j <= i, plus the carried state
//                       S_kv = sum phi(k) v^T and s_k = sum phi(k)), or the
//                       two global sums when non-causal. A state can be
//                       carried in (scaled) and returned, which is the decode
//                       step: a fixed-size state instead of a growing cache.
//   Long causal calls split the sequence into segments that run in
//   parallel: linear_segsum_kernel sums each segment, linear_scan_kernel
//   turns the sums into each segment's starting state (in the caller's
//   workspace), and linear_attn_kernel runs one CTA per segment.
// These options are O(S Df D) and small next to the softmax path; the
// kernels favour simple, exact fp32 code over tensor cores.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

// Order-preserving float <-> int map for atomicMax on floats.
__device__ __forceinline__ int ord_enc(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : (i ^ 0x7fffffff);
}
__device__ __forceinline__ float ord_dec(int i) { return __int_as_float(i >= 0 ? i : (i ^ 0x7fffffff)); }

__device__ __forceinline__ float load_elem(const void* base, long long idx, bool f32) {
  return f32 ? reinterpret_cast<const float*>(base)[idx]
             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}

// phi = elu(x) + 1, four features per thread: one 16-byte (fp32) or 8-byte
// (bf16) load and one 16-byte store, in output order (b, h, s, d). At most
// 2^31 groups of four, so that the flat index splits into (b, h, s, d) with
// 32-bit multiply-high divisions. Each thread issues kPhiUnroll loads before
// it stores anything, so that enough bytes are in flight to cover the DRAM
// latency on inputs of a few tens of MB. With p.planes set the output is the
// bf16 hi/lo planes [2][B * H][S][Dfp] that the tensor-core linear attention
// reads, instead of fp32 phi.
constexpr int kPhiUnroll = 4;

__global__ void __launch_bounds__(256)
    phi_linear_vec_kernel(PhiParams p, DivU32 dq4, DivU32 ds, DivU32 dh) {
  const uint32_t n = (uint32_t)((long long)p.B * p.H * p.S * dq4.d);
  const uint32_t stride = gridDim.x * blockDim.x;
  const long long plane_elems = (long long)p.B * p.H * p.S * p.Dfp;
  for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += kPhiUnroll * stride) {
    float v[kPhiUnroll][4];
#pragma unroll
    for (int u = 0; u < kPhiUnroll; ++u) {
      const uint32_t i = i0 + u * stride;
      if (i >= n) break;
      const uint32_t r = dq4.div(i);
      const int c = (int)(i - r * dq4.d) * 4;
      const uint32_t bh = ds.div(r);
      const int s = (int)(r - bh * ds.d);
      const uint32_t b = dh.div(bh);
      const int h = (int)(bh - b * dh.d);
      const long long xoff = (long long)b * p.sb + (long long)s * p.ss + (long long)h * p.sh + c;
      if (p.in_f32) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(
            reinterpret_cast<const float*>(p.x) + xoff));
        v[u][0] = x.x, v[u][1] = x.y, v[u][2] = x.z, v[u][3] = x.w;
      } else {
        const uint2 x = __ldg(reinterpret_cast<const uint2*>(
            reinterpret_cast<const __nv_bfloat16*>(p.x) + xoff));
        v[u][0] = bf16lo_to_f32(x.x), v[u][1] = bf16hi_to_f32(x.x);
        v[u][2] = bf16lo_to_f32(x.y), v[u][3] = bf16hi_to_f32(x.y);
      }
    }
#pragma unroll
    for (int u = 0; u < kPhiUnroll; ++u) {
      const uint32_t i = i0 + u * stride;
      if (i >= n) break;
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = v[u][e] > 0.0f ? v[u][e] + 1.0f : expf(fminf(v[u][e], 0.0f));
      if (p.planes) {
        // bf16 hi = bf16(y), lo = bf16(y - hi) at row r, columns c..c+3.
        const uint32_t r = dq4.div(i);
        const long long o = (long long)r * p.Dfp + (i - r * dq4.d) * 4;
        const uint32_t h01 = pack_bf16x2(y[0], y[1]), h23 = pack_bf16x2(y[2], y[3]);
        const uint32_t l01 = pack_bf16x2(y[0] - bf16lo_to_f32(h01), y[1] - bf16hi_to_f32(h01));
        const uint32_t l23 = pack_bf16x2(y[2] - bf16lo_to_f32(h23), y[3] - bf16hi_to_f32(h23));
        *reinterpret_cast<uint2*>(p.planes + o) = make_uint2(h01, h23);
        *reinterpret_cast<uint2*>(p.planes + plane_elems + o) = make_uint2(l01, l23);
      } else {
        *reinterpret_cast<float4*>(p.phi + (long long)i * 4) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
  }
}

// phi = elu(x) + 1: one warp per (b, s, h) row, elementwise (any alignment).
__global__ void __launch_bounds__(256) phi_linear_kernel(PhiParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long rows = (long long)p.B * p.S * p.H;
  for (long long r = (long long)blockIdx.x * 8 + warp; r < rows; r += (long long)gridDim.x * 8) {
    const int h = (int)(r % p.H);
    const long long bs = r / p.H;
    const int s = (int)(bs % p.S), b = (int)(bs / p.S);
    const long long xoff = b * p.sb + s * p.ss + h * p.sh;
    float* out = p.phi + (((long long)b * p.H + h) * p.S + s) * p.Df;
    for (int d = lane; d < p.Dh; d += 32) {
      const float v = load_elem(p.x, xoff + d, p.in_f32);
      out[d] = v > 0.0f ? v + 1.0f : expf(fminf(v, 0.0f));
    }
  }
}

// Performer projections w.x' (x' = x / Dh^(1/4)) as a tiled fp32 GEMM: one
// CTA per 64 rows of one (b, h), features in chunks of 64 staged in shared
// memory with the rows; each thread accumulates a 4 x 4 tile.
constexpr int kPtRows = 64, kPtFeat = 64, kPtThreads = 256;
constexpr int kPerfMaxHeadDim = 256;

__host__ __device__ inline int perf_smem_floats(int Dh) {
  return (kPtRows + kPtFeat) * (Dh + 1) + 2 * kPtRows;
}

// kMode 0: global stabilizer, the max of w.x' over the tile's rows and all
//          features, folded into stab[b*H + h] (ordered-int atomic max);
//       1: phi with each row's own stabilizer (queries);
//       2: phi with the global stabilizer in stab (keys).
template <int kMode>
__global__ void __launch_bounds__(kPtThreads) phi_perf_kernel(PhiParams p) {
  extern __shared__ float sm[];
  const int Dh = p.Dh, ld = Dh + 1;
  float* xs = sm;                          // [64][Dh + 1] scaled rows
  float* ws = xs + kPtRows * ld;           // [64][Dh + 1] feature chunk of omega
  float* sq = ws + kPtFeat * ld;           // [64] |x'|^2 / 2
  int* rmax = reinterpret_cast<int*>(sq + kPtRows);  // [64] row maxima, ordered ints
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int s0 = blockIdx.x * kPtRows;
  const int nrow = min(kPtRows, p.S - s0);
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const float inv = rsqrtf(sqrtf((float)Dh));
  for (int i = tid; i < kPtRows * Dh; i += kPtThreads) {
    const int r = i / Dh, d = i % Dh;
    xs[r * ld + d] = (r < nrow) ? load_elem(p.x, b * p.sb + (long long)(s0 + r) * p.ss +
                                                   h * p.sh + d, p.in_f32) * inv
                                : 0.0f;
  }
  __syncthreads();
  if (tid < kPtRows) {
    float a = 0.0f;
    for (int d = 0; d < Dh; ++d) a = fmaf(xs[tid * ld + d], xs[tid * ld + d], a);
    sq[tid] = 0.5f * a;
    rmax[tid] = ord_enc(-INFINITY);
  }
  float acc[4][4];
  auto chunk = [&](int f0) {
    __syncthreads();  // the previous chunk's readers are done with ws
    for (int i = tid; i < kPtFeat * Dh; i += kPtThreads) {
      const int f = i / Dh, d = i % Dh;
      ws[f * ld + d] = (f0 + f < p.Df) ? p.omega[(long long)(f0 + f) * Dh + d] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int d = 0; d < Dh; ++d) {
      float xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[(ty * 4 + i) * ld + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = ws[(tx * 4 + j) * ld + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
    }
  };
  auto valid = [&](int f0, int i, int j) { return ty * 4 + i < nrow && f0 + tx * 4 + j < p.Df; };
  if (kMode == 0) {
    float m = -INFINITY;
    for (int f0 = 0; f0 < p.Df; f0 += kPtFeat) {
      chunk(f0);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (valid(f0, i, j) && acc[i][j] == acc[i][j]) m = fmaxf(m, acc[i][j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0 && m > -INFINITY)
      atomicMax(reinterpret_cast<int*>(p.stab) + bh, ord_enc(m));
    return;
  }
  if (kMode == 1 && p.Df <= 4 * kPtFeat) {
    // Up to four feature chunks: keep every projection in registers, so the
    // GEMM runs once (row maxima, then the features from the kept values).
    float keep[4][4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c * kPtFeat >= p.Df) break;
      chunk(c * kPtFeat);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          keep[c][i][j] = acc[i][j];
          if (valid(c * kPtFeat, i, j) && acc[i][j] == acc[i][j]) m = fmaxf(m, acc[i][j]);
        }
        if (m > -INFINITY) atomicMax(rmax + ty * 4 + i, ord_enc(m));
      }
    }
    __syncthreads();  // row maxima complete
    const float norm = rsqrtf((float)p.Df);
    float* out = p.phi + ((long long)bh * p.S + s0) * p.Df;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c * kPtFeat >= p.Df) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        const float st = ord_dec(rmax[r]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (valid(c * kPtFeat, i, j))
            out[(long long)r * p.Df + c * kPtFeat + tx * 4 + j] =
                expf(keep[c][i][j] - sq[r] - st) * norm;
      }
    }
    return;
  }
  if (kMode == 1) {  // row maxima first
    for (int f0 = 0; f0 < p.Df; f0 += kPtFeat) {
      chunk(f0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (valid(f0, i, j) && acc[i][j] == acc[i][j]) m = fmaxf(m, acc[i][j]);
        if (m > -INFINITY) atomicMax(rmax + ty * 4 + i, ord_enc(m));
      }
    }
  }
  const float gstab = (kMode == 2) ? ord_dec(reinterpret_cast<const int*>(p.stab)[bh]) : 0.0f;
  const float norm = rsqrtf((float)p.Df);
  float* out = p.phi + ((long long)bh * p.S + s0) * p.Df;
  for (int f0 = 0; f0 < p.Df; f0 += kPtFeat) {
    chunk(f0);  // its leading barrier also orders the row maxima above
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      const float st = (kMode == 2) ? gstab : ord_dec(rmax[r]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (valid(f0, i, j))
          out[(long long)r * p.Df + f0 + tx * 4 + j] = expf(acc[i][j] - sq[r] - st) * norm;
    }
  }
}

__global__ void phi_init_kernel(PhiParams p) {
  const int n = p.B * p.H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    reinterpret_cast<int*>(p.stab)[i] = ord_enc(p.stab_floor ? p.stab_floor[i] : -INFINITY);
}

__global__ void phi_decode_kernel(PhiParams p) {
  const int n = p.B * p.H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    int* e = reinterpret_cast<int*>(p.stab) + i;
    p.stab[i] = ord_dec(*e);
  }
}

int perf_max_head_dim() { return kPerfMaxHeadDim; }

// The elu + 1 map's vectorised kernel: four features per thread from aligned
// rows, at most 2^31 groups of four.
static bool phi_linear_vec_ok(const PhiParams& p) {
  const int esz = p.in_f32 ? 4 : 2;
  const long long n = (long long)p.B * p.S * p.H * (p.Dh / 4);
  return p.Dh % 4 == 0 && (reinterpret_cast<uintptr_t>(p.x) % (4 * esz)) == 0 &&
         ((p.sb | p.ss | p.sh) % 4) == 0 &&
         (reinterpret_cast<uintptr_t>(p.planes ? static_cast<void*>(p.planes)
                                               : static_cast<void*>(p.phi)) % 16) == 0 &&
         n <= (1ll << 31) && (!p.planes || p.Dfp % 4 == 0);
}

bool phi_planes_direct(const PhiParams& p) { return p.kernel == 0 && phi_linear_vec_ok(p); }

cudaError_t launch_phi(const PhiParams& p, cudaStream_t stream) {
  const long long rows = (long long)p.B * p.S * p.H;
  if (p.planes && !phi_planes_direct(p)) return cudaErrorInvalidValue;
  if (p.kernel == 0) {
    const long long n = rows * (p.Dh / 4);
    if (rows > 0 && phi_linear_vec_ok(p)) {
      phi_linear_vec_kernel<<<(int)min((n + 255) / 256, 148ll * 16), 256, 0, stream>>>(
          p, DivU32::make((uint32_t)(p.Dh / 4)), DivU32::make((uint32_t)p.S),
          DivU32::make((uint32_t)p.H));
    } else if (rows > 0) {
      phi_linear_kernel<<<(int)min((rows + 7) / 8, 148ll * 16), 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
  }
  const int smem = perf_smem_floats(p.Dh) * (int)sizeof(float);
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const int most = perf_smem_floats(kPerfMaxHeadDim) * (int)sizeof(float);
    e = cudaFuncSetAttribute(phi_perf_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(phi_perf_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(phi_perf_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const dim3 grid((p.S + kPtRows - 1) / kPtRows, p.B * p.H);
  if (p.global_stab) {
    phi_init_kernel<<<max(1, (p.B * p.H + 255) / 256), 256, 0, stream>>>(p);
    if (rows > 0) {
      phi_perf_kernel<0><<<grid, kPtThreads, smem, stream>>>(p);
      phi_perf_kernel<2><<<grid, kPtThreads, smem, stream>>>(p);
    }
    phi_decode_kernel<<<max(1, (p.B * p.H + 255) / 256), 256, 0, stream>>>(p);
  } else if (rows > 0) {
    phi_perf_kernel<1><<<grid, kPtThreads, smem, stream>>>(p);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------ attention
constexpr int kLinChunk = 16;   // rows per chunk
constexpr int kLinCols = 32;    // V columns per CTA
constexpr int kLinThreads = 256;

// Shared-memory layout of both attention kernels, in floats. The S_kv slice
// and the V chunk come first so their rows stay 16-byte aligned for float4
// access; the phi chunks are padded to Df + 1 so column-wise walks avoid bank
// conflicts.
constexpr int kLinPart = kLinChunk * kLinCols + kLinChunk;  // emit's second-half partials
__host__ __device__ inline int lin_smem_floats(int Df) {
  // S_kv slice [Df][32], V chunk [16][32], partials [16][32] + [16],
  // scores [16][16], s_k [Df], phi(q) and phi(k) chunks [16][Df + 1]
  return Df * kLinCols + kLinChunk * kLinCols + kLinPart + kLinChunk * kLinChunk + Df +
         2 * kLinChunk * (Df + 1);
}

// S_kv[f][c] += sum_j phi(k_j)[f] v_j[c] over a chunk, register-tiled: thread
// t owns columns 4 (t % 8) .. + 3 of rows t / 8, t / 8 + 32, ..., two rows at
// a time, so each step of j feeds eight independent FMAs from one float4 of V
// and two phi values.
__device__ __forceinline__ void lin_accumulate(float* kv, const float* vc, const float* kc, int ld,
                                               int Df, int tid) {
  const int cq = tid % 8, fg = tid / 8;
  for (int f0 = fg; f0 < Df; f0 += 64) {
    const int f1 = f0 + 32;
    const bool has1 = f1 < Df;
    float4 a0 = *reinterpret_cast<const float4*>(kv + f0 * kLinCols + 4 * cq);
    float4 a1 = has1 ? *reinterpret_cast<const float4*>(kv + f1 * kLinCols + 4 * cq)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kLinChunk; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(vc + j * kLinCols + 4 * cq);
      const float k0 = kc[j * ld + f0];
      const float k1 = has1 ? kc[j * ld + f1] : 0.0f;
      a0.x = fmaf(k0, v.x, a0.x);
      a0.y = fmaf(k0, v.y, a0.y);
      a0.z = fmaf(k0, v.z, a0.z);
      a0.w = fmaf(k0, v.w, a0.w);
      a1.x = fmaf(k1, v.x, a1.x);
      a1.y = fmaf(k1, v.y, a1.y);
      a1.z = fmaf(k1, v.z, a1.z);
      a1.w = fmaf(k1, v.w, a1.w);
    }
    *reinterpret_cast<float4*>(kv + f0 * kLinCols + 4 * cq) = a0;
    if (has1) *reinterpret_cast<float4*>(kv + f1 * kLinCols + 4 * cq) = a1;
  }
}

// Next-chunk prefetch: with kPer > 0 (Df <= kPer * kLinThreads / kLinChunk)
// each thread holds its kPer elements of the next chunk's phi rows, and its
// share of the V slice, in registers while the current chunk computes, so a
// chunk's global loads are in flight during the previous chunk's arithmetic.
// kPer = 0: loads at the top of each chunk (feature counts above 256).
constexpr int kLinVPer = kLinChunk * kLinCols / kLinThreads;  // V elements per thread

template <int kPer>
__device__ __forceinline__ void lin_fetch_rows(float (&dst)[kPer], const float* src, int nrow,
                                               int Df, int tid) {
#pragma unroll
  for (int m = 0; m < kPer; ++m) {
    const int i = tid + m * kLinThreads;
    const int r = i / Df, f = i - r * Df;
    dst[m] = (i < kLinChunk * Df && r < nrow) ? src[(long long)r * Df + f] : 0.0f;
  }
}

template <int kPer>
__device__ __forceinline__ void lin_commit_rows(const float (&src)[kPer], float* dst, int ld,
                                                int Df, int tid) {
#pragma unroll
  for (int m = 0; m < kPer; ++m) {
    const int i = tid + m * kLinThreads;
    if (i < kLinChunk * Df) {
      const int r = i / Df, f = i - r * Df;
      dst[r * ld + f] = src[m];
    }
  }
}

template <int kPer>
__global__ void __launch_bounds__(kLinThreads) linear_attn_kernel(LinearParams p) {
  extern __shared__ __align__(16) float sm[];
  const int Df = p.Df, ld = Df + 1;
  float* kv = sm;                            // [Df][32]
  float* vc = kv + Df * kLinCols;            // [16][32]
  float* part = vc + kLinChunk * kLinCols;   // [16][32] numerators + [16] denominators
  float* sc = part + kLinPart;               // [16][16]
  float* ks = sc + kLinChunk * kLinChunk;    // [Df]
  float* qc = ks + Df;                       // [16][Df + 1]
  float* kc = qc + kLinChunk * ld;           // [16][Df + 1]
  const int tid = threadIdx.x;
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int hkv = h / (p.H / p.Hkv);
  const int d0 = blockIdx.y * kLinCols;
  const int ncol = min(kLinCols, p.D - d0);
  const long long bk = (long long)b * p.Hkv + hkv;
  // Causal with segments: this CTA covers rows [r0, r1) of one segment and
  // starts from the segment's exclusive prefix in the workspace.
  const int seg = blockIdx.z;
  const int r0 = p.causal ? seg * p.seg_len : 0;
  const int r1 = p.causal ? min(p.S, r0 + p.seg_len) : p.S;
  const float* phq = p.phi_q + ((long long)b * p.H + h) * p.S * Df;
  const float* phk = p.phi_k + bk * p.S * Df;
  const bool from_carry = p.causal && p.n_seg > 1;
  const float* kv_src = from_carry ? p.carry_kv + (long long)seg * p.B * p.Hkv * Df * p.D : p.kv_in;
  const float* ks_src = from_carry ? p.carry_ks + (long long)seg * p.B * p.Hkv * Df : p.ks_in;
  const float scale = (!from_carry && p.state_scale) ? p.state_scale[bk] : 1.0f;

  // carried state (or zero)
  for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
    const int f = i / kLinCols, c = i % kLinCols;
    kv[i] = (kv_src && c < ncol) ? kv_src[(bk * Df + f) * p.D + d0 + c] * scale : 0.0f;
  }
  for (int f = tid; f < Df; f += kLinThreads) ks[f] = ks_src ? ks_src[bk * Df + f] * scale : 0.0f;
  __syncthreads();

  auto load_rows = [&](const float* src, float* dst, int s0, int nrow) {
    for (int i = tid; i < kLinChunk * Df; i += kLinThreads) {
      const int r = i / Df, f = i % Df;
      dst[r * ld + f] = (r < nrow) ? src[(long long)(s0 + r) * Df + f] : 0.0f;
    }
  };
  auto load_v = [&](int s0, int nrow) {
    for (int i = tid; i < kLinChunk * kLinCols; i += kLinThreads) {
      const int r = i / kLinCols, c = i % kLinCols;
      vc[i] = (r < nrow && c < ncol)
                  ? load_elem(p.v, b * p.v_sb + (long long)(s0 + r) * p.v_ss + hkv * p.v_sh + d0 + c,
                              p.v_f32)
                  : 0.0f;
    }
  };
  // S_kv += phi(K_c)^T V_c, s_k += sum phi(K_c) (rows past nrow are zero)
  auto accumulate = [&]() {
    lin_accumulate(kv, vc, kc, ld, Df, tid);
    for (int f = tid; f < Df; f += kLinThreads) {
      float acc = ks[f];
#pragma unroll
      for (int j = 0; j < kLinChunk; ++j) acc += kc[j * ld + f];
      ks[f] = acc;
    }
  };
  // Out rows of the chunk: phi(q) . state (+ the causal part in sc), over
  // the denominators phi(q) . s_k (+ the scores' row sums). Thread t takes
  // row (t / 8) % 16, columns 4 (t % 8) .. + 3, and half kh = t / 128 of the
  // features; the second half's partial sums meet the first's in shared
  // memory. The denominator of a row is split over its 8 lanes.
  auto emit = [&](int s0, int nrow, bool with_scores) {
    const int cq = tid % 8, r = (tid / 8) % kLinChunk, kh = tid / 128;
    const int fh = (Df + 1) / 2, fa = kh * fh, fb = min(Df, fa + fh);
    const float* qr = qc + r * ld;
    float4 n0 = make_float4(0.f, 0.f, 0.f, 0.f), n1 = n0;
    int f = fa;
    for (; f + 1 < fb; f += 2) {  // two interleaved partial sums
      const float q0 = qr[f], q1 = qr[f + 1];
      const float4 s0v = *reinterpret_cast<const float4*>(kv + f * kLinCols + 4 * cq);
      const float4 s1v = *reinterpret_cast<const float4*>(kv + (f + 1) * kLinCols + 4 * cq);
      n0.x = fmaf(q0, s0v.x, n0.x);
      n0.y = fmaf(q0, s0v.y, n0.y);
      n0.z = fmaf(q0, s0v.z, n0.z);
      n0.w = fmaf(q0, s0v.w, n0.w);
      n1.x = fmaf(q1, s1v.x, n1.x);
      n1.y = fmaf(q1, s1v.y, n1.y);
      n1.z = fmaf(q1, s1v.z, n1.z);
      n1.w = fmaf(q1, s1v.w, n1.w);
    }
    if (f < fb) {
      const float q0 = qr[f];
      const float4 s0v = *reinterpret_cast<const float4*>(kv + f * kLinCols + 4 * cq);
      n0.x = fmaf(q0, s0v.x, n0.x);
      n0.y = fmaf(q0, s0v.y, n0.y);
      n0.z = fmaf(q0, s0v.z, n0.z);
      n0.w = fmaf(q0, s0v.w, n0.w);
    }
    float4 num = make_float4(n0.x + n1.x, n0.y + n1.y, n0.z + n1.z, n0.w + n1.w);
    float den = 0.0f;
    for (int g = fa + cq; g < fb; g += 8) den = fmaf(qr[g], ks[g], den);
#pragma unroll
    for (int m = 4; m > 0; m >>= 1) den += __shfl_xor_sync(0xffffffffu, den, m);
    if (kh == 1) {
      *reinterpret_cast<float4*>(part + r * kLinCols + 4 * cq) = num;
      if (cq == 0) part[kLinChunk * kLinCols + r] = den;
    }
    __syncthreads();
    if (kh == 0) {
      const float4 o2 = *reinterpret_cast<const float4*>(part + r * kLinCols + 4 * cq);
      num.x += o2.x;
      num.y += o2.y;
      num.z += o2.z;
      num.w += o2.w;
      den += part[kLinChunk * kLinCols + r];
      if (with_scores)
        for (int j = 0; j <= r; ++j) {
          const float sv = sc[r * kLinChunk + j];
          const float4 v = *reinterpret_cast<const float4*>(vc + j * kLinCols + 4 * cq);
          num.x = fmaf(sv, v.x, num.x);
          num.y = fmaf(sv, v.y, num.y);
          num.z = fmaf(sv, v.z, num.z);
          num.w = fmaf(sv, v.w, num.w);
          den += sv;
        }
      den += p.eps;
      if (r < nrow) {
        const float vals[4] = {num.x / den, num.y / den, num.z / den, num.w / den};
        const long long off = b * p.o_sb + (long long)(s0 + r) * p.o_ss + h * p.o_sh + d0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 4 * cq + e;
          if (c >= ncol) continue;
          if (p.o_f32)
            reinterpret_cast<float*>(p.o)[off + c] = vals[e];
          else
            reinterpret_cast<__nv_bfloat16*>(p.o)[off + c] = __float2bfloat16(vals[e]);
        }
      }
    }
  };

  constexpr int kP = kPer > 0 ? kPer : 1;
  float rq[kP], rk[kP], rv[kLinVPer];
  auto fetch_v = [&](int s0, int nrow) {
#pragma unroll
    for (int m = 0; m < kLinVPer; ++m) {
      const int i = tid + m * kLinThreads, r = i / kLinCols, c = i % kLinCols;
      rv[m] = (r < nrow && c < ncol)
                  ? load_elem(p.v, b * p.v_sb + (long long)(s0 + r) * p.v_ss + hkv * p.v_sh + d0 + c,
                              p.v_f32)
                  : 0.0f;
    }
  };
  auto commit_v = [&]() {
#pragma unroll
    for (int m = 0; m < kLinVPer; ++m) vc[tid + m * kLinThreads] = rv[m];
  };

  if (p.causal) {
    if constexpr (kPer > 0) {
      if (r0 < r1) {
        const int n0 = min(kLinChunk, r1 - r0);
        lin_fetch_rows<kPer>(rq, phq + (long long)r0 * Df, n0, Df, tid);
        lin_fetch_rows<kPer>(rk, phk + (long long)r0 * Df, n0, Df, tid);
        fetch_v(r0, n0);
      }
    }
    for (int s0 = r0; s0 < r1; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, r1 - s0);
      if constexpr (kPer > 0) {
        lin_commit_rows<kPer>(rq, qc, ld, Df, tid);
        lin_commit_rows<kPer>(rk, kc, ld, Df, tid);
        commit_v();
        __syncthreads();
        const int s1 = s0 + kLinChunk;
        if (s1 < r1) {
          const int n1 = min(kLinChunk, r1 - s1);
          lin_fetch_rows<kPer>(rq, phq + (long long)s1 * Df, n1, Df, tid);
          lin_fetch_rows<kPer>(rk, phk + (long long)s1 * Df, n1, Df, tid);
          fetch_v(s1, n1);
        }
      } else {
        load_rows(phq + (long long)s0 * Df, qc, 0, nrow);
        load_rows(phk + (long long)s0 * Df, kc, 0, nrow);
        load_v(s0, nrow);
        __syncthreads();
      }
      {  // scores phi(q_i).phi(k_j) for j <= i inside the chunk, four partial sums
        const int i = tid / kLinChunk, j = tid % kLinChunk;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        if (j <= i) {
          const float* qi = qc + i * ld;
          const float* kj = kc + j * ld;
          int f = 0;
          for (; f + 3 < Df; f += 4) {
            a0 = fmaf(qi[f], kj[f], a0);
            a1 = fmaf(qi[f + 1], kj[f + 1], a1);
            a2 = fmaf(qi[f + 2], kj[f + 2], a2);
            a3 = fmaf(qi[f + 3], kj[f + 3], a3);
          }
          for (; f < Df; ++f) a0 = fmaf(qi[f], kj[f], a0);
        }
        sc[i * kLinChunk + j] = (a0 + a1) + (a2 + a3);
      }
      __syncthreads();
      emit(s0, nrow, true);  // uses the state before this chunk
      __syncthreads();
      accumulate();
      __syncthreads();
    }
  } else {
    // keys and values into the state, then the queries against it
    if constexpr (kPer > 0) {
      lin_fetch_rows<kPer>(rk, phk, min(kLinChunk, p.S), Df, tid);
      fetch_v(0, min(kLinChunk, p.S));
    }
    for (int s0 = 0; s0 < p.S; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, p.S - s0);
      if constexpr (kPer > 0) {
        lin_commit_rows<kPer>(rk, kc, ld, Df, tid);
        commit_v();
        __syncthreads();
        const int s1 = s0 + kLinChunk;
        if (s1 < p.S) {
          lin_fetch_rows<kPer>(rk, phk + (long long)s1 * Df, min(kLinChunk, p.S - s1), Df, tid);
          fetch_v(s1, min(kLinChunk, p.S - s1));
        }
      } else {
        load_rows(phk + (long long)s0 * Df, kc, 0, nrow);
        load_v(s0, nrow);
        __syncthreads();
      }
      accumulate();
      __syncthreads();
    }
    if constexpr (kPer > 0) lin_fetch_rows<kPer>(rq, phq, min(kLinChunk, p.S), Df, tid);
    for (int s0 = 0; s0 < p.S; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, p.S - s0);
      if constexpr (kPer > 0) {
        lin_commit_rows<kPer>(rq, qc, ld, Df, tid);
        __syncthreads();
        const int s1 = s0 + kLinChunk;
        if (s1 < p.S)
          lin_fetch_rows<kPer>(rq, phq + (long long)s1 * Df, min(kLinChunk, p.S - s1), Df, tid);
      } else {
        load_rows(phq + (long long)s0 * Df, qc, 0, nrow);
        __syncthreads();
      }
      emit(s0, nrow, false);
      __syncthreads();
    }
  }
  // state out: one query head per kv group writes it (with segments the scan
  // kernel writes the total instead)
  if (h % (p.H / p.Hkv) == 0 && !from_carry) {
    if (p.kv_out)
      for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
        const int f = i / kLinCols, c = i % kLinCols;
        if (c < ncol) p.kv_out[(bk * Df + f) * p.D + d0 + c] = kv[i];
      }
    if (p.ks_out && blockIdx.y == 0)
      for (int f = tid; f < Df; f += kLinThreads) p.ks_out[bk * Df + f] = ks[f];
  }
}

// Phase A of the segmented causal pass: per (segment, b, kv head, column
// slice) the segment's sums of phi(k) v^T and phi(k) into the workspace.
template <int kPer>
__global__ void __launch_bounds__(kLinThreads) linear_segsum_kernel(LinearParams p) {
  extern __shared__ __align__(16) float sm[];
  const int Df = p.Df, ld = Df + 1;
  float* kv = sm;                        // [Df][32]
  float* vc = kv + Df * kLinCols;        // [16][32]
  float* ks = vc + kLinChunk * kLinCols; // [Df]
  float* kc = ks + Df;                   // [16][Df + 1]
  const int tid = threadIdx.x;
  const int bk = blockIdx.x, b = bk / p.Hkv, hkv = bk % p.Hkv;
  const int d0 = blockIdx.y * kLinCols;
  const int ncol = min(kLinCols, p.D - d0);
  const int seg = blockIdx.z;
  const int r0 = seg * p.seg_len, r1 = min(p.S, r0 + p.seg_len);
  const float* phk = p.phi_k + (long long)bk * p.S * Df;
  for (int i = tid; i < Df * kLinCols; i += kLinThreads) kv[i] = 0.0f;
  for (int f = tid; f < Df; f += kLinThreads) ks[f] = 0.0f;
  constexpr int kP = kPer > 0 ? kPer : 1;
  float rk[kP], rv[kLinVPer];
  auto fetch = [&](int s0, int nrow) {
    if constexpr (kPer > 0) lin_fetch_rows<kPer>(rk, phk + (long long)s0 * Df, nrow, Df, tid);
#pragma unroll
    for (int m = 0; m < kLinVPer; ++m) {
      const int i = tid + m * kLinThreads, r = i / kLinCols, c = i % kLinCols;
      rv[m] = (r < nrow && c < ncol)
                  ? load_elem(p.v, b * p.v_sb + (long long)(s0 + r) * p.v_ss + hkv * p.v_sh + d0 + c,
                              p.v_f32)
                  : 0.0f;
    }
  };
  if (r0 < r1) fetch(r0, min(kLinChunk, r1 - r0));
  for (int s0 = r0; s0 < r1; s0 += kLinChunk) {
    const int nrow = min(kLinChunk, r1 - s0);
    __syncthreads();
    if constexpr (kPer > 0) {
      lin_commit_rows<kPer>(rk, kc, ld, Df, tid);
    } else {
      for (int i = tid; i < kLinChunk * Df; i += kLinThreads) {
        const int r = i / Df, f = i % Df;
        kc[r * ld + f] = (r < nrow) ? phk[(long long)(s0 + r) * Df + f] : 0.0f;
      }
    }
#pragma unroll
    for (int m = 0; m < kLinVPer; ++m) vc[tid + m * kLinThreads] = rv[m];
    __syncthreads();
    if (s0 + kLinChunk < r1) fetch(s0 + kLinChunk, min(kLinChunk, r1 - s0 - kLinChunk));
    lin_accumulate(kv, vc, kc, ld, Df, tid);
    for (int f = tid; f < Df; f += kLinThreads) {
      float acc = ks[f];
#pragma unroll
      for (int j = 0; j < kLinChunk; ++j) acc += kc[j * ld + f];
      ks[f] = acc;
    }
  }
  __syncthreads();
  float* okv = p.carry_kv + (long long)seg * p.B * p.Hkv * Df * p.D;
  for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
    const int f = i / kLinCols, c = i % kLinCols;
    if (c < ncol) okv[((long long)bk * Df + f) * p.D + d0 + c] = kv[i];
  }
  if (blockIdx.y == 0) {
    float* oks = p.carry_ks + (long long)seg * p.B * p.Hkv * Df;
    for (int f = tid; f < Df; f += kLinThreads) oks[(long long)bk * Df + f] = ks[f];
  }
}

// Phase B: segment sums -> exclusive prefixes in place, starting from the
// carried state (times its scale); the total goes to kv_out / ks_out.
__global__ void linear_scan_kernel(LinearParams p) {
  const long long nkv = (long long)p.B * p.Hkv * p.Df * p.D;
  const long long nks = (long long)p.B * p.Hkv * p.Df;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nkv + nks;
       i += (long long)gridDim.x * blockDim.x) {
    const bool is_kv = i < nkv;
    const long long e = is_kv ? i : i - nkv;
    const long long bk = is_kv ? e / ((long long)p.Df * p.D) : e / p.Df;
    float* buf = is_kv ? p.carry_kv : p.carry_ks;
    const long long stride = is_kv ? nkv : nks;
    const float* init = is_kv ? p.kv_in : p.ks_in;
    float run = init ? init[e] * (p.state_scale ? p.state_scale[bk] : 1.0f) : 0.0f;
    for (int z = 0; z < p.n_seg; ++z) {
      const float t = buf[z * stride + e];
      buf[z * stride + e] = run;
      run += t;
    }
    float* out = is_kv ? p.kv_out : p.ks_out;
    if (out) out[e] = run;
  }
}

// Segments of the causal pass: enough CTAs for two waves, segments of at
// least 256 rows.
// Segments of the causal pass (segments of at least 256 rows): the count
// whose CTAs best fill whole waves, taking the first that fills them to 95%.
// A wave is 148 SMs times the CTAs one SM holds: two (the attention kernel's
// registers allow two), fewer when shared memory does not.
int linear_segments(int B, int H, int S, int D, int Df) {
  const long long ctas = (long long)B * H * ((D + kLinCols - 1) / kLinCols);
  const int smem = lin_smem_floats(Df) * (int)sizeof(float);
  const long long slots = 148ll * max(1, min(2, (227 * 1024) / max(smem, 1)));
  const int max_n = max(1, min(S / 256, 64));
  int best = 1;
  double best_util = 0.0;
  for (int n = 1; n <= max_n; ++n) {
    const long long c = ctas * n;
    const double util = (double)c / (double)(((c + slots - 1) / slots) * slots);
    if (util > best_util + 1e-9) {
      best = n;
      best_util = util;
    }
    if (util >= 0.95) break;
  }
  return best;
}

size_t linear_workspace_bytes(int B, int H, int Hkv, int S, int Df, int D, int causal) {
  const int n = causal ? linear_segments(B, H, S, D, Df) : 1;
  if (n <= 1) return 0;
  return (size_t)n * B * Hkv * ((size_t)Df * D + Df) * sizeof(float);
}

int linear_attn_max_features() {
  // lin_smem_floats(Df) = (kLinCols + 1 + 2 kLinChunk) Df + the Df-free terms
  const int fixed = kLinChunk * kLinCols + kLinPart + kLinChunk * kLinChunk + 2 * kLinChunk;
  return (227 * 1024 / (int)sizeof(float) - fixed) / (kLinCols + 1 + 2 * kLinChunk);
}

cudaError_t launch_linear_attn(const LinearParams& p, cudaStream_t stream) {
  if (p.B == 0 || p.H == 0 || p.D == 0) return cudaSuccess;
  const int smem = lin_smem_floats(p.Df) * (int)sizeof(float);
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    const void* fns[8] = {(const void*)linear_attn_kernel<0>, (const void*)linear_attn_kernel<4>,
                          (const void*)linear_attn_kernel<8>, (const void*)linear_attn_kernel<16>,
                          (const void*)linear_segsum_kernel<0>,
                          (const void*)linear_segsum_kernel<4>,
                          (const void*)linear_segsum_kernel<8>,
                          (const void*)linear_segsum_kernel<16>};
    for (int i = 0; i < 8 && e == cudaSuccess; ++i) e = cudaFuncSetAttribute(fns[i], a, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  // prefetch width: phi elements per thread per chunk
  const int per = p.Df <= 64 ? 4 : p.Df <= 128 ? 8 : p.Df <= 256 ? 16 : 0;
  const int nslice = (p.D + kLinCols - 1) / kLinCols;
  LinearParams q = p;
  q.n_seg = p.causal ? linear_segments(p.B, p.H, p.S, p.D, p.Df) : 1;
  q.seg_len = (p.S + q.n_seg - 1) / max(q.n_seg, 1);
  if (q.n_seg > 1) {
    if (!p.carry_kv || !p.carry_ks) return cudaErrorInvalidValue;  // the ABI checks the workspace
    const dim3 sg(p.B * p.Hkv, nslice, q.n_seg);
    switch (per) {
      case 4: linear_segsum_kernel<4><<<sg, kLinThreads, smem, stream>>>(q); break;
      case 8: linear_segsum_kernel<8><<<sg, kLinThreads, smem, stream>>>(q); break;
      case 16: linear_segsum_kernel<16><<<sg, kLinThreads, smem, stream>>>(q); break;
      default: linear_segsum_kernel<0><<<sg, kLinThreads, smem, stream>>>(q); break;
    }
    const long long n = (long long)p.B * p.Hkv * p.Df * (p.D + 1);
    linear_scan_kernel<<<(int)min((n + 255) / 256, 148ll * 8), 256, 0, stream>>>(q);
  }
  dim3 grid(p.B * p.H, nslice, q.n_seg);
  switch (per) {
    case 4: linear_attn_kernel<4><<<grid, kLinThreads, smem, stream>>>(q); break;
    case 8: linear_attn_kernel<8><<<grid, kLinThreads, smem, stream>>>(q); break;
    case 16: linear_attn_kernel<16><<<grid, kLinThreads, smem, stream>>>(q); break;
    default: linear_attn_kernel<0><<<grid, kLinThreads, smem, stream>>>(q); break;
  }
  return cudaGetLastError();
}

}  // namespace enl
