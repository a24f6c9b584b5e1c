// K4: linearized attention (the reference's attention_kernel="linear" and
// "performer" options), nn/attention_kernels.py:58-143 and the cached step of
// nn/kvcache.py:217-260.
//
// Both kernels replace softmax(q.k) by phi(q).phi(k), so attention
// reassociates into phi(Q) (phi(K)^T V) / (phi(Q) . sum phi(K)) and never
// forms a score matrix. Two kernels, fp32 arithmetic throughout:
//   phi_kernel          feature map of one head view into (B, H, S, Df) fp32:
//                       elu(x) + 1, or exp(w.x' - |x'|^2/2 - stab)/sqrt(Df)
//                       with x' = x / Dh^(1/4) and a row or per-(b, h) global
//                       stabilizer (phi_max_kernel reduces the global one);
//   linear_attn_kernel  per (b, query head, 32-column slice of V): causal
//                       prefix sums over 16-row chunks (intra-chunk scores
//                       phi(q_i).phi(k_j), j <= i, plus the carried state
//                       S_kv = sum phi(k) v^T and s_k = sum phi(k)), or the
//                       two global sums when non-causal. A state can be
//                       carried in (scaled) and returned, which is the decode
//                       step: a fixed-size state instead of a growing cache.
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

constexpr int kPhiMaxFeatPerLane = 32;  // Df <= 1024

// One warp per (b, s, h) row. Performer: lane l owns features l, l + 32, ...
__device__ __forceinline__ void performer_row(const PhiParams& p, long long xoff, float* xs,
                                              int lane, float* proj, float& sq) {
  const float inv = rsqrtf(sqrtf((float)p.Dh));  // Dh^(-1/4)
  float s2 = 0.0f;
  for (int d = lane; d < p.Dh; d += 32) {
    const float v = load_elem(p.x, xoff + d, p.in_f32) * inv;
    xs[d] = v;
    s2 += v * v;
  }
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  sq = 0.5f * s2;
#pragma unroll 1
  for (int k = 0; k < kPhiMaxFeatPerLane; ++k) {
    const int f = lane + 32 * k;
    if (f >= p.Df) break;
    const float* w = p.omega + (long long)f * p.Dh;
    float acc = 0.0f;
    for (int d = 0; d < p.Dh; ++d) acc = fmaf(xs[d], __ldg(w + d), acc);
    proj[k] = acc;
  }
}

__global__ void phi_init_kernel(PhiParams p) {
  const int n = p.B * p.H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    reinterpret_cast<int*>(p.stab)[i] = ord_enc(p.stab_floor ? p.stab_floor[i] : -INFINITY);
}

// Global stabilizer: max over rows and features of w.x' per (b, h).
__global__ void __launch_bounds__(256) phi_max_kernel(PhiParams p) {
  extern __shared__ float xs_all[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* xs = xs_all + warp * p.Dh;
  const long long rows = (long long)p.B * p.S * p.H;
  for (long long r = (long long)blockIdx.x * 8 + warp; r < rows; r += (long long)gridDim.x * 8) {
    const int h = (int)(r % p.H);
    const long long bs = r / p.H;
    const int s = (int)(bs % p.S), b = (int)(bs / p.S);
    float proj[kPhiMaxFeatPerLane];
    float sq;
    performer_row(p, b * p.sb + s * p.ss + h * p.sh, xs, lane, proj, sq);
    float m = -INFINITY;
    for (int k = 0; k < kPhiMaxFeatPerLane && lane + 32 * k < p.Df; ++k)
      if (proj[k] == proj[k]) m = fmaxf(m, proj[k]);  // NaN rows do not vote
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && m > -INFINITY) atomicMax(reinterpret_cast<int*>(p.stab) + b * p.H + h, ord_enc(m));
    __syncwarp();
  }
}

__global__ void __launch_bounds__(256) phi_kernel(PhiParams p) {
  extern __shared__ float xs_all[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* xs = xs_all + warp * p.Dh;
  const long long rows = (long long)p.B * p.S * p.H;
  const float norm = rsqrtf((float)p.Df);
  for (long long r = (long long)blockIdx.x * 8 + warp; r < rows; r += (long long)gridDim.x * 8) {
    const int h = (int)(r % p.H);
    const long long bs = r / p.H;
    const int s = (int)(bs % p.S), b = (int)(bs / p.S);
    const long long xoff = b * p.sb + s * p.ss + h * p.sh;
    float* out = p.phi + (((long long)b * p.H + h) * p.S + s) * p.Df;
    if (p.kernel == 0) {
      for (int d = lane; d < p.Dh; d += 32) {
        const float v = load_elem(p.x, xoff + d, p.in_f32);
        out[d] = v > 0.0f ? v + 1.0f : expf(fminf(v, 0.0f));  // elu(v) + 1
      }
      continue;
    }
    float proj[kPhiMaxFeatPerLane];
    float sq;
    performer_row(p, xoff, xs, lane, proj, sq);
    float stab;
    if (p.global_stab) {
      stab = ord_dec(reinterpret_cast<const int*>(p.stab)[b * p.H + h]);
    } else {
      stab = -INFINITY;
      for (int k = 0; k < kPhiMaxFeatPerLane && lane + 32 * k < p.Df; ++k) stab = fmaxf(stab, proj[k]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) stab = fmaxf(stab, __shfl_xor_sync(0xffffffffu, stab, o));
    }
    for (int k = 0; k < kPhiMaxFeatPerLane && lane + 32 * k < p.Df; ++k)
      out[lane + 32 * k] = expf(proj[k] - sq - stab) * norm;
    __syncwarp();
  }
}

__global__ void phi_decode_kernel(PhiParams p) {
  const int n = p.B * p.H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    int* e = reinterpret_cast<int*>(p.stab) + i;
    p.stab[i] = ord_dec(*e);
  }
}

cudaError_t launch_phi(const PhiParams& p, cudaStream_t stream) {
  const long long rows = (long long)p.B * p.S * p.H;
  const int smem = 8 * p.Dh * (int)sizeof(float);
  const int blocks = (int)min((rows + 7) / 8, 148ll * 16);
  if (p.kernel == 1 && p.global_stab) {
    phi_init_kernel<<<max(1, (p.B * p.H + 255) / 256), 256, 0, stream>>>(p);
    if (rows > 0) phi_max_kernel<<<blocks, 256, smem, stream>>>(p);
  }
  if (rows > 0) phi_kernel<<<blocks, 256, smem, stream>>>(p);
  if (p.kernel == 1 && p.global_stab)
    phi_decode_kernel<<<max(1, (p.B * p.H + 255) / 256), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

// ------------------------------------------------------------ attention
constexpr int kLinChunk = 16;   // rows per chunk
constexpr int kLinCols = 32;    // V columns per CTA
constexpr int kLinThreads = 256;

__host__ __device__ inline int lin_smem_floats(int Df) {
  // S_kv slice [Df][32], s_k [Df], phi(q) and phi(k) chunks [16][Df + 1],
  // V chunk [16][32], scores [16][16], denominators [16]
  return Df * kLinCols + Df + 2 * kLinChunk * (Df + 1) + kLinChunk * kLinCols +
         kLinChunk * kLinChunk + kLinChunk;
}

__global__ void __launch_bounds__(kLinThreads) linear_attn_kernel(LinearParams p) {
  extern __shared__ float sm[];
  const int Df = p.Df, ld = Df + 1;
  float* kv = sm;                          // [Df][32]
  float* ks = kv + Df * kLinCols;          // [Df]
  float* qc = ks + Df;                     // [16][Df + 1]
  float* kc = qc + kLinChunk * ld;         // [16][Df + 1]
  float* vc = kc + kLinChunk * ld;         // [16][32]
  float* sc = vc + kLinChunk * kLinCols;   // [16][16]
  float* dn = sc + kLinChunk * kLinChunk;  // [16]
  const int tid = threadIdx.x;
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const int hkv = h / (p.H / p.Hkv);
  const int d0 = blockIdx.y * kLinCols;
  const int ncol = min(kLinCols, p.D - d0);
  const long long bk = (long long)b * p.Hkv + hkv;
  const float* phq = p.phi_q + ((long long)b * p.H + h) * p.S * Df;
  const float* phk = p.phi_k + bk * p.S * Df;
  const float scale = p.state_scale ? p.state_scale[bk] : 1.0f;

  // carried state (or zero)
  for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
    const int f = i / kLinCols, c = i % kLinCols;
    kv[i] = (p.kv_in && c < ncol) ? p.kv_in[(bk * Df + f) * p.D + d0 + c] * scale : 0.0f;
  }
  for (int f = tid; f < Df; f += kLinThreads) ks[f] = p.ks_in ? p.ks_in[bk * Df + f] * scale : 0.0f;
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
    for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
      const int f = i / kLinCols, c = i % kLinCols;
      float acc = kv[i];
#pragma unroll
      for (int j = 0; j < kLinChunk; ++j) acc = fmaf(kc[j * ld + f], vc[j * kLinCols + c], acc);
      kv[i] = acc;
    }
    for (int f = tid; f < Df; f += kLinThreads) {
      float acc = ks[f];
#pragma unroll
      for (int j = 0; j < kLinChunk; ++j) acc += kc[j * ld + f];
      ks[f] = acc;
    }
  };
  // out rows of the chunk: (causal part in sc) + phi(q) . state
  auto emit = [&](int s0, int nrow, bool with_scores) {
    // denominators
    if (tid < kLinChunk) {
      const int r = tid;
      float den = 0.0f;
      for (int f = 0; f < Df; ++f) den = fmaf(qc[r * ld + f], ks[f], den);
      if (with_scores)
        for (int j = 0; j <= r; ++j) den += sc[r * kLinChunk + j];
      dn[r] = den + p.eps;
    }
    __syncthreads();
    for (int i = tid; i < kLinChunk * kLinCols; i += kLinThreads) {
      const int r = i / kLinCols, c = i % kLinCols;
      if (r >= nrow || c >= ncol) continue;
      float num = 0.0f;
      for (int f = 0; f < Df; ++f) num = fmaf(qc[r * ld + f], kv[f * kLinCols + c], num);
      if (with_scores)
        for (int j = 0; j <= r; ++j) num = fmaf(sc[r * kLinChunk + j], vc[j * kLinCols + c], num);
      const float o = num / dn[r];
      const long long off = b * p.o_sb + (long long)(s0 + r) * p.o_ss + h * p.o_sh + d0 + c;
      if (p.o_f32)
        reinterpret_cast<float*>(p.o)[off] = o;
      else
        reinterpret_cast<__nv_bfloat16*>(p.o)[off] = __float2bfloat16(o);
    }
  };

  if (p.causal) {
    for (int s0 = 0; s0 < p.S; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, p.S - s0);
      load_rows(phq + (long long)s0 * Df, qc, 0, nrow);
      load_rows(phk + (long long)s0 * Df, kc, 0, nrow);
      load_v(s0, nrow);
      __syncthreads();
      {  // scores phi(q_i).phi(k_j) for j <= i inside the chunk
        const int i = tid / kLinChunk, j = tid % kLinChunk;
        float acc = 0.0f;
        if (j <= i)
          for (int f = 0; f < Df; ++f) acc = fmaf(qc[i * ld + f], kc[j * ld + f], acc);
        sc[i * kLinChunk + j] = acc;
      }
      __syncthreads();
      emit(s0, nrow, true);  // uses the state before this chunk
      __syncthreads();
      accumulate();
      __syncthreads();
    }
  } else {
    for (int s0 = 0; s0 < p.S; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, p.S - s0);
      load_rows(phk + (long long)s0 * Df, kc, 0, nrow);
      load_v(s0, nrow);
      __syncthreads();
      accumulate();
      __syncthreads();
    }
    for (int s0 = 0; s0 < p.S; s0 += kLinChunk) {
      const int nrow = min(kLinChunk, p.S - s0);
      load_rows(phq + (long long)s0 * Df, qc, 0, nrow);
      __syncthreads();
      emit(s0, nrow, false);
      __syncthreads();
    }
  }
  // state out: one query head per kv group writes it
  if (h % (p.H / p.Hkv) == 0) {
    if (p.kv_out)
      for (int i = tid; i < Df * kLinCols; i += kLinThreads) {
        const int f = i / kLinCols, c = i % kLinCols;
        if (c < ncol) p.kv_out[(bk * Df + f) * p.D + d0 + c] = kv[i];
      }
    if (p.ks_out && blockIdx.y == 0)
      for (int f = tid; f < Df; f += kLinThreads) p.ks_out[bk * Df + f] = ks[f];
  }
}

int linear_attn_max_features() {
  return (227 * 1024 / (int)sizeof(float) - (kLinChunk * kLinCols + kLinChunk * kLinChunk +
                                              kLinChunk + 2 * kLinChunk)) /
         (kLinCols + 1 + 2 * kLinChunk);
}

cudaError_t launch_linear_attn(const LinearParams& p, cudaStream_t stream) {
  if (p.B == 0 || p.H == 0 || p.D == 0) return cudaSuccess;
  const int smem = lin_smem_floats(p.Df) * (int)sizeof(float);
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(linear_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(p.B * p.H, (p.D + kLinCols - 1) / kLinCols);
  linear_attn_kernel<<<grid, kLinThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace enl
