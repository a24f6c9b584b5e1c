// K2: bandwidth-bound split-KV decode, plus the log-sum-exp merge.
//
// Replaces the one-token attention of the reference's cached step,
// nn/kvcache.py:198-213 (scores / sqrt(Dh), ALiBi at absolute positions,
// softmax, attn @ V). The reference re-concatenates and re-reads the whole
// cache each step; here the cache is a preallocated device buffer
// (B, Hkv, capacity, D) and each step streams the live slots exactly once.
//
// Grid: (n_splits, B * Hkv). A CTA owns one contiguous slot range of one
// (batch, kv head) and all H/Hkv query heads that share it (GQA group-major:
// query head h reads kv head h / (H/Hkv), nn/forward.py:165-171), so every K/V
// byte is read once per step whatever the group size. D/8 lanes share a key
// row: each lane loads 16 contiguous bytes (128-bit, L1 no-allocate), so a
// warp reads whole 256-byte rows back to back. Scores reduce across the lane
// group with xor-shuffles; the softmax runs online in the log2 domain.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Eight consecutive head-dim elements of one lane: one 16-byte load of bf16,
// two of fp32 (raw words; unpack8 converts).
template <bool kF32>
struct Chunk {
  uint4 w[kF32 ? 2 : 1];
};

template <bool kF32>
__device__ __forceinline__ Chunk<kF32> ld_chunk(const uint8_t* p) {
  Chunk<kF32> c;
  c.w[0] = ld_stream(p);
  if constexpr (kF32) c.w[1] = ld_stream(p + 16);
  return c;
}

template <bool kF32>
__device__ __forceinline__ Chunk<kF32> zero_chunk() {
  Chunk<kF32> c;
#pragma unroll
  for (int i = 0; i < (kF32 ? 2 : 1); ++i) c.w[i] = make_uint4(0, 0, 0, 0);
  return c;
}

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  f[0] = bf16lo_to_f32(w.x);
  f[1] = bf16hi_to_f32(w.x);
  f[2] = bf16lo_to_f32(w.y);
  f[3] = bf16hi_to_f32(w.y);
  f[4] = bf16lo_to_f32(w.z);
  f[5] = bf16hi_to_f32(w.z);
  f[6] = bf16lo_to_f32(w.w);
  f[7] = bf16hi_to_f32(w.w);
}

template <bool kF32>
__device__ __forceinline__ void unpack8(const Chunk<kF32>& c, float (&f)[8]) {
  if constexpr (kF32) {
    f[0] = __uint_as_float(c.w[0].x);
    f[1] = __uint_as_float(c.w[0].y);
    f[2] = __uint_as_float(c.w[0].z);
    f[3] = __uint_as_float(c.w[0].w);
    f[4] = __uint_as_float(c.w[1].x);
    f[5] = __uint_as_float(c.w[1].y);
    f[6] = __uint_as_float(c.w[1].z);
    f[7] = __uint_as_float(c.w[1].w);
  } else {
    unpack8(c.w[0], f);
  }
}

template <int D, int G>
struct DecodeCfg {
  static constexpr int kThreads = 128;
  static constexpr int kLanesPerKey = D / 8;
  static constexpr int kKeysPerWarp = 32 / kLanesPerKey;
  static constexpr int kGroups = (kThreads / 32) * kKeysPerWarp;  // key groups per CTA
  static constexpr int kUnroll = (G >= 4) ? 2 : 4;  // bounded by registers at large G
};

template <int D, int G, bool kF32>
__global__ void __launch_bounds__(128) attn_decode_kernel(const DecodeParams p) {
  constexpr int kEsz = kF32 ? 4 : 2;  // element bytes
  using Cfg = DecodeCfg<D, G>;
  constexpr int LPK = Cfg::kLanesPerKey;
  constexpr int NG = Cfg::kGroups;
  constexpr int U = Cfg::kUnroll;

  const int split = blockIdx.x;
  const int bkv = blockIdx.y;
  const int b = bkv / p.Hkv;
  const int hkv = bkv % p.Hkv;
  const int lane = threadIdx.x % 32;
  const int warp = threadIdx.x / 32;
  const int sub = lane % LPK;                        // which 8-element slice of D
  const int group = warp * Cfg::kKeysPerWarp + lane / LPK;

  const int s_begin = p.slot_begin + split * p.split_len;
  const int s_end = min(p.slot_end, s_begin + p.split_len);

  // Lanes whose 8-element slice lies past the tensors' head dim read zeros.
  const bool lane_live = sub * 8 < p.d_real;
  // Queries of the GQA group, pre-scaled into the log2 domain.
  float q[G][8];
  float slope2[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int h = hkv * G + g;
    const uint8_t* qp = reinterpret_cast<const uint8_t*>(p.q) +
                        ((long long)b * p.q_sb + (long long)h * p.q_sh + sub * 8) * kEsz;
    unpack8(lane_live ? ld_chunk<kF32>(qp) : zero_chunk<kF32>(), q[g]);
#pragma unroll
    for (int i = 0; i < 8; ++i) q[g][i] *= p.scale_log2;
    slope2[g] = p.alibi ? p.alibi[h] * 1.4426950408889634f : 0.0f;
  }

  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.0f;
  }

  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(p.k) +
                         ((long long)b * p.k_sb + (long long)hkv * p.k_sh + sub * 8) * kEsz;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(p.v) +
                         ((long long)b * p.v_sb + (long long)hkv * p.v_sh + sub * 8) * kEsz;
  const long long k_ss = p.k_ss * kEsz, v_ss = p.v_ss * kEsz;  // bytes per slot

  // The loop bound is warp-uniform (the shuffles below need the whole warp);
  // each lane group masks its own slots past the end of the split.
  const int group_in_warp = lane / LPK;
  for (int sw = s_begin + warp * Cfg::kKeysPerWarp; sw < s_end; sw += NG * U) {
    const int s0 = sw + group_in_warp;
    Chunk<kF32> kr[U], vr[U];
    bool valid[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int slot = s0 + u * NG;
      valid[u] = slot < s_end;
      if (valid[u] && lane_live) {
        kr[u] = ld_chunk<kF32>(kbase + (long long)slot * k_ss);
        vr[u] = ld_chunk<kF32>(vbase + (long long)slot * v_ss);
      } else {
        kr[u] = zero_chunk<kF32>();
        vr[u] = zero_chunk<kF32>();
      }
    }
    float kf[U][8], vf[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      unpack8(kr[u], kf[u]);
      unpack8(vr[u], vf[u]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(q[g][i], kf[u][i], d);
#pragma unroll
        for (int off = LPK / 2; off > 0; off /= 2) d += __shfl_xor_sync(0xffffffffu, d, off);
        if (slope2[g] != 0.0f) {
          // ALiBi at absolute positions: -slope * (pos_q - pos_k), nn/kvcache.py:199-203.
          const float dist = (float)(p.q_minus_k0 - (long long)(s0 + u * NG));
          d = fmaf(-slope2[g], dist, d);
        }
        s[u] = valid[u] ? d : -INFINITY;
      }
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u) mx = fmaxf(mx, s[u]);
      if (mx != -INFINITY) {
        const float corr = fast_exp2(m[g] - mx);  // exp2(-inf) == 0 on the first keys
        l[g] *= corr;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[g][i] *= corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float pu = fast_exp2(s[u] - mx);
          l[g] += pu;
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[g][i] = fmaf(pu, vf[u][i], acc[g][i]);
        }
        m[g] = mx;
      }
    }
  }

  // Merge the NG key groups of this CTA through shared memory.
  __shared__ float sm_m[G][NG];
  __shared__ float sm_l[G][NG];
  __shared__ float sm_acc[G][NG][D];
  if (sub == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[g][group] = m[g];
      sm_l[g][group] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) sm_acc[g][group][sub * 8 + i] = acc[g][i];
  __syncthreads();

  for (int idx = threadIdx.x; idx < G * D; idx += Cfg::kThreads) {
    const int g = idx / D;
    const int d = idx % D;
    if (d >= p.d_real) continue;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < NG; ++k) M = fmaxf(M, sm_m[g][k]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int k = 0; k < NG; ++k) {
        const float w = fast_exp2(sm_m[g][k] - M);
        L = fmaf(w, sm_l[g][k], L);
        O = fmaf(w, sm_acc[g][k][d], O);
      }
    }
    const int h = hkv * G + g;
    const float lse = (M == -INFINITY) ? -INFINITY : (M + log2f(L)) * 0.6931471805599453f;
    if (p.n_splits == 1) {
      const float val = O / L;  // 0/0 -> NaN when no key was visible
      if (p.out_fp32) {
        reinterpret_cast<float*>(p.o)[(long long)b * p.o_sb + (long long)h * p.o_sh + d] = val;
      } else {
        reinterpret_cast<__nv_bfloat16*>(p.o)[(long long)b * p.o_sb + (long long)h * p.o_sh + d] =
            __float2bfloat16_rn(val);
      }
      if (d == 0 && p.lse) p.lse[(long long)b * p.H + h] = lse;
    } else {
      const long long row = ((long long)split * p.B + b) * p.H + h;
      p.part_o[row * D + d] = (L > 0.0f) ? O / L : 0.0f;
      if (d == 0) p.part_lse[row] = lse;
    }
  }
}

template <int D, int G>
static cudaError_t launch_decode_g(const DecodeParams& p, cudaStream_t stream) {
  dim3 grid(p.n_splits, p.B * p.Hkv);
  if (p.in_fp32)
    attn_decode_kernel<D, G, true><<<grid, DecodeCfg<D, G>::kThreads, 0, stream>>>(p);
  else
    attn_decode_kernel<D, G, false><<<grid, DecodeCfg<D, G>::kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream) {
  const int G = p.H / p.Hkv;
  cudaError_t e;
  switch (G) {
    case 1: e = launch_decode_g<D, 1>(p, stream); break;
    case 2: e = launch_decode_g<D, 2>(p, stream); break;
    case 4: e = launch_decode_g<D, 4>(p, stream); break;
    case 8: e = launch_decode_g<D, 8>(p, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess || p.n_splits == 1) return e;
  return launch_lse_merge(p.part_o, p.part_lse, p.n_splits, (long long)p.B * p.H * D,
                          (long long)p.B * p.H, p.B, p.H, D, p.d_real, p.o, p.o_sb, p.o_sh,
                          p.out_fp32, p.lse, stream);
}

template cudaError_t launch_decode<64>(const DecodeParams&, cudaStream_t);
template cudaError_t launch_decode<128>(const DecodeParams&, cudaStream_t);

// out = sum_i e^{lse_i - lse*} o_i / sum_i e^{lse_i - lse*}; parts whose
// lse is -inf (no visible key) carry no weight. One block of 128 threads per
// (batch, head), one output column per thread. The parts' weights are
// computed once per block, 128 parts at a time, into shared memory, so each
// thread's pass over the parts is a stream of independent loads; the sums
// keep the parts' order (the weight total is accumulated by one thread).
constexpr int kMergeThreads = 128;
__global__ void __launch_bounds__(kMergeThreads)
    lse_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                     int n_parts, long long stride_o, long long stride_lse, int B, int H, int D,
                     int d_out, void* o, long long o_sb, long long o_sh, int out_fp32,
                     float* lse_out) {
  __shared__ float s_red[kMergeThreads / 32];
  __shared__ float s_w[kMergeThreads], s_l[kMergeThreads];
  __shared__ float s_W;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  float m = -INFINITY;
  for (int i = tid; i < n_parts; i += kMergeThreads) m = fmaxf(m, part_lse[i * stride_lse + bh]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (tid % 32 == 0) s_red[tid / 32] = m;
  __syncthreads();
  float M = s_red[0];
#pragma unroll
  for (int k = 1; k < kMergeThreads / 32; ++k) M = fmaxf(M, s_red[k]);
  float W = 0.0f;  // thread 0's running total, in part order
  for (int d0 = 0; d0 < d_out; d0 += kMergeThreads) {
    const int d = d0 + tid;
    float acc = 0.0f;
    for (int c0 = 0; c0 < n_parts; c0 += kMergeThreads) {
      const int n = min(kMergeThreads, n_parts - c0);
      __syncthreads();  // the previous chunk's weights have been read
      if (tid < n) {
        const float li = part_lse[(c0 + tid) * stride_lse + bh];
        s_l[tid] = li;
        s_w[tid] = (M != -INFINITY) ? __expf(li - M) : 0.0f;
      }
      __syncthreads();
      if (d0 == 0 && tid == 0 && M != -INFINITY)
        for (int k = 0; k < n; ++k) W += s_w[k];
      if (d < d_out && M != -INFINITY) {
        const float* po = part_o + (long long)c0 * stride_o + (long long)bh * D + d;
#pragma unroll 8
        for (int k = 0; k < n; ++k)
          if (s_l[k] != -INFINITY) acc = fmaf(s_w[k], po[k * stride_o], acc);
      }
    }
    if (d0 == 0) {
      if (tid == 0) s_W = W;
      __syncthreads();
      W = s_W;
    }
    if (d < d_out) {
      const float val = acc / W;  // NaN when nothing was visible, like the reference
      if (out_fp32)
        reinterpret_cast<float*>(o)[(long long)b * o_sb + (long long)h * o_sh + d] = val;
      else
        reinterpret_cast<__nv_bfloat16*>(o)[(long long)b * o_sb + (long long)h * o_sh + d] =
            __float2bfloat16_rn(val);
    }
  }
  if (tid == 0 && lse_out) lse_out[bh] = (M == -INFINITY) ? M : M + logf(W);
}

cudaError_t launch_lse_merge(const float* part_o, const float* part_lse, int n_parts,
                             long long part_stride_o, long long part_stride_lse, int B, int H,
                             int D, int d_out, void* o, long long o_sb, long long o_sh,
                             int out_fp32, float* lse, cudaStream_t stream) {
  lse_merge_kernel<<<B * H, kMergeThreads, 0, stream>>>(part_o, part_lse, n_parts, part_stride_o,
                                              part_stride_lse, B, H, D, d_out, o, o_sb, o_sh,
                                              out_fp32, lse);
  return cudaGetLastError();
}

}  // namespace enl
