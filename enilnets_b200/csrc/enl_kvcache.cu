// K3: KV-cache append, the batch-axis cache gather used by beam search, and
// the RoPE rotation applied to freshly projected Q/K.
//
// Append replaces the reference's per-step `np.concatenate([prev, new],
// axis=2)` (nn/kvcache.py:156-162), which copies the whole cache every step:
// here only the n_new new rows are written, 16 bytes per thread, into a
// preallocated (B, Hkv, capacity, D) buffer. Gather replaces
// KVCache.reorder's `k[idx]` (nn/kvcache.py:42-61) for the live slots only.
// RoPE follows nn/forward.py:80-88 (rotate-half) with angles precomputed on
// the host in float64 as nn/forward.py:46-55 computes them.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

// One thread moves one 16-byte chunk of one new row.
__global__ void kv_append_kernel(uint8_t* __restrict__ cache, long long c_sb, long long c_sh,
                                 long long c_ss, const uint8_t* __restrict__ src, long long s_sb,
                                 long long s_st, long long s_sh, int B, int Hkv, int n_new,
                                 int row_chunks, long long slot0) {
  const long long total = (long long)B * n_new * Hkv * row_chunks;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % row_chunks);
    long long r = i / row_chunks;
    const int h = (int)(r % Hkv);
    r /= Hkv;
    const int t = (int)(r % n_new);
    const int b = (int)(r / n_new);
    const uint4 w =
        *reinterpret_cast<const uint4*>(src + b * s_sb + t * s_st + h * s_sh + c * 16);
    *reinterpret_cast<uint4*>(cache + b * c_sb + h * c_sh + (slot0 + t) * c_ss + c * 16) = w;
  }
}

cudaError_t launch_kv_append(void* cache, long long c_sb, long long c_sh, long long c_ss,
                             const void* src, long long s_sb, long long s_st, long long s_sh,
                             int B, int Hkv, int n_new, int D, int elem_bytes, long long slot0,
                             cudaStream_t stream) {
  const int row_chunks = D * elem_bytes / 16;
  const long long total = (long long)B * n_new * Hkv * row_chunks;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = min((total + threads - 1) / threads, 148ll * 16);
  // Strides arrive in elements; the kernel works in bytes.
  kv_append_kernel<<<(int)blocks, threads, 0, stream>>>(
      reinterpret_cast<uint8_t*>(cache), c_sb * elem_bytes, c_sh * elem_bytes, c_ss * elem_bytes,
      reinterpret_cast<const uint8_t*>(src), s_sb * elem_bytes, s_st * elem_bytes,
      s_sh * elem_bytes, B, Hkv, n_new, row_chunks, slot0);
  return cudaGetLastError();
}

__global__ void kv_gather_kernel(uint8_t* __restrict__ dst, long long d_sb, long long d_sh,
                                 long long d_ss, const uint8_t* __restrict__ src, long long s_sb,
                                 long long s_sh, long long s_ss, const long long* __restrict__ index,
                                 int B_out, int B_src, int Hkv, int slot_begin, int n_slots,
                                 int row_chunks) {
  const long long total = (long long)B_out * Hkv * n_slots * row_chunks;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % row_chunks);
    long long r = i / row_chunks;
    const int s = slot_begin + (int)(r % n_slots);
    r /= n_slots;
    const int h = (int)(r % Hkv);
    const int bo = (int)(r / Hkv);
    const long long bs = index[bo];
    if (bs < 0 || bs >= B_src) {
      report_error(kDevBadIndex, bo);
      continue;
    }
    const uint4 w = *reinterpret_cast<const uint4*>(src + bs * s_sb + h * s_sh + s * s_ss + c * 16);
    *reinterpret_cast<uint4*>(dst + bo * d_sb + h * d_sh + s * d_ss + c * 16) = w;
  }
}

cudaError_t launch_kv_gather(void* dst, long long d_sb, long long d_sh, long long d_ss,
                             const void* src, long long s_sb, long long s_sh, long long s_ss,
                             const long long* index, int B_out, int B_src, int Hkv,
                             int slot_begin, int slot_end, int D, int elem_bytes,
                             cudaStream_t stream) {
  const int row_chunks = D * elem_bytes / 16;
  const int n_slots = slot_end - slot_begin;
  const long long total = (long long)B_out * Hkv * n_slots * row_chunks;
  if (total <= 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = min((total + threads - 1) / threads, 148ll * 16);
  kv_gather_kernel<<<(int)blocks, threads, 0, stream>>>(
      reinterpret_cast<uint8_t*>(dst), d_sb * elem_bytes, d_sh * elem_bytes, d_ss * elem_bytes,
      reinterpret_cast<const uint8_t*>(src), s_sb * elem_bytes, s_sh * elem_bytes,
      s_ss * elem_bytes, index, B_out, B_src, Hkv, slot_begin, n_slots, row_chunks);
  return cudaGetLastError();
}

// x1' = x1 cos - x2 sin, x2' = x2 cos + x1 sin over the two halves of the head.
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, long long x_sb, long long x_ss, long long x_sh,
                            int B, int S, int H, int half, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, long long row0, long long n_rows) {
  const long long total = (long long)B * S * H * half;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(i % half);
    long long r = i / half;
    const int h = (int)(r % H);
    r /= H;
    const int s = (int)(r % S);
    const int b = (int)(r / S);
    const long long trow = row0 + s;
    if (trow < 0 || trow >= n_rows) {
      report_error(kDevBadIndex, s);
      continue;
    }
    const float c = cos_t[trow * half + k];
    const float sn = sin_t[trow * half + k];
    T* base = x + b * x_sb + s * x_ss + h * x_sh;
    const float x1 = static_cast<float>(base[k]);
    const float x2 = static_cast<float>(base[k + half]);
    base[k] = static_cast<T>(x1 * c - x2 * sn);
    base[k + half] = static_cast<T>(x2 * c + x1 * sn);
  }
}

cudaError_t launch_rope(void* x, long long x_sb, long long x_ss, long long x_sh, int B, int S,
                        int H, int D, int elem_bytes, const float* cos_t, const float* sin_t,
                        long long table_row0, long long n_rows, cudaStream_t stream) {
  const int half = D / 2;
  const long long total = (long long)B * S * H * half;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = min((total + threads - 1) / threads, 148ll * 16);
  if (elem_bytes == 2)
    rope_kernel<__nv_bfloat16><<<(int)blocks, threads, 0, stream>>>(
        reinterpret_cast<__nv_bfloat16*>(x), x_sb, x_ss, x_sh, B, S, H, half, cos_t, sin_t,
        table_row0, n_rows);
  else
    rope_kernel<float><<<(int)blocks, threads, 0, stream>>>(reinterpret_cast<float*>(x), x_sb,
                                                            x_ss, x_sh, B, S, H, half, cos_t,
                                                            sin_t, table_row0, n_rows);
  return cudaGetLastError();
}

}  // namespace enl
