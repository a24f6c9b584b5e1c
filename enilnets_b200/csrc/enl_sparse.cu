// Block-sparse layout masks for K1's sparse mode.
//
// nn/sparse_attention.py:96-142 lets query block qb (positions
// [qb*bs, qb*bs + bs)) see the key blocks block_selection (:48-84) chose for
// it, minus keys past the sequence end (:132) and, when causal, keys after
// the query (:134). The gather there becomes, here, a per-query-tile list of
// 128-key tiles (built on the host) and one 64-bit column mask per (entry,
// tile half, query row), which this kernel fills: bit c of
// masks[(2e + h) * 128 + r] is set iff query row 128*qt + r may see key
// 128*tile_kt[e] + 64h + c. Rows past seq_q get an empty mask.
#include "enl_common.cuh"
#include "enl_kernels.h"

namespace enl {

// Bits [a, b] of a 64-bit word (0 <= a <= b <= 63).
__device__ __forceinline__ unsigned long long bit_range(int a, int b) {
  const unsigned long long hi = (b >= 63) ? ~0ull : ((1ull << (b + 1)) - 1ull);
  return hi & ~((1ull << a) - 1ull);
}

// One CTA per query tile, one thread per (tile half, row).
__global__ void __launch_bounds__(256) sparse_mask_kernel(SparseMaskParams p) {
  const int qt = blockIdx.x;
  const int half = threadIdx.x / 128, r = threadIdx.x % 128;
  const int e0 = p.tile_ptr[qt], e1 = p.tile_ptr[qt + 1];
  if (e0 < 0 || e1 > p.n_entries || e0 > e1) {
    if (threadIdx.x == 0) report_error(kDevBadIndex, qt);
    return;
  }
  const long long row = (long long)qt * 128 + r;
  const long long qpos = p.q_pos0 + row;
  const long long qb = qpos / p.block_size;  // positions are >= 0
  const long long qsel = qb - p.qb0;
  const bool live = row < p.seq_q && qsel >= 0 && qsel < p.n_qblocks;
  if (row < p.seq_q && !live) report_error(kDevBadIndex, (int)row);
  int s0 = 0, s1 = 0;
  if (live) {
    s0 = p.sel_ptr[qsel];
    s1 = p.sel_ptr[qsel + 1];
    if (s0 < 0 || s1 > p.n_sel || s0 > s1) {
      report_error(kDevBadIndex, (int)row);
      s0 = s1 = 0;
    }
  }
  // Largest key index this row may see: the sequence end, and under a
  // causal mask its own position.
  long long jmax = (long long)p.seq_kv - 1;
  if (p.causal) jmax = min(jmax, qpos - p.k_pos0);
  for (int e = e0; e < e1; ++e) {
    const long long j0 = (long long)p.tile_kt[e] * 128 + 64 * half;  // key index of bit 0
    unsigned long long m = 0;
    for (int s = s0; s < s1; ++s) {
      // key block kb holds positions [kb*bs, kb*bs + bs), key indices shifted by k_pos0
      const long long klo = (long long)p.sel_kb[s] * p.block_size - p.k_pos0;
      const long long a = max(max(klo, j0), 0ll);
      const long long b = min(min(klo + p.block_size - 1, j0 + 63), jmax);
      if (a <= b) m |= bit_range((int)(a - j0), (int)(b - j0));
    }
    p.masks[((long long)e * 2 + half) * 128 + r] = m;
  }
}

cudaError_t launch_sparse_masks(const SparseMaskParams& p, cudaStream_t stream) {
  if (p.n_qtiles <= 0) return cudaSuccess;
  sparse_mask_kernel<<<p.n_qtiles, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace enl
