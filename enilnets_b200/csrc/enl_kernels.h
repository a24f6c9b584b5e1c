// Internal launch interface between the C-ABI layer (enl_abi.cu) and the
// kernels. Not installed; the public surface is include/enl_attn.h.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace enl {

// K1 prefill. Q is (B, Sq, H, D), K/V (B, Skv, Hkv, D) with arbitrary b/s/h
// strides (head dim contiguous) described by the tensor maps; O has the same
// logical shape as Q. Query row r sits at absolute position q_pos0 + r, key j
// at k_pos0 + j.
struct PrefillParams {
  int B, H, Hkv, Sq, Skv;
  int d_real;                  // head dim of the tensors (<= the kernel's D; the rest is TMA zero fill)
  void* o;
  long long o_sb, o_ss, o_sh;  // element strides of O
  int out_fp32;                // 0: bf16 output, 1: fp32 output
  float* lse;                  // (B, H, Sq) natural-log LSE, or null
  int causal;                  // key j allowed only if pos_k <= pos_q
  int window;                  // < 0: none; else |pos_q - pos_k| <= window
  int additive;                // 1: graph/sequence.py -1e9 additive rule; 0: -inf exclusion
  const int* kv_len;           // (B) valid key prefix per batch row, or null
  const float* alibi;          // (H) ALiBi slopes (natural-log units), or null
  long long q_pos0, k_pos0;
  float scale_log2;            // softmax scale * log2(e)
  // Persistent schedule: n_items = n_bh * ceil(Sq / 128) work items over
  // min(n_items, n_ctas) CTAs, in sections of sec_bh (batch, head) pairs.
  // The pairs are all B * H of them (units null) or units[0 .. n_bh), each
  // b * H + h.
  int n_items, n_ctas, sec_bh;
  int n_bh;
  const int* units;
  // Block-sparse mode (nn/sparse_attention.py:96-142), when sp_ptr is set:
  // query tile qt visits the key tiles sp_kt[sp_ptr[qt] .. sp_ptr[qt + 1]),
  // and row r of entry e sees key column c of half h (keys 64h + c of the
  // tile) iff bit c of sp_mask[(2e + h) * 128 + r] is set. The masks carry
  // causality and the sequence end; causal/window/kv_len do not apply.
  const int* sp_ptr;
  const int* sp_kt;
  const unsigned long long* sp_mask;
  int sp_entries;
  // Arbitrary key-padding mask (graph/sequence.py:162-168 takes any boolean
  // (B, S) mask), when kv_mask is set: bit c of kv_mask[b * kv_mask_sb + w]
  // set = key 64 w + c of batch row b is real. A key must also lie below
  // kv_len[b] when both are given. mask_tiles[b * n_qt + qt] = {lo, hi, safe,
  // 0}: the key tiles [lo, hi) query tile qt of batch row b visits and
  // whether each of its rows has an unmasked key (launch_mask_tiles).
  const unsigned long long* kv_mask;
  long long kv_mask_sb;
  const int4* mask_tiles;
};

// K6 projection GEMM (enl_gemm.cu): Y[m, n] = sum_k X[m, k] W[n, k] + bias[n],
// then rotate-half RoPE on columns n < rope_cols in heads of rope_d columns at
// position rope_pos0 + (m % rope_seq), with fp32 tables (rows, rope_d / 2).
struct ProjParams {
  int M, N, K;
  const float* bias;  // (N) or null
  int out_fp32;
  int rope_cols, rope_d, rope_seq;
  long long rope_pos0;
  const float* rope_cos;
  const float* rope_sin;
};
template <bool kSplit>
cudaError_t launch_proj_gemm(const CUtensorMap& tx, const CUtensorMap& txlo,
                             const CUtensorMap& tw, const CUtensorMap& twlo,
                             const CUtensorMap& ty, const ProjParams& p, int n_sms,
                             cudaStream_t stream);
// fp32 (rows, cols) with row stride ld -> contiguous bf16 planes hi, lo.
cudaError_t launch_split_matrix(const float* src, long long ld, long long rows, int cols,
                                void* hi, void* lo, cudaStream_t stream);

// Fill p.mask_tiles (B * ceil(Sq / 128) entries) from p.kv_mask, p.kv_len and
// the causal/window bounds; must run before the prefill launch on the same
// stream.
cudaError_t launch_mask_tiles(const PrefillParams& p, int4* tiles, cudaStream_t stream);

// kSplit: the tensor maps cover (hi, lo) bf16 planes of fp32 inputs
// interleaved per head (head coordinate 2h + plane), see launch_split_planes.
// to: bf16 map over O with the Q maps' box and swizzle, used for bf16 output
// of the bf16 path (otherwise ignored).
template <int D, bool kSplit>
cudaError_t launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const CUtensorMap& to, const PrefillParams& p, cudaStream_t stream);

// fp32 src[b, s, h, :] (element strides, 16-byte aligned rows) ->
// dst[b][s][h][plane][D] bf16 with plane 0 = bf16(x), plane 1 = bf16(x - hi).
cudaError_t launch_split_planes(const float* src, long long sb, long long ss, long long sh, int B,
                                int S, int H, int D, void* dst, cudaStream_t stream);

// K5 attention backward (enl_backward.cu).
struct BwdPrepParams {
  int B, H, Sq, s_pad, d_real;
  const void* o;  // forward output (B, Sq, H, D), bf16 or fp32
  long long o_sb, o_ss, o_sh;
  int o_f32;
  const void* dout;  // (B, Sq, H, D), bf16 or fp32
  long long do_sb, do_ss, do_sh;
  int do_f32;
  const float* lse;  // (B, H, Sq) natural-log LSE of the forward
  float* lse2;       // out (B * H, s_pad): LSE * log2(e), +inf on pad rows
  float* dsum;       // out (B * H, s_pad): rowsum(dO * O), 0 on pad rows
};
struct BwdParams {
  int B, H, Hkv, Sq, Skv, d_real;
  int causal;  // key j visible to query i only when j <= i
  int window;  // < 0: none; else |i - j| <= window
  const float* alibi;  // (H) slopes or null
  float scale, scale_log2;
  const float* lse2;
  const float* dsum;
  int s_pad;
  float* dq;  // (B, Sq, H, D) fp32
  long long dq_sb, dq_ss, dq_sh;
  float* dk;  // (B, Skv, Hkv, D) fp32, summed over each kv head's query heads
  long long dk_sb, dk_ss, dk_sh;
  float* dv;
  long long dv_sb, dv_ss, dv_sh;
  int out_vec4;  // dq, dk, dv 16-byte aligned with strides multiple of 4: float4 stores
};
cudaError_t launch_backward(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const CUtensorMap& tdo, const BwdPrepParams& prep, const BwdParams& p,
                            int D, bool split, cudaStream_t stream);

// Column masks of a block-sparse layout (enl_sparse.cu).
struct SparseMaskParams {
  const int* tile_ptr;  // (n_qtiles + 1) entry ranges per query tile
  const int* tile_kt;   // (n_entries) key tile of each entry
  unsigned long long* masks;  // (n_entries, 2, 128) out
  int n_qtiles, n_entries;
  const int* sel_ptr;   // (n_qblocks + 1) selection ranges per query block
  const int* sel_kb;    // (n_sel) selected key blocks
  int n_qblocks, n_sel;
  long long qb0;        // query block of sel_ptr[0]
  int block_size, seq_q, seq_kv, causal;
  long long q_pos0, k_pos0;
};
cudaError_t launch_sparse_masks(const SparseMaskParams& p, cudaStream_t stream);

// K2 split-KV decode: one query token per (b, h) against cached slots.
struct DecodeParams {
  int B, H, Hkv;
  int d_real;  // head dim of the tensors (<= the kernel's D); lanes past it read zeros
  int in_fp32;     // 0: bf16 q and cache, 1: fp32
  const void* q;  // q[b, h, :]
  long long q_sb, q_sh;
  const void* k;  // cache[b, hkv, slot, :]
  const void* v;
  long long k_sb, k_sh, k_ss;
  long long v_sb, v_sh, v_ss;
  int slot_begin, slot_end;  // key slots to read, already narrowed by the window
  long long q_minus_k0;      // q position minus the position of slot 0
  const float* alibi;        // (H) or null
  float scale_log2;
  int n_splits, split_len;
  void* o;  // final output o[b, h, :] (n_splits == 1)
  long long o_sb, o_sh;
  int out_fp32;
  float* lse;       // (B, H) or null (n_splits == 1)
  float* part_o;    // (n_splits, B, H, D) fp32 normalised partials
  float* part_lse;  // (n_splits, B, H)
};

template <int D>
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream);

// LSE merge of n_parts normalised partials (o_i, lse_i) into one output.
// part_o rows hold D floats; the first d_out of them are written to o.
cudaError_t launch_lse_merge(const float* part_o, const float* part_lse, int n_parts,
                             long long part_stride_o, long long part_stride_lse, int B, int H,
                             int D, int d_out, void* o, long long o_sb, long long o_sh,
                             int out_fp32, float* lse, cudaStream_t stream);

// K3 cache append: cache[b, h, slot0 + t, :] = src[b, t, h, :].
cudaError_t launch_kv_append(void* cache, long long c_sb, long long c_sh, long long c_ss,
                             const void* src, long long s_sb, long long s_st, long long s_sh,
                             int B, int Hkv, int n_new, int D, int elem_bytes, long long slot0,
                             cudaStream_t stream);

// Batch-axis gather of cache rows: dst[i, h, s, :] = src[index[i], h, s, :]
// for s in [slot_begin, slot_end).
cudaError_t launch_kv_gather(void* dst, long long d_sb, long long d_sh, long long d_ss,
                             const void* src, long long s_sb, long long s_sh, long long s_ss,
                             const long long* index, int B_out, int B_src, int Hkv,
                             int slot_begin, int slot_end, int D, int elem_bytes,
                             cudaStream_t stream);

// RoPE rotate-half in place on x[b, s, h, :] using a (n_pos, D/2) cos/sin table.
cudaError_t launch_rope(void* x, long long x_sb, long long x_ss, long long x_sh, int B, int S,
                        int H, int D, int elem_bytes, const float* cos_t, const float* sin_t,
                        long long table_row0, long long n_rows, cudaStream_t stream);

// Linearized attention feature map (enl_linear.cu): x[b, s, h, :] (strided,
// bf16 or fp32) -> phi[b, h, s, :] fp32, Df = Dh for kernel 0 (elu + 1) or
// the rows of omega for kernel 1 (Performer). With global_stab, stab[b*H + h]
// receives the stabilizer (the max of w.x' over the call's rows, no lower
// than stab_floor when given); otherwise each row uses its own max.
struct PhiParams {
  const void* x;
  long long sb, ss, sh;
  int B, S, H, Dh;
  bool in_f32;
  int kernel;
  const float* omega;
  int Df;
  int global_stab;
  const float* stab_floor;
  float* stab;
  float* phi;        // (B, H, S, Df) fp32 out, or null when planes is set
  uint16_t* planes;  // [2][B * H][S][Dfp] bf16 hi/lo planes out (elu + 1, vectorised path)
  int Dfp;
};
cudaError_t launch_phi(const PhiParams& p, cudaStream_t stream);
// Whether launch_phi writes planes directly for these arguments (else the
// caller maps to fp32 and splits with launch_rows_planes).
bool phi_planes_direct(const PhiParams& p);
int perf_max_head_dim();  // Performer feature maps take head_dim up to this

// Linear attention over phi(Q) (B, H, S, Df) and phi(K) (B, Hkv, S, Df) with
// V[b, s, hkv, :] (strided); o[b, s, h, :]. Causal runs prefix sums starting
// from the carried state (kv_in (B, Hkv, Df, D), ks_in (B, Hkv, Df), each
// times state_scale[b*Hkv + hkv]) and returns the final sums in kv_out/ks_out.
struct LinearParams {
  const float* phi_q;
  const float* phi_k;
  const void* v;
  long long v_sb, v_ss, v_sh;
  bool v_f32;
  void* o;
  long long o_sb, o_ss, o_sh;
  bool o_f32;
  int B, H, Hkv, S, Df, D;
  int causal;
  const float* kv_in;
  const float* ks_in;
  const float* state_scale;
  float* kv_out;
  float* ks_out;
  float eps;
  float* carry_kv;  // workspace: per-segment prefixes (n_seg, B, Hkv, Df, D)
  float* carry_ks;  // (n_seg, B, Hkv, Df)
  int n_seg, seg_len;  // set by launch_linear_attn
};
cudaError_t launch_linear_attn(const LinearParams& p, cudaStream_t stream);

// K4 on tcgen05 (enl_linear_tc.cu): chunked linear attention over bf16 hi/lo
// planes. Dp = V' columns (D + 1 rounded up to 16); Dfp, Sp: row strides of the
// feature- and sequence-contiguous planes (multiples of 8).
struct LinTcParams {
  int B, H, Hkv, S, Df, D, Dp, Dfp, Sp, n_chunks, causal, tmem_cols;
  float* u;      // (B * Hkv, n_chunks, Dp, Df) chunk states, transposed
  uint16_t* st;  // [2][B * Hkv * n_chunks][Dp][Dfp] exclusive prefix states, transposed
  const float* kv_in;
  const float* ks_in;
  const float* state_scale;
  float* kv_out;
  float* ks_out;
  void* o;
  long long o_sb, o_ss, o_sh;
  int o_f32;
  float eps;
};
// Performer feature map on tcgen05 (enl_linear_tc.cu), Df <= 256.
struct PerfTcParams {
  int B, S, H, Dh, Dhp, Df;
  uint16_t* xp;      // [2][B * H][S][Dhp] bf16 planes of x
  float* stab;       // (B * H): mode 0 atomic-max target (ordered ints), mode 2 input
  float* phi;        // (B, H, S, Df) fp32 out, or null when planes is set
  uint16_t* planes;  // [2][B * H][S][Dfp] bf16 hi/lo planes out
  int Dfp;
  int n_sm;          // SMs of the device (grid of the persistent form)
};
bool perf_tc_supported(int Dh, int Df);
cudaError_t launch_perf_prep(const void* x, long long sb, long long ss, long long sh, int f32,
                             const float* omega, const PerfTcParams& p, uint16_t* wp,
                             cudaStream_t stream);
cudaError_t launch_perf_tc(const CUtensorMap& tx, const CUtensorMap& tw, const PerfTcParams& p,
                           int mode, cudaStream_t stream);
// Queries (global_stab 0): one pass with row stabilizers. Keys: the
// stabilizer (floored by stab_floor) as a max pass, then the map.
cudaError_t launch_perf_tc_maps(const CUtensorMap& tx, const CUtensorMap& tw,
                                const PerfTcParams& p, int global_stab, const float* stab_floor,
                                cudaStream_t stream);
// Row planes of an fp32 (R, Df) matrix: dst[plane][R][Dfp] bf16 hi/lo.
cudaError_t launch_rows_planes(const float* src, long long R, int Df, int Dfp, uint16_t* dst,
                               cudaStream_t stream);
cudaError_t launch_lin_prep(const float* phi_q, const float* phi_k, const void* v, long long v_sb,
                            long long v_ss, long long v_sh, int v_f32, const LinTcParams& p,
                            uint16_t* qp, uint16_t* kp, uint16_t* vt, cudaStream_t stream);
cudaError_t launch_lin_tc(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tvt,
                          const CUtensorMap& tst, const LinTcParams& p, cudaStream_t stream);
size_t linear_workspace_bytes(int B, int H, int Hkv, int S, int Df, int D, int causal);
int linear_attn_max_features();

}  // namespace enl
