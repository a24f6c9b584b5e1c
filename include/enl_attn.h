/*
 * enl_attn.h -- C ABI of libenl_b200.so, the B200 (sm_100a) attention
 * inference path behind the Enilnets attention layers.
 *
 * Plain C: pointers, fixed-width integers and sizes only. Every entry point
 * returns an int status (ENL_OK == 0); on failure enl_last_error() returns a
 * thread-local message. Launches are asynchronous on the caller's stream
 * (a cudaStream_t passed as void*, NULL = legacy default stream). Device
 * pointers are caller-owned; the library never allocates device memory.
 *
 * Layout conventions: every tensor has a contiguous head dimension; the
 * other axes are described by element strides, so projection outputs of
 * shape (batch, seq, heads * head_dim) are consumed in place.
 */
#ifndef ENL_ATTN_H_
#define ENL_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ENL_ABI_VERSION 8

/* Status codes. The Python binding maps INVALID/UNSUPPORTED to ValueError
 * (the reference raises ValueError for bad layer configurations,
 * nn/layers.py:210-327) and CUDA/DEVICE to RuntimeError (core/backend.py:106-113). */
enum {
  ENL_OK = 0,
  ENL_ERR_INVALID = 1,     /* bad argument: shape, stride, alignment, null pointer */
  ENL_ERR_UNSUPPORTED = 2, /* valid request outside what the kernels cover */
  ENL_ERR_CUDA = 3,        /* CUDA runtime / driver error */
  ENL_ERR_DEVICE = 4       /* a kernel recorded an error in the device error word */
};

enum { ENL_DTYPE_BF16 = 0, ENL_DTYPE_FP32 = 1 };

/* How masked scores are treated.
 * EXCLUDE : masked scores are -inf (nn/forward.py:102-117, the nn/ layers).
 * ADDITIVE: each violated mask term adds -1e9 (graph/sequence.py:162-176);
 *           a row whose every key is masked keeps the keys with the fewest
 *           violations, exactly as the float64 reference does. */
enum { ENL_MASK_EXCLUDE = 0, ENL_MASK_ADDITIVE = 1 };

/* ---------------------------------------------------------------- prefill */
typedef struct enl_prefill_args {
  const void* q; /* (batch, seq_q, num_heads, head_dim) */
  const void* k; /* (batch, seq_kv, num_kv_heads, head_dim) */
  const void* v; /* (batch, seq_kv, num_kv_heads, head_dim) */
  void* o;       /* (batch, seq_q, num_heads, head_dim), out_dtype */
  float* lse;    /* (batch, num_heads, seq_q) natural-log LSE, or NULL */
  int32_t batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim;
  int64_t q_stride_b, q_stride_s, q_stride_h; /* element strides */
  int64_t k_stride_b, k_stride_s, k_stride_h;
  int64_t v_stride_b, v_stride_s, v_stride_h;
  int64_t o_stride_b, o_stride_s, o_stride_h;
  int32_t in_dtype;  /* ENL_DTYPE_BF16, or ENL_DTYPE_FP32 (split-bf16 path, needs workspace) */
  int32_t out_dtype; /* ENL_DTYPE_BF16 or ENL_DTYPE_FP32 */
  int32_t causal;    /* key allowed only when pos_k <= pos_q */
  int32_t window;    /* < 0: none; else |pos_q - pos_k| <= window */
  int32_t mask_mode; /* ENL_MASK_EXCLUDE or ENL_MASK_ADDITIVE */
  const int32_t* kv_valid_len; /* device (batch,): keys [0, len) are real; NULL = all */
  const float* alibi_slopes;   /* device (num_heads,): ALiBi slopes; NULL = none */
  int64_t q_pos0;              /* absolute position of query row 0 */
  int64_t k_pos0;              /* absolute position of key row 0 */
  float scale;                 /* softmax scale, normally 1/sqrt(head_dim) */
  void* workspace;             /* device scratch for fp32 inputs and kv_mask, */
  size_t workspace_bytes;      /* >= enl_prefill_workspace_bytes(), 256-byte aligned */
  /* Arbitrary key-padding mask, for masks that are not a prefix of real keys
   * (left padding, holes): graph/sequence.py:162-168 adds -1e9 for any
   * boolean (batch, seq) mask. Bit c of kv_mask[b * kv_mask_stride_b + w]
   * set = key 64 w + c of batch row b is real. Device memory, NULL = none;
   * with kv_valid_len also set a key must pass both. Bits past seq_kv are
   * ignored. Needs the workspace (per-query-tile key ranges). */
  const uint64_t* kv_mask;
  int64_t kv_mask_stride_b; /* 64-bit words per batch row, >= ceil(seq_kv / 64) */
  /* Which (batch, head) units to compute: device list of n_units entries
   * b * num_heads + h (a rank's share of a batch x head partition); NULL =
   * all batch * num_heads. Rows of units not listed are not written. */
  const int32_t* units;
  int32_t n_units;
} enl_prefill_args;

/* Fused attention prefill: softmax(Q K^T * scale + bias + mask) V.
 * Replaces the score/softmax/context math of nn/forward.py:525-551 (MHA),
 * nn/flash_attention.py:42-80 (tiled softmax), nn/forward.py:578-586 (cross
 * attention), the cached multi-token step nn/kvcache.py:198-213, and the
 * key-padding rule of graph/sequence.py:159-183. head_dim: any multiple of 8
 * up to 128 (the kernel runs at 64 or 128 with TMA zero fill).
 *
 * bf16 inputs: one bf16 MMA per product, fp32 accumulation.
 * fp32 inputs (the reference's default float32 models): q, k, v are first
 * split into bf16 planes hi = bf16(x), lo = bf16(x - hi) in the workspace,
 * and every product is hi*hi + hi*lo + lo*hi on the bf16 tensor cores (the
 * softmax probabilities are split the same way), for about 2^-16 relative
 * error, tighter than tf32. fp32 rows must be 16-byte aligned. */
int enl_attn_prefill(const enl_prefill_args* args, void* stream);

/* Workspace bytes enl_attn_prefill needs for these arguments: the bf16
 * planes of fp32 inputs, plus 16 bytes per (batch row, 128-row query tile)
 * with kv_mask; 0 for bf16 inputs without kv_mask. */
size_t enl_prefill_workspace_bytes(const enl_prefill_args* args);

/* ----------------------------------------------------------------- decode */
typedef struct enl_decode_args {
  const void* q; /* (batch, num_heads, head_dim): one query token per row */
  int64_t q_stride_b, q_stride_h;
  const void* k_cache; /* (batch, num_kv_heads, capacity, head_dim) */
  const void* v_cache;
  int64_t cache_stride_b, cache_stride_h, cache_stride_s; /* shared by K and V */
  void* o; /* (batch, num_heads, head_dim), out_dtype */
  int64_t o_stride_b, o_stride_h;
  float* lse; /* (batch, num_heads) natural-log LSE, or NULL */
  int32_t batch, num_heads, num_kv_heads, head_dim;
  int32_t slot_begin, slot_end; /* live cache slots [slot_begin, slot_end) */
  int64_t pos_slot0;            /* absolute position of cache slot 0 */
  int64_t q_pos;                /* absolute position of the query token */
  int32_t window;               /* < 0: none */
  const float* alibi_slopes;    /* device (num_heads,) or NULL */
  float scale;
  int32_t in_dtype, out_dtype;
  int32_t n_splits; /* KV splits per (batch, kv head); 0 = choose automatically */
  void* workspace;  /* device scratch, >= enl_decode_workspace_bytes(); may be NULL if 1 split */
  size_t workspace_bytes;
} enl_decode_args;

/* Split-KV single-token decode with log-sum-exp merge of the splits.
 * Replaces the attention half of nn/kvcache.py:_attention_step (lines
 * 198-213) for one new token; head_dim a multiple of 8 up to 128,
 * num_heads/num_kv_heads in {1, 2, 4, 8}. in_dtype (q and both caches):
 * ENL_DTYPE_BF16 or ENL_DTYPE_FP32; the arithmetic is fp32 either way. */
int enl_attn_decode(const enl_decode_args* args, void* stream);

/* Scratch held by enl_attn_decode_noalloc on every device that loads the library. */
#define ENL_DECODE_NOALLOC_SCRATCH_BYTES (4u << 20)

/* enl_attn_decode for callers that cannot allocate device memory: a host
 * that owns all device memory and gives plugins no allocation hook, or a
 * token loop where a cudaMalloc (which may synchronise the device) is not
 * allowed. Same arguments and results as enl_attn_decode; args->workspace is
 * ignored and the split partials go to a fixed scratch array inside the
 * library (ENL_DECODE_NOALLOC_SCRATCH_BYTES per device, kept until exit).
 * Requests whose partials would not fit (for the split count actually run,
 * after the slot range is narrowed by causality and the window) are
 * rejected with ENL_ERR_INVALID. The first call on a device looks up the
 * scratch address, so make it before any stream capture; the address
 * belongs to that call's CUDA context, so keep that context alive (no
 * cudaDeviceReset) while the entry point is in use. All calls on a device
 * share the scratch: calls whose kernels overlap on the GPU race and must
 * be ordered on one stream.
 * No counterpart in the reference, which never splits the key sequence. */
int enl_attn_decode_noalloc(const enl_decode_args* args, void* stream);

/* The split count enl_attn_decode uses for n_splits == 0. */
int enl_decode_auto_splits(int32_t batch, int32_t num_kv_heads, int32_t n_slots);

/* Scratch bytes enl_attn_decode needs for a given split count. */
size_t enl_decode_workspace_bytes(int32_t batch, int32_t num_heads, int32_t head_dim,
                                  int32_t n_splits);

/* Merge n_parts normalised partial outputs (part_o: (n_parts, batch, heads,
 * head_dim) fp32; part_lse: (n_parts, batch, heads)) by log-sum-exp. Used
 * after an NCCL all-gather of per-GPU partials in sequence-sharded decode.
 * No reference counterpart: the reference never splits the KV sequence. */
int enl_lse_merge(const float* part_o, const float* part_lse, int32_t n_parts, int32_t batch,
                  int32_t num_heads, int32_t head_dim, void* o, int64_t o_stride_b,
                  int64_t o_stride_h, int32_t out_dtype, float* lse, void* stream);

/* enl_lse_merge with the parts part_o_stride / part_lse_stride floats apart
 * (each part's (batch, heads, head_dim) and (batch, heads) contiguous), so a
 * gathered buffer of packed [out | lse] parts is merged in place. */
int enl_lse_merge_strided(const float* part_o, int64_t part_o_stride, const float* part_lse,
                          int64_t part_lse_stride, int32_t n_parts, int32_t batch,
                          int32_t num_heads, int32_t head_dim, void* o, int64_t o_stride_b,
                          int64_t o_stride_h, int32_t out_dtype, float* lse, void* stream);

/* -------------------------------------------------------------- KV cache */
/* cache[b, h, slot0 + t, :] = src[b, t, h, :] for t < n_new. Replaces the
 * whole-cache np.concatenate of nn/kvcache.py:156-162. Fails with
 * ENL_ERR_INVALID when slot0 + n_new > capacity. */
int enl_kv_append(void* cache, int64_t cache_stride_b, int64_t cache_stride_h,
                  int64_t cache_stride_s, const void* src, int64_t src_stride_b,
                  int64_t src_stride_t, int64_t src_stride_h, int32_t batch,
                  int32_t num_kv_heads, int32_t n_new, int32_t head_dim, int32_t dtype,
                  int64_t slot0, int64_t capacity, void* stream);

/* dst[i, h, s, :] = src[index[i], h, s, :] for s in [slot_begin, slot_end).
 * Replaces KVCache.reorder / expand (nn/kvcache.py:42-66) on device. index is
 * a device int64 array of batch_out entries; out-of-range entries set the
 * device error word and are skipped. dst must not alias src. */
int enl_kv_gather(void* dst, int64_t dst_stride_b, int64_t dst_stride_h, int64_t dst_stride_s,
                  const void* src, int64_t src_stride_b, int64_t src_stride_h,
                  int64_t src_stride_s, const int64_t* index, int32_t batch_out,
                  int32_t batch_src, int32_t num_kv_heads, int32_t slot_begin, int32_t slot_end,
                  int32_t head_dim, int32_t dtype, void* stream);

/* In-place rotate-half RoPE on x[b, s, h, :] (nn/forward.py:80-88) with
 * float32 tables cos/sin of shape (table_rows, head_dim/2) computed as
 * nn/forward.py:46-55 does; sequence row s uses table row table_row0 + s. */
int enl_rope_apply(void* x, int64_t stride_b, int64_t stride_s, int64_t stride_h, int32_t batch,
                   int32_t seq, int32_t num_heads, int32_t head_dim, int32_t dtype,
                   const float* cos_table, const float* sin_table, int64_t table_row0,
                   int64_t table_rows, void* stream);

/* ------------------------------------------------------------ projections */
typedef struct enl_project_args {
  const void* x;       /* (M, K) rows, x_stride_m elements apart */
  int64_t x_stride_m;
  int32_t x_dtype;     /* ENL_DTYPE_BF16, or ENL_DTYPE_FP32 (split-bf16 path, needs w_lo
                          and workspace) */
  const void* w;       /* (N, K) bf16 weight of x @ W.T, rows w_stride_n elements apart;
                          for fp32 x its hi plane bf16(W) */
  const void* w_lo;    /* fp32 x: (N, K) bf16 lo plane bf16(W - bf16(W)), same strides */
  int64_t w_stride_n;
  const float* bias;   /* (N) fp32, or NULL */
  void* y;             /* (M, N) rows, y_stride_m elements apart */
  int64_t y_stride_m;
  int32_t y_dtype;     /* ENL_DTYPE_BF16 or ENL_DTYPE_FP32 */
  int32_t M, N, K;     /* M >= 0 (M == 0: nothing to do, x and y may be NULL) */
  /* RoPE fused into the epilogue (nn/forward.py:80-88): columns n < rope_cols,
   * heads of rope_head_dim columns, rotate-half at position
   * rope_pos0 + (m % rope_seq) with fp32 tables (rope_rows, rope_head_dim / 2)
   * as nn/forward.py:46-55 computes them. rope_cols = 0: no rotation.
   * rope_head_dim: 8, 16, 32, 64 or 128. */
  int32_t rope_cols, rope_head_dim, rope_seq;
  int64_t rope_pos0;
  const float* rope_cos;
  const float* rope_sin;
  int64_t rope_rows;
  void* workspace;     /* fp32 x: >= enl_project_workspace_bytes(), 256-byte aligned */
  size_t workspace_bytes;
} enl_project_args;

/* y = x W^T + bias, then the RoPE rotation of the Q/K columns: the attention
 * layers' projections (nn/forward.py:428-430 and :551, the cross-attention
 * projections of nn/forward.py:567-586, the cached step's of
 * nn/kvcache.py:148-154). tcgen05 MMAs on CTA pairs, fp32 accumulation.
 * fp32 x: the split-bf16 path, x is split into hi/lo bf16 planes in the
 * workspace and every product is hi*hi + hi*lo + lo*hi (about 2^-16
 * relative error). K and N multiples of 8; rows 16-byte aligned. */
int enl_project(const enl_project_args* args, void* stream);

/* Workspace bytes enl_project needs (the bf16 planes of fp32 x; 0 for bf16). */
size_t enl_project_workspace_bytes(const enl_project_args* args);

/* fp32 (rows, cols) matrix with row stride ld elements -> contiguous bf16
 * planes hi = bf16(x), lo = bf16(x - hi), for the weights of the split-bf16
 * projections. cols a multiple of 4, rows 16-byte aligned. */
int enl_split_bf16(const float* src, int64_t ld, int64_t rows, int32_t cols, void* hi, void* lo,
                   void* stream);

/* ---------------------------------------------------- linearized attention */
/* The reference's attention_kernel = "linear" (phi = elu + 1) and "performer"
 * (FAVOR+) options: nn/attention_kernels.py:58-143, nn/forward.py:456-478 and
 * the cached step of nn/kvcache.py:217-260. Arithmetic is fp32. */
enum { ENL_PHI_LINEAR = 0, ENL_PHI_PERFORMER = 1 };

typedef struct enl_phi_args {
  const void* x; /* x[b, s, h, :], bf16 or fp32, strides in elements */
  int64_t x_stride_b, x_stride_s, x_stride_h;
  int32_t batch, seq, num_heads, head_dim;
  int32_t in_dtype;        /* ENL_DTYPE_BF16 or ENL_DTYPE_FP32 */
  int32_t kernel;          /* ENL_PHI_LINEAR or ENL_PHI_PERFORMER */
  const float* omega;      /* performer: (num_features, head_dim) fp32, row-major;
                              performer head_dim up to 256 */
  int32_t num_features;    /* performer: rows of omega, 1..1024 */
  int32_t global_stab;     /* performer: 1 = one stabilizer per (b, h) (keys),
                              0 = one per row (queries) */
  const float* stab_floor; /* global: optional lower bound per (b, h) */
  float* stab;             /* global: receives the stabilizer per (b, h) */
  float* phi;              /* out (batch, num_heads, seq, Df) fp32, contiguous;
                              Df = head_dim (linear) or num_features; NULL when
                              phi_planes is given */
  void* workspace;         /* >= enl_phi_workspace_bytes(), 256-byte aligned */
  size_t workspace_bytes;
  void* phi_planes;        /* optional out instead of phi: bf16 planes
                              [2][batch * num_heads][seq][Dfp], hi = bf16(phi) then
                              lo = bf16(phi - hi), Dfp = Df rounded up to 8,
                              16-byte aligned: the operand layout of the
                              tensor-core enl_linear_attention (phi_q_planes /
                              phi_k_planes), so that phi makes no fp32 round trip */
} enl_phi_args;

/* Workspace bytes enl_linear_feature_map needs: the bf16 hi/lo planes of x
 * and omega for the tensor-core Performer map (num_features <= 256), and an
 * fp32 phi when planes are asked of a map that writes fp32 only; 0
 * otherwise. */
size_t enl_phi_workspace_bytes(const enl_phi_args* args);

/* phi(x) (nn/attention_kernels.py:58-74): elu(x) + 1, or
 * exp(w.x' - |x'|^2 / 2 - stab) / sqrt(num_features) with x' = x / head_dim^(1/4)
 * and stab the row max of w.x' (queries) or its max over every row of the
 * call and stab_floor (keys, nn/attention_kernels.py:38-55). Performer maps
 * with up to 256 features run the projections w.x as split-bf16 tcgen05 MMAs
 * (needs the workspace); larger ones on the CUDA cores. */
int enl_linear_feature_map(const enl_phi_args* args, void* stream);

typedef struct enl_linear_args {
  const float* phi_q; /* (batch, num_heads, seq, num_features) fp32 */
  const float* phi_k; /* (batch, num_kv_heads, seq, num_features) fp32 */
  const void* v;      /* v[b, s, kv_head, :], strides in elements */
  int64_t v_stride_b, v_stride_s, v_stride_h;
  int32_t v_dtype;
  void* o; /* o[b, s, h, :] */
  int64_t o_stride_b, o_stride_s, o_stride_h;
  int32_t out_dtype;
  int32_t batch, num_heads, num_kv_heads, seq, num_features, head_dim;
  int32_t causal;
  /* Causal only, each nullable: a carried state added to every prefix,
   * kv (batch, num_kv_heads, num_features, head_dim) and ksum (batch,
   * num_kv_heads, num_features), both times state_scale[b * num_kv_heads +
   * kv_head]; kv_out / ksum_out receive the sums after the last row. */
  const float* kv_in;
  const float* ksum_in;
  const float* state_scale;
  float* kv_out;
  float* ksum_out;
  float eps; /* denominator guard, 1e-20 in the reference */
  void* workspace; /* device scratch for the segmented causal pass, */
  size_t workspace_bytes; /* >= enl_linear_workspace_bytes() */
  /* Optional, both or neither, instead of phi_q / phi_k (which may then be
   * NULL): their bf16 hi/lo planes as enl_phi_args.phi_planes writes them,
   * [2][batch * num_heads][seq][Dfp] and [2][batch * num_kv_heads][seq][Dfp].
   * Only where enl_linear_planes_ok(head_dim, num_features). */
  const void* phi_q_planes;
  const void* phi_k_planes;
} enl_linear_args;

/* o = phi(Q) S_kv / (phi(Q) . s_k + eps) with S_kv = sum phi(k) v^T and
 * s_k = sum phi(k) over keys s <= t (causal, prefix sums) or all keys
 * (nn/attention_kernels.py:119-143). num_features <= enl_linear_max_features(). */
int enl_linear_attention(const enl_linear_args* args, void* stream);
int enl_linear_max_features(void);
/* 1 when enl_linear_attention runs these sizes on the tensor pipe and takes
 * phi planes (head_dim <= 128, num_features <= 1024), else 0. */
int enl_linear_planes_ok(int32_t head_dim, int32_t num_features);

/* Workspace bytes enl_linear_attention needs for these arguments: causal
 * calls long enough to run in parallel sequence segments keep one partial
 * state per segment; 0 otherwise. */
size_t enl_linear_workspace_bytes(const enl_linear_args* args);

/* --------------------------------------------------------------- backward */
typedef struct enl_backward_args {
  const void* q;    /* in_dtype (batch, seq_q, num_heads, head_dim), as given to the forward */
  const void* k;    /* in_dtype (batch, seq_kv, num_kv_heads, head_dim) */
  const void* v;    /* in_dtype (batch, seq_kv, num_kv_heads, head_dim) */
  const void* o;    /* forward output (batch, seq_q, num_heads, head_dim), o_dtype */
  const void* dout; /* in_dtype gradient of o, same shape */
  const float* lse; /* (batch, num_heads, seq_q) natural-log LSE from enl_attn_prefill */
  float* dq;        /* fp32 (batch, seq_q, num_heads, head_dim) */
  float* dk;        /* fp32 (batch, seq_kv, num_kv_heads, head_dim), summed over the group */
  float* dv;        /* fp32, as dk */
  int32_t batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim;
  int64_t q_stride_b, q_stride_s, q_stride_h; /* element strides */
  int64_t k_stride_b, k_stride_s, k_stride_h;
  int64_t v_stride_b, v_stride_s, v_stride_h;
  int64_t o_stride_b, o_stride_s, o_stride_h;
  int64_t do_stride_b, do_stride_s, do_stride_h;
  int64_t dq_stride_b, dq_stride_s, dq_stride_h;
  int64_t dk_stride_b, dk_stride_s, dk_stride_h;
  int64_t dv_stride_b, dv_stride_s, dv_stride_h;
  int32_t o_dtype;           /* ENL_DTYPE_BF16 or ENL_DTYPE_FP32 */
  int32_t causal;            /* as in the forward; query and key positions both start at 0 */
  int32_t window;            /* < 0: none */
  const float* alibi_slopes; /* device (num_heads,) or NULL */
  float scale;               /* the forward's softmax scale */
  void* workspace;           /* >= enl_backward_workspace_bytes(), 256-byte aligned */
  size_t workspace_bytes;
  int32_t in_dtype; /* q, k, v, dout: ENL_DTYPE_BF16, or ENL_DTYPE_FP32 (split-bf16 operands,
                       head_dim <= 64; 16-byte aligned, strides multiples of 4 elements) */
} enl_backward_args;

/* Attention backward: dQ, dK, dV of softmax(Q K^T * scale + bias + mask) V
 * from dO, recomputing the probabilities from the forward's LSE, as
 * nn/flash_attention.py:83-114 does with its row statistics. bf16 operands,
 * or fp32 operands split into bf16 hi/lo planes (three MMAs per product, as
 * the fp32 prefill), fp32 accumulation and outputs; head_dim a multiple of 8
 * up to 128 (up to 64 for fp32). With GQA, dK and dV of a kv head sum its
 * query heads (the adjoint of the reference's _repeat_kv,
 * nn/forward.py:165-171). */
int enl_attn_backward(const enl_backward_args* args, void* stream);

/* Workspace bytes enl_attn_backward needs: two fp32 rows per query, padded
 * to whole 128-row tiles, plus (fp32 inputs) the bf16 hi/lo planes of q, k,
 * v and dout. */
size_t enl_backward_workspace_bytes(const enl_backward_args* args);

/* -------------------------------------------------- block-sparse attention */
/* Which keys each query sees under a sparse_pattern, as 128 x 128 tiles.
 * The gather of nn/sparse_attention.py:107-135 (block_selection's index and
 * valid tables, the tail padding and the causal rule) becomes a per-query-
 * tile list of key tiles plus a column mask per query row. Query tile t
 * (rows [128t, 128t + 128)) visits the key tiles tile_kt[tile_ptr[t] ..
 * tile_ptr[t + 1]); row r of entry e sees key 128*tile_kt[e] + 64h + c iff
 * bit c of masks[(2e + h) * 128 + r] is set (h = 0, 1). All device memory. */
typedef struct enl_sparse_layout {
  const int32_t* tile_ptr;  /* (ceil(seq_q / 128) + 1) */
  const int32_t* tile_kt;   /* (n_entries) */
  const uint64_t* masks;    /* (n_entries, 2, 128) */
  int32_t n_entries;
} enl_sparse_layout;

typedef struct enl_sparse_mask_args {
  const int32_t* tile_ptr; /* device, as in enl_sparse_layout */
  const int32_t* tile_kt;  /* device */
  uint64_t* masks;         /* device out, (n_entries, 2, 128) */
  int32_t n_entries;
  /* block_selection's valid entries as a CSR over query blocks
   * [qb0, qb0 + n_qblocks): query block qb0 + i selects the key blocks
   * sel_kb[sel_ptr[i] .. sel_ptr[i + 1]) (absolute block numbers). */
  const int32_t* sel_ptr;  /* device (n_qblocks + 1) */
  const int32_t* sel_kb;   /* device (n_sel) */
  int32_t n_qblocks, n_sel;
  int64_t qb0;
  int32_t block_size;
  int32_t seq_q, seq_kv;
  int64_t q_pos0, k_pos0;  /* absolute positions of query row 0 and key row 0 */
  int32_t causal;          /* also drop keys after the query's position */
} enl_sparse_mask_args;

/* Fill the masks of a layout whose tile lists the caller built. */
int enl_sparse_build_masks(const enl_sparse_mask_args* args, void* stream);

/* Block-sparse attention: enl_attn_prefill with the keys of each query
 * restricted to its layout. Replaces nn/sparse_attention.py:96-142 (forward)
 * and the scores of nn/kvcache.py:263-306 (cached step, with q_pos0/k_pos0).
 * The layout carries causality and the sequence end; args->causal only picks
 * the ALiBi distance (signed when causal, absolute otherwise, :125-128).
 * Needs window < 0, mask_mode ENL_MASK_EXCLUDE and kv_valid_len NULL: every
 * row sees at least its own key, so there are no fully masked rows. */
int enl_attn_prefill_sparse(const enl_prefill_args* args, const enl_sparse_layout* layout,
                            void* stream);

/* ------------------------------------------------------------- utilities */
/* Read (and with clear != 0 reset) the device error word of the current
 * device. Synchronises the device. *code == 0 means no kernel reported. */
int enl_device_error(int32_t* code, int32_t* info, int32_t clear);

/* Message for the last failing call on this thread ("" if none). */
const char* enl_last_error(void);

/* Site code that enl_selftest_wait_timeout records in the device error word. */
#define ENL_SELFTEST_SITE 99

/* Diagnostic of the failure path every kernel wait takes: launches one warp
 * that waits on a barrier nothing arrives on, for budget_ns (1 us .. 100 ms),
 * then records a wait timeout (code 1, info ENL_SELFTEST_SITE) in the device
 * error word and returns. No trap and no hang: the context stays usable and
 * enl_device_error() reports the status. */
int enl_selftest_wait_timeout(int64_t budget_ns, void* stream);

/* Diagnostic of the exponentials K1 computes on the FMA pipe (one pair in
 * four of its softmax exponentials, on tiles without masked scores): for
 * each x[i] (device fp32, n entries) writes the scalar cubic, the packed
 * (f32x2) cubic and CUDA's exp2f of x[i]. Documented bound: relative error
 * <= 7.7e-5 for x in [-125, 8]; inputs below -125 give 2^-125. */
int enl_selftest_exp2(const float* x, float* y_poly, float* y_poly2, float* y_ref, int32_t n,
                      void* stream);

int enl_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ENL_ATTN_H_ */
