// C-ABI entry points of libenl_b200.so (declared in include/enl_attn.h):
// argument validation, TMA tensor-map construction and kernel launches.
#include <algorithm>
#include <cstdio>
#include <cstdarg>
#include <string>

#include "enl_attn.h"
#include "enl_common.cuh"
#include "enl_kernels.h"

// K1 work items come in sections of (batch, head) pairs whose K/V take about
// this many MiB, a quarter of the 126 MB L2 by default.
#ifndef ENL_PREFILL_SECTION_MB
#define ENL_PREFILL_SECTION_MB 32
#endif

namespace enl {
namespace {

thread_local std::string t_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(ENL_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D bf16 map over (head_dim, seq, heads, batch) with 128-byte swizzled
// boxes of 64 x 128 elements: exactly the K-major SW128 layout the UMMA
// descriptors in enl_prefill.cu expect.
int make_qkv_map(CUtensorMap* map, const void* base, int D, int S, int H, int B, int64_t ss,
                 int64_t sh, int64_t sb, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ENL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ENL_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name,
                (int)r);
  return ENL_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D bf16 map (inner, rows, depth) with element strides row_ld and depth_ld,
// 128-byte swizzled boxes of 64 x box_rows x 1.
int make_3d_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t depth,
                int64_t row_ld, int64_t depth_ld, uint32_t box_rows, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ENL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)depth};
  cuuint64_t strides[2] = {(cuuint64_t)(row_ld * 2), (cuuint64_t)(depth_ld * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ENL_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name,
                (int)r);
  return ENL_OK;
}

// Sizes of the tensor-core linear-attention path (enl_linear_tc.cu): which
// calls it takes (head_dim <= 128, at most 1024 features) and its workspace.
struct LinTcPlan {
  bool use;
  int Dp, Dfp, Sp, n_chunks;
  size_t off_qp, off_kp, off_vt, off_u, off_st, total;
};
bool lin_tc_sizes(int head_dim, int num_features) {
  return head_dim >= 1 && head_dim <= 128 && num_features >= 1 && num_features <= 1024;
}
bool lin_planes_given(const enl_linear_args* a) { return a->phi_q_planes && a->phi_k_planes; }
// With phi planes given, the qp / kp regions are empty and the caller's
// planes are read in their place.
LinTcPlan lin_tc_plan(const enl_linear_args* a) {
  LinTcPlan pl{};
  pl.use = lin_tc_sizes(a->head_dim, a->num_features) && a->seq >= 1 && a->batch >= 1;
  if (!pl.use) return pl;
  const bool given = lin_planes_given(a);
  const size_t B = a->batch, H = a->num_heads, Hk = a->num_kv_heads, S = a->seq;
  const size_t Df = a->num_features;
  pl.Dp = ((a->head_dim + 1 + 15) / 16) * 16;
  pl.Dfp = (int)((Df + 7) / 8 * 8);
  pl.Sp = (int)((S + 7) / 8 * 8);
  pl.n_chunks = (int)((S + 127) / 128);
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t off = 0;
  pl.off_qp = off;
  if (!given) off += al(2 * B * H * S * pl.Dfp * 2);
  pl.off_kp = off;
  if (!given) off += al(2 * B * Hk * S * pl.Dfp * 2);
  pl.off_vt = off;
  off += al(2 * B * Hk * (size_t)pl.Dp * pl.Sp * 2);
  pl.off_u = off;
  off += al(B * Hk * (size_t)pl.n_chunks * Df * pl.Dp * 4);
  pl.off_st = off;
  off += al(2 * B * Hk * (size_t)pl.n_chunks * pl.Dp * pl.Dfp * 2);
  pl.total = off;
  return pl;
}

// 2-D map over a row-major (rows, cols) matrix with a 128-byte swizzled box of
// box_cols x box_rows elements (box_cols * element size = 128 bytes).
int make_2d_map(CUtensorMap* map, const void* base, bool fp32, int64_t cols, int64_t rows,
                int64_t ld, uint32_t box_cols, uint32_t box_rows, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ENL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int esz = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ENL_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name,
                (int)r);
  return ENL_OK;
}

// SM count of the current device, cached per device.
int sm_count(int* out) {
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(ENL_ERR_UNSUPPORTED, "device ordinal %d >= 64", dev);
  if (cached[dev] == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(multiProcessorCount)");
    cached[dev] = n;
  }
  *out = cached[dev];
  return ENL_OK;
}

int check_strides_16B(const char* name, int64_t sb, int64_t ss, int64_t sh, int elem_bytes) {
  const int64_t v[3] = {sb, ss, sh};
  for (int i = 0; i < 3; ++i)
    if (v[i] < 0 || (v[i] * elem_bytes) % 16 != 0)
      return fail(ENL_ERR_INVALID,
                  "%s strides (%lld, %lld, %lld) must be non-negative multiples of 16 bytes",
                  name, (long long)sb, (long long)ss, (long long)sh);
  return ENL_OK;
}

}  // namespace
}  // namespace enl

using namespace enl;

extern "C" {

const char* enl_last_error(void) { return t_last_error.c_str(); }

int enl_abi_version(void) { return ENL_ABI_VERSION; }

int enl_device_error(int32_t* code, int32_t* info, int32_t clear) {
  int c = 0, i = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "enl_device_error: cudaDeviceSynchronize");
  e = cudaMemcpyFromSymbol(&c, g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&i, g_device_error_info, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "enl_device_error: read");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error_info, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "enl_device_error: clear");
  }
  if (code) *code = c;
  if (info) *info = i;
  return ENL_OK;
}

}  // extern "C"

namespace enl {
namespace {

// enl_attn_prefill, and enl_attn_prefill_sparse when layout is set.
int prefill_impl(const enl_prefill_args* a, const enl_sparse_layout* layout, void* stream) {
  if (!a) return fail(ENL_ERR_INVALID, "enl_attn_prefill: args is NULL");
  if (!a->q || !a->k || !a->v || !a->o)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: q, k, v and o must be non-NULL");
  if (a->batch < 1 || a->num_heads < 1 || a->num_kv_heads < 1 || a->seq_q < 1 || a->seq_kv < 1)
    return fail(ENL_ERR_INVALID,
                "enl_attn_prefill: batch=%d num_heads=%d num_kv_heads=%d seq_q=%d seq_kv=%d "
                "must all be >= 1",
                a->batch, a->num_heads, a->num_kv_heads, a->seq_q, a->seq_kv);
  if (a->num_heads % a->num_kv_heads != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: num_kv_heads=%d must divide num_heads=%d",
                a->num_kv_heads, a->num_heads);
  if (a->head_dim < 8 || a->head_dim > 128 || a->head_dim % 8 != 0)
    return fail(ENL_ERR_UNSUPPORTED,
                "enl_attn_prefill: head_dim=%d (supported: multiples of 8 up to 128)",
                a->head_dim);
  if (a->in_dtype != ENL_DTYPE_BF16 && a->in_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: in_dtype=%d", a->in_dtype);
  const bool split = a->in_dtype == ENL_DTYPE_FP32;
  const int esz = split ? 4 : 2;
  if (a->out_dtype != ENL_DTYPE_BF16 && a->out_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: out_dtype=%d", a->out_dtype);
  if (a->mask_mode != ENL_MASK_EXCLUDE && a->mask_mode != ENL_MASK_ADDITIVE)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: mask_mode=%d", a->mask_mode);
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o))
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: q, k, v, o must be 16-byte aligned");
  int st;
  if ((st = check_strides_16B("q", a->q_stride_b, a->q_stride_s, a->q_stride_h, esz))) return st;
  if ((st = check_strides_16B("k", a->k_stride_b, a->k_stride_s, a->k_stride_h, esz))) return st;
  if ((st = check_strides_16B("v", a->v_stride_b, a->v_stride_s, a->v_stride_h, esz))) return st;
  if ((st = check_strides_16B("o", a->o_stride_b, a->o_stride_s, a->o_stride_h,
                              a->out_dtype == ENL_DTYPE_FP32 ? 4 : 2)))
    return st;
  if (a->kv_mask) {
    if ((reinterpret_cast<uintptr_t>(a->kv_mask) & 7u) != 0)
      return fail(ENL_ERR_INVALID, "enl_attn_prefill: kv_mask must be 8-byte aligned");
    if (a->kv_mask_stride_b < (a->seq_kv + 63) / 64)
      return fail(ENL_ERR_INVALID,
                  "enl_attn_prefill: kv_mask_stride_b=%lld words is less than ceil(seq_kv/64)=%d",
                  (long long)a->kv_mask_stride_b, (a->seq_kv + 63) / 64);
    const size_t need = enl_prefill_workspace_bytes(a);
    if (!a->workspace || a->workspace_bytes < need)
      return fail(ENL_ERR_INVALID,
                  "enl_attn_prefill: kv_mask needs a %zu-byte workspace (got %zu)", need,
                  a->workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
      return fail(ENL_ERR_INVALID, "enl_attn_prefill: workspace must be 256-byte aligned");
  }
  if ((long long)a->batch * a->num_heads > 65535)
    return fail(ENL_ERR_UNSUPPORTED, "enl_attn_prefill: batch*num_heads=%lld exceeds 65535",
                (long long)a->batch * a->num_heads);

  // The kernel runs at D = 64 or 128; smaller head dims are zero-filled by
  // TMA (the tensor maps keep the real extent) and never stored.
  const int D = a->head_dim <= 64 ? 64 : 128;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap tq, tk, tv;
  if (!split) {
    if ((st = make_qkv_map(&tq, a->q, a->head_dim, a->seq_q, a->num_heads, a->batch,
                           a->q_stride_s, a->q_stride_h, a->q_stride_b, "q")))
      return st;
    if ((st = make_qkv_map(&tk, a->k, a->head_dim, a->seq_kv, a->num_kv_heads, a->batch,
                           a->k_stride_s, a->k_stride_h, a->k_stride_b, "k")))
      return st;
    if ((st = make_qkv_map(&tv, a->v, a->head_dim, a->seq_kv, a->num_kv_heads, a->batch,
                           a->v_stride_s, a->v_stride_h, a->v_stride_b, "v")))
      return st;
  } else {
    // fp32: (hi, lo) planes of q, k, v in the workspace, then tensor maps
    // over them with the planes as 2 * heads "heads" of a contiguous tensor.
    const size_t need = enl_prefill_workspace_bytes(a);
    if (!a->workspace || a->workspace_bytes < need)
      return fail(ENL_ERR_INVALID,
                  "enl_attn_prefill: fp32 inputs need a %zu-byte workspace (got %zu)", need,
                  a->workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
      return fail(ENL_ERR_INVALID, "enl_attn_prefill: workspace must be 256-byte aligned");
    const int Dr = a->head_dim;
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
    struct Op {
      const void* src;
      int64_t sb, ss, sh;
      int S, H;
      CUtensorMap* map;
      const char* name;
    } ops[3] = {{a->q, a->q_stride_b, a->q_stride_s, a->q_stride_h, a->seq_q, a->num_heads, &tq, "q"},
                {a->k, a->k_stride_b, a->k_stride_s, a->k_stride_h, a->seq_kv, a->num_kv_heads, &tk, "k"},
                {a->v, a->v_stride_b, a->v_stride_s, a->v_stride_h, a->seq_kv, a->num_kv_heads, &tv, "v"}};
    for (const Op& op : ops) {
      const int64_t hs = Dr, ss = 2ll * op.H * Dr, bs = ss * op.S;  // plane tensor strides
      cudaError_t e = launch_split_planes(reinterpret_cast<const float*>(op.src), op.sb, op.ss,
                                          op.sh, a->batch, op.S, op.H, Dr, ws, s);
      if (e != cudaSuccess) return cuda_fail(e, "enl_attn_prefill: split planes");
      if ((st = make_qkv_map(op.map, ws, Dr, op.S, 2 * op.H, a->batch, ss, hs, bs, op.name)))
        return st;
      ws += (((size_t)a->batch * bs * 2) + 255) & ~size_t(255);
    }
  }

  PrefillParams p;
  p.d_real = a->head_dim;
  p.B = a->batch;
  p.H = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.Sq = a->seq_q;
  p.Skv = a->seq_kv;
  p.o = a->o;
  p.o_sb = a->o_stride_b;
  p.o_ss = a->o_stride_s;
  p.o_sh = a->o_stride_h;
  p.out_fp32 = a->out_dtype == ENL_DTYPE_FP32;
  p.lse = a->lse;
  p.causal = a->causal != 0;
  p.window = a->window < 0 ? -1 : a->window;
  p.additive = a->mask_mode == ENL_MASK_ADDITIVE;
  p.kv_len = a->kv_valid_len;
  p.alibi = a->alibi_slopes;
  p.q_pos0 = a->q_pos0;
  p.k_pos0 = a->k_pos0;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.sp_ptr = layout ? layout->tile_ptr : nullptr;
  p.sp_kt = layout ? layout->tile_kt : nullptr;
  p.sp_mask = layout ? reinterpret_cast<const unsigned long long*>(layout->masks) : nullptr;
  p.sp_entries = layout ? layout->n_entries : 0;
  p.kv_mask = reinterpret_cast<const unsigned long long*>(a->kv_mask);
  p.kv_mask_sb = a->kv_mask_stride_b;
  p.mask_tiles = nullptr;
  if (a->kv_mask) {
    // The tile ranges sit after the fp32 planes (if any) in the workspace.
    enl_prefill_args planes_only = *a;
    planes_only.kv_mask = nullptr;
    int4* tiles = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(a->workspace) +
                                          enl_prefill_workspace_bytes(&planes_only));
    p.mask_tiles = tiles;
  }
  // One persistent CTA per SM. Sections of (batch, head) pairs whose K/V
  // fit in about a quarter of L2 keep the concurrently running items on
  // shared keys.
  if (a->units && a->n_units < 0)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: n_units=%d must be >= 0", a->n_units);
  if (a->units && (reinterpret_cast<uintptr_t>(a->units) & 3u) != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill: units must be 4-byte aligned");
  p.units = a->units;
  p.n_bh = a->units ? a->n_units : a->batch * a->num_heads;
  {
    const long long n_qt = (a->seq_q + 127) / 128;
    const long long n_items = (long long)p.n_bh * n_qt;
    if (n_items > (1ll << 30))
      return fail(ENL_ERR_UNSUPPORTED, "enl_attn_prefill: %lld query tiles exceed 2^30", n_items);
    p.n_items = (int)n_items;
    int sms = 0;
    if ((st = sm_count(&sms))) return st;
    p.n_ctas = sms;
    const int G = a->num_heads / a->num_kv_heads;
    const double kv_bytes_per_head =
        4.0 * a->seq_kv * D * (split ? 2 : 1) / G;  // K and V, bf16, shared by G heads
    const double budget = ENL_PREFILL_SECTION_MB * double(1 << 20);
    long long sec = (long long)(budget / kv_bytes_per_head);
    const long long n_bh = std::max(1, p.n_bh);
    p.sec_bh = (int)std::max(1ll, std::min(n_bh, sec));
  }

  if (p.mask_tiles) {
    cudaError_t e = launch_mask_tiles(p, const_cast<int4*>(p.mask_tiles), s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_attn_prefill: mask tiles launch");
  }

  // O map for the kernel's TMA-store epilogue (bf16 output of bf16 inputs).
  CUtensorMap to = tq;
  if (!split && a->out_dtype == ENL_DTYPE_BF16 &&
      (st = make_qkv_map(&to, a->o, a->head_dim, a->seq_q, a->num_heads, a->batch, a->o_stride_s,
                         a->o_stride_h, a->o_stride_b, "o")))
    return st;

  cudaError_t e;
  if (split)
    e = (D == 128) ? launch_prefill<128, true>(tq, tk, tv, to, p, s)
                   : launch_prefill<64, true>(tq, tk, tv, to, p, s);
  else
    e = (D == 128) ? launch_prefill<128, false>(tq, tk, tv, to, p, s)
                   : launch_prefill<64, false>(tq, tk, tv, to, p, s);
  if (e != cudaSuccess) return cuda_fail(e, "enl_attn_prefill launch");
  return ENL_OK;
}

}  // namespace
}  // namespace enl

extern "C" {

int enl_attn_prefill(const enl_prefill_args* a, void* stream) {
  return prefill_impl(a, nullptr, stream);
}

int enl_attn_prefill_sparse(const enl_prefill_args* a, const enl_sparse_layout* l,
                            void* stream) {
  if (!a || !l) return fail(ENL_ERR_INVALID, "enl_attn_prefill_sparse: args or layout is NULL");
  if (!l->tile_ptr || !l->tile_kt || !l->masks || l->n_entries < 0)
    return fail(ENL_ERR_INVALID,
                "enl_attn_prefill_sparse: layout needs tile_ptr, tile_kt, masks and "
                "n_entries >= 0");
  if ((reinterpret_cast<uintptr_t>(l->masks) & 7u) != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_prefill_sparse: masks must be 8-byte aligned");
  if (a->window >= 0 || a->mask_mode != ENL_MASK_EXCLUDE || a->kv_valid_len || a->kv_mask)
    return fail(ENL_ERR_INVALID,
                "enl_attn_prefill_sparse: the layout is the whole mask; window must be < 0, "
                "mask_mode ENL_MASK_EXCLUDE and kv_valid_len and kv_mask NULL");
  return prefill_impl(a, l, stream);
}

size_t enl_project_workspace_bytes(const enl_project_args* a) {
  if (!a || a->x_dtype != ENL_DTYPE_FP32 || a->M < 1 || a->K < 1) return 0;
  const size_t plane = ((size_t)a->M * a->K * 2 + 255) & ~size_t(255);
  return 2 * plane;
}

int enl_project(const enl_project_args* a, void* stream) {
  if (!a) return fail(ENL_ERR_INVALID, "enl_project: args is NULL");
  // With M == 0 there are no rows: x and y may be NULL (an empty tensor's
  // address); the call checks its other arguments and does nothing.
  if ((a->M != 0 && (!a->x || !a->y)) || !a->w)
    return fail(ENL_ERR_INVALID, "enl_project: x, w and y must be non-NULL");
  if (a->M < 0 || a->N < 1 || a->K < 1)
    return fail(ENL_ERR_INVALID, "enl_project: M=%d N=%d K=%d (M >= 0, N and K >= 1)", a->M,
                a->N, a->K);
  if (a->K % 8 != 0 || a->N % 8 != 0)
    return fail(ENL_ERR_UNSUPPORTED, "enl_project: K=%d and N=%d must be multiples of 8", a->K,
                a->N);
  if (a->x_dtype != ENL_DTYPE_BF16 && a->x_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_project: x_dtype=%d", a->x_dtype);
  if (a->y_dtype != ENL_DTYPE_BF16 && a->y_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_project: y_dtype=%d", a->y_dtype);
  const bool split = a->x_dtype == ENL_DTYPE_FP32;
  if (split && !a->w_lo)
    return fail(ENL_ERR_INVALID, "enl_project: fp32 x needs the weight's lo plane w_lo");
  if (!split && a->w_lo)
    return fail(ENL_ERR_INVALID, "enl_project: w_lo is only used with fp32 x");
  const int xsz = split ? 4 : 2, ysz = a->y_dtype == ENL_DTYPE_FP32 ? 4 : 2;
  if ((a->x && !aligned16(a->x)) || !aligned16(a->w) || (a->y && !aligned16(a->y)) ||
      (a->w_lo && !aligned16(a->w_lo)))
    return fail(ENL_ERR_INVALID, "enl_project: x, w, w_lo and y must be 16-byte aligned");
  if (a->x_stride_m < a->K || (a->x_stride_m * xsz) % 16 != 0 || a->w_stride_n < a->K ||
      (a->w_stride_n * 2) % 16 != 0 || a->y_stride_m < a->N || (a->y_stride_m * ysz) % 16 != 0)
    return fail(ENL_ERR_INVALID,
                "enl_project: row strides (x %lld, w %lld, y %lld) must cover a row and be "
                "multiples of 16 bytes",
                (long long)a->x_stride_m, (long long)a->w_stride_n, (long long)a->y_stride_m);
  if (a->bias && (reinterpret_cast<uintptr_t>(a->bias) & 15u) != 0)
    return fail(ENL_ERR_INVALID, "enl_project: bias must be 16-byte aligned");
  if (a->rope_cols < 0 || a->rope_cols > a->N)
    return fail(ENL_ERR_INVALID, "enl_project: rope_cols=%d outside [0, N=%d]", a->rope_cols,
                a->N);
  if (a->rope_cols > 0) {
    const int d = a->rope_head_dim;
    if (d != 8 && d != 16 && d != 32 && d != 64 && d != 128)
      return fail(ENL_ERR_UNSUPPORTED,
                  "enl_project: rope_head_dim=%d (fused RoPE: 8, 16, 32, 64 or 128)", d);
    if (a->rope_cols % d != 0)
      return fail(ENL_ERR_INVALID, "enl_project: rope_cols=%d is not whole heads of %d",
                  a->rope_cols, d);
    if (!a->rope_cos || !a->rope_sin || a->rope_seq < 1 || a->rope_pos0 < 0)
      return fail(ENL_ERR_INVALID,
                  "enl_project: RoPE needs cos/sin tables, rope_seq >= 1 and rope_pos0 >= 0");
    const long long last = a->rope_pos0 + std::min<long long>(a->rope_seq, std::max(a->M, 1)) - 1;
    if (last >= a->rope_rows)
      return fail(ENL_ERR_INVALID, "enl_project: RoPE position %lld beyond the %lld table rows",
                  last, (long long)a->rope_rows);
    if ((reinterpret_cast<uintptr_t>(a->rope_cos) & 15u) ||
        (reinterpret_cast<uintptr_t>(a->rope_sin) & 15u))
      return fail(ENL_ERR_INVALID, "enl_project: RoPE tables must be 16-byte aligned");
  }
  if (a->M == 0) return ENL_OK;
  int st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  CUtensorMap tx, txlo, tw, twlo, ty;
  if (split) {
    const size_t need = enl_project_workspace_bytes(a);
    if (!a->workspace || a->workspace_bytes < need)
      return fail(ENL_ERR_INVALID, "enl_project: fp32 x needs a %zu-byte workspace (got %zu)",
                  need, a->workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
      return fail(ENL_ERR_INVALID, "enl_project: workspace must be 256-byte aligned");
    uint8_t* hi = reinterpret_cast<uint8_t*>(a->workspace);
    uint8_t* lo = hi + need / 2;
    cudaError_t e = launch_split_matrix(reinterpret_cast<const float*>(a->x), a->x_stride_m, a->M,
                                        a->K, hi, lo, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_project: split x");
    if ((st = make_2d_map(&tx, hi, false, a->K, a->M, a->K, 64, 128, "x hi"))) return st;
    if ((st = make_2d_map(&txlo, lo, false, a->K, a->M, a->K, 64, 128, "x lo"))) return st;
    if ((st = make_2d_map(&twlo, a->w_lo, false, a->K, a->N, a->w_stride_n, 64, 128, "w lo")))
      return st;
  } else {
    if ((st = make_2d_map(&tx, a->x, false, a->K, a->M, a->x_stride_m, 64, 128, "x"))) return st;
    txlo = tx;
  }
  if ((st = make_2d_map(&tw, a->w, false, a->K, a->N, a->w_stride_n, 64, 128, "w"))) return st;
  if (!split) twlo = tw;
  const bool yf32 = a->y_dtype == ENL_DTYPE_FP32;
  if ((st = make_2d_map(&ty, a->y, yf32, a->N, a->M, a->y_stride_m, yf32 ? 32 : 64, 32, "y")))
    return st;
  ProjParams p;
  p.M = a->M;
  p.N = a->N;
  p.K = a->K;
  p.bias = a->bias;
  p.out_fp32 = yf32;
  p.rope_cols = a->rope_cols;
  p.rope_d = a->rope_cols > 0 ? a->rope_head_dim : 128;
  p.rope_seq = a->rope_cols > 0 ? a->rope_seq : 0;
  p.rope_pos0 = a->rope_pos0;
  p.rope_cos = a->rope_cos;
  p.rope_sin = a->rope_sin;
  int sms = 0;
  if ((st = sm_count(&sms))) return st;
  cudaError_t e = split ? launch_proj_gemm<true>(tx, txlo, tw, twlo, ty, p, sms, s)
                        : launch_proj_gemm<false>(tx, txlo, tw, twlo, ty, p, sms, s);
  if (e != cudaSuccess) return cuda_fail(e, "enl_project launch");
  return ENL_OK;
}

int enl_split_bf16(const float* src, int64_t ld, int64_t rows, int32_t cols, void* hi, void* lo,
                   void* stream) {
  if (!src || !hi || !lo) return fail(ENL_ERR_INVALID, "enl_split_bf16: NULL pointer");
  if (rows < 0 || cols < 0 || cols % 4 != 0 || ld < cols || ld % 4 != 0)
    return fail(ENL_ERR_INVALID, "enl_split_bf16: rows=%lld cols=%d ld=%lld (cols, ld multiples "
                "of 4, ld >= cols)", (long long)rows, cols, (long long)ld);
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(hi) & 7u) ||
      (reinterpret_cast<uintptr_t>(lo) & 7u))
    return fail(ENL_ERR_INVALID, "enl_split_bf16: src must be 16-byte and planes 8-byte aligned");
  cudaError_t e = launch_split_matrix(src, ld, rows, cols, hi, lo,
                                      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_split_bf16 launch");
  return ENL_OK;
}

namespace {
// Bytes of the row statistics (lse2, dsum), each rounded to 256.
size_t bwd_rows_bytes(const enl_backward_args* a) {
  const size_t s_pad = ((size_t)a->seq_q + 127) / 128 * 128;
  return ((size_t)a->batch * a->num_heads * s_pad * sizeof(float) + 255) & ~size_t(255);
}
// Bytes of one operand's bf16 (hi, lo) planes, rounded to 256.
size_t bwd_planes_bytes(const enl_backward_args* a, int S, int H) {
  return ((size_t)a->batch * S * H * a->head_dim * 2 * sizeof(uint16_t) + 255) & ~size_t(255);
}
}  // namespace

size_t enl_backward_workspace_bytes(const enl_backward_args* a) {
  if (!a || a->batch < 1 || a->num_heads < 1 || a->seq_q < 1) return 0;
  size_t total = 2 * bwd_rows_bytes(a);
  if (a->in_dtype == ENL_DTYPE_FP32 && a->seq_kv >= 1 && a->num_kv_heads >= 1 &&
      a->head_dim >= 1)
    total += 2 * bwd_planes_bytes(a, a->seq_q, a->num_heads) +
             2 * bwd_planes_bytes(a, a->seq_kv, a->num_kv_heads);
  return total;
}

int enl_attn_backward(const enl_backward_args* a, void* stream) {
  if (!a) return fail(ENL_ERR_INVALID, "enl_attn_backward: args is NULL");
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv)
    return fail(ENL_ERR_INVALID,
                "enl_attn_backward: q, k, v, o, dout, lse, dq, dk and dv must be non-NULL");
  if (a->batch < 1 || a->num_heads < 1 || a->num_kv_heads < 1 || a->seq_q < 1 || a->seq_kv < 1)
    return fail(ENL_ERR_INVALID,
                "enl_attn_backward: batch=%d num_heads=%d num_kv_heads=%d seq_q=%d seq_kv=%d "
                "must all be >= 1",
                a->batch, a->num_heads, a->num_kv_heads, a->seq_q, a->seq_kv);
  if (a->num_heads % a->num_kv_heads != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_backward: num_kv_heads=%d must divide num_heads=%d",
                a->num_kv_heads, a->num_heads);
  if (a->head_dim < 8 || a->head_dim > 128 || a->head_dim % 8 != 0)
    return fail(ENL_ERR_UNSUPPORTED,
                "enl_attn_backward: head_dim=%d (supported: multiples of 8 up to 128)",
                a->head_dim);
  if (a->o_dtype != ENL_DTYPE_BF16 && a->o_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_backward: o_dtype=%d", a->o_dtype);
  if (a->in_dtype != ENL_DTYPE_BF16 && a->in_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_backward: in_dtype=%d", a->in_dtype);
  const bool split = a->in_dtype == ENL_DTYPE_FP32;
  if (split && a->head_dim > 64)
    return fail(ENL_ERR_UNSUPPORTED,
                "enl_attn_backward: fp32 inputs (split-bf16 operands) cover head_dim <= 64 "
                "(got %d): the planes of a 128-wide head do not fit in shared memory",
                a->head_dim);
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->dout))
    return fail(ENL_ERR_INVALID, "enl_attn_backward: q, k, v, dout must be 16-byte aligned");
  int st;
  const int esz = split ? 4 : 2;
  if ((st = check_strides_16B("q", a->q_stride_b, a->q_stride_s, a->q_stride_h, esz))) return st;
  if ((st = check_strides_16B("k", a->k_stride_b, a->k_stride_s, a->k_stride_h, esz))) return st;
  if ((st = check_strides_16B("v", a->v_stride_b, a->v_stride_s, a->v_stride_h, esz))) return st;
  if ((st = check_strides_16B("dout", a->do_stride_b, a->do_stride_s, a->do_stride_h, esz)))
    return st;
  const long long n_kt = (a->seq_kv + 127) / 128, n_qt = (a->seq_q + 127) / 128;
  if (n_kt * a->batch * a->num_kv_heads > (1ll << 31) - 1 ||
      n_qt * a->batch * a->num_heads > (1ll << 31) - 1)
    return fail(ENL_ERR_UNSUPPORTED, "enl_attn_backward: too many tiles for one launch");
  const size_t need = enl_backward_workspace_bytes(a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(ENL_ERR_INVALID, "enl_attn_backward: needs a %zu-byte workspace (got %zu)", need,
                a->workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_backward: workspace must be 256-byte aligned");

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t rows_bytes = bwd_rows_bytes(a);
  CUtensorMap tq, tk, tv, tdo;
  struct Op {
    const void* src;
    int64_t sb, ss, sh;
    int S, H;
    CUtensorMap* map;
    const char* name;
  } ops[4] = {
      {a->q, a->q_stride_b, a->q_stride_s, a->q_stride_h, a->seq_q, a->num_heads, &tq, "q"},
      {a->k, a->k_stride_b, a->k_stride_s, a->k_stride_h, a->seq_kv, a->num_kv_heads, &tk, "k"},
      {a->v, a->v_stride_b, a->v_stride_s, a->v_stride_h, a->seq_kv, a->num_kv_heads, &tv, "v"},
      {a->dout, a->do_stride_b, a->do_stride_s, a->do_stride_h, a->seq_q, a->num_heads, &tdo,
       "dout"}};
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace) + 2 * rows_bytes;
  for (const Op& op : ops) {
    if (!split) {
      if ((st = make_qkv_map(op.map, op.src, a->head_dim, op.S, op.H, a->batch, op.ss, op.sh,
                             op.sb, op.name)))
        return st;
      continue;
    }
    // fp32: (hi, lo) planes in the workspace, mapped with the planes as
    // 2 * heads "heads" of a contiguous tensor, as the fp32 prefill does.
    const int Dr = a->head_dim;
    const int64_t hs = Dr, ss = 2ll * op.H * Dr, bs = ss * op.S;
    cudaError_t e = launch_split_planes(reinterpret_cast<const float*>(op.src), op.sb, op.ss,
                                        op.sh, a->batch, op.S, op.H, Dr, ws, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_attn_backward: split planes");
    if ((st = make_qkv_map(op.map, ws, Dr, op.S, 2 * op.H, a->batch, ss, hs, bs, op.name)))
      return st;
    ws += bwd_planes_bytes(a, op.S, op.H);
  }

  const int s_pad = (int)(n_qt * 128);
  float* lse2 = reinterpret_cast<float*>(a->workspace);
  float* dsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a->workspace) + rows_bytes);
  BwdPrepParams q;
  q.B = a->batch;
  q.H = a->num_heads;
  q.Sq = a->seq_q;
  q.s_pad = s_pad;
  q.d_real = a->head_dim;
  q.o = a->o;
  q.o_sb = a->o_stride_b;
  q.o_ss = a->o_stride_s;
  q.o_sh = a->o_stride_h;
  q.o_f32 = a->o_dtype == ENL_DTYPE_FP32;
  q.dout = a->dout;
  q.do_f32 = split;
  q.do_sb = a->do_stride_b;
  q.do_ss = a->do_stride_s;
  q.do_sh = a->do_stride_h;
  q.lse = a->lse;
  q.lse2 = lse2;
  q.dsum = dsum;

  BwdParams p;
  p.B = a->batch;
  p.H = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.Sq = a->seq_q;
  p.Skv = a->seq_kv;
  p.d_real = a->head_dim;
  p.causal = a->causal != 0;
  p.window = a->window < 0 ? -1 : a->window;
  p.alibi = a->alibi_slopes;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.lse2 = lse2;
  p.dsum = dsum;
  p.s_pad = s_pad;
  p.dq = a->dq;
  p.dq_sb = a->dq_stride_b;
  p.dq_ss = a->dq_stride_s;
  p.dq_sh = a->dq_stride_h;
  p.dk = a->dk;
  p.dk_sb = a->dk_stride_b;
  p.dk_ss = a->dk_stride_s;
  p.dk_sh = a->dk_stride_h;
  p.dv = a->dv;
  p.dv_sb = a->dv_stride_b;
  p.dv_ss = a->dv_stride_s;
  p.dv_sh = a->dv_stride_h;
  {
    auto v4 = [](const void* ptr, int64_t x, int64_t y, int64_t z) {
      return aligned16(ptr) && x % 4 == 0 && y % 4 == 0 && z % 4 == 0;
    };
    p.out_vec4 = v4(a->dq, a->dq_stride_b, a->dq_stride_s, a->dq_stride_h) &&
                 v4(a->dk, a->dk_stride_b, a->dk_stride_s, a->dk_stride_h) &&
                 v4(a->dv, a->dv_stride_b, a->dv_stride_s, a->dv_stride_h);
  }
  const int D = a->head_dim <= 64 ? 64 : 128;
  cudaError_t e = launch_backward(tq, tk, tv, tdo, q, p, D, split, s);
  if (e != cudaSuccess) return cuda_fail(e, "enl_attn_backward launch");
  return ENL_OK;
}

int enl_sparse_build_masks(const enl_sparse_mask_args* a, void* stream) {
  if (!a) return fail(ENL_ERR_INVALID, "enl_sparse_build_masks: args is NULL");
  if (!a->tile_ptr || !a->tile_kt || !a->masks || !a->sel_ptr || (!a->sel_kb && a->n_sel > 0))
    return fail(ENL_ERR_INVALID, "enl_sparse_build_masks: NULL device pointer");
  if (a->block_size < 1 || a->seq_q < 1 || a->seq_kv < 1 || a->n_entries < 0 ||
      a->n_qblocks < 1 || a->n_sel < 0 || a->q_pos0 < 0 || a->k_pos0 < 0 || a->qb0 < 0)
    return fail(ENL_ERR_INVALID,
                "enl_sparse_build_masks: block_size=%d seq_q=%d seq_kv=%d n_entries=%d "
                "n_qblocks=%d n_sel=%d q_pos0=%lld k_pos0=%lld qb0=%lld out of range",
                a->block_size, a->seq_q, a->seq_kv, a->n_entries, a->n_qblocks, a->n_sel,
                (long long)a->q_pos0, (long long)a->k_pos0, (long long)a->qb0);
  if ((reinterpret_cast<uintptr_t>(a->masks) & 7u) != 0)
    return fail(ENL_ERR_INVALID, "enl_sparse_build_masks: masks must be 8-byte aligned");
  SparseMaskParams p;
  p.tile_ptr = a->tile_ptr;
  p.tile_kt = a->tile_kt;
  p.masks = reinterpret_cast<unsigned long long*>(a->masks);
  p.n_qtiles = (a->seq_q + 127) / 128;
  p.n_entries = a->n_entries;
  p.sel_ptr = a->sel_ptr;
  p.sel_kb = a->sel_kb;
  p.n_qblocks = a->n_qblocks;
  p.n_sel = a->n_sel;
  p.qb0 = a->qb0;
  p.block_size = a->block_size;
  p.seq_q = a->seq_q;
  p.seq_kv = a->seq_kv;
  p.causal = a->causal != 0;
  p.q_pos0 = a->q_pos0;
  p.k_pos0 = a->k_pos0;
  cudaError_t e = launch_sparse_masks(p, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_sparse_build_masks launch");
  return ENL_OK;
}

size_t enl_prefill_workspace_bytes(const enl_prefill_args* a) {
  if (!a || a->batch < 1 || a->seq_q < 1 || a->seq_kv < 1) return 0;
  size_t total = 0;
  if (a->in_dtype == ENL_DTYPE_FP32) {
    auto planes = [&](int S, int H) {
      return (((size_t)a->batch * S * H * 2 * a->head_dim * 2) + 255) & ~size_t(255);
    };
    total += planes(a->seq_q, a->num_heads) + 2 * planes(a->seq_kv, a->num_kv_heads);
  }
  if (a->kv_mask) total += (size_t)a->batch * ((a->seq_q + 127) / 128) * 16;
  return total;
}

int enl_decode_auto_splits(int32_t batch, int32_t num_kv_heads, int32_t n_slots) {
  if (batch < 1 || num_kv_heads < 1 || n_slots < 1) return 1;
  const long long units = (long long)batch * num_kv_heads;
  int sms = 0;
  const std::string saved = t_last_error;  // a query that fails here is not the caller's error
  if (sm_count(&sms) != ENL_OK || sms < 1) sms = 148;  // no device: size for a B200
  t_last_error = saved;
  const long long target_ctas = (long long)sms * 32;  // enough CTAs to balance the SMs
  long long splits = (target_ctas + units - 1) / units;
  const long long max_splits = (n_slots + 511) / 512;  // keep >= ~512 slots per split
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 1024) splits = 1024;
  return (int)splits;
}

size_t enl_decode_workspace_bytes(int32_t batch, int32_t num_heads, int32_t head_dim,
                                  int32_t n_splits) {
  if (n_splits <= 1) return 0;
  const int dk = head_dim <= 64 ? 64 : 128;  // the kernel's (zero-extended) head dim
  return (size_t)n_splits * batch * num_heads * (dk + 1) * sizeof(float);
}

namespace enl {
// The slot range a decode actually streams -- [slot_begin, slot_end)
// narrowed by causality (keys after the query are invisible) and by the
// sliding window -- and the split count and length it runs with.
void decode_plan(const enl_decode_args* a, long long* lo_out, long long* hi_out, int* splits_out,
                 int* split_len_out) {
  long long lo = a->slot_begin, hi = a->slot_end;
  const long long q_slot = a->q_pos - a->pos_slot0;  // slot holding the query position
  if (hi > q_slot + 1) hi = q_slot + 1;
  if (a->window >= 0 && lo < q_slot - a->window) lo = q_slot - a->window;
  if (hi < lo) hi = lo;
  const int n_slots = (int)(hi - lo);
  int splits = a->n_splits > 0 ? a->n_splits : enl_decode_auto_splits(a->batch, a->num_kv_heads,
                                                                      n_slots > 0 ? n_slots : 1);
  if (n_slots <= 1) splits = 1;
  int split_len = (n_slots + splits - 1) / splits;
  if (split_len < 1) split_len = 1;
  splits = (n_slots + split_len - 1) / split_len;
  if (splits < 1) splits = 1;
  *lo_out = lo;
  *hi_out = hi;
  *splits_out = splits;
  *split_len_out = split_len;
}
}  // namespace enl

int enl_attn_decode(const enl_decode_args* a, void* stream) {
  if (!a) return fail(ENL_ERR_INVALID, "enl_attn_decode: args is NULL");
  if (!a->q || !a->k_cache || !a->v_cache || !a->o)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: q, k_cache, v_cache and o must be non-NULL");
  if (a->batch < 1 || a->num_heads < 1 || a->num_kv_heads < 1)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: batch/num_heads/num_kv_heads must be >= 1");
  if (a->num_heads % a->num_kv_heads != 0)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: num_kv_heads=%d must divide num_heads=%d",
                a->num_kv_heads, a->num_heads);
  const int G = a->num_heads / a->num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(ENL_ERR_UNSUPPORTED,
                "enl_attn_decode: num_heads/num_kv_heads=%d (supported: 1, 2, 4, 8)", G);
  if (a->head_dim < 8 || a->head_dim > 128 || a->head_dim % 8 != 0)
    return fail(ENL_ERR_UNSUPPORTED,
                "enl_attn_decode: head_dim=%d (supported: multiples of 8 up to 128)",
                a->head_dim);
  const int Dk = a->head_dim <= 64 ? 64 : 128;  // kernel head dim (zero-extended)
  if (a->in_dtype != ENL_DTYPE_BF16 && a->in_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: in_dtype=%d", a->in_dtype);
  const int esz = a->in_dtype == ENL_DTYPE_FP32 ? 4 : 2;
  if (a->out_dtype != ENL_DTYPE_BF16 && a->out_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: out_dtype=%d", a->out_dtype);
  if (a->slot_begin < 0 || a->slot_end < a->slot_begin)
    return fail(ENL_ERR_INVALID, "enl_attn_decode: slot range [%d, %d) is invalid",
                a->slot_begin, a->slot_end);
  if (!aligned16(a->q) || !aligned16(a->k_cache) || !aligned16(a->v_cache))
    return fail(ENL_ERR_INVALID, "enl_attn_decode: q and caches must be 16-byte aligned");
  int st;
  if ((st = check_strides_16B("q", a->q_stride_b, 0, a->q_stride_h, esz))) return st;
  if ((st = check_strides_16B("cache", a->cache_stride_b, a->cache_stride_s, a->cache_stride_h,
                              esz)))
    return st;

  // Narrow the slot range by causality and the window, so the kernel only
  // streams what it attends.
  long long lo, hi;
  int splits, split_len;
  decode_plan(a, &lo, &hi, &splits, &split_len);
  const long long q_slot = a->q_pos - a->pos_slot0;
  if (splits > 1) {
    const size_t need = enl_decode_workspace_bytes(a->batch, a->num_heads, Dk, splits);
    if (!a->workspace || a->workspace_bytes < need)
      return fail(ENL_ERR_INVALID,
                  "enl_attn_decode: %d splits need a %zu-byte workspace (got %zu)", splits, need,
                  a->workspace_bytes);
  }

  DecodeParams p;
  p.d_real = a->head_dim;
  p.B = a->batch;
  p.H = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.in_fp32 = esz == 4;
  p.q = a->q;
  p.q_sb = a->q_stride_b;
  p.q_sh = a->q_stride_h;
  p.k = a->k_cache;
  p.v = a->v_cache;
  p.k_sb = p.v_sb = a->cache_stride_b;
  p.k_sh = p.v_sh = a->cache_stride_h;
  p.k_ss = p.v_ss = a->cache_stride_s;
  p.slot_begin = (int)lo;
  p.slot_end = (int)hi;
  p.q_minus_k0 = q_slot;
  p.alibi = a->alibi_slopes;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.n_splits = splits;
  p.split_len = split_len;
  p.o = a->o;
  p.o_sb = a->o_stride_b;
  p.o_sh = a->o_stride_h;
  p.out_fp32 = a->out_dtype == ENL_DTYPE_FP32;
  p.lse = a->lse;
  p.part_o = reinterpret_cast<float*>(a->workspace);
  p.part_lse = p.part_o ? p.part_o + (size_t)splits * a->batch * a->num_heads * Dk : nullptr;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = (Dk == 128) ? launch_decode<128>(p, s) : launch_decode<64>(p, s);
  if (e != cudaSuccess) return cuda_fail(e, "enl_attn_decode launch");
  return ENL_OK;
}

int enl_lse_merge(const float* part_o, const float* part_lse, int32_t n_parts, int32_t batch,
                  int32_t num_heads, int32_t head_dim, void* o, int64_t o_stride_b,
                  int64_t o_stride_h, int32_t out_dtype, float* lse, void* stream) {
  if (!part_o || !part_lse || !o)
    return fail(ENL_ERR_INVALID, "enl_lse_merge: part_o, part_lse and o must be non-NULL");
  if (n_parts < 1 || batch < 1 || num_heads < 1 || head_dim < 1)
    return fail(ENL_ERR_INVALID, "enl_lse_merge: sizes must be >= 1");
  if (out_dtype != ENL_DTYPE_BF16 && out_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_lse_merge: out_dtype=%d", out_dtype);
  cudaError_t e = launch_lse_merge(part_o, part_lse, n_parts, (long long)batch * num_heads * head_dim,
                                   (long long)batch * num_heads, batch, num_heads, head_dim,
                                   head_dim, o, o_stride_b, o_stride_h,
                                   out_dtype == ENL_DTYPE_FP32, lse,
                                   reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_lse_merge launch");
  return ENL_OK;
}

int enl_lse_merge_strided(const float* part_o, int64_t part_o_stride, const float* part_lse,
                          int64_t part_lse_stride, int32_t n_parts, int32_t batch,
                          int32_t num_heads, int32_t head_dim, void* o, int64_t o_stride_b,
                          int64_t o_stride_h, int32_t out_dtype, float* lse, void* stream) {
  if (!part_o || !part_lse || !o)
    return fail(ENL_ERR_INVALID, "enl_lse_merge_strided: part_o, part_lse and o must be non-NULL");
  if (n_parts < 1 || batch < 1 || num_heads < 1 || head_dim < 1)
    return fail(ENL_ERR_INVALID, "enl_lse_merge_strided: sizes must be >= 1");
  const long long bhd = (long long)batch * num_heads * head_dim, bh = (long long)batch * num_heads;
  if ((n_parts > 1 && (part_o_stride < bhd || part_lse_stride < bh)) || part_o_stride < 0 ||
      part_lse_stride < 0)
    return fail(ENL_ERR_INVALID, "enl_lse_merge_strided: part strides (%lld, %lld) overlap the "
                "parts", (long long)part_o_stride, (long long)part_lse_stride);
  if (out_dtype != ENL_DTYPE_BF16 && out_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_lse_merge_strided: out_dtype=%d", out_dtype);
  cudaError_t e = launch_lse_merge(part_o, part_lse, n_parts, part_o_stride, part_lse_stride,
                                   batch, num_heads, head_dim, head_dim, o, o_stride_b, o_stride_h,
                                   out_dtype == ENL_DTYPE_FP32, lse,
                                   reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_lse_merge_strided launch");
  return ENL_OK;
}

int enl_kv_append(void* cache, int64_t cache_stride_b, int64_t cache_stride_h,
                  int64_t cache_stride_s, const void* src, int64_t src_stride_b,
                  int64_t src_stride_t, int64_t src_stride_h, int32_t batch,
                  int32_t num_kv_heads, int32_t n_new, int32_t head_dim, int32_t dtype,
                  int64_t slot0, int64_t capacity, void* stream) {
  if (!cache || !src) return fail(ENL_ERR_INVALID, "enl_kv_append: cache and src must be non-NULL");
  if (dtype != ENL_DTYPE_BF16 && dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_kv_append: dtype=%d", dtype);
  const int eb = dtype == ENL_DTYPE_FP32 ? 4 : 2;
  if (batch < 0 || num_kv_heads < 1 || n_new < 0 || head_dim < 1)
    return fail(ENL_ERR_INVALID, "enl_kv_append: bad sizes");
  if ((head_dim * eb) % 16 != 0)
    return fail(ENL_ERR_INVALID, "enl_kv_append: head_dim * element size must be a multiple of 16");
  if (slot0 < 0 || slot0 + n_new > capacity)
    return fail(ENL_ERR_INVALID, "enl_kv_append: slots [%lld, %lld) exceed capacity %lld",
                (long long)slot0, (long long)(slot0 + n_new), (long long)capacity);
  if (!aligned16(cache) || !aligned16(src))
    return fail(ENL_ERR_INVALID, "enl_kv_append: buffers must be 16-byte aligned");
  int st;
  if ((st = check_strides_16B("cache", cache_stride_b, cache_stride_s, cache_stride_h, eb)))
    return st;
  if ((st = check_strides_16B("src", src_stride_b, src_stride_t, src_stride_h, eb))) return st;
  cudaError_t e = launch_kv_append(cache, cache_stride_b, cache_stride_h, cache_stride_s, src,
                                   src_stride_b, src_stride_t, src_stride_h, batch, num_kv_heads,
                                   n_new, head_dim, eb, slot0,
                                   reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_kv_append launch");
  return ENL_OK;
}

int enl_kv_gather(void* dst, int64_t dst_stride_b, int64_t dst_stride_h, int64_t dst_stride_s,
                  const void* src, int64_t src_stride_b, int64_t src_stride_h,
                  int64_t src_stride_s, const int64_t* index, int32_t batch_out,
                  int32_t batch_src, int32_t num_kv_heads, int32_t slot_begin, int32_t slot_end,
                  int32_t head_dim, int32_t dtype, void* stream) {
  if (!dst || !src || !index)
    return fail(ENL_ERR_INVALID, "enl_kv_gather: dst, src and index must be non-NULL");
  if (dst == src) return fail(ENL_ERR_INVALID, "enl_kv_gather: dst must not alias src");
  if (dtype != ENL_DTYPE_BF16 && dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_kv_gather: dtype=%d", dtype);
  const int eb = dtype == ENL_DTYPE_FP32 ? 4 : 2;
  if (batch_out < 0 || batch_src < 1 || num_kv_heads < 1 || slot_begin < 0 ||
      slot_end < slot_begin || (head_dim * eb) % 16 != 0)
    return fail(ENL_ERR_INVALID, "enl_kv_gather: bad sizes");
  if (!aligned16(dst) || !aligned16(src))
    return fail(ENL_ERR_INVALID, "enl_kv_gather: buffers must be 16-byte aligned");
  int st;
  if ((st = check_strides_16B("dst", dst_stride_b, dst_stride_s, dst_stride_h, eb))) return st;
  if ((st = check_strides_16B("src", src_stride_b, src_stride_s, src_stride_h, eb))) return st;
  cudaError_t e = launch_kv_gather(dst, dst_stride_b, dst_stride_h, dst_stride_s, src,
                                   src_stride_b, src_stride_h, src_stride_s,
                                   reinterpret_cast<const long long*>(index), batch_out,
                                   batch_src, num_kv_heads, slot_begin, slot_end, head_dim, eb,
                                   reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_kv_gather launch");
  return ENL_OK;
}

int enl_rope_apply(void* x, int64_t stride_b, int64_t stride_s, int64_t stride_h, int32_t batch,
                   int32_t seq, int32_t num_heads, int32_t head_dim, int32_t dtype,
                   const float* cos_table, const float* sin_table, int64_t table_row0,
                   int64_t table_rows, void* stream) {
  if (!x || !cos_table || !sin_table)
    return fail(ENL_ERR_INVALID, "enl_rope_apply: x and tables must be non-NULL");
  if (head_dim < 2 || head_dim % 2 != 0)
    return fail(ENL_ERR_INVALID, "enl_rope_apply: head_dim=%d must be even", head_dim);
  if (dtype != ENL_DTYPE_BF16 && dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_rope_apply: dtype=%d", dtype);
  if (batch < 0 || seq < 0 || num_heads < 1)
    return fail(ENL_ERR_INVALID, "enl_rope_apply: bad sizes");
  if (table_row0 < 0 || table_row0 + seq > table_rows)
    return fail(ENL_ERR_INVALID, "enl_rope_apply: table rows [%lld, %lld) exceed %lld",
                (long long)table_row0, (long long)(table_row0 + seq), (long long)table_rows);
  cudaError_t e = launch_rope(x, stride_b, stride_s, stride_h, batch, seq, num_heads, head_dim,
                              dtype == ENL_DTYPE_FP32 ? 4 : 2, cos_table, sin_table, table_row0,
                              table_rows, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_rope_apply launch");
  return ENL_OK;
}

int enl_linear_max_features(void) { return enl::linear_attn_max_features(); }

int enl_linear_planes_ok(int32_t head_dim, int32_t num_features) {
  return lin_tc_sizes(head_dim, num_features) ? 1 : 0;
}

size_t enl_linear_workspace_bytes(const enl_linear_args* a) {
  if (!a || a->batch < 1 || a->num_heads < 1 || a->num_kv_heads < 1 || a->seq < 1) return 0;
  const LinTcPlan pl = lin_tc_plan(a);
  if (pl.use) return pl.total;
  return enl::linear_workspace_bytes(a->batch, a->num_heads, a->num_kv_heads, a->seq,
                                     a->num_features, a->head_dim, a->causal);
}

}  // extern "C"

namespace {
// The feature map's kernel parameters from the ABI arguments (phi / planes
// pointers left for the caller to set).
enl::PhiParams phi_params(const enl_phi_args* a) {
  enl::PhiParams p{};
  p.x = a->x;
  p.sb = a->x_stride_b;
  p.ss = a->x_stride_s;
  p.sh = a->x_stride_h;
  p.B = a->batch;
  p.S = a->seq;
  p.H = a->num_heads;
  p.Dh = a->head_dim;
  p.in_f32 = a->in_dtype == ENL_DTYPE_FP32;
  p.kernel = a->kernel;
  p.omega = a->omega;
  p.Df = a->kernel == ENL_PHI_LINEAR ? a->head_dim : a->num_features;
  p.Dfp = (p.Df + 7) / 8 * 8;
  p.global_stab = a->kernel == ENL_PHI_PERFORMER && a->global_stab;
  p.stab_floor = a->stab_floor;
  p.stab = a->stab;
  return p;
}

bool phi_on_tensor_cores(const enl_phi_args* a) {
  return a->kernel == ENL_PHI_PERFORMER && enl::perf_tc_supported(a->head_dim, a->num_features) &&
         a->num_features >= 1 && a->num_features % 4 == 0;
}

// Planes from a map that writes fp32 only: the map goes to an fp32 phi in the
// workspace, then a split pass writes the planes.
bool phi_planes_via_fp32(const enl_phi_args* a) {
  if (!a->phi_planes || phi_on_tensor_cores(a)) return false;
  enl::PhiParams p = phi_params(a);
  p.planes = reinterpret_cast<uint16_t*>(a->phi_planes);
  return !enl::phi_planes_direct(p);
}
}  // namespace

extern "C" {

size_t enl_phi_workspace_bytes(const enl_phi_args* a) {
  if (!a || a->batch < 1 || a->seq < 1 || a->num_heads < 1) return 0;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  if (phi_on_tensor_cores(a)) {
    const size_t Dhp = (a->head_dim + 7) / 8 * 8;
    return al(2 * (size_t)a->batch * a->num_heads * a->seq * Dhp * 2) +
           al(2 * (size_t)a->num_features * Dhp * 2);
  }
  if (phi_planes_via_fp32(a)) {
    const size_t Df = a->kernel == ENL_PHI_LINEAR ? a->head_dim : a->num_features;
    return al((size_t)a->batch * a->num_heads * a->seq * Df * 4);
  }
  return 0;
}

int enl_linear_feature_map(const enl_phi_args* a, void* stream) {
  if (!a || !a->x || (!a->phi && !a->phi_planes))
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: args, x and phi (or phi_planes) must "
                "be non-NULL");
  if (a->batch < 0 || a->seq < 0 || a->num_heads < 1 || a->head_dim < 1 || a->head_dim > 1024)
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: bad sizes (batch %d, seq %d, heads %d, "
                "head_dim %d)", a->batch, a->seq, a->num_heads, a->head_dim);
  if (a->in_dtype != ENL_DTYPE_BF16 && a->in_dtype != ENL_DTYPE_FP32)
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: in_dtype=%d", a->in_dtype);
  if (a->kernel != ENL_PHI_LINEAR && a->kernel != ENL_PHI_PERFORMER)
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: kernel=%d", a->kernel);
  if (a->kernel == ENL_PHI_PERFORMER) {
    if (!a->omega || a->num_features < 1 || a->num_features > 1024)
      return fail(ENL_ERR_INVALID, "enl_linear_feature_map: performer needs omega and "
                  "1 <= num_features <= 1024 (got %d)", a->num_features);
    if (a->global_stab && !a->stab)
      return fail(ENL_ERR_INVALID, "enl_linear_feature_map: a global stabilizer needs stab");
    if (a->head_dim > enl::perf_max_head_dim())
      return fail(ENL_ERR_UNSUPPORTED, "enl_linear_feature_map: performer head_dim %d > %d",
                  a->head_dim, enl::perf_max_head_dim());
  }
  if (a->phi_planes && (reinterpret_cast<uintptr_t>(a->phi_planes) & 15u) != 0)
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: phi_planes must be 16-byte aligned");
  enl::PhiParams p = phi_params(a);
  const size_t need = enl_phi_workspace_bytes(a);
  if (need > 0 && (!a->workspace || a->workspace_bytes < need ||
                   (reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0))
    return fail(ENL_ERR_INVALID, "enl_linear_feature_map: needs a 256-byte aligned workspace of "
                "%zu bytes (enl_phi_workspace_bytes)", need);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (phi_on_tensor_cores(a)) {
    // Tensor-core Performer map: planes of x and omega, then the projections
    // on tcgen05 with the stabilizer in the epilogue, which writes fp32 phi or
    // its planes.
    if (!a->phi_planes && (reinterpret_cast<uintptr_t>(a->phi) & 15u) != 0)
      return fail(ENL_ERR_INVALID, "enl_linear_feature_map: phi must be 16-byte aligned for the "
                  "tensor-core map");
    const int Dhp = (a->head_dim + 7) / 8 * 8;
    const size_t xbytes = ((2 * (size_t)a->batch * a->num_heads * a->seq * Dhp * 2) + 255) &
                          ~size_t(255);
    enl::PerfTcParams t{};
    t.B = a->batch;
    t.S = a->seq;
    t.H = a->num_heads;
    t.Dh = a->head_dim;
    t.Dhp = Dhp;
    t.Df = a->num_features;
    t.Dfp = p.Dfp;
    t.xp = reinterpret_cast<uint16_t*>(a->workspace);
    uint16_t* wp = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(a->workspace) + xbytes);
    t.stab = a->stab;
    t.phi = a->phi_planes ? nullptr : a->phi;
    t.planes = reinterpret_cast<uint16_t*>(a->phi_planes);
    if (int st_sm = sm_count(&t.n_sm)) return st_sm;
    cudaError_t e = enl::launch_perf_prep(a->x, a->x_stride_b, a->x_stride_s, a->x_stride_h,
                                          a->in_dtype == ENL_DTYPE_FP32, a->omega, t, wp, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_linear_feature_map: prep launch");
    CUtensorMap tx, tw;
    const long long BH = (long long)t.B * t.H;
    const int Dfn = (t.Df + 15) / 16 * 16;
    int st;
    if ((st = make_3d_map(&tx, t.xp, t.Dh, t.S, 2 * BH, Dhp, (int64_t)t.S * Dhp, 128, "x")))
      return st;
    if ((st = make_3d_map(&tw, wp, t.Dh, t.Df, 2, Dhp, (int64_t)t.Df * Dhp, Dfn, "omega")))
      return st;
    e = enl::launch_perf_tc_maps(tx, tw, t, p.global_stab, a->stab_floor, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_linear_feature_map launch");
    return ENL_OK;
  }
  const bool via_fp32 = phi_planes_via_fp32(a);
  p.phi = via_fp32 ? reinterpret_cast<float*>(a->workspace) : a->phi_planes ? nullptr : a->phi;
  p.planes = via_fp32 ? nullptr : reinterpret_cast<uint16_t*>(a->phi_planes);
  cudaError_t e = enl::launch_phi(p, s);
  if (e == cudaSuccess && via_fp32)
    e = enl::launch_rows_planes(p.phi, (long long)p.B * p.H * p.S, p.Df, p.Dfp,
                                reinterpret_cast<uint16_t*>(a->phi_planes), s);
  if (e != cudaSuccess) return cuda_fail(e, "enl_linear_feature_map launch");
  return ENL_OK;
}

int enl_linear_attention(const enl_linear_args* a, void* stream) {
  if (!a || !a->v || !a->o)
    return fail(ENL_ERR_INVALID, "enl_linear_attention: args, v and o must be non-NULL");
  if ((a->phi_q_planes == nullptr) != (a->phi_k_planes == nullptr))
    return fail(ENL_ERR_INVALID, "enl_linear_attention: phi_q_planes and phi_k_planes come in "
                "pairs");
  const bool given = lin_planes_given(a);
  if (!given && (!a->phi_q || !a->phi_k))
    return fail(ENL_ERR_INVALID, "enl_linear_attention: phi_q and phi_k (or their planes) must "
                "be non-NULL");
  if (given && !lin_tc_sizes(a->head_dim, a->num_features))
    return fail(ENL_ERR_UNSUPPORTED, "enl_linear_attention: phi planes need head_dim <= 128 and "
                "num_features <= 1024 (got %d, %d)", a->head_dim, a->num_features);
  if (given && ((reinterpret_cast<uintptr_t>(a->phi_q_planes) |
                 reinterpret_cast<uintptr_t>(a->phi_k_planes)) & 15u) != 0)
    return fail(ENL_ERR_INVALID, "enl_linear_attention: phi planes must be 16-byte aligned");
  if (a->batch < 0 || a->seq < 0 || a->num_heads < 1 || a->num_kv_heads < 1 || a->head_dim < 1 ||
      a->num_features < 1)
    return fail(ENL_ERR_INVALID, "enl_linear_attention: bad sizes");
  if (a->num_heads % a->num_kv_heads != 0)
    return fail(ENL_ERR_INVALID, "enl_linear_attention: num_heads %d is not a multiple of "
                "num_kv_heads %d", a->num_heads, a->num_kv_heads);
  if (a->num_features > enl::linear_attn_max_features())
    return fail(ENL_ERR_UNSUPPORTED, "enl_linear_attention: num_features %d > %d",
                a->num_features, enl::linear_attn_max_features());
  if ((a->v_dtype != ENL_DTYPE_BF16 && a->v_dtype != ENL_DTYPE_FP32) ||
      (a->out_dtype != ENL_DTYPE_BF16 && a->out_dtype != ENL_DTYPE_FP32))
    return fail(ENL_ERR_INVALID, "enl_linear_attention: v_dtype=%d out_dtype=%d", a->v_dtype,
                a->out_dtype);
  if (!a->causal && (a->kv_in || a->ksum_in || a->kv_out || a->ksum_out))
    return fail(ENL_ERR_INVALID, "enl_linear_attention: a carried state needs causal attention");
  if ((a->kv_in == nullptr) != (a->ksum_in == nullptr) ||
      (a->kv_out == nullptr) != (a->ksum_out == nullptr))
    return fail(ENL_ERR_INVALID, "enl_linear_attention: kv and ksum come in pairs");
  enl::LinearParams p{};
  p.phi_q = a->phi_q;
  p.phi_k = a->phi_k;
  p.v = a->v;
  p.v_sb = a->v_stride_b;
  p.v_ss = a->v_stride_s;
  p.v_sh = a->v_stride_h;
  p.v_f32 = a->v_dtype == ENL_DTYPE_FP32;
  p.o = a->o;
  p.o_sb = a->o_stride_b;
  p.o_ss = a->o_stride_s;
  p.o_sh = a->o_stride_h;
  p.o_f32 = a->out_dtype == ENL_DTYPE_FP32;
  p.B = a->batch;
  p.H = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.S = a->seq;
  p.Df = a->num_features;
  p.D = a->head_dim;
  p.causal = a->causal;
  p.kv_in = a->kv_in;
  p.ks_in = a->ksum_in;
  p.state_scale = a->state_scale;
  p.kv_out = a->kv_out;
  p.ks_out = a->ksum_out;
  p.eps = a->eps;
  const size_t need = enl_linear_workspace_bytes(a);
  if (need > 0) {
    if (!a->workspace || a->workspace_bytes < need)
      return fail(ENL_ERR_INVALID, "enl_linear_attention: needs a workspace of %zu bytes "
                  "(enl_linear_workspace_bytes), got %zu", need,
                  a->workspace ? a->workspace_bytes : (size_t)0);
  }
  const LinTcPlan pl = lin_tc_plan(a);
  if (pl.use) {
    // Tensor-core path: bf16 hi/lo planes of phi(Q), phi(K) (both layouts)
    // and V' in the workspace, chunk states, their scan, chunk outputs.
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0)
      return fail(ENL_ERR_INVALID, "enl_linear_attention: workspace must be 256-byte aligned");
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
    const uint16_t* qp = given ? reinterpret_cast<const uint16_t*>(a->phi_q_planes)
                               : reinterpret_cast<const uint16_t*>(ws + pl.off_qp);
    const uint16_t* kp = given ? reinterpret_cast<const uint16_t*>(a->phi_k_planes)
                               : reinterpret_cast<const uint16_t*>(ws + pl.off_kp);
    uint16_t* vt = reinterpret_cast<uint16_t*>(ws + pl.off_vt);
    enl::LinTcParams t{};
    t.B = a->batch;
    t.H = a->num_heads;
    t.Hkv = a->num_kv_heads;
    t.S = a->seq;
    t.Df = a->num_features;
    t.D = a->head_dim;
    t.Dp = pl.Dp;
    t.Dfp = pl.Dfp;
    t.Sp = pl.Sp;
    t.n_chunks = pl.n_chunks;
    t.causal = a->causal != 0;
    t.tmem_cols = 128 + pl.Dp <= 256 ? 256 : 512;
    t.u = reinterpret_cast<float*>(ws + pl.off_u);
    t.st = reinterpret_cast<uint16_t*>(ws + pl.off_st);
    t.kv_in = a->kv_in;
    t.ks_in = a->ksum_in;
    t.state_scale = a->state_scale;
    t.kv_out = a->kv_out;
    t.ks_out = a->ksum_out;
    t.o = a->o;
    t.o_sb = a->o_stride_b;
    t.o_ss = a->o_stride_s;
    t.o_sh = a->o_stride_h;
    t.o_f32 = a->out_dtype == ENL_DTYPE_FP32;
    t.eps = a->eps;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = enl::launch_lin_prep(
        given ? nullptr : a->phi_q, given ? nullptr : a->phi_k, a->v, a->v_stride_b,
        a->v_stride_s, a->v_stride_h, a->v_dtype == ENL_DTYPE_FP32, t,
        const_cast<uint16_t*>(qp), const_cast<uint16_t*>(kp), vt, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_linear_attention: prep launch");
    const long long BHq = (long long)t.B * t.H, BHk = (long long)t.B * t.Hkv;
    CUtensorMap tq, tk, tvt, tst;
    int st;
    if ((st = make_3d_map(&tq, qp, t.Df, t.S, 2 * BHq, t.Dfp, (int64_t)t.S * t.Dfp, 128, "phi_q")))
      return st;
    if ((st = make_3d_map(&tk, kp, t.Df, t.S, 2 * BHk, t.Dfp, (int64_t)t.S * t.Dfp, 128, "phi_k")))
      return st;
    if ((st = make_3d_map(&tvt, vt, t.S, t.Dp, 2 * BHk, t.Sp, (int64_t)t.Dp * t.Sp, t.Dp, "v^T")))
      return st;
    if ((st = make_3d_map(&tst, t.st, t.Df, t.Dp, 2 * BHk * t.n_chunks, t.Dfp,
                          (int64_t)t.Dp * t.Dfp, t.Dp, "state^T")))
      return st;
    e = enl::launch_lin_tc(tq, tk, tvt, tst, t, s);
    if (e != cudaSuccess) return cuda_fail(e, "enl_linear_attention launch");
    return ENL_OK;
  }
  if (need > 0) {
    // (n_seg, B, Hkv, Df, D) partial S_kv, then (n_seg, B, Hkv, Df) partial s_k
    const size_t per_seg = (size_t)a->batch * a->num_kv_heads * a->num_features;
    const size_t n_seg = need / sizeof(float) / (per_seg * ((size_t)a->head_dim + 1));
    p.carry_kv = reinterpret_cast<float*>(a->workspace);
    p.carry_ks = p.carry_kv + n_seg * per_seg * a->head_dim;
  }
  cudaError_t e = enl::launch_linear_attn(p, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "enl_linear_attention launch");
  return ENL_OK;
}

}  // extern "C"
