// enl_attn_decode_noalloc: the split-KV decode for callers that cannot
// allocate device memory.
//
// Some hosts cannot hand this library a workspace: an inference server or
// plugin host that owns every byte of device memory through its own pool and
// gives plugins no allocation hook, or a latency-critical token loop where a
// cudaMalloc (which may synchronise the whole device) is not allowed. For
// them the split partials live in a fixed scratch array compiled into the
// library instead of in caller memory.
//
// Limits and sharing rules:
//   * The scratch holds at most ENL_DECODE_NOALLOC_SCRATCH_BYTES (4 MiB).
//     A request whose split partials (n_splits * batch * heads * (head_dim+1)
//     floats, for the split count the decode really runs with after the slot
//     range is narrowed by causality and the window) would not fit is
//     rejected with ENL_ERR_INVALID.
//   * Every GPU that loads the library keeps its own copy of the array until
//     the process exits.
//   * All calls on a device share that one array and it keeps whatever the
//     last call wrote. Nothing in it needs to start at zero: each split writes
//     its partial in full before the merge reads it. Two calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race
//     on the array and corrupt each other's results; order them on one stream.
//   * The first call on a device looks up the array's device address (one
//     cudaGetSymbolAddress, with that device current). Make that first call
//     before any stream capture.
//   * The address belongs to the CUDA context current at that first call.
//     A call from a different context looks it up again, but a
//     cudaDeviceReset destroys the context and a new one may reuse its
//     handle, so keep the first call's context alive for as long as this
//     entry point is used (do not reset the device in between).
#include <mutex>

#include "enl_attn.h"
#include "enl_common.cuh"

namespace enl {
namespace {

constexpr size_t kNoallocScratchBytes = ENL_DECODE_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch itself. Host code must never use this name as a device
// address: on the host it is only a stand-in symbol.
static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchBytes / sizeof(float)];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};  // context the address was looked up in

// The driver's cuCtxGetCurrent, through the runtime's entry-point query (the
// library does not link libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn;
}

// Device address of the scratch on the current device: looked up once per
// device, again only when the calling context differs from the one it was
// looked up in.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "enl_attn_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(ENL_ERR_UNSUPPORTED, "enl_attn_decode_noalloc: device %d >= %d", dev,
                kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  CUcontext ctx = nullptr;
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (get_ctx && g_noalloc_ptr[dev]) get_ctx(&ctx);
  if (!g_noalloc_ptr[dev] || (get_ctx && ctx != g_noalloc_ctx[dev])) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also makes the context current
    if (e != cudaSuccess)
      return cuda_fail(e, "enl_attn_decode_noalloc: cudaGetSymbolAddress(scratch)");
    if (get_ctx) get_ctx(&ctx);
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return ENL_OK;
}

}  // namespace
}  // namespace enl

extern "C" int enl_attn_decode_noalloc(const enl_decode_args* a, void* stream) {
  using namespace enl;
  if (!a) return fail(ENL_ERR_INVALID, "enl_attn_decode_noalloc: args is NULL");
  // Sizes first, so a bad size is reported as itself rather than as an
  // oversized scratch request; enl_attn_decode checks everything else.
  if (a->batch < 1 || a->num_heads < 1 || a->num_kv_heads < 1 || a->head_dim < 1)
    return fail(ENL_ERR_INVALID,
                "enl_attn_decode_noalloc: batch/num_heads/num_kv_heads/head_dim must be >= 1");
  if (a->slot_begin < 0 || a->slot_end < a->slot_begin)
    return fail(ENL_ERR_INVALID, "enl_attn_decode_noalloc: slot range [%d, %d) is invalid",
                a->slot_begin, a->slot_end);
  // The split partials of the split count the decode will run with.
  long long lo, hi;
  int splits, split_len;
  decode_plan(a, &lo, &hi, &splits, &split_len);
  const size_t need = enl_decode_workspace_bytes(a->batch, a->num_heads, a->head_dim, splits);
  if (need > kNoallocScratchBytes)
    return fail(ENL_ERR_INVALID,
                "enl_attn_decode_noalloc: batch=%d num_heads=%d head_dim=%d with %d splits "
                "needs %zu bytes of scratch, more than the %zu bytes this entry point holds; "
                "pass fewer n_splits or call enl_attn_decode with your own workspace",
                a->batch, a->num_heads, a->head_dim, splits, need,
                (size_t)kNoallocScratchBytes);
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != ENL_OK) return st;
  enl_decode_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kNoallocScratchBytes;
  return enl_attn_decode(&b, stream);
}
