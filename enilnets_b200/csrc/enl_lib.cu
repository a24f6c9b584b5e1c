// Single translation unit of libenl_b200.so: the kernels share one device
// error word, so they are compiled together rather than with relocatable
// device code.
#include "enl_abi.cu"
#include "enl_prefill.cu"
#include "enl_decode.cu"
#include "enl_kvcache.cu"
#include "enl_decode_noalloc.cu"
#include "enl_selftest.cu"
#include "enl_linear.cu"
#include "enl_linear_tc.cu"
#include "enl_sparse.cu"
#include "enl_backward.cu"
#include "enl_gemm.cu"
