// SwiGLU FFN entry point that allocates no device memory.
//
// tk_swiglu_ffn needs an [m, f] scratch buffer for the activation between the
// gate|up GEMM and the down GEMM, and takes it from the caller. Some callers
// have no way to provide one: a host application that owns all device memory
// and hands the library only its inputs and outputs (a plugin interface with a
// fixed memory budget), or a latency-critical serving loop that must not call
// cudaMalloc / cudaFree, which can synchronise the device and take
// milliseconds. tk_swiglu_ffn_noalloc keeps that scratch in a fixed array in
// the library's own device memory instead, so the call allocates nothing.
//
// Limits and behaviour:
//  * The array holds TK_FFN_NOALLOC_SCRATCH_BYTES (8 MiB): m * f * 2 bytes must
//    fit, otherwise the call returns TK_ERR_INVALID. Every GPU that loads the
//    library keeps these 8 MiB until the process exits.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture starts.
//  * All calls on a device share the one array, which keeps the last call's
//    contents. Nothing in it has to start at zero: the gate|up kernel writes
//    every element the down kernel then reads. Calls whose work overlaps on the
//    GPU (e.g. on two streams at once) race on the array and must be ordered by
//    the caller.
#include <cstdio>
#include <mutex>

#include "tk_common.cuh"
#include "tk_host.h"

#define TK_FFN_NOALLOC_SCRATCH_BYTES (8u << 20)

static __device__ __align__(256) unsigned char g_ffn_scratch[TK_FFN_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};  // per-device address of g_ffn_scratch
}  // namespace

extern "C" int tk_swiglu_ffn_noalloc(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up,
                                     const void* w_down, void* out, const void* residual, int64_t m, int64_t hidden,
                                     int64_t f, int dtype, void* stream) {
  using namespace tk;
  if (!half_dtype(dtype)) return fail_invalid("swiglu_ffn_noalloc: dtype must be F16 or BF16");
  if (m < 0 || f <= 0 || hidden <= 0) return fail_invalid("swiglu_ffn_noalloc: invalid sizes");
  const uint64_t need = static_cast<uint64_t>(m) * static_cast<uint64_t>(f) * 2u;
  if (need > TK_FFN_NOALLOC_SCRATCH_BYTES) {
    char buf[200];
    std::snprintf(buf, sizeof(buf),
                  "swiglu_ffn_noalloc: m * f * 2 = %llu bytes exceeds the fixed %u-byte scratch array; "
                  "use tk_swiglu_ffn with a caller-provided buffer",
                  static_cast<unsigned long long>(need), TK_FFN_NOALLOC_SCRATCH_BYTES);
    return fail_invalid(buf);
  }
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_UNSUPPORTED, "swiglu_ffn_noalloc: device index out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_ffn_scratch), "cudaGetSymbolAddress(scratch)")) return rc;
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  return tk_swiglu_ffn(x, x_row_stride, w_gate, w_up, w_down, scratch, out, residual, m, hidden, f, dtype, stream);
}
