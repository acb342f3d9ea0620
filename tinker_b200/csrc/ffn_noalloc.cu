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
//  * The first call in each CUDA context looks up the array's device address
//    (cudaGetSymbolAddress, with that context's device current) and caches it
//    under the context's unique ID, so a context created later on the same
//    device (after cudaDeviceReset, or a host's own non-primary context) gets
//    its own lookup; make that first call before any stream capture starts.
//  * All calls on a device share the one array, which keeps the last call's
//    contents. Nothing in it has to start at zero: the gate|up kernel writes
//    every element the down kernel then reads. Calls whose work overlaps on the
//    GPU (e.g. on two streams at once) race on the array and must be ordered by
//    the caller.
#include <cuda.h>

#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "tk_common.cuh"
#include "tk_host.h"

#define TK_FFN_NOALLOC_SCRATCH_BYTES (8u << 20)

static __device__ __align__(256) unsigned char g_ffn_scratch[TK_FFN_NOALLOC_SCRATCH_BYTES];

namespace {
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

std::mutex g_scratch_mu;
std::unordered_map<unsigned long long, void*> g_scratch_ptr;  // context ID -> address of g_ffn_scratch

// The unique ID of the calling thread's current context (0 if there is none yet or the driver
// cannot tell); IDs are never reused within a process, unlike context handles.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the scratch array in the current context.
int scratch_address(void** out) {
  using namespace tk;
  unsigned long long id = current_context_id();
  if (id) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    auto it = g_scratch_ptr.find(id);
    if (it != g_scratch_ptr.end()) {
      *out = it->second;
      return TK_OK;
    }
  }
  void* p = nullptr;  // this also makes the device's primary context current if none was
  if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_ffn_scratch), "cudaGetSymbolAddress(scratch)")) return rc;
  if (!id) id = current_context_id();
  if (id) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    g_scratch_ptr[id] = p;
  }
  *out = p;
  return TK_OK;
}
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
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  return tk_swiglu_ffn(x, x_row_stride, w_gate, w_up, w_down, scratch, out, residual, m, hidden, f, dtype, stream);
}
