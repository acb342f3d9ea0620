// Host-side helpers shared by the entry points: per-thread error messages,
// argument checks, device properties, and TMA tensor-map encoding with a cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/tinker_b200.h"

namespace tk {

// Record `msg` as this thread's last error and return `code`.
int set_error(int code, const std::string& msg);
inline int fail_invalid(const std::string& msg) { return set_error(TK_ERR_INVALID, msg); }

// Check a CUDA runtime status; on failure records it and returns TK_ERR_CUDA.
int check_cuda(cudaError_t e, const char* what);

// Launch-error check after a <<<>>> launch.
inline int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  size_t smem_optin = 0;
};
// Properties of the current device (cached per device).
int current_device_info(DeviceInfo* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline int elem_size(int dt) { return dt == TK_F32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == TK_F16 || dt == TK_BF16 || dt == TK_F32; }
inline bool half_dtype(int dt) { return dt == TK_F16 || dt == TK_BF16; }

// Programmatic dependent launch on (default) or off (TINKER_B200_PDL=0 in the environment).
bool pdl_enabled();

// Launch `kern` with cudaLaunchKernelEx: programmatic stream serialisation when
// PDL is enabled (the kernel overlaps its set-up with the previous kernel and
// orders its dependent reads with griddepcontrol.wait), and a cluster of
// `cluster_x` CTAs along x when cluster_x > 1.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
                  const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}

// 2-D tensor map over a row-major [rows, cols] matrix of 2-byte elements
// (row stride in elements), box [box_rows, box_cols], 128-byte swizzle.
// Cached by all of its arguments, so repeated calls with the same buffer are cheap.
int tensor_map_2d(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols,
                  uint64_t row_stride, uint32_t box_rows, uint32_t box_cols);

// 3-D tensor map over [d2, d1, d0] (d0 contiguous) with strides s1, s2 in
// elements, box [b2, b1, b0], 128-byte swizzle.
int tensor_map_3d(CUtensorMap* out, const void* base, int dtype, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2);

// Byte ranges a kernel pulls into L2 for the kernels launched after it (the weights of the
// next projections of a decoder block), so that their weight streams start from L2 instead of
// HBM: the launch chain leaves HBM mostly idle, and these ranges never depend on the previous
// kernel (a later write still lands in L2, the point of coherence), so every CTA issues its
// share at its start. The host rounds each range inward to 16-byte boundaries.
constexpr int L2_PF_MAX = 8;
struct L2Prefetch {
  const char* base[L2_PF_MAX];
  int64_t bytes[L2_PF_MAX];
  int n;
};

// The ranges of a tk_epilogue (NULL pointer or size <= 0: unused slot), each rounded inward
// to 16-byte boundaries; ranges left empty are dropped.
inline void l2_prefetch_from(const void* const* ptrs, const int64_t* bytes, L2Prefetch* out) {
  *out = L2Prefetch{};
  for (int i = 0; i < L2_PF_MAX; ++i) {
    if (!ptrs[i] || bytes[i] <= 0) continue;
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(ptrs[i]) + 15) & ~uintptr_t(15);
    const uintptr_t hi = (reinterpret_cast<uintptr_t>(ptrs[i]) + static_cast<uintptr_t>(bytes[i])) & ~uintptr_t(15);
    if (hi <= lo) continue;
    out->base[out->n] = reinterpret_cast<const char*>(lo);
    out->bytes[out->n] = static_cast<int64_t>(hi - lo);
    ++out->n;
  }
}

// Weight-streaming products for 1..MAX_M rows (gemv.cu): y = x W^T over up to three weight
// blocks stacked along n (nrows[i] rows each, w[i] null when absent), with the GEMM epilogue
// options, or SwiGLU of gate w[0] and up w[1] (n output columns). Used by the GEMM entry points
// for small M.
namespace gemv {
constexpr int MAX_M = 8;
int run(int dtype, const void* x, int64_t lda, const void* const w[3], const int64_t nrows[3], bool swiglu, void* y,
        int64_t ldy, int64_t m, int64_t n, int64_t k, const void* residual, const float* ssq_in, int ssq_parts,
        float ssq_inv_k, float ssq_eps, float* ssq_out, cudaStream_t st);
}  // namespace gemv

}  // namespace tk
