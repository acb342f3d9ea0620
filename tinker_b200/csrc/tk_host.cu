// Host runtime of the library: error reporting, device queries, tensor maps,
// and the small entry points (version, device check, device error word).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "tk_common.cuh"
#include "tk_host.h"

__device__ int g_tk_device_error = 0;

namespace tk {

static thread_local std::string t_last_error;

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TK_OK;
  return set_error(TK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TINKER_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int current_device_info(DeviceInfo* out) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].device != dev) {
    DeviceInfo d;
    d.device = dev;
    if (int rc = check_cuda(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev),
                            "cudaDeviceGetAttribute"))
      return rc;
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.smem_optin = static_cast<size_t>(optin);
    cache[dev] = d;
  }
  *out = cache[dev];
  return TK_OK;
}

// ---- tensor maps ----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  uint64_t v[12];
  bool operator==(const MapKey& o) const { return std::memcmp(v, o.v, sizeof(v)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t x : k.v) h = (h ^ x) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

static std::mutex g_map_mu;
static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

static int encode(CUtensorMap* out, const MapKey& key, const void* base, int dtype, cuuint32_t rank,
                  const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return TK_OK;
    }
  }
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(TK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMapDataType t = dtype == TK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, t, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d) for rank %u base %p", int(r),
                  unsigned(rank), base);
    return set_error(TK_ERR_INVALID, buf);
  }
  std::lock_guard<std::mutex> lock(g_map_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, *out);
  return TK_OK;
}

int tensor_map_2d(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols,
                  uint64_t row_stride, uint32_t box_rows, uint32_t box_cols) {
  if (!aligned16(base)) return fail_invalid("TMA base address must be 16-byte aligned");
  if ((row_stride * 2) % 16 != 0) return fail_invalid("row stride must be a multiple of 8 elements");
  MapKey key{{reinterpret_cast<uint64_t>(base), uint64_t(dtype), rows, cols, row_stride, box_rows, box_cols, 2,
              0, 0, 0, 0}};
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  return encode(out, key, base, dtype, 2, dims, strides, box);
}

int tensor_map_3d(CUtensorMap* out, const void* base, int dtype, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
  if (!aligned16(base)) return fail_invalid("TMA base address must be 16-byte aligned");
  if ((s1 * 2) % 16 != 0 || (s2 * 2) % 16 != 0) return fail_invalid("strides must be multiples of 8 elements");
  MapKey key{{reinterpret_cast<uint64_t>(base), uint64_t(dtype), d0, d1, d2, s1, s2, b0, b1, b2, 3, 0}};
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1 * 2, s2 * 2};
  cuuint32_t box[3] = {b0, b1, b2};
  return encode(out, key, base, dtype, 3, dims, strides, box);
}

}  // namespace tk

// ---- small entry points ------------------------------------------------------------
extern "C" int tk_version(void) { return 100; }

extern "C" const char* tk_last_error(void) { return tk::t_last_error.c_str(); }

extern "C" int tk_check_device(int device) {
  int major = 0, minor = 0;
  if (int rc = tk::check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device),
                              "cudaDeviceGetAttribute"))
    return rc;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "device %d is sm_%d%d; this library is built for sm_100a only", device, major,
                  minor);
    return tk::set_error(TK_ERR_UNSUPPORTED, buf);
  }
  return TK_OK;
}

extern "C" int tk_device_error(int* code, int clear) {
  if (!code) return tk::fail_invalid("code must not be NULL");
  if (int rc = tk::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize")) return rc;
  if (int rc = tk::check_cuda(cudaMemcpyFromSymbol(code, g_tk_device_error, sizeof(int)), "read error word"))
    return rc;
  if (clear) {
    int zero = 0;
    if (int rc = tk::check_cuda(cudaMemcpyToSymbol(g_tk_device_error, &zero, sizeof(int)), "clear error word"))
      return rc;
  }
  return TK_OK;
}
