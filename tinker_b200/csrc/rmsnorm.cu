// Single-pass RMSNorm (optionally fused with the residual add) and the SwiGLU
// activation: HBM-bound kernels built on 16-byte vector loads and stores.
//
// RMSNorm: each row is read exactly once. A row is split over TPR threads; each
// thread keeps its NV 16-byte vectors in registers, so the statistics pass and
// the scaling pass share one HBM read (the reference's Triton kernel reads X
// twice, tinker/kernels/fused_rmsnorm.py:37-52). The sum of squares is reduced
// with warp shuffles and, for rows wider than one warp, through shared memory.
#include <algorithm>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace {

// 16-byte vector of the row dtype, converted to/from float.
template <int DT> struct Vec;
template <> struct Vec<TK_F32> {
  static constexpr int N = 4;
  __device__ static void to_f(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ static uint4 from_f(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <int DT> struct VecHalf {
  static constexpr int N = 8;
  using D = Dt<DT>;
  __device__ static void to_f(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      typename D::T2 h = *reinterpret_cast<const typename D::T2*>(&w[i]);
      float2 p = D::unpack(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ static uint4 from_f(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      typename D::T2 h = D::pack(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Vec<TK_F16> : VecHalf<TK_F16> {};
template <> struct Vec<TK_BF16> : VecHalf<TK_BF16> {};

// Round a float through the row dtype (the residual stream is stored in that dtype).
template <int DT> __device__ __forceinline__ float round_dt(float v);
template <> __device__ __forceinline__ float round_dt<TK_F32>(float v) { return v; }
template <> __device__ __forceinline__ float round_dt<TK_F16>(float v) { return __half2float(__float2half_rn(v)); }
template <> __device__ __forceinline__ float round_dt<TK_BF16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// WV: the weight has the row dtype and a 16-byte aligned base, so each thread loads its weight
// vectors with the same 16-byte loads as the row, issued together with them (before the
// reduction, off its critical path); otherwise the weights are read element by element after it.
template <int DT, int NV, int TPR, bool ADD, bool WV>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const void* __restrict__ x, int64_t xs,
                                                           const void* __restrict__ res, const void* __restrict__ w,
                                                           int wdt, void* y, int64_t ys, void* res_out,
                                                           int64_t rows, int dim, float eps) {
  using V = Vec<DT>;
  constexpr int E = V::N;
  constexpr int WARPS = TPR / 32;
  __shared__ float red[256 / 32];
  pdl_launch_dependents();
  pdl_wait();  // x (and the residual) are written by earlier kernels
  const int t = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const int nvec = dim / E;

  float v[NV][E];
  uint4 wr[WV ? NV : 1];
  float ss = 0.f;
  if constexpr (WV) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = t + i * TPR;
      if (active && c < nvec) wr[i] = reinterpret_cast<const uint4*>(w)[c];
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = t + i * TPR;
    if (active && c < nvec) {
      uint4 u = reinterpret_cast<const uint4*>(static_cast<const char*>(x) + (row * xs) * (DT == TK_F32 ? 4 : 2))[c];
      V::to_f(u, v[i]);
      if constexpr (ADD) {
        uint4 r = reinterpret_cast<const uint4*>(static_cast<const char*>(res) + (row * xs) * (DT == TK_F32 ? 4 : 2))[c];
        float rf[E];
        V::to_f(r, rf);
#pragma unroll
        for (int e = 0; e < E; ++e) v[i][e] = round_dt<DT>(v[i][e] + rf[e]);
        reinterpret_cast<uint4*>(static_cast<char*>(res_out) + (row * xs) * (DT == TK_F32 ? 4 : 2))[c] = V::from_f(v[i]);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if constexpr (WARPS > 1) {
    // a row spans WARPS warps; blockDim.y rows share the block, each with its own slots
    if ((t & 31) == 0) red[threadIdx.y * WARPS + (t >> 5)] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < WARPS; ++i) ss += red[threadIdx.y * WARPS + i];
  }
  const float rrms = rsqrtf(ss / static_cast<float>(dim) + eps);
  if (!active) return;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = t + i * TPR;
    if (c < nvec) {
      float o[E], wf[E];
      if constexpr (WV) {
        V::to_f(wr[i], wf);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) wf[e] = load_as_f32(w, static_cast<int64_t>(c) * E + e, wdt);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = v[i][e] * rrms * wf[e];
      reinterpret_cast<uint4*>(static_cast<char*>(y) + (row * ys) * (DT == TK_F32 ? 4 : 2))[c] = V::from_f(o);
    }
  }
}

// Generic path for any dim / alignment: one block per row, two passes over the row.
template <int DT, bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const void* __restrict__ x, int64_t xs,
                                                              const void* __restrict__ res, const void* __restrict__ w,
                                                              int wdt, void* y, int64_t ys, void* res_out,
                                                              int64_t rows, int dim, float eps) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  float ss = 0.f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float a = load_as_f32(x, row * xs + c, DT);
    if constexpr (ADD) {
      a = round_dt<DT>(a + load_as_f32(res, row * xs + c, DT));
      if (DT == TK_F32) reinterpret_cast<float*>(res_out)[row * xs + c] = a;
      else if (DT == TK_F16) reinterpret_cast<__half*>(res_out)[row * xs + c] = __float2half_rn(a);
      else reinterpret_cast<__nv_bfloat16*>(res_out)[row * xs + c] = __float2bfloat16_rn(a);
    }
    ss = fmaf(a, a, ss);
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) ss += red[i];
  const float rrms = rsqrtf(ss / static_cast<float>(dim) + eps);
  // ADD: the rounded sum was written by this same thread above, so re-reading it is safe
  const void* src = ADD ? res_out : x;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    const float o = load_as_f32(src, row * xs + c, DT) * rrms * load_as_f32(w, c, wdt);
    if (DT == TK_F32) reinterpret_cast<float*>(y)[row * ys + c] = o;
    else if (DT == TK_F16) reinterpret_cast<__half*>(y)[row * ys + c] = __float2half_rn(o);
    else reinterpret_cast<__nv_bfloat16*>(y)[row * ys + c] = __float2bfloat16_rn(o);
  }
}

template <int DT, bool ADD>
int launch_rmsnorm(const void* x, int64_t xs, const void* res, const void* w, int wdt, void* y, int64_t ys,
                   void* res_out, int64_t rows, int64_t dim, float eps, cudaStream_t st) {
  constexpr int E = DT == TK_F32 ? 4 : 8;
  const int es = DT == TK_F32 ? 4 : 2;
  const bool vec_ok = dim % E == 0 && (xs * es) % 16 == 0 && (ys * es) % 16 == 0 && aligned16(x) && aligned16(y) &&
                      (!ADD || (aligned16(res) && aligned16(res_out)));
  const int64_t nvec = dim / E;
  const bool wv = wdt == DT && aligned16(w);
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (vec_ok && nvec <= 2048) {
#define TK_RMS_LAUNCH(NV, TPR)                                                                                 \
  {                                                                                                            \
    dim3 block(TPR, TPR >= 128 ? 1 : 128 / TPR);                                                               \
    dim3 grid(static_cast<unsigned>((rows + block.y - 1) / block.y));                                          \
    if (wv)                                                                                                    \
      return launch_kernel(rmsnorm_vec_kernel<DT, NV, TPR, ADD, true>, grid, block, 0, st, 1,                  \
                           "rmsnorm_vec_kernel", x, xs, res, w, wdt, y, ys, res_out, rows, static_cast<int>(dim), \
                           eps);                                                                               \
    return launch_kernel(rmsnorm_vec_kernel<DT, NV, TPR, ADD, false>, grid, block, 0, st, 1, "rmsnorm_vec_kernel", \
                         x, xs, res, w, wdt, y, ys, res_out, rows, static_cast<int>(dim), eps);                \
  }
    if (rows < 4 * static_cast<int64_t>(dev.sm_count)) {
      // few rows: one row per block and one vector per thread, to spread a small
      // problem over as many SMs (and as many loads in flight) as possible
      if (nvec <= 64) TK_RMS_LAUNCH(1, 64)
      if (nvec <= 128) TK_RMS_LAUNCH(1, 128)
      if (nvec <= 256) TK_RMS_LAUNCH(1, 256)
      if (nvec <= 512) TK_RMS_LAUNCH(2, 256)
    }
    if (nvec <= 32) TK_RMS_LAUNCH(1, 32)
    if (nvec <= 64) TK_RMS_LAUNCH(2, 32)
    if (nvec <= 128) TK_RMS_LAUNCH(4, 32)
    if (nvec <= 256) TK_RMS_LAUNCH(4, 64)
    if (nvec <= 512) TK_RMS_LAUNCH(4, 128)
    if (nvec <= 1024) TK_RMS_LAUNCH(4, 256)
    TK_RMS_LAUNCH(8, 256)
#undef TK_RMS_LAUNCH
  }
  return launch_kernel(rmsnorm_scalar_kernel<DT, ADD>, dim3(static_cast<unsigned>(rows)), dim3(256), 0, st, 1,
                       "rmsnorm_scalar_kernel", x, xs, res, w, wdt, y, ys, res_out, rows, static_cast<int>(dim), eps);
}

template <bool ADD>
int rmsnorm_dispatch(const void* x, int64_t xs, const void* res, const void* w, int wdt, void* y, int64_t ys,
                     void* res_out, int64_t rows, int64_t dim, float eps, int dtype, void* stream) {
  if (!valid_dtype(dtype) || !valid_dtype(wdt)) return fail_invalid("rmsnorm: dtype must be F16, BF16 or F32");
  if (rows < 0 || dim <= 0 || dim > (1 << 24)) return fail_invalid("rmsnorm: invalid rows/dim");
  if (xs < dim || ys < dim) return fail_invalid("rmsnorm: row stride smaller than dim");
  if (!(eps >= 0.f)) return fail_invalid("rmsnorm: eps must be >= 0");
  if (rows == 0) return TK_OK;  // empty tensors may carry NULL data pointers
  if (!x || !w || !y || (ADD && (!res || !res_out))) return fail_invalid("rmsnorm: NULL pointer");
  if (rows > 0x7fffffffLL) return fail_invalid("rmsnorm: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case TK_F16: return launch_rmsnorm<TK_F16, ADD>(x, xs, res, w, wdt, y, ys, res_out, rows, dim, eps, st);
    case TK_BF16: return launch_rmsnorm<TK_BF16, ADD>(x, xs, res, w, wdt, y, ys, res_out, rows, dim, eps, st);
    default: return launch_rmsnorm<TK_F32, ADD>(x, xs, res, w, wdt, y, ys, res_out, rows, dim, eps, st);
  }
}

// ---- SwiGLU activation ---------------------------------------------------------
// silu(a) * b in fp32. For 16-bit rows (one rounding to 11 or 8 significant bits follows) the fast
// exponential and division intrinsics are used; fp32 rows keep expf and the IEEE division.
template <int DT>
__device__ __forceinline__ float silu_mul(float a, float b) {
  if constexpr (DT == TK_F32) return a / (1.0f + expf(-a)) * b;
  else return __fdividef(a, 1.0f + __expf(-a)) * b;
}

template <int DT>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const void* __restrict__ g, int64_t gs,
                                                          const void* __restrict__ u, int64_t us, void* o, int64_t os,
                                                          int64_t rows, int64_t vpr) {
  using V = Vec<DT>;
  constexpr int E = V::N;
  constexpr int ES = DT == TK_F32 ? 4 : 2;
  const int64_t total = rows * vpr;
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vpr, c = i - r * vpr;
    float a[E], b[E], out[E];
    V::to_f(reinterpret_cast<const uint4*>(static_cast<const char*>(g) + r * gs * ES)[c], a);
    V::to_f(reinterpret_cast<const uint4*>(static_cast<const char*>(u) + r * us * ES)[c], b);
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = silu_mul<DT>(a[e], b[e]);
    reinterpret_cast<uint4*>(static_cast<char*>(o) + r * os * ES)[c] = V::from_f(out);
  }
}

// Contiguous gate, up and output: a flat array of 16-byte vectors. Each thread loads U vectors of
// each input (a block covers 256 x U consecutive vectors, coalesced per step) before it computes,
// so 2U loads are in flight per thread; no index division.
template <int DT, int U>
__global__ void __launch_bounds__(256) swiglu_flat_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u,
                                                           uint4* __restrict__ o, int64_t total) {
  using V = Vec<DT>;
  constexpr int E = V::N;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (256 * U) + threadIdx.x;
  uint4 ga[U], ua[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + k * 256;
    if (i < total) {
      ga[k] = g[i];
      ua[k] = u[i];
    }
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + k * 256;
    if (i < total) {
      float a[E], b[E], out[E];
      V::to_f(ga[k], a);
      V::to_f(ua[k], b);
#pragma unroll
      for (int e = 0; e < E; ++e) out[e] = silu_mul<DT>(a[e], b[e]);
      o[i] = V::from_f(out);
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(256) swiglu_scalar_kernel(const void* __restrict__ g, int64_t gs,
                                                             const void* __restrict__ u, int64_t us, void* o,
                                                             int64_t os, int64_t rows, int64_t n) {
  const int64_t total = rows * n;
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    const float a = load_as_f32(g, r * gs + c, DT), b = load_as_f32(u, r * us + c, DT);
    const float out = silu_mul<DT>(a, b);
    if (DT == TK_F32) reinterpret_cast<float*>(o)[r * os + c] = out;
    else if (DT == TK_F16) reinterpret_cast<__half*>(o)[r * os + c] = __float2half_rn(out);
    else reinterpret_cast<__nv_bfloat16*>(o)[r * os + c] = __float2bfloat16_rn(out);
  }
}

template <int DT>
int launch_swiglu(const void* g, int64_t gs, const void* u, int64_t us, void* o, int64_t os, int64_t rows,
                  int64_t n, cudaStream_t st) {
  constexpr int E = DT == TK_F32 ? 4 : 8;
  const int es = DT == TK_F32 ? 4 : 2;
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * 8;
  const bool vec_ok = n % E == 0 && (gs * es) % 16 == 0 && (us * es) % 16 == 0 && (os * es) % 16 == 0 &&
                      aligned16(g) && aligned16(u) && aligned16(o);
  if (vec_ok && gs == n && us == n && os == n) {
    // four vectors per thread once that still leaves at least four blocks per SM; smaller problems
    // take one vector per thread, to spread over more SMs
    const int64_t total = rows * (n / E);
    const int64_t blocks4 = (total + 256 * 4 - 1) / (256 * 4);
    if (blocks4 > 0x7fffffffLL) return fail_invalid("swiglu: too many elements");
    if (blocks4 >= 4 * static_cast<int64_t>(dev.sm_count))
      return launch_kernel(swiglu_flat_kernel<DT, 4>, dim3(static_cast<unsigned>(blocks4)), dim3(256), 0, st, 1,
                           "swiglu_flat_kernel", static_cast<const uint4*>(g), static_cast<const uint4*>(u),
                           static_cast<uint4*>(o), total);
    return launch_kernel(swiglu_flat_kernel<DT, 1>, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0,
                         st, 1, "swiglu_flat_kernel", static_cast<const uint4*>(g), static_cast<const uint4*>(u),
                         static_cast<uint4*>(o), total);
  }
  if (vec_ok) {
    const int64_t total = rows * (n / E);
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(cap, (total + 255) / 256)));
    return launch_kernel(swiglu_vec_kernel<DT>, dim3(grid), dim3(256), 0, st, 1, "swiglu_vec_kernel", g, gs, u, us,
                         o, os, rows, n / E);
  }
  const int64_t total = rows * n;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(cap, (total + 255) / 256)));
  return launch_kernel(swiglu_scalar_kernel<DT>, dim3(grid), dim3(256), 0, st, 1, "swiglu_scalar_kernel", g, gs, u,
                       us, o, os, rows, n);
}

// parts[(c / 32) * m + r] = sum of x[r, c .. c+31]^2: one thread per (row, 32-column chunk),
// chunks of a row on consecutive threads (the 64-byte loads of a warp are contiguous).
template <int DT>
__global__ void __launch_bounds__(256) row_sumsq_kernel(const void* __restrict__ x, int64_t xs, int64_t m,
                                                         int chunks, float* __restrict__ parts) {
  pdl_launch_dependents();
  pdl_wait();  // x is written by an earlier kernel
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= m * chunks) return;
  const int64_t r = t / chunks;
  const int c = static_cast<int>(t - r * chunks);
  using V = Vec<DT>;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + r * xs + c * 32);
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < 32 / V::N; ++q) {
    float f[V::N];
    V::to_f(src[q], f);
#pragma unroll
    for (int i = 0; i < V::N; ++i) ss = fmaf(f[i], f[i], ss);
  }
  parts[static_cast<int64_t>(c) * m + r] = ss;
}

// out[r, c .. c+31] = table[tokens[r], c .. c+31] and parts[(c / 32) * m + r] = the chunk's sum of
// squares: a model's embedding gather together with the row statistics its first folded RMSNorm
// reads, one thread per (row, 32-column chunk), the 64-byte copies of a warp contiguous. A token
// outside [0, vocab) records TK_DEVERR_TOKEN and gives a zero row.
template <int DT>
__global__ void __launch_bounds__(256) embedding_rows_kernel(const int64_t* __restrict__ tokens,
                                                              const void* __restrict__ table, int64_t vocab,
                                                              int64_t hidden, void* __restrict__ out, int64_t m,
                                                              int chunks, float* __restrict__ parts) {
  pdl_launch_dependents();
  pdl_wait();  // the token ids may be written by an earlier kernel
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= m * chunks) return;
  const int64_t r = t / chunks;
  const int c = static_cast<int>(t - r * chunks);
  using V = Vec<DT>;
  const int64_t tok = __ldg(tokens + r);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + r * hidden + c * 32);
  float ss = 0.f;
  if (tok < 0 || tok >= vocab) {
    if (c == 0) record_device_error(TK_DEVERR_TOKEN);
#pragma unroll
    for (int q = 0; q < 32 / V::N; ++q) dst[q] = make_uint4(0, 0, 0, 0);
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(table) + tok * hidden + c * 32);
#pragma unroll
    for (int q = 0; q < 32 / V::N; ++q) {
      const uint4 u = __ldg(src + q);
      dst[q] = u;
      float f[V::N];
      V::to_f(u, f);
#pragma unroll
      for (int i = 0; i < V::N; ++i) ss = fmaf(f[i], f[i], ss);
    }
  }
  if (parts) parts[static_cast<int64_t>(c) * m + r] = ss;
}

}  // namespace
}  // namespace tk

extern "C" int tk_embedding_rows(const int64_t* tokens, const void* table, int64_t vocab, int64_t hidden, void* out,
                                 float* row_ssq_out, int64_t rows, int dtype, void* stream) {
  using namespace tk;
  if (!half_dtype(dtype)) return fail_invalid("embedding_rows: dtype must be F16 or BF16");
  if (rows < 0 || vocab <= 0 || hidden <= 0 || hidden % 32 != 0)
    return fail_invalid("embedding_rows: hidden must be a positive multiple of 32");
  if (rows == 0) return TK_OK;
  if (!tokens || !table || !out || !aligned16(table) || !aligned16(out))
    return fail_invalid("embedding_rows: NULL or unaligned pointer");
  const int chunks = static_cast<int>(hidden / 32);
  const int64_t threads = rows * chunks;
  const dim3 grid(static_cast<unsigned>((threads + 255) / 256)), block(256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return launch_kernel(embedding_rows_kernel<TK_F16>, grid, block, 0, st, 1, "embedding_rows_kernel", tokens, table,
                         vocab, hidden, out, rows, chunks, row_ssq_out);
  return launch_kernel(embedding_rows_kernel<TK_BF16>, grid, block, 0, st, 1, "embedding_rows_kernel", tokens, table,
                       vocab, hidden, out, rows, chunks, row_ssq_out);
}

extern "C" int tk_row_sumsq(const void* x, int64_t x_row_stride, int64_t m, int64_t k, float* parts, int dtype,
                            void* stream) {
  using namespace tk;
  if (!half_dtype(dtype)) return fail_invalid("row_sumsq: dtype must be F16 or BF16");
  if (m < 0 || k <= 0 || k % 32 != 0 || x_row_stride < k || x_row_stride % 8 != 0)
    return fail_invalid("row_sumsq: k must be a positive multiple of 32 and the row stride >= k, a multiple of 8");
  if (m == 0) return TK_OK;
  if (!x || !parts || !aligned16(x)) return fail_invalid("row_sumsq: NULL or unaligned pointer");
  const int chunks = static_cast<int>(k / 32);
  const int64_t threads = m * chunks;
  const dim3 grid(static_cast<unsigned>((threads + 255) / 256)), block(256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return launch_kernel(row_sumsq_kernel<TK_F16>, grid, block, 0, st, 1, "row_sumsq_kernel", x, x_row_stride, m,
                         chunks, parts);
  return launch_kernel(row_sumsq_kernel<TK_BF16>, grid, block, 0, st, 1, "row_sumsq_kernel", x, x_row_stride, m,
                       chunks, parts);
}

extern "C" int tk_rmsnorm(const void* x, int64_t x_row_stride, const void* weight, int w_dtype, void* y,
                          int64_t y_row_stride, int64_t rows, int64_t dim, float eps, int dtype, void* stream) {
  return tk::rmsnorm_dispatch<false>(x, x_row_stride, nullptr, weight, w_dtype, y, y_row_stride, nullptr, rows, dim,
                                     eps, dtype, stream);
}

extern "C" int tk_add_rmsnorm(const void* x, const void* residual, const void* weight, int w_dtype, void* y,
                              void* residual_out, int64_t rows, int64_t dim, float eps, int dtype, void* stream) {
  return tk::rmsnorm_dispatch<true>(x, dim, residual, weight, w_dtype, y, dim, residual_out, rows, dim, eps, dtype,
                                    stream);
}

extern "C" int tk_swiglu(const void* gate, int64_t gate_row_stride, const void* up, int64_t up_row_stride, void* out,
                         int64_t out_row_stride, int64_t rows, int64_t n, int dtype, void* stream) {
  using namespace tk;
  if (!valid_dtype(dtype)) return fail_invalid("swiglu: dtype must be F16, BF16 or F32");
  if (rows < 0 || n < 0) return fail_invalid("swiglu: negative size");
  if (gate_row_stride < n || up_row_stride < n || out_row_stride < n)
    return fail_invalid("swiglu: row stride smaller than n");
  if (rows == 0 || n == 0) return TK_OK;  // empty tensors may carry NULL data pointers
  if (!gate || !up || !out) return fail_invalid("swiglu: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case TK_F16: return launch_swiglu<TK_F16>(gate, gate_row_stride, up, up_row_stride, out, out_row_stride, rows, n, st);
    case TK_BF16: return launch_swiglu<TK_BF16>(gate, gate_row_stride, up, up_row_stride, out, out_row_stride, rows, n, st);
    default: return launch_swiglu<TK_F32>(gate, gate_row_stride, up, up_row_stride, out, out_row_stride, rows, n, st);
  }
}
