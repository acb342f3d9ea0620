// One decode step of a whole decoder stack in one persistent kernel (at most 8 sequences, one new
// token each): the kernel boundaries of the per-block path become grid barriers.
//
// Per layer, five phases (the per-block path's five launches): the q|k|v product with the
// attention RMSNorm folded into its weights, KV-cache attention (RoPE of the new rows, cache
// append, split-K over the cached keys: kv_attention.cuh, run by the first four warps of a CTA),
// o_proj + residual, gate|up + SwiGLU with the FFN RMSNorm folded in, down + residual; the products
// are weight streams (every weight byte used by all rows at once), each CTA taking 8-column items
// with one column per warp. After the last layer the final RMSNorm. Row statistics of the residual
// stream are kept in 8-column parts, so the CTA that stores a column block also stores its part.
//
// Phases are separated by a grid barrier (a counter in global memory that every CTA increments
// once per barrier, zeroed before the launch) whose wait is bounded by %globaltimer: on a timeout, or once any kernel has
// recorded a device error, the barrier returns false and every CTA leaves. The launch is
// cooperative (every CTA resident), and activations written by other SMs are read through L2
// (ld.global.cg), since L1 is not coherent across SMs.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kv_attention.cuh"
#include "tk_host.h"

namespace tk {
namespace step {

constexpr int THREADS = 256;  // 8 warps; attention items run on warps 0-3
constexpr int WARPS = THREADS / 32;
constexpr int COLS = WARPS;   // output columns per product item (one per warp) = columns per statistics part

struct Layer {
  const void* wq;
  const void* wk;
  const void* wv;
  const void* wo;
  const void* wg;
  const void* wu;
  const void* wd;
  float eps_attn, eps_ffn;
};

struct Params {
  const Layer* layers;              // [num_layers] device copy
  const kvattn::Params* kv;         // [num_layers] device copy (cache pointers per layer)
  int num_layers;
  int m;                            // sequences
  int hidden, q_width, kv_width, inter;
  int kv_items;                     // attention items per layer (chunks x kv heads x row blocks x sequences)
  int kv_chunks, kv_units_y;        // grid shape of those items (x: chunks, y: kv heads x row blocks)
  const void* final_w;
  float final_eps;
  void* x;        // [m, hidden]: the embedding rows in; the last block's output after the step
  void* y;        // [m, hidden]: the final RMSNorm of x (the LM head's input)
  void* h;        // [m, hidden]
  void* qkv;      // [m, q_width + 2 * kv_width]
  void* attn;     // [m, q_width]
  void* act;      // [m, inter]
  float* ssq_x;   // [hidden / COLS, m]
  float* ssq_h;   // [hidden / COLS, m]
  unsigned* bar;  // arrival counter (zeroed before each launch)
  int withhold_cta;  // test hook: this CTA does not arrive at the first grid barrier (-1: none)
};

// ---- grid barrier ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int device_error_now() {
  return *reinterpret_cast<volatile int*>(&g_tk_device_error);
}

// Every CTA arrives; returns false (in every thread of the CTA) when the step must stop. The
// counter only grows during a launch (zeroed before it): barrier k waits for k * gridDim.x
// arrivals. `k` counts this CTA's barriers (the same sequence in every CTA).
// `arrive` false (only the tk_decode_step_withhold_arrival test hook) makes the CTA wait without
// arriving, so that every CTA's bounded wait runs out.
__device__ __forceinline__ bool grid_barrier(unsigned* bar, unsigned& k, bool arrive = true) {
  __shared__ int s_ok;
  __syncthreads();
  ++k;
  if (threadIdx.x == 0) {
    int ok = device_error_now() == 0;
    if (ok) {
      __threadfence();  // publish this CTA's writes
      if (arrive) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
      const unsigned target = k * gridDim.x;
      const uint64_t t0 = globaltimer();
      while (ld_acquire(bar) < target) {
        if (device_error_now()) {
          ok = 0;
          break;
        }
        if (globaltimer() - t0 > TK_WAIT_LIMIT_NS) {
          record_device_error(TK_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// ---- weight-streaming products ----------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void cvt8(const uint4& u, uint64_t (&f)[4]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = Dt<DT>::unpack(*reinterpret_cast<const typename Dt<DT>::T2*>(&w[j]));
    f[j] = pack_f32x2(t.x, t.y);
  }
}

// 1/rms of rows 0..m-1 from `parts` statistics parts (warp r computes row r) into rstd[];
// all 1 without statistics.
template <int M>
__device__ __forceinline__ void row_rstd(const float* ssq, int parts, int m, float inv_k, float eps, float* rstd) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < m) {
    float s = 0.f;
    if (ssq)
      for (int i = lane; i < parts; i += 32) s += __ldcg(ssq + static_cast<int64_t>(i) * m + warp);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) rstd[warp] = ssq ? rsqrtf(s * inv_k + eps) : 1.f;
  }
  __syncthreads();
}

struct Product {
  const void* x;  // [m, k] (row stride k)
  const void* w0; int64_t n0;
  const void* w1; int64_t n1;
  const void* w2;  // w0|w1|w2 stacked along n; SwiGLU: w0 gate, w1 up
  int n, k;
  const void* residual;  // [m, n] or null
  void* y;               // [m, n]
  float* ssq_out;        // [n / COLS, m] or null
};

// Items first, first + stride, ... (n_items <= J of them) of a product, all at once: each warp
// computes output column item*COLS + warp of every item, loading each input row chunk once for
// all items. rstd: the input rows' 1/rms.
template <int DT, int M, int J, bool SWIGLU>
__device__ __forceinline__ void product_items(const Product& P, int first, int stride, int n_items, int m,
                                              const float* rstd, float (*sq_s)[WARPS][M]) {
  using T = typename Dt<DT>::T;
  constexpr int ROWS = SWIGLU ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = P.k >> 3;
  const T* wrow[J][ROWS];
  int cols[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int col = (first + j * stride) * COLS + warp;
    cols[j] = (j < n_items && col < P.n) ? col : -1;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      wrow[j][r] = nullptr;
      if (cols[j] >= 0) {
        if (SWIGLU) {
          wrow[j][r] = reinterpret_cast<const T*>(r == 0 ? P.w0 : P.w1) + static_cast<int64_t>(col) * P.k;
        } else {
          const int blk = col < P.n0 ? 0 : col < P.n0 + P.n1 ? 1 : 2;
          const int64_t local = blk == 0 ? col : blk == 1 ? col - P.n0 : col - P.n0 - P.n1;
          const void* base = blk == 0 ? P.w0 : blk == 1 ? P.w1 : P.w2;
          wrow[j][r] = reinterpret_cast<const T*>(base) + local * P.k;
        }
      }
    }
  }
  uint64_t acc[J][ROWS][M];
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int i = 0; i < M; ++i) acc[j][r][i] = 0ull;
  const T* xb = reinterpret_cast<const T*>(P.x);
#pragma unroll(J * ROWS > 2 ? 2 : 4)
  for (int c = lane; c < kc; c += 32) {
    uint4 wv[J][ROWS];
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
        wv[j][r] = wrow[j][r] ? __ldcs(reinterpret_cast<const uint4*>(wrow[j][r]) + c) : make_uint4(0, 0, 0, 0);
    uint64_t xf[M][4];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const uint4 xv = i < m ? __ldcg(reinterpret_cast<const uint4*>(xb + static_cast<int64_t>(i) * P.k) + c)
                             : make_uint4(0, 0, 0, 0);
      cvt8<DT>(xv, xf[i]);
    }
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        uint64_t wf[4];
        cvt8<DT>(wv[j][r], wf);
#pragma unroll
        for (int i = 0; i < M; ++i)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[j][r][i] = fma_f32x2(wf[q], xf[i][q], acc[j][r][i]);
      }
  }
#pragma unroll
  for (int j = 0; j < J; ++j) {
    float sum[ROWS][M];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int i = 0; i < M; ++i) {
        float lo, hi;
        unpack_f32x2(acc[j][r][i], lo, hi);
        float s = lo + hi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sum[r][i] = s;
      }
    const int col = cols[j];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      float sq = 0.f;
      if (i < m && col >= 0) {
        float v;
        if (SWIGLU) {
          const float g = sum[0][i] * rstd[i], u = sum[1][i] * rstd[i];
          v = __fdividef(g, 1.0f + __expf(-g)) * u;
        } else {
          v = sum[0][i] * rstd[i];
          if (P.residual)
            v += Dt<DT>::to_f(__ldcg(reinterpret_cast<const T*>(P.residual) + static_cast<int64_t>(i) * P.n + col));
        }
        const T t = Dt<DT>::from_f(v);
        const float rv = Dt<DT>::to_f(t);
        sq = rv * rv;
        if (lane == i) reinterpret_cast<T*>(P.y)[static_cast<int64_t>(i) * P.n + col] = t;
      }
      if (lane == 0) sq_s[j][warp][i] = sq;
    }
  }
  if (P.ssq_out) {  // part (item) = the COLS columns of one item, summed over the warps in order
    __syncthreads();
    for (int t = threadIdx.x; t < n_items * m; t += THREADS) {
      const int j = t / m, i = t % m;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += sq_s[j][w][i];
      P.ssq_out[static_cast<int64_t>(first + j * stride) * m + i] = s;
    }
    __syncthreads();  // sq_s is rewritten by the next group
  }
}

// Pull into L2 the weight rows this CTA's items of a product will read (issued one phase ahead:
// the weights do not depend on the barrier in between). Threads [t0, t0 + nt) take part.
__device__ __forceinline__ void prefetch_product(const Product& P, bool swiglu, int t0, int nt) {
  const int items = (P.n + COLS - 1) / COLS;
  const int lines = (P.k * 2 + 127) / 128;  // 128-byte lines per weight row
  const int nrows = swiglu ? 2 * COLS : COLS;
  for (int item = blockIdx.x; item < items; item += gridDim.x)
    for (int idx = static_cast<int>(threadIdx.x) - t0; idx >= 0 && idx < nrows * lines; idx += nt) {
      const int r = idx / lines, line = idx % lines;
      const int col = item * COLS + r % COLS;
      if (col >= P.n) continue;
      const char* row;
      if (swiglu) {
        row = static_cast<const char*>(r < COLS ? P.w0 : P.w1) + static_cast<int64_t>(col) * P.k * 2;
      } else {
        const int blk = col < P.n0 ? 0 : col < P.n0 + P.n1 ? 1 : 2;
        const int64_t local = blk == 0 ? col : blk == 1 ? col - P.n0 : col - P.n0 - P.n1;
        row = static_cast<const char*>(blk == 0 ? P.w0 : blk == 1 ? P.w1 : P.w2) + local * P.k * 2;
      }
      prefetch_l2(row + static_cast<int64_t>(line) * 128);
    }
}

// Items per warp pass: several when the rows are few (registers allow it), so that a CTA's share
// of a phase is one round of loads.
template <int M>
struct ItemsPerPass {
  static constexpr int value = M <= 2 ? 4 : M <= 4 ? 2 : 1;
};

template <int DT, int M, bool SWIGLU>
__device__ __forceinline__ void product(const Product& P, int m, const float* ssq_in, int parts, float inv_k,
                                        float eps) {
  constexpr int J = ItemsPerPass<M>::value;
  __shared__ float rstd[M];
  __shared__ float sq_s[J][WARPS][M];
  row_rstd<M>(ssq_in, parts, m, inv_k, eps, rstd);
  const int items = (P.n + COLS - 1) / COLS;
  const int mine = items > static_cast<int>(blockIdx.x) ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  for (int g = 0; g < mine; g += J)
    product_items<DT, M, J, SWIGLU>(P, blockIdx.x + g * gridDim.x, gridDim.x, min(J, mine - g), m, rstd, sq_s);
}

template <int DT, int D, int R, int M>
__global__ void __launch_bounds__(THREADS, 1) decode_step_kernel(const Params p) {
  using T = typename Dt<DT>::T;
  extern __shared__ __align__(128) uint8_t smem[];
  const int m = p.m;
  const float inv_h = 1.f / static_cast<float>(p.hidden);
  const int parts_h = p.hidden / COLS;
  unsigned nbar = 0;  // grid barriers passed

  // row statistics of the input rows (the embedding output), in COLS-column parts
  for (int idx = blockIdx.x * THREADS + threadIdx.x; idx < parts_h * m; idx += gridDim.x * THREADS) {
    const int part = idx / m, row = idx % m;
    const T* src = reinterpret_cast<const T*>(p.x) + static_cast<int64_t>(row) * p.hidden + part * COLS;
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src));
    uint64_t f[4];
    cvt8<DT>(u, f);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a, b;
      unpack_f32x2(f[j], a, b);
      s = fmaf(a, a, fmaf(b, b, s));
    }
    p.ssq_x[static_cast<int64_t>(part) * m + row] = s;
  }
  if (!grid_barrier(p.bar, nbar, p.withhold_cta != static_cast<int>(blockIdx.x))) return;

  auto qkv_of = [&](const Layer& L) {
    return Product{p.x, L.wq, p.q_width, L.wk, p.kv_width, L.wv, p.q_width + 2 * p.kv_width, p.hidden,
                   nullptr, p.qkv, nullptr};
  };
  prefetch_product(qkv_of(p.layers[0]), false, 0, THREADS);
  for (int l = 0; l < p.num_layers; ++l) {
    const Layer L = p.layers[l];
    const Product Po{p.attn, L.wo, p.hidden, nullptr, 0, nullptr, p.hidden, p.q_width, p.x, p.h, p.ssq_h};
    const Product Pg{p.h, L.wg, p.inter, L.wu, p.inter, nullptr, p.inter, p.hidden, nullptr, p.act, nullptr};
    const Product Pd{p.act, L.wd, p.hidden, nullptr, 0, nullptr, p.hidden, p.inter, p.h, p.x, p.ssq_x};
    const kvattn::Params& kv = p.kv[l];
    // q|k|v with the attention RMSNorm folded in; the cached keys/values of this CTA's attention
    // items go to L2 meanwhile
    {
      const int kv_len = __ldcg(kv.start_dev) + 1;
      for (int item = blockIdx.x; item < p.kv_items; item += gridDim.x) {
        if (item % p.kv_chunks || kv_len < 1 || kv_len > kv.cap) continue;
        const int rest = item / p.kv_chunks;
        const int yy = rest % p.kv_units_y, b = rest / p.kv_units_y;
        const int64_t row0 = (static_cast<int64_t>(b) * kv.num_kv_heads + yy / kv.n_rb) * kv.cap;
        const int64_t bytes = static_cast<int64_t>(kv_len) * D * 2;
        for (int64_t o = static_cast<int64_t>(threadIdx.x) * 128; o < bytes; o += THREADS * 128) {
          prefetch_l2(static_cast<const char*>(kv.kc) + row0 * D * 2 + o);
          prefetch_l2(static_cast<const char*>(kv.vc) + row0 * D * 2 + o);
        }
      }
      product<DT, M, false>(qkv_of(L), m, p.ssq_x, parts_h, inv_h, L.eps_attn);
    }
    if (!grid_barrier(p.bar, nbar)) return;
    // attention against the cache (warps 0-3 of a CTA per item); warps 4-7 pull o_proj's rows
    if (threadIdx.x < kvattn::THREADS) {
      for (int item = blockIdx.x; item < p.kv_items; item += gridDim.x) {
        const int chunk = item % p.kv_chunks;
        const int rest = item / p.kv_chunks;
        const int yy = rest % p.kv_units_y, b = rest / p.kv_units_y;
        kvattn::kv_attention_item<DT, D, R>(kv, chunk, yy / kv.n_rb, yy % kv.n_rb, b, b * p.kv_units_y + yy,
                                            item == 0, smem);
        kvattn::kv_sync();  // the next item reuses the shared memory
      }
    } else {
      prefetch_product(Po, false, kvattn::THREADS, THREADS - kvattn::THREADS);
    }
    if (!grid_barrier(p.bar, nbar)) return;
    // o_proj + residual x -> h, statistics of h
    prefetch_product(Pg, true, 0, THREADS);
    product<DT, M, false>(Po, m, nullptr, 0, 0.f, 0.f);
    if (!grid_barrier(p.bar, nbar)) return;
    // gate|up + SwiGLU with the FFN RMSNorm folded in
    prefetch_product(Pd, false, 0, THREADS);
    product<DT, M, true>(Pg, m, p.ssq_h, parts_h, inv_h, L.eps_ffn);
    if (!grid_barrier(p.bar, nbar)) return;
    // down + residual h -> x, statistics of x for the next layer
    if (l + 1 < p.num_layers) prefetch_product(qkv_of(p.layers[l + 1]), false, 0, THREADS);
    product<DT, M, false>(Pd, m, nullptr, 0, 0.f, 0.f);
    if (!grid_barrier(p.bar, nbar)) return;
  }

  // final RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, one rounding
  {
    __shared__ float rstd[M];
    row_rstd<M>(p.ssq_x, parts_h, m, inv_h, p.final_eps, rstd);
    const T* w = reinterpret_cast<const T*>(p.final_w);
    for (int idx = blockIdx.x * THREADS + threadIdx.x; idx < m * p.hidden; idx += gridDim.x * THREADS) {
      const int row = idx / p.hidden, c = idx % p.hidden;
      const float v = Dt<DT>::to_f(__ldcg(reinterpret_cast<const T*>(p.x) + idx)) * rstd[row] * Dt<DT>::to_f(w[c]);
      reinterpret_cast<T*>(p.y)[idx] = Dt<DT>::from_f(v);
    }
  }
}

// ---- host side ----------------------------------------------------------------------------------
struct Plan {
  Params p;
  int dtype, head_dim, rows_cta, grid;
  size_t smem;
};

std::mutex g_mu;
std::unordered_map<const void*, Plan> g_plans;  // keyed by the scratch pointer

inline size_t align_up(size_t x) { return (x + 255) / 256 * 256; }

struct Layout {
  size_t layers, kv, h, qkv, attn, act, ssq_x, ssq_h, bar, kv_ws, total;
  int64_t kv_ws_bytes;
};

Layout layout(int num_layers, int batch, int hidden, int num_heads, int num_kv_heads, int head_dim, int inter,
              int capacity, int sm_count) {
  Layout L{};
  const int q_width = num_heads * head_dim, kv_width = num_kv_heads * head_dim;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes);
    return at;
  };
  L.layers = take(sizeof(Layer) * num_layers);
  L.kv = take(sizeof(kvattn::Params) * num_layers);
  L.h = take(size_t(batch) * hidden * 2);
  L.qkv = take(size_t(batch) * (q_width + 2 * kv_width) * 2);
  L.attn = take(size_t(batch) * q_width * 2);
  L.act = take(size_t(batch) * inter * 2);
  L.ssq_x = take(size_t(hidden / COLS) * batch * 4);
  L.ssq_h = take(size_t(hidden / COLS) * batch * 4);
  L.bar = take(16);
  const kvattn::Plan kp = kvattn::make_plan(batch, num_kv_heads, num_heads / num_kv_heads, capacity, head_dim, sm_count);
  L.kv_ws_bytes = static_cast<int64_t>(kp.bytes());
  L.kv_ws = take(kp.bytes());
  L.total = o;
  return L;
}

template <int DT, int D, int R, int M>
int launch(const Plan& pl, cudaStream_t st) {
  auto kern = decode_step_kernel<DT, D, R, M>;
  static std::mutex mu;
  static int per_sm[64] = {};  // 0 until configured; written and read under mu
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  int resident = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    resident = per_sm[dev.device];
  }
  if (!resident) {
    std::lock_guard<std::mutex> lock(mu);
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(pl.smem)),
                            "cudaFuncSetAttribute(decode_step)"))
      return rc;
    int n = 0;
    if (int rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, THREADS, pl.smem),
                            "cudaOccupancyMaxActiveBlocksPerMultiprocessor(decode_step)"))
      return rc;
    if (n < 1) return set_error(TK_ERR_UNSUPPORTED, "decode_step: the kernel does not fit on an SM");
    per_sm[dev.device] = n;
    resident = n;
  }
  if (int rc = check_cuda(cudaMemsetAsync(pl.p.bar, 0, 2 * sizeof(unsigned), st), "decode_step barrier reset"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(dev.sm_count * resident);  // every CTA resident
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, pl.p), "decode_step");
}

template <int DT, int D, int R>
int launch_m(const Plan& pl, cudaStream_t st) {
  switch (pl.p.m) {
    case 1: return launch<DT, D, R, 1>(pl, st);
    case 2: return launch<DT, D, R, 2>(pl, st);
    case 3:
    case 4: return launch<DT, D, R, 4>(pl, st);
    default: return launch<DT, D, R, 8>(pl, st);
  }
}

template <int DT, int D>
int launch_r(const Plan& pl, cudaStream_t st) {
  switch (pl.rows_cta) {
    case 1: return launch_m<DT, D, 1>(pl, st);
    case 4: return launch_m<DT, D, 4>(pl, st);
    default: return launch_m<DT, D, 8>(pl, st);
  }
}

template <int D>
size_t kv_smem(int rows_cta) {
  return rows_cta == 1 ? kvattn::Smem<D, 1>::TOTAL : rows_cta == 4 ? kvattn::Smem<D, 4>::TOTAL
                                                                   : kvattn::Smem<D, 8>::TOTAL;
}

}  // namespace step
}  // namespace tk

extern "C" int64_t tk_decode_step_scratch_bytes(int num_layers, int batch, int hidden, int num_heads, int num_kv_heads,
                                                int head_dim, int intermediate, int capacity) {
  using namespace tk;
  if (num_layers <= 0 || batch <= 0 || hidden <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      intermediate <= 0 || capacity <= 0)
    return 0;
  DeviceInfo di;
  if (current_device_info(&di)) return -1;
  return static_cast<int64_t>(
      step::layout(num_layers, batch, hidden, num_heads, num_kv_heads, head_dim, intermediate, capacity, di.sm_count)
          .total);
}

extern "C" int tk_decode_step_setup(const tk_step_layer* layers, int num_layers, int batch, int hidden, int num_heads,
                                    int num_kv_heads, int head_dim, int intermediate, const float* cos_table,
                                    const float* sin_table, int64_t table_rows, int capacity, const int* position,
                                    const void* final_norm_weight, float final_eps, int dtype, void* scratch,
                                    int64_t scratch_bytes) {
  using namespace tk;
  using namespace tk::step;
  if (!half_dtype(dtype)) return fail_invalid("decode_step: dtype must be F16 or BF16");
  if (head_dim != 64 && head_dim != 128) return set_error(TK_ERR_UNSUPPORTED, "decode_step: head_dim must be 64 or 128");
  if (batch < 1 || batch > 8) return set_error(TK_ERR_UNSUPPORTED, "decode_step: 1 to 8 sequences");
  if (num_layers < 1 || num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads || num_heads / num_kv_heads > 8)
    return fail_invalid("decode_step: heads (at most 8 query heads per kv head)");
  if (hidden % 32 || intermediate % 8 || hidden > 65536 || intermediate > 65536)
    return fail_invalid("decode_step: hidden must be a multiple of 32 and intermediate of 8");
  if (capacity < 1 || capacity > table_rows) return fail_invalid("decode_step: capacity beyond the RoPE table");
  if (!layers || !cos_table || !sin_table || !position || !final_norm_weight || !scratch)
    return fail_invalid("decode_step: NULL pointer");
  if (!aligned16(scratch) || !aligned16(cos_table) || !aligned16(sin_table))
    return fail_invalid("decode_step: pointers must be 16-byte aligned");
  DeviceInfo di;
  if (int rc = current_device_info(&di)) return rc;
  const Layout L = layout(num_layers, batch, hidden, num_heads, num_kv_heads, head_dim, intermediate, capacity,
                          di.sm_count);
  if (scratch_bytes < static_cast<int64_t>(L.total)) return fail_invalid("decode_step: scratch too small");
  const int q_width = num_heads * head_dim, kv_width = num_kv_heads * head_dim;
  char* base = static_cast<char*>(scratch);
  std::vector<Layer> hl(num_layers);
  std::vector<kvattn::Params> hk(num_layers);
  const int groups = num_heads / num_kv_heads;
  const kvattn::Plan kp = kvattn::make_plan(batch, num_kv_heads, groups, capacity, head_dim, di.sm_count);
  for (int i = 0; i < num_layers; ++i) {
    const tk_step_layer& s = layers[i];
    if (!s.wq || !s.wk || !s.wv || !s.wo || !s.wg || !s.wu || !s.wd || !s.k_cache || !s.v_cache)
      return fail_invalid("decode_step: NULL layer pointer");
    for (const void* w : {s.wq, s.wk, s.wv, s.wo, s.wg, s.wu, s.wd, static_cast<const void*>(s.k_cache),
                          static_cast<const void*>(s.v_cache)})
      if (!aligned16(w)) return fail_invalid("decode_step: weights and caches must be 16-byte aligned");
    hl[i] = Layer{s.wq, s.wk, s.wv, s.wo, s.wg, s.wu, s.wd, s.eps_attn, s.eps_ffn};
    kvattn::Params& k = hk[i];
    k = kvattn::Params{};
    k.q = base + L.qkv;
    k.qs = q_width + 2 * kv_width;
    k.k = base + L.qkv + size_t(q_width) * 2;
    k.ks = k.qs;
    k.v = base + L.qkv + size_t(q_width + kv_width) * 2;
    k.vs = k.qs;
    k.kc = s.k_cache;
    k.vc = s.v_cache;
    k.cap = capacity;
    k.cos_t = cos_table;
    k.sin_t = sin_table;
    k.table_rows = table_rows;
    k.out = base + L.attn;
    k.os = q_width;
    k.seq = 1;
    k.num_kv_heads = num_kv_heads;
    k.groups = groups;
    k.rows = groups;
    k.start_pos = 0;
    k.start_dev = position;
    k.n_rb = kp.n_rb;
    k.n_chunks = kp.n_chunks;
    k.scale_log2 = static_cast<float>((1.0 / std::sqrt(double(head_dim))) * 1.4426950408889634);
    if (kp.bytes() > 0) {
      char* ws = base + L.kv_ws;
      k.counters = reinterpret_cast<int*>(ws);
      k.part_ml = reinterpret_cast<float2*>(ws + kp.counters_bytes);
      k.part_o = reinterpret_cast<float*>(ws + kp.counters_bytes + kp.ml_bytes);
    }
  }
  if (int rc = check_cuda(cudaMemset(scratch, 0, L.total), "decode_step scratch clear")) return rc;
  if (int rc = check_cuda(cudaMemcpy(base + L.layers, hl.data(), sizeof(Layer) * num_layers, cudaMemcpyHostToDevice),
                          "decode_step layer table"))
    return rc;
  if (int rc = check_cuda(cudaMemcpy(base + L.kv, hk.data(), sizeof(kvattn::Params) * num_layers,
                                     cudaMemcpyHostToDevice),
                          "decode_step attention table"))
    return rc;
  Plan pl{};
  Params& p = pl.p;
  p.layers = reinterpret_cast<const Layer*>(base + L.layers);
  p.kv = reinterpret_cast<const kvattn::Params*>(base + L.kv);
  p.num_layers = num_layers;
  p.m = batch;
  p.hidden = hidden;
  p.q_width = q_width;
  p.kv_width = kv_width;
  p.inter = intermediate;
  p.kv_chunks = kp.n_chunks;
  p.kv_units_y = num_kv_heads * kp.n_rb;
  p.kv_items = kp.n_chunks * p.kv_units_y * batch;
  p.final_w = final_norm_weight;
  p.final_eps = final_eps;
  p.h = base + L.h;
  p.qkv = base + L.qkv;
  p.attn = base + L.attn;
  p.act = base + L.act;
  p.ssq_x = reinterpret_cast<float*>(base + L.ssq_x);
  p.ssq_h = reinterpret_cast<float*>(base + L.ssq_h);
  p.bar = reinterpret_cast<unsigned*>(base + L.bar);
  p.withhold_cta = -1;
  pl.dtype = dtype;
  pl.head_dim = head_dim;
  pl.rows_cta = kp.rows_cta;
  pl.smem = head_dim == 64 ? kv_smem<64>(kp.rows_cta) : kv_smem<128>(kp.rows_cta);
  std::lock_guard<std::mutex> lock(g_mu);
  g_plans[scratch] = pl;
  return TK_OK;
}

extern "C" int tk_decode_step(void* x, void* y, void* scratch, void* stream) {
  using namespace tk;
  using namespace tk::step;
  Plan pl;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_plans.find(scratch);
    if (it == g_plans.end()) return fail_invalid("decode_step: scratch was not prepared by tk_decode_step_setup");
    pl = it->second;
  }
  if (!x || !y || !aligned16(x) || !aligned16(y)) return fail_invalid("decode_step: x and y must be 16-byte aligned");
  pl.p.x = x;
  pl.p.y = y;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pl.dtype == TK_F16)
    return pl.head_dim == 64 ? launch_r<TK_F16, 64>(pl, st) : launch_r<TK_F16, 128>(pl, st);
  return pl.head_dim == 64 ? launch_r<TK_BF16, 64>(pl, st) : launch_r<TK_BF16, 128>(pl, st);
}

extern "C" int tk_decode_step_withhold_arrival(void* scratch, int cta) {
  using namespace tk;
  std::lock_guard<std::mutex> lock(tk::step::g_mu);
  auto it = tk::step::g_plans.find(scratch);
  if (it == tk::step::g_plans.end())
    return fail_invalid("decode_step: scratch was not prepared by tk_decode_step_setup");
  if (cta < -1) return fail_invalid("decode_step_withhold_arrival: cta must be >= -1");
  it->second.p.withhold_cta = cta;
  return TK_OK;
}

extern "C" int tk_decode_step_release(void* scratch) {
  std::lock_guard<std::mutex> lock(tk::step::g_mu);
  tk::step::g_plans.erase(scratch);
  return TK_OK;
}
