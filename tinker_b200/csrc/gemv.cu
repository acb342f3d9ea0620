// Weight-streaming products for a handful of rows (decode steps: M = batch <= 8).
//
// y[m, n] = x[m, :] . W[n, :] for every n, with the epilogue options of the tcgen05 GEMM
// (gemm.cu): the 1/rms row scale of an RMSNorm folded into W (ssq_in), a residual add, the
// per-32-column sums of squares of the stored rows (ssq_out), or SwiGLU of a gate|up pair.
// With so few rows every weight byte is used M times, so the work is a stream over W at HBM
// speed; a tensor-core tile of 128 rows would be >94% padding and its set-up (TMEM, barriers,
// split-K cluster reduction) costs more than the stream. One warp owns CPW weight rows
// (CPW output columns, or CPW gate + CPW up rows for SwiGLU); its lanes take interleaved
// 16-byte chunks of K, so a warp reads CPW * 512 contiguous bytes per step; products are
// packed fp32 FMAs, then one butterfly reduction per (row, m). A CTA of 8 warps covers
// 8 * CPW columns; with ssq_out, a cluster of CL CTAs covers one 32-column chunk and its rank
// 0 adds the CTAs' sums of squares from distributed shared memory (fixed order).
#include <algorithm>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace gemv {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;

struct Params {
  const void* x;
  int64_t lda;
  const void* w[3];  // weight blocks stacked along n (rows n0, n1, n2); for SwiGLU w[0] gate, w[1] up
  int64_t n0, n1;
  void* y;
  int64_t ldy;
  const void* residual;  // [m, n], row stride ldy
  const float* ssq_in;   // [ssq_parts, m]
  int ssq_parts;
  float ssq_inv_k, ssq_eps;
  float* ssq_out;  // [ceil(n / 32), m]
  int m, n, k;
};

template <int DT>
__device__ __forceinline__ void cvt8(const uint4& u, uint64_t (&f)[4]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = Dt<DT>::unpack(*reinterpret_cast<const typename Dt<DT>::T2*>(&w[j]));
    f[j] = pack_f32x2(t.x, t.y);
  }
}

__device__ __forceinline__ float row_scale(const Params& p, int row) {
  if (!p.ssq_in) return 1.f;
  float s = 0.f;
  for (int i = 0; i < p.ssq_parts; ++i) s += p.ssq_in[static_cast<int64_t>(i) * p.m + row];
  return rsqrtf(s * p.ssq_inv_k + p.ssq_eps);
}

// SWIGLU: column j needs gate row j and up row j (ROWS = 2 * CPW weight rows per warp).
// KS: warps per column group, each on 1/KS of K (the partial sums meet in shared memory): a
// long row (the down projection of a decode step) then takes fewer rounds of loads per lane.
// CL: CTAs per cluster ((WARPS / KS) * CPW * CL == 32 when ssq_out is used).
template <int DT, int M, int CPW, bool SWIGLU, int CL, int KS>
__global__ void __launch_bounds__(THREADS) gemv_kernel(const Params p) {
  using T = typename Dt<DT>::T;
  constexpr int ROWS = SWIGLU ? 2 * CPW : CPW;
  constexpr int CWARPS = WARPS / KS;  // column groups per CTA
  __shared__ float ssq_s[WARPS][M];
  __shared__ float cta_ssq[M];
  __shared__ float part[KS > 1 ? CWARPS : 1][KS > 1 ? ROWS : 1][KS > 1 ? M : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kpart = warp / CWARPS;                                 // which 1/KS of K
  const int col0 = (blockIdx.x * CWARPS + warp % CWARPS) * CPW;  // first output column of this warp
  const int kc = p.k >> 3;                                        // 16-byte chunks per row
  const int kbeg = kpart * kc / KS, kend = (kpart + 1) * kc / KS;

  // weight row pointers (null past the end)
  const T* wrow[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int c = col0 + (SWIGLU ? r % CPW : r);
    wrow[r] = nullptr;
    if (c < p.n) {
      if (SWIGLU) {
        wrow[r] = reinterpret_cast<const T*>(p.w[r < CPW ? 0 : 1]) + static_cast<int64_t>(c) * p.k;
      } else {
        const int64_t nn = c;
        const int blk = nn < p.n0 ? 0 : nn < p.n0 + p.n1 ? 1 : 2;
        const int64_t local = blk == 0 ? nn : blk == 1 ? nn - p.n0 : nn - p.n0 - p.n1;
        const void* base = blk == 0 ? p.w[0] : blk == 1 ? p.w[1] : p.w[2];
        wrow[r] = reinterpret_cast<const T*>(base) + local * p.k;
      }
    }
  }
  // the weights do not depend on the previous kernel: start pulling them into L2
  for (int r = 0; r < ROWS; ++r)
    if (wrow[r])
      for (int c = kbeg + lane * 8; c < kend; c += 32 * 8) prefetch_l2(wrow[r] + static_cast<int64_t>(c) * 8);
  pdl_wait();

  uint64_t acc[ROWS][M];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0ull;
  const T* xb = reinterpret_cast<const T*>(p.x);
#pragma unroll 4  // a 1024-wide row in one round of loads per lane
  for (int c = kbeg + lane; c < kend; c += 32) {
    uint4 wv[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
      wv[r] = wrow[r] ? __ldcs(reinterpret_cast<const uint4*>(wrow[r]) + c) : make_uint4(0, 0, 0, 0);
    uint4 xv[M];
#pragma unroll
    for (int m = 0; m < M; ++m)
      xv[m] = m < p.m ? __ldg(reinterpret_cast<const uint4*>(xb + static_cast<int64_t>(m) * p.lda) + c)
                      : make_uint4(0, 0, 0, 0);
    uint64_t xf[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m) cvt8<DT>(xv[m], xf[m]);
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      uint64_t wf[4];
      cvt8<DT>(wv[r], wf);
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][m] = fma_f32x2(wf[j], xf[m][j], acc[r][m]);
    }
  }
  pdl_launch_dependents();

  // butterfly reduction: every lane ends with every (row, m) sum
  float sum[ROWS][M];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float lo, hi;
      unpack_f32x2(acc[r][m], lo, hi);
      float s = lo + hi;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      sum[r][m] = s;
    }
  if constexpr (KS > 1) {  // the warps of the second half of K hand their sums to the first
    if (kpart == 1 && lane == 0)
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) part[warp % CWARPS][r][m] = sum[r][m];
    __syncthreads();
    if (kpart == 0)
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) sum[r][m] += part[warp][r][m];
  }

  // epilogue: lane (c * M + m) stores output column col0 + c of row m
  float sq[M];
#pragma unroll
  for (int m = 0; m < M; ++m) sq[m] = 0.f;
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int col = col0 + c;
      if (kpart != 0 || m >= p.m || col >= p.n) continue;  // one writer per column
      const float sc = row_scale(p, m);
      float v;
      if (SWIGLU) {
        const float g = sum[c][m] * sc, u = sum[CPW + c][m] * sc;
        v = __fdividef(g, 1.0f + __expf(-g)) * u;
      } else {
        v = sum[c][m] * sc;
        if (p.residual)
          v += Dt<DT>::to_f(reinterpret_cast<const T*>(p.residual)[static_cast<int64_t>(m) * p.ldy + col]);
      }
      const T t = Dt<DT>::from_f(v);
      const float rv = Dt<DT>::to_f(t);
      sq[m] = fmaf(rv, rv, sq[m]);
      if (lane == c * M + m) reinterpret_cast<T*>(p.y)[static_cast<int64_t>(m) * p.ldy + col] = t;
    }
  if (!SWIGLU && p.ssq_out) {  // the CL CTAs of a cluster = one 32-column chunk
    if (lane == 0)
#pragma unroll
      for (int m = 0; m < M; ++m) ssq_s[warp][m] = sq[m];
    __syncthreads();
    if (threadIdx.x < M) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += ssq_s[w][threadIdx.x];
      cta_ssq[threadIdx.x] = s;
    }
    if constexpr (CL == 1) {
      if (threadIdx.x < p.m && threadIdx.x < M)
        p.ssq_out[static_cast<int64_t>(blockIdx.x) * p.m + threadIdx.x] = cta_ssq[threadIdx.x];
    } else {
      cluster_sync();  // every CTA's cta_ssq written
      if (cluster_ctarank() == 0 && threadIdx.x < p.m && threadIdx.x < M) {
        float s = 0.f;
#pragma unroll
        for (int r = 0; r < CL; ++r) s += ld_cluster_f32(mapa_shared(smem_u32(&cta_ssq[threadIdx.x]), r));
        p.ssq_out[static_cast<int64_t>(blockIdx.x / CL) * p.m + threadIdx.x] = s;
      }
      cluster_sync();  // the peers keep their shared memory until rank 0 has read it
    }
  }
}

template <int DT, int M, int CPW, bool SWIGLU, int CL, int KS = 1>
int launch_m(const Params& p, cudaStream_t st) {
  const int cols = (WARPS / KS) * CPW;
  const int grid = ((p.n + cols - 1) / cols + CL - 1) / CL * CL;  // whole clusters
  return launch_kernel(gemv_kernel<DT, M, CPW, SWIGLU, CL, KS>, dim3(grid), dim3(THREADS), 0, st, CL, "gemv", p);
}

template <int DT, int CPW, bool SWIGLU, int CL>
int launch_cpw(const Params& p, cudaStream_t st) {
  switch (p.m) {
    case 1: return launch_m<DT, 1, CPW, SWIGLU, CL>(p, st);
    case 2: return launch_m<DT, 2, CPW, SWIGLU, CL>(p, st);
    case 3:
    case 4: return launch_m<DT, 4, CPW, SWIGLU, CL>(p, st);
    default: return launch_m<DT, 8, CPW, SWIGLU, CL>(p, st);
  }
}

template <int DT>
int launch_dt(const Params& p, bool swiglu, int cpw, cudaStream_t st) {
  if (swiglu) return cpw == 1 ? launch_cpw<DT, 1, true, 1>(p, st) : launch_cpw<DT, 2, true, 1>(p, st);
  // one row against a long weight row (K >= 2048, e.g. the down projection of a decode step):
  // two warps per column, each on half of K; 4 columns per CTA, 8 CTAs per 32-column chunk
  if (p.ssq_out && p.m == 1 && p.k >= 2048) return launch_m<DT, 1, 1, false, 8, 2>(p, st);
  if (p.ssq_out) return launch_cpw<DT, 1, false, 4>(p, st);  // 8 columns per CTA, 4 CTAs per chunk
  if (cpw == 4) return launch_cpw<DT, 4, false, 1>(p, st);
  return cpw == 2 ? launch_cpw<DT, 2, false, 1>(p, st) : launch_cpw<DT, 1, false, 1>(p, st);
}

int run(int dtype, const void* x, int64_t lda, const void* const w[3], const int64_t nrows[3], bool swiglu, void* y,
        int64_t ldy, int64_t m, int64_t n, int64_t k, const void* residual, const float* ssq_in, int ssq_parts,
        float ssq_inv_k, float ssq_eps, float* ssq_out, cudaStream_t st) {
  if (m < 1 || m > MAX_M) return fail_invalid("gemv: 1 <= m <= 8 rows");
  if (k % 8 != 0 || lda % 8 != 0 || ldy < 1) return fail_invalid("gemv: k and the row stride must be multiples of 8");
  if (!aligned16(x) || !aligned16(w[0]) || (w[1] && !aligned16(w[1])) || (w[2] && !aligned16(w[2])))
    return fail_invalid("gemv: x and the weights must be 16-byte aligned");
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  Params p{};
  p.x = x;
  p.lda = lda;
  p.w[0] = w[0];
  p.w[1] = w[1] ? w[1] : w[0];
  p.w[2] = w[2] ? w[2] : w[0];
  p.n0 = nrows[0];
  p.n1 = nrows[1];
  p.y = y;
  p.ldy = ldy;
  p.residual = residual;
  p.ssq_in = ssq_in;
  p.ssq_parts = ssq_parts;
  p.ssq_inv_k = ssq_inv_k;
  p.ssq_eps = ssq_eps;
  p.ssq_out = ssq_out;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  // columns per warp: the most that still gives about two CTAs per SM (one with ssq_out, whose
  // 32-column chunks are split over clusters of 4 CTAs)
  const int max_cpw = swiglu ? 2 : 4;
  int cpw = 1;
  while (cpw < max_cpw && (n + WARPS * cpw * 2 - 1) / (WARPS * cpw * 2) >= 2 * dev.sm_count) cpw *= 2;
  return dtype == TK_F16 ? launch_dt<TK_F16>(p, swiglu, cpw, st) : launch_dt<TK_BF16>(p, swiglu, cpw, st);
}

}  // namespace gemv
}  // namespace tk
