// tcgen05 GEMM y[m, n] = x[m, k] . w[n, k]^T for the projections of the
// decoder: the fused q|k|v projection, o_proj, the gate|up projection with the
// SwiGLU epilogue, and down_proj (optionally adding the residual).
//
// Structure (one persistent CTA per SM slot, 192 threads):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per k-block
//               into a STAGES-deep ring of 128-byte-swizzled shared-memory slots.
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into one of two fp32 accumulators in TMEM and
//               frees ring slots / publishes accumulators with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (each thread owns one
//               output row), SwiGLU or residual add in fp32, one rounding,
//               16-byte stores. Two accumulators let the epilogue of tile i
//               overlap the main loop of tile i+1.
// The weight may be split into up to three row blocks (q, k and v projection
// weights used as one GEMM without concatenating them); for the SwiGLU
// epilogue each B tile holds BN/2 rows of the gate weight followed by the same
// BN/2 rows of the up weight, so gate and up of one output column sit in the
// same accumulator tile.
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <numeric>
#include <string>
#include <tuple>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of 2-byte elements
constexpr int THREADS = 192;
// 2-SM pair kernel: warps 0 (TMA), 1 (MMA) and eight epilogue warps, two per TMEM lane quarter
// (each covers half of the tile's columns), so the epilogue of tile i keeps pace with the
// main loop of tile i + 1 even when K is short.
constexpr int PAIR_THREADS = 320;
constexpr int PAIR_EPI_WARPS = 8;
constexpr int GROUP_M = 16;  // rasterisation: GROUP_M m-tiles sweep all n-tiles together

enum Epi { EPI_STORE = 0, EPI_SWIGLU = 1 };

struct Params {
  int m, n, k;       // n: output columns (for SwiGLU the width of h)
  int num_kb;        // k-blocks of BK
  int m_tiles, n_tiles;
  int seg1, seg2;    // first n-tile of weight block 1 and 2 (plain epilogue)
  void* y;
  int64_t ldy;
  const void* residual;  // optional, [m, n] with row stride ldy
  // RoPE epilogue (plain store only): columns [0, rope_cols) are the q and k heads of a
  // fused q|k|v projection; row r sits at position rope_start + r % rope_seq.
  int rope_cols;         // 0: no RoPE
  int rope_seq, rope_start, rope_half_d;
  const float* rope_cos;  // [table_rows, rope_half_d] float32
  const float* rope_sin;
  // RMSNorm folded into this GEMM (its weight already multiplied into the weights): the
  // result of row r is scaled by 1/sqrt(sum_i ssq_in[i * m + r] * ssq_inv_k + ssq_eps).
  const float* ssq_in;   // [ssq_parts, m] partial sums of squares of x's rows, or null
  int ssq_parts;
  float ssq_inv_k, ssq_eps;
  // Plain store: ssq_out[(col / 32) * m + r] = sum of squares of the 32 stored (rounded)
  // values of row r from column col on, the input of a folded RMSNorm downstream.
  float* ssq_out;
  // Nonzero: no kernel since the stream last waited for all earlier work wrote the weights,
  // so their first tiles may go to shared memory before griddepcontrol.wait.
  int weights_prefetch;
  L2Prefetch pf;  // weights of later kernels pulled into L2 (every CTA a share, at its start)
};

// 1/rms of input row `row` for a folded RMSNorm (1 when there is none or the row is padding).
__device__ __forceinline__ float row_rstd(const Params& p, int row) {
  if (!p.ssq_in || row >= p.m) return 1.f;
  float s = 0.f;
  for (int i = 0; i < p.ssq_parts; ++i) s += p.ssq_in[static_cast<int64_t>(i) * p.m + row];
  return rsqrtf(s * p.ssq_inv_k + p.ssq_eps);
}

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& mt, int& nt) {
  const int per_group = GROUP_M * p.n_tiles;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gm = min(p.m_tiles - first_m, GROUP_M);
  const int r = t - g * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int BAR_OFF = RING;
  static constexpr int NUM_BARS = 2 * STAGES + 4;
  static constexpr int TOTAL = 1024 /*align slack*/ + RING + NUM_BARS * 8 + 16;
  static constexpr uint32_t TMEM_COLS = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128
                                                         : (2 * BN) <= 256 ? 256 : 512;
};

// silu(g) * u = g / (1 + e^-g) * u in fp32 with the fast exponential and division (a few ulp of
// fp32; the result is rounded to 16 bits right after).
__device__ __forceinline__ float swiglu_f(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

__device__ __forceinline__ void scale32(float (&v)[32], float s) {
  if (s != 1.f) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= s;
  }
}

template <int DT>
__device__ __forceinline__ void store_row32(void* y, int64_t ldy, int row, int col, int n, const float (&v)[32],
                                            const void* residual, float* ssq = nullptr) {
  using D = Dt<DT>;
  using T = typename D::T;
  T* dst = reinterpret_cast<T*>(y) + static_cast<int64_t>(row) * ldy + col;
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = v[i];
  if (residual) {
    const T* r = reinterpret_cast<const T*>(residual) + static_cast<int64_t>(row) * ldy + col;
    if (col + 32 <= n) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = reinterpret_cast<const uint4*>(r)[q];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = D::unpack(*reinterpret_cast<const typename D::T2*>(&w[j]));
          o[q * 8 + 2 * j] += f.x;
          o[q * 8 + 2 * j + 1] += f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < n) o[i] += D::to_f(r[i]);
    }
  }
  float sq = 0.f;
  if (col + 32 <= n) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        typename D::T2 h = D::pack(o[q * 8 + 2 * j], o[q * 8 + 2 * j + 1]);
        if (ssq) {
          const float2 r = D::unpack(h);
          sq = fmaf(r.x, r.x, fmaf(r.y, r.y, sq));
        }
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col + i < n) {
        const T t = D::from_f(o[i]);
        dst[i] = t;
        const float r = D::to_f(t);
        sq = fmaf(r, r, sq);
      }
  }
  if (ssq) *ssq = sq;
}

// Where a plain-store epilogue puts the row sum of squares of its 32-column chunk (or null).
__device__ __forceinline__ float* ssq_slot(const Params& p, int row, int col) {
  return p.ssq_out ? p.ssq_out + static_cast<int64_t>(col >> 5) * p.m + row : nullptr;
}

// RoPE of the 32 accumulator columns [col, col + 32) of row `row`, all inside one q or
// k head: each value is first rounded to the output dtype (the value the projection
// stores, which the reference's RoPE kernel then reads, tinker/kernels/fused_attention.py
// :53-69), then each interleaved pair (x0, x1) becomes (x0 c - x1 s, x0 s + x1 c) in fp32
// with the angle of pair (col mod head_dim) / 2 at the row's position; the caller rounds
// the result once more when it stores it.
template <int DT>
__device__ __forceinline__ void rope_chunk32(float (&v)[32], int row, int col, const Params& p) {
  using D = Dt<DT>;
  const int64_t pos = static_cast<int64_t>(p.rope_start) + row % p.rope_seq;
  const int i0 = (col % (2 * p.rope_half_d)) >> 1;  // multiple of 16
  const float4* c4 = reinterpret_cast<const float4*>(p.rope_cos + pos * p.rope_half_d + i0);
  const float4* s4 = reinterpret_cast<const float4*>(p.rope_sin + pos * p.rope_half_d + i0);
  float c[16], s[16];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 a = c4[q], b = s4[q];
    c[4 * q] = a.x; c[4 * q + 1] = a.y; c[4 * q + 2] = a.z; c[4 * q + 3] = a.w;
    s[4 * q] = b.x; s[4 * q + 1] = b.y; s[4 * q + 2] = b.z; s[4 * q + 3] = b.w;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x0 = D::to_f(D::from_f(v[2 * i]));
    const float x1 = D::to_f(D::from_f(v[2 * i + 1]));
    v[2 * i] = x0 * c[i] - x1 * s[i];
    v[2 * i + 1] = x0 * s[i] + x1 * c[i];
  }
}

// First 16 values of v to columns [col, col + 16) of row `row` (columns >= n dropped).
template <int DT>
__device__ __forceinline__ void store_row16(void* y, int64_t ldy, int row, int col, int n, const float* v) {
  using D = Dt<DT>;
  using T = typename D::T;
  T* dst = reinterpret_cast<T*>(y) + static_cast<int64_t>(row) * ldy + col;
  if (col + 16 <= n) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        typename D::T2 h = D::pack(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (col + i < n) dst[i] = D::from_f(v[i]);
  }
}

template <int DT, int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tb2, const Params p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring_a = smem;
  uint8_t* ring_b = smem + STAGES * S::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::NUM_BARS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 3 && p.pf.n) l2_prefetch_share(p.pf, blockIdx.x, gridDim.x, lane);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb0);
      if (EPI == EPI_SWIGLU || p.seg1 < p.n_tiles) prefetch_tmap(&tb1);
      if (EPI == EPI_STORE && p.seg2 < p.n_tiles) prefetch_tmap(&tb2);
      const uint64_t pol_w = policy_evict_first();  // weights are streamed once per tile row
      const uint64_t pol_a = policy_evict_last();   // activations are re-read by every n-tile
      auto load_b = [&](int stage, int nt, int kb) {
        uint8_t* sb = ring_b + stage * S::B_BYTES;
        if constexpr (EPI == EPI_SWIGLU) {
          tma_load_2d_hint(sb, &tb0, &full[stage], kb * BK, nt * (BN / 2), pol_w);
          tma_load_2d_hint(sb + (BN / 2) * 128, &tb1, &full[stage], kb * BK, nt * (BN / 2), pol_w);
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_load_2d_hint(sb, tb, &full[stage], kb * BK, row0, pol_w);
        }
      };
      auto prefetch_b = [&](int nt, int kb) {
        if constexpr (EPI == EPI_SWIGLU) {
          tma_prefetch_2d(&tb0, kb * BK, nt * (BN / 2));
          tma_prefetch_2d(&tb1, kb * BK, nt * (BN / 2));
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_prefetch_2d(tb, kb * BK, row0);
        }
      };
      // Pull the first tile's weight tiles into L2 while the previous kernel finishes; shared
      // memory is only written after griddepcontrol.wait (a weight written by that kernel could
      // still be in flight), so the ring fills from L2 right after it.
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < total_tiles) {
        int mt0, nt0;
        tile_coords(blockIdx.x, p, mt0, nt0);
        pre = min(STAGES, p.num_kb);
        if (!p.weights_prefetch) {
          for (int kb = 0; kb < pre; ++kb) prefetch_b(nt0, kb);
          pdl_wait();
        }
        for (int kb = 0; kb < pre; ++kb) {
          mbar_arrive_expect_tx(&full[kb], S::A_BYTES + S::B_BYTES);
          load_b(kb, nt0, kb);
        }
        if (p.weights_prefetch) pdl_wait();
      } else {
        pdl_wait();
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int mt, nt;
        tile_coords(t, p, mt, nt);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(t == static_cast<int>(blockIdx.x) && kb < pre)) {
            if (!mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], S::A_BYTES + S::B_BYTES);
            load_b(stage, nt, kb);
          }
          tma_load_2d_hint(ring_a + stage * S::A_BYTES, &ta, &full[stage], kb * BK, mt * BM, pol_a);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(Dt<DT>::umma_fmt, BM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int i = 0;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(ring_a + stage * S::A_BYTES);
          const uint32_t b0 = smem_u32(ring_b + stage * S::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = make_sw128_desc(a0 + kk * 32, 0, 1024);
            const uint64_t bd = make_sw128_desc(b0 + kk * 32, 0, 1024);
            umma_f16_ss(d, ad, bd, idesc, (kb | kk) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int i = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++i) {
      int mt, nt;
      tile_coords(t, p, mt, nt);
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int row = mt * BM + row_in_tile;
      const float rs = row_rstd(p, row);
      if constexpr (EPI == EPI_SWIGLU && BN / 2 < 32) {
        // 16 gate columns followed by 16 up columns
        float g[32], u[16];
        tmem_load16x2(taddr, taddr + BN / 2, g, u);
#pragma unroll
        for (int j = 0; j < 16; ++j) g[j] = swiglu_f(g[j] * rs, u[j] * rs);
        if (row < p.m) store_row16<DT>(p.y, p.ldy, row, nt * (BN / 2), p.n, g);
      } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float g[32], u[32];
          tmem_load32x2(taddr + c, taddr + BN / 2 + c, g, u);
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = swiglu_f(g[j] * rs, u[j] * rs);
          if (row < p.m) store_row32<DT>(p.y, p.ldy, row, nt * (BN / 2) + c, p.n, g, nullptr);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_load32(taddr + c, v);
          scale32(v, rs);
          if (nt * BN + c < p.rope_cols) rope_chunk32<DT>(v, row, nt * BN + c, p);
          if (row < p.m) store_row32<DT>(p.y, p.ldy, row, nt * BN + c, p.n, v, p.residual, ssq_slot(p, row, nt * BN + c));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// 2-SM variant for large problems: a cluster of two CTAs (a pair) computes one
// 256 x BN output tile with tcgen05.mma.cta_group::2. Each CTA holds 128 rows of
// the A tile and BN/2 rows of the B tile in its own shared memory, so per flop a
// CTA pulls 2/3 of the operand bytes a 1-SM 128 x BN tile needs - the 1-SM kernel
// is bound by L2->SM bandwidth at large M. Both CTAs' TMA loads count on the
// leader's full barrier; the leader's single MMA thread commits to barriers in
// both CTAs (multicast commit); each CTA's epilogue drains its own 128 TMEM lanes
// and both release the accumulator on the leader's barrier. For the SwiGLU
// epilogue rank 0 loads the gate rows and rank 1 the matching up rows, so every
// accumulator holds gate in columns [0, BN/2) and up in [BN/2, BN).
// ---------------------------------------------------------------------------------
template <int BN, int STAGES>
struct PairSmem {
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int RING = STAGES * STAGE;
  static constexpr int NUM_BARS = 2 * STAGES + 4;
  static constexpr int TOTAL = 1024 + RING + NUM_BARS * 8 + 16;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
};

constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;  // shared::cluster address of the same offset in the pair leader

template <int DT, int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(PAIR_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                     const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tb2, const Params p) {
  using S = PairSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::RING);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::NUM_BARS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());  // 0: leader, 1: follower
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int total_tiles = p.m_tiles * p.n_tiles;  // m_tiles counts 256-row tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * PAIR_EPI_WARPS);  // every epilogue warp of both CTAs of the pair
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  cluster_sync();  // both CTAs' barriers and TMEM exist before any cross-CTA signal
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 3 && p.pf.n) l2_prefetch_share(p.pf, blockIdx.x, gridDim.x, lane);

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb0);
      if (EPI == EPI_SWIGLU || p.seg1 < p.n_tiles) prefetch_tmap(&tb1);
      if (EPI == EPI_STORE && p.seg2 < p.n_tiles) prefetch_tmap(&tb2);
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      auto full_bar = [&](int stage) { return smem_u32(&full[stage]) & kPeerBitMask; };
      auto load_b = [&](int stage, int nt, int kb) {
        uint8_t* sb = ring + stage * S::STAGE + S::A_BYTES;
        if constexpr (EPI == EPI_SWIGLU) {
          tma_load_2d_pair(sb, rank == 0 ? &tb0 : &tb1, full_bar(stage), kb * BK, nt * (BN / 2), pol_w);
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_load_2d_pair(sb, tb, full_bar(stage), kb * BK, row0 + rank * (BN / 2), pol_w);
        }
      };
      auto prefetch_b = [&](int nt, int kb) {
        if constexpr (EPI == EPI_SWIGLU) {
          tma_prefetch_2d(rank == 0 ? &tb0 : &tb1, kb * BK, nt * (BN / 2));
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_prefetch_2d(tb, kb * BK, row0 + rank * (BN / 2));
        }
      };
      // weight tiles into L2 before the wait, into shared memory after it (see gemm_kernel)
      int pre = 0;
      if (pair < total_tiles) {
        int mt0, nt0;
        tile_coords(pair, p, mt0, nt0);
        pre = min(STAGES, p.num_kb);
        if (!p.weights_prefetch) {
          for (int kb = 0; kb < pre; ++kb) prefetch_b(nt0, kb);
          pdl_wait();
        }
        for (int kb = 0; kb < pre; ++kb) {
          if (rank == 0) mbar_arrive_expect_tx(&full[kb], 2 * S::STAGE);
          load_b(kb, nt0, kb);
        }
        if (p.weights_prefetch) pdl_wait();
      } else {
        pdl_wait();
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < total_tiles && ok; t += npairs) {
        int mt, nt;
        tile_coords(t, p, mt, nt);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(t == pair && kb < pre)) {
            if (!mbar_wait(&empty[stage], phase ^ 1)) { ok = false; break; }
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * S::STAGE);
            load_b(stage, nt, kb);
          }
          tma_load_2d_pair(ring + stage * S::STAGE, &ta, full_bar(stage), kb * BK, mt * 256 + rank * 128, pol_a);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(Dt<DT>::umma_fmt, 256, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int i = 0;
      for (int t = pair; t < total_tiles && ok; t += npairs, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(ring + stage * S::STAGE);
          const uint32_t b0 = a0 + S::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_ss_pair(d, make_sw128_desc(a0 + kk * 32, 0, 1024), make_sw128_desc(b0 + kk * 32, 0, 1024),
                             idesc, (kb | kk) != 0);
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit_pair(&tfull[acc], 0x3);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) / 4;  // which half of the tile's columns this warp stores
    const int row_in_tile = rank * 128 + quarter * 32 + lane;
    const uint32_t tempty_leader = smem_u32(&tempty[0]) & kPeerBitMask;
    int i = 0;
    for (int t = pair; t < total_tiles; t += npairs, ++i) {
      int mt, nt;
      tile_coords(t, p, mt, nt);
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int row = mt * 256 + row_in_tile;
      const float rs = row_rstd(p, row);
      if constexpr (EPI == EPI_SWIGLU) {
        static_assert(BN % 128 == 0, "each half of the SwiGLU columns must be whole 32-column chunks");
#pragma unroll 1
        for (int c = half * (BN / 4); c < (half + 1) * (BN / 4); c += 32) {
          float g[32], u[32];
          tmem_load32x2(taddr + c, taddr + BN / 2 + c, g, u);
#pragma unroll
          for (int j = 0; j < 32; ++j) g[j] = swiglu_f(g[j] * rs, u[j] * rs);
          if (row < p.m) store_row32<DT>(p.y, p.ldy, row, nt * (BN / 2) + c, p.n, g, nullptr);
        }
      } else {
        static_assert(BN % 64 == 0, "each half of the columns must be whole 32-column chunks");
#pragma unroll 1
        for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
          float v[32];
          tmem_load32(taddr + c, v);
          scale32(v, rs);
          if (nt * BN + c < p.rope_cols) rope_chunk32<DT>(v, row, nt * BN + c, p);
          if (row < p.m) store_row32<DT>(p.y, p.ldy, row, nt * BN + c, p.n, v, p.residual, ssq_slot(p, row, nt * BN + c));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&tempty[acc]);
        else mbar_arrive_remote(tempty_leader + acc * 8);
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // every MMA, every epilogue and every remote arrival of the pair is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// Split-K variant for few output tiles (weight streaming at M <= a few hundred).
//
// A cluster of `split` CTAs shares one output tile; CTA r of the cluster runs
// k-blocks [r*num_kb/split, (r+1)*num_kb/split) into its own TMEM accumulator,
// so each CTA streams 1/split of the activation block and of the weight tile.
// The partial sums are then reduced through distributed shared memory: the 128
// rows are owned in groups of 16 (group g -> CTA g % split); every CTA writes
// the rows it does not own into the owner's receive buffer (st.shared::cluster),
// and after a cluster barrier each owner adds the partials to its own and runs
// the epilogue (SwiGLU / residual / store) for its rows.
// ---------------------------------------------------------------------------------
template <int BN>
struct SplitSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int ROW_F = BN + 4;  // padded fp32 row of the receive buffer (no bank conflicts)
  static constexpr int MAX_STAGES = 8;
  static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  __host__ __device__ static constexpr int rows_owned_max(int split) {
    return split > 1 ? ((8 + split - 1) / split) * 16 : 0;
  }
  __host__ __device__ static constexpr int recv_bytes(int split) {
    return split > 1 ? (split - 1) * rows_owned_max(split) * ROW_F * 4 : 0;
  }
  __host__ __device__ static constexpr int bar_off(int split, int stages) { return stages * STAGE + recv_bytes(split); }
  __host__ __device__ static constexpr int total(int split, int stages) {
    return 1024 + bar_off(split, stages) + (2 * MAX_STAGES + 2) * 8 + 16;
  }
};

template <int DT, int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_splitk_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                       const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tb2,
                       const Params p, const int split, const int stages) {
  using S = SplitSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* recv = reinterpret_cast<float*>(smem + stages * S::STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bar_off(split, stages));
  uint64_t* full = bars;
  uint64_t* empty = bars + S::MAX_STAGES;
  uint64_t* tfull = bars + 2 * S::MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S::MAX_STAGES + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int nt = blockIdx.y;
  const int mt = blockIdx.z;
  const int kb0 = (rank * p.num_kb) / split;
  const int kb1 = ((rank + 1) * p.num_kb) / split;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  cluster_sync();  // every CTA of the cluster is running before any remote shared-memory write
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 3 && p.pf.n)
    l2_prefetch_share(p.pf, blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z),
                      gridDim.x * gridDim.y * gridDim.z, lane);

  if (warp == 0) {
    if (elect_one()) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb0);
      if (EPI == EPI_SWIGLU || p.seg1 < p.n_tiles) prefetch_tmap(&tb1);
      if (EPI == EPI_STORE && p.seg2 < p.n_tiles) prefetch_tmap(&tb2);
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      auto load_b = [&](int stage, int kb) {
        uint8_t* sb = ring + stage * S::STAGE + S::A_BYTES;
        if constexpr (EPI == EPI_SWIGLU) {
          tma_load_2d_hint(sb, &tb0, &full[stage], kb * BK, nt * (BN / 2), pol_w);
          tma_load_2d_hint(sb + (BN / 2) * 128, &tb1, &full[stage], kb * BK, nt * (BN / 2), pol_w);
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_load_2d_hint(sb, tb, &full[stage], kb * BK, row0, pol_w);
        }
      };
      // weight tiles into L2 before the wait, into shared memory after it (see gemm_kernel)
      const int pre = min(stages, kb1 - kb0);
      for (int i = 0; i < pre && !p.weights_prefetch; ++i) {
        const int kb = kb0 + i;
        if constexpr (EPI == EPI_SWIGLU) {
          tma_prefetch_2d(&tb0, kb * BK, nt * (BN / 2));
          tma_prefetch_2d(&tb1, kb * BK, nt * (BN / 2));
        } else {
          const CUtensorMap* tb = nt < p.seg1 ? &tb0 : (nt < p.seg2 ? &tb1 : &tb2);
          const int row0 = nt < p.seg1 ? nt * BN : (nt < p.seg2 ? (nt - p.seg1) * BN : (nt - p.seg2) * BN);
          tma_prefetch_2d(tb, kb * BK, row0);
        }
      }
      if (!p.weights_prefetch) pdl_wait();
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], S::STAGE);
        load_b(i, kb0 + i);
      }
      if (p.weights_prefetch) pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (kb - kb0 >= pre) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) break;
          mbar_arrive_expect_tx(&full[stage], S::STAGE);
          load_b(stage, kb);
        }
        tma_load_2d_hint(ring + stage * S::STAGE, &ta, &full[stage], kb * BK, mt * BM, pol_a);
        if (++stage == stages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_f16(Dt<DT>::umma_fmt, BM, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(ring + stage * S::STAGE);
        const uint32_t b0 = a0 + S::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16_ss(tmem_base, make_sw128_desc(a0 + kk * 32, 0, 1024), make_sw128_desc(b0 + kk * 32, 0, 1024),
                      idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == stages) { stage = 0; phase ^= 1; }
      }
      if (ok) umma_commit(tfull);
    }
  }

  // epilogue warps: send the rows other CTAs own (tcgen05.ld is warp-wide, so a warp
  // loads whenever any of its lanes needs its row)
  const int quarter = warp & 3;
  const int group = quarter * 2 + (lane >> 4);  // 16-row group of this lane's row
  const int owner = group % split;
  const int local_row = (group / split) * 16 + (lane & 15);
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  bool have_acc = false;
  if (warp >= 2) {
    have_acc = mbar_wait(tfull, 0);
    tc_fence_after();
    if (have_acc && __any_sync(0xffffffffu, owner != rank)) {
      const int slot = rank < owner ? rank : rank - 1;
      const uint32_t remote =
          mapa_shared(smem_u32(recv + (slot * S::rows_owned_max(split) + local_row) * S::ROW_F), owner);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_load32(taddr + c, v);
        if (owner != rank) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_cluster_v4(remote + (c + 4 * j) * 4, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
    }
  }
  cluster_sync();  // all partials have landed in their owners' receive buffers

  if (warp >= 2 && have_acc && __any_sync(0xffffffffu, owner == rank)) {
    const bool mine = owner == rank;
    const int row = mt * BM + quarter * 32 + lane;
    const float rs = row_rstd(p, row);
    const float* rbase = recv + local_row * S::ROW_F;
    const int rstride = S::rows_owned_max(split) * S::ROW_F;
    if constexpr (EPI == EPI_SWIGLU && BN / 2 < 32) {
      float g[32], u[16];
      tmem_load16x2(taddr, taddr + BN / 2, g, u);
      for (int s2 = 0; mine && s2 < split - 1; ++s2) {
        const float* r = rbase + s2 * rstride;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          g[j] += r[j];
          u[j] += r[BN / 2 + j];
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) g[j] = swiglu_f(g[j] * rs, u[j] * rs);
      if (mine && row < p.m) store_row16<DT>(p.y, p.ldy, row, nt * (BN / 2), p.n, g);
    } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
      for (int c = 0; c < BN / 2; c += 32) {
        float g[32], u[32];
        tmem_load32x2(taddr + c, taddr + BN / 2 + c, g, u);
        for (int s2 = 0; mine && s2 < split - 1; ++s2) {
          const float4* rg = reinterpret_cast<const float4*>(rbase + s2 * rstride + c);
          const float4* ru = reinterpret_cast<const float4*>(rbase + s2 * rstride + BN / 2 + c);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 a = rg[j], b = ru[j];
            g[4 * j] += a.x; g[4 * j + 1] += a.y; g[4 * j + 2] += a.z; g[4 * j + 3] += a.w;
            u[4 * j] += b.x; u[4 * j + 1] += b.y; u[4 * j + 2] += b.z; u[4 * j + 3] += b.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) g[j] = swiglu_f(g[j] * rs, u[j] * rs);
        if (mine && row < p.m) store_row32<DT>(p.y, p.ldy, row, nt * (BN / 2) + c, p.n, g, nullptr);
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_load32(taddr + c, v);
        for (int s2 = 0; mine && s2 < split - 1; ++s2) {
          const float4* r = reinterpret_cast<const float4*>(rbase + s2 * rstride + c);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 a = r[j];
            v[4 * j] += a.x; v[4 * j + 1] += a.y; v[4 * j + 2] += a.z; v[4 * j + 3] += a.w;
          }
        }
        scale32(v, rs);
        if (mine && nt * BN + c < p.rope_cols) rope_chunk32<DT>(v, row, nt * BN + c, p);
        if (mine && row < p.m)
          store_row32<DT>(p.y, p.ldy, row, nt * BN + c, p.n, v, p.residual, ssq_slot(p, row, nt * BN + c));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------

// Plan limits, checked on the host before every launch of the three GEMM kernels.
// TMEM: a CTA's columns times the CTAs that can share an SM (by shared memory, threads
// and registers) stay within the SM's 512 columns, so a tcgen05.alloc never waits for
// columns held by another CTA - a CTA blocked in its alloc while its cluster peers wait
// for it at a cluster barrier, and the columns' owners wait for theirs, would never
// finish. Cached per (kernel, shared memory, device).
template <typename... KArgs>
static int check_tmem_residency(void (*kern)(KArgs...), int threads, size_t smem, uint32_t cols, const char* what) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, size_t, int>, int> cache;
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kern), smem, dev.device);
  int resident = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) resident = it->second;
  }
  if (!resident) {
    if (int rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, threads, smem),
                            "cudaOccupancyMaxActiveBlocksPerMultiprocessor(gemm)"))
      return rc;
    if (resident < 1) return set_error(TK_ERR_UNSUPPORTED, std::string(what) + ": the plan does not fit on an SM");
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = resident;
  }
  if (static_cast<uint64_t>(resident) * cols > 512u)
    return set_error(TK_ERR_UNSUPPORTED, std::string(what) + ": " + std::to_string(resident) +
                                             " resident CTAs x " + std::to_string(cols) +
                                             " TMEM columns exceed the SM's 512");
  return TK_OK;
}

// Split-K plan limits: every CTA of a cluster accumulates at least one k-block (a CTA without
// one would add an unwritten accumulator to the others), clusters of at most 8 CTAs (the
// portable size), a ring that fits the barrier array, and shared memory within the device's
// opt-in limit.
static int check_splitk_plan(int split, int stages, int num_kb, size_t smem, size_t smem_cap) {
  if (split < 1 || split > 8 || split > num_kb)
    return set_error(TK_ERR_UNSUPPORTED, "gemm split-K plan: split " + std::to_string(split) + " for " +
                                             std::to_string(num_kb) + " k-blocks (must be 1..min(8, k-blocks))");
  if (stages < 1 || stages > SplitSmem<32>::MAX_STAGES)
    return set_error(TK_ERR_UNSUPPORTED, "gemm split-K plan: " + std::to_string(stages) + " ring stages");
  if (smem > smem_cap)
    return set_error(TK_ERR_UNSUPPORTED, "gemm split-K plan: " + std::to_string(smem) +
                                             " bytes of shared memory exceed the device limit");
  return TK_OK;
}

template <int DT, int BN, int EPI, int STAGES>
int launch(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const CUtensorMap& tb2,
           const Params& p, int ctas_per_sm, cudaStream_t st) {
  using S = Smem<BN, STAGES>;
  auto kern = gemm_kernel<DT, BN, EPI, STAGES>;
  static bool configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!configured[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL),
                            "cudaFuncSetAttribute(gemm)"))
      return rc;
    configured[dev.device] = true;
  }
  if (int rc = check_tmem_residency(kern, THREADS, S::TOTAL, S::TMEM_COLS, "gemm_kernel")) return rc;
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = std::max(1, std::min(tiles, dev.sm_count * ctas_per_sm));
  return launch_kernel(kern, dim3(grid), dim3(THREADS), S::TOTAL, st, 1, "gemm_kernel", ta, tb0, tb1, tb2, p);
}

template <int DT, int BN, int EPI, int STAGES>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const CUtensorMap& tb2,
                const Params& p, cudaStream_t st) {
  using S = PairSmem<BN, STAGES>;
  auto kern = gemm_pair_kernel<DT, BN, EPI, STAGES>;
  static int max_pairs[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!max_pairs[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL),
                            "cudaFuncSetAttribute(gemm_pair)"))
      return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(PAIR_THREADS);
    cfg.dynamicSmemBytes = S::TOTAL;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (int rc = check_cuda(cudaOccupancyMaxActiveClusters(&n, kern, &cfg), "cudaOccupancyMaxActiveClusters")) return rc;
    max_pairs[dev.device] = std::max(1, n);
  }
  if (int rc = check_tmem_residency(kern, PAIR_THREADS, S::TOTAL, S::TMEM_COLS, "gemm_pair_kernel")) return rc;
  const int tiles = p.m_tiles * p.n_tiles;
  const int pairs = std::max(1, std::min(tiles, max_pairs[dev.device]));
  return launch_kernel(kern, dim3(2 * pairs), dim3(PAIR_THREADS), S::TOTAL, st, 2, "gemm_pair_kernel", ta, tb0, tb1, tb2,
                       p);
}

// Pair (2-SM) tiles pay off once there are enough 256-row tiles to keep every SM pair busy.
static bool use_pair(int64_t m, int64_t n_tiles, int sms) { return m >= 512 && ((m + 255) / 256) * n_tiles >= sms / 2; }

template <int DT, int BN, int EPI>
int launch_splitk(const CUtensorMap& ta, const CUtensorMap& tb0, const CUtensorMap& tb1, const CUtensorMap& tb2,
                  const Params& p, int split, int stages, cudaStream_t st) {
  using S = SplitSmem<BN>;
  auto kern = gemm_splitk_kernel<DT, BN, EPI>;
  static bool configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!configured[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(dev.smem_optin)),
                            "cudaFuncSetAttribute(gemm_splitk)"))
      return rc;
    configured[dev.device] = true;
  }
  const size_t smem = S::total(split, stages);
  if (int rc = check_splitk_plan(split, stages, p.num_kb, smem, dev.smem_optin)) return rc;
  if (int rc = check_tmem_residency(kern, THREADS, smem, S::TMEM_COLS, "gemm_splitk_kernel")) return rc;
  return launch_kernel(kern, dim3(split, p.n_tiles, p.m_tiles), dim3(THREADS), smem, st, split,
                       "gemm_splitk_kernel", ta, tb0, tb1, tb2, p, split, stages);
}

// Tile plan for problems with few output tiles: split K over a cluster of `split`
// CTAs when that keeps all CTAs in one wave and cuts the bytes each CTA must pull.
constexpr int DEEP_STAGES = 8;  // ring of the single-wave plain kernel (see plan_small_m)
struct SmallPlan {
  int bn = 0, split = 1, stages = 4;
};
static int splitk_smem(int bn, int split, int stages) {
  switch (bn) {
    case 256: return SplitSmem<256>::total(split, stages);
    case 128: return SplitSmem<128>::total(split, stages);
    case 64: return SplitSmem<64>::total(split, stages);
    default: return SplitSmem<32>::total(split, stages);
  }
}
// How many clusters of `split` CTAs of the split-K kernel can be resident at once
// with `smem` bytes of shared memory each (queried once per configuration).
template <int DT, int EPI>
static int max_active_clusters(int bn, int split, int smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  DeviceInfo dev;
  if (current_device_info(&dev)) return 0;
  const auto key = std::make_tuple(dev.device, bn, split, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  void (*kern)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Params, int, int) =
      bn == 64 ? gemm_splitk_kernel<DT, 64, EPI> : gemm_splitk_kernel<DT, 32, EPI>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dev.smem_optin)) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split, 1, 1);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

// Cost model (µs) for a CTA's critical path at M <= a few hundred rows on B200, fitted to A/B timings
// of the 268M decoder's projections at 128 rows inside its CUDA graph: ~1.8 of set-up and first
// load; ~1.0 per round trip of the ring (at these sizes a k-block's TMA round trip from L2 costs
// more than its transfer, so a CTA's stream takes ceil(k-blocks / stages) round trips) plus the
// bytes at ~200 GB/s per SM; for split > 1 a DSMEM reduction of ~0.5 + 0.35 per extra CTA of
// the cluster + (partial bytes sent) / 25 GB/s; an owner epilogue that grows with BN. Plans of one
// wave with one CTA per SM get a deep ring (8 stages, split-K: as many as the CTA's k-blocks);
// other split-K plans <= 4 stages (two CTAs per SM) and must fit in one wave of co-resident
// clusters. Splits stay <= 4 and BN <= 64; splits are tried from the largest down, and a later
// candidate must be 3 % cheaper to replace an earlier one.
// Measured against the earlier bandwidth-only model: o_proj at 128 rows moves from split 4 to
// split 2 (one round trip either way, half the exchange partners): 564 -> 548 us per forward.
template <int DT, int EPI>
static SmallPlan plan_small_m(int64_t m_tiles, int64_t n_out, int num_kb, int sms, int64_t constraint,
                              size_t smem_cap) {
  constexpr bool swiglu = EPI == EPI_SWIGLU;
  SmallPlan best;
  double best_cost = 1e30;
  static const int bns[] = {64, 32};
  for (int bn : bns) {
    const int64_t per_tile_n = swiglu ? bn / 2 : bn;
    if (!swiglu && constraint % bn != 0) continue;
    const int64_t n_tiles = (n_out + per_tile_n - 1) / per_tile_n;
    const int64_t tiles = m_tiles * n_tiles;
    for (int split = 4; split >= 1; --split) {
      if (split > num_kb) continue;
      const int64_t ctas = tiles * split;
      const int kb = (num_kb + split - 1) / split;  // k-blocks of the busiest CTA
      const bool one_wave = ctas <= sms;
      int stages = 0;
      if (split > 1) {
        const int want = std::min(4, kb);
        for (int s = want; s >= 2; --s)
          if (static_cast<size_t>(splitk_smem(bn, split, s)) <= smem_cap) { stages = s; break; }
        if (stages < std::min(want, 3)) continue;
        if (tiles > max_active_clusters<DT, EPI>(bn, split, splitk_smem(bn, split, stages)))
          continue;  // the split kernel must run in one wave
        if (one_wave && kb > stages) {
          const int deep = std::min(SplitSmem<32>::MAX_STAGES, kb);
          const int smem = splitk_smem(bn, split, deep);
          if (static_cast<size_t>(smem) <= smem_cap && tiles <= max_active_clusters<DT, EPI>(bn, split, smem))
            stages = deep;
        }
      } else {
        stages = one_wave && kb > 4 ? DEEP_STAGES : 4;
      }
      const int trips = (kb + stages - 1) / stages;
      const double load = double(kb) * (BM * BK * 2 + bn * BK * 2);
      const double red = split > 1 ? 128.0 * bn * 4 * (split - 1) / split : 0.0;
      const double per_sm = split > 1 ? std::max(1.0, double(ctas) / sms) : double((ctas + sms - 1) / sms);
      const double cost = 1.8 + per_sm * (trips * 1.0 + load / 200e3) +
                          (split > 1 ? 0.5 + 0.35 * (split - 1) + red / 25e3 : 0.0) + 0.25 * bn / 32;
      if (cost < best_cost * 0.97) {
        best_cost = cost;
        best.bn = bn;
        best.split = split;
        best.stages = stages;
      }
    }
  }
  return best;
}

// Largest BN (from the candidates) whose tile count still fills the GPU, else the
// smallest: few, fat tiles when M is large; many thin tiles for weight streaming.
static int pick_bn(int64_t m_tiles, int64_t n, int sms, const int* cands, int ncand, int64_t div_constraint) {
  for (int i = 0; i < ncand; ++i) {
    const int bn = cands[i];
    if (div_constraint % bn != 0) continue;
    const int64_t tiles = m_tiles * ((n + bn - 1) / bn);
    if (tiles >= sms) return bn;
  }
  for (int i = ncand - 1; i >= 0; --i)
    if (div_constraint % cands[i] == 0) return cands[i];
  return 0;
}

// Epilogue options beyond the plain store (see tk_epilogue in the header).
struct Extras {
  const void* residual = nullptr;
  int rope_cols = 0, rope_seq = 1, rope_start = 0, rope_half_d = 0;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  const float* ssq_in = nullptr;
  int ssq_parts = 0;
  float ssq_inv_k = 0.f, ssq_eps = 0.f;
  float* ssq_out = nullptr;
  int weights_prefetch = 0;
  L2Prefetch pf{};
};

void apply_extras(Params& p, const Extras& e) {
  p.residual = e.residual;
  p.rope_cols = e.rope_cols;
  p.rope_seq = e.rope_seq;
  p.rope_start = e.rope_start;
  p.rope_half_d = e.rope_half_d;
  p.rope_cos = e.rope_cos;
  p.rope_sin = e.rope_sin;
  p.ssq_in = e.ssq_in;
  p.ssq_parts = e.ssq_parts;
  p.ssq_inv_k = e.ssq_inv_k;
  p.ssq_eps = e.ssq_eps;
  p.ssq_out = e.ssq_out;
  p.weights_prefetch = e.weights_prefetch;
  p.pf = e.pf;
}

template <int DT>
int run_linear(const void* x, int64_t lda, const void* w0, int64_t n0, const void* w1, int64_t n1, const void* w2,
               int64_t n2, void* y, int64_t ldy, int64_t m, int64_t k, cudaStream_t st, const Extras& ex) {
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  const int64_t n = n0 + n1 + n2;
  if (m <= gemv::MAX_M && ex.rope_cols == 0) {  // a few rows: stream the weights once (gemv.cu)
    const void* w[3] = {w0, n1 ? w1 : nullptr, n2 ? w2 : nullptr};
    const int64_t nr[3] = {n0, n1, n2};
    return gemv::run(DT, x, lda, w, nr, false, y, ldy, m, n, k, ex.residual, ex.ssq_in, ex.ssq_parts, ex.ssq_inv_k,
                     ex.ssq_eps, ex.ssq_out, st);
  }
  const int64_t m_tiles = (m + BM - 1) / BM;
  // all but the last weight block must be whole tiles
  const int64_t constraint = (n1 || n2) ? std::gcd(n0, n1 ? n1 : n0) : 256;
  static const int cands[] = {256, 128, 64, 32};
  int bn = pick_bn(m_tiles, n, dev.sm_count, cands, 4, constraint);
  if (bn == 0) return fail_invalid("linear: weight block sizes must be multiples of 32");
  SmallPlan plan;
  // One M tile and a wide weight (an LM head: 32000 x 1024 at 128 rows) whose 256-column tiles
  // fill most of the SMs once: one round of wide tiles streams the weight at the HBM rate,
  // where 128-column tiles would take two uneven rounds and narrower ones re-read the
  // activation block from L2 once per tile.
  const int64_t wide_tiles = (n + 255) / 256;
  const bool one_wide_round = m_tiles == 1 && constraint % 256 == 0 && 4 * wide_tiles >= 3 * dev.sm_count &&
                              wide_tiles <= dev.sm_count;
  if (one_wide_round) {
    bn = 256;
  } else if (m_tiles <= 2 || m_tiles * ((n + bn - 1) / bn) < dev.sm_count) {
    plan = plan_small_m<DT, EPI_STORE>(m_tiles, n, static_cast<int>((k + BK - 1) / BK), dev.sm_count, constraint,
                                       dev.smem_optin);
    if (plan.bn) bn = plan.bn;
  }
  Params p{};
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.num_kb = static_cast<int>((k + BK - 1) / BK);
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>((n + bn - 1) / bn);
  p.seg1 = n1 || n2 ? static_cast<int>(n0 / bn) : p.n_tiles;
  p.seg2 = n2 ? static_cast<int>((n0 + n1) / bn) : p.n_tiles;
  p.y = y;
  p.ldy = ldy;
  apply_extras(p, ex);
  CUtensorMap ta, tb0, tb1, tb2;
  if (int rc = tensor_map_2d(&ta, x, DT, m, k, lda, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&tb0, w0, DT, n0, k, k, bn, BK)) return rc;
  tb1 = tb0;
  tb2 = tb0;
  if (n1)
    if (int rc = tensor_map_2d(&tb1, w1, DT, n1, k, k, bn, BK)) return rc;
  if (n2)
    if (int rc = tensor_map_2d(&tb2, w2, DT, n2, k, k, bn, BK)) return rc;
  // 2-SM pair tiles (256 rows) for large M: BN 256 when the weight blocks allow it, else 128
  {
    const int pbn = (constraint % 256 == 0 && n >= 1024) ? 256 : (constraint % 128 == 0 ? 128 : 0);
    if (pbn && plan.split <= 1 && use_pair(m, (n + pbn - 1) / pbn, dev.sm_count)) {
      Params q = p;
      q.m_tiles = static_cast<int>((m + 255) / 256);
      q.n_tiles = static_cast<int>((n + pbn - 1) / pbn);
      q.seg1 = n1 || n2 ? static_cast<int>(n0 / pbn) : q.n_tiles;
      q.seg2 = n2 ? static_cast<int>((n0 + n1) / pbn) : q.n_tiles;
      CUtensorMap pa, pb0, pb1, pb2;
      if (int rc = tensor_map_2d(&pa, x, DT, m, k, lda, 128, BK)) return rc;
      if (int rc = tensor_map_2d(&pb0, w0, DT, n0, k, k, pbn / 2, BK)) return rc;
      pb1 = pb0;
      pb2 = pb0;
      if (n1)
        if (int rc = tensor_map_2d(&pb1, w1, DT, n1, k, k, pbn / 2, BK)) return rc;
      if (n2)
        if (int rc = tensor_map_2d(&pb2, w2, DT, n2, k, k, pbn / 2, BK)) return rc;
      if (pbn == 256) return launch_pair<DT, 256, EPI_STORE, 6>(pa, pb0, pb1, pb2, q, st);
      return launch_pair<DT, 128, EPI_STORE, 8>(pa, pb0, pb1, pb2, q, st);
    }
  }
  if (plan.split > 1) {
    switch (bn) {
      case 256: return launch_splitk<DT, 256, EPI_STORE>(ta, tb0, tb1, tb2, p, plan.split, plan.stages, st);
      case 128: return launch_splitk<DT, 128, EPI_STORE>(ta, tb0, tb1, tb2, p, plan.split, plan.stages, st);
      case 64: return launch_splitk<DT, 64, EPI_STORE>(ta, tb0, tb1, tb2, p, plan.split, plan.stages, st);
      default: return launch_splitk<DT, 32, EPI_STORE>(ta, tb0, tb1, tb2, p, plan.split, plan.stages, st);
    }
  }
  switch (bn) {
    case 256: return launch<DT, 256, EPI_STORE, 4>(ta, tb0, tb1, tb2, p, 1, st);
    case 128: return launch<DT, 128, EPI_STORE, 5>(ta, tb0, tb1, tb2, p, 1, st);
    case 64:
      if (plan.stages == DEEP_STAGES) return launch<DT, 64, EPI_STORE, DEEP_STAGES>(ta, tb0, tb1, tb2, p, 1, st);
      return launch<DT, 64, EPI_STORE, 4>(ta, tb0, tb1, tb2, p, 2, st);
    default:
      if (plan.stages == DEEP_STAGES) return launch<DT, 32, EPI_STORE, DEEP_STAGES>(ta, tb0, tb1, tb2, p, 1, st);
      return launch<DT, 32, EPI_STORE, 4>(ta, tb0, tb1, tb2, p, 2, st);
  }
}

template <int DT>
int run_gate_up(const void* x, int64_t lda, const void* wg, const void* wu, void* h, int64_t m, int64_t hidden,
                int64_t f, cudaStream_t st, const Extras& ex) {
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (m <= gemv::MAX_M) {  // a few rows: stream the weights once (gemv.cu)
    const void* w[3] = {wg, wu, nullptr};
    const int64_t nr[3] = {f, f, 0};
    return gemv::run(DT, x, lda, w, nr, true, h, f, m, f, hidden, nullptr, ex.ssq_in, ex.ssq_parts, ex.ssq_inv_k,
                     ex.ssq_eps, nullptr, st);
  }
  const int64_t m_tiles = (m + BM - 1) / BM;
  // BN counts gate + up rows; each tile produces BN/2 columns of h
  static const int cands_half[] = {128, 64, 32, 16};
  int half = 0;
  for (int c : cands_half)
    if (m_tiles * ((f + c - 1) / c) >= dev.sm_count) { half = c; break; }
  SmallPlan plan;
  if (!half) half = 16;
  if (m_tiles <= 2 || m_tiles * ((f + half - 1) / half) < dev.sm_count) {
    plan = plan_small_m<DT, EPI_SWIGLU>(m_tiles, f, static_cast<int>((hidden + BK - 1) / BK), dev.sm_count, 1,
                                        dev.smem_optin);
    if (plan.bn) half = plan.bn / 2;
  }
  if (use_pair(m, (f + 127) / 128, dev.sm_count)) {
    // pair tiles: rank 0 loads 128 gate rows, rank 1 the same 128 up rows
    Params q{};
    q.m = static_cast<int>(m);
    q.n = static_cast<int>(f);
    q.k = static_cast<int>(hidden);
    q.num_kb = static_cast<int>((hidden + BK - 1) / BK);
    q.m_tiles = static_cast<int>((m + 255) / 256);
    q.n_tiles = static_cast<int>((f + 127) / 128);
    q.seg1 = q.seg2 = q.n_tiles;
    q.y = h;
    q.ldy = f;
    apply_extras(q, ex);
    CUtensorMap pa, pg, pu;
    if (int rc = tensor_map_2d(&pa, x, DT, m, hidden, lda, 128, BK)) return rc;
    if (int rc = tensor_map_2d(&pg, wg, DT, f, hidden, hidden, 128, BK)) return rc;
    if (int rc = tensor_map_2d(&pu, wu, DT, f, hidden, hidden, 128, BK)) return rc;
    return launch_pair<DT, 256, EPI_SWIGLU, 6>(pa, pg, pu, pu, q, st);
  }
  Params p{};
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(f);
  p.k = static_cast<int>(hidden);
  p.num_kb = static_cast<int>((hidden + BK - 1) / BK);
  p.m_tiles = static_cast<int>(m_tiles);
  p.n_tiles = static_cast<int>((f + half - 1) / half);
  p.seg1 = p.seg2 = p.n_tiles;
  p.y = h;
  p.ldy = f;
  apply_extras(p, ex);
  CUtensorMap ta, tg, tu;
  if (int rc = tensor_map_2d(&ta, x, DT, m, hidden, lda, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&tg, wg, DT, f, hidden, hidden, half, BK)) return rc;
  if (int rc = tensor_map_2d(&tu, wu, DT, f, hidden, hidden, half, BK)) return rc;
  if (plan.split > 1) {
    switch (half) {
      case 128: return launch_splitk<DT, 256, EPI_SWIGLU>(ta, tg, tu, tu, p, plan.split, plan.stages, st);
      case 64: return launch_splitk<DT, 128, EPI_SWIGLU>(ta, tg, tu, tu, p, plan.split, plan.stages, st);
      case 32: return launch_splitk<DT, 64, EPI_SWIGLU>(ta, tg, tu, tu, p, plan.split, plan.stages, st);
      default: return launch_splitk<DT, 32, EPI_SWIGLU>(ta, tg, tu, tu, p, plan.split, plan.stages, st);
    }
  }
  switch (half) {
    case 128: return launch<DT, 256, EPI_SWIGLU, 4>(ta, tg, tu, tu, p, 1, st);
    case 64: return launch<DT, 128, EPI_SWIGLU, 5>(ta, tg, tu, tu, p, 1, st);
    case 32:
      if (plan.stages == DEEP_STAGES) return launch<DT, 64, EPI_SWIGLU, DEEP_STAGES>(ta, tg, tu, tu, p, 1, st);
      return launch<DT, 64, EPI_SWIGLU, 4>(ta, tg, tu, tu, p, 2, st);
    default:
      if (plan.stages == DEEP_STAGES) return launch<DT, 32, EPI_SWIGLU, DEEP_STAGES>(ta, tg, tu, tu, p, 1, st);
      return launch<DT, 32, EPI_SWIGLU, 4>(ta, tg, tu, tu, p, 2, st);
  }
}

}  // namespace gemm
}  // namespace tk

using namespace tk;

static int check_gemm_common(int dtype, const void* x, int64_t lda, int64_t m, int64_t k) {
  if (!half_dtype(dtype)) return fail_invalid("GEMM dtype must be F16 or BF16");
  if (m < 0 || k <= 0) return fail_invalid("GEMM: invalid m/k");
  if (!x && m > 0) return fail_invalid("GEMM: NULL input");
  if (k % 8 != 0 || lda % 8 != 0) return fail_invalid("GEMM: k and the row stride must be multiples of 8");
  if (lda < k) return fail_invalid("GEMM: row stride smaller than k");
  if (m > 0x7fffffffLL || k > 0x7fffffffLL) return fail_invalid("GEMM: size too large");
  return TK_OK;
}

static_assert(L2_PF_MAX == TK_L2_PREFETCH_MAX, "tk_epilogue prefetch slots");

namespace {

// Host-side checks of the epilogue options; fills the device-side Extras.
int extras_from(const tk_epilogue* e, int64_t m, int64_t k, int64_t n, int64_t rope_cols, bool plain_store,
                gemm::Extras* ex, const char* what) {
  *ex = gemm::Extras{};
  if (!e) return TK_OK;
  if (e->residual && !plain_store) return fail_invalid("epilogue: a residual needs the plain store");
  ex->residual = e->residual;
  if (e->row_ssq_in) {
    if (e->row_ssq_parts <= 0 || !(e->row_ssq_eps >= 0.f)) return fail_invalid("epilogue: bad row_ssq_parts / eps");
    ex->ssq_in = e->row_ssq_in;
    ex->ssq_parts = e->row_ssq_parts;
    ex->ssq_inv_k = 1.0f / static_cast<float>(k);
    ex->ssq_eps = e->row_ssq_eps;
  }
  if (e->row_ssq_out) {
    if (!plain_store) return fail_invalid("epilogue: row_ssq_out needs the plain store");
    ex->ssq_out = e->row_ssq_out;
  }
  ex->weights_prefetch = e->weights_prefetch ? 1 : 0;
  l2_prefetch_from(e->l2_prefetch, e->l2_prefetch_bytes, &ex->pf);
  if (e->rope_head_dim) {
    const int hd = e->rope_head_dim;
    if (!plain_store || hd < 32 || hd % 32 != 0 || rope_cols % hd != 0 || rope_cols > n)
      return fail_invalid("epilogue: RoPE needs the plain store, head_dim a multiple of 32 and whole q/k heads");
    if (e->rope_seq <= 0 || e->rope_start < 0 || m % e->rope_seq != 0)
      return fail_invalid("epilogue: RoPE rows must be [batch, seq] tokens with seq > 0");
    if (int64_t(e->rope_start) + e->rope_seq > e->rope_table_rows)
      return fail_invalid("epilogue: start_pos + seq exceeds the RoPE table length");
    if (!e->rope_cos || !e->rope_sin || !aligned16(e->rope_cos) || !aligned16(e->rope_sin))
      return fail_invalid("epilogue: RoPE tables must be non-NULL and 16-byte aligned");
    ex->rope_cols = static_cast<int>(rope_cols);
    ex->rope_seq = e->rope_seq;
    ex->rope_start = e->rope_start;
    ex->rope_half_d = hd / 2;
    ex->rope_cos = static_cast<const float*>(e->rope_cos);
    ex->rope_sin = static_cast<const float*>(e->rope_sin);
  }
  (void)what;
  return TK_OK;
}

}  // namespace

extern "C" int tk_linear_ex(const void* x, int64_t x_row_stride, const void* w0, int64_t n0, const void* w1,
                            int64_t n1, const void* w2, int64_t n2, void* y, int64_t y_row_stride, int64_t m,
                            int64_t k, const tk_epilogue* epi, int dtype, void* stream) {
  if (int rc = check_gemm_common(dtype, x, x_row_stride, m, k)) return rc;
  if (n0 <= 0 || n1 < 0 || n2 < 0 || (n2 && !n1)) return fail_invalid("linear: invalid weight blocks");
  if ((n1 || n2) && (n0 % 32 != 0 || n1 % 32 != 0)) return fail_invalid("linear: weight blocks 0 and 1 must be multiples of 32 rows");
  const int64_t n = n0 + n1 + n2;
  if (n > INT32_MAX || m > INT32_MAX) return fail_invalid("linear: too large");
  gemm::Extras ex;
  if (int rc = extras_from(epi, m, k, n, n0 + n1, true, &ex, "linear")) return rc;
  if (m == 0) return TK_OK;
  if (!w0 || (n1 && !w1) || (n2 && !w2)) return fail_invalid("linear: NULL weight");
  if (!y || y_row_stride < n || y_row_stride % 8 != 0) return fail_invalid("linear: bad output or stride");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return gemm::run_linear<TK_F16>(x, x_row_stride, w0, n0, w1, n1, w2, n2, y, y_row_stride, m, k, st, ex);
  return gemm::run_linear<TK_BF16>(x, x_row_stride, w0, n0, w1, n1, w2, n2, y, y_row_stride, m, k, st, ex);
}

extern "C" int tk_linear(const void* x, int64_t x_row_stride, const void* w0, int64_t n0, const void* w1, int64_t n1,
                         const void* w2, int64_t n2, void* y, int64_t y_row_stride, const void* residual, int64_t m,
                         int64_t k, int dtype, void* stream) {
  tk_epilogue e{};
  e.residual = residual;
  return tk_linear_ex(x, x_row_stride, w0, n0, w1, n1, w2, n2, y, y_row_stride, m, k, &e, dtype, stream);
}

extern "C" int tk_linear_rope(const void* x, int64_t x_row_stride, const void* wq, int64_t nq, const void* wk,
                              int64_t nk, const void* wv, int64_t nv, void* y, int64_t y_row_stride, int64_t m,
                              int64_t k, int seq, int start_pos, int head_dim, const void* cos_table,
                              const void* sin_table, int64_t table_rows, int dtype, void* stream) {
  if (head_dim <= 0 || nq <= 0 || nk <= 0 || nv <= 0 || nq % head_dim != 0 || nk % head_dim != 0 || nv % 32 != 0)
    return fail_invalid("linear_rope: q and k widths must be multiples of head_dim, v a multiple of 32");
  tk_epilogue e{};
  e.rope_seq = seq;
  e.rope_start = start_pos;
  e.rope_head_dim = head_dim;
  e.rope_cos = cos_table;
  e.rope_sin = sin_table;
  e.rope_table_rows = table_rows;
  return tk_linear_ex(x, x_row_stride, wq, nq, wk, nk, wv, nv, y, y_row_stride, m, k, &e, dtype, stream);
}

extern "C" int tk_gate_up_swiglu_ex(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up,
                                    void* h, int64_t m, int64_t hidden, int64_t f, const tk_epilogue* epi, int dtype,
                                    void* stream) {
  if (int rc = check_gemm_common(dtype, x, x_row_stride, m, hidden)) return rc;
  if (f <= 0 || f % 8 != 0) return fail_invalid("gate_up_swiglu: f must be a positive multiple of 8");
  gemm::Extras ex;
  if (int rc = extras_from(epi, m, hidden, f, 0, false, &ex, "gate_up_swiglu")) return rc;
  if (m == 0) return TK_OK;
  if (!w_gate || !w_up || !h) return fail_invalid("gate_up_swiglu: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16) return gemm::run_gate_up<TK_F16>(x, x_row_stride, w_gate, w_up, h, m, hidden, f, st, ex);
  return gemm::run_gate_up<TK_BF16>(x, x_row_stride, w_gate, w_up, h, m, hidden, f, st, ex);
}

extern "C" int tk_gate_up_swiglu(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up, void* h,
                                 int64_t m, int64_t hidden, int64_t f, int dtype, void* stream) {
  return tk_gate_up_swiglu_ex(x, x_row_stride, w_gate, w_up, h, m, hidden, f, nullptr, dtype, stream);
}

extern "C" int tk_swiglu_ffn(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up,
                             const void* w_down, void* h_scratch, void* out, const void* residual, int64_t m,
                             int64_t hidden, int64_t f, int dtype, void* stream) {
  if (hidden % 8 != 0) return fail_invalid("swiglu_ffn: hidden must be a multiple of 8");
  if (m == 0) return TK_OK;
  if (!w_down || !h_scratch || !out) return fail_invalid("swiglu_ffn: NULL pointer");
  if (int rc = tk_gate_up_swiglu(x, x_row_stride, w_gate, w_up, h_scratch, m, hidden, f, dtype, stream)) return rc;
  return tk_linear(h_scratch, f, w_down, hidden, nullptr, 0, nullptr, 0, out, hidden, residual, m, f, dtype, stream);
}
