// Fused RoPE + GQA/MQA/MHA causal attention on tcgen05 tensor cores.
//
// One CTA computes a PAIR of 128-row query tiles (a = 2 * blk, b = 2 * blk + 1) of one
// (batch, query head). The pair index is the grid's slowest dimension, so the heaviest pairs of
// every head and sequence start first. Roles working through mbarriers (warp numbers for head_dim
// 64; head_dim 128 has eight softmax warps and the other roles start at warp 8):
//   * warp 16 (TMA): loads the two raw Q tiles once, then streams K_0, V_0, K_1, V_1, ...
//     of KV head h / groups through a ring of 4 (head_dim 64) or 3 (head_dim 128) slots,
//     straight from the [batch, seq, heads, head_dim] projection layout (token strides
//     are free, so q/k/v may be column slices of one fused q|k|v output) into
//     128-byte-swizzled shared memory. Tile b needs one key tile more than tile a.
//   * warps 18-19 (RoPE, drop-in entry only): rotate the interleaved pairs of every K row
//     in place in shared memory, in fp32, rounding back to the input dtype as the
//     reference does before its attention kernel (tinker/kernels/fused_attention.py
//     :203-214, :53-69). The softmax warps rotate their Q tile the same way, once.
//   * warp 17 (MMA, one thread): S_a = Q_a K_j^T and S_b = Q_b K_j^T as tcgen05.mma
//     (M=128, N=128, K=head_dim) into two TMEM S buffers - the next S of a tile as soon as
//     its softmax has read the current one into registers - then O_a += P_a V_j and
//     O_b += P_b V_j with V as an MN-major operand into two TMEM O accumulators, P read
//     from TMEM at head_dim 64 and from shared memory at head_dim 128.
//   * softmax warpgroups (see Roles), thread = query row: read S with tcgen05.ld, mask the
//     diagonal tile, run the online softmax with exp2, write P (rounded to the input dtype)
//     and rescale the running O in TMEM. The running maximum is only moved when a tile
//     raises it by more than 2^8 (a lazy rescale): P stays below 256 and O is rescaled on
//     few tiles. The final O / l is written by the same threads.
// Causal tiles above the diagonal are skipped. The arithmetic follows _attention_kernel
// (tinker/kernels/fused_attention.py:74-154): scale 1/sqrt(head_dim), running max / sum
// in fp32, output divided by the sum.
#include <algorithm>
#include <cmath>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace attn {

constexpr int BQ = 128;   // query rows per softmax warpgroup (one tcgen05 M=128 tile)
constexpr int BKV = 128;  // keys per K/V tile
// Warp roles. head_dim 64 runs four softmax warpgroups, two per query tile, each on one half of
// the key columns of its rows (warps 0-3: tile a, columns 0-63; 4-7: tile b, 0-63; 8-11: tile a,
// 64-127; 12-15: tile b, 64-127), exchanging the row maximum per step through shared memory; it
// measured a few percent faster than two. head_dim 128 has no shared memory left for the
// exchange buffer and runs two (warps 0-3: tile a, 4-7: tile b, whole rows).
template <int D>
struct Roles {
  static constexpr bool SPLIT = D == 64;
  static constexpr int SOFTMAX_WARPS = SPLIT ? 16 : 8;
  static constexpr int SOFTMAX_THREADS = SOFTMAX_WARPS * 32;
  static constexpr int TMA_WARP = SOFTMAX_WARPS;
  static constexpr int MMA_WARP = SOFTMAX_WARPS + 1;
  static constexpr int ROPE_WARP0 = SOFTMAX_WARPS + 2;  // two warps rotate the K tiles (two rows per thread)
  static constexpr int THREADS = (SOFTMAX_WARPS + 4) * 32;
};
constexpr int ROPE_K_THREADS = 64;
constexpr float LAZY_RESCALE_LOG2 = 8.0f;  // move the running max only when it grows by more than 2^8


template <int D>
struct Smem {
  static constexpr int Q_BYTES = BQ * D * 2;      // one query tile
  static constexpr int T_BYTES = BKV * D * 2;     // one K or V tile
  static constexpr int STAGES = D == 64 ? 4 : 3;  // K/V ring: K_0, V_0, K_1, V_1, ... through STAGES slots
  static constexpr int P_BYTES = BQ * BKV * 2;    // one P tile
  static constexpr int Q_OFF = 0;                 // Q_a, Q_b
  static constexpr int RING_OFF = Q_OFF + 2 * Q_BYTES;
  static constexpr int P_OFF = RING_OFF + STAGES * T_BYTES;  // P_a, P_b
  static constexpr int BAR_OFF = P_OFF + 2 * P_BYTES;
  static constexpr int NUM_BARS = 24;
  // head_dim 64: the softmax halves' per-row partial maxima (and at the end their sums),
  // [tile][step parity][half][row] fp32
  static constexpr int RED_SPLIT_OFF = BAR_OFF + NUM_BARS * 8 + 16;
  static constexpr int TOTAL = 1024 + RED_SPLIT_OFF + (Roles<D>::SPLIT ? 2 * 2 * 2 * BQ * 4 : 0);
  // single-tile CTAs (no query tile b): the per-row partial max and sum of the two column
  // halves, [4][128] fp32, in tile b's Q slot
  static constexpr int RED_OFF = Q_OFF + Q_BYTES;
  // S_a: 0-127, S_b: 128-255, O_a: 256.., O_b: 256 + head_dim..; head_dim 64 keeps P in the last
  // 128 columns (P_a: 384-447, P_b: 448-511, 16-bit pairs) as the A operand of P.V
  static constexpr uint32_t TMEM_COLS = 512;
};

// mbarrier slots
enum : int {
  B_Q_FULL = 0,    // both Q tiles landed (TMA transaction bytes)
  B_Q_READY = 1,   // Q tiles rotated (256 softmax threads)
  B_FULL = 2,      // [4] ring slot landed
  B_EMPTY = 6,     // [4] ring slot consumed (UMMA commit)
  B_K_READY = 10,  // [2] K_j rotated, indexed by j & 1 (64 RoPE threads)
  B_S_FULL = 12,   // [2] S_a / S_b written (UMMA commit)
  B_P_FULL = 14,   // [2] P_a / P_b written and O rescaled (128 threads of the warpgroup)
  B_PV_DONE = 16,  // [2] P.V of a / b finished (UMMA commit)
  B_S_FREE = 18,   // [2] S_a / S_b read into registers (128 threads of the warpgroup)
};

struct Params {
  int batch, seq, num_heads, num_kv_heads, groups, start_pos, n_qtiles;
  int64_t table_rows;
  const void* cos_t;
  const void* sin_t;
  int table_dtype;
  void* out;
  int64_t out_tok_stride;
  float scale_log2;  // (1/sqrt(head_dim)) * log2(e)
};

// Load 4 consecutive table entries (pair indices i0..i0+3) of row `pos` as fp32.
__device__ __forceinline__ void load_cs4(const void* t, int dt, int64_t off, float* v) {
  if (dt == TK_F32) {
    const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t) + off);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(t) + off);
    const uint32_t w[2] = {u.x, u.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float2 p;
      if (dt == TK_F16) p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      v[2 * i] = p.x;
      v[2 * i + 1] = p.y;
    }
  }
}

// RoPE of one row of a swizzled [128 x D] tile, in 64-column blocks: the 32 cos and
// 32 sin values of a block are loaded first (all in flight at once), then the
// block's 8 chunks of the row are rotated in place in fp32 and rounded back.
__device__ __forceinline__ void rope_load_block(const Params& p, int64_t pos, int blk, int half_d, float (&c)[32],
                                                float (&s)[32]) {
  const int64_t off = pos * half_d + blk * 32;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    load_cs4(p.cos_t, p.table_dtype, off + ch * 4, c + ch * 4);
    load_cs4(p.sin_t, p.table_dtype, off + ch * 4, s + ch * 4);
  }
}

template <int DT>
__device__ __forceinline__ void rope_apply_block(uint8_t* tile, int r, int blk, const float (&c)[32],
                                                 const float (&s)[32]) {
  using Dx = Dt<DT>;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    uint4* addr = reinterpret_cast<uint4*>(tile + blk * (128 * 128) + r * 128 + ((ch ^ (r & 7)) * 16));
    uint4 u = *addr;
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = Dx::unpack(*reinterpret_cast<typename Dx::T2*>(&w[i]));
      const float cc = c[ch * 4 + i], ss = s[ch * 4 + i];
      typename Dx::T2 o = Dx::pack(x.x * cc - x.y * ss, x.x * ss + x.y * cc);
      w[i] = *reinterpret_cast<uint32_t*>(&o);
    }
    *addr = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int DT, int D>
__device__ __forceinline__ void rope_row_inplace(uint8_t* tile, int r, int64_t pos, const Params& p) {
#pragma unroll
  for (int blk = 0; blk < D / 64; ++blk) {
    float c[32], s[32];
    rope_load_block(p, pos, blk, D / 2, c, s);
    rope_apply_block<DT>(tile, r, blk, c, s);
  }
}

template <int DT, int D, bool ROPE>
__global__ void __launch_bounds__(Roles<D>::THREADS, 1)
    rope_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const Params p) {
  using S = Smem<D>;
  using R = Roles<D>;
  using Dx = Dt<DT>;
  constexpr int NS = S::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + S::RING_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::NUM_BARS);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // CTA = query tiles a = 2*blk and b = 2*blk + 1 of one (batch, head); heaviest pairs first
  const int n_pairs = (p.n_qtiles + 1) >> 1;
  // the pair index is the grid's slowest dimension, so CTAs start heaviest pair first across all
  // heads and sequences (longest-first list scheduling over the SMs)
  const int blk = n_pairs - 1 - static_cast<int>(blockIdx.z);
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int kvh = h / p.groups;
  const bool has_b = 2 * blk + 1 < p.n_qtiles;
  const int n_a = 2 * blk + 1;             // key tiles of query tile a (causal)
  const int n_kv = has_b ? n_a + 1 : n_a;  // key tiles loaded (query tile b needs one more)
  // a sequence of at most 128 rows: one query tile and one key tile per CTA, so both softmax
  // warpgroups work on it, each on one half of the key columns
  const bool single = p.n_qtiles == 1;

  if (tid == 0) {
    mbar_init(bars + B_Q_FULL, 1);
    mbar_init(bars + B_Q_READY, R::SOFTMAX_THREADS);
    for (int i = 0; i < NS; ++i) {
      mbar_init(bars + B_FULL + i, 1);
      mbar_init(bars + B_EMPTY + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bars + B_K_READY + i, ROPE_K_THREADS);
      mbar_init(bars + B_S_FULL + i, 1);
      mbar_init(bars + B_P_FULL + i, R::SPLIT || single ? 256 : 128);
      mbar_init(bars + B_PV_DONE + i, 1);
      mbar_init(bars + B_S_FREE + i, R::SPLIT ? 256 : 128);
    }
    fence_mbar_init();
  }
  if (warp == R::MMA_WARP) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == R::TMA_WARP) {
    // ---------------- TMA producer: Q_a|Q_b, then K_0, V_0, K_1, V_1, ... ----------------
    if (lane == 0) {
      pdl_launch_dependents();
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      pdl_wait();  // q, k, v are written by the previous kernel
      mbar_arrive_expect_tx(bars + B_Q_FULL, (has_b ? 2 : 1) * S::Q_BYTES);
      for (int t = 0; t < (has_b ? 2 : 1); ++t)
#pragma unroll
        for (int cb = 0; cb < D / 64; ++cb)
          tma_load_3d(smem + S::Q_OFF + t * S::Q_BYTES + cb * 128 * 128, &tq, bars + B_Q_FULL, h * D + cb * 64,
                      (2 * blk + t) * BQ, b);
      for (int i = 0; i < 2 * n_kv; ++i) {
        const int slot = i % NS;
        if (i >= NS && !mbar_wait(bars + B_EMPTY + slot, ((i / NS) - 1) & 1)) break;
        const CUtensorMap* m = (i & 1) ? &tv : &tk;
        uint8_t* dst = ring + slot * S::T_BYTES;
        mbar_arrive_expect_tx(bars + B_FULL + slot, S::T_BYTES);
#pragma unroll
        for (int cb = 0; cb < D / 64; ++cb)
          tma_load_3d(dst + cb * 128 * 128, m, bars + B_FULL + slot, kvh * D + cb * 64, (i >> 1) * BKV, b);
      }
    }
  } else if (warp == R::MMA_WARP) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(Dx::umma_fmt, BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_f16(Dx::umma_fmt, BQ, D, 0, 1);
      const uint32_t q_a = smem_u32(smem + S::Q_OFF), q_b = q_a + S::Q_BYTES;
      const uint32_t p_a = smem_u32(smem + S::P_OFF), p_b = p_a + S::P_BYTES;
      // Descriptors are built once per operand base; each K=16 step adds its byte offset / 16 to the
      // start-address field (bases and offsets stay below 256 KB, so the 14-bit field never carries).
      // This thread shares its scheduler with two busy softmax warps, so its instruction count per
      // MMA decides how soon the next S is issued.
      auto issue_s = [&](uint64_t q_desc, uint64_t k_desc, uint32_t t_s) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off16 = static_cast<uint64_t>(((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4);
          umma_f16_ss(t_s, q_desc + off16, k_desc + off16, idesc_s, kk != 0);
        }
      };
      auto issue_pv = [&](uint64_t p_desc, uint32_t p_tmem, uint64_t v_desc, uint32_t t_o, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          if constexpr (R::SPLIT) {  // P in tensor memory: 8 columns per K=16 step
            umma_f16_ts(t_o, p_tmem + kk * 8, v_desc + static_cast<uint64_t>(kk * 16 * 128 / 16), idesc_o,
                        (acc || kk > 0) ? 1u : 0u);
          } else {
            const uint64_t aoff16 = static_cast<uint64_t>(((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4);
            umma_f16_ss(t_o, p_desc + aoff16, v_desc + static_cast<uint64_t>(kk * 16 * 128 / 16), idesc_o,
                        (acc || kk > 0) ? 1u : 0u);
          }
        }
      };
      // K_j is ring item 2j, V_j item 2j + 1
      auto wait_k = [&](int j) -> bool {
        if constexpr (ROPE) return mbar_wait(bars + B_K_READY + (j & 1), (j >> 1) & 1);
        const int i = 2 * j;
        return mbar_wait(bars + B_FULL + i % NS, (i / NS) & 1);
      };
      auto k_desc = [&](int i) { return make_sw128_desc(smem_u32(ring + (i % NS) * S::T_BYTES), 0, 1024); };
      auto v_desc = [&](int i) { return make_sw128_desc(smem_u32(ring + (i % NS) * S::T_BYTES), BKV * 128, 1024); };
      const uint64_t qd_a = make_sw128_desc(q_a, 0, 1024), qd_b = make_sw128_desc(q_b, 0, 1024);
      const uint64_t pd_a = make_sw128_desc(p_a, 0, 1024), pd_b = make_sw128_desc(p_b, 0, 1024);
      const uint32_t t_sa = tmem_base, t_sb = tmem_base + 128;
      const uint32_t t_oa = tmem_base + 256, t_ob = tmem_base + 256 + D;

      // with RoPE the softmax warps publish the rotated Q tiles (Q_READY after they saw Q_FULL);
      // without it nobody touches Q, so wait for the TMA transaction itself
      bool ok = mbar_wait(bars + (ROPE ? B_Q_READY : B_Q_FULL), 0) && wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_s(qd_a, k_desc(0), t_sa);
        umma_commit(bars + B_S_FULL + 0);
        if (has_b) {
          issue_s(qd_b, k_desc(0), t_sb);
          umma_commit(bars + B_S_FULL + 1);
        }
        umma_commit(bars + B_EMPTY + 0);  // K_0 consumed
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int iv = 2 * j + 1;
        // S_{j+1} of each tile as soon as its softmax has read S_j into registers (S_FREE): the
        // next Q K^T runs while the softmax of step j is still computing
        if (j + 1 < n_kv) {
          if (!wait_k(j + 1)) break;
          if (j + 1 < n_a) {
            if (!mbar_wait(bars + B_S_FREE + 0, j & 1)) break;
            tc_fence_after();
            issue_s(qd_a, k_desc(iv + 1), t_sa);
            umma_commit(bars + B_S_FULL + 0);
          }
          if (has_b) {
            if (!mbar_wait(bars + B_S_FREE + 1, j & 1)) break;
            tc_fence_after();
            issue_s(qd_b, k_desc(iv + 1), t_sb);
            umma_commit(bars + B_S_FULL + 1);
          }
          umma_commit(bars + B_EMPTY + (iv + 1) % NS);  // K_{j+1} consumed
        }
        if (!mbar_wait(bars + B_FULL + iv % NS, (iv / NS) & 1)) break;  // V_j
        if (j < n_a) {
          if (!mbar_wait(bars + B_P_FULL + 0, j & 1)) break;
          tc_fence_after();
          issue_pv(pd_a, tmem_base + 384, v_desc(iv), t_oa, j > 0);
          umma_commit(bars + B_PV_DONE + 0);
        }
        if (has_b) {
          if (!mbar_wait(bars + B_P_FULL + 1, j & 1)) break;
          tc_fence_after();
          issue_pv(pd_b, tmem_base + 448, v_desc(iv), t_ob, j > 0);
          umma_commit(bars + B_PV_DONE + 1);
        }
        umma_commit(bars + B_EMPTY + iv % NS);  // V_j consumed
      }
    }
  } else if (warp >= R::ROPE_WARP0) {
    // ---------------- RoPE of the K tiles (rows t and t + 64) ----------------
    if constexpr (ROPE) {
      pdl_wait();  // the tables may have been written by the previous kernel
      const int t = tid - R::ROPE_WARP0 * 32;
      for (int j = 0; j < n_kv; ++j) {
        const int i = 2 * j;
        uint8_t* kt = ring + (i % NS) * S::T_BYTES;
        const int64_t pos0 = static_cast<int64_t>(p.start_pos) + j * BKV + t;
        const bool v0 = j * BKV + t < p.seq, v1 = j * BKV + t + 64 < p.seq;
        float c[32], sn[32];
        if (v0) rope_load_block(p, pos0, 0, D / 2, c, sn);  // in flight while the K tile lands
        if (!mbar_wait(bars + B_FULL + i % NS, (i / NS) & 1)) break;
        // rows past the sequence are zero-filled by TMA and left alone
        if (v0) {
          rope_apply_block<DT>(kt, t, 0, c, sn);
#pragma unroll
          for (int cb = 1; cb < D / 64; ++cb) {
            rope_load_block(p, pos0, cb, D / 2, c, sn);
            rope_apply_block<DT>(kt, t, cb, c, sn);
          }
        }
        if (v1) {
#pragma unroll
          for (int cb = 0; cb < D / 64; ++cb) {
            rope_load_block(p, pos0 + 64, cb, D / 2, c, sn);
            rope_apply_block<DT>(kt, t + 64, cb, c, sn);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(bars + B_K_READY + (j & 1));
      }
    }
  } else if (!R::SPLIT && warp < 8 && single) {
    // ---------------- one key tile: warpgroup h takes key columns [64 h, 64 h + 64) of row r ----------------
    const int h2 = warp >> 2;
    const int r = tid & 127;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + S::RED_OFF);  // [max h0, max h1, sum h0, sum h1][row]
    uint8_t* sq = smem + S::Q_OFF;
    uint8_t* sp = smem + S::P_OFF;
    bool ok = true;
    if constexpr (ROPE) {
      const bool valid = h2 == 0 && r < p.seq;
      float c[32], sn[32];
      pdl_wait();  // the tables may have been written by the previous kernel
      if (valid) rope_load_block(p, static_cast<int64_t>(p.start_pos) + r, 0, D / 2, c, sn);
      ok = mbar_wait(bars + B_Q_FULL, 0);
      if (ok && valid) {
        rope_apply_block<DT>(sq, r, 0, c, sn);
#pragma unroll
        for (int cb = 1; cb < D / 64; ++cb) {
          rope_load_block(p, static_cast<int64_t>(p.start_pos) + r, cb, D / 2, c, sn);
          rope_apply_block<DT>(sq, r, cb, c, sn);
        }
      }
      fence_proxy_async_smem();
    }
    mbar_arrive(bars + B_Q_READY);
    ok = ok && mbar_wait(bars + B_S_FULL + 0, 0);
    tc_fence_after();
    float sv[64];
    tmem_load64(tmem_base + lane_off + h2 * 64, sv);
#pragma unroll
    for (int c = 0; c < 64; ++c)
      if (h2 * 64 + c > r) sv[c] = -INFINITY;  // causal mask of the diagonal tile
    float mx8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
    for (int c = 8; c < 64; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
    red[h2 * BQ + r] = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
    named_sync(1, R::SOFTMAX_THREADS);
    // column 0 is never masked, so the row maximum is finite
    const float neg_m = -fmaxf(red[r], red[BQ + r]) * p.scale_log2;
    const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2), negm2 = pack_f32x2(neg_m, neg_m);
    uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 64; c += 2) {
      const uint64_t e = fma_f32x2(pack_f32x2(sv[c], sv[c + 1]), scale2, negm2);
      float e0, e1;
      unpack_f32x2(e, e0, e1);
      sv[c] = exp2_approx(e0);
      sv[c + 1] = exp2_approx(e1);
      rs2[(c >> 1) & 3] = add_f32x2(rs2[(c >> 1) & 3], pack_f32x2(sv[c], sv[c + 1]));
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        typename Dx::T2 hv = Dx::pack(sv[c * 8 + 2 * i], sv[c * 8 + 2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(sp + h2 * (128 * 128) + r * 128 + ((c ^ (r & 7)) * 16)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(bars + B_P_FULL + 0);  // 256 arrivals: both halves of P
    float rp[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack_f32x2(rs2[i], rp[2 * i], rp[2 * i + 1]);
    red[(2 + h2) * BQ + r] = ((rp[0] + rp[1]) + (rp[2] + rp[3])) + ((rp[4] + rp[5]) + (rp[6] + rp[7]));
    named_sync(1, R::SOFTMAX_THREADS);
    const float inv_l = 1.0f / (red[2 * BQ + r] + red[3 * BQ + r]);
    // O / l: warpgroup h2 writes output columns [h2 D/2, h2 D/2 + D/2) of row r
    if (ok && mbar_wait(bars + B_PV_DONE + 0, 0)) {
      tc_fence_after();
      using T = typename Dx::T;
      T* dst = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.seq + r) * p.out_tok_stride +
               static_cast<int64_t>(h) * D;
#pragma unroll
      for (int c = h2 * (D / 2); c < (h2 + 1) * (D / 2); c += 32) {
        float o[32];
        tmem_load32(tmem_base + 256 + lane_off + c, o);
        if (r < p.seq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              typename Dx::T2 hv = Dx::pack(o[q * 8 + 2 * i] * inv_l, o[q * 8 + 2 * i + 1] * inv_l);
              w[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
            reinterpret_cast<uint4*>(dst + c)[q] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  } else if (R::SPLIT && warp < R::SOFTMAX_WARPS) {
    // ---------------- softmax, head_dim 64: tile x, key columns [64 hh, 64 hh + 64) of row r ----------------
    const int x = (warp >> 2) & 1;
    const int hh = warp >> 3;
    const int r = tid & 127;
    const int qt = 2 * blk + x;
    const int q_row = qt * BQ + r;
    const bool active = x == 0 || has_b;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem_base + x * 128 + hh * 64;
    const uint32_t t_o = tmem_base + 256 + x * D + hh * (D / 2);
    uint8_t* sq = smem + S::Q_OFF + x * S::Q_BYTES;
    const uint32_t t_p = tmem_base + 384 + x * 64 + hh * 32;  // this half's 64 keys of P, packed in pairs
    float* red = reinterpret_cast<float*>(smem + S::RED_SPLIT_OFF) + x * (2 * 2 * BQ);
    bool ok = true;
    if constexpr (ROPE) {
      const int64_t qpos = static_cast<int64_t>(p.start_pos) + q_row;
      const bool valid = active && hh == 0 && q_row < p.seq;
      float c[32], sn[32];
      pdl_wait();  // the tables may have been written by the previous kernel
      if (valid) rope_load_block(p, qpos, 0, D / 2, c, sn);  // in flight while the Q tile lands
      ok = mbar_wait(bars + B_Q_FULL, 0);
      if (ok && valid) rope_apply_block<DT>(sq, r, 0, c, sn);
      fence_proxy_async_smem();
    }
    mbar_arrive(bars + B_Q_READY);
    const int n_x = x == 0 ? n_a : n_a + 1;
    float m_run = -INFINITY, l_run = 0.f;
    // every step reaches the halves' barrier, also after a timed-out wait (the other half waits there)
    for (int j = 0; active && j < n_x; ++j) {
      if (ok) ok = mbar_wait(bars + B_S_FULL + x, j & 1);
      tc_fence_after();
      float sv[64];
      tmem_load64(t_s + lane_off, sv);
      // S is in registers: the MMA may write the next tile's scores over it
      tc_fence_before();
      mbar_arrive(bars + B_S_FREE + x);
      if (j == qt) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (j * BKV + hh * 64 + c > q_row) sv[c] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int c = 8; c < 64; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
      // the row maximum of this step: both halves' partial maxima, double-buffered by step parity
      // (a half overwrites a slot only after the barrier of the next step, which its partner
      // passes only once it has read the slot)
      float* rj = red + (j & 1) * (2 * BQ);
      rj[hh * BQ + r] = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                              fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      named_sync(1 + x, 256);
      const float mx = fmaxf(rj[r], rj[BQ + r]) * p.scale_log2;
      // lazy rescale: keep the old maximum unless this tile exceeds it by more than 2^8 (both
      // halves see the same maxima, so they take the same decision)
      float m_use = m_run, alpha = 1.f;
      if (mx > m_run + LAZY_RESCALE_LOG2) {
        m_use = mx;
        alpha = exp2_approx(m_run - mx);
      }
      const float neg_m = -m_use;
      const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2), negm2 = pack_f32x2(neg_m, neg_m);
      uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const uint64_t e = fma_f32x2(pack_f32x2(sv[c], sv[c + 1]), scale2, negm2);
        float e0, e1;
        unpack_f32x2(e, e0, e1);
        sv[c] = exp2_approx(e0);
        sv[c + 1] = exp2_approx(e1);
        rs2[(c >> 1) & 3] = add_f32x2(rs2[(c >> 1) & 3], pack_f32x2(sv[c], sv[c + 1]));
      }
      float rp[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack_f32x2(rs2[i], rp[2 * i], rp[2 * i + 1]);
      l_run = l_run * alpha + (((rp[0] + rp[1]) + (rp[2] + rp[3])) + ((rp[4] + rp[5]) + (rp[6] + rp[7])));
      m_run = m_use;
      if (j > 0 && ok) {
        // P and the O accumulator are still in use by the previous P.V
        ok = mbar_wait(bars + B_PV_DONE + x, (j - 1) & 1);
        tc_fence_after();
      }
      {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          typename Dx::T2 hv = Dx::pack(sv[2 * i], sv[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&hv);
        }
        tmem_st32u(t_p + lane_off, w);  // waits for its own completion
      }
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
        for (int c = 0; c < D / 2; c += 32) {
          float o[32];
          tmem_load32(t_o + lane_off + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(t_o + lane_off + c, o);
        }
      }
      tc_fence_before();
      mbar_arrive(bars + B_P_FULL + x);
    }
    if (active) {
      // the row sum: both halves' partial sums, through the parity slot no step still reads
      float* rs_buf = red + (n_x & 1) * (2 * BQ);
      rs_buf[hh * BQ + r] = l_run;
      named_sync(1 + x, 256);
      const float inv_l = 1.0f / (rs_buf[r] + rs_buf[BQ + r]);
      if (ok && mbar_wait(bars + B_PV_DONE + x, (n_x - 1) & 1)) {
        tc_fence_after();
        using T = typename Dx::T;
        T* dst = reinterpret_cast<T*>(p.out) +
                 (static_cast<int64_t>(b) * p.seq + q_row) * p.out_tok_stride + static_cast<int64_t>(h) * D + hh * (D / 2);
#pragma unroll
        for (int c = 0; c < D / 2; c += 32) {
          float o[32];
          tmem_load32(t_o + lane_off + c, o);
          if (q_row < p.seq) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                typename Dx::T2 hv = Dx::pack(o[q * 8 + 2 * i] * inv_l, o[q * 8 + 2 * i + 1] * inv_l);
                w[i] = *reinterpret_cast<uint32_t*>(&hv);
              }
              reinterpret_cast<uint4*>(dst + c)[q] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
    }
  } else if (!R::SPLIT && warp < 8) {
    // ---------------- softmax / correction / output: warpgroup x, thread = query row ----------------
    const int x = warp >> 2;
    const int r = tid & 127;
    const int qt = 2 * blk + x;
    const int q_row = qt * BQ + r;
    const bool active = x == 0 || has_b;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem_base + x * 128;
    const uint32_t t_o = tmem_base + 256 + x * D;
    uint8_t* sq = smem + S::Q_OFF + x * S::Q_BYTES;
    uint8_t* sp = smem + S::P_OFF + x * S::P_BYTES;
    bool ok = true;
    if constexpr (ROPE) {
      const int64_t qpos = static_cast<int64_t>(p.start_pos) + q_row;
      const bool valid = active && q_row < p.seq;
      float c[32], sn[32];
      pdl_wait();  // the tables may have been written by the previous kernel
      if (valid) rope_load_block(p, qpos, 0, D / 2, c, sn);  // in flight while the Q tile lands
      ok = mbar_wait(bars + B_Q_FULL, 0);
      if (ok && valid) {
        rope_apply_block<DT>(sq, r, 0, c, sn);
#pragma unroll
        for (int cb = 1; cb < D / 64; ++cb) {
          rope_load_block(p, qpos, cb, D / 2, c, sn);
          rope_apply_block<DT>(sq, r, cb, c, sn);
        }
      }
      fence_proxy_async_smem();
    }
    mbar_arrive(bars + B_Q_READY);

    const int n_x = x == 0 ? n_a : n_a + 1;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; active && ok && j < n_x; ++j) {
      if (!mbar_wait(bars + B_S_FULL + x, j & 1)) { ok = false; break; }
      tc_fence_after();
      float sv[BKV];
      tmem_load128(t_s + lane_off, sv);
      // S is in registers: the MMA may write the next tile's scores over it
      tc_fence_before();
      mbar_arrive(bars + B_S_FREE + x);

      // mask the diagonal tile, then the row maximum over eight independent chains
      if (j == qt) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (j * BKV + c > q_row) sv[c] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int c = 8; c < BKV; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * p.scale_log2;
      // lazy rescale: keep the old maximum unless this tile exceeds it by more than 2^8
      float m_use = m_run, alpha = 1.f;
      if (mx > m_run + LAZY_RESCALE_LOG2) {
        m_use = mx;
        alpha = exp2_approx(m_run - mx);
      }
      // p = 2^(s * scale * log2(e) - m): one FMA and one MUFU.EX2 per score
      const float neg_m = -m_use;
      // packed f32x2 FMA / add: two scores per instruction
      const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2), negm2 = pack_f32x2(neg_m, neg_m);
      uint64_t rs2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < BKV; c += 2) {
        const uint64_t e = fma_f32x2(pack_f32x2(sv[c], sv[c + 1]), scale2, negm2);
        float e0, e1;
        unpack_f32x2(e, e0, e1);
        sv[c] = exp2_approx(e0);
        sv[c + 1] = exp2_approx(e1);
        rs2[(c >> 1) & 3] = add_f32x2(rs2[(c >> 1) & 3], pack_f32x2(sv[c], sv[c + 1]));
      }
      float rp[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack_f32x2(rs2[i], rp[2 * i], rp[2 * i + 1]);
      const float rs = ((rp[0] + rp[1]) + (rp[2] + rp[3])) + ((rp[4] + rp[5]) + (rp[6] + rp[7]));
      l_run = l_run * alpha + rs;
      m_run = m_use;

      if (j > 0) {
        // P and the O accumulator are still in use by the previous P.V
        if (!mbar_wait(bars + B_PV_DONE + x, (j - 1) & 1)) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < BKV / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          typename Dx::T2 hv = Dx::pack(sv[c * 8 + 2 * i], sv[c * 8 + 2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&hv);
        }
        uint8_t* dst = sp + (c >> 3) * (128 * 128) + r * 128 + (((c & 7) ^ (r & 7)) * 16);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float o[32];
          tmem_load32(t_o + lane_off + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(t_o + lane_off + c, o);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bars + B_P_FULL + x);
    }

    if (active && ok && mbar_wait(bars + B_PV_DONE + x, (n_x - 1) & 1)) {
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      using T = typename Dx::T;
      T* dst = reinterpret_cast<T*>(p.out) +
               (static_cast<int64_t>(b) * p.seq + q_row) * p.out_tok_stride + static_cast<int64_t>(h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_load32(t_o + lane_off + c, o);
        if (q_row < p.seq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              typename Dx::T2 hv = Dx::pack(o[q * 8 + 2 * i] * inv_l, o[q * 8 + 2 * i + 1] * inv_l);
              w[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
            reinterpret_cast<uint4*>(dst + c)[q] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == R::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

template <int DT, int D, bool ROPE>
int launch(const void* q, int64_t qs, const void* k, int64_t ks, const void* v, int64_t vs, Params p,
           cudaStream_t st) {
  using S = Smem<D>;
  CUtensorMap tq, tk_, tv;
  const uint64_t B = p.batch, Sq = p.seq;
  if (int rc = tensor_map_3d(&tq, q, DT, uint64_t(p.num_heads) * D, Sq, B, qs, qs * Sq, 64, BQ, 1)) return rc;
  if (int rc = tensor_map_3d(&tk_, k, DT, uint64_t(p.num_kv_heads) * D, Sq, B, ks, ks * Sq, 64, BKV, 1)) return rc;
  if (int rc = tensor_map_3d(&tv, v, DT, uint64_t(p.num_kv_heads) * D, Sq, B, vs, vs * Sq, 64, BKV, 1)) return rc;
  auto kern = rope_attention_kernel<DT, D, ROPE>;
  static bool configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!configured[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL),
                            "cudaFuncSetAttribute(attention)"))
      return rc;
    configured[dev.device] = true;
  }
  return launch_kernel(kern, dim3(p.num_heads, p.batch, (p.n_qtiles + 1) / 2), dim3(Roles<D>::THREADS), S::TOTAL, st, 1,
                       ROPE ? "rope_attention_kernel" : "causal_attention_kernel", tq, tk_, tv, p);
}

// RoPE of q and k in one pass, into out [batch, seq, (num_heads + num_kv_heads) * D] (q heads,
// then k heads). One thread per (token, group of heads_per_thread heads, 8-column chunk of a
// head): it loads the 4 cos and 4 sin values of its chunk once and rotates that chunk in each
// head of its group (few heads per thread when there are few tokens, all of them when many).
template <int DT>
__global__ void __launch_bounds__(256) rope_qk_kernel(const void* __restrict__ q, int64_t qs,
                                                       const void* __restrict__ k, int64_t ks, void* __restrict__ out,
                                                       int64_t os, Params p, int head_dim, int64_t tokens,
                                                       int heads_per_thread) {
  using Dx = Dt<DT>;
  pdl_launch_dependents();
  pdl_wait();  // q and k are written by the previous kernel
  const int chunks = head_dim / 8;
  const int heads = p.num_heads + p.num_kv_heads;
  const int groups = (heads + heads_per_thread - 1) / heads_per_thread;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= tokens * groups * chunks) return;
  const int64_t tok = t / (groups * chunks);
  const int rem = static_cast<int>(t - tok * groups * chunks);
  const int grp = rem / chunks;
  const int col = (rem - grp * chunks) * 8;
  const int64_t pos = static_cast<int64_t>(p.start_pos) + tok % p.seq;
  float c[4], sn[4];
  load_cs4(p.cos_t, p.table_dtype, pos * (head_dim / 2) + col / 2, c);
  load_cs4(p.sin_t, p.table_dtype, pos * (head_dim / 2) + col / 2, sn);
  const uint16_t* qrow = reinterpret_cast<const uint16_t*>(q) + tok * qs + col;
  const uint16_t* krow = reinterpret_cast<const uint16_t*>(k) + tok * ks + col;
  uint16_t* orow = reinterpret_cast<uint16_t*>(out) + tok * os + col;
  const int h1 = min(heads, (grp + 1) * heads_per_thread);
  for (int h = grp * heads_per_thread; h < h1; ++h) {
    const uint16_t* src = h < p.num_heads ? qrow + h * head_dim : krow + (h - p.num_heads) * head_dim;
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = Dx::unpack(*reinterpret_cast<typename Dx::T2*>(&w[i]));
      typename Dx::T2 o = Dx::pack(x.x * c[i] - x.y * sn[i], x.x * sn[i] + x.y * c[i]);
      w[i] = *reinterpret_cast<uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(orow + h * head_dim) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <bool ROPE>
int dispatch(const void* q, int64_t qs, const void* k, int64_t ks, const void* v, int64_t vs, const Params& p,
             int dtype, int head_dim, cudaStream_t st) {
  if (dtype == TK_F16) {
    if (head_dim == 64) return launch<TK_F16, 64, ROPE>(q, qs, k, ks, v, vs, p, st);
    return launch<TK_F16, 128, ROPE>(q, qs, k, ks, v, vs, p, st);
  }
  if (head_dim == 64) return launch<TK_BF16, 64, ROPE>(q, qs, k, ks, v, vs, p, st);
  return launch<TK_BF16, 128, ROPE>(q, qs, k, ks, v, vs, p, st);
}

// Argument checks shared by both entry points; fills the kernel parameters.
int prepare(const char* what, const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
            const void* v, int64_t v_tok_stride, void* out, int64_t out_tok_stride, int batch, int seq,
            int num_heads, int num_kv_heads, int head_dim, int dtype, Params* p, bool* empty) {
  *empty = false;
  if (!half_dtype(dtype)) return fail_invalid("attention: dtype must be F16 or BF16");
  if (head_dim != 64 && head_dim != 128) return set_error(TK_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0) return fail_invalid("attention: invalid sizes");
  if (num_heads % num_kv_heads != 0) return fail_invalid("attention: num_heads must be a multiple of num_kv_heads");
  if (q_tok_stride < int64_t(num_heads) * head_dim || k_tok_stride < int64_t(num_kv_heads) * head_dim ||
      v_tok_stride < int64_t(num_kv_heads) * head_dim || out_tok_stride < int64_t(num_heads) * head_dim)
    return fail_invalid("attention: token stride smaller than heads * head_dim");
  if (q_tok_stride % 8 || k_tok_stride % 8 || v_tok_stride % 8 || out_tok_stride % 8)
    return fail_invalid("attention: token strides must be multiples of 8 elements");
  if (num_heads > 65535 || batch > 65535 || (int64_t(seq) + 2 * BQ - 1) / (2 * BQ) > 65535)
    return fail_invalid("attention: too many heads, batches or query tiles");
  if (batch == 0 || seq == 0) {  // empty tensors may carry NULL data pointers
    *empty = true;
    return TK_OK;
  }
  if (!q || !k || !v || !out) return fail_invalid("attention: NULL pointer");
  if (!aligned16(out)) return fail_invalid("attention: out must be 16-byte aligned");
  (void)what;
  *p = Params{};
  p->batch = batch;
  p->seq = seq;
  p->num_heads = num_heads;
  p->num_kv_heads = num_kv_heads;
  p->groups = num_heads / num_kv_heads;
  p->n_qtiles = (seq + BQ - 1) / BQ;
  p->out = out;
  p->out_tok_stride = out_tok_stride;
  p->scale_log2 = static_cast<float>((1.0 / std::sqrt(double(head_dim))) * 1.4426950408889634);
  return TK_OK;
}

}  // namespace attn
}  // namespace tk

extern "C" int tk_rope_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                                 const void* v, int64_t v_tok_stride, const void* cos_table, const void* sin_table,
                                 int table_dtype, int64_t table_rows, void* out, int64_t out_tok_stride, int batch,
                                 int seq, int num_heads, int num_kv_heads, int head_dim, int start_pos, int dtype,
                                 void* stream) {
  using namespace tk;
  if (!valid_dtype(table_dtype)) return fail_invalid("rope_attention: table dtype must be F16, BF16 or F32");
  if (start_pos < 0) return fail_invalid("rope_attention: invalid sizes");
  attn::Params p{};
  bool empty = false;
  if (int rc = attn::prepare("rope_attention", q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, out,
                             out_tok_stride, batch, seq, num_heads, num_kv_heads, head_dim, dtype, &p, &empty))
    return rc;
  if (int64_t(start_pos) + seq > table_rows)
    return fail_invalid("rope_attention: start_pos + seq exceeds the RoPE table length");
  if (empty) return TK_OK;
  if (!cos_table || !sin_table) return fail_invalid("rope_attention: NULL pointer");
  if (!aligned16(cos_table) || !aligned16(sin_table))
    return fail_invalid("rope_attention: the RoPE tables must be 16-byte aligned");
  p.start_pos = start_pos;
  p.table_rows = table_rows;
  p.cos_t = cos_table;
  p.sin_t = sin_table;
  p.table_dtype = table_dtype;
  return attn::dispatch<true>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, dtype, head_dim,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int tk_causal_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                                   const void* v, int64_t v_tok_stride, void* out, int64_t out_tok_stride, int batch,
                                   int seq, int num_heads, int num_kv_heads, int head_dim, int dtype, void* stream) {
  using namespace tk;
  attn::Params p{};
  bool empty = false;
  if (int rc = attn::prepare("causal_attention", q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, out,
                             out_tok_stride, batch, seq, num_heads, num_kv_heads, head_dim, dtype, &p, &empty))
    return rc;
  if (empty) return TK_OK;
  return attn::dispatch<false>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, dtype, head_dim,
                               static_cast<cudaStream_t>(stream));
}

extern "C" int tk_rope_qk(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                          const void* cos_table, const void* sin_table, int table_dtype, int64_t table_rows,
                          void* out, int64_t out_tok_stride, int batch, int seq, int num_heads, int num_kv_heads,
                          int head_dim, int start_pos, int dtype, void* stream) {
  using namespace tk;
  if (!half_dtype(dtype)) return fail_invalid("rope_qk: dtype must be F16 or BF16");
  if (!valid_dtype(table_dtype)) return fail_invalid("rope_qk: table dtype must be F16, BF16 or F32");
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0 || start_pos < 0 || head_dim <= 0 ||
      head_dim % 8 != 0)
    return fail_invalid("rope_qk: invalid sizes (head_dim must be a positive multiple of 8)");
  const int64_t width = int64_t(num_heads + num_kv_heads) * head_dim;
  if (q_tok_stride < int64_t(num_heads) * head_dim || k_tok_stride < int64_t(num_kv_heads) * head_dim ||
      out_tok_stride < width)
    return fail_invalid("rope_qk: token stride smaller than heads * head_dim");
  if (q_tok_stride % 8 || k_tok_stride % 8 || out_tok_stride % 8)
    return fail_invalid("rope_qk: token strides must be multiples of 8 elements");
  if (int64_t(start_pos) + seq > table_rows)
    return fail_invalid("rope_qk: start_pos + seq exceeds the RoPE table length");
  if (batch == 0 || seq == 0) return TK_OK;
  if (!q || !k || !cos_table || !sin_table || !out) return fail_invalid("rope_qk: NULL pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(out) || !aligned16(cos_table) || !aligned16(sin_table))
    return fail_invalid("rope_qk: q, k, out and the RoPE tables must be 16-byte aligned");
  attn::Params p{};
  p.seq = seq;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.start_pos = start_pos;
  p.table_rows = table_rows;
  p.cos_t = cos_table;
  p.sin_t = sin_table;
  p.table_dtype = table_dtype;
  const int64_t tokens = int64_t(batch) * seq;
  // enough threads to fill the GPU (~8 blocks of 256 per SM), as many heads per thread as that allows
  const int heads = num_heads + num_kv_heads;
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  const int64_t want = int64_t(dev.sm_count) * 8 * 256;
  const int64_t per_head = tokens * (head_dim / 8);
  const int hpt_max = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(heads, per_head * heads / want)));
  const int groups = (heads + hpt_max - 1) / hpt_max;
  const int hpt = (heads + groups - 1) / groups;  // equal groups
  const int64_t threads = per_head * groups;
  const dim3 grid(static_cast<unsigned>((threads + 255) / 256)), block(256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return launch_kernel(attn::rope_qk_kernel<TK_F16>, grid, block, 0, st, 1, "rope_qk_kernel", q, q_tok_stride, k,
                         k_tok_stride, out, out_tok_stride, p, head_dim, tokens, hpt);
  return launch_kernel(attn::rope_qk_kernel<TK_BF16>, grid, block, 0, st, 1, "rope_qk_kernel", q, q_tok_stride, k,
                       k_tok_stride, out, out_tok_stride, p, head_dim, tokens, hpt);
}
