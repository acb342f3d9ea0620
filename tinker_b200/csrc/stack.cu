// The whole decoder stack of a short prefill (batch x seq <= 128 rows) in ONE persistent
// kernel: token embedding, for every layer the q|k|v projection (attention RMSNorm folded
// into the weights, RoPE in the epilogue), causal GQA attention, o_proj + residual,
// gate|up + SwiGLU (FFN RMSNorm folded), down + residual, then the final RMSNorm.
//
// Why: at 128 rows every projection is a weight stream of 2-12 MB that HBM delivers in
// 0.3-2 us, while a kernel boundary costs several microseconds of set-up, drain and
// dependency latency; the per-block path is 5 launches per layer. Here the stages of a
// layer are separated by arrival counters instead, and a CTA loads the weight tiles of
// its next work item into shared memory as soon as its tensor cores have finished the
// previous item - weights never depend on the previous stage, only the activations do -
// so the weight stream of stage n+1 overlaps the tail of stage n.
//
// One CTA per SM (cooperative launch: every CTA is resident, so CTAs may wait on one
// another), 192 threads:
//   warp 0      TMA producer: weight tiles of the CTA's next item into the W region as
//               soon as the previous item's MMAs are done, then - once the stage it
//               depends on is complete - the activation k-blocks into the A region
//               (attention items: Q, K and V tiles of one head)
//   warp 1      allocates all 512 TMEM columns once; one lane issues tcgen05.mma:
//               GEMM items accumulate 128 x BN in TMEM columns [0, 128); attention
//               items S = Q K^T into [128, 256) and O = P V into [256, 320)
//   warps 2-5   epilogue, 128 threads (TMEM lane quarter = warp % 4): GEMM items write
//               their fp32 partial tile to an L2-resident buffer, count it on the tile's
//               counter, wait for the tile's other k-splits, then reduce the 16-row groups
//               they own (group g -> k-split g % split, fixed summation order, so results
//               are deterministic) and run the epilogue; attention items run the softmax
//               (thread = query row) and write P to shared memory for the P.V MMA.
//
// Work division: stage s of the schedule (embedding, 5 per layer, final norm) has items
// (n-tile, k-split) - or (sequence, head) for attention - dealt to CTAs round-robin. A
// CTA arrives on the stage's counter after its last item of the stage; consumers wait
// for all gridDim.x arrivals. A stage being complete implies every earlier stage is
// (each CTA walks the stages in order). Activations are read with ld.global.cg / TMA
// (never a stale L1 line); counters use release/acquire at gpu scope.
//
// Every wait is bounded (TK_WAIT_LIMIT_NS) and fails fast once any CTA has recorded a
// device error; on failure a thread skips its work but keeps walking the schedule, so
// the epilogue warps' named barriers stay aligned, the producer waits for its own TMA
// copies in flight, and every CTA frees its TMEM and returns. The last CTA to finish
// returns every counter to zero for the next launch.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace stack {

constexpr int THREADS = 192;
constexpr int EPI_THREADS = 128;
constexpr int BM = 128;  // rows: the whole prefill is one M tile
constexpr int BK = 64;   // one 128-byte swizzle atom of 2-byte elements
constexpr int MAX_KB = 6;      // k-blocks per item (the W and A regions)
constexpr int MAX_SPLIT = 16;  // k-splits per tile (splits past the 8 row groups only add partials)
constexpr int MAX_BN = 128;
constexpr int HEAD_DIM = 64;
constexpr int KB_A_BYTES = BM * BK * 2;               // 16 KB
constexpr int W_REGION = MAX_KB * MAX_BN * BK * 2;    // 96 KB
constexpr int A_REGION = MAX_KB * KB_A_BYTES;         // 96 KB
constexpr int ATT_Q = 0, ATT_K = 16384, ATT_V = 32768, ATT_P = 49152;  // P: 128 x 128 keys, 32 KB
constexpr int BAR_OFF = W_REGION + A_REGION;

enum Bar : int {
  B_W_FULL = 0,
  B_A_FULL = 1,  // [MAX_KB]; attention: 0 = Q, 1 = K, 2 = V
  B_MMA_DONE = B_A_FULL + MAX_KB,
  B_W_FREE,
  B_A_FREE,
  B_ACC_FREE,
  B_S_FULL,
  B_P_FULL,
  B_O_FULL,
  B_O_FREE,
  B_PROD_DONE,  // the producer has issued and seen land all its copies
  NUM_BARS
};
constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;  // tmem slot, flags
constexpr int RSTD_OFF = BAR_OFF + 256;            // [BM] 1/rms of the stage's input rows
constexpr int SMEM_BYTES = 1024 + RSTD_OFF + BM * 4;

constexpr uint32_t T_ACC = 0, T_S = 128, T_O = 256, TMEM_COLS = 512;

enum GemmKind { G_QKV = 0, G_O = 1, G_GU = 2, G_D = 3 };
// trace events (tk_stack_trace): producer saw the stage's dependency / issued its first weight
// tiles; MMA committed the stage's last item; epilogue saw its first accumulator / its first
// tile's k-splits / the stage's dependency, arrived on the stage; attention S ready
enum TraceEvent { EV_DEP = 0, EV_W = 1, EV_MMA = 2, EV_ACC = 3, EV_TILE = 4, EV_EDEP = 5, EV_ARRIVE = 6, EV_S = 7,
                  EV_PW = 8, EV_RED = 9, EV_O = 10, TRACE_EVENTS = 12 };
enum : int { K_QKV = 0, K_ATT = 1, K_O = 2, K_GU = 3, K_D = 4, STAGES_PER_LAYER = 5 };

struct Gemm {
  int n;       // output columns (G_GU: the SwiGLU width)
  int k;       // reduction length
  int bn;      // accumulator columns per tile (G_GU: bn/2 gate + bn/2 up)
  int tiles, split, num_kb;
};

// tensor maps in the scratch buffer: activations, then L_MAPS per layer
enum { M_X = 0, M_ATTN = 1, M_H = 2, M_ACT = 3, M_QKV = 4, M_LAYER0 = 8 };
enum { L_WQ = 0, L_WK, L_WV, L_WO, L_WG, L_WU, L_WD, L_MAPS = 8 };

struct Params {
  int num_layers, m, seq, hidden, heads, kv_heads, inter, q_w, kv_w, start_pos;
  Gemm g[4];
  const CUtensorMap* maps;
  const float* eps;  // [2 * num_layers]: attention-norm eps, FFN-norm eps (folded norms)
  const int64_t* tokens;
  const void* emb;
  int64_t vocab;
  void* x;     // [BM, hidden]: the residual stream (block inputs / outputs)
  void* qkv;   // [BM, q_w + 2 kv_w]
  void* attn;  // [BM, q_w]
  void* h;     // [BM, hidden]
  void* act;   // [BM, inter]
  void* y;     // [m, hidden]: final RMSNorm of the last block's output
  float* ssq_x;  // [hidden / 32, BM] sums of squares of x's 32-column chunks
  float* ssq_h;  // [hidden / 32, BM]
  float* partial;
  unsigned* counters;  // [n_counters]: stage arrivals, exit, then per-(layer, GEMM, tile) k-split arrivals
  int n_counters, max_tiles;
  const float* cos_t;
  const float* sin_t;
  int64_t table_rows;
  const void* final_w;
  float final_eps;
  float scale_log2;  // log2(e) / sqrt(head_dim)
  // diagnostics (null: off): %globaltimer of event e of stage s in CTA c at
  // trace[(c * exit_counter(num_layers) + s) * TRACE_EVENTS + e]
  unsigned long long* trace;
};

__host__ __device__ inline int stage_of(int layer, int kind) { return 1 + STAGES_PER_LAYER * layer + kind; }
__host__ __device__ inline int norm_stage(int layers) { return 1 + STAGES_PER_LAYER * layers; }
__host__ __device__ inline int exit_counter(int layers) { return norm_stage(layers) + 1; }
// set by the first wait of this launch that ran out: every other wait then gives up at once
__host__ __device__ inline int abort_word(int layers) { return exit_counter(layers) + 1; }
__host__ __device__ inline int tile_counter(const Params& p, int layer, int gk, int tile) {
  return abort_word(p.num_layers) + 1 + (layer * 4 + gk) * p.max_tiles + tile;
}

#define TK_TRACE(s, e)                                                                               \
  do {                                                                                               \
    if (p.trace) p.trace[(static_cast<size_t>(blockIdx.x) * exit_counter(p.num_layers) + (s)) * TRACE_EVENTS + (e)] = \
        globaltimer();                                                                               \
  } while (0)

// ---- cross-CTA synchronisation ------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool aborted(const unsigned* abort) { return *reinterpret_cast<const volatile unsigned*>(abort) != 0; }
__device__ __forceinline__ void give_up(unsigned* abort) {
  record_device_error(TK_DEVERR_TIMEOUT);
  atomicExch(abort, 1u);
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// named barrier of the four epilogue warps
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Wait until *c >= target (acquire). False when the wait runs out (device error 1 recorded,
// the launch's abort word set) or another wait of this launch already ran out. Polls with
// relaxed loads and a short back-off (up to 296 pollers share a counter) and fences once.
__device__ bool wait_count(const unsigned* c, unsigned target, unsigned* abort) {
  if (ld_acquire_u32(c) >= target) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 16; ++i) {
      if (ld_relaxed_u32(c) >= target) {
        fence_acquire_gpu();
        return true;
      }
      __nanosleep(32);
    }
    if (aborted(abort)) return false;
    if (globaltimer() - t0 > TK_WAIT_LIMIT_NS) {
      give_up(abort);
      return false;
    }
  }
}
// Bounded mbarrier wait with the same give-up rules.
__device__ bool wait_bar(uint64_t* bar, uint32_t parity, unsigned* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (aborted(abort)) return false;
    if (globaltimer() - t0 > TK_WAIT_LIMIT_NS) {
      give_up(abort);
      return false;
    }
  }
}

// ---- small epilogue helpers ---------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t idx, float (&v)[8]) {
  using D = Dt<DT>;
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(static_cast<const typename D::T*>(base) + idx));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = D::unpack(*reinterpret_cast<const typename D::T2*>(&w[j]));
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
// Round 8 values to DT, store them (16 bytes) and return the sum of squares of the rounded values.
template <int DT>
__device__ __forceinline__ float store8(void* base, int64_t idx, const float (&v)[8]) {
  using D = Dt<DT>;
  uint32_t w[4];
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    typename D::T2 hv = D::pack(v[2 * j], v[2 * j + 1]);
    const float2 r = D::unpack(hv);
    sq = fmaf(r.x, r.x, fmaf(r.y, r.y, sq));
    w[j] = *reinterpret_cast<uint32_t*>(&hv);
  }
  *reinterpret_cast<uint4*>(static_cast<typename D::T*>(base) + idx) = make_uint4(w[0], w[1], w[2], w[3]);
  return sq;
}
// v[0..8) += sum over k-splits sp = 0..split-1 of the 8 floats at src + sp * stride, in split
// order (deterministic); the loads of six splits are issued before any of them is added, so a
// deep split costs ceil(split / 6) L2 round trips, not one per split.
__device__ __forceinline__ void add8(float (&v)[8], const float4& a, const float4& b) {
  v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
  v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
}
__device__ __forceinline__ void sum_partials8(const float* src, int64_t stride, int split, float (&v)[8]) {
  for (int s0 = 0; s0 < split; s0 += 6) {
    float4 a[6], b[6];
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      if (s0 + j < split) {
        const float4* q = reinterpret_cast<const float4*>(src + (s0 + j) * stride);
        a[j] = __ldcg(q);
        b[j] = __ldcg(q + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < 6; ++j)
      if (s0 + j < split) add8(v, a[j], b[j]);
  }
}
// The same for the gate and the up halves of a gate|up tile at once (four splits per round).
__device__ __forceinline__ void sum_partials8x2(const float* src_g, const float* src_u, int64_t stride, int split,
                                                float (&g)[8], float (&u)[8]) {
  for (int s0 = 0; s0 < split; s0 += 4) {
    float4 a[4], b[4], c[4], d[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s0 + j < split) {
        const float4* q = reinterpret_cast<const float4*>(src_g + (s0 + j) * stride);
        const float4* w = reinterpret_cast<const float4*>(src_u + (s0 + j) * stride);
        a[j] = __ldcg(q);
        b[j] = __ldcg(q + 1);
        c[j] = __ldcg(w);
        d[j] = __ldcg(w + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s0 + j < split) {
        add8(g, a[j], b[j]);
        add8(u, c[j], d[j]);
      }
    }
  }
}
// Sum of the `parts` 32-column sums of squares of row `row` ([parts, BM] layout), in part order,
// with eight loads in flight.
__device__ __forceinline__ float row_ssq(const float* ssq, int parts, int row) {
  float t = 0.f;
  for (int i0 = 0; i0 < parts; i0 += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = i0 + j < parts ? __ldcg(ssq + (i0 + j) * BM + row) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += v[j];
  }
  return t;
}
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

// ---- the kernel ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(THREADS, 1) stack_kernel(const __grid_constant__ Params p) {
  using Dx = Dt<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_reg = smem;
  uint8_t* a_reg = smem + W_REGION;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
  int* flag_s = reinterpret_cast<int*>(smem + MISC_OFF + 16);
  float* rstd_s = reinterpret_cast<float*>(smem + RSTD_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned grid = gridDim.x;
  const int L = p.num_layers;
  unsigned* abort = p.counters + abort_word(L);

  if (threadIdx.x == 0) {
    mbar_init(bars + B_W_FULL, 1);
    for (int i = 0; i < MAX_KB; ++i) mbar_init(bars + B_A_FULL + i, 1);
    mbar_init(bars + B_MMA_DONE, 1);
    mbar_init(bars + B_W_FREE, 1);
    mbar_init(bars + B_A_FREE, 1);
    mbar_init(bars + B_ACC_FREE, EPI_THREADS);
    mbar_init(bars + B_S_FULL, 1);
    mbar_init(bars + B_P_FULL, EPI_THREADS);
    mbar_init(bars + B_O_FULL, 1);
    mbar_init(bars + B_O_FREE, EPI_THREADS);
    mbar_init(bars + B_PROD_DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // =================================== TMA producer ===================================
    if (lane == 0) {
      int n_gemm = 0, n_item = 0;
      int w_arms = 0, a_arms[MAX_KB] = {0, 0, 0, 0, 0, 0};
      bool ok = true;
      for (int l = 0; l < L; ++l) {
        const CUtensorMap* lm = p.maps + M_LAYER0 + l * L_MAPS;
        for (int kind = 0; kind < STAGES_PER_LAYER; ++kind) {
          const int s = stage_of(l, kind);
          bool dep = false;
          if (kind == K_ATT) {
            const int items = (p.m / p.seq) * p.heads;
            for (int it = blockIdx.x; it < items; it += grid) {
              ok = ok && (n_item == 0 || wait_bar(bars + B_A_FREE, (n_item - 1) & 1, abort));
              if (ok && !dep) {
                ok = wait_count(p.counters + s - 1, grid, abort);
                fence_proxy_async_global();
                dep = true;
                TK_TRACE(s, EV_DEP);
              }
              if (ok) {
                const int b = it / p.heads, hd = it % p.heads, kvh = hd / (p.heads / p.kv_heads);
                const int row0 = b * p.seq;
                const int xs[3] = {hd * HEAD_DIM, p.q_w + kvh * HEAD_DIM, p.q_w + p.kv_w + kvh * HEAD_DIM};
                const int dst[3] = {ATT_Q, ATT_K, ATT_V};
#pragma unroll
                for (int t = 0; t < 3; ++t) {
                  mbar_arrive_expect_tx(bars + B_A_FULL + t, BM * HEAD_DIM * 2);
                  ++a_arms[t];
                  tma_load_2d(a_reg + dst[t], p.maps + M_QKV, bars + B_A_FULL + t, xs[t], row0);
                }
              }
              ++n_item;
            }
            continue;
          }
          const int gk = kind == K_QKV ? G_QKV : kind - 1;
          const Gemm& G = p.g[gk];
          const CUtensorMap* amap = p.maps + (gk == G_QKV ? M_X : gk == G_O ? M_ATTN : gk == G_GU ? M_H : M_ACT);
          const int items = G.tiles * G.split;
          for (int it = blockIdx.x; it < items; it += grid) {
            const int tile = it / G.split, r = it % G.split;
            const int kb0 = r * G.num_kb / G.split, kb1 = (r + 1) * G.num_kb / G.split;
            // weights first: they do not depend on the previous stage
            ok = ok && (n_gemm == 0 || wait_bar(bars + B_W_FREE, (n_gemm - 1) & 1, abort));
            if (it == static_cast<int>(blockIdx.x)) TK_TRACE(s, EV_W);
            if (ok) {
              mbar_arrive_expect_tx(bars + B_W_FULL, (kb1 - kb0) * G.bn * BK * 2);
              ++w_arms;
              for (int kb = kb0; kb < kb1; ++kb) {
                uint8_t* dst = w_reg + (kb - kb0) * G.bn * BK * 2;
                if (gk == G_GU) {
                  tma_load_2d(dst, lm + L_WG, bars + B_W_FULL, kb * BK, tile * (G.bn / 2));
                  tma_load_2d(dst + (G.bn / 2) * 128, lm + L_WU, bars + B_W_FULL, kb * BK, tile * (G.bn / 2));
                } else if (gk == G_QKV) {
                  const int c0 = tile * G.bn;
                  const int blk = c0 < p.q_w ? L_WQ : (c0 < p.q_w + p.kv_w ? L_WK : L_WV);
                  const int row0 = blk == L_WQ ? c0 : (blk == L_WK ? c0 - p.q_w : c0 - p.q_w - p.kv_w);
                  tma_load_2d(dst, lm + blk, bars + B_W_FULL, kb * BK, row0);
                } else {
                  tma_load_2d(dst, lm + (gk == G_O ? L_WO : L_WD), bars + B_W_FULL, kb * BK, tile * G.bn);
                }
              }
            }
            // then the activations, once the stage they come from is complete
            ok = ok && (n_item == 0 || wait_bar(bars + B_A_FREE, (n_item - 1) & 1, abort));
            if (ok && !dep) {
              ok = wait_count(p.counters + s - 1, grid, abort);
              fence_proxy_async_global();
              dep = true;
              TK_TRACE(s, EV_DEP);
            }
            if (ok) {
              for (int kb = kb0; kb < kb1; ++kb) {
                mbar_arrive_expect_tx(bars + B_A_FULL + (kb - kb0), KB_A_BYTES);
                ++a_arms[kb - kb0];
                tma_load_2d(a_reg + (kb - kb0) * KB_A_BYTES, amap, bars + B_A_FULL + (kb - kb0), kb * BK, 0);
              }
            }
            ++n_gemm;
            ++n_item;
          }
        }
      }
      // wait for this CTA's own copies in flight before it may exit (only ever pending after a
      // failure; bounded, and not cut short by the abort word)
      if (w_arms) mbar_wait(bars + B_W_FULL, (w_arms - 1) & 1);
      for (int i = 0; i < MAX_KB; ++i)
        if (a_arms[i]) mbar_wait(bars + B_A_FULL + i, (a_arms[i] - 1) & 1);
      mbar_arrive(bars + B_PROD_DONE);  // no counter of this launch is polled by this CTA any more
    }
  } else if (warp == 1) {
    // ==================================== MMA issuer ====================================
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_f16(Dx::umma_fmt, BM, BM, 0, 0);
      const uint32_t idesc_o = make_idesc_f16(Dx::umma_fmt, BM, HEAD_DIM, 0, 1);
      const uint32_t w0 = smem_u32(w_reg), a0 = smem_u32(a_reg);
      int n_gemm = 0, n_att = 0;
      uint32_t a_par = 0;  // phase parity of each A_FULL barrier
      bool ok = true;
      auto wait_a = [&](int i) {
        ok = ok && wait_bar(bars + B_A_FULL + i, (a_par >> i) & 1, abort);
        a_par ^= 1u << i;
      };
      for (int l = 0; l < L; ++l) {
        for (int kind = 0; kind < STAGES_PER_LAYER; ++kind) {
          if (kind == K_ATT) {
            const int items = (p.m / p.seq) * p.heads;
            for (int it = blockIdx.x; it < items; it += grid) {
              wait_a(0);
              wait_a(1);
              if (ok) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < HEAD_DIM / 16; ++kk)
                  umma_f16_ss(tmem + T_S, make_sw128_desc(a0 + ATT_Q + kk * 32, 0, 1024),
                              make_sw128_desc(a0 + ATT_K + kk * 32, 0, 1024), idesc_s, kk > 0);
                umma_commit(bars + B_S_FULL);
              }
              ok = ok && wait_bar(bars + B_P_FULL, n_att & 1, abort);
              ok = ok && (n_att == 0 || wait_bar(bars + B_O_FREE, (n_att - 1) & 1, abort));
              wait_a(2);
              if (ok) {
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BM / 16; ++kk)
                  umma_f16_ss(tmem + T_O, make_sw128_desc(a0 + ATT_P + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024),
                              make_sw128_desc(a0 + ATT_V + kk * 16 * 128, BM * 128, 1024), idesc_o, kk > 0);
                umma_commit(bars + B_O_FULL);
                umma_commit(bars + B_A_FREE);
              }
              TK_TRACE(stage_of(l, kind), EV_MMA);
              ++n_att;
            }
            continue;
          }
          const int gk = kind == K_QKV ? G_QKV : kind - 1;
          const Gemm& G = p.g[gk];
          const uint32_t idesc = make_idesc_f16(Dx::umma_fmt, BM, G.bn, 0, 0);
          const int items = G.tiles * G.split;
          for (int it = blockIdx.x; it < items; it += grid) {
            const int r = it % G.split;
            const int nkb = (r + 1) * G.num_kb / G.split - r * G.num_kb / G.split;
            ok = ok && wait_bar(bars + B_W_FULL, n_gemm & 1, abort);
            ok = ok && (n_gemm == 0 || wait_bar(bars + B_ACC_FREE, (n_gemm - 1) & 1, abort));
            for (int kb = 0; kb < nkb; ++kb) {
              wait_a(kb);
              if (ok) {
                tc_fence_after();
                const uint32_t wa = w0 + kb * G.bn * BK * 2, aa = a0 + kb * KB_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                  umma_f16_ss(tmem + T_ACC, make_sw128_desc(aa + kk * 32, 0, 1024),
                              make_sw128_desc(wa + kk * 32, 0, 1024), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              }
            }
            if (ok) {
              umma_commit(bars + B_MMA_DONE);
              umma_commit(bars + B_W_FREE);
              umma_commit(bars + B_A_FREE);
            }
            TK_TRACE(stage_of(l, kind), EV_MMA);
            ++n_gemm;
          }
        }
      }
    }
  } else {
    // ===================================== epilogue =====================================
    const int et = threadIdx.x - 64;                 // 0..127: SIMT work index
    const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
    const int trow = quarter * 32 + lane;            // TMEM row (= output row) of this thread
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int H = p.hidden;
    const int parts = H / 32;
    bool ok = true;
    int n_gemm = 0, n_att = 0;

    // arrive on stage s's counter once every epilogue thread is done with the stage
    auto arrive = [&](int s) {
      __threadfence();
      epi_sync();
      if (et == 0) {
        red_release_add(p.counters + s, 1);
        TK_TRACE(s, EV_ARRIVE);
      }
    };
    // all 128 threads: wait for stage s to be complete (thread 0 polls), ok made uniform
    auto depend = [&](int s) {
      if (et == 0) {
        flag_s[0] = (ok && wait_count(p.counters + s, grid, abort)) ? 1 : 0;
        TK_TRACE(s + 1, EV_EDEP);
      }
      epi_sync();
      ok = ok && flag_s[0] != 0;
      epi_sync();
    };

    // ---- stage 0: token embedding rows and their sums of squares ----
    for (int r = blockIdx.x; r < p.m; r += grid) {
      int64_t tok = p.tokens[r];
      if (tok < 0 || tok >= p.vocab) {
        if (et == 0) record_device_error(TK_DEVERR_TOKEN);
        tok = 0;
      }
      for (int c0 = et * 8; c0 < ((H + 255) / 256) * 256; c0 += EPI_THREADS * 8) {
        float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float sq = 0.f;
        if (c0 < H) {
          load8<DT>(p.emb, tok * H + c0, v);
          sq = store8<DT>(p.x, static_cast<int64_t>(r) * H + c0, v);
        }
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        if (c0 < H && (et & 3) == 0) p.ssq_x[(c0 >> 5) * BM + r] = sq;
      }
    }
    arrive(0);

    for (int l = 0; l < L; ++l) {
      for (int kind = 0; kind < STAGES_PER_LAYER; ++kind) {
        const int s = stage_of(l, kind);
        if (kind == K_ATT) {
          const int items = (p.m / p.seq) * p.heads;
          for (int it = blockIdx.x; it < items; it += grid) {
            const int b = it / p.heads, hd = it % p.heads;
            const int i = trow;  // query row within the sequence's tile
            ok = ok && wait_bar(bars + B_S_FULL, n_att & 1, abort);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
            if (et == 0) TK_TRACE(s, EV_S);
            float l_sum = 1.f;
            if (ok) {
              tc_fence_after();
              // causal within the sequence: key j visible iff j <= i and j < seq. S is read from
              // TMEM in two 64-key halves, twice (maximum, then exponentials), to bound registers.
              const int jmax = min(i, p.seq - 1);
              float mx = -INFINITY;
#pragma unroll 1
              for (int hh = 0; hh < 2; ++hh) {
                float sv[64];
                tmem_load64(tmem + T_S + lane_off + hh * 64, sv);
#pragma unroll
                for (int j = 0; j < 64; ++j)
                  if (hh * 64 + j <= jmax) mx = fmaxf(mx, sv[j]);
              }
              const float neg_m = -mx * p.scale_log2;
              float acc = 0.f;
              uint8_t* prow = a_reg + ATT_P;
#pragma unroll 1
              for (int hh = 0; hh < 2; ++hh) {
                float sv[64];
                tmem_load64(tmem + T_S + lane_off + hh * 64, sv);
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                  sv[j] = hh * 64 + j <= jmax ? exp2_approx(fmaf(sv[j], p.scale_log2, neg_m)) : 0.f;
                  acc += sv[j];
                }
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                  uint32_t w[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    typename Dx::T2 hv = Dx::pack(sv[c * 8 + 2 * q], sv[c * 8 + 2 * q + 1]);
                    w[q] = *reinterpret_cast<uint32_t*>(&hv);
                  }
                  uint8_t* dst = prow + hh * (BM * 128) + i * 128 + (((c & 7) ^ (i & 7)) * 16);
                  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
                }
              }
              l_sum = acc;
              fence_proxy_async_smem();
            }
            tc_fence_before();
            mbar_arrive(bars + B_P_FULL);
            ok = ok && wait_bar(bars + B_O_FULL, n_att & 1, abort);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
            if (et == 0) TK_TRACE(s, EV_O);
            if (ok) {
              tc_fence_after();
              const float inv_l = 1.0f / l_sum;
              const int64_t orow = static_cast<int64_t>(b) * p.seq + i;
#pragma unroll
              for (int c = 0; c < HEAD_DIM; c += 32) {
                float o[32];
                tmem_load32(tmem + T_O + lane_off + c, o);
                if (i < p.seq) {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = o[q * 8 + e] * inv_l;
                    store8<DT>(p.attn, orow * p.q_w + hd * HEAD_DIM + c + q * 8, v);
                  }
                }
              }
            }
            tc_fence_before();
            mbar_arrive(bars + B_O_FREE);
            ++n_att;
          }
          arrive(s);
          continue;
        }

        const int gk = kind == K_QKV ? G_QKV : kind - 1;
        const Gemm& G = p.g[gk];
        const int items = G.tiles * G.split;
        if (static_cast<int>(blockIdx.x) < items) {
          depend(s - 1);  // residual rows and row statistics of earlier stages
          if (gk == G_QKV || gk == G_GU) {  // 1/rms of the input rows of the folded RMSNorm
            const float* ssq = gk == G_QKV ? p.ssq_x : p.ssq_h;
            const float eps = p.eps[2 * l + (gk == G_GU ? 1 : 0)];
            const float t = row_ssq(ssq, parts, et);
            rstd_s[et] = rsqrtf(t * (1.0f / static_cast<float>(H)) + eps);
            epi_sync();
          }
        }
        const int out_per_tile = gk == G_GU ? G.bn / 2 : G.bn;
        const int cpr = out_per_tile / 8;  // 8-column chunks per row
        for (int it = blockIdx.x; it < items; it += grid) {
          const int tile = it / G.split, r = it % G.split;
          float* part = p.partial + static_cast<int64_t>(tile * G.split + r) * BM * G.bn;
          // 1. this k-split's accumulator rows to the partial buffer
          ok = ok && wait_bar(bars + B_MMA_DONE, n_gemm & 1, abort);
          ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
          if (et == 0 && it == static_cast<int>(blockIdx.x)) TK_TRACE(s, EV_ACC);
          if (ok) {
            tc_fence_after();
            float4* dst = reinterpret_cast<float4*>(part + static_cast<int64_t>(trow) * G.bn);
            for (int c = 0; c < G.bn; c += 32) {
              float v[32];
              tmem_load32(tmem + T_ACC + lane_off + c, v);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                __stcg(dst + c / 4 + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
            }
          }
          tc_fence_before();
          mbar_arrive(bars + B_ACC_FREE);
          // 2. wait for the tile's other k-splits
          __threadfence();
          epi_sync();
          if (et == 0 && it == static_cast<int>(blockIdx.x)) TK_TRACE(s, EV_PW);
          if (et == 0) {
            int good = ok ? 1 : 0;
            if (good) {
              unsigned* cnt = p.counters + tile_counter(p, l, gk, tile);
              red_release_add(cnt, 1);
              good = wait_count(cnt, G.split, abort) ? 1 : 0;
              __threadfence();
              if (it == static_cast<int>(blockIdx.x)) TK_TRACE(s, EV_TILE);
            }
            flag_s[0] = good;
          }
          epi_sync();
          ok = ok && flag_s[0] != 0;
          epi_sync();
          // 3. reduce this k-split's share of the tile's (row, 8-column chunk) units - the m * cpr
          // units in even shares whose bounds are multiples of 4, so the four units of a 32-column
          // chunk stay together - then the epilogue. All loads a unit needs (every k-split's
          // partial, the residual, the RoPE angles) go out before any result is used.
          const int total = p.m * cpr;
          const int align = cpr % 4 == 0 ? 4 : 1;  // 4 for the stages that write row statistics
          auto bound = [&](int q) { return q >= G.split ? total : min(total, (q * total / G.split + align - 1) / align * align); };
          const int u0 = bound(r), u1 = bound(r + 1);
          const float* tile_part = p.partial + static_cast<int64_t>(tile * G.split) * BM * G.bn;
          const int64_t pstride = static_cast<int64_t>(BM) * G.bn;
          for (int base = u0; base < u1; base += EPI_THREADS) {
            const int u = base + et;
            const bool valid = ok && u < u1;
            const int row = valid ? u / cpr : 0, ch = valid ? u % cpr : 0;
            float sq = 0.f;
            int col = 0;
            if (valid) {
              if (gk == G_GU) {
                float gv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, uv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                const float* src = tile_part + static_cast<int64_t>(row) * G.bn + ch * 8;
                sum_partials8x2(src, src + G.bn / 2, pstride, G.split, gv, uv);
                col = tile * (G.bn / 2) + ch * 8;
                if (col < G.n) {
                  const float rs = rstd_s[row];
                  float v[8];
#pragma unroll
                  for (int e = 0; e < 8; ++e) v[e] = silu_mul(gv[e] * rs, uv[e] * rs);
                  store8<DT>(p.act, static_cast<int64_t>(row) * p.inter + col, v);
                }
              } else if (gk == G_QKV) {
                col = tile * G.bn + ch * 8;
                const bool rope = col < p.q_w + p.kv_w;
                const int64_t pos = static_cast<int64_t>(p.start_pos) + row % p.seq;
                const int i0 = (col % HEAD_DIM) >> 1;
                float4 c4 = make_float4(1.f, 1.f, 1.f, 1.f), s4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (rope) {
                  c4 = __ldg(reinterpret_cast<const float4*>(p.cos_t + pos * (HEAD_DIM / 2) + i0));
                  s4 = __ldg(reinterpret_cast<const float4*>(p.sin_t + pos * (HEAD_DIM / 2) + i0));
                }
                float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                sum_partials8(tile_part + static_cast<int64_t>(row) * G.bn + ch * 8, pstride, G.split, v);
                const float rs = rstd_s[row];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] *= rs;
                if (rope) {
                  // the projection's value rounded to the model dtype, then the interleaved pair
                  // rotation in fp32 at the row's position (rounded again when stored)
                  const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float x0 = Dx::to_f(Dx::from_f(v[2 * e])), x1 = Dx::to_f(Dx::from_f(v[2 * e + 1]));
                    v[2 * e] = x0 * cs[e] - x1 * sn[e];
                    v[2 * e + 1] = x0 * sn[e] + x1 * cs[e];
                  }
                }
                store8<DT>(p.qkv, static_cast<int64_t>(row) * (p.q_w + 2 * p.kv_w) + col, v);
              } else {
                // o_proj adds x and writes h; down_proj adds h and writes the block output x
                col = tile * G.bn + ch * 8;
                const void* res = gk == G_O ? p.x : p.h;
                void* out = gk == G_O ? p.h : p.x;
                float rv[8];
                load8<DT>(res, static_cast<int64_t>(row) * H + col, rv);
                float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                sum_partials8(tile_part + static_cast<int64_t>(row) * G.bn + ch * 8, pstride, G.split, v);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += rv[e];
                sq = store8<DT>(out, static_cast<int64_t>(row) * H + col, v);
              }
            }
            if (gk == G_O || gk == G_D) {
              // row statistics for the next folded RMSNorm: the four lanes of a 32-column chunk
              sq += __shfl_xor_sync(0xffffffffu, sq, 1);
              sq += __shfl_xor_sync(0xffffffffu, sq, 2);
              if (valid && (et & 3) == 0) (gk == G_O ? p.ssq_h : p.ssq_x)[(col >> 5) * BM + row] = sq;
            }
          }
          if (et == 0) TK_TRACE(s, EV_RED);
          ++n_gemm;
        }
        arrive(s);
      }
    }

    // ---- final RMSNorm of the last block's output ----
    const int sn = norm_stage(L);
    if (static_cast<int>(blockIdx.x) < p.m) depend(sn - 1);
    for (int r = blockIdx.x; ok && r < p.m; r += grid) {
      const float t = row_ssq(p.ssq_x, parts, r);
      const float rs = rsqrtf(t * (1.0f / static_cast<float>(H)) + p.final_eps);
      for (int c0 = et * 8; c0 < H; c0 += EPI_THREADS * 8) {
        float v[8], w[8];
        load8<DT>(p.x, static_cast<int64_t>(r) * H + c0, v);
        load8<DT>(p.final_w, c0, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * rs * w[e];
        store8<DT>(p.y, static_cast<int64_t>(r) * H + c0, v);
      }
    }
    arrive(sn);

    // ---- exit: the last CTA returns every counter to zero for the next launch (once its
    // producer, the only other poller, is done: nobody reads a counter after the reset) ----
    if (et == 0) {
      mbar_wait(bars + B_PROD_DONE, 0);
      flag_s[1] = atomicAdd(p.counters + exit_counter(L), 1u) == grid - 1 ? 1 : 0;
    }
    epi_sync();
    if (flag_s[1]) {
      __threadfence();
      for (int i = et; i < p.n_counters; i += EPI_THREADS) p.counters[i] = 0;
      __threadfence();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct Plan {
  Params p;
  int dtype = 0, grid = 0;
};
std::mutex g_mu;
std::unordered_map<const void*, Plan> g_plans;  // keyed by the scratch pointer

// Tile / k-split plan of one projection: every item's k-range fits the MAX_KB-block W and A
// regions, and the estimated time - rounds of items over the CTAs times the per-CTA bytes
// (weights, the activation k-slice, the fp32 partial written and read back) at ~100 GB/s
// per SM, plus ~1 us for the k-split hand-off - is smallest.
static bool plan_gemm(int n_out, int k, bool swiglu, bool needs_ssq, const int* blocks, int nblocks, int grid,
                      Gemm* out) {
  static const int bns[] = {128, 96, 64, 32};
  const int num_kb = (k + BK - 1) / BK;
  double best = 1e30;
  bool found = false;
  for (int bn : bns) {
    if (swiglu && (bn / 2) % 16) continue;
    if (needs_ssq && bn % 32) continue;  // the row statistics cover 32-column chunks
    if (!swiglu && needs_ssq && (128 % (bn / 8))) continue;
    bool ok = true;
    for (int i = 0; i < nblocks; ++i) ok = ok && blocks[i] % bn == 0;  // tiles never straddle weight blocks
    if (!ok) continue;
    const int per_tile = swiglu ? bn / 2 : bn;
    if ((128 % (per_tile / 8)) != 0) continue;  // 8-column units tile the 128 epilogue threads evenly
    const int tiles = (n_out + per_tile - 1) / per_tile;
    for (int split = 1; split <= MAX_SPLIT; ++split) {
      const int kb_max = (num_kb + split - 1) / split;
      if (kb_max > MAX_KB || split > num_kb) continue;
      const int items = tiles * split;
      const int rounds = (items + grid - 1) / grid;
      const double bytes = kb_max * (bn * BK * 2.0 + KB_A_BYTES) + (split > 1 ? 2.0 * BM * bn * 4 : 0.0);
      const double cost = rounds * (bytes / 100e3 + (split > 1 ? 1.0 : 0.0));
      if (cost < best * 0.98) {
        best = cost;
        *out = Gemm{n_out, k, bn, tiles, split, num_kb};
        found = true;
      }
    }
  }
  return found;
}

struct Layout {
  size_t maps, eps, counters, x, qkv, attn, h, act, ssq_x, ssq_h, partial, total;
  int n_counters, max_tiles;
  Gemm g[4];
};

static int make_layout(int num_layers, int batch, int seq, int hidden, int heads, int kv_heads, int head_dim,
                       int inter, int grid, Layout* L) {
  if (num_layers < 1 || batch < 1 || seq < 1 || static_cast<int64_t>(batch) * seq > BM)
    return fail_invalid("stack: batch * seq must be 1..128 rows");
  if (head_dim != HEAD_DIM) return fail_invalid("stack: head_dim must be 64");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads) return fail_invalid("stack: heads must be a multiple of kv heads");
  if (hidden < 64 || hidden % 64 || inter < 64 || inter % 64)
    return fail_invalid("stack: hidden and intermediate sizes must be multiples of 64");
  const int q_w = heads * head_dim, kv_w = kv_heads * head_dim;
  {
    const int blocks[3] = {q_w, kv_w, kv_w};
    if (!plan_gemm(q_w + 2 * kv_w, hidden, false, false, blocks, 3, grid, &L->g[G_QKV]))
      return fail_invalid("stack: no tile plan for the q|k|v projection");
    const int bo[1] = {hidden};
    if (!plan_gemm(hidden, q_w, false, true, bo, 1, grid, &L->g[G_O]))
      return fail_invalid("stack: no tile plan for o_proj");
    if (!plan_gemm(inter, hidden, true, false, nullptr, 0, grid, &L->g[G_GU]))
      return fail_invalid("stack: no tile plan for gate|up");
    if (!plan_gemm(hidden, inter, false, true, bo, 1, grid, &L->g[G_D]))
      return fail_invalid("stack: no tile plan for down_proj");
  }
  L->max_tiles = 0;
  size_t partial_floats = 0;
  for (const Gemm& g : L->g) {
    L->max_tiles = std::max(L->max_tiles, g.tiles);
    partial_floats = std::max(partial_floats, static_cast<size_t>(g.tiles) * g.split * BM * g.bn);
  }
  L->n_counters = abort_word(num_layers) + 1 + num_layers * 4 * L->max_tiles;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 255) & ~size_t(255);
    return at;
  };
  L->maps = take(sizeof(CUtensorMap) * (M_LAYER0 + L_MAPS * num_layers));
  L->eps = take(sizeof(float) * 2 * num_layers);
  L->counters = take(sizeof(unsigned) * L->n_counters);
  L->x = take(size_t(BM) * hidden * 2);
  L->qkv = take(size_t(BM) * (q_w + 2 * kv_w) * 2);
  L->attn = take(size_t(BM) * q_w * 2);
  L->h = take(size_t(BM) * hidden * 2);
  L->act = take(size_t(BM) * inter * 2);
  L->ssq_x = take(size_t(hidden / 32) * BM * 4);
  L->ssq_h = take(size_t(hidden / 32) * BM * 4);
  L->partial = take(partial_floats * 4);
  L->total = o;
  return TK_OK;
}

static int grid_size(int* grid) {
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  *grid = dev.sm_count;
  return TK_OK;
}

template <int DT>
static int launch(const Plan& pl, cudaStream_t st) {
  auto kern = stack_kernel<DT>;
  static std::mutex mu;
  static int configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev.device]) {
      if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                              "cudaFuncSetAttribute(stack)"))
        return rc;
      int n = 0;
      if (int rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, THREADS, SMEM_BYTES),
                              "cudaOccupancyMaxActiveBlocksPerMultiprocessor(stack)"))
        return rc;
      // one CTA per SM: every CTA resident (the cooperative launch checks it) and the 512 TMEM
      // columns each CTA takes never wait for another CTA's
      if (n != 1) return set_error(TK_ERR_UNSUPPORTED, "stack: expected exactly one resident CTA per SM");
      configured[dev.device] = 1;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, pl.p), "stack_kernel launch");
}

}  // namespace stack
}  // namespace tk

using namespace tk;

extern "C" int64_t tk_stack_scratch_bytes(int num_layers, int batch, int seq, int hidden, int num_heads,
                                          int num_kv_heads, int head_dim, int intermediate) {
  int grid = 0;
  if (stack::grid_size(&grid)) return -1;
  stack::Layout L;
  if (stack::make_layout(num_layers, batch, seq, hidden, num_heads, num_kv_heads, head_dim, intermediate, grid, &L))
    return -1;
  return static_cast<int64_t>(L.total);
}

extern "C" int tk_stack_setup(const tk_stack_layer* layers, int num_layers, int batch, int seq, int hidden,
                              int num_heads, int num_kv_heads, int head_dim, int intermediate, const void* embedding,
                              int64_t vocab, const float* cos_table, const float* sin_table, int64_t table_rows,
                              int start_pos, const void* final_norm_weight, float final_eps, int dtype, void* scratch,
                              int64_t scratch_bytes) {
  using namespace tk::stack;
  if (!half_dtype(dtype)) return fail_invalid("stack: dtype must be F16 or BF16");
  if (!layers || !embedding || !cos_table || !sin_table || !final_norm_weight || !scratch)
    return fail_invalid("stack: NULL pointer");
  if (vocab < 1) return fail_invalid("stack: empty embedding table");
  if (!aligned16(embedding) || !aligned16(final_norm_weight) || !aligned16(cos_table) || !aligned16(sin_table))
    return fail_invalid("stack: embedding, norm weight and RoPE tables must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(scratch) & 255) return fail_invalid("stack: scratch must be 256-byte aligned");
  if (start_pos < 0 || static_cast<int64_t>(start_pos) + seq > table_rows)
    return fail_invalid("stack: positions beyond the RoPE table");
  int grid = 0;
  if (int rc = grid_size(&grid)) return rc;
  Layout L;
  if (int rc = make_layout(num_layers, batch, seq, hidden, num_heads, num_kv_heads, head_dim, intermediate, grid, &L))
    return rc;
  if (scratch_bytes < static_cast<int64_t>(L.total)) return fail_invalid("stack: scratch too small");
  const int q_w = num_heads * head_dim, kv_w = num_kv_heads * head_dim;
  char* base = static_cast<char*>(scratch);
  std::vector<CUtensorMap> maps(M_LAYER0 + L_MAPS * num_layers);
  std::memset(maps.data(), 0, sizeof(CUtensorMap) * maps.size());
  const int m = batch * seq;
  // activation maps: [m rows, K] row-major, box 64 columns x 128 rows (rows >= m read as zeros)
  if (int rc = tensor_map_2d(&maps[M_X], base + L.x, dtype, m, hidden, hidden, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&maps[M_ATTN], base + L.attn, dtype, m, q_w, q_w, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&maps[M_H], base + L.h, dtype, m, hidden, hidden, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&maps[M_ACT], base + L.act, dtype, m, intermediate, intermediate, BM, BK)) return rc;
  if (int rc = tensor_map_2d(&maps[M_QKV], base + L.qkv, dtype, m, q_w + 2 * kv_w, q_w + 2 * kv_w, BM, BK)) return rc;
  std::vector<float> eps(2 * num_layers);
  for (int i = 0; i < num_layers; ++i) {
    const tk_stack_layer& s = layers[i];
    if (!s.wq || !s.wk || !s.wv || !s.wo || !s.wg || !s.wu || !s.wd) return fail_invalid("stack: NULL layer weight");
    for (const void* w : {s.wq, s.wk, s.wv, s.wo, s.wg, s.wu, s.wd})
      if (!aligned16(w)) return fail_invalid("stack: weights must be 16-byte aligned");
    CUtensorMap* lm = &maps[M_LAYER0 + i * L_MAPS];
    const Gemm& gq = L.g[G_QKV];
    const Gemm& go = L.g[G_O];
    const Gemm& gg = L.g[G_GU];
    const Gemm& gd = L.g[G_D];
    if (int rc = tensor_map_2d(&lm[L_WQ], s.wq, dtype, q_w, hidden, hidden, gq.bn, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WK], s.wk, dtype, kv_w, hidden, hidden, gq.bn, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WV], s.wv, dtype, kv_w, hidden, hidden, gq.bn, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WO], s.wo, dtype, hidden, q_w, q_w, go.bn, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WG], s.wg, dtype, intermediate, hidden, hidden, gg.bn / 2, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WU], s.wu, dtype, intermediate, hidden, hidden, gg.bn / 2, BK)) return rc;
    if (int rc = tensor_map_2d(&lm[L_WD], s.wd, dtype, hidden, intermediate, intermediate, gd.bn, BK)) return rc;
    eps[2 * i] = s.eps_attn;
    eps[2 * i + 1] = s.eps_ffn;
  }
  if (int rc = check_cuda(cudaMemset(scratch, 0, L.total), "stack scratch clear")) return rc;
  if (int rc = check_cuda(cudaMemcpy(base + L.maps, maps.data(), sizeof(CUtensorMap) * maps.size(),
                                     cudaMemcpyHostToDevice),
                          "stack tensor maps"))
    return rc;
  if (int rc = check_cuda(cudaMemcpy(base + L.eps, eps.data(), sizeof(float) * eps.size(), cudaMemcpyHostToDevice),
                          "stack eps table"))
    return rc;
  Plan pl;
  Params& p = pl.p;
  p = Params{};
  p.num_layers = num_layers;
  p.m = m;
  p.seq = seq;
  p.hidden = hidden;
  p.heads = num_heads;
  p.kv_heads = num_kv_heads;
  p.inter = intermediate;
  p.q_w = q_w;
  p.kv_w = kv_w;
  p.start_pos = start_pos;
  for (int i = 0; i < 4; ++i) p.g[i] = L.g[i];
  p.maps = reinterpret_cast<const CUtensorMap*>(base + L.maps);
  p.eps = reinterpret_cast<const float*>(base + L.eps);
  p.emb = embedding;
  p.vocab = vocab;
  p.x = base + L.x;
  p.qkv = base + L.qkv;
  p.attn = base + L.attn;
  p.h = base + L.h;
  p.act = base + L.act;
  p.ssq_x = reinterpret_cast<float*>(base + L.ssq_x);
  p.ssq_h = reinterpret_cast<float*>(base + L.ssq_h);
  p.partial = reinterpret_cast<float*>(base + L.partial);
  p.counters = reinterpret_cast<unsigned*>(base + L.counters);
  p.n_counters = L.n_counters;
  p.max_tiles = L.max_tiles;
  p.cos_t = cos_table;
  p.sin_t = sin_table;
  p.table_rows = table_rows;
  p.final_w = final_norm_weight;
  p.final_eps = final_eps;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(head_dim)));
  pl.dtype = dtype;
  pl.grid = grid;
  std::lock_guard<std::mutex> lock(g_mu);
  g_plans[scratch] = pl;
  return TK_OK;
}

extern "C" int tk_stack_forward(const int64_t* tokens, void* y, void* scratch, void* stream) {
  using namespace tk::stack;
  Plan pl;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_plans.find(scratch);
    if (it == g_plans.end()) return fail_invalid("stack: scratch was not prepared by tk_stack_setup");
    pl = it->second;
  }
  if (!tokens || !y || !aligned16(y)) return fail_invalid("stack: tokens and a 16-byte aligned y are required");
  pl.p.tokens = tokens;
  pl.p.y = y;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return pl.dtype == TK_F16 ? launch<TK_F16>(pl, st) : launch<TK_BF16>(pl, st);
}

extern "C" int tk_stack_plan(void* scratch, int* out, int n) {
  using namespace tk::stack;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_plans.find(scratch);
  if (it == g_plans.end()) return fail_invalid("stack: scratch was not prepared by tk_stack_setup");
  const Params& p = it->second.p;
  for (int i = 0; i < 4 && 4 * i + 3 < n; ++i) {
    out[4 * i] = p.g[i].bn;
    out[4 * i + 1] = p.g[i].tiles;
    out[4 * i + 2] = p.g[i].split;
    out[4 * i + 3] = p.g[i].num_kb;
  }
  if (n > 16) out[16] = it->second.grid;
  return TK_OK;
}

extern "C" int tk_stack_trace(void* scratch, unsigned long long* trace) {
  using namespace tk::stack;
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_plans.find(scratch);
  if (it == g_plans.end()) return fail_invalid("stack: scratch was not prepared by tk_stack_setup");
  it->second.p.trace = trace;
  return TK_OK;
}

extern "C" int tk_stack_release(void* scratch) {
  std::lock_guard<std::mutex> lock(tk::stack::g_mu);
  tk::stack::g_plans.erase(scratch);
  return TK_OK;
}
