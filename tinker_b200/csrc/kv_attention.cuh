// Device code of the KV-cache attention shared by its own kernel (kv_attention.cu) and the fused
// decode step (decode_step.cu): launch parameters, helpers, the shared-memory layout and the work of
// one CTA. What it computes and how is described in kv_attention.cu.
#pragma once

#include <math.h>

#include "tk_common.cuh"

namespace tk {
namespace kvattn {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int KT = 32;                   // keys per warp tile, one per lane
constexpr int CHUNK_KEYS = 256;          // keys per CTA at the finest split of the key axis

struct Params {
  const void* q;  // [batch * seq, ...] rows, head h at column h * D (no RoPE yet)
  int64_t qs;
  const void* k;  // new keys (no RoPE yet), head j at column j * D
  int64_t ks;
  const void* v;
  int64_t vs;
  void* kc;  // [batch, num_kv_heads, cap, D] cache, rotated keys
  void* vc;
  int cap;
  const float* cos_t;  // [table_rows, D / 2] float32
  const float* sin_t;
  int64_t table_rows;
  void* out;  // [batch * seq, ...] rows, head h at column h * D
  int64_t os;
  int seq, num_kv_heads, groups, rows;  // rows = groups * seq query rows per (sequence, kv head)
  int start_pos;
  const int* start_dev;  // if set, the position is read from here
  int n_rb, n_chunks;
  float scale_log2;  // log2(e) / sqrt(D)
  int* counters;     // [units] arrival counters, zero between launches
  float2* part_ml;   // [units, n_chunks, rows_cta] (running max, sum)
  float* part_o;     // [units, n_chunks, rows_cta, D]
};

template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t off, float (&f)[8]) {
  using Tr = Dt<DT>;
  // through L2: in the fused decode step these rows are written by other SMs of the same kernel
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const typename Tr::T*>(base) + off));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = Tr::unpack(*reinterpret_cast<const typename Tr::T2*>(&w[j]));
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// Rotate the 4 interleaved pairs in f (pair indices i0..i0+3 of a head) by the angles of
// table row `pos`, round each result to DT; returns the packed values and leaves the rounded
// values in f.
template <int DT>
__device__ __forceinline__ uint4 rope8(float (&f)[8], const Params& p, int64_t pos, int i0, int half_d) {
  using Tr = Dt<DT>;
  const float4 c = *reinterpret_cast<const float4*>(p.cos_t + pos * half_d + i0);
  const float4 s = *reinterpret_cast<const float4*>(p.sin_t + pos * half_d + i0);
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {s.x, s.y, s.z, s.w};
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x0 = f[2 * i], x1 = f[2 * i + 1];
    const typename Tr::T2 h = Tr::pack(x0 * cc[i] - x1 * ss[i], x0 * ss[i] + x1 * cc[i]);
    const float2 r = Tr::unpack(h);
    f[2 * i] = r.x;
    f[2 * i + 1] = r.y;
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int DT>
__device__ __forceinline__ float2 unpack_word(uint32_t w) {
  return Dt<DT>::unpack(*reinterpret_cast<const typename Dt<DT>::T2*>(&w));
}

template <int DT>
__device__ __forceinline__ uint32_t pack_word(float a, float b) {
  const typename Dt<DT>::T2 h = Dt<DT>::pack(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Store DL consecutive fp32 values as DT at `dst` (DL = 2 or 4).
template <int DT, int DL>
__device__ __forceinline__ void store_out(void* dst, const float* v) {
  if constexpr (DL == 2) {
    *reinterpret_cast<uint32_t*>(dst) = pack_word<DT>(v[0], v[1]);
  } else {
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_word<DT>(v[0], v[1]), pack_word<DT>(v[2], v[3]));
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Barrier of the THREADS threads that run an attention item (named barrier 1, so a larger CTA
// whose other warps do something else can run items too).
__device__ __forceinline__ void kv_sync() { asm volatile("bar.sync 1, %0;" ::"n"(THREADS) : "memory"); }

// Shared memory of one CTA: per warp and stage a tile of KT keys (k rows padded by 16 bytes, so
// that the lane-per-key 128-bit reads of a quarter warp fall in distinct banks; v rows dense),
// the CTA's q rows in fp32 and each warp's probabilities. After the key loop the ring holds the
// warps' (max, sum) and O rows for the merge.
template <int D, int R>
struct Smem {
  static constexpr int STAGES = D == 64 ? 3 : 2;
  static constexpr int K_ROW = 2 * D + 16;
  static constexpr int V_ROW = 2 * D;
  static constexpr int K_TILE = KT * K_ROW;
  static constexpr int STAGE = K_TILE + KT * V_ROW;
  static constexpr int RING = STAGES * WARPS * STAGE;
  static constexpr int Q_OFF = RING;                   // float [R][D], pre-scaled by log2(e)/sqrt(D)
  static constexpr int P_OFF = Q_OFF + R * D * 4;      // float [WARPS][R][KT]
  static constexpr int FLAG_OFF = P_OFF + WARPS * R * KT * 4;
  static constexpr int TOTAL = FLAG_OFF + 16;
  static constexpr int ML_BYTES = WARPS * R * 8;       // merge: float2 [WARPS][R] at the ring's start
  static_assert(ML_BYTES % 16 == 0 || R == 1, "merge O rows must stay 16-byte aligned");
  static_assert(32 + WARPS * R * D * 4 + ML_BYTES <= RING, "the merge buffers must fit in the ring");
};

// One CTA's share of a launch: key chunk `chunk` of (sequence b, kv head kvh, row block rb);
// `unit` numbers (b, kvh, rb) for the split-K scratch; `report`: this CTA records a bad position.
// Run by the first THREADS threads of the CTA (named barrier 1), with `smem` 128-byte aligned
// and Smem<D, R>::TOTAL bytes long.
template <int DT, int D, int R>
__device__ __forceinline__ void kv_attention_item(const Params& p, int chunk, int kvh, int rb, int b, int unit,
                                                  bool report, uint8_t* smem) {
  using S = Smem<D, R>;
  using T = typename Dt<DT>::T;
  constexpr int C16 = D / 8;  // 16-byte chunks per row
  constexpr int DL = D / 32;  // output columns per lane (2 or 4)
  constexpr int HALF = D / 2;
  float* q_s = reinterpret_cast<float*>(smem + S::Q_OFF);
  float* p_s = reinterpret_cast<float*>(smem + S::P_OFF);
  int* last_s = reinterpret_cast<int*>(smem + S::FLAG_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int start = p.start_dev ? __ldcg(p.start_dev) : p.start_pos;  // the position may be fresh: read it from L2
  const int64_t end = static_cast<int64_t>(start) + p.seq;
  if (start < 0 || end > p.cap || end > p.table_rows) {
    if (threadIdx.x == 0 && report) record_device_error(TK_DEVERR_POSITION);
    return;
  }
  const int kv_len = static_cast<int>(end);
  // chunks in use for this length (the launch covers the longest): a short context is not split,
  // so it needs no combine; CTAs past them leave before touching memory
  const int n_chunks = min(p.n_chunks, (kv_len + CHUNK_KEYS - 1) / CHUNK_KEYS);
  if (chunk >= n_chunks) return;
  const int n_tiles = (kv_len + KT - 1) / KT;
  const int per = (n_tiles + n_chunks - 1) / n_chunks;  // tiles per chunk
  const int t_lo = chunk * per;
  const int t_hi = min(n_tiles, t_lo + per);
  const int hi = min(kv_len, t_hi * KT);
  const int cached_hi = min(hi, start);  // keys below this come from the cache
  const int64_t cache_row0 = (static_cast<int64_t>(b) * p.num_kv_heads + kvh) * p.cap;
  const T* kc = reinterpret_cast<const T*>(p.kc);
  const T* vc = reinterpret_cast<const T*>(p.vc);
  const uint32_t ring = smem_u32(smem);

  // this warp's tiles: t_lo + warp, t_lo + warp + WARPS, ...
  const int first = t_lo + warp;
  const int n_my = first < t_hi ? (t_hi - first + WARPS - 1) / WARPS : 0;
  auto issue = [&](int i) {  // cp.async of the warp's i-th tile into stage i % STAGES
    const int t = first + WARPS * i;
    const uint32_t kb = ring + ((i % S::STAGES) * WARPS + warp) * S::STAGE;
    const uint32_t vb = kb + S::K_TILE;
#pragma unroll
    for (int j = 0; j < C16; ++j) {
      const int idx = lane + 32 * j;
      const int row = idx / C16, c = idx % C16;
      const int kp = t * KT + row;
      const bool cached = kp < cached_hi;  // new keys are written in after the copy, the rest is zero
      const int64_t off = (cache_row0 + (cached ? kp : 0)) * D + c * 8;
      cp_async16(kb + row * S::K_ROW + c * 16, kc + off, cached ? 16u : 0u);
      cp_async16(vb + row * S::V_ROW + c * 16, vc + off, cached ? 16u : 0u);
    }
  };
#pragma unroll
  for (int i = 0; i < S::STAGES - 1; ++i) {
    if (i < n_my) issue(i);
    cp_async_commit();
  }

  // q rows of the CTA: RoPE at their positions, rounded to DT, times log2(e)/sqrt(D)
  for (int idx = threadIdx.x; idx < R * C16; idx += THREADS) {
    const int lr = idx / C16, c = idx % C16;
    const int gr = rb * R + lr;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (gr < p.rows) {
      const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
      load8<DT>(p.q, (static_cast<int64_t>(b) * p.seq + s) * p.qs + static_cast<int64_t>(h) * D + c * 8, f);
      (void)rope8<DT>(f, p, start + s, c * 4, HALF);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] *= p.scale_log2;
    }
    float4* dst = reinterpret_cast<float4*>(q_s + lr * D + c * 8);
    dst[0] = make_float4(f[0], f[1], f[2], f[3]);
    dst[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  kv_sync();

  float m[R], l[R];
  uint64_t o2[R][DL / 2];  // O columns lane*DL .. lane*DL+DL-1 as packed pairs
  int qpos[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int gr = rb * R + r;
    qpos[r] = gr < p.rows ? start + gr / p.groups : -1;  // -1: padding row, every key masked
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int d = 0; d < DL / 2; ++d) o2[r][d] = 0ull;
  }
  float* pw = p_s + warp * R * KT;

  for (int i = 0; i < n_my; ++i) {
    if (i + S::STAGES - 1 < n_my) issue(i + S::STAGES - 1);
    cp_async_commit();
    cp_async_wait<S::STAGES - 1>();
    __syncwarp();  // every lane's copies of tile i have landed
    const int t0 = (first + WARPS * i) * KT;
    uint8_t* kbuf = smem + ((i % S::STAGES) * WARPS + warp) * S::STAGE;
    uint8_t* vbuf = kbuf + S::K_TILE;
    if (t0 + KT > start && t0 < hi) {
      // the tile holds new keys: rotate them in (and append them to the cache, row block 0)
      const int r0 = max(t0, start), n_new = min(t0 + KT, hi) - r0;
      for (int idx = lane; idx < n_new * C16; idx += 32) {
        const int kp = r0 + idx / C16, c = idx % C16;
        const int64_t trow = static_cast<int64_t>(b) * p.seq + (kp - start);
        float f[8];
        load8<DT>(p.k, trow * p.ks + static_cast<int64_t>(kvh) * D + c * 8, f);
        const uint4 kw = rope8<DT>(f, p, kp, c * 4, HALF);
        const uint4 vw = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.v) + trow * p.vs +
                                                                static_cast<int64_t>(kvh) * D + c * 8));
        *reinterpret_cast<uint4*>(kbuf + (kp - t0) * S::K_ROW + c * 16) = kw;
        *reinterpret_cast<uint4*>(vbuf + (kp - t0) * S::V_ROW + c * 16) = vw;
        if (rb == 0) {
          const int64_t crow = (cache_row0 + kp) * D + c * 8;
          *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.kc) + crow) = kw;
          *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.vc) + crow) = vw;
        }
      }
      __syncwarp();
    }

    // score of key t0 + lane for every row: two packed accumulators per row
    uint64_t acc[R][2];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = 0ull;
    const uint8_t* krow = kbuf + lane * S::K_ROW;
#pragma unroll
    for (int j = 0; j < C16; ++j) {
      const uint4 kw = *reinterpret_cast<const uint4*>(krow + j * 16);
      const float2 k0 = unpack_word<DT>(kw.x), k1 = unpack_word<DT>(kw.y);
      const float2 k2 = unpack_word<DT>(kw.z), k3 = unpack_word<DT>(kw.w);
      const uint64_t kk0 = pack_f32x2(k0.x, k0.y), kk1 = pack_f32x2(k1.x, k1.y);
      const uint64_t kk2 = pack_f32x2(k2.x, k2.y), kk3 = pack_f32x2(k3.x, k3.y);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const ulonglong2 qa = *reinterpret_cast<const ulonglong2*>(q_s + r * D + 8 * j);
        const ulonglong2 qb = *reinterpret_cast<const ulonglong2*>(q_s + r * D + 8 * j + 4);
        acc[r][0] = fma_f32x2(qa.x, kk0, acc[r][0]);
        acc[r][1] = fma_f32x2(qa.y, kk1, acc[r][1]);
        acc[r][0] = fma_f32x2(qb.x, kk2, acc[r][0]);
        acc[r][1] = fma_f32x2(qb.y, kk3, acc[r][1]);
      }
    }
    const int kp = t0 + lane;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float a0, a1, b0, b1;
      unpack_f32x2(acc[r][0], a0, a1);
      unpack_f32x2(acc[r][1], b0, b1);
      const float sr = (kp < hi && kp <= qpos[r]) ? (a0 + a1) + (b0 + b1) : -INFINITY;
      const float mn = fmaxf(m[r], warp_max(sr));
      float pr = 0.f;
      if (mn != -INFINITY) {  // warp-uniform: some key of this row seen so far
        pr = exp2_approx(sr - mn);
        if (mn != m[r]) {
          const float alpha = exp2_approx(m[r] - mn);
          const uint64_t a2 = pack_f32x2(alpha, alpha);
          l[r] *= alpha;
#pragma unroll
          for (int d = 0; d < DL / 2; ++d) o2[r][d] = fma_f32x2(o2[r][d], a2, 0ull);
        }
        m[r] = mn;
      }
      l[r] += pr;  // per-lane partial sum, reduced after the loop
      pw[r * KT + lane] = pr;
    }
    __syncwarp();

    // O += P V over the tile's keys
#pragma unroll 2
    for (int k = 0; k < KT; k += 4) {
      float4 p4[R];
#pragma unroll
      for (int r = 0; r < R; ++r) p4[r] = *reinterpret_cast<const float4*>(pw + r * KT + k);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint64_t vv[DL / 2];
        if constexpr (DL == 2) {
          const float2 v = unpack_word<DT>(*reinterpret_cast<const uint32_t*>(vbuf + (k + kk) * S::V_ROW + lane * 4));
          vv[0] = pack_f32x2(v.x, v.y);
        } else {
          const uint2 w = *reinterpret_cast<const uint2*>(vbuf + (k + kk) * S::V_ROW + lane * 8);
          const float2 v0 = unpack_word<DT>(w.x), v1 = unpack_word<DT>(w.y);
          vv[0] = pack_f32x2(v0.x, v0.y);
          vv[1] = pack_f32x2(v1.x, v1.y);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float pk = kk == 0 ? p4[r].x : kk == 1 ? p4[r].y : kk == 2 ? p4[r].z : p4[r].w;
          const uint64_t pp = pack_f32x2(pk, pk);
#pragma unroll
          for (int d = 0; d < DL / 2; ++d) o2[r][d] = fma_f32x2(pp, vv[d], o2[r][d]);
        }
      }
    }
    __syncwarp();  // the stage and pw are rewritten by the next iterations
  }
  cp_async_wait<0>();
  pdl_launch_dependents();
#pragma unroll
  for (int r = 0; r < R; ++r) l[r] = warp_sum(l[r]);

  // merge the warps' rows in shared memory (the ring is free now)
  kv_sync();
  float2* ml_s = reinterpret_cast<float2*>(smem);                 // [WARPS][R]
  float* o_s = reinterpret_cast<float*>(smem + (S::ML_BYTES + 15) / 16 * 16);  // [WARPS][R][D]
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (lane == 0) ml_s[warp * R + r] = make_float2(m[r], l[r]);
    float* dst = o_s + (warp * R + r) * D + lane * DL;
    if constexpr (DL == 2) {
      *reinterpret_cast<uint64_t*>(dst) = o2[r][0];
    } else {
      *reinterpret_cast<ulonglong2*>(dst) = make_ulonglong2(o2[r][0], o2[r][1]);
    }
  }
  kv_sync();

  constexpr int D4 = D / 4;
  for (int idx = threadIdx.x; idx < R * D4; idx += THREADS) {
    const int r = idx / D4, d = (idx % D4) * 4;
    const int gr = rb * R + r;
    if (gr >= p.rows) continue;
    float M = -INFINITY, L = 0.f;
    float acc4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float2 ml = ml_s[w * R + r];
      if (ml.y == 0.f) continue;  // no key of this row in warp w's tiles
      const float4 ov = *reinterpret_cast<const float4*>(o_s + (w * R + r) * D + d);
      const float mn = fmaxf(M, ml.x);
      const float a = exp2_approx(M - mn), e = exp2_approx(ml.x - mn);
      L = L * a + ml.y * e;
      acc4[0] = acc4[0] * a + ov.x * e;
      acc4[1] = acc4[1] * a + ov.y * e;
      acc4[2] = acc4[2] * a + ov.z * e;
      acc4[3] = acc4[3] * a + ov.w * e;
      M = mn;
    }
    if (n_chunks == 1) {  // the only chunk: normalise and store
      const float inv = 1.f / L;
      float v[4] = {acc4[0] * inv, acc4[1] * inv, acc4[2] * inv, acc4[3] * inv};
      const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
      store_out<DT, 4>(reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.seq + s) * p.os +
                           static_cast<int64_t>(h) * D + d, v);
    } else {
      const int64_t slot = (static_cast<int64_t>(unit) * p.n_chunks + chunk) * R + r;
      if (d == 0) p.part_ml[slot] = make_float2(M, L);
      *reinterpret_cast<float4*>(p.part_o + slot * D + d) = make_float4(acc4[0], acc4[1], acc4[2], acc4[3]);
    }
  }
  if (n_chunks == 1) return;

  __threadfence();
  kv_sync();
  if (threadIdx.x == 0) *last_s = atomicAdd(p.counters + unit, 1) == n_chunks - 1;
  kv_sync();
  if (!*last_s) return;
  __threadfence();

  // last CTA of this unit: merge the chunks' partial rows
  for (int idx = threadIdx.x; idx < R * D4; idx += THREADS) {
    const int r = idx / D4, d = (idx % D4) * 4;
    const int gr = rb * R + r;
    if (gr >= p.rows) continue;
    float M = -INFINITY, L = 0.f;
    float acc4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < n_chunks; ++c) {
      const int64_t slot = (static_cast<int64_t>(unit) * p.n_chunks + c) * R + r;
      const float2 ml = __ldcg(p.part_ml + slot);
      if (ml.y == 0.f) continue;  // no key of this row in chunk c
      const float4 ov = __ldcg(reinterpret_cast<const float4*>(p.part_o + slot * D + d));
      const float mn = fmaxf(M, ml.x);
      const float a = exp2_approx(M - mn), e = exp2_approx(ml.x - mn);
      L = L * a + ml.y * e;
      acc4[0] = acc4[0] * a + ov.x * e;
      acc4[1] = acc4[1] * a + ov.y * e;
      acc4[2] = acc4[2] * a + ov.z * e;
      acc4[3] = acc4[3] * a + ov.w * e;
      M = mn;
    }
    const float inv = 1.f / L;
    float v[4] = {acc4[0] * inv, acc4[1] * inv, acc4[2] * inv, acc4[3] * inv};
    const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
    store_out<DT, 4>(reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.seq + s) * p.os +
                         static_cast<int64_t>(h) * D + d, v);
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;  // ready for the next launch
}

// Launch shape of one kv_attention launch and its split-K scratch (host side, kv_attention.cu).
struct Plan {
  int rows_cta, n_rb, n_chunks;
  int64_t units;
  size_t counters_bytes, ml_bytes, o_bytes;
  size_t bytes() const { return n_chunks > 1 ? counters_bytes + ml_bytes + o_bytes : 0; }
};

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Rows per CTA, row blocks and key chunks for `rows` query rows per (sequence, kv head) attending
// to at most `max_kv` keys.
Plan make_plan(int batch, int num_kv_heads, int rows, int max_kv, int head_dim, int sm_count);

}  // namespace kvattn
}  // namespace tk
