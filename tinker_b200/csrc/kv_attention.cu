// Attention of a few new tokens per sequence against a KV cache (decode steps and short
// chunks), plus the plain cache append used after a prompt's tensor-core attention.
//
// What it computes: for a sequence whose keys/values 0..start-1 are cached and whose S new
// tokens sit at positions start..start+S-1, rows start..start+S-1 of the reference's causal
// RoPE + GQA attention over the whole sequence (tinker/kernels/fused_attention.py:176-192;
// mask q >= kv :132, scale 1/sqrt(D) :216, interleaved RoPE :44-69 with fp32 angles). The
// reference has no cache and recomputes the whole sequence for every new token
// (tinker/modules/attention.py:51 only shifts the RoPE positions); here every cached key is
// read once per step.
//
// One launch, per (key chunk, kv head x row block, sequence) CTA:
//   * RoPE of the new q rows and k rows at their positions (fp32 angles, each result rounded
//     to the model dtype, as the projection epilogue does on the prompt path);
//   * the append of the new rotated k rows and v rows to the cache (row block 0 only; no
//     other CTA of the launch reads those cache rows, they take them from the inputs);
//   * flash-decoding over a contiguous key range: the rows of a CTA are the query rows of
//     the `groups` query heads that share its kv head, so a key/value tile in shared memory
//     serves all of them; two keys per lane for q.k, running max/sum per row, p.V with the
//     lane owning D/32 output columns;
//   * the split-K combine: each CTA stores (max, sum, unnormalised O) of its rows, the last
//     CTA of a (sequence, kv head, row block) to arrive (atomic counter, reset by that CTA)
//     merges them. No CTA waits for another.
// The position may come from device memory (`start_dev`), so one CUDA graph serves every
// decode step; an out-of-range position records TK_DEVERR_POSITION and leaves `out` as is.
// The work is memory-bound (2 * kv_len * D * 2 bytes per kv head and sequence against
// 4 * groups * kv_len * D flops): SIMT, not tensor cores.
#include <math.h>

#include <algorithm>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace kvattn {

constexpr int THREADS = 128;
constexpr int WARPS = THREADS / 32;
constexpr int KT = 64;  // keys per shared-memory tile (two per lane)

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
  const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const typename Tr::T*>(base) + off);
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

template <int DT, int D, int RPW>
__global__ void __launch_bounds__(THREADS) kv_attention_kernel(const Params p) {
  using T = typename Dt<DT>::T;
  constexpr int R = WARPS * RPW;  // query rows per CTA; warp w owns rows w, w + WARPS, ...
  constexpr int C8 = D / 8;       // 16-byte chunks per row
  constexpr int KW = D / 2 + 1;   // padded k row in words: lanes reading different keys hit different banks
  constexpr int VW = D / 2;
  constexpr int DL = D / 32;      // output columns per lane
  __shared__ __align__(16) float q_s[R][D];
  __shared__ uint32_t k_s[KT][KW];
  __shared__ __align__(16) uint32_t v_s[KT][VW];
  __shared__ __align__(16) float p_s[R][KT];
  __shared__ int last_s;

  const int chunk = blockIdx.x;
  const int kvh = blockIdx.y / p.n_rb;
  const int rb = blockIdx.y % p.n_rb;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int HALF = D / 2;

  pdl_wait();  // q/k/v come from the previous kernel; the position may be written by a copy before it
  const int start = p.start_dev ? *p.start_dev : p.start_pos;
  const int64_t end = static_cast<int64_t>(start) + p.seq;
  if (start < 0 || end > p.cap || end > p.table_rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
      record_device_error(TK_DEVERR_POSITION);
    return;
  }
  const int kv_len = static_cast<int>(end);
  const int n_tiles = (kv_len + KT - 1) / KT;
  const int per = (n_tiles + p.n_chunks - 1) / p.n_chunks;  // tiles per chunk
  const int lo = chunk * per * KT;
  const int hi = min(kv_len, lo + per * KT);
  const int64_t cache_row0 = (static_cast<int64_t>(b) * p.num_kv_heads + kvh) * p.cap;
  const T* kc_in = reinterpret_cast<const T*>(p.kc);
  const T* vc_in = reinterpret_cast<const T*>(p.vc);

  float m[RPW], l[RPW], o[RPW][DL];
  int qpos[RPW];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int gr = rb * R + warp + WARPS * i;
    qpos[i] = gr < p.rows ? start + gr / p.groups : -1;  // -1: padding row, every key masked
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) o[i][d] = 0.f;
  }

  if (lo < hi) {
    // q rows: RoPE at their positions, rounded to DT, times log2(e)/sqrt(D)
    for (int idx = threadIdx.x; idx < R * C8; idx += THREADS) {
      const int lr = idx / C8, c = idx % C8;
      const int gr = rb * R + lr;
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (gr < p.rows) {
        const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
        load8<DT>(p.q, (static_cast<int64_t>(b) * p.seq + s) * p.qs + static_cast<int64_t>(h) * D + c * 8, f);
        (void)rope8<DT>(f, p, start + s, c * 4, HALF);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] *= p.scale_log2;
      }
      float4* dst = reinterpret_cast<float4*>(&q_s[lr][c * 8]);
      dst[0] = make_float4(f[0], f[1], f[2], f[3]);
      dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    }

    for (int t0 = lo; t0 < hi; t0 += KT) {
      __syncthreads();  // q_s written; the previous tile's k_s / v_s / p_s reads are done
      for (int idx = threadIdx.x; idx < KT * C8; idx += THREADS) {
        const int key = idx / C8, c = idx % C8;
        const int kp = t0 + key;
        uint4 kw = make_uint4(0, 0, 0, 0), vw = make_uint4(0, 0, 0, 0);
        if (kp < hi) {
          const int64_t crow = (cache_row0 + kp) * D + c * 8;
          if (kp < start) {
            kw = *reinterpret_cast<const uint4*>(kc_in + crow);
            vw = *reinterpret_cast<const uint4*>(vc_in + crow);
          } else {
            const int64_t trow = static_cast<int64_t>(b) * p.seq + (kp - start);
            float f[8];
            load8<DT>(p.k, trow * p.ks + static_cast<int64_t>(kvh) * D + c * 8, f);
            kw = rope8<DT>(f, p, kp, c * 4, HALF);
            vw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.v) + trow * p.vs +
                                                 static_cast<int64_t>(kvh) * D + c * 8);
            if (rb == 0) {
              *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.kc) + crow) = kw;
              *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.vc) + crow) = vw;
            }
          }
        }
        uint32_t* kd = &k_s[key][c * 4];
        kd[0] = kw.x;
        kd[1] = kw.y;
        kd[2] = kw.z;
        kd[3] = kw.w;
        *reinterpret_cast<uint4*>(&v_s[key][c * 4]) = vw;
      }
      __syncthreads();

      // scores of keys t0 + lane and t0 + lane + 32 for each of the warp's rows
      float sc[RPW][2];
#pragma unroll
      for (int i = 0; i < RPW; ++i) sc[i][0] = sc[i][1] = 0.f;
#pragma unroll 4
      for (int w2 = 0; w2 < D / 4; ++w2) {
        const float2 a0 = unpack_word<DT>(k_s[lane][2 * w2]);
        const float2 a1 = unpack_word<DT>(k_s[lane][2 * w2 + 1]);
        const float2 b0 = unpack_word<DT>(k_s[lane + 32][2 * w2]);
        const float2 b1 = unpack_word<DT>(k_s[lane + 32][2 * w2 + 1]);
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          const float4 qv = *reinterpret_cast<const float4*>(&q_s[warp + WARPS * i][4 * w2]);
          sc[i][0] = fmaf(qv.x, a0.x, fmaf(qv.y, a0.y, fmaf(qv.z, a1.x, fmaf(qv.w, a1.y, sc[i][0]))));
          sc[i][1] = fmaf(qv.x, b0.x, fmaf(qv.y, b0.y, fmaf(qv.z, b1.x, fmaf(qv.w, b1.y, sc[i][1]))));
        }
      }
      const int kp0 = t0 + lane, kp1 = t0 + lane + 32;
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const float s0 = (kp0 < hi && kp0 <= qpos[i]) ? sc[i][0] : -INFINITY;
        const float s1 = (kp1 < hi && kp1 <= qpos[i]) ? sc[i][1] : -INFINITY;
        const float mn = fmaxf(m[i], warp_max(fmaxf(s0, s1)));
        float p0 = 0.f, p1 = 0.f, alpha = 1.f;
        if (mn != -INFINITY) {  // some key of this row seen so far
          alpha = exp2f(m[i] - mn);
          p0 = exp2f(s0 - mn);
          p1 = exp2f(s1 - mn);
        }
        m[i] = mn;
        l[i] = l[i] * alpha + (p0 + p1);  // per-lane partial sum, reduced at the end
#pragma unroll
        for (int d = 0; d < DL; ++d) o[i][d] *= alpha;
        p_s[warp + WARPS * i][lane] = p0;
        p_s[warp + WARPS * i][lane + 32] = p1;
      }
      __syncwarp();

      // O += P V over the tile's keys (the lane's DL columns)
      const int kn = min(KT, hi - t0);
      for (int k4 = 0; k4 < kn; k4 += 4) {
        float4 pv[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) pv[i] = *reinterpret_cast<const float4*>(&p_s[warp + WARPS * i][k4]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          float vv[DL];
          if constexpr (DL == 2) {
            const float2 t = unpack_word<DT>(v_s[k4 + kk][lane]);
            vv[0] = t.x;
            vv[1] = t.y;
          } else {
            const uint2 w = *reinterpret_cast<const uint2*>(&v_s[k4 + kk][2 * lane]);
            const float2 t0v = unpack_word<DT>(w.x), t1v = unpack_word<DT>(w.y);
            vv[0] = t0v.x;
            vv[1] = t0v.y;
            vv[2] = t1v.x;
            vv[3] = t1v.y;
          }
#pragma unroll
          for (int i = 0; i < RPW; ++i) {
            const float pk = kk == 0 ? pv[i].x : kk == 1 ? pv[i].y : kk == 2 ? pv[i].z : pv[i].w;
#pragma unroll
            for (int d = 0; d < DL; ++d) o[i][d] = fmaf(pk, vv[d], o[i][d]);
          }
        }
      }
    }
  }
  pdl_launch_dependents();
#pragma unroll
  for (int i = 0; i < RPW; ++i) l[i] = warp_sum(l[i]);

  if (p.n_chunks == 1) {  // the only chunk: normalise and store
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      if (qpos[i] < 0) continue;
      const int gr = rb * R + warp + WARPS * i;
      const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
      const float inv = 1.f / l[i];
      float v[DL];
#pragma unroll
      for (int d = 0; d < DL; ++d) v[d] = o[i][d] * inv;
      T* dst = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.seq + s) * p.os +
               static_cast<int64_t>(h) * D + lane * DL;
      store_out<DT, DL>(dst, v);
    }
    return;
  }

  const int unit = b * gridDim.y + blockIdx.y;
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int64_t slot = (static_cast<int64_t>(unit) * p.n_chunks + chunk) * R + warp + WARPS * i;
    if (lane == 0) p.part_ml[slot] = make_float2(m[i], l[i]);
    float* dst = p.part_o + slot * D + lane * DL;
    if constexpr (DL == 2) {
      *reinterpret_cast<float2*>(dst) = make_float2(o[i][0], o[i][1]);
    } else {
      *reinterpret_cast<float4*>(dst) = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(p.counters + unit, 1) == p.n_chunks - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();

  // last CTA of this unit: merge the chunks' partial rows
  constexpr int D4 = D / 4;
  for (int idx = threadIdx.x; idx < R * D4; idx += THREADS) {
    const int lr = idx / D4, d = (idx % D4) * 4;
    const int gr = rb * R + lr;
    if (gr >= p.rows) continue;
    float M = -INFINITY, L = 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < p.n_chunks; ++c) {
      const int64_t slot = (static_cast<int64_t>(unit) * p.n_chunks + c) * R + lr;
      const float2 ml = __ldcg(p.part_ml + slot);
      if (ml.y == 0.f) continue;  // no key of this row in chunk c
      const float4 ov = __ldcg(reinterpret_cast<const float4*>(p.part_o + slot * D + d));
      const float mn = fmaxf(M, ml.x);
      const float a = exp2f(M - mn), w = exp2f(ml.x - mn);
      L = L * a + ml.y * w;
      acc[0] = acc[0] * a + ov.x * w;
      acc[1] = acc[1] * a + ov.y * w;
      acc[2] = acc[2] * a + ov.z * w;
      acc[3] = acc[3] * a + ov.w * w;
      M = mn;
    }
    const float inv = 1.f / L;
    float v[4] = {acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv};
    const int s = gr / p.groups, h = kvh * p.groups + gr % p.groups;
    T* dst = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.seq + s) * p.os +
             static_cast<int64_t>(h) * D + d;
    store_out<DT, 4>(dst, v);
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;  // ready for the next launch
}

// Copy S new rows of k (already rotated) and v per sequence into the cache at `start`.
template <int DT>
__global__ void __launch_bounds__(256) kv_append_kernel(const void* k, int64_t ks, const void* v, int64_t vs,
                                                         void* kc, void* vc, int seq, int num_kv_heads, int d8,
                                                         int cap, int start, int64_t total) {
  using T = typename Dt<DT>::T;
  pdl_wait();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  // idx = ((b * seq + s) * num_kv_heads + j) * d8 + c
  const int c = static_cast<int>(idx % d8);
  const int64_t r = idx / d8;
  const int j = static_cast<int>(r % num_kv_heads);
  const int64_t t = r / num_kv_heads;  // b * seq + s
  const int64_t bb = t / seq;
  const int s = static_cast<int>(t - bb * seq);
  const int D = d8 * 8;
  const int64_t col = static_cast<int64_t>(j) * D + c * 8;
  const int64_t crow = ((bb * num_kv_heads + j) * cap + start + s) * D + c * 8;
  const uint4 kw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(k) + t * ks + col);
  const uint4 vw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(v) + t * vs + col);
  pdl_launch_dependents();
  *reinterpret_cast<uint4*>(reinterpret_cast<T*>(kc) + crow) = kw;
  *reinterpret_cast<uint4*>(reinterpret_cast<T*>(vc) + crow) = vw;
}

struct Plan {
  int rpw, rows_cta, n_rb, n_chunks;
  int64_t units;
  size_t counters_bytes, ml_bytes, o_bytes;
  size_t bytes() const { return n_chunks > 1 ? counters_bytes + ml_bytes + o_bytes : 0; }
};

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Rows per CTA, row blocks and key chunks for a launch whose key count is at most `max_kv`;
// about two CTAs per SM unless the keys run out. The workspace a plan needs grows with max_kv.
Plan make_plan(int batch, int num_kv_heads, int rows, int max_kv, int head_dim, int sm_count) {
  Plan pl{};
  pl.rpw = rows <= WARPS ? 1 : rows <= 2 * WARPS ? 2 : 4;
  pl.rows_cta = WARPS * pl.rpw;
  pl.n_rb = (rows + pl.rows_cta - 1) / pl.rows_cta;
  pl.units = static_cast<int64_t>(batch) * num_kv_heads * pl.n_rb;
  const int max_tiles = std::max(1, (max_kv + KT - 1) / KT);
  const int64_t target = 2 * static_cast<int64_t>(std::max(sm_count, 1));
  pl.n_chunks = static_cast<int>(std::min<int64_t>(max_tiles, std::max<int64_t>(1, (target + pl.units - 1) / pl.units)));
  pl.counters_bytes = round_up(static_cast<size_t>(pl.units) * sizeof(int), 256);
  const size_t slots = static_cast<size_t>(pl.units) * pl.n_chunks * pl.rows_cta;
  pl.ml_bytes = round_up(slots * sizeof(float2), 256);
  pl.o_bytes = slots * head_dim * sizeof(float);
  return pl;
}

int check_sizes(const char* what, int batch, int seq, int num_heads, int num_kv_heads, int head_dim, int cap,
                int dtype) {
  const std::string w(what);
  if (!half_dtype(dtype)) return fail_invalid(w + ": dtype must be F16 or BF16");
  if (head_dim != 64 && head_dim != 128) return set_error(TK_ERR_UNSUPPORTED, w + ": head_dim must be 64 or 128");
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0 || cap < 0) return fail_invalid(w + ": invalid sizes");
  if (num_heads % num_kv_heads != 0) return fail_invalid(w + ": num_heads must be a multiple of num_kv_heads");
  if (batch > 65535) return fail_invalid(w + ": too many sequences");
  return TK_OK;
}

template <int DT, int D, int RPW>
int launch(const Params& p, dim3 grid, cudaStream_t st) {
  return launch_kernel(kv_attention_kernel<DT, D, RPW>, grid, dim3(THREADS), 0, st, 1, "kv_attention", p);
}

template <int DT, int D>
int launch_rpw(int rpw, const Params& p, dim3 grid, cudaStream_t st) {
  switch (rpw) {
    case 1: return launch<DT, D, 1>(p, grid, st);
    case 2: return launch<DT, D, 2>(p, grid, st);
    default: return launch<DT, D, 4>(p, grid, st);
  }
}

}  // namespace kvattn
}  // namespace tk

extern "C" int64_t tk_kv_attention_workspace(int batch, int num_heads, int num_kv_heads, int head_dim, int seq,
                                             int max_kv) {
  using namespace tk;
  if (batch <= 0 || seq <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || max_kv <= 0)
    return 0;
  DeviceInfo di;
  if (current_device_info(&di)) return -1;
  const int rows = num_heads / num_kv_heads * seq;
  return static_cast<int64_t>(kvattn::make_plan(batch, num_kv_heads, rows, max_kv, head_dim, di.sm_count).bytes());
}

extern "C" int tk_kv_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                               const void* v, int64_t v_tok_stride, void* k_cache, void* v_cache, int capacity,
                               const float* cos_table, const float* sin_table, int64_t table_rows, void* out,
                               int64_t out_tok_stride, int batch, int seq, int num_heads, int num_kv_heads,
                               int head_dim, int start_pos, const int* start_pos_device, void* workspace,
                               int64_t workspace_bytes, int dtype, void* stream) {
  using namespace tk;
  using namespace tk::kvattn;
  if (int rc = check_sizes("kv_attention", batch, seq, num_heads, num_kv_heads, head_dim, capacity, dtype)) return rc;
  if (q_tok_stride < int64_t(num_heads) * head_dim || k_tok_stride < int64_t(num_kv_heads) * head_dim ||
      v_tok_stride < int64_t(num_kv_heads) * head_dim || out_tok_stride < int64_t(num_heads) * head_dim)
    return fail_invalid("kv_attention: token stride smaller than heads * head_dim");
  if (q_tok_stride % 8 || k_tok_stride % 8 || v_tok_stride % 8 || out_tok_stride % 8)
    return fail_invalid("kv_attention: token strides must be multiples of 8 elements");
  if (!start_pos_device) {
    if (start_pos < 0) return fail_invalid("kv_attention: start_pos must be >= 0");
    if (int64_t(start_pos) + seq > capacity) return fail_invalid("kv_attention: start_pos + seq exceeds the cache");
    if (int64_t(start_pos) + seq > table_rows)
      return fail_invalid("kv_attention: start_pos + seq exceeds the RoPE table length");
  }
  if (batch == 0 || seq == 0) return TK_OK;
  if (!q || !k || !v || !k_cache || !v_cache || !cos_table || !sin_table || !out)
    return fail_invalid("kv_attention: NULL pointer");
  for (const void* ptr : {q, k, v, static_cast<const void*>(k_cache), static_cast<const void*>(v_cache),
                          static_cast<const void*>(cos_table), static_cast<const void*>(sin_table),
                          static_cast<const void*>(out)})
    if (!aligned16(ptr)) return fail_invalid("kv_attention: pointers must be 16-byte aligned");
  DeviceInfo di;
  if (int rc = current_device_info(&di)) return rc;
  const int rows = num_heads / num_kv_heads * seq;
  // with a device position the launch must cover any position: plan for a full cache
  const int max_kv = start_pos_device ? capacity : start_pos + seq;
  const Plan pl = make_plan(batch, num_kv_heads, rows, max_kv, head_dim, di.sm_count);
  if (int64_t(num_kv_heads) * pl.n_rb > 65535) return fail_invalid("kv_attention: too many query rows per kv head");
  if (pl.bytes() > 0) {
    if (!workspace || workspace_bytes < static_cast<int64_t>(pl.bytes()))
      return fail_invalid("kv_attention: workspace missing or smaller than tk_kv_attention_workspace()");
    if (!aligned16(workspace)) return fail_invalid("kv_attention: workspace must be 16-byte aligned");
  }
  Params p{};
  p.q = q;
  p.qs = q_tok_stride;
  p.k = k;
  p.ks = k_tok_stride;
  p.v = v;
  p.vs = v_tok_stride;
  p.kc = k_cache;
  p.vc = v_cache;
  p.cap = capacity;
  p.cos_t = cos_table;
  p.sin_t = sin_table;
  p.table_rows = table_rows;
  p.out = out;
  p.os = out_tok_stride;
  p.seq = seq;
  p.num_kv_heads = num_kv_heads;
  p.groups = num_heads / num_kv_heads;
  p.rows = rows;
  p.start_pos = start_pos;
  p.start_dev = start_pos_device;
  p.n_rb = pl.n_rb;
  p.n_chunks = pl.n_chunks;
  p.scale_log2 = static_cast<float>((1.0 / std::sqrt(double(head_dim))) * 1.4426950408889634);
  if (pl.bytes() > 0) {
    char* ws = static_cast<char*>(workspace);
    p.counters = reinterpret_cast<int*>(ws);
    p.part_ml = reinterpret_cast<float2*>(ws + pl.counters_bytes);
    p.part_o = reinterpret_cast<float*>(ws + pl.counters_bytes + pl.ml_bytes);
  }
  const dim3 grid(pl.n_chunks, num_kv_heads * pl.n_rb, batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return head_dim == 64 ? launch_rpw<TK_F16, 64>(pl.rpw, p, grid, st) : launch_rpw<TK_F16, 128>(pl.rpw, p, grid, st);
  return head_dim == 64 ? launch_rpw<TK_BF16, 64>(pl.rpw, p, grid, st) : launch_rpw<TK_BF16, 128>(pl.rpw, p, grid, st);
}

extern "C" int tk_kv_append(const void* k, int64_t k_tok_stride, const void* v, int64_t v_tok_stride, void* k_cache,
                            void* v_cache, int capacity, int batch, int seq, int num_kv_heads, int head_dim,
                            int start_pos, int dtype, void* stream) {
  using namespace tk;
  using namespace tk::kvattn;
  if (int rc = check_sizes("kv_append", batch, seq, num_kv_heads, num_kv_heads, head_dim, capacity, dtype)) return rc;
  if (k_tok_stride < int64_t(num_kv_heads) * head_dim || v_tok_stride < int64_t(num_kv_heads) * head_dim)
    return fail_invalid("kv_append: token stride smaller than num_kv_heads * head_dim");
  if (k_tok_stride % 8 || v_tok_stride % 8) return fail_invalid("kv_append: token strides must be multiples of 8 elements");
  if (start_pos < 0 || int64_t(start_pos) + seq > capacity)
    return fail_invalid("kv_append: start_pos + seq exceeds the cache");
  if (batch == 0 || seq == 0) return TK_OK;
  if (!k || !v || !k_cache || !v_cache) return fail_invalid("kv_append: NULL pointer");
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail_invalid("kv_append: pointers must be 16-byte aligned");
  const int64_t total = int64_t(batch) * seq * num_kv_heads * (head_dim / 8);
  const int64_t blocks = (total + 255) / 256;
  if (blocks > 0x7fffffff) return fail_invalid("kv_append: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16)
    return launch_kernel(kv_append_kernel<TK_F16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, 1,
                         "kv_append", k, k_tok_stride, v, v_tok_stride, k_cache, v_cache, seq, num_kv_heads,
                         head_dim / 8, capacity, start_pos, total);
  return launch_kernel(kv_append_kernel<TK_BF16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, 1,
                       "kv_append", k, k_tok_stride, v, v_tok_stride, k_cache, v_cache, seq, num_kv_heads,
                       head_dim / 8, capacity, start_pos, total);
}
