// Fused RoPE + GQA/MQA/MHA causal attention on tcgen05 tensor cores.
//
// One CTA (4 warps, thread i owns query row i of the tile) computes a 128-row
// query tile of one (batch, query head):
//   * TMA loads the raw Q tile once and, per 128-key tile, the raw K and V tiles
//     of KV head h / groups straight from the [batch, seq, heads, head_dim]
//     projection layout (token strides are free, so q/k/v may be column slices of
//     one fused QKV output) into 128-byte-swizzled shared memory.
//   * RoPE is applied on load: each thread rotates the interleaved pairs of its
//     Q row (once) and its K row (every tile) in place in shared memory, in fp32,
//     rounding back to the input dtype as the reference does before its
//     attention kernel (tinker/kernels/fused_attention.py:203-214, :53-69).
//   * S = Q K^T runs as tcgen05.mma (M=128, N=128, K=head_dim) into TMEM; the
//     online softmax reads S with tcgen05.ld, writes P (rounded to the input
//     dtype) to shared memory and rescales the running O in TMEM; O += P V is a
//     second tcgen05.mma with V as an MN-major operand.
//   * Causal tiles above the diagonal are skipped; only the diagonal tile is masked.
// The arithmetic follows _attention_kernel (tinker/kernels/fused_attention.py:74-154):
// scale 1/sqrt(head_dim), running max / sum in fp32, output divided by the sum.
#include <cmath>

#include "tk_common.cuh"
#include "tk_host.h"

namespace tk {
namespace attn {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int THREADS = 128;

template <int D>
struct Smem {
  static constexpr int Q_BYTES = BQ * D * 2;
  static constexpr int K_BYTES = BKV * D * 2;
  static constexpr int V_BYTES = BKV * D * 2;
  static constexpr int P_BYTES = BQ * BKV * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + K_BYTES;
  static constexpr int P_OFF = V_OFF + V_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int TOTAL = 1024 + BAR_OFF + 4 * 8 + 16;
  static constexpr uint32_t TMEM_COLS = 256;  // S: 128 columns, O: head_dim columns
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
__device__ __forceinline__ void load_cs4(const void* t, int dt, int64_t off, float (&v)[4]) {
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

// Rotate row `r` of a swizzled [128 x D] tile in place by the RoPE angle of position `pos`.
template <int DT, int D>
__device__ __forceinline__ void rope_row_inplace(uint8_t* tile, int r, int64_t pos, const Params& p) {
  using Dx = Dt<DT>;
  const int64_t trow = pos * (D / 2);
#pragma unroll
  for (int blk = 0; blk < D / 64; ++blk) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      uint4* addr = reinterpret_cast<uint4*>(tile + blk * (128 * 128) + r * 128 + ((ch ^ (r & 7)) * 16));
      uint4 u = *addr;
      uint32_t w[4] = {u.x, u.y, u.z, u.w};
      const int i0 = blk * 32 + ch * 4;  // first pair index of this 16-byte chunk
      float c[4], s[4];
      load_cs4(p.cos_t, p.table_dtype, trow + i0, c);
      load_cs4(p.sin_t, p.table_dtype, trow + i0, s);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x = Dx::unpack(*reinterpret_cast<typename Dx::T2*>(&w[i]));
        typename Dx::T2 o = Dx::pack(x.x * c[i] - x.y * s[i], x.x * s[i] + x.y * c[i]);
        w[i] = *reinterpret_cast<uint32_t*>(&o);
      }
      *addr = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <int DT, int D>
__global__ void __launch_bounds__(THREADS, 1)
    rope_attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv, const Params p) {
  using S = Smem<D>;
  using Dx = Dt<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem + S::Q_OFF;
  uint8_t* sk = smem + S::K_OFF;
  uint8_t* sv = smem + S::V_OFF;
  uint8_t* sp = smem + S::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* s_done = bars + 1;
  uint64_t* pv_done = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x);  // heaviest tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.groups;
  const int q0 = qt * BQ;
  const int n_kv = qt + 1;  // causal: key tiles 0..qt

  if (tid == 0) {
    mbar_init(kv_full, 1);
    mbar_init(s_done, 1);
    mbar_init(pv_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t t_s = tmem_base;
  const uint32_t t_o = tmem_base + 128;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  {
    // the RoPE table rows this thread rotates with (Q row, first K row) do not depend
    // on the previous kernel: start pulling them into L1 while it finishes
    const int es = p.table_dtype == TK_F32 ? 4 : 2;
    const int row_bytes = (D / 2) * es;
    const int64_t qpos = static_cast<int64_t>(p.start_pos) + q0 + tid;
    const int64_t kpos = static_cast<int64_t>(p.start_pos) + tid;
    if (q0 + tid < p.seq && qpos < p.table_rows)
      for (int b = 0; b < row_bytes; b += 128) {
        prefetch_l1(static_cast<const char*>(p.cos_t) + qpos * row_bytes + b);
        prefetch_l1(static_cast<const char*>(p.sin_t) + qpos * row_bytes + b);
      }
    if (tid < p.seq && kpos < p.table_rows)
      for (int b = 0; b < row_bytes; b += 128) {
        prefetch_l1(static_cast<const char*>(p.cos_t) + kpos * row_bytes + b);
        prefetch_l1(static_cast<const char*>(p.sin_t) + kpos * row_bytes + b);
      }
  }

  if (tid == 0) {
    pdl_launch_dependents();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    pdl_wait();  // q, k, v are written by the previous kernel
    mbar_arrive_expect_tx(kv_full, S::Q_BYTES + S::K_BYTES + S::V_BYTES);
#pragma unroll
    for (int blk = 0; blk < D / 64; ++blk) {
      tma_load_3d(sq + blk * 128 * 128, &tq, kv_full, h * D + blk * 64, q0, b);
      tma_load_3d(sk + blk * 128 * 128, &tk, kv_full, kvh * D + blk * 64, 0, b);
      tma_load_3d(sv + blk * 128 * 128, &tv, kv_full, kvh * D + blk * 64, 0, b);
    }
  }

  constexpr uint32_t idesc_s = make_idesc_f16(Dx::umma_fmt, BQ, BKV, 0, 0);
  constexpr uint32_t idesc_o = make_idesc_f16(Dx::umma_fmt, BQ, D, 0, 1);
  const int q_row = q0 + tid;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int j = 0; j < n_kv; ++j) {
    if (!mbar_wait(kv_full, j & 1)) { ok = false; break; }
    // RoPE on load (rows past the sequence are zero-filled by TMA and left alone)
    if (j == 0 && q_row < p.seq) rope_row_inplace<DT, D>(sq, tid, static_cast<int64_t>(p.start_pos) + q_row, p);
    const int k_row = j * BKV + tid;
    if (k_row < p.seq) rope_row_inplace<DT, D>(sk, tid, static_cast<int64_t>(p.start_pos) + k_row, p);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        umma_f16_ss(t_s, make_sw128_desc(smem_u32(sq) + off, 0, 1024), make_sw128_desc(smem_u32(sk) + off, 0, 1024),
                    idesc_s, kk != 0);
      }
      umma_commit(s_done);
    }
    if (!mbar_wait(s_done, j & 1)) { ok = false; break; }
    tc_fence_after();

    // ---- online softmax on row tid ----
    float s[BKV];
#pragma unroll
    for (int c = 0; c < BKV; c += 32) tmem_ld32(t_s + lane_off + c, *reinterpret_cast<float(*)[32]>(&s[c]));
    tmem_wait_ld();
    const bool diag = (j == qt);
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < BKV; ++c) {
      float v = s[c] * p.scale_log2;
      if (diag && (j * BKV + c) > q_row) v = -INFINITY;
      s[c] = v;
      mx = fmaxf(mx, v);
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = exp2f(m_run - m_new);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < BKV; ++c) {
      s[c] = exp2f(s[c] - m_new);
      rs += s[c];
    }
    l_run = l_run * alpha + rs;
    m_run = m_new;

    if (j > 0) {
      // P and the O accumulator are still in use by the previous P.V
      if (!mbar_wait(pv_done, (j - 1) & 1)) { ok = false; break; }
      tc_fence_after();
    }
#pragma unroll
    for (int c = 0; c < BKV / 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        typename Dx::T2 hv = Dx::pack(s[c * 8 + 2 * i], s[c * 8 + 2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&hv);
      }
      uint8_t* dst = sp + (c >> 3) * (128 * 128) + tid * 128 + (((c & 7) ^ (tid & 7)) * 16);
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(t_o + lane_off + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tmem_st32(t_o + lane_off + c, o);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {
        const uint32_t aoff = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        const uint64_t ad = make_sw128_desc(smem_u32(sp) + aoff, 0, 1024);
        const uint64_t bd = make_sw128_desc(smem_u32(sv) + kk * 16 * 128, BKV * 128, 1024);
        umma_f16_ss(t_o, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(pv_done);
      if (j + 1 < n_kv) {
        // K and V of the next tile overwrite buffers the P.V just issued still reads
        if (mbar_wait(pv_done, j & 1)) {
          mbar_arrive_expect_tx(kv_full, S::K_BYTES + S::V_BYTES);
#pragma unroll
          for (int blk = 0; blk < D / 64; ++blk) {
            tma_load_3d(sk + blk * 128 * 128, &tk, kv_full, kvh * D + blk * 64, (j + 1) * BKV, b);
            tma_load_3d(sv + blk * 128 * 128, &tv, kv_full, kvh * D + blk * 64, (j + 1) * BKV, b);
          }
        }
      }
    }
  }

  if (ok && mbar_wait(pv_done, (n_kv - 1) & 1)) {
    tc_fence_after();
    const float inv_l = 1.0f / l_run;
    using T = typename Dx::T;
    T* dst = reinterpret_cast<T*>(p.out) +
             (static_cast<int64_t>(b) * p.seq + q_row) * p.out_tok_stride + static_cast<int64_t>(h) * D;
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      float o[32];
      tmem_ld32(t_o + lane_off + c, o);
      tmem_wait_ld();
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

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

template <int DT, int D>
int launch(const void* q, int64_t qs, const void* k, int64_t ks, const void* v, int64_t vs, Params p,
           cudaStream_t st) {
  using S = Smem<D>;
  CUtensorMap tq, tk_, tv;
  const uint64_t B = p.batch, Sq = p.seq;
  if (int rc = tensor_map_3d(&tq, q, DT, uint64_t(p.num_heads) * D, Sq, B, qs, qs * Sq, 64, BQ, 1)) return rc;
  if (int rc = tensor_map_3d(&tk_, k, DT, uint64_t(p.num_kv_heads) * D, Sq, B, ks, ks * Sq, 64, BKV, 1)) return rc;
  if (int rc = tensor_map_3d(&tv, v, DT, uint64_t(p.num_kv_heads) * D, Sq, B, vs, vs * Sq, 64, BKV, 1)) return rc;
  auto kern = rope_attention_kernel<DT, D>;
  static bool configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!configured[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL),
                            "cudaFuncSetAttribute(attention)"))
      return rc;
    configured[dev.device] = true;
  }
  return launch_kernel(kern, dim3(p.n_qtiles, p.num_heads, p.batch), dim3(THREADS), S::TOTAL, st, 1,
                       "rope_attention_kernel", tq, tk_, tv, p);
}

}  // namespace attn
}  // namespace tk

extern "C" int tk_rope_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                                 const void* v, int64_t v_tok_stride, const void* cos_table, const void* sin_table,
                                 int table_dtype, int64_t table_rows, void* out, int64_t out_tok_stride, int batch,
                                 int seq, int num_heads, int num_kv_heads, int head_dim, int start_pos, int dtype,
                                 void* stream) {
  using namespace tk;
  if (!half_dtype(dtype)) return fail_invalid("rope_attention: dtype must be F16 or BF16");
  if (!valid_dtype(table_dtype)) return fail_invalid("rope_attention: table dtype must be F16, BF16 or F32");
  if (head_dim != 64 && head_dim != 128) return set_error(TK_ERR_UNSUPPORTED, "rope_attention: head_dim must be 64 or 128");
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0 || start_pos < 0)
    return fail_invalid("rope_attention: invalid sizes");
  if (num_heads % num_kv_heads != 0) return fail_invalid("rope_attention: num_heads must be a multiple of num_kv_heads");
  if (q_tok_stride < int64_t(num_heads) * head_dim || k_tok_stride < int64_t(num_kv_heads) * head_dim ||
      v_tok_stride < int64_t(num_kv_heads) * head_dim || out_tok_stride < int64_t(num_heads) * head_dim)
    return fail_invalid("rope_attention: token stride smaller than heads * head_dim");
  if (q_tok_stride % 8 || k_tok_stride % 8 || v_tok_stride % 8 || out_tok_stride % 8)
    return fail_invalid("rope_attention: token strides must be multiples of 8 elements");
  if (int64_t(start_pos) + seq > table_rows)
    return fail_invalid("rope_attention: start_pos + seq exceeds the RoPE table length");
  if (num_heads > 65535 || batch > 65535) return fail_invalid("rope_attention: too many heads or batches");
  if (batch == 0 || seq == 0) return TK_OK;  // empty tensors may carry NULL data pointers
  if (!q || !k || !v || !cos_table || !sin_table || !out) return fail_invalid("rope_attention: NULL pointer");
  if (!aligned16(out) || !aligned16(cos_table) || !aligned16(sin_table))
    return fail_invalid("rope_attention: out and the RoPE tables must be 16-byte aligned");
  attn::Params p{};
  p.batch = batch;
  p.seq = seq;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.groups = num_heads / num_kv_heads;
  p.start_pos = start_pos;
  p.n_qtiles = (seq + attn::BQ - 1) / attn::BQ;
  p.table_rows = table_rows;
  p.cos_t = cos_table;
  p.sin_t = sin_table;
  p.table_dtype = table_dtype;
  p.out = out;
  p.out_tok_stride = out_tok_stride;
  p.scale_log2 = static_cast<float>((1.0 / std::sqrt(double(head_dim))) * 1.4426950408889634);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TK_F16) {
    if (head_dim == 64) return attn::launch<TK_F16, 64>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, st);
    return attn::launch<TK_F16, 128>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, st);
  }
  if (head_dim == 64) return attn::launch<TK_BF16, 64>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, st);
  return attn::launch<TK_BF16, 128>(q, q_tok_stride, k, k_tok_stride, v, v_tok_stride, p, st);
}
