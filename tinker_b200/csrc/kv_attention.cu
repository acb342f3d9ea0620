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
//     the `groups` query heads that share its kv head (up to 8, in every warp's registers),
//     so each cached key is converted once for all of them. The 4 warps take interleaved
//     32-key tiles, each with its own cp.async pipeline (2-3 stages) into shared memory;
//     q.k with one key per lane, p.V with the lane owning D/32 output columns, both in
//     packed fp32 FMAs; the warps' (max, sum, O) rows are merged in shared memory;
//   * the split-K combine across CTAs: each stores (max, sum, unnormalised O) of its rows,
//     the last CTA of a (sequence, kv head, row block) to arrive (atomic counter, reset by
//     that CTA) merges them. No CTA waits for another.
// The position may come from device memory (`start_dev`), so one CUDA graph serves every
// decode step; an out-of-range position records TK_DEVERR_POSITION and leaves `out` as is.
// The work is memory-bound (2 * kv_len * D * 2 bytes per kv head and sequence against
// 4 * groups * kv_len * D flops): SIMT, not tensor cores.
#include <algorithm>

#include "kv_attention.cuh"
#include "tk_host.h"

namespace tk {
namespace kvattn {

template <int DT, int D, int R>
__global__ void __launch_bounds__(THREADS) kv_attention_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  {
    // The cached rows below the position were written by earlier steps, not by the previous kernel:
    // pull the first CHUNK_KEYS of this CTA's share into L2 while that kernel finishes (a hint
    // only, so a position that is about to change does no harm; longer ranges are left to the
    // cp.async pipeline, which a larger prefetch only competes with).
    const int start = p.start_dev ? __ldcg(p.start_dev) : p.start_pos;  // L2: never a stale L1 line
    const int kv_len = start + p.seq;
    if (start > 0 && kv_len <= p.cap) {
      const int n_chunks = min(p.n_chunks, (kv_len + CHUNK_KEYS - 1) / CHUNK_KEYS);
      const int n_tiles = (kv_len + KT - 1) / KT;
      const int per = (n_tiles + n_chunks - 1) / n_chunks;
      const int lo = blockIdx.x * per * KT, hi = min(min(start, lo + per * KT), lo + CHUNK_KEYS);
      if (static_cast<int>(blockIdx.x) < n_chunks && lo < hi) {
        const int64_t row0 = (static_cast<int64_t>(blockIdx.z) * p.num_kv_heads + blockIdx.y / p.n_rb) * p.cap + lo;
        const int64_t bytes = static_cast<int64_t>(hi - lo) * D * 2;
        const char* kc = static_cast<const char*>(p.kc) + row0 * D * 2;
        const char* vc = static_cast<const char*>(p.vc) + row0 * D * 2;
        for (int64_t o = static_cast<int64_t>(threadIdx.x) * 128; o < bytes; o += THREADS * 128) {
          prefetch_l2(kc + o);
          prefetch_l2(vc + o);
        }
      }
    }
  }
  pdl_wait();  // q/k/v come from the previous kernel; the position may be written just before
  kv_attention_item<DT, D, R>(p, blockIdx.x, blockIdx.y / p.n_rb, blockIdx.y % p.n_rb, blockIdx.z,
                              blockIdx.z * gridDim.y + blockIdx.y,
                              blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0, smem);
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


// Rows per CTA (1, 4 or 8: every warp holds all of them), row blocks, and key chunks for a
// launch attending to at most `max_kv` keys: enough chunks for about 1.5 CTAs per SM, each at
// least CHUNK_KEYS keys long (the kernel uses fewer when the actual length is shorter).
// n_chunks never decreases with max_kv, so the workspace sized for a cache's capacity covers
// every position.
Plan make_plan(int batch, int num_kv_heads, int rows, int max_kv, int head_dim, int sm_count) {
  Plan pl{};
  pl.rows_cta = rows == 1 ? 1 : rows <= 4 ? 4 : 8;
  pl.n_rb = (rows + pl.rows_cta - 1) / pl.rows_cta;
  pl.units = static_cast<int64_t>(batch) * num_kv_heads * pl.n_rb;
  const int64_t max_chunks = std::max(1, (max_kv + CHUNK_KEYS - 1) / CHUNK_KEYS);
  const int64_t want = (3 * static_cast<int64_t>(std::max(sm_count, 1)) / 2 + pl.units - 1) / pl.units;
  pl.n_chunks = static_cast<int>(std::max<int64_t>(1, std::min(max_chunks, want)));
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

template <int DT, int D, int R>
int launch(const Params& p, dim3 grid, cudaStream_t st) {
  using S = Smem<D, R>;
  auto kern = kv_attention_kernel<DT, D, R>;
  static bool configured[64] = {};
  DeviceInfo dev;
  if (int rc = current_device_info(&dev)) return rc;
  if (!configured[dev.device]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL),
                            "cudaFuncSetAttribute(kv_attention)"))
      return rc;
    configured[dev.device] = true;
  }
  return launch_kernel(kern, grid, dim3(THREADS), S::TOTAL, st, 1, "kv_attention", p);
}

template <int DT, int D>
int launch_rows(int rows_cta, const Params& p, dim3 grid, cudaStream_t st) {
  switch (rows_cta) {
    case 1: return launch<DT, D, 1>(p, grid, st);
    case 4: return launch<DT, D, 4>(p, grid, st);
    default: return launch<DT, D, 8>(p, grid, st);
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
    return head_dim == 64 ? launch_rows<TK_F16, 64>(pl.rows_cta, p, grid, st) : launch_rows<TK_F16, 128>(pl.rows_cta, p, grid, st);
  return head_dim == 64 ? launch_rows<TK_BF16, 64>(pl.rows_cta, p, grid, st) : launch_rows<TK_BF16, 128>(pl.rows_cta, p, grid, st);
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
