/*
 * tinker_b200.h - C ABI of the B200 (sm_100a) fused-kernel library.
 *
 * This library replaces everything under the reference's tinker/kernels/
 * (eb1386/TinKer) with hand-written CUDA for sm_100a. Each entry point takes
 * plain device pointers, element strides and sizes, a dtype code and a CUDA
 * stream handle (cudaStream_t passed as void*; NULL = legacy default stream),
 * enqueues its kernels on that stream and returns without synchronising.
 * Outputs are written to caller-owned buffers; inputs are never modified.
 *
 * Return value: TK_OK, or an error code with a message available from
 * tk_last_error() (per calling thread). Argument checks run on the host before
 * any launch, so a rejected call leaves the device untouched.
 */
#ifndef TINKER_B200_H_
#define TINKER_B200_H_

#include <stdint.h>

/* Every entry point is exported; everything else in the library is hidden, so
 * that its CUDA registration symbols cannot interpose with another library's. */
#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element type codes */
#define TK_F16 0
#define TK_BF16 1
#define TK_F32 2

/* status codes */
#define TK_OK 0
#define TK_ERR_INVALID 1     /* bad shape, stride, dtype or alignment */
#define TK_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define TK_ERR_UNSUPPORTED 3 /* not an sm_100 device, or a size the kernels do not cover */

/* Library version (major*10000 + minor*100 + patch). */
TK_API int tk_version(void);

/* Message for the last non-TK_OK return on this thread ("" if none). */
TK_API const char* tk_last_error(void);

/* TK_OK if `device` is an sm_100 (B200-class) GPU the kernels were built for. */
TK_API int tk_check_device(int device);

/* Read (and optionally clear) the sticky device-side error word of the current
 * device. Non-zero means a kernel gave up and its outputs are invalid: 1 = a
 * bounded wait timed out, 2 = a position read from device memory lay beyond a KV
 * cache or RoPE table, 3 = a token id read from device memory lay outside the
 * embedding table. Synchronises the device; meant for tests and debugging. */
TK_API int tk_device_error(int* code, int clear);

/*
 * RMSNorm over the last axis: y = x * rsqrt(mean(x^2) + eps) * weight, float32
 * statistics, one rounding to `dtype`.
 * Replaces fused_rmsnorm / _rmsnorm_triton / _rmsnorm_kernel
 * (tinker/kernels/fused_rmsnorm.py:70-74, :55-61, :12-52).
 * x, y: [rows, dim] with row strides in elements; weight: [dim] of `w_dtype`.
 * dtype, w_dtype in {TK_F16, TK_BF16, TK_F32}.
 */
TK_API int tk_rmsnorm(const void* x, int64_t x_row_stride, const void* weight, int w_dtype, void* y,
               int64_t y_row_stride, int64_t rows, int64_t dim, float eps, int dtype, void* stream);

/*
 * Row sums of squares for an RMSNorm folded into the next GEMM (tk_epilogue.row_ssq_in):
 * parts[(c / 32) * m + r] = sum of x[r, c .. c+31]^2 in float32, for every 32-column
 * chunk c of k columns (k a multiple of 32). The statistics pass of
 * _rmsnorm_kernel (tinker/kernels/fused_rmsnorm.py:12-52) without its normalisation,
 * for rows no GEMM epilogue produced (the embedding output).
 */
TK_API int tk_row_sumsq(const void* x, int64_t x_row_stride, int64_t m, int64_t k, float* parts, int dtype,
                 void* stream);

/*
 * The embedding gather of a decoder's first step with the row statistics of its output:
 * out[r, :] = table[tokens[r], :] ([rows, hidden] contiguous, table [vocab, hidden] contiguous,
 * tokens int64 on the device) and, if row_ssq_out is not NULL, row_ssq_out[(c / 32) * rows + r] =
 * the sum of squares of out[r, c .. c+31] - the row_ssq_in of the first folded RMSNorm, so that
 * tk_row_sumsq need not run. Replaces `x = self.embedding(tokens)` of the reference's decoder
 * (benchmarks/bench_e2e.py:95,104; nn.Embedding without padding_idx / max_norm) plus the
 * statistics pass of its first RMSNorm. A token outside [0, vocab) records device error 3
 * (tk_device_error) and gives a zero row. hidden a multiple of 32; dtype in {F16, BF16}.
 */
TK_API int tk_embedding_rows(const int64_t* tokens, const void* table, int64_t vocab, int64_t hidden, void* out,
                             float* row_ssq_out, int64_t rows, int dtype, void* stream);

/*
 * Residual add fused with RMSNorm: s = x + residual (rounded to dtype), written
 * to residual_out; y = rmsnorm(s). The residual update of the reference decoder
 * block (benchmarks/bench_e2e.py:112-115) followed by its next norm
 * (tinker/kernels/fused_rmsnorm.py:70). All tensors contiguous [rows, dim].
 * residual_out may alias x or residual.
 */
TK_API int tk_add_rmsnorm(const void* x, const void* residual, const void* weight, int w_dtype, void* y,
                   void* residual_out, int64_t rows, int64_t dim, float eps, int dtype, void* stream);

/*
 * SwiGLU activation out = silu(gate) * up, float32 math, one rounding.
 * Replaces fused_swiglu / _swiglu_triton / _swiglu_kernel
 * (tinker/kernels/fused_swiglu.py:61-66, :47-54, :13-44).
 * gate, up, out: [rows, n] with row strides in elements; dtype in {F16, BF16, F32}.
 */
TK_API int tk_swiglu(const void* gate, int64_t gate_row_stride, const void* up, int64_t up_row_stride, void* out,
              int64_t out_row_stride, int64_t rows, int64_t n, int dtype, void* stream);

/*
 * Fused RoPE + GQA/MQA/MHA causal attention on tcgen05 tensor cores.
 * Replaces fused_attention / _attention_triton / _rope_kernel / _attention_kernel
 * (tinker/kernels/fused_attention.py:234-238, :195-231, :19-69, :74-154).
 * q: [batch, seq, num_heads, head_dim], k, v: [batch, seq, num_kv_heads, head_dim],
 * out: [batch, seq, num_heads, head_dim]; the *_tok_stride arguments are the
 * element strides between consecutive tokens (so q, k and v may be column
 * slices of one fused QKV projection). Interleaved-pair RoPE at positions
 * start_pos + s uses cos_table/sin_table [table_rows, head_dim/2] of
 * `table_dtype`; softmax scale 1/sqrt(head_dim); query head h reads KV head
 * h / (num_heads / num_kv_heads). dtype in {F16, BF16}; head_dim in {64, 128}.
 */
TK_API int tk_rope_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride, const void* v,
                      int64_t v_tok_stride, const void* cos_table, const void* sin_table, int table_dtype,
                      int64_t table_rows, void* out, int64_t out_tok_stride, int batch, int seq, int num_heads,
                      int num_kv_heads, int head_dim, int start_pos, int dtype, void* stream);

/*
 * RoPE of q and k in one pass: out[b, s, :] = [rope(q heads) | rope(k heads)], each interleaved
 * pair rotated in fp32 at position start_pos + s and rounded to dtype, exactly as
 * tk_rope_attention rotates on load (the reference's _rope_kernel,
 * tinker/kernels/fused_attention.py:19-69, on its permuted copies :199-214). Feeds
 * tk_causal_attention for long sequences, where rotating on load would re-read the cos/sin
 * rows of every key tile in every CTA. out: token stride >= (num_heads + num_kv_heads) *
 * head_dim; head_dim a multiple of 8; all strides multiples of 8 elements.
 */
TK_API int tk_rope_qk(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride, const void* cos_table,
               const void* sin_table, int table_dtype, int64_t table_rows, void* out, int64_t out_tok_stride,
               int batch, int seq, int num_heads, int num_kv_heads, int head_dim, int start_pos, int dtype,
               void* stream);

/*
 * The same causal GQA attention on q and k that already carry RoPE (the q|k|v
 * projection applied it in its epilogue, tk_linear_rope): the kernel of
 * tk_rope_attention without the rotation. Together with tk_linear_rope it
 * replaces the q/k/v projections plus fused_attention in TinKerAttention.forward
 * (tinker/modules/attention.py:55-70, tinker/kernels/fused_attention.py:195-231).
 */
TK_API int tk_causal_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride,
                        const void* v, int64_t v_tok_stride, void* out, int64_t out_tok_stride, int batch,
                        int seq, int num_heads, int num_kv_heads, int head_dim, int dtype, void* stream);

/*
 * Attention of S new tokens per sequence against a KV cache (decode steps, short
 * chunks), one launch: RoPE of the new q and k rows at positions start..start+S-1
 * (float32 tables [table_rows, head_dim/2], results rounded to dtype), the append of
 * the rotated k rows and the v rows to the cache, and causal GQA attention of the new
 * rows over cache positions 0..start+S-1. Equals rows start..start+S-1 of the
 * reference's causal RoPE attention over the whole sequence
 * (tinker/kernels/fused_attention.py:176-192, :195-231), which has no cache and
 * recomputes the sequence (tinker/modules/attention.py:51, README.md:102).
 * q [batch*seq, >= num_heads*head_dim], k/v [batch*seq, >= num_kv_heads*head_dim]
 * (projections without RoPE, token strides in elements); k_cache/v_cache
 * [batch, num_kv_heads, capacity, head_dim] contiguous; out like q.
 * start_pos_device: if not NULL the position is read from this device int at run
 * time (a CUDA graph replays for every step); a position with start+S beyond the
 * cache or the table then records device error 2 and leaves out unchanged.
 * workspace: zero-filled device memory of tk_kv_attention_workspace() bytes (may be
 * 0: then NULL is fine); the kernel returns it to zeros, so it is reused without a
 * memset, but launches that overlap on the GPU must not share it.
 */
TK_API int tk_kv_attention(const void* q, int64_t q_tok_stride, const void* k, int64_t k_tok_stride, const void* v,
                           int64_t v_tok_stride, void* k_cache, void* v_cache, int capacity, const float* cos_table,
                           const float* sin_table, int64_t table_rows, void* out, int64_t out_tok_stride, int batch,
                           int seq, int num_heads, int num_kv_heads, int head_dim, int start_pos,
                           const int* start_pos_device, void* workspace, int64_t workspace_bytes, int dtype,
                           void* stream);

/* Workspace bytes tk_kv_attention needs for these sizes when start+S <= max_kv
 * (pass the cache capacity when the position comes from device memory). 0 when
 * none is needed or the sizes are invalid, -1 without a device. */
TK_API int64_t tk_kv_attention_workspace(int batch, int num_heads, int num_kv_heads, int head_dim, int seq,
                                         int max_kv);

/*
 * Copy S rows of k (already rotated) and v per sequence into a KV cache at
 * start_pos: the cache fill after a prompt's tk_linear_rope + tk_causal_attention.
 * Layouts as tk_kv_attention.
 */
TK_API int tk_kv_append(const void* k, int64_t k_tok_stride, const void* v, int64_t v_tok_stride, void* k_cache,
                        void* v_cache, int capacity, int batch, int seq, int num_kv_heads, int head_dim,
                        int start_pos, int dtype, void* stream);

/*
 * One decode step of a whole decoder stack in ONE persistent cooperative kernel (batch <= 8
 * sequences, one new token each): for every layer the q|k|v product (attention RMSNorm folded
 * into wq/wk/wv), tk_kv_attention's work, o_proj + residual, gate|up + SwiGLU (FFN RMSNorm folded
 * into wg/wu), down + residual, separated by grid barriers instead of kernel boundaries; then the
 * final RMSNorm. The per-block path of the same step is 5 launches per layer (tk_linear /
 * tk_kv_attention / tk_linear_ex / tk_gate_up_swiglu_ex / tk_linear_ex); the reference has no
 * cached decoding at all (tinker/modules/attention.py:51, README.md:102).
 *
 * tk_decode_step_setup (synchronous, not capturable; zero-fills `scratch` of
 * tk_decode_step_scratch_bytes() bytes and copies the layer table into it): weights [out, in]
 * row-major in `dtype`, caches [batch, num_kv_heads, capacity, head_dim], float32 RoPE tables,
 * `position`: device int32 read when the kernel runs (the first new token's position).
 * tk_decode_step (capturable): x [batch, hidden] holds the embedding rows and is overwritten
 * with the last block's output; y [batch, hidden] receives the final RMSNorm of it. Appends the
 * step's keys and values to the caches. Waits are bounded; a device error stops the step.
 */
typedef struct tk_step_layer {
  const void* wq;
  const void* wk;
  const void* wv;
  const void* wo;
  const void* wg;
  const void* wu;
  const void* wd;
  void* k_cache;
  void* v_cache;
  float eps_attn;
  float eps_ffn;
} tk_step_layer;

TK_API int64_t tk_decode_step_scratch_bytes(int num_layers, int batch, int hidden, int num_heads, int num_kv_heads,
                                            int head_dim, int intermediate, int capacity);
TK_API int tk_decode_step_setup(const tk_step_layer* layers, int num_layers, int batch, int hidden, int num_heads,
                                int num_kv_heads, int head_dim, int intermediate, const float* cos_table,
                                const float* sin_table, int64_t table_rows, int capacity, const int* position,
                                const void* final_norm_weight, float final_eps, int dtype, void* scratch,
                                int64_t scratch_bytes);
TK_API int tk_decode_step(void* x, void* y, void* scratch, void* stream);
/*
 * Test hook for the failure path (no counterpart in the reference): with cta >= 0, CTA `cta` of
 * the next tk_decode_step launches on `scratch` does not arrive at the step's first grid
 * barrier, so every CTA's bounded wait there runs out after TK_WAIT_LIMIT_NS (2 s): the step
 * records device error 1 (tk_device_error), every CTA returns and the outputs are invalid;
 * cta = -1 (the default after tk_decode_step_setup) turns it off. Nothing is faulted.
 */
TK_API int tk_decode_step_withhold_arrival(void* scratch, int cta);
/* Forget the plan tk_decode_step_setup stored for `scratch` (before freeing it). */
TK_API int tk_decode_step_release(void* scratch);

/*
 * Epilogue options of tk_linear_ex / tk_gate_up_swiglu_ex (zero-initialise, then set):
 *  residual       [m, n] with y's row stride, added before the one rounding (plain store).
 *  row_ssq_in     [row_ssq_parts, m] float32 partial sums of squares of x's rows: the
 *                 accumulator of row r is scaled by 1/sqrt(sum / k + row_ssq_eps), i.e. the
 *                 GEMM consumes rmsnorm(x) whose weight has been multiplied into w's
 *                 columns (TinKerRMSNorm + the projection that follows it,
 *                 tinker/modules/normalization.py:29-31 then attention.py:55 /
 *                 feed_forward.py:27-28).
 *  row_ssq_out    plain store only: [ceil(n / 32), m] float32, the sum of squares of the
 *                 32 stored (rounded) values of row r from column 32 j on, at [j * m + r];
 *                 the row_ssq_in of the next folded RMSNorm.
 *  rope_*         plain store only, rope_head_dim > 0: the columns [0, n0 + n1) (the q
 *                 and k heads) are rounded to dtype and rotated as in tk_linear_rope.
 *  weights_prefetch  nonzero only if no kernel enqueued since the stream last waited for all
 *                 earlier work writes the weights (e.g. inside a CUDA graph that never writes
 *                 them): the first weight tiles are then loaded into shared memory before the
 *                 previous kernel has finished (programmatic dependent launch). With 0 they are
 *                 only prefetched into L2 until it has.
 *  l2_prefetch, l2_prefetch_bytes  up to TK_L2_PREFETCH_MAX device byte ranges (NULL / 0 =
 *                 unused) that the launch pulls into L2 for the kernels enqueued after it, e.g.
 *                 the weights of a decoder block's later projections: every CTA issues a share
 *                 at its start, so their streams start from L2 instead of HBM while the launch
 *                 chain keeps HBM mostly idle. A hint only: nothing is written, each range is
 *                 rounded inward to 16-byte boundaries, and the ranges must stay allocated until
 *                 the launch has finished.
 */
#define TK_L2_PREFETCH_MAX 8
typedef struct tk_epilogue {
  const void* residual;
  const float* row_ssq_in;
  int row_ssq_parts;
  float row_ssq_eps;
  float* row_ssq_out;
  int rope_seq;
  int rope_start;
  int rope_head_dim;
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_table_rows;
  int weights_prefetch;
  const void* l2_prefetch[TK_L2_PREFETCH_MAX];
  int64_t l2_prefetch_bytes[TK_L2_PREFETCH_MAX];
} tk_epilogue;

/*
 * tk_linear with the epilogue options above (NULL = plain store).
 */
TK_API int tk_linear_ex(const void* x, int64_t x_row_stride, const void* w0, int64_t n0, const void* w1, int64_t n1,
                 const void* w2, int64_t n2, void* y, int64_t y_row_stride, int64_t m, int64_t k,
                 const tk_epilogue* epi, int dtype, void* stream);

/*
 * y[m, n] = x[m, k] . w[n, k]^T on tcgen05 (nn.Linear without bias), fp32
 * accumulation in TMEM. Replaces the nn.Linear projections the reference's
 * modules run through cuBLAS (tinker/modules/attention.py:53-55,64;
 * tinker/modules/feed_forward.py:27-30). The weight may be given as up to three
 * row blocks w0 [n0, k], w1 [n1, k], w2 [n2, k] that are concatenated along n
 * (n = n0 + n1 + n2; pass NULL / 0 for unused blocks), which is how the q, k and
 * v projections run as one GEMM. Row strides in elements; dtype in {F16, BF16};
 * k and the strides must be multiples of 8; n0, n1 multiples of 32.
 * If residual is non-NULL, y = x . w^T + residual ([m, n], row stride y_row_stride).
 */
TK_API int tk_linear(const void* x, int64_t x_row_stride, const void* w0, int64_t n0, const void* w1, int64_t n1,
              const void* w2, int64_t n2, void* y, int64_t y_row_stride, const void* residual, int64_t m,
              int64_t k, int dtype, void* stream);

/*
 * The fused q|k|v projection with RoPE in its epilogue: y = x . cat(wq, wk, wv)^T
 * where the q and k columns of every row are rounded to dtype and then rotated
 * (interleaved pairs, fp32 math) at position start_pos + (row mod seq), i.e. the
 * rows are [batch, seq] tokens. cos_table / sin_table: float32 [table_rows,
 * head_dim/2]. Replaces q_proj/k_proj/v_proj plus the RoPE kernel launches of
 * TinKerAttention.forward (tinker/modules/attention.py:55-70,
 * tinker/kernels/fused_attention.py:203-214, :19-69); the result feeds
 * tk_causal_attention.
 */
TK_API int tk_linear_rope(const void* x, int64_t x_row_stride, const void* wq, int64_t nq, const void* wk, int64_t nk,
                   const void* wv, int64_t nv, void* y, int64_t y_row_stride, int64_t m, int64_t k, int seq,
                   int start_pos, int head_dim, const void* cos_table, const void* sin_table, int64_t table_rows,
                   int dtype, void* stream);

/*
 * h[m, f] = silu(x . w_gate^T) * (x . w_up^T): the gate and up projections as
 * one tcgen05 GEMM whose epilogue applies SwiGLU to the fp32 accumulators.
 * Replaces gate_proj/up_proj + fused_swiglu in TinKerSwiGLU.forward
 * (tinker/modules/feed_forward.py:26-30, tinker/kernels/fused_swiglu.py:61-66).
 * x: [m, hidden] (row stride x_row_stride), w_gate, w_up: [f, hidden]
 * contiguous, h: [m, f] contiguous. f multiple of 32, hidden multiple of 8.
 */
TK_API int tk_gate_up_swiglu(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up, void* h,
                      int64_t m, int64_t hidden, int64_t f, int dtype, void* stream);

/*
 * tk_gate_up_swiglu with epilogue options (only row_ssq_in / row_ssq_eps apply: the
 * RMSNorm before the FFN folded into w_gate and w_up).
 */
TK_API int tk_gate_up_swiglu_ex(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up, void* h,
                         int64_t m, int64_t hidden, int64_t f, const tk_epilogue* epi, int dtype, void* stream);

/*
 * Whole SwiGLU FFN: out = (silu(x Wg^T) * (x Wu^T)) Wd^T (+ residual).
 * Replaces TinKerSwiGLU.forward (tinker/modules/feed_forward.py:26-30).
 * h_scratch is caller-provided scratch of m * f elements of dtype holding the
 * activation between the two GEMMs. out: [m, hidden] contiguous; residual NULL
 * or [m, hidden] contiguous (may alias out).
 */
TK_API int tk_swiglu_ffn(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up, const void* w_down,
                  void* h_scratch, void* out, const void* residual, int64_t m, int64_t hidden, int64_t f,
                  int dtype, void* stream);

/*
 * tk_swiglu_ffn without the scratch argument: the same FFN, with the [m, f]
 * activation kept in a fixed 8 MiB array inside the library's own device
 * memory, so the call allocates no device memory. No counterpart in the
 * reference: it is for callers that cannot allocate - hosts that own all device
 * memory and pass only inputs and outputs, or loops that must not call
 * cudaMalloc/cudaFree. Requires m * f * 2 <= 8 MiB (else TK_ERR_INVALID). The
 * first call in each CUDA context looks up the array's address; make it before
 * any stream capture starts. All calls on a device share the array, so calls that
 * overlap on the GPU race and must be ordered by the caller.
 */
TK_API int tk_swiglu_ffn_noalloc(const void* x, int64_t x_row_stride, const void* w_gate, const void* w_up,
                          const void* w_down, void* out, const void* residual, int64_t m, int64_t hidden,
                          int64_t f, int dtype, void* stream);

/*
 * The whole decoder stack of a short prefill (batch * seq <= 128 rows) in ONE persistent
 * kernel: token embedding, then per layer the q|k|v projection (attention RMSNorm folded
 * into wq/wk/wv, RoPE in the epilogue), causal GQA attention, o_proj + residual, gate|up +
 * SwiGLU (FFN RMSNorm folded into wg/wu), down + residual; then the final RMSNorm. The
 * arithmetic of the per-block path (tk_linear_rope, tk_causal_attention, tk_linear_ex,
 * tk_gate_up_swiglu_ex) with kernel boundaries replaced by arrival counters; it replaces the
 * reference's patched forward of the model's blocks and final norm (benchmarks/bench_e2e.py
 * :112-138 with tinker/modules/*.py, tinker/kernels/*.py), whose CUDA graph replays one kernel
 * launch per operation (tinker/optimize.py:153-173). head_dim 64; hidden and intermediate
 * multiples of 64; weights [out, in] row-major in `dtype`, 16-byte aligned.
 *
 * tk_stack_setup (synchronous, not capturable): plans the tiles, encodes the tensor maps of
 * every weight into `scratch` (tk_stack_scratch_bytes() bytes, 256-byte aligned) and zeroes
 * its counters. Weights, tables and the embedding must stay at their addresses while the plan
 * is used. tk_stack_forward (capturable, no host synchronisation): tokens [batch * seq] int64
 * on the device; y [batch * seq, hidden] receives the final RMSNorm of the last block's output
 * (the LM head's input). Token ids outside [0, vocab) record device error 3 and read row 0.
 * Every wait is bounded: a launch whose wait runs out records device error 1, skips the rest
 * of its work (outputs invalid) and still leaves the scratch ready for the next launch. Calls
 * sharing one scratch must not overlap on the GPU.
 */
typedef struct tk_stack_layer {
  const void* wq;
  const void* wk;
  const void* wv;
  const void* wo;
  const void* wg;
  const void* wu;
  const void* wd;
  float eps_attn;
  float eps_ffn;
} tk_stack_layer;

TK_API int64_t tk_stack_scratch_bytes(int num_layers, int batch, int seq, int hidden, int num_heads, int num_kv_heads,
                                      int head_dim, int intermediate);
TK_API int tk_stack_setup(const tk_stack_layer* layers, int num_layers, int batch, int seq, int hidden, int num_heads,
                          int num_kv_heads, int head_dim, int intermediate, const void* embedding, int64_t vocab,
                          const float* cos_table, const float* sin_table, int64_t table_rows, int start_pos,
                          const void* final_norm_weight, float final_eps, int dtype, void* scratch,
                          int64_t scratch_bytes);
TK_API int tk_stack_forward(const int64_t* tokens, void* y, void* scratch, void* stream);
/* The tile plan of a prepared scratch: out[4 * g .. 4 * g + 3] = (accumulator columns, tiles,
 * k-splits, k-blocks) of projection g (0 q|k|v, 1 o_proj, 2 gate|up, 3 down); out[16] = CTAs. */
TK_API int tk_stack_plan(void* scratch, int* out, int n);
/* Diagnostics (no reference counterpart): with `trace` non-NULL, later tk_stack_forward launches
 * on `scratch` write %globaltimer stamps (ns) of 8 events per CTA and schedule stage to
 * trace[(cta * (2 + 5 * num_layers) + stage) * 8 + event] (events: producer saw the stage's
 * dependency, producer issued its first weight tiles, MMA committed, epilogue saw its first
 * accumulator, its first tile's k-splits, the stage's dependency, arrived; attention S ready).
 * NULL turns it off (the default). */
TK_API int tk_stack_trace(void* scratch, unsigned long long* trace);
/* Forget the plan tk_stack_setup stored for `scratch` (before freeing it). */
TK_API int tk_stack_release(void* scratch);

#ifdef __cplusplus
}
#endif

#endif /* TINKER_B200_H_ */
