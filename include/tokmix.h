/* tokmix.h -- C ABI of libtokmix.so, the sm_100a (B200) prefill token-mixer kernels.
 *
 * Two entry points replace the two kernel extensions the reference's plugin modules bind (the
 * GDN one has two further variants below, and a single-token decode step follows them):
 *
 *   tokmix_fa2_fwd      replaces  flash_attention_2_forward(q, k, v, sm_scale, causal)
 *                       kernels_optimized/flash_attention_2.cu:1121-1258, bound at
 *                       kernels_optimized/flash_attention_2.py:139-140 (kernel_fn)
 *   tokmix_gdn_prefill  replaces  qwen35moe_gdn_prefill_bf16tc(q, k, v, g, beta, state, scale)
 *                       kernels_optimized/qwen35moe_gdn_prefill.cu:1203-1264, bound at
 *                       kernels_optimized/qwen35moe_gdn_prefill.py:149-161 (kernel_fn)
 *
 * Conventions (all entry points):
 *   - every pointer argument is DEVICE memory of the current device; the library allocates and
 *     frees no device memory (TMEM is allocated and released inside each kernel);
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream) and the call
 *     returns without synchronising;
 *   - the return value is TOKMIX_OK or one of the TOKMIX_ERR_* codes; the text of the last
 *     error of the calling thread is returned by tokmix_last_error();
 *   - `status` (optional, device memory, one uint32 initialised to 0 by the caller) receives
 *     the kernels' device-side status bits: every pipeline wait inside a kernel is bounded, and
 *     a wait that runs out sets a TOKMIX_DEV_* bit here and ends the kernel early instead of
 *     hanging the GPU.  The caller reads it after synchronising.
 */
#ifndef TOKMIX_H_
#define TOKMIX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define TOKMIX_OK 0
#define TOKMIX_ERR_INVALID_ARGUMENT 1 /* shape / pointer / alignment argument rejected */
#define TOKMIX_ERR_UNSUPPORTED 2      /* valid request this build has no kernel for */
#define TOKMIX_ERR_LAUNCH 3           /* the CUDA launch itself failed */
#define TOKMIX_ERR_DEVICE 4           /* wrong device (needs compute capability 10.0) */

/* device status bits written into *status by the kernels */
#define TOKMIX_DEV_TIMEOUT_TMA 0x1u
#define TOKMIX_DEV_TIMEOUT_MMA 0x2u
#define TOKMIX_DEV_TIMEOUT_PIPE 0x4u
#define TOKMIX_DEV_BAD_ARGS 0x8u

/* tensor layouts for attention */
#define TOKMIX_LAYOUT_BHSD 0 /* [batch, heads, seq, head_dim]  (the reference's contract) */
#define TOKMIX_LAYOUT_BSHD 1 /* [batch, seq, heads, head_dim] */

/* element types */
#define TOKMIX_DTYPE_BF16 0
#define TOKMIX_DTYPE_FP32 1
#define TOKMIX_DTYPE_FP16 2

/* Causal / non-causal attention forward, bf16 in and out, fp32 softmax and accumulation.
 *
 *   o = softmax(q k^T * sm_scale + mask) v
 *
 * q, o: [batch, heads_q, seqlen_q, head_dim] (BHSD) or [batch, seqlen_q, heads_q, head_dim] (BSHD)
 * k, v: same layout with heads_kv and seqlen_kv.  Contiguous; base pointers 16-byte aligned.
 * heads_q must be a multiple of heads_kv; query head h reads key/value head h / (heads_q/heads_kv).
 * head_dim in {64, 128, 256}.  causal != 0 masks key j for query i when j > i (top-left aligned, as
 * torch's scaled_dot_product_attention(is_causal=True)).
 * Replaces flash_attention_2_forward (kernels_optimized/flash_attention_2.cu:1121-1258), which
 * supported only BHSD, heads_q == heads_kv and head_dim == 128. */
int tokmix_fa2_fwd(const void* q, const void* k, const void* v, void* o, int batch, int heads_q, int heads_kv,
                   int seqlen_q, int seqlen_kv, int head_dim, int layout, int causal, float sm_scale,
                   uint32_t* status, void* stream);

/* Steps before the recurrence that the GDN prefill entry points can do inside their first stage
 * (the `gates` argument; NULL = neither).  The reference takes normalised q, k and ready g, beta
 * (kernels/qwen35moe_gdn_prefill.py:107-136).
 *   Gates (a != NULL): the Qwen3.5 gated-delta-net gates from the raw projections, computed while
 *   each chunk is prepared (the g, beta arguments are then ignored):
 *     g = -exp(a_log[h]) * softplus(a + dt_bias[h]),  beta = sigmoid(b)      (fp32 arithmetic)
 *   a, b: device [total_tokens, heads_v] in `dtype` (TOKMIX_DTYPE_BF16 or TOKMIX_DTYPE_FP32);
 *   a_log, dt_bias: device fp32 [heads_v].  The arithmetic is tokmix_gdn_gates' own, so the
 *   results equal those of running tokmix_gdn_gates first, bit for bit.
 *   q/k normalisation (qk_l2norm != 0): every q and k row becomes x / sqrt(sum x^2 + l2norm_eps)
 *   (fp32 arithmetic, bf16 result) as it is staged for the first product, with the summation of
 *   tokmix_l2norm_rows, so the results equal those of running tokmix_l2norm_rows on bf16 q and k
 *   first, bit for bit.  The schedules that prepare chunks apart from their state chains
 *   (tokmix_gdn_prefill_split, tokmix_gdn_prefill_segmented) write the normalised keys to
 *   k_normed (device bf16 [total_tokens, heads_k, 128]) for the chains to read; the one-CTA-per-unit
 *   kernel (tokmix_gdn_prefill) needs no such buffer (k_normed may be NULL there). */
typedef struct tokmix_gdn_stage1 {
  const void* a;
  const void* b;
  int dtype;
  const float* a_log;
  const float* dt_bias;
  int qk_l2norm;
  float l2norm_eps;
  void* k_normed;
} tokmix_gdn_stage1;

/* Gated-delta-rule (GDN) prefill, chunked on the tensor cores.
 *
 * Token layout: q, k [total_tokens, heads_k, 128]; v, out [total_tokens, heads_v, 128];
 * g, beta [total_tokens, heads_v] fp32 (g is the log decay, beta the write strength).
 * A batch [B, T, ...] is the same memory with total_tokens = B*T and B sequences of T tokens.
 * Sequence n covers tokens [cu_seqlens[n], cu_seqlens[n+1]).
 * State layout: initial_state / final_state [num_seqs, heads_v, 128 (v), 128 (k)] fp32
 * (initial_state may be NULL for a zero initial state; final_state may alias initial_state).
 * Value head h reads key head h % heads_k (as kernels/qwen35moe_gdn_prefill.cu:48).
 * io_dtype is the type of q, k, v and out: TOKMIX_DTYPE_BF16 (the only one this build runs).
 * gates: NULL (g and beta as given), or the raw projections to compute them from (above).
 *
 * cu_seqlens_dev:   device int32 [num_seqs + 1]
 * seq_order_dev:    device int32 [num_seqs], the order in which sequences are scheduled
 *                   (longest first balances the GPU); may be NULL for 0..num_seqs-1.
 * Replaces qwen35moe_gdn_prefill_bf16tc (kernels_optimized/qwen35moe_gdn_prefill.cu:1203-1264),
 * which supported only fp32 I/O, a batch of equal lengths, heads_k=16, heads_v=32. */
int tokmix_gdn_prefill(const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* initial_state, void* out, float* final_state, const int32_t* cu_seqlens_dev,
                       const int32_t* seq_order_dev, int num_seqs, int total_tokens, int heads_k, int heads_v,
                       int head_dim_k, int head_dim_v, float scale, int io_dtype, const tokmix_gdn_stage1* gates,
                       uint32_t* status, void* stream);

/* Gated-delta-rule prefill for a batch of equal-length sequences that allocates nothing.
 *
 * For callers that cannot allocate device memory while they run an op (graph executors that
 * plan every buffer in advance, C / FFI callers without a device allocator).  Same maths and
 * arguments as tokmix_gdn_prefill with batched layout q, k [batch, seqlen, heads_k, 128],
 * v, out [batch, seqlen, heads_v, 128], g, beta [batch, seqlen, heads_v], states
 * [batch, heads_v, 128, 128]; the per-sequence token offsets (and the device status word when
 * `status` is NULL) live in a library-owned device array of about 16 KB per device instead of
 * caller memory.  batch must be <= 4095.  The first call on a device looks up that array's
 * address on the current device; make it before capturing the stream into a CUDA graph.  The
 * address is kept for the life of the process: after cudaDeviceReset (or anything else that
 * replaces the device's primary context) reload the library before calling again.  All calls on
 * a device share the array: calls that may overlap on the GPU (different streams without
 * ordering) race on it.  With status == NULL each call clears the library's status word when it
 * starts and the kernels' timeout bits go there; read it with tokmix_gdn_noalloc_status after
 * synchronising.  Every argument check runs before anything is enqueued.  No counterpart in the
 * reference. */
int tokmix_gdn_prefill_noalloc(const void* q, const void* k, const void* v, const float* g, const float* beta,
                               const float* initial_state, void* out, float* final_state, int batch, int seqlen,
                               int heads_k, int heads_v, int head_dim_k, int head_dim_v, float scale, int io_dtype,
                               uint32_t* status, void* stream);

/* The library-owned status word of the current device that tokmix_gdn_prefill_noalloc writes
 * when it is called with status == NULL: copied to *host_status synchronously (call it after
 * synchronising the stream of the prefill), then zeroed if clear != 0.  Allocates nothing.  No
 * counterpart in the reference. */
int tokmix_gdn_noalloc_status(uint32_t* host_status, int clear);

/* Gated-delta-rule prefill in two launches, for problems with few (sequence, value head) units
 * (fewer than the GPU has SMs): a chunk-parallel preparation kernel (one CTA per chunk and value
 * head) writes every chunk's tensor-core operands to `workspace`; a state-chain kernel (one CTA
 * per sequence and value head) consumes them.  Same maths, arguments and results as
 * tokmix_gdn_prefill (up to fp32 summation order), plus:
 *   chunk_base_dev:   device int32 [num_seqs + 1], chunk_base[n] = sum over m < n of
 *                     ceil(len_m / 64); chunk_base[num_seqs] = total_chunks
 *   record_order_dev: device int32 [total_chunks * heads_v] or NULL: the records
 *                     (global chunk * heads_v + value head) in chunk-major order (chunk 0 of every
 *                     sequence and head first).  When given and the device can run it, both
 *                     stages share ONE cooperative launch: chain CTAs consume each chunk's record
 *                     as soon as preparation CTAs on the other SMs have written it.  NULL (or a
 *                     device where the cooperative launch is refused) gives two ordinary launches.
 *   checkpoints:      NULL, or device fp32 [total_chunks, heads_v, 128, 128]: the state after each
 *                     chunk, checkpoints[chunk_base[n] + c] = the state of sequence n after its
 *                     tokens [0, 64 (c + 1)) (its last entry equals that sequence's final state)
 *   workspace:        device memory of at least tokmix_gdn_split_workspace_bytes(total_chunks,
 *                     heads_v) bytes, 16-byte aligned (contents need no initialisation)
 * No counterpart in the reference (its prefill is one kernel chain per layer call). */
int tokmix_gdn_prefill_split(const void* q, const void* k, const void* v, const float* g, const float* beta,
                             const float* initial_state, void* out, float* final_state, float* checkpoints,
                             const int32_t* cu_seqlens_dev, const int32_t* chunk_base_dev, const int32_t* record_order_dev, int num_seqs,
                             int total_tokens, int total_chunks, int heads_k, int heads_v, int head_dim_k,
                             int head_dim_v, float scale, int io_dtype, const tokmix_gdn_stage1* gates,
                             void* workspace, long long workspace_bytes, uint32_t* status, void* stream);

/* Workspace size of tokmix_gdn_prefill_split in bytes (-1 for negative arguments). */
long long tokmix_gdn_split_workspace_bytes(int total_chunks, int heads_v);

/* Gated-delta-rule prefill with long sequences cut into segments that run side by side, for
 * problems whose longest sequence would otherwise set the time (a few long sequences, or a
 * head slice of them on one GPU of several).  Same maths, arguments and results as
 * tokmix_gdn_prefill (up to fp32 summation order and one extra bf16 rounding of the outputs of
 * later segments), plus:
 *   cu_seqlens_host:    host int32 [num_seqs + 1], the same offsets as cu_seqlens_dev (the
 *                       segment plan is made on the host)
 *   chunk_base_dev:     as for tokmix_gdn_prefill_split
 *   max_segment_chunks: a sequence of more than this many 64-token chunks is cut into the
 *                       fewest near-equal segments of at most this many chunks
 *   plan_dev:           NULL, or a device copy (16-byte aligned) of the tables that
 *                       tokmix_gdn_segmented_plan writes for the same offsets, heads_v and
 *                       max_segment_chunks (kept by a caller that repeats a shape); with NULL the
 *                       call uploads them into the workspace itself, from pageable host memory,
 *                       which makes the host wait for the stream
 *   workspace:          device memory of tokmix_gdn_segmented_workspace_bytes(...) bytes,
 *                       16-byte aligned (preparation records, the segments' transition
 *                       outputs and states, room for the plan's tables)
 * Four launches on `stream`: chunk-parallel preparation; one state chain per segment and value
 * head -- the first segment from the sequence's initial state, every later segment twice, from a
 * zero state (its own contribution) and from the identity with zero values (its transition,
 * whose end state and outputs are linear in the segment's true entry state); a combine kernel
 * that chains the entry states E(j+1) = E(j) M(j) + N(j) in fp32 and writes the final states;
 * and a tensor-core GEMM that adds each later segment's entry-state share R E^T to its outputs.
 * No counterpart in the reference (its chunk scan runs each sequence's chunks in order,
 * kernels_optimized/qwen35moe_gdn_prefill.cu:1131-1153). */
int tokmix_gdn_prefill_segmented(const void* q, const void* k, const void* v, const float* g, const float* beta,
                                 const float* initial_state, void* out, float* final_state,
                                 const int32_t* cu_seqlens_dev, const int32_t* chunk_base_dev,
                                 const int32_t* cu_seqlens_host, int num_seqs, int total_tokens, int total_chunks,
                                 int heads_k, int heads_v, int head_dim_k, int head_dim_v, float scale, int io_dtype,
                                 const tokmix_gdn_stage1* gates, int max_segment_chunks, const void* plan_dev,
                                 void* workspace, long long workspace_bytes, uint32_t* status, void* stream);

/* Workspace size of tokmix_gdn_prefill_segmented in bytes (-1 for inconsistent arguments). */
long long tokmix_gdn_segmented_workspace_bytes(const int32_t* cu_seqlens_host, int num_seqs, int heads_v,
                                               int max_segment_chunks);

/* Size in bytes of the segment plan's tables (-1 for inconsistent arguments), and the tables
 * written to plan_host (host memory of at least that size), for a device copy passed as
 * tokmix_gdn_prefill_segmented's plan_dev. */
long long tokmix_gdn_segmented_plan_bytes(const int32_t* cu_seqlens_host, int num_seqs, int heads_v,
                                          int max_segment_chunks);
int tokmix_gdn_segmented_plan(const int32_t* cu_seqlens_host, int num_seqs, int heads_v, int max_segment_chunks,
                              void* plan_host, long long plan_bytes);

/* One decode step of the gated delta rule: one new token per sequence, bf16 in and out, fp32 state.
 *
 *   for every sequence b, value head h (key head h % heads_k) and value row c:
 *   gamma = exp(g);  kv = S[c] . k;  delta = (v[c] - gamma kv) beta
 *   S[c] = gamma S[c] + delta k;  out[c] = scale (S[c] . q)            (with the updated S)
 *
 * q, k: [batch, heads_k, 128]; v, out: [batch, heads_v, 128]; g, beta: [batch, heads_v] fp32;
 * state_in (NULL = zero state) and state_out: [batch, heads_v, 128 (v), 128 (k)] fp32 -- the
 * reference's [v_col, k_row] layout; state_out may equal state_in (update in place).  All
 * tensors contiguous and 16-byte aligned.  Same maths as one token of tokmix_gdn_prefill.
 * Replaces the single-token step the reference takes inside its prefill
 * (kernels_optimized/qwen35moe_gdn_prefill.cu:865-934; maths kernels/qwen35moe_gdn_prefill.cu:55-99). */
int tokmix_gdn_decode(const void* q, const void* k, const void* v, const float* g, const float* beta,
                      const float* state_in, float* state_out, void* out, int batch, int heads_k, int heads_v,
                      int head_dim_k, int head_dim_v, float scale, int io_dtype, void* stream);

/* Per-row L2 normalisation (the GDN qk_l2norm option): y[r] = x[r] / sqrt(sum x[r]^2 + eps), fp32
 * arithmetic.  x: [rows, dim] bf16 (x_dtype TOKMIX_DTYPE_BF16) or fp32; y: [rows, dim] bf16; dim
 * must be 128; both 16-byte aligned.  The reference leaves this step to its caller
 * (kernels/qwen35moe_gdn_prefill.py:107-136 takes normalised q and k). */
int tokmix_l2norm_rows(const void* x, int x_dtype, void* y, long long rows, int dim, float eps, void* stream);

/* The Qwen3.5 gated-delta-net gates from the raw projections (the GDN gates option):
 *   g = -exp(a_log[h]) * softplus(a + dt_bias[h]),  beta = sigmoid(b)      (fp32 arithmetic)
 * a, b: [tokens, heads_v] bf16 (ab_dtype TOKMIX_DTYPE_BF16) or fp32; a_log, dt_bias: [heads_v] fp32;
 * g, beta: [tokens, heads_v] fp32 outputs.  The reference takes g and beta ready-made
 * (kernels/qwen35moe_gdn_prefill.py:107-136). */
int tokmix_gdn_gates(const void* a, const void* b, int ab_dtype, const float* a_log, const float* dt_bias, float* g,
                     float* beta, long long tokens, int heads_v, void* stream);

/* ---- the harness's other registered row-wise ops (HBM-bound; no counterpart kernels in the
 * reference, whose configs check them against references/<op>.py) ---- */

/* RMS norm (references/rms_norm.py:6-10): out = x / sqrt(mean(x^2) + eps) * weight, fp32 arithmetic.
 * x, out: [rows, n]; weight: [n]; dtype TOKMIX_DTYPE_BF16 or TOKMIX_DTYPE_FP16; n a multiple of 8. */
int tokmix_rms_norm(const void* x, const void* weight, void* out, int rows, int n, int dtype, float eps,
                    void* stream);

/* SwiGLU with FP8 input quantisation (references/swiglu_input_quant.py:6-30).  x: [m, 2n] bf16 = [x0 | x1];
 * out: [m, n] bf16 = bf16(x0 * x1 * sigmoid(x1)) (fp32 arithmetic); x_fp8: [m, 2n] e4m3 =
 * e4m3(bf16(x * bf16(1 / scale))) with scale = max(amax |block|, eps) / 448 per 128-column block;
 * x_scale: [2n / 128, m] fp32.  n must be a multiple of 128. */
int tokmix_swiglu_input_quant(const void* x, void* out, void* x_fp8, float* x_scale, int m, int n, float eps,
                              void* stream);

/* Partial rotary embedding of packed QKV (references/qkv_part_rope.py:6-45).  qkv, out: [batch, seq, heads,
 * head_dim] bf16; cos, sin: [seq, (head_dim - nope_dim) / 2] fp32.  out = qkv with the last head_dim - nope_dim
 * columns of the first q_heads + kv_heads heads rotated: (x0, x1) -> (x0 cos - x1 sin, x0 sin + x1 cos) over
 * the column pairs (j, j + half); negative_sin != 0 negates sin.  head_dim, nope_dim multiples of 8. */
int tokmix_qkv_part_rope(const void* qkv, const float* cos, const float* sin, void* out, int batch, int seq, int heads,
                         int head_dim, int q_heads, int kv_heads, int nope_dim, int negative_sin, void* stream);

/* Self-test of the bounded waits every pipelined kernel relies on: one small kernel waits on an
 * event that never happens -- which = 0: a transaction barrier whose bytes never land (a TMA load
 * that never completes; sets TOKMIX_DEV_TIMEOUT_TMA), 1: a hand-off barrier missing an arrival
 * (TOKMIX_DEV_TIMEOUT_PIPE), 2: the ready flag *flag (device uint32; TOKMIX_DEV_TIMEOUT_PIPE while
 * it stays 0, success if the caller set it) -- with a limit of limit_ns (1e3 .. 1e9 ns), while a
 * second warp waits on the same event with the library's own 2 s limit and must stop as soon as
 * the first gives up.  result (device int32[2] or NULL) receives what each warp's wait returned
 * (1 satisfied, 0 gave up); *status (device uint32) the bits.  Nothing is in flight in this
 * kernel, so the run ends cleanly.  The reference's counterpart is host-side only (its bench
 * harness puts a timeout around each run, tools/bench.py:138-169). */
int tokmix_selftest_wait_timeout(int which, long long limit_ns, const uint32_t* flag, int32_t* result,
                                 uint32_t* status, void* stream);

/* Text of the last error reported on the calling thread ("" if none). */
const char* tokmix_last_error(void);

/* Library version string, e.g. "tokmix 0.1.0 sm_100a". */
const char* tokmix_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TOKMIX_H_ */
