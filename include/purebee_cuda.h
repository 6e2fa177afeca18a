/*
 * purebee_cuda.h - C ABI of the B200 (sm_100a) backend for PureBee's
 * quantized Llama inference path.
 *
 * Plain C: opaque handles, plain pointers and sizes.  Every entry point
 * returns PB_OK (0) or a PB_ERR_* status; pb_last_error() gives the message.
 * There is no CPU fallback: every compute entry point runs a CUDA kernel.
 *
 * Pointer conventions:
 *   - arguments named *_host are host memory (copied in or out by the call);
 *   - arguments named *_dev are device memory from pb_malloc (or any device
 *     allocation on the context's device);
 *   - calls that only take device pointers are asynchronous on the context
 *     stream; calls that return host data block until it is ready, with the
 *     deadline set by pb_set_timeout_ms (PB_ERR_TIMEOUT when it passes).
 *
 * Each declaration names the reference interface it replaces (file:line in
 * sammcj/purebee).
 */
#ifndef PUREBEE_CUDA_H
#define PUREBEE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PB_ABI_VERSION 1

/* status codes (the reference throws Error with a message; the shim maps a
 * non-zero status plus pb_last_error() to `throw new Error(msg)`) */
#define PB_OK 0
#define PB_ERR_ARG 1      /* bad argument (engine.js:97, engine.js:122 size checks) */
#define PB_ERR_OOM 2      /* device allocation failed */
#define PB_ERR_CUDA 3     /* CUDA runtime error */
#define PB_ERR_TIMEOUT 4  /* host wait passed its deadline (thread-pool.js:232-238) */
#define PB_ERR_DEVICE 5   /* a kernel raised its error word (bounds, bounded wait) */
#define PB_ERR_STATE 6    /* call not valid in the current state */
#define PB_ERR_NOTFOUND 7 /* name not in memory (memory.js:126) */

/* GGML tensor types (gguf.js:30-33) */
#define PB_TYPE_F32 0
#define PB_TYPE_F16 1
#define PB_TYPE_Q4_0 2
#define PB_TYPE_Q4_1 3
#define PB_TYPE_Q8_0 8
/* GGUF decode only (pb_gguf_dequant; a model loads a Q6_K embedding or
 * output.weight as a dequantized f32 table, as streaming-loader.js:324-335
 * does): 256-value blocks of 210 bytes, gguf.js:317-355. */
#define PB_TYPE_Q6_K 14
/* OR'ed into the type of pb_qmat_upload / pb_qmat_from_device: store the
 * matrix as a table read one row per lane (the layout pb_qmat_head needs)
 * instead of the matvec layout. */
#define PB_QMAT_TABLE 0x100

typedef struct pb_ctx pb_ctx;
typedef struct pb_qmat pb_qmat;
typedef struct pb_model pb_model;

/* ------------------------------------------------------------------ */
/* context                                                              */
/* ------------------------------------------------------------------ */

/* Replaces wasm-q4.js:647-668 init() / wasm-simd.js:339-362 init(): binds a
 * device, creates the stream, runs the Q4_0 self-test (wasm-q4.js:673-704). */
int pb_init(int device, pb_ctx** out);
int pb_shutdown(pb_ctx* ctx);
const char* pb_last_error(const pb_ctx* ctx);
int pb_abi_version(void);
/* Host-wait deadline for blocking calls (default 10000 ms). */
int pb_set_timeout_ms(pb_ctx* ctx, int timeout_ms);
/* purebee.js:193-197 SYNC(): wait for all queued work, bounded by the deadline. */
int pb_sync(pb_ctx* ctx);
/* The cudaStream_t the context enqueues on, as an opaque pointer. */
void* pb_stream(pb_ctx* ctx);
/* Device error word: non-zero once a kernel recorded an error. */
int pb_device_error(pb_ctx* ctx, int* code_out);
/* Kernel launches issued by this context so far. */
int64_t pb_launch_count(pb_ctx* ctx);

/* Record the device-pointer calls made on the context between
 * pb_capture_begin and pb_capture_end into a replayable graph (no
 * counterpart in the reference, which has no device: this is how a caller
 * replays a fixed sequence of calls, a layer loop or a benchmark loop,
 * without paying the host launch cost per call).  Only calls that take
 * device pointers may be recorded; calls that copy host data or wait return
 * an error while recording.  pb_graph_launch enqueues one replay on the
 * context stream. */
typedef struct pb_graph pb_graph;
int pb_capture_begin(pb_ctx* ctx);
int pb_capture_end(pb_ctx* ctx, pb_graph** out);
int pb_graph_launch(pb_ctx* ctx, pb_graph* g);
int pb_graph_free(pb_graph* g);

/* ------------------------------------------------------------------ */
/* device memory (memory.js:87-155 PureBeeMemory, now device resident)   */
/* ------------------------------------------------------------------ */

int pb_malloc(pb_ctx* ctx, size_t bytes, void** dptr);
int pb_free(pb_ctx* ctx, void* dptr);
/* memory.js:102-121 write(): host -> device (blocking on completion) */
int pb_upload(pb_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
/* memory.js:124-128 read(): device -> host (blocking, deadline) */
int pb_download(pb_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);
int pb_memset(pb_ctx* ctx, void* dst_dev, int value, size_t bytes);
int pb_memcpy_d2d(pb_ctx* ctx, void* dst_dev, const void* src_dev, size_t bytes);

/* ------------------------------------------------------------------ */
/* quantized matrices resident on the device                            */
/* ------------------------------------------------------------------ */

/* Upload GGUF blocks of an [N rows][K cols] matrix (K % 32 == 0) and repack
 * them into a device layout.  type: PB_TYPE_Q4_0, PB_TYPE_Q4_1 or
 * PB_TYPE_Q8_0, plus PB_QMAT_TABLE for an LM-head table (pb_qmat_head);
 * without it the matrix is laid out for pb_qmat_matvec.  Replaces the raw
 * cache of streaming-loader.js:119-162 / 245-262 (raw GGUF bytes kept
 * resident for the Q4 path). */
int pb_qmat_upload(pb_ctx* ctx, int type, const void* gguf_host, int N, int K, pb_qmat** out);
/* Same from GGUF bytes already on the device. */
int pb_qmat_from_device(pb_ctx* ctx, int type, const void* gguf_dev, int N, int K, pb_qmat** out);
/* Write the matrix back as GGUF bytes (bit-exact round trip). */
int pb_qmat_download_gguf(pb_ctx* ctx, const pb_qmat* m, void* gguf_host);
int pb_qmat_free(pb_ctx* ctx, pb_qmat* m);
int pb_qmat_info(const pb_qmat* m, int* type, int* N, int* K);

/* ------------------------------------------------------------------ */
/* the Q4 matvec and LM head (wasm-q4.js module API)                    */
/* ------------------------------------------------------------------ */

/* y[n] = sum_k W[n,k] x[k] over a resident Q4_0 / Q4_1 matrix, with the
 * f32 lane order of wasm-q4.js:118-267 / 275-435 (bit-exact).  Rows
 * [row0, row0 + rows) only, so a caller can split rows across devices like
 * thread-pool.js:165-246; rows <= 0 means all rows.  row0 must be a
 * multiple of 8 (rows are stored in 8-row tiles); anything else is
 * PB_ERR_ARG. */
int pb_qmat_matvec(pb_ctx* ctx, const pb_qmat* w, const float* x_dev, float* y_dev, int row0, int rows);
/* Arithmetic of the resident Q4_0 matvec: pb_qmat_matvec and every model
 * decode step on the context (a model re-records its step graph when the
 * mode changes).
 *   PB_MATVEC_FAST (default): the same exact (q - 8) * x products, summed
 *     with one FMA per weight in a different order: y within an f32
 *     relative tolerance of wasm-q4.js:118-267 (north_star's per-op bar),
 *     greedy tokens unchanged (tests check both over whole workloads);
 *   PB_MATVEC_EXACT: the WASM lane order with separate multiply and add,
 *     bit for bit (the parity mode).
 * pb_q4_0_matvec / pb_q4_1_matvec (the module functions) and Q4_1 matrices
 * always run the exact kernel. */
#define PB_MATVEC_FAST 0
#define PB_MATVEC_EXACT 1
int pb_set_matvec_mode(pb_ctx* ctx, int mode);
int pb_matvec_mode(const pb_ctx* ctx);
/* Fast mode, Q4_0 matrices in the row layout with a tensor-core copy: the
 * int8 tensor-core kernel runs the matvecs of a matrix of at least `rows`
 * rows, the f32 kernel those of smaller ones (default 32768: the LM head;
 * environment PB_MVI_MIN_ROWS at pb_init).  Both agree with the exact kernel
 * within the fast mode's tolerance.  A tuning knob with no counterpart in
 * the reference. */
int pb_set_mvi_min_rows(pb_ctx* ctx, int rows);
/* Fast mode: on = 1 runs the Q4_0 row-layout matvecs with K % 128 == 0 and
 * K <= 16384 on the tcgen05 int8 kernel (the same integer digits as the int8
 * kernel above, the products on the 5th-generation tensor cores) for the
 * matrices uploaded while it is on (they get the kernel's tile-contiguous
 * copy); other matrices, and every matrix with on = 0 (the default, as it
 * measures slower than the kernels above; environment PB_MVT=1 at pb_init
 * turns it on), take the choice pb_set_mvi_min_rows makes.  A tuning knob
 * with no counterpart in the reference. */
int pb_set_mvt(pb_ctx* ctx, int on);
/* Fast mode, the one-sequence decode step: on = 1 runs each layer's RMSNorm
 * -> q/k/v projection (RoPE, KV write) and its decode attention as one
 * kernel, the 8 CTAs attending for a kv head computing that head group's
 * projection rows first; the same bits as the two kernels.  Off by default
 * (environment PB_FUSE_ATTN=1 at pb_init turns it on): measured slower, the
 * projection then runs on 64 SMs.  Recorded decode graphs are re-recorded
 * after a change.  A tuning knob with no counterpart in the reference. */
int pb_set_fuse_attn(pb_ctx* ctx, int on);
/* wasm-q4.js:716-747 q4_0_matvec(x, rawBuf, N, K): host buffers in and out. */
int pb_q4_0_matvec(pb_ctx* ctx, const float* x_host, const uint8_t* raw_host, int N, int K, float* y_host);
/* wasm-q4.js:758-785 q4_1_matvec(x, rawBuf, N, K) */
int pb_q4_1_matvec(pb_ctx* ctx, const float* x_host, const uint8_t* raw_host, int N, int K, float* y_host);
/* Batched form of the Q4_0 matvec (the batched prefill / decode config):
 * C[M][N] = X[M][K] . W[N][K]^T on the tensor cores (tcgen05, f16 operands,
 * f32 accumulation), W a resident Q4_0 matrix (either layout).  Each operand is
 * rounded to f16 once, so C agrees with the reference's f32 arithmetic
 * (wasm-q4.js:118-267, wasm-simd.js:71-91) within a relative tolerance, not
 * bit for bit.  x_dev 16-byte aligned, ldx a multiple of 4. */
int pb_q4_gemm(pb_ctx* ctx, const pb_qmat* w, const float* x_dev, int M, int ldx, float* c_dev, int ldc);
/* The same product with f16 activations x16_dev [M][K] (row-major, device):
 * M <= 64 runs the warp-specialised decode-size kernel (TMA-fed Q4_0 payload
 * and activations, half-precision dequant with the same values as the
 * fused kernel), M >= 512 the persistent TMA kernel.  With the activations
 * already rounded to f16, M <= 64 gives the same bits as pb_q4_gemm. */
int pb_q4_gemm_f16(pb_ctx* ctx, const pb_qmat* w, const void* x16_dev, int M, float* c_dev, int ldc);
/* pb_q4_gemm with a precision choice: terms == 1 is pb_q4_gemm; terms == 3
 * splits both operands into f16 pairs, hi = f16(v) and lo = f16(v - hi) (the
 * weight value (q-8)*d splits exactly, x keeps about 22 bits), and sums
 * hi*hi + hi*lo + lo*hi on the tensor cores, for three times the tensor-core
 * work.  C then agrees with the reference's f32 arithmetic within the
 * tensor cores' f32 accumulation error.  The batched model uses terms == 3.
 * Both forms decode the block scale as wasm-q4.js:88-109 does (a zero
 * exponent is +0). */
int pb_q4_gemm_ex(pb_ctx* ctx, const pb_qmat* w, const float* x_dev, int M, int ldx, float* c_dev, int ldc,
                  int terms);
/* The three-term product with activations already split: xhl_dev holds each
 * row of K values as 2K halves, per 64-wide K group its 64 hi halves then its
 * 64 lo halves (the layout the batched model's producers write).  M <= 64 or
 * M >= 512 with K % 64 == 0; the same bits as pb_q4_gemm_ex(terms = 3) on the
 * f32 activations the pairs came from. */
int pb_q4_gemm_hl(pb_ctx* ctx, const pb_qmat* w, const void* xhl_dev, int M, float* c_dev, int ldc);
/* wasm-q4.js:798-839 lmHead(hidden, embData, V, D): f32 row-major table on
 * the host, batch_dot lane order (wasm-q4.js:447-566). */
int pb_lm_head(pb_ctx* ctx, const float* h_host, const float* emb_host, int V, int D, float* logits_host);
/* Head over a resident table (Q4_0 / Q8_0, uploaded with PB_QMAT_TABLE;
 * dequantized exactly as gguf.js:239-286 does), batch_dot lane order, fused
 * greedy argmax (llama-streaming.js:899-909).  argmax_dev may be NULL. */
int pb_qmat_head(pb_ctx* ctx, const pb_qmat* emb, const float* h_dev, float* logits_dev, int* argmax_dev);
/* argmax over logits: first index of the strict maximum. */
int pb_argmax(pb_ctx* ctx, const float* logits_dev, int n, int* idx_dev);

/* ------------------------------------------------------------------ */
/* engine.js / purebee.js operators on device buffers                   */
/* ------------------------------------------------------------------ */

/* engine.js:119-167 / 180-244 TENSOR_MUL and LINEAR with f32 weights:
 * C[M,N] = bias + A[M,K] B[K,N], f32 multiply then add per k in k order
 * (wasm-simd.js:71-91).  bias_dev may be NULL. */
int pb_matmul_f32(pb_ctx* ctx, const float* A_dev, int M, int K, const float* B_dev, int N,
                  const float* bias_dev, float* C_dev);
/* engine.js:259-269 -> quantize.js:224-266 matmul_q8 (LINEAR on a
 * QuantizedTensor): W is quantize.js format (a) over a flat [K,N] array. */
int pb_matmul_q8a(pb_ctx* ctx, const float* A_dev, int M, int K, const float* scales_dev,
                  const int8_t* q_dev, int N, const float* bias_dev, float* out_dev);
int pb_rmsnorm(pb_ctx* ctx, const float* x_dev, int seq, int dim, const float* w_dev, double eps,
               float* out_dev);                                         /* engine.js:429-449 */
int pb_softmax(pb_ctx* ctx, const float* in_dev, int rows, int cols, float* out_dev); /* engine.js:279-303 */
int pb_layernorm(pb_ctx* ctx, const float* x_dev, int seq, int dim, const float* w_dev,
                 const float* b_dev, double eps, float* out_dev);       /* engine.js:315-344 */
int pb_gelu(pb_ctx* ctx, const float* x_dev, int64_t n, float* out_dev);         /* engine.js:354-360 */
int pb_silu(pb_ctx* ctx, const float* x_dev, int64_t n, float* out_dev);         /* engine.js:459-463 */
int pb_elementmul(pb_ctx* ctx, const float* a_dev, const float* b_dev, int64_t n, float* out_dev); /* engine.js:474-484 */
int pb_tensoradd(pb_ctx* ctx, const float* a_dev, const float* b_dev, int64_t n, float* out_dev);  /* engine.js:96-106 */
int pb_attention(pb_ctx* ctx, const float* Q_dev, const float* K_dev, const float* V_dev, int seqQ, int seqK,
                 int dK, int dV, int causal, float* out_dev);           /* engine.js:374-415 */
/* pb_attention without allocating: no counterpart in the reference (it
 * computes the same engine.js:374-415 attention, bit for bit equal to
 * pb_attention).  pb_attention grows the context scratch on demand
 * (cudaFree + cudaMalloc, which synchronise the whole device); this call
 * instead keeps the seqQ x seqK scores and probabilities in one fixed device
 * array of PB_NOALLOC_ATTN_BYTES per device, whose address pb_init looks up,
 * so the call itself makes no allocation and no set-up.
 * Limits: 2 * (4 * seqQ * seqK rounded up to 256) <= PB_NOALLOC_ATTN_BYTES
 * (seqQ * seqK <= 524288) and seqQ <= 65535, else PB_ERR_ARG before anything
 * is launched (pb_attention has the same seqQ limit).
 * The array is shared by every context and stream on the device: calls that
 * overlap in time race on it, so the caller serialises them (one stream, or
 * an event between streams). */
#define PB_NOALLOC_ATTN_BYTES (4u << 20)
int pb_attention_noalloc(pb_ctx* ctx, const float* Q_dev, const float* K_dev, const float* V_dev, int seqQ,
                         int seqK, int dK, int dV, int causal, float* out_dev);
/* llama-streaming.js:310-339 _applyRoPE on q [seq, n_heads*hd], k [seq, n_kv*hd] in place */
int pb_rope(pb_ctx* ctx, float* q_dev, float* k_dev, int seq, int start_pos, int n_heads, int n_kv,
            int head_dim, double theta);
/* llama-streaming.js:422-464 / 543-573: attention of seq queries at
 * start_pos.. over a [seq_len, kv_dim] K/V cache (causal). */
int pb_attn_cached(pb_ctx* ctx, const float* q_dev, const float* kc_dev, const float* vc_dev, int seq,
                   int start_pos, int n_heads, int n_kv, int head_dim, float* out_dev);
/* llama-streaming.js:543-573: the attention of one query q [n_heads *
 * head_dim] at position pos over a [max_len, n_kv * head_dim] K/V cache
 * holding rows 0..pos, as the decode step runs it: the positions split over
 * the GPU's SMs, the splits merged in a fixed order.  In the exact matvec
 * mode, and for head_dim != 64, dots and sums run in double (the
 * reference's arithmetic, within an f32 rounding); in the fast mode
 * (head_dim 64, max_len <= 2048) in f32 with the splits of a kv head merged
 * through one thread-block cluster.  At most 8 query heads per kv head,
 * head_dim % 4 == 0 and <= 128.  Blocks until done. */
int pb_attn_decode(pb_ctx* ctx, const float* q_dev, const float* kc_dev, const float* vc_dev, int pos, int n_heads,
                   int n_kv, int head_dim, int max_len, float* out_dev);
/* llama-streaming.js:590-595 fused SiLU(gate)*up */
int pb_swiglu(pb_ctx* ctx, const float* g_dev, const float* u_dev, int n, float* out_dev);

/* ------------------------------------------------------------------ */
/* quantizers and decoders                                              */
/* ------------------------------------------------------------------ */

/* quantize.js:79-109 quantize_q8 / :124-161 quantize_q4 (format (a)) */
int pb_quantize_q8a(pb_ctx* ctx, const float* x_dev, int64_t n, float* scales_dev, int8_t* q_dev);
int pb_quantize_q4a(pb_ctx* ctx, const float* x_dev, int64_t n, float* scales_dev, uint8_t* q_dev);
/* quantize.js:170-208 dequantize_q8 / dequantize_q4 */
int pb_dequantize_q8a(pb_ctx* ctx, const float* scales_dev, const int8_t* q_dev, int64_t n, float* out_dev);
int pb_dequantize_q4a(pb_ctx* ctx, const float* scales_dev, const uint8_t* q_dev, int64_t n, float* out_dev);
/* gguf.js:219-355 loadTensorData for F32/F16/Q4_0/Q4_1/Q8_0/Q6_K blocks
 * (raw_dev holds ceil(n / block) whole blocks) */
int pb_gguf_dequant(pb_ctx* ctx, int type, const void* raw_dev, int64_t n, float* out_dev);
/* GGUF Q4_0 / Q8_0 block encoders (not in the reference, which only decodes
 * GGUF; used to build quantized synthetic models on the device). */
int pb_gguf_quantize(pb_ctx* ctx, int type, const float* x_dev, int64_t n, void* raw_dev);

/* ------------------------------------------------------------------ */
/* seeded synthetic inputs                                              */
/* ------------------------------------------------------------------ */

int pb_synth_weights(pb_ctx* ctx, float* out_dev, int64_t n, uint64_t seed, uint64_t tensor_id, double stdev);
int pb_synth_activation(pb_ctx* ctx, float* out_dev, int64_t n, uint64_t seed, uint64_t stream);
int pb_synth_tokens(int* out_host, int n, uint64_t seed, int lo, int hi);

/* ------------------------------------------------------------------ */
/* the model runtime (llama-streaming.js StreamingLlamaRuntime and       */
/* llama.js LlamaRuntime)                                               */
/* ------------------------------------------------------------------ */

#define PB_MODEL_STREAMING_Q4 0 /* GGUF Q4_0 layers (llama-streaming.js) */
#define PB_MODEL_LLAMA_Q8A 1    /* quantize.js Q8 layers, f32 embedding (llama.js) */

typedef struct pb_model_config {
  int kind;       /* PB_MODEL_* */
  int emb_type;   /* PB_TYPE_Q4_0 / PB_TYPE_Q8_0 (streaming) or PB_TYPE_F32 (llama.js) */
  int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab, seq_len;
  double rope_theta;
  double eps;
} pb_model_config;

int pb_model_create(pb_ctx* ctx, const pb_model_config* cfg, pb_model** out);
int pb_model_free(pb_model* m);
/* Random-init weights N(0, stdev) from the seed (device generator), norm
 * gains 1, quantized on the device. */
int pb_model_init_synthetic(pb_model* m, uint64_t seed, double stdev);
/* Set / get one tensor.  which: 0 embedding, 1..7 = wq wk wv wo w1 w2 w3,
 * 8 = attention norm, 9 = ffn norm (layer), 10 = final norm, 11 = untied LM
 * head (after pb_model_attach_head).  Streaming models take GGUF bytes;
 * llama.js models take (scales f32[], int8 q[]) packed back to back for 1..7
 * and f32 for the embedding. */
/* Give a streaming model its own LM head table (GGUF output.weight, Q4_0 or
 * Q8_0) instead of the tied embedding (streaming-loader.js:77-86
 * sharedWeights, llama-streaming.js:616-679). */
int pb_model_attach_head(pb_model* m, int type);
int pb_model_set_tensor(pb_model* m, int layer, int which, const void* host, size_t bytes);
int pb_model_get_tensor(pb_model* m, int layer, int which, void* host, size_t bytes);
/* llama-streaming.js:738-815 / llama.js:204-371 forward(tokens, startPos):
 * logits of the last position copied to logits_host (may be NULL). */
int pb_model_forward(pb_model* m, const int* tokens_host, int n, int start_pos, float* logits_host);
/* One graph-replayed decode step for token `token` at `pos`; writes the
 * greedy next token (llama-streaming.js:899-909). */
int pb_model_decode(pb_model* m, int token, int pos, int* next_host, float* logits_host);
/* llama-streaming.js:914-970 generate(prompt, maxTokens, {greedy, eosId}) */
int pb_model_generate(pb_model* m, const int* prompt_host, int n_prompt, int max_tokens, int eos_id,
                      int* out_host, int out_cap, int* n_out);
/* Device-resident decode loop for timing: `steps` greedy steps starting from
 * the token already in the model's token slot at `pos0`; tokens stay on the
 * device (out_dev may be NULL). */
int pb_model_decode_loop(pb_model* m, int pos0, int steps, int* out_dev);
/* forward(tokenIds, startPos, {maxLayers}) (llama-streaming.js:738-815):
 * only the first max_layers layers run (0: all), then the final norm and head;
 * the layers actually run (early exit included) go to layers_used. */
int pb_model_forward_ex(pb_model* m, const int* tokens_host, int n, int start_pos, int max_layers, float* logits_host,
                        int* layers_used);
int pb_model_decode_ex(pb_model* m, int token, int pos, int max_layers, int* next_host, float* logits_host,
                       int* layers_used);
/* options.earlyExitThreshold / earlyExitInterval (llama-streaming.js:202-203):
 * single-token steps check the top-8 confidence of the partial hidden state
 * every `interval` layers and stop at or above the threshold (0: off).  The
 * reference's check throws (an undefined `candidates`, :717); this is the
 * intended rule with tailCount = V - 8. */
int pb_model_set_early_exit(pb_model* m, double threshold, int interval);
int pb_model_exit_stats(const pb_model* m, int* layers_used, int* last_exit_layer, int* early_exits);
/* sample(logits, topK, temperature) over the logits of the last forward. */
int pb_model_sample(pb_model* m, int top_k, double temperature, uint64_t seed, uint64_t counter, int* token_host);
int pb_model_set_token(pb_model* m, int token);
int pb_model_reset_cache(pb_model* m);             /* llama-streaming.js:828-837 */
int pb_model_rollback_cache(pb_model* m, int pos); /* llama-streaming.js:845-862 */
int pb_model_kv(pb_model* m, int layer, int which_v, float* host, size_t floats);
/* Llama-3 RoPE frequency scaling, off by default.  The reference applies
 * none: llama-streaming.js:316-336 rotates by pos / theta^(i/hd), and
 * gguf.js:378-410 never maps rope_freqs.weight; so every parity check keeps
 * it off.  A caller that wants the published Llama 3.1 / 3.2 rule (Llama-3.2-1B:
 * factor 32, low_freq_factor 1, high_freq_factor 4, original_max_pos 8192)
 * turns it on here; factor <= 0 turns it off.  Pair frequency f, wavelength
 * w = 2 pi / f, C = original_max_pos: f if w < C / high; f / factor if
 * w > C / low; else (1 - s) f / factor + s f with s = (C / w - low) / (high - low). */
int pb_model_set_rope_scaling(pb_model* m, double factor, double low_freq_factor, double high_freq_factor,
                              int original_max_pos);
int pb_model_rope_scaling(const pb_model* m, double* factor_out); /* 0 when off */
/* The pair frequencies freqs_out[head_dim / 2] of that rule (host only, no
 * device needed; factor <= 0 gives the reference's 1 / theta^(i/hd)). */
int pb_rope_freqs(double theta, int head_dim, double factor, double low_freq_factor, double high_freq_factor,
                  int original_max_pos, double* freqs_out);
/* Algorithmic bytes one decode step reads at cache length `pos+1`. */
int64_t pb_model_decode_bytes(const pb_model* m, int pos);
/* Kernel launches of one decode step. */
int pb_model_decode_launches(const pb_model* m);

/* ------------------------------------------------------------------ */
/* sampling (llama-streaming.js:868-894 sample(logits, topK, temperature)) */
/* ------------------------------------------------------------------ */

/* Top-K of logits / temperature (ties to the lower index, as the stable JS
 * sort), softmax over them in double, then the first index whose running
 * probability reaches r.  The reference draws r from Math.random(); here r =
 * pb_sample_uniform(seed, counter), uniform in [0, 1) with 53 bits.
 * logits and token live on the device; enqueued on the context stream.
 * 0 < top_k <= 256, temperature > 0; NaN logits are never chosen. */
int pb_sample_topk(pb_ctx* ctx, const float* logits_dev, int V, int top_k, double temperature, uint64_t seed,
                   uint64_t counter, int* token_dev);
double pb_sample_uniform(uint64_t seed, uint64_t counter);
/* llama-streaming.js:914-970 generate(prompt, maxTokens, {temperature,
 * topK}) with device sampling: draw i uses pb_sample_uniform(seed, i) (the
 * prefill's token is draw 0); decode steps replay one recorded graph. */
int pb_model_generate_sampled(pb_model* m, const int* prompt_host, int n_prompt, int max_tokens, int eos_id, int top_k,
                              double temperature, uint64_t seed, int* out_host, int out_cap, int* n_out);

/* ------------------------------------------------------------------ */
/* GGUF files (gguf.js:76-194 GGUFParser, :402-424 extractConfig;        */
/* streaming-loader.js:35-87 parseHeader, :245-262 loadTensorRaw)        */
/* ------------------------------------------------------------------ */

/* A parsed GGUF v2/v3 file: metadata and the tensor index in host memory,
 * tensor bytes read on demand.  Errors: PB_ERR_ARG with the message in
 * pb_gguf_last_error() (the reference throws Error with a message). */
typedef struct pb_gguf pb_gguf;
const char* pb_gguf_last_error(void);
int pb_gguf_open(const char* path, pb_gguf** out);
int pb_gguf_close(pb_gguf* g);
int pb_gguf_version(const pb_gguf* g);
int64_t pb_gguf_data_start(const pb_gguf* g); /* aligned start of the tensor data */
int64_t pb_gguf_alignment(const pb_gguf* g);  /* general.alignment, default 32 */
/* Metadata: value types are GGUF's (0 u8 .. 12 f64; 8 string, 9 array).
 * String values are returned as borrowed pointers with their byte length.
 * Keys and tensor names are returned as NUL-terminated C strings: GGUF keys
 * are ASCII identifiers, and a name with an embedded NUL byte reads up to it. */
int pb_gguf_meta_count(const pb_gguf* g);
int pb_gguf_meta_find(const pb_gguf* g, const char* key); /* index or -1 */
int pb_gguf_meta_key(const pb_gguf* g, int i, const char** key);
int pb_gguf_meta_type(const pb_gguf* g, int i, int* type, int* arr_type, int64_t* arr_len);
int pb_gguf_meta_int(const pb_gguf* g, int i, int64_t* v);
int pb_gguf_meta_float(const pb_gguf* g, int i, double* v);
int pb_gguf_meta_string(const pb_gguf* g, int i, const char** s, int64_t* len);
int pb_gguf_meta_array_string(const pb_gguf* g, int i, int64_t j, const char** s, int64_t* len);
int pb_gguf_meta_array_number(const pb_gguf* g, int i, int64_t j, double* v);
/* Tensor index: dims[4] (unused dims 1), absolute file offset, byte size. */
int pb_gguf_tensor_count(const pb_gguf* g);
int pb_gguf_tensor_find(const pb_gguf* g, const char* name); /* index or -1 */
int pb_gguf_tensor_info(const pb_gguf* g, int i, const char** name, int* type, int* n_dims, int64_t* dims,
                        int64_t* file_offset, int64_t* bytes);
int pb_gguf_tensor_read(const pb_gguf* g, int i, void* host, size_t bytes);
/* extractConfig with the reference's defaults; vocab from the tokenizer's
 * token list; a streaming (Q4_0) model with a Q4_0 or Q8_0 embedding. */
int pb_gguf_config(const pb_gguf* g, pb_model_config* cfg);
/* Create a streaming model from the file (every tensor uploaded once into the
 * packed device layout; output.weight, when present, as an untied head).
 * seq_len > 0 overrides the file's context length. */
int pb_model_load_gguf(pb_ctx* ctx, const pb_gguf* g, int seq_len, pb_model** out);

/* ------------------------------------------------------------------ */
/* batched serving (the batched configuration; the reference serves one  */
/* sequence at a time, llama-streaming.js:738-815)                        */
/* ------------------------------------------------------------------ */

/* n_seqs (<= 256) independent sequences over a streaming model's weights
 * (Q4_0 embedding), each with its own KV cache.  The projections and the LM
 * head run as tensor-core GEMMs (pb_q4_gemm / pb_q4_gemm_f16: f16 operands,
 * f32 sums; decode steps of up to 64 sequences take the decode-size kernel),
 * so logits agree with the one-sequence path within a relative tolerance. */
typedef struct pb_batch pb_batch;
int pb_batch_create(pb_model* m, int n_seqs, pb_batch** out);
int pb_batch_free(pb_batch* b);
/* Prefill tokens_host [n_seqs][n_prompt] from position 0; next_host
 * [n_seqs] gets each sequence's greedy token, logits_host [n_seqs][vocab]
 * (optional) the last position's logits. */
int pb_batch_prefill(pb_batch* b, const int* tokens_host, int n_prompt, int* next_host, float* logits_host);
/* `steps` greedy decode steps of every sequence (one replayed CUDA graph per
 * step); tokens_host [steps][n_seqs] (optional) gets the generated tokens,
 * logits_host [n_seqs][vocab] (optional) the last step's logits. */
int pb_batch_decode(pb_batch* b, int steps, int* tokens_host, float* logits_host);
/* GEMM precision of the batch: 3 (the default) runs every projection and the
 * head as the three-term product of pb_q4_gemm_ex; 1 rounds each operand to
 * f16 once (a third of the tensor-core work, logits about 3e-3 of their
 * scale from the one-sequence path at the Llama-3.2-1B shape).  Set between
 * steps.  No counterpart in the reference, which serves one sequence. */
int pb_batch_set_precision(pb_batch* b, int terms);

/* ------------------------------------------------------------------ */
/* row split over GPUs (thread-pool.js:165-246 splits a matvec's output   */
/* rows over worker threads, thread-pool.js:174-203 for the row ranges;   */
/* here one rank per GPU holds a row range of every projection and of    */
/* the LM head, and in-place all-gathers complete the activations)       */
/* ------------------------------------------------------------------ */

/* Which rows rank `rank` of `world` holds.  Query heads and kv heads are
 * split evenly (each rank attends over its own heads and holds their KV
 * cache); wo and w2 by output rows in dim / world chunks, the interleaved
 * gate|up matrix in 2F / world row chunks (hidden units [rank*F/world, ...));
 * the vocab in chunks of vocab_chunk rows (a multiple of 32; the last rank
 * takes the rest).  Needs n_kv_heads, dim / 64 and hidden_dim / 64
 * divisible by world; PB_ERR_ARG otherwise.  Host only. */
typedef struct pb_split_plan {
  int world, rank;
  int n_heads, n_kv_heads;      /* this rank's heads */
  int q_row0, k_row0, v_row0;   /* first rows held of wq, wk, wv, as rows of [wq; wk; wv] */
  int qkv_rows;                 /* (n_heads + 2 n_kv_heads) * head_dim */
  int dim_chunk, hidden_chunk;  /* dim / world, hidden_dim / world */
  int vocab_row0, vocab_rows, vocab_chunk;
} pb_split_plan;
int pb_batch_split_plan(const pb_model_config* c, int world, int rank, pb_split_plan* out);

#define PB_COMM_ID_BYTES 128
typedef struct pb_comm pb_comm;
/* A new NCCL unique id (on one rank; the caller sends it to the others). */
int pb_comm_id(void* id_out);
/* Join communicator `id` as `rank` of `world` on ctx's device (collective
 * over the ranks).  Release every batch that uses it before pb_comm_free. */
int pb_comm_init(pb_ctx* ctx, int world, int rank, const void* id, pb_comm** out);
int pb_comm_free(pb_comm* c);
int pb_comm_rank(const pb_comm* c);
int pb_comm_world(const pb_comm* c);
/* recv_dev [world][bytes] <- every rank's send_dev [bytes], on ctx's stream */
int pb_comm_allgather(pb_comm* c, const void* send_dev, void* recv_dev, size_t bytes);
/* 1 when the ranks exchange over peer memory: pb_comm_init opened every
 * rank's buffers in every process (CUDA IPC over NVLink) and all ranks
 * agreed; then a row-split batch's all-gathers are one kernel each that
 * stores this rank's chunk into the peers' buffers and waits (bounded by the
 * context timeout) for theirs.  0: NCCL all-gathers (also with PB_NO_P2P=1). */
int pb_comm_peer_access(const pb_comm* c);
/* Register a device buffer (a whole pb_malloc allocation, the same size on
 * every rank; collective) for in-place all-gathers: pb_comm_allgather_inplace
 * sends chunk `rank` (chunk_bytes, a multiple of 8, from buf + rank *
 * chunk_bytes) to every rank's copy, over peer memory when the communicator
 * has peer access, else with NCCL. */
typedef struct pb_peerbuf pb_peerbuf;
int pb_comm_register(pb_comm* c, void* buf_dev, pb_peerbuf** out);
int pb_comm_deregister(pb_comm* c, pb_peerbuf* pb);
int pb_comm_allgather_inplace(pb_comm* c, pb_peerbuf* pb, size_t chunk_bytes);
/* The peer exchange kernels' bounded waits, on this device alone: two-rank
 * exchanges (the bulk kernel, then the low-latency one) whose peer never
 * signals.  Returns PB_OK with *raised_code = PB_DEVERR_WAIT (2) when both
 * waits gave up after about timeout_ms each (the device error word is then
 * cleared and the context stays usable), else the first other code seen. */
int pb_comm_selftest_wait(pb_ctx* ctx, int timeout_ms, int* raised_code);

/* This process's rank of a row-split batch over comm's ranks: every rank
 * calls prefill / decode with the same arguments (asking for logits_host on
 * every rank or on none: the logits are gathered collectively), and every
 * rank gets the same tokens and logits, with the same bits as
 * pb_batch_create on one GPU.  The exchanges are in-place all-gathers on the
 * context stream, four per layer plus the argmax keys, recorded into the
 * decode graph: one peer-memory kernel each when pb_comm_peer_access is 1,
 * else NCCL all-gathers. */
int pb_batch_create_split(pb_model* m, int n_seqs, pb_comm* comm, pb_batch** out);
/* All `world` ranks of a row split in this process, on ctx's one device,
 * with device copies in place of the all-gathers: the split's arithmetic on
 * one GPU (tests compare it with pb_batch_create bit for bit). */
int pb_batch_create_group(pb_model* m, int n_seqs, int world, pb_batch** out);

#ifdef __cplusplus
}
#endif
#endif
