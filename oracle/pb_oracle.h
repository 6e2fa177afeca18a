/*
 * pb_oracle.h - CPU restatement of sammcj/purebee's quantized Llama hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * library and the timed CPU baseline of bench.py.  The product path never
 * links or calls it.  Each function names the reference file:line it follows.
 *
 * Arithmetic conventions (the reference is JavaScript):
 *   - scalar JS code computes in IEEE double and rounds to float when a value
 *     is stored into a Float32Array; here that is `double` plus a (float) cast;
 *   - the WASM SIMD kernels compute in float with separate multiply and add
 *     (no FMA) in a fixed lane order; here that is `float` code built with
 *     -ffp-contract=off.
 *
 * Parity pinning: the reference cannot run in this image (no JavaScript
 * engine).  The restatement is pinned by the reference's own known-answer
 * tests (wasm-q4.js:673-704, wasm-simd.js:367-385, main.js:65-96), replayed in
 * tests/test_oracle_kat.py, and cross-checked against the reference's
 * double-precision JS fallback kernels (llama-streaming.js:72-151).
 */
#ifndef PB_ORACLE_H
#define PB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- threading (bit-neutral row splits, thread-pool.js:165-246) ---- */
void orc_set_threads(int n);
int orc_get_threads(void);

/* ---- f16 decode ---- */
float orc_f16_exact(uint16_t bits);   /* gguf.js:55-70 */
float orc_f16_wasm(uint16_t bits);    /* wasm-q4.js:88-109 */
uint16_t orc_f32_to_f16(float f);     /* IEEE round-to-nearest-even encode */

/* ---- GGUF block decode (gguf.js:219-315) ---- */
void orc_dequant_q4_0(const uint8_t* raw, int64_t n, float* out);
void orc_dequant_q4_1(const uint8_t* raw, int64_t n, float* out);
void orc_dequant_q8_0(const uint8_t* raw, int64_t n, float* out);
void orc_dequant_f16(const uint8_t* raw, int64_t n, float* out);
void orc_dequant_q6_k(const uint8_t* raw, int64_t n, float* out); /* gguf.js:317-355 */

/* ---- GGUF block encode (not in the reference; the build's own definition) ---- */
void orc_quantize_gguf_q4_0(const float* x, int64_t n, uint8_t* out);
void orc_quantize_gguf_q8_0(const float* x, int64_t n, uint8_t* out);

/* ---- quantized matvecs ---- */
void orc_q4_0_matvec_wasm(const float* x, const uint8_t* raw, int N, int K, float* y); /* wasm-q4.js:118-267 */
void orc_q4_1_matvec_wasm(const float* x, const uint8_t* raw, int N, int K, float* y); /* wasm-q4.js:275-435 */
void orc_q4_0_matvec_js(const float* x, const uint8_t* raw, int N, int K, float* y);   /* llama-streaming.js:72-104 */
void orc_q4_1_matvec_js(const float* x, const uint8_t* raw, int N, int K, float* y);   /* llama-streaming.js:115-151 */

/* ---- f32 kernels ---- */
void orc_batch_dot(const float* x, const float* W, int N, int K, float* out);           /* wasm-q4.js:447-566 */
void orc_matmul_wasm(const float* A, int M, int K, const float* B, int N,
                     const float* bias, float* C);                                       /* wasm-simd.js:71-91, 469-506 */

/* ---- quantize.js format (a) ---- */
void orc_quantize_q8a(const float* data, int64_t n, float* scales, int8_t* q);          /* quantize.js:79-109 */
void orc_quantize_q4a(const float* data, int64_t n, float* scales, uint8_t* q);         /* quantize.js:124-161 */
void orc_dequantize_q8a(const float* scales, const int8_t* q, int64_t n, float* out);    /* quantize.js:170-181 */
void orc_dequantize_q4a(const float* scales, const uint8_t* q, int64_t n, float* out);  /* quantize.js:189-208 */
void orc_matmul_q8(const float* a, int M, int K, const float* scales, const int8_t* q, int N,
                   const float* bias, float* out);                                       /* quantize.js:224-266 */

/* ---- engine.js ops ---- */
void orc_rmsnorm(const float* x, int seq, int dim, const float* w, double eps, float* out); /* engine.js:429-449 */
void orc_softmax(const float* in, int rows, int cols, float* out);                         /* engine.js:279-303 */
void orc_layernorm(const float* x, int seq, int dim, const float* w, const float* b,
                   double eps, float* out);                                                /* engine.js:315-344 */
void orc_gelu(const float* x, int64_t n, float* out);                                      /* engine.js:354-360 */
void orc_silu(const float* x, int64_t n, float* out);                                      /* engine.js:459-463 */
void orc_elementmul(const float* a, const float* b, int64_t n, float* out);                /* engine.js:474-484 */
void orc_tensoradd(const float* a, const float* b, int64_t n, float* out);                 /* engine.js:96-106 */
void orc_attention(const float* Q, const float* K, const float* V, int seqQ, int seqK, int dK,
                   int dV, int causal, float* out);                                        /* engine.js:374-415 */

/* ---- llama pieces ---- */
void orc_rope(float* q, float* k, int seq, int start_pos, int dim, int n_heads, int n_kv,
              int head_dim, double theta);                                                 /* llama-streaming.js:310-339 */
void orc_attn_cached(const float* q, const float* kcache, const float* vcache, int seq,
                     int start_pos, int dim, int n_heads, int n_kv, int head_dim, float* out); /* llama-streaming.js:422-464, 543-573 */
void orc_swiglu_fused(const float* g, const float* u, int n, float* out);                  /* llama-streaming.js:590-595 */
int orc_argmax(const float* logits, int n);                                                /* llama-streaming.js:899-909 */

/* ---- synthetic inputs (same generator as the CUDA library) ---- */
void orc_synth_weights(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, double stdev);
void orc_synth_activation(float* out, int64_t n, uint64_t seed, uint64_t stream);
void orc_synth_tokens(int* out, int n, uint64_t seed, int lo, int hi);

/* ---- whole model ---- */
enum { ORC_KIND_STREAMING_Q4 = 0, ORC_KIND_LLAMA_Q8A = 1 };
enum { ORC_EMB_Q4_0 = 2, ORC_EMB_Q8_0 = 8, ORC_EMB_F32 = 0 };

typedef struct orc_config {
  int kind;        /* ORC_KIND_* */
  int emb_type;    /* ORC_EMB_* (streaming: Q4_0 or Q8_0; llama.js: F32) */
  int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab, seq_len;
  double rope_theta;
  double eps;
} orc_config;

typedef struct orc_model orc_model;

orc_model* orc_model_create(const orc_config* cfg);
void orc_model_free(orc_model* m);
/* Fill every tensor from the synthetic generator (weights N(0, stdev), norm gains 1). */
void orc_model_init_synthetic(orc_model* m, uint64_t seed, double stdev);
/* Raw tensor storage access (GGUF bytes for the streaming kind, Q8a for llama.js).
 * which: 0 = embedding, 1..7 = wq wk wv wo w1 w2 w3; returns bytes and a pointer. */
uint8_t* orc_model_tensor(orc_model* m, int layer, int which, int64_t* nbytes);
float* orc_model_q8a_scales(orc_model* m, int layer, int which, int64_t* count);
/* Re-derive cached f32 tables after raw bytes were replaced. */
void orc_model_refresh(orc_model* m);
/* Untied LM head from GGUF bytes (emb_type ORC_EMB_Q4_0 / ORC_EMB_Q8_0), or an
 * f32 table (ORC_EMB_F32, already dequantized). */
int orc_model_set_head(orc_model* m, int emb_type, const uint8_t* raw);
/* llama-streaming.js:868-894 sample() with the uniform draw r given. */
int orc_sample(const float* logits, int V, int topK, double temperature, double r);
double orc_sample_uniform(uint64_t seed, uint64_t counter);
/* forward(tokens, startPos) -> logits[vocab] (llama-streaming.js:738-815, llama.js:204-371) */
int orc_forward(orc_model* m, const int* tokens, int n, int start_pos, float* logits);
/* forward(tokenIds, startPos, {maxLayers}) with the early exit
 * (llama-streaming.js:746-803); exit_threshold 0 turns it off. */
int orc_forward_ex(orc_model* m, const int* tokens, int n, int start_pos, int max_layers, double exit_threshold,
                   int exit_interval, float* logits, int* layers_used);
double orc_exit_prob(const float* logits, int V);
/* generate, greedy (llama-streaming.js:914-970, llama.js:452-505); returns tokens written */
int orc_generate(orc_model* m, const int* prompt, int n_prompt, int max_tokens, int eos_id,
                 int* out_tokens, int out_cap);
void orc_reset_cache(orc_model* m);              /* llama-streaming.js:828-837 */
void orc_rollback_cache(orc_model* m, int pos);  /* llama-streaming.js:845-862 */
float* orc_kv(orc_model* m, int layer, int which_v);

#ifdef __cplusplus
}
#endif
#endif
