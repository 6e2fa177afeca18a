// pb_model.cu - the Llama runtime of llama-streaming.js (GGUF Q4_0 layers)
// and llama.js (quantize.js Q8 layers) with every tensor resident on the
// device and the decode step captured in a CUDA graph.
//
// Decode step (seq == 1, llama-streaming.js:505-606), per layer:
//   rmsnorm -> fused [wq; wk; wv] Q4_0 matvec -> RoPE + KV append ->
//   attention over the cache -> wo matvec (+ residual epilogue) -> rmsnorm ->
//   fused [w1; w3] matvec -> SwiGLU -> w2 matvec (+ residual epilogue)
// then the final rmsnorm and the head with the fused argmax.  Position and
// token live in device memory, so one captured graph replays every step.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "pb_internal.cuh"
#include "pb_synth.h"

// from pb_ops.cu / pb_q4.cu
void pb_rope_table(double theta, int hd, int start, int n, double2* out);
void pb_rope_table_freqs(const double* freqs, int hd, int start, int n, double2* out);
int pb_launch_attn_cached(pb_ctx* ctx, const float* q, int q_stride, const float* kc, const float* vc, int seq,
                          int start_pos, const int* pos_dev, int n_heads, int n_kv, int hd, float* out, int max_len,
                          int nseq, pb_seq_geo geo);
int pb_launch_prefill_q4(pb_ctx* ctx, const pb_qmat* w, const float* X, int ldx, int M, float* C, int ldc);
int pb_launch_attn_decode(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                          int n_heads, int n_kv, int hd, float* out, int max_len, int nseq, pb_seq_geo geo,
                          float* ws = nullptr, size_t ws_floats = 0, int* counters = nullptr,
                          __half* out16 = nullptr, int hl16 = 0);

int pb_attn_dec1_splits(int n_kv, int max_len, int sm_count);
bool pb_attn_dec_fast_ok(int n_heads, int n_kv, int hd, int max_len);
bool pb_qkv_attn_ok(const pb_qmat* w, int n_heads, int n_kv, int hd, int max_len);
int pb_launch_qkv_attn(pb_ctx* ctx, const pb_qmat* w, const float* x, float* qkv_out, const pb_mv_epi& e, int n_heads,
                       int n_kv, float* out);
int pb_launch_attn_dec_fast(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                            int n_heads, int n_kv, int hd, float* out, int max_len);
size_t pb_attn_dec1_ws_doubles(int n_heads, int n_kv, int hd, int nsplit);
bool pb_attn_dec1_ok(int n_heads, int n_kv, int hd);
int pb_launch_attn_dec1(pb_ctx* ctx, const float* q, const float* kc, const float* vc, const int* pos_dev,
                        int n_heads, int n_kv, int hd, float* out, int max_len, int nsplit, double* ws,
                        unsigned int* counters);

int pb_launch_attn_prefill(pb_ctx* ctx, const float* q, int q_stride, const float* kc, const float* vc, int seq,
                               int start_pos, int n_heads, int n_kv, int hd, float* out, int nseq, pb_seq_geo geo, int terms = 1,
                               const __half* khl = nullptr, const __half* vhl = nullptr, int64_t hl_seq_stride = 0,
                               __half* out16 = nullptr);
bool pb_attn_decode_ok(int n_heads, int n_kv, int hd, int max_len);
bool pb_attn_decode_group_ok(int n_heads, int n_kv, int hd, int max_len);
__global__ void k_rope_kv(float* __restrict__ q, int q_stride, const float* __restrict__ k, int k_stride,
                          const float* __restrict__ v, int v_stride, int n_heads, int n_kv, int hd,
                          const double2* __restrict__ tab, int start_pos, const int* __restrict__ pos_dev,
                          float* __restrict__ kc, float* __restrict__ vc, int max_len, int rows_per_seq,
                          int64_t cache_seq_stride, int* err, int rows, int rows_per_cta, __half* __restrict__ khl,
                          __half* __restrict__ vhl, int64_t hl_seq_stride);
__global__ void k_glu(const float* __restrict__ g, int g_stride, const float* __restrict__ u, int u_stride, int F,
                      int mode, int interleave4, float* __restrict__ out);
__global__ void k_embed(int type, const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc,
                        const float* __restrict__ f32tiles, int V, int dim, const int* __restrict__ toks,
                        const unsigned long long* __restrict__ key_dev, int* __restrict__ tok_out,
                        unsigned long long* __restrict__ key_reset, float* __restrict__ x, int* err);
__global__ void k_step_end(unsigned long long* __restrict__ key, int* __restrict__ tok_dev, int* __restrict__ pos_dev,
                           int* __restrict__ hist, int hist_len);
__global__ void k_elementwise(int op, const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                              float* __restrict__ out);

struct pb_model {
  pb_ctx* ctx = nullptr;
  pb_model_config c{};
  int kv_dim = 0;
  // streaming weights
  pb_qmat* emb = nullptr;                 // Q4_0 / Q8_0 tiles [V][dim]
  pb_qmat* head = nullptr;                // untied output.weight tiles [V][dim] (nullptr: the head is emb)
  std::vector<pb_qmat*> qkv, wo, gu, w2;  // per layer
  // llama.js weights
  float* emb_f32 = nullptr;               // tiles [V/32][dim][32]
  pb_qmat emb_f32_view;                   // head view of emb_f32
  // a streaming model's dequantized tables (a GGUF embedding or output.weight
  // of a type kept as f32, e.g. Q6_K, F16): emb_f32 above, and an untied head
  float* head_f32 = nullptr;              // tiles [V/32][dim][32]
  pb_qmat head_f32_view;
  // the quantized head table in the matvec (row) layout, for the fast
  // kernel's coalesced loads; built on first use, dropped when the table changes
  pb_qmat* head_rows = nullptr;
  std::vector<float*> q8s;                // scales per (layer, which 1..7)
  std::vector<int8_t*> q8q;
  // norms and cache
  float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr;
  float *kc = nullptr, *vc = nullptr;
  double2* rope_tab = nullptr;
  // one-sequence decode attention split over positions: per-split partials
  // and the per-kv-head arrival counters (zero between launches)
  int attn_splits = 0;
  double* attn_ws = nullptr;
  unsigned int* attn_cnt = nullptr;
  double rope_scaling[4] = {0, 0, 0, 0};  // factor, low, high, original context (factor 0: off)
  // activations (sized for max_m rows)
  int max_m = 0;
  float *x = nullptr, *xn = nullptr, *qkvo = nullptr, *att = nullptr, *guo = nullptr, *hb = nullptr, *proj = nullptr,
        *logits = nullptr;
  int* toks = nullptr;
  int* tok_dev = nullptr;  // [0] token, [1] position
  int* hist = nullptr;     // greedy tokens by position
  unsigned long long* key = nullptr;
  // decode graph
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // the sampling decode step (pb_model_generate_sampled): its own graph, the
  // draw counter and the candidate keys on the device
  cudaGraph_t sgraph = nullptr;
  cudaGraphExec_t sexec = nullptr;
  int s_topk = 0;
  double s_temp = 0.0;
  uint64_t s_seed = 0;
  uint64_t* samp_ctr = nullptr;
  uint64_t* samp_cand = nullptr;
  int* samp_tok = nullptr;
  double* exit_prob = nullptr;
  // early exit (llama-streaming.js:202-203, :746-789) and layer-limited
  // decode steps (forward(..., {maxLayers}), the speculative draft)
  double exit_threshold = 0.0;
  int exit_interval = 4;
  int layers_used = 0, last_exit_layer = -1, early_exits = 0;
  std::vector<cudaGraph_t> lgraph;  // decode steps over the first L layers, index L
  std::vector<cudaGraphExec_t> lexec;
  int launches_per_step = 0;
  int graph_mode = -1;  // graph_key of the context when the recorded graphs were made
  float* h_logits_pinned = nullptr;
  int* h_io_pinned = nullptr;
};

static size_t kv_floats(const pb_model* m) { return (size_t)m->c.n_layers * m->c.seq_len * m->kv_dim; }
static float* kcache(pb_model* m, int l) { return m->kc + (size_t)l * m->c.seq_len * m->kv_dim; }
static float* vcache(pb_model* m, int l) { return m->vc + (size_t)l * m->c.seq_len * m->kv_dim; }

// matrix shape (rows = outputs, cols = inputs) of tensor `which` (1..7)
static void mshape(const pb_model_config& c, int which, int* rows, int* cols) {
  int kv = c.n_kv_heads * c.head_dim;
  switch (which) {
    case 1: *rows = c.dim; *cols = c.dim; break;
    case 2: case 3: *rows = kv; *cols = c.dim; break;
    case 4: *rows = c.dim; *cols = c.dim; break;
    case 5: case 7: *rows = c.hidden_dim; *cols = c.dim; break;
    default: *rows = c.dim; *cols = c.hidden_dim; break;
  }
}

static void free_graph(pb_model* m);

static int ensure_act(pb_model* m, int M) {
  if (M <= m->max_m) return PB_OK;
  pb_ctx* ctx = m->ctx;
  PB_TRY(pb_wait(ctx));
  free_graph(m);  // a captured graph holds the old buffer addresses
  cudaFree(m->x); cudaFree(m->xn); cudaFree(m->qkvo); cudaFree(m->att); cudaFree(m->guo); cudaFree(m->hb);
  cudaFree(m->proj); cudaFree(m->toks);
  const pb_model_config& c = m->c;
  size_t qkvw = (size_t)c.dim + 2 * m->kv_dim;
  PB_TRY_CUDA(ctx, cudaMalloc(&m->x, (size_t)M * c.dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->xn, (size_t)M * c.dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->qkvo, (size_t)M * qkvw * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->att, (size_t)M * c.dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->guo, (size_t)M * 2 * c.hidden_dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->hb, (size_t)M * c.hidden_dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->proj, (size_t)M * c.dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&m->toks, (size_t)M * 4));
  m->max_m = M;
  return PB_OK;
}

static void free_graph(pb_model* m) {
  if (m->exec) cudaGraphExecDestroy(m->exec);
  if (m->graph) cudaGraphDestroy(m->graph);
  if (m->sexec) cudaGraphExecDestroy(m->sexec);
  if (m->sgraph) cudaGraphDestroy(m->sgraph);
  m->exec = nullptr;
  m->graph = nullptr;
  m->sexec = nullptr;
  m->sgraph = nullptr;
  for (auto& e : m->lexec)
    if (e) cudaGraphExecDestroy(e);
  for (auto& g : m->lgraph)
    if (g) cudaGraphDestroy(g);
  m->lexec.clear();
  m->lgraph.clear();
}

extern "C" int pb_model_free(pb_model* m) {
  if (!m) return PB_OK;
  pb_ctx* ctx = m->ctx;
  if (ctx) pb_wait(ctx);
  free_graph(m);
  cudaFree(m->samp_ctr);
  cudaFree(m->samp_cand);
  cudaFree(m->samp_tok);
  cudaFree(m->exit_prob);
  pb_qmat_free(nullptr, m->emb);
  pb_qmat_free(nullptr, m->head);
  pb_qmat_free(nullptr, m->head_rows);
  for (auto* p : m->qkv) pb_qmat_free(nullptr, p);
  for (auto* p : m->wo) pb_qmat_free(nullptr, p);
  for (auto* p : m->gu) pb_qmat_free(nullptr, p);
  for (auto* p : m->w2) pb_qmat_free(nullptr, p);
  for (auto* p : m->q8s) cudaFree(p);
  for (auto* p : m->q8q) cudaFree(p);
  cudaFree(m->emb_f32);
  cudaFree(m->head_f32);
  cudaFree(m->rms_att); cudaFree(m->rms_ffn); cudaFree(m->rms_final);
  cudaFree(m->kc); cudaFree(m->vc); cudaFree(m->rope_tab);
  cudaFree(m->attn_ws); cudaFree(m->attn_cnt);
  cudaFree(m->x); cudaFree(m->xn); cudaFree(m->qkvo); cudaFree(m->att); cudaFree(m->guo); cudaFree(m->hb);
  cudaFree(m->proj); cudaFree(m->logits); cudaFree(m->toks); cudaFree(m->tok_dev); cudaFree(m->hist);
  cudaFree(m->key);
  if (m->h_logits_pinned) cudaFreeHost(m->h_logits_pinned);
  if (m->h_io_pinned) cudaFreeHost(m->h_io_pinned);
  delete m;
  return PB_OK;
}

__global__ void k_fill(float* p, int64_t n, float v) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

// An f32 table [V][dim] stored as tiles [V/32][dim][32] (lanes = rows), with
// the head view the head kernels take.
static int alloc_f32_table(pb_model* m, float** tab, pb_qmat* view) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  const size_t ntile = (size_t)((c.vocab + 31) / 32) * 32;
  if (cudaMalloc(tab, ntile * c.dim * 4) != cudaSuccess) return pb_set_error(ctx, PB_ERR_OOM, "f32 table");
  cudaMemsetAsync(*tab, 0, ntile * c.dim * 4, ctx->stream);
  *view = pb_qmat();
  view->type = PB_TYPE_F32;
  view->N = c.vocab;
  view->K = c.dim;
  view->N_pad = (int)ntile;
  view->nb = c.dim / 32;
  view->qs = (uint8_t*)*tab;
  return PB_OK;
}

extern "C" int pb_model_create(pb_ctx* ctx, const pb_model_config* cfg, pb_model** out) {
  if (!ctx || !cfg || !out) return PB_ERR_ARG;
  *out = nullptr;
  const pb_model_config& c = *cfg;
  if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
      c.vocab <= 0 || c.seq_len <= 0 || c.n_heads % c.n_kv_heads || c.n_heads * c.head_dim != c.dim ||
      (c.head_dim & 1) || c.dim % 32 || c.hidden_dim % 32 || (c.n_kv_heads * c.head_dim) % 32)
    return pb_set_error(ctx, PB_ERR_ARG, "invalid model config");
  if (c.kind != PB_MODEL_STREAMING_Q4 && c.kind != PB_MODEL_LLAMA_Q8A)
    return pb_set_error(ctx, PB_ERR_ARG, "unknown model kind %d", c.kind);
  if (c.kind == PB_MODEL_STREAMING_Q4 && c.emb_type != PB_TYPE_Q4_0 && c.emb_type != PB_TYPE_Q8_0 &&
      c.emb_type != PB_TYPE_F32)
    return pb_set_error(ctx, PB_ERR_ARG, "streaming models take a Q4_0, Q8_0 or f32 (dequantized) embedding");
  if (c.kind == PB_MODEL_LLAMA_Q8A && c.emb_type != PB_TYPE_F32)
    return pb_set_error(ctx, PB_ERR_ARG, "llama.js models take an f32 embedding");
  pb_model* m = new pb_model();
  m->ctx = ctx;
  m->c = c;
  m->kv_dim = c.n_kv_heads * c.head_dim;
  int rc = PB_OK;
  auto fail = [&](int code) { pb_model_free(m); return code; };
  const int L = c.n_layers;
  if (c.kind == PB_MODEL_STREAMING_Q4) {
    if (c.emb_type == PB_TYPE_F32) {
      if ((rc = alloc_f32_table(m, &m->emb_f32, &m->emb_f32_view))) return fail(rc);
    } else {
      rc = pb_qmat_alloc(ctx, c.emb_type, PB_LAYOUT_TILED8, c.vocab, c.dim, &m->emb);
      if (rc) return fail(rc);
    }
    m->qkv.assign(L, nullptr); m->wo.assign(L, nullptr); m->gu.assign(L, nullptr); m->w2.assign(L, nullptr);
    for (int l = 0; l < L; ++l) {
      if ((rc = pb_qmat_alloc(ctx, PB_TYPE_Q4_0, PB_LAYOUT_ROWS, c.dim + 2 * m->kv_dim, c.dim, &m->qkv[l]))) return fail(rc);
      if ((rc = pb_qmat_alloc(ctx, PB_TYPE_Q4_0, PB_LAYOUT_ROWS, c.dim, c.dim, &m->wo[l]))) return fail(rc);
      if ((rc = pb_qmat_alloc(ctx, PB_TYPE_Q4_0, PB_LAYOUT_ROWS, 2 * c.hidden_dim, c.dim, &m->gu[l]))) return fail(rc);
      if ((rc = pb_qmat_alloc(ctx, PB_TYPE_Q4_0, PB_LAYOUT_ROWS, c.dim, c.hidden_dim, &m->w2[l]))) return fail(rc);
    }
  } else {
    if ((rc = alloc_f32_table(m, &m->emb_f32, &m->emb_f32_view))) return fail(rc);
    m->q8s.assign((size_t)L * 7, nullptr);
    m->q8q.assign((size_t)L * 7, nullptr);
    for (int l = 0; l < L; ++l)
      for (int w = 1; w <= 7; ++w) {
        int r, k;
        mshape(c, w, &r, &k);
        int64_t n = (int64_t)r * k, nblk = (n + 31) / 32;
        if (cudaMalloc(&m->q8s[l * 7 + w - 1], nblk * 4) != cudaSuccess ||
            cudaMalloc(&m->q8q[l * 7 + w - 1], nblk * 32) != cudaSuccess)
          return fail(pb_set_error(ctx, PB_ERR_OOM, "Q8 weights"));
      }
  }
  size_t nd = (size_t)L * c.dim;
  if (cudaMalloc(&m->rms_att, nd * 4) || cudaMalloc(&m->rms_ffn, nd * 4) || cudaMalloc(&m->rms_final, c.dim * 4) ||
      cudaMalloc(&m->kc, kv_floats(m) * 4) || cudaMalloc(&m->vc, kv_floats(m) * 4) ||
      cudaMalloc(&m->logits, (size_t)c.vocab * 4) || cudaMalloc(&m->tok_dev, 16) ||
      cudaMalloc(&m->hist, (size_t)(c.seq_len + 1) * 4) || cudaMalloc(&m->key, 16) ||
      cudaMalloc(&m->rope_tab, (size_t)c.seq_len * (c.head_dim / 2) * sizeof(double2)))
    return fail(pb_set_error(ctx, PB_ERR_OOM, "model buffers"));
  k_fill<<<pb_cdiv(nd, 256), 256, 0, ctx->stream>>>(m->rms_att, nd, 1.0f);
  k_fill<<<pb_cdiv(nd, 256), 256, 0, ctx->stream>>>(m->rms_ffn, nd, 1.0f);
  k_fill<<<pb_cdiv(c.dim, 256), 256, 0, ctx->stream>>>(m->rms_final, c.dim, 1.0f);
  cudaMemsetAsync(m->kc, 0, kv_floats(m) * 4, ctx->stream);
  cudaMemsetAsync(m->vc, 0, kv_floats(m) * 4, ctx->stream);
  cudaMemsetAsync(m->key, 0, 16, ctx->stream);
  cudaMemsetAsync(m->tok_dev, 0, 16, ctx->stream);
  cudaMemsetAsync(m->hist, 0, (size_t)(c.seq_len + 1) * 4, ctx->stream);
  if (pb_attn_dec1_ok(c.n_heads, c.n_kv_heads, c.head_dim)) {
    m->attn_splits = pb_attn_dec1_splits(c.n_kv_heads, c.seq_len, ctx->sm_count);
    // tuning override of the split count (positions per split stay within the kernel's bound)
    if (const char* e = getenv("PB_ATTN_SPLITS")) {
      const int v = atoi(e);
      if (v > 0 && v >= pb_attn_dec1_splits(c.n_kv_heads, c.seq_len, 1)) m->attn_splits = v;
    }
    const size_t wsd = pb_attn_dec1_ws_doubles(c.n_heads, c.n_kv_heads, c.head_dim, m->attn_splits);
    if (cudaMalloc(&m->attn_ws, wsd * 8) != cudaSuccess || cudaMalloc(&m->attn_cnt, (size_t)c.n_kv_heads * 4))
      return fail(pb_set_error(ctx, PB_ERR_OOM, "decode attention workspace"));
    cudaMemsetAsync(m->attn_cnt, 0, (size_t)c.n_kv_heads * 4, ctx->stream);
  }
  // RoPE rotation table built on the host as the reference builds it
  std::vector<double2> tab((size_t)c.seq_len * (c.head_dim / 2));
  pb_rope_table(c.rope_theta, c.head_dim, 0, c.seq_len, tab.data());
  cudaMemcpyAsync(m->rope_tab, tab.data(), tab.size() * sizeof(double2), cudaMemcpyHostToDevice, ctx->stream);
  if (cudaMallocHost(&m->h_logits_pinned, (size_t)c.vocab * 4) != cudaSuccess ||
      cudaMallocHost(&m->h_io_pinned, 64) != cudaSuccess)
    return fail(pb_set_error(ctx, PB_ERR_OOM, "pinned buffers"));
  if ((rc = ensure_act(m, 1))) return fail(rc);
  if ((rc = pb_wait(ctx))) return fail(rc);
  *out = m;
  return PB_OK;
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------

// Row offset of tensor `which` inside its fused matrix.
static pb_qmat* fused_target(pb_model* m, int l, int which, int* row_off, int* interleave4) {
  const pb_model_config& c = m->c;
  *interleave4 = 0;
  switch (which) {
    case 1: *row_off = 0; return m->qkv[l];
    case 2: *row_off = c.dim; return m->qkv[l];
    case 3: *row_off = c.dim + m->kv_dim; return m->qkv[l];
    case 4: *row_off = 0; return m->wo[l];
    case 5: *row_off = 0; *interleave4 = 1; return m->gu[l];
    case 7: *row_off = 4; *interleave4 = 1; return m->gu[l];
    default: *row_off = 0; return m->w2[l];
  }
}

// GGUF rows -> the device layout at a row offset of an existing matrix
// interleave4: GGUF row i goes to tile row 8*(i/4) + i%4 + row_off, so an
// 8-row tile holds gate rows 4i..4i+3 (row_off 0) and up rows 4i..4i+3
// (row_off 4) and the gate|up matvec can finish SwiGLU in its epilogue.
__global__ void k_pack_rows(const uint8_t* __restrict__ src, int rows, int row_off, int interleave4, int nb, int type,
                            int layout, uint8_t* __restrict__ qs, uint16_t* __restrict__ d, int unpack) {
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (int64_t)rows * nb) return;
  int i = (int)(t / nb), b = (int)(t % nb);
  int n = interleave4 ? 8 * (i >> 2) + (i & 3) + row_off : i + row_off;
  int bb = type == PB_TYPE_Q4_0 ? 18 : 34, pl = type == PB_TYPE_Q4_0 ? 16 : 32;
  uint8_t* g = (uint8_t*)src + t * bb;
  int64_t slot = pb_slot(layout, n, b, nb);
  if (!unpack) {
    d[slot] = (uint16_t)(g[0] | (g[1] << 8));
    for (int i = 0; i < pl; ++i) qs[slot * pl + i] = g[2 + i];
  } else {
    g[0] = (uint8_t)(d[slot] & 0xff);
    g[1] = (uint8_t)(d[slot] >> 8);
    for (int i = 0; i < pl; ++i) g[2 + i] = qs[slot * pl + i];
  }
}

// row-major f32 [V][dim] <-> tiles [V/32][dim][32]
__global__ void k_tile_f32(const float* __restrict__ src, int V, int dim, float* __restrict__ tiles, int untile) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)V * dim) return;
  int v = (int)(i / dim), d = (int)(i % dim);
  size_t t = ((size_t)(v >> 5) * dim + d) * 32 + (v & 31);
  if (!untile) tiles[t] = src[i];
  else ((float*)src)[i] = tiles[t];
}

static int pack_rows(pb_model* m, pb_qmat* dst, const void* gguf_dev, int rows, int row_off, int interleave4) {
  pb_ctx* ctx = m->ctx;
  dst->mma_ok = false;  // the tensor-core copy no longer mirrors the matrix
  int64_t tot = (int64_t)rows * dst->nb;
  k_pack_rows<<<pb_cdiv(tot, 256), 256, 0, ctx->stream>>>((const uint8_t*)gguf_dev, rows, row_off, interleave4,
                                                          dst->nb, dst->type, dst->layout, dst->qs, dst->d, 0);
  PB_LAUNCHED(ctx, "k_pack_rows");
  return PB_OK;
}

extern "C" int pb_model_init_synthetic(pb_model* m, uint64_t seed, double stdev) {
  if (!m) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  free_graph(m);
  pb_qmat_free(ctx, m->head_rows);
  m->head_rows = nullptr;
  // largest tensor: embedding or an FFN matrix
  int64_t ne = (int64_t)c.vocab * c.dim;
  int64_t nf = (int64_t)c.hidden_dim * c.dim;
  int64_t nmax = ne > nf ? ne : nf;
  float* tmp = nullptr;
  uint8_t* gg = nullptr;
  PB_TRY_CUDA(ctx, cudaMalloc(&tmp, nmax * 4));
  int rc = PB_OK;
  if (cudaMalloc(&gg, nmax / 32 * 34 + 64) != cudaSuccess) {
    cudaFree(tmp);
    return pb_set_error(ctx, PB_ERR_OOM, "synthetic init buffer");
  }
  auto gen = [&](uint64_t tid, int64_t n) { return pb_synth_weights(ctx, tmp, n, seed, tid, stdev); };
  // embedding (tensor id 0)
  if ((rc = gen(0, ne))) goto done;
  if (c.kind == PB_MODEL_STREAMING_Q4 && c.emb_type != PB_TYPE_F32) {
    if ((rc = pb_gguf_quantize(ctx, c.emb_type, tmp, ne, gg))) goto done;
    if ((rc = pack_rows(m, m->emb, gg, c.vocab, 0, 0))) goto done;
  } else {
    k_tile_f32<<<pb_cdiv(ne, 256), 256, 0, ctx->stream>>>(tmp, c.vocab, c.dim, m->emb_f32, 0);
    if ((rc = pb_check_launch(ctx, "k_tile_f32"))) goto done;
  }
  for (int l = 0; l < c.n_layers; ++l)
    for (int w = 1; w <= 7; ++w) {
      int r, k;
      mshape(c, w, &r, &k);
      int64_t n = (int64_t)r * k;
      if ((rc = gen(1 + 7 * (uint64_t)l + (w - 1), n))) goto done;
      if (c.kind == PB_MODEL_STREAMING_Q4) {
        if ((rc = pb_gguf_quantize(ctx, PB_TYPE_Q4_0, tmp, n, gg))) goto done;
        int off, il;
        pb_qmat* dst = fused_target(m, l, w, &off, &il);
        if ((rc = pack_rows(m, dst, gg, r, off, il))) goto done;
      } else {
        if ((rc = pb_quantize_q8a(ctx, tmp, n, m->q8s[l * 7 + w - 1], m->q8q[l * 7 + w - 1]))) goto done;
      }
    }
  rc = pb_wait(ctx);
done:
  cudaStreamSynchronize(ctx->stream);
  cudaFree(tmp);
  cudaFree(gg);
  return rc;
}

// The quantized LM head table: output.weight when the file has one, else the
// tied embedding (llama-streaming.js:616-679, streaming-loader.js
// sharedWeights); nullptr when the head is an f32 table.
static pb_qmat* head_of(const pb_model* m) {
  if (m->head) return m->head;
  return m->head_f32 ? nullptr : m->emb;
}

// The head table and the head kernel's arithmetic: batch_dot order with the
// exact dequant over Q4_0 / Q8_0 tiles (mode 0), batch_dot order over a
// dequantized f32 table (mode 2: what the reference keeps for every other
// GGUF type, streaming-loader.js:324-335, e.g. Q6_K or F16), or llama.js's
// double-precision dot over its f32 embedding (mode 1).
static const pb_qmat* head_table(const pb_model* m, int* mode) {
  if (m->c.kind == PB_MODEL_LLAMA_Q8A) { *mode = 1; return &m->emb_f32_view; }
  if (m->head) { *mode = 0; return m->head; }
  if (m->head_f32) { *mode = 2; return &m->head_f32_view; }
  if (m->emb) { *mode = 0; return m->emb; }
  *mode = 2;
  return &m->emb_f32_view;
}

// Give a streaming model an untied LM head (GGUF output.weight) of `type`
// (Q4_0 / Q8_0 kept quantized, or PB_TYPE_F32 for a dequantized table), set
// afterwards as tensor 11.
extern "C" int pb_model_attach_head(pb_model* m, int type) {
  if (!m) return PB_ERR_ARG;
  if (m->c.kind != PB_MODEL_STREAMING_Q4 || (type != PB_TYPE_Q4_0 && type != PB_TYPE_Q8_0 && type != PB_TYPE_F32))
    return pb_set_error(m->ctx, PB_ERR_ARG, "an untied head needs a streaming model and a Q4_0, Q8_0 or f32 table");
  free_graph(m);
  pb_qmat_free(m->ctx, m->head);
  m->head = nullptr;
  pb_qmat_free(m->ctx, m->head_rows);
  m->head_rows = nullptr;
  cudaFree(m->head_f32);
  m->head_f32 = nullptr;
  if (type == PB_TYPE_F32) return alloc_f32_table(m, &m->head_f32, &m->head_f32_view);
  return pb_qmat_alloc(m->ctx, type, PB_LAYOUT_TILED8, m->c.vocab, m->c.dim, &m->head);
}

static size_t tensor_bytes(const pb_model* m, int which) {
  const pb_model_config& c = m->c;
  if (which == 11) {
    if (m->head_f32) return (size_t)c.vocab * c.dim * 4;
    return m->head ? (size_t)((int64_t)c.vocab * c.dim / 32) * (m->head->type == PB_TYPE_Q4_0 ? 18 : 34) : 0;
  }
  if (which >= 8) return (size_t)c.dim * 4;
  if (which == 0) {
    int64_t ne = (int64_t)c.vocab * c.dim;
    if (c.kind == PB_MODEL_LLAMA_Q8A || c.emb_type == PB_TYPE_F32) return (size_t)ne * 4;
    return (size_t)(ne / 32) * (c.emb_type == PB_TYPE_Q4_0 ? 18 : 34);
  }
  int r, k;
  mshape(c, which, &r, &k);
  int64_t n = (int64_t)r * k;
  if (c.kind == PB_MODEL_STREAMING_Q4) return (size_t)(n / 32) * 18;
  int64_t nb = (n + 31) / 32;
  return (size_t)(nb * 4 + nb * 32);
}

static int model_tensor_io(pb_model* m, int layer, int which, void* host, size_t bytes, int get) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  if (which < 0 || which > 11 || (which >= 1 && which <= 9 && (layer < 0 || layer >= c.n_layers)))
    return pb_set_error(ctx, PB_ERR_ARG, "bad tensor (layer %d, which %d)", layer, which);
  if (which == 11 && !m->head && !m->head_f32)
    return pb_set_error(ctx, PB_ERR_ARG, "the model has no untied head (pb_model_attach_head)");
  size_t need = tensor_bytes(m, which);
  if (bytes != need) return pb_set_error(ctx, PB_ERR_ARG, "tensor %d needs %zu bytes, got %zu", which, need, bytes);
  if (!get) free_graph(m);
  if (!get && (which == 0 || which == 11)) {
    pb_qmat_free(ctx, m->head_rows);
    m->head_rows = nullptr;
  }
  if (which >= 8 && which <= 10) {
    float* p = which == 8 ? m->rms_att + (size_t)layer * c.dim : which == 9 ? m->rms_ffn + (size_t)layer * c.dim
                                                                            : m->rms_final;
    return get ? pb_download(ctx, host, p, bytes) : pb_upload(ctx, p, host, bytes);
  }
  if (c.kind == PB_MODEL_LLAMA_Q8A && which >= 1) {
    int64_t nb = (int64_t)(bytes / 36);
    float* s = m->q8s[layer * 7 + which - 1];
    int8_t* q = m->q8q[layer * 7 + which - 1];
    if (get) {
      PB_TRY(pb_download(ctx, host, s, nb * 4));
      return pb_download(ctx, (char*)host + nb * 4, q, nb * 32);
    }
    PB_TRY(pb_upload(ctx, s, host, nb * 4));
    return pb_upload(ctx, q, (const char*)host + nb * 4, nb * 32);
  }
  PB_TRY(pb_ensure_scratch(ctx, bytes));
  float* f32_tab = which == 11 ? m->head_f32 : (which == 0 && (c.kind == PB_MODEL_LLAMA_Q8A || c.emb_type == PB_TYPE_F32))
                                                  ? m->emb_f32 : nullptr;
  if (f32_tab) {  // f32 table, stored as tiles
    int64_t ne = (int64_t)c.vocab * c.dim;
    if (!get) PB_TRY_CUDA(ctx, cudaMemcpyAsync(ctx->scratch, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    k_tile_f32<<<pb_cdiv(ne, 256), 256, 0, ctx->stream>>>((float*)ctx->scratch, c.vocab, c.dim, f32_tab, get);
    PB_LAUNCHED(ctx, "k_tile_f32");
    if (get) PB_TRY_CUDA(ctx, cudaMemcpyAsync(host, ctx->scratch, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return pb_wait(ctx);
  }
  pb_qmat* dst;
  int rows, off = 0, il = 0;
  if (which == 0 || which == 11) {
    dst = which == 0 ? m->emb : m->head;
    rows = c.vocab;
  } else {
    int k;
    mshape(c, which, &rows, &k);
    dst = fused_target(m, layer, which, &off, &il);
  }
  if (!get) {
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(ctx->scratch, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    dst->mma_ok = false;
  }
  int64_t tot = (int64_t)rows * dst->nb;
  k_pack_rows<<<pb_cdiv(tot, 256), 256, 0, ctx->stream>>>((const uint8_t*)ctx->scratch, rows, off, il, dst->nb,
                                                          dst->type, dst->layout, dst->qs, dst->d, get);
  PB_LAUNCHED(ctx, "k_pack_rows");
  if (get) PB_TRY_CUDA(ctx, cudaMemcpyAsync(host, ctx->scratch, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_model_set_tensor(pb_model* m, int layer, int which, const void* host, size_t bytes) {
  if (!m || !host) return PB_ERR_ARG;
  return model_tensor_io(m, layer, which, (void*)host, bytes, 0);
}
extern "C" int pb_model_get_tensor(pb_model* m, int layer, int which, void* host, size_t bytes) {
  if (!m || !host) return PB_ERR_ARG;
  return model_tensor_io(m, layer, which, host, bytes, 1);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

// Rows of k_rope_kv per CTA: one for decode batches (many CTAs for few rows),
// 16 at prefill sizes (458K CTAs of 128 elements per layer otherwise).
static int rope_rows_per_cta(int rows) { return rows >= 4096 ? 16 : 1; }

static int launch_norm(pb_model* m, const float* x, int M, const float* w, float* out, __half* out16 = nullptr,
                       int xc = 0, int hl = 0) {
  pb_launch_rmsnorm(m->ctx->stream, x, M, m->c.dim, w, m->c.eps, out, out16, xc, hl, m->ctx->pdl);
  PB_LAUNCHED(m->ctx, "k_rmsnorm");
  return PB_OK;
}

static int launch_q8a(pb_model* m, int l, int which, const float* A, int M, float* out) {
  int r, k;
  mshape(m->c, which, &r, &k);
  return pb_matmul_q8a(m->ctx, A, M, k, m->q8s[l * 7 + which - 1], m->q8q[l * 7 + which - 1], r, nullptr, out);
}

// Prefetch hint: the payload and scales of w (the payload capped at cap
// bytes) in slots i, i + 1 of the epilogue's L2 list.
static void l2_hint(pb_mv_epi* e, int i, const pb_qmat* w, size_t cap = ~(size_t)0) {
  if (!w) return;
  const size_t nblk = (size_t)w->N_pad * w->nb;
  const size_t qb = nblk * (w->type == PB_TYPE_Q8_0 ? 32 : 16);
  e->l2_next[i] = w->qs;
  e->l2_next_bytes[i] = qb < cap ? qb : cap;
  e->l2_next[i + 1] = w->d;
  e->l2_next_bytes[i + 1] = (nblk * 2) & ~(size_t)15;
}

// Decode attention of the one sequence at *pos_dev (llama-streaming.js
// :543-573): the position-split kernel when the shape fits it, else one CTA
// per query head.
static int launch_attn_decode1(pb_model* m, int l, const float* q, const int* pos_dev) {
  const pb_model_config& c = m->c;
  // fast mode: the f32, cluster-merged form
  if (m->ctx->matvec_mode == PB_MATVEC_FAST && pb_attn_dec_fast_ok(c.n_heads, c.n_kv_heads, c.head_dim, c.seq_len))
    return pb_launch_attn_dec_fast(m->ctx, q, kcache(m, l), vcache(m, l), pos_dev, c.n_heads, c.n_kv_heads,
                                   c.head_dim, m->att, c.seq_len);
  if (m->attn_ws)
    return pb_launch_attn_dec1(m->ctx, q, kcache(m, l), vcache(m, l), pos_dev, c.n_heads, c.n_kv_heads, c.head_dim,
                               m->att, c.seq_len, m->attn_splits, m->attn_ws, m->attn_cnt);
  return pb_launch_attn_decode(m->ctx, q, kcache(m, l), vcache(m, l), pos_dev, c.n_heads, c.n_kv_heads, c.head_dim,
                               m->att, c.seq_len, 1, pb_seq_geo());
}

// Decode layer (M == 1) of the streaming model: four fused matvecs and the
// attention (llama-streaming.js:505-606).
static int run_layer_decode_q4(pb_model* m, int l) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  const int dim = c.dim, kv = m->kv_dim;
  const int* pos_dev = m->tok_dev + 1;
  const bool last = l + 1 == c.n_layers;
  // Each matvec also prefetches into L2 the weights of the matvecs after it,
  // so HBM keeps streaming while the attention and the chains run.
  pb_mv_epi e;
  // RMSNorm -> [wq; wk; wv] -> RoPE on q, k; k, v into the cache at pos
  e.kind = PB_EPI_ROPE_KV;
  e.norm_w = m->rms_att + (size_t)l * dim;
  e.eps = c.eps;
  e.rope_tab = m->rope_tab;
  e.pos_dev = pos_dev;
  e.q_rows = dim;
  e.kv_rows = kv;
  e.head_dim = c.head_dim;
  e.max_len = c.seq_len;
  e.kc = kcache(m, l);
  e.vc = vcache(m, l);
  l2_hint(&e, 0, m->wo[l]);
  l2_hint(&e, 2, m->w2[l]);
  if (ctx->matvec_mode == PB_MATVEC_FAST && ctx->fuse_attn && pb_fast_uses_mvf(ctx, m->qkv[l]) &&
      pb_qkv_attn_ok(m->qkv[l], c.n_heads, c.n_kv_heads, c.head_dim, c.seq_len)) {
    // one kernel: the 8 CTAs attending for a kv head compute its projection rows first
    PB_TRY(pb_launch_qkv_attn(ctx, m->qkv[l], m->x, m->qkvo, e, c.n_heads, c.n_kv_heads, m->att));
  } else {
    PB_TRY(pb_launch_matvec(ctx, m->qkv[l], m->x, m->qkvo, 0, dim + 2 * kv, &e));
    PB_TRY(launch_attn_decode1(m, l, m->qkvo, pos_dev));
  }
  // wo with the residual add
  pb_mv_epi r;
  r.kind = PB_EPI_RESIDUAL;
  r.residual = m->x;
  l2_hint(&r, 0, m->gu[l]);
  PB_TRY(pb_launch_matvec(ctx, m->wo[l], m->att, m->x, 0, dim, &r));
  // RMSNorm -> [w1 | w3] interleaved -> SwiGLU
  pb_mv_epi g;
  g.kind = PB_EPI_SWIGLU4;
  g.norm_w = m->rms_ffn + (size_t)l * dim;
  g.eps = c.eps;
  g.h_out = m->hb;
  if (!last) {
    l2_hint(&g, 0, m->qkv[l + 1]);
    l2_hint(&g, 2, m->wo[l + 1]);
  }
  PB_TRY(pb_launch_matvec(ctx, m->gu[l], m->x, nullptr, 0, 2 * c.hidden_dim, &g));
  // w2 with the residual add
  pb_mv_epi r2 = r;
  r2.l2_next[0] = r2.l2_next[1] = nullptr;
  r2.l2_next_bytes[0] = r2.l2_next_bytes[1] = 0;
  if (!last) l2_hint(&r2, 0, m->gu[l + 1]);
  else if (head_of(m)) l2_hint(&r2, 0, head_of(m), (size_t)48 << 20);
  PB_TRY(pb_launch_matvec(ctx, m->w2[l], m->hb, m->x, 0, dim, &r2));
  return PB_OK;
}

// One layer for M rows at start_pos (prefill, and every llama.js layer).
static int run_layer(pb_model* m, int l, int M, int start_pos, bool dev_pos) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  if (c.kind == PB_MODEL_STREAMING_Q4 && M == 1 && dev_pos) return run_layer_decode_q4(m, l);
  const int dim = c.dim, F = c.hidden_dim, kv = m->kv_dim;
  const int qkvw = dim + 2 * kv;
  const int* pos_dev = dev_pos ? m->tok_dev + 1 : nullptr;
  PB_TRY(launch_norm(m, m->x, M, m->rms_att + (size_t)l * dim, m->xn));
  float *q, *k, *v;
  int qs_, ks_, vs_;
  if (c.kind == PB_MODEL_STREAMING_Q4) {
    PB_TRY(pb_launch_prefill_q4(ctx, m->qkv[l], m->xn, dim, M, m->qkvo, qkvw));
    q = m->qkvo; k = m->qkvo + dim; v = m->qkvo + dim + kv;
    qs_ = ks_ = vs_ = qkvw;
  } else {
    q = m->qkvo; k = m->qkvo + (size_t)M * dim; v = k + (size_t)M * kv;
    qs_ = dim; ks_ = kv; vs_ = kv;
    PB_TRY(launch_q8a(m, l, 1, m->xn, M, q));
    PB_TRY(launch_q8a(m, l, 2, m->xn, M, k));
    PB_TRY(launch_q8a(m, l, 3, m->xn, M, v));
  }
  {
    int tot = (c.n_heads + c.n_kv_heads) * (c.head_dim / 2) + kv;
    const int rpc = rope_rows_per_cta(M);
    k_rope_kv<<<dim3(pb_cdiv(tot, 128), pb_cdiv(M, rpc)), 128, 0, ctx->stream>>>(
        q, qs_, k, ks_, v, vs_, c.n_heads, c.n_kv_heads, c.head_dim, m->rope_tab, start_pos, pos_dev, kcache(m, l),
        vcache(m, l), c.seq_len, M, 0, ctx->d_err, M, rpc, nullptr, nullptr, 0);
    PB_LAUNCHED(ctx, "k_rope_kv");
  }
  if (M == 1 && pos_dev && (m->attn_ws || pb_attn_decode_ok(c.n_heads, c.n_kv_heads, c.head_dim, c.seq_len)))
    PB_TRY(launch_attn_decode1(m, l, q, pos_dev));
  else
    PB_TRY(pb_launch_attn_cached(ctx, q, qs_, kcache(m, l), vcache(m, l), M, start_pos, pos_dev, c.n_heads,
                                 c.n_kv_heads, c.head_dim, m->att, c.seq_len, 1, pb_seq_geo()));
  // output projection + residual
  if (c.kind == PB_MODEL_STREAMING_Q4) PB_TRY(pb_launch_prefill_q4(ctx, m->wo[l], m->att, dim, M, m->proj, dim));
  else PB_TRY(launch_q8a(m, l, 4, m->att, M, m->proj));
  k_elementwise<<<pb_cdiv((int64_t)M * dim, 256), 256, 0, ctx->stream>>>(0, m->x, m->proj, (int64_t)M * dim, m->x);
  PB_LAUNCHED(ctx, "k_elementwise");
  PB_TRY(launch_norm(m, m->x, M, m->rms_ffn + (size_t)l * dim, m->xn));
  // FFN: SILU then ELEMENT_MUL (llama.js:329-332, llama-streaming.js:478-481)
  const float *g, *u;
  int gs, us, il;
  if (c.kind == PB_MODEL_STREAMING_Q4) {
    PB_TRY(pb_launch_prefill_q4(ctx, m->gu[l], m->xn, dim, M, m->guo, 2 * F));
    g = m->guo; u = m->guo; gs = us = 2 * F; il = 1;  // interleaved [g4 | u4] columns
  } else {
    PB_TRY(launch_q8a(m, l, 5, m->xn, M, m->guo));
    PB_TRY(launch_q8a(m, l, 7, m->xn, M, m->guo + (size_t)M * F));
    g = m->guo; u = m->guo + (size_t)M * F; gs = us = F; il = 0;
  }
  k_glu<<<dim3(pb_cdiv(F, 256), M), 256, 0, ctx->stream>>>(g, gs, u, us, F, 1, il, m->hb);
  PB_LAUNCHED(ctx, "k_glu");
  if (c.kind == PB_MODEL_STREAMING_Q4) PB_TRY(pb_launch_prefill_q4(ctx, m->w2[l], m->hb, F, M, m->proj, dim));
  else PB_TRY(launch_q8a(m, l, 6, m->hb, M, m->proj));
  k_elementwise<<<pb_cdiv((int64_t)M * dim, 256), 256, 0, ctx->stream>>>(0, m->x, m->proj, (int64_t)M * dim, m->x);
  PB_LAUNCHED(ctx, "k_elementwise");
  return PB_OK;
}

static int launch_embed(pb_model* m, const int* toks, int M) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  dim3 grid(pb_cdiv(c.dim, 256), M);
  if (m->emb)
    k_embed<<<grid, 256, 0, ctx->stream>>>(c.emb_type, m->emb->qs, m->emb->d, nullptr, c.vocab, c.dim, toks, nullptr,
                                           nullptr, nullptr, m->x, ctx->d_err);
  else
    k_embed<<<grid, 256, 0, ctx->stream>>>(PB_TYPE_F32, nullptr, nullptr, m->emb_f32, c.vocab, c.dim, toks, nullptr,
                                           nullptr, nullptr, m->x, ctx->d_err);
  PB_LAUNCHED(ctx, "k_embed");
  return PB_OK;
}

// The copies the fast mode reads: the layer matrices' tensor-core copies and
// the row-layout copy of the quantized head table (the tiled table serves
// the exact batch_dot kernel and the embedding lookup; its row copy gets a
// tensor-core copy of its own).  Allocates: called before any recording.
static int ensure_head_rows(pb_model* m) {
  pb_ctx* ctx = m->ctx;
  if (ctx->matvec_mode != PB_MATVEC_FAST || m->c.kind != PB_MODEL_STREAMING_Q4) return PB_OK;
  // the layer matrices' tensor-core copies (rebuilt after their weights change)
  for (auto* v : {&m->qkv, &m->wo, &m->gu, &m->w2})
    for (pb_qmat* w : *v)
      if (w && !w->mma_ok) PB_TRY(pb_qmat_build_mma(ctx, w));
  if (m->head_rows) return PB_OK;
  const pb_qmat* t = head_of(m);
  if (!t || (t->type != PB_TYPE_Q4_0 && t->type != PB_TYPE_Q8_0)) return PB_OK;
  const size_t bytes = (size_t)t->N * t->nb * (t->type == PB_TYPE_Q4_0 ? 18 : 34);
  PB_TRY(pb_ensure_scratch(ctx, bytes));
  const int64_t tot = (int64_t)t->N * t->nb;
  k_pack_rows<<<pb_cdiv(tot, 256), 256, 0, ctx->stream>>>((const uint8_t*)ctx->scratch, t->N, 0, 0, t->nb, t->type,
                                                          t->layout, t->qs, t->d, 1);
  PB_LAUNCHED(ctx, "k_pack_rows");
  PB_TRY(pb_qmat_from_device(ctx, t->type, ctx->scratch, t->N, t->K, &m->head_rows));
  return pb_wait(ctx);
}

// Final RMSNorm (fused into the head kernel) and the LM head with the greedy
// argmax (llama-streaming.js:616-642, :899-909; llama.js:340-367).
static int launch_head(pb_model* m, const float* last_x) {
  int mode = 0;
  const pb_qmat* t = head_table(m, &mode);
  if (mode == 0 && m->ctx->matvec_mode == PB_MATVEC_FAST)
    return pb_launch_head_fast(m->ctx, m->head_rows ? m->head_rows : t, last_x, m->rms_final, m->c.eps, m->logits,
                               m->key);
  return pb_launch_head_norm(m->ctx, t, last_x, m->rms_final, m->c.eps, m->logits, m->key, mode);
}

// Enqueue one decode step that reads token and position from m->tok_dev.
static int enqueue_decode_step(pb_model* m, int layers) {
  pb_ctx* ctx = m->ctx;
  PB_TRY(launch_embed(m, m->tok_dev, 1));
  for (int l = 0; l < layers; ++l) PB_TRY(run_layer(m, l, 1, 0, true));
  PB_TRY(launch_head(m, m->x));
  k_step_end<<<1, 32, 0, ctx->stream>>>(m->key, m->tok_dev, m->tok_dev + 1, m->hist, m->c.seq_len + 1);
  PB_LAUNCHED(ctx, "k_step_end");
  return PB_OK;
}

static int ensure_sample_buffers(pb_model* m) {
  if (m->samp_ctr) return PB_OK;
  PB_TRY_CUDA(m->ctx, cudaMalloc(&m->samp_ctr, 8));
  PB_TRY_CUDA(m->ctx, cudaMalloc(&m->samp_cand, pb_sample_cand_count(m->c.vocab, 256) * 8));
  PB_TRY_CUDA(m->ctx, cudaMalloc(&m->samp_tok, 16));
  PB_TRY_CUDA(m->ctx, cudaMalloc(&m->exit_prob, 16));
  return PB_OK;
}

// Recorded graphs hold the kernels of the context's matvec mode and fusion
// setting at recording time; a change drops them so the next step records
// again.
static int graph_key(const pb_ctx* ctx) { return ctx->matvec_mode | (ctx->fuse_attn ? 2 : 0); }
static void check_graph_mode(pb_model* m) {
  if (m->graph_mode != graph_key(m->ctx)) {
    free_graph(m);
    m->graph_mode = graph_key(m->ctx);
  }
}

static int ensure_graph(pb_model* m) {
  check_graph_mode(m);
  if (m->exec) return PB_OK;
  PB_TRY(ensure_head_rows(m));
  pb_ctx* ctx = m->ctx;
  PB_TRY(ensure_act(m, 1));
  int64_t before = ctx->launches;
  PB_TRY_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_decode_step(m, m->c.n_layers);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (rc != PB_OK) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "decode graph capture");
  m->launches_per_step = (int)(ctx->launches - before);
  e = cudaGraphInstantiate(&m->exec, g, 0);
  if (e != cudaSuccess) { cudaGraphDestroy(g); return pb_cuda_error(ctx, e, "decode graph instantiate"); }
  m->graph = g;
  return PB_OK;
}

extern "C" int pb_model_forward_ex(pb_model* m, const int* tokens, int n, int start_pos, int max_layers,
                                   float* logits_host, int* layers_used) {
  if (!m || !tokens || n <= 0) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  if (start_pos < 0 || start_pos + n > c.seq_len)
    return pb_set_error(ctx, PB_ERR_ARG, "positions [%d, %d) exceed the cache length %d", start_pos, start_pos + n, c.seq_len);
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= c.vocab) return pb_set_error(ctx, PB_ERR_ARG, "token %d out of range", tokens[i]);
  if (n == 1) {  // the graph-captured decode step
    int next;
    return pb_model_decode_ex(m, tokens[0], start_pos, max_layers, &next, logits_host, layers_used);
  }
  PB_TRY(ensure_head_rows(m));
  const int L = max_layers <= 0 || max_layers > c.n_layers ? c.n_layers : max_layers;
  PB_TRY(ensure_act(m, n));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->toks, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
  PB_TRY(launch_embed(m, m->toks, n));
  for (int l = 0; l < L; ++l) PB_TRY(run_layer(m, l, n, start_pos, false));
  m->layers_used = L;
  m->last_exit_layer = L - 1;
  if (layers_used) *layers_used = L;
  PB_TRY(launch_head(m, m->x + (size_t)(n - 1) * c.dim));
  // leave the greedy token in the token slot, as a decode step would
  m->h_io_pinned[0] = 0;
  k_step_end<<<1, 32, 0, ctx->stream>>>(m->key, m->tok_dev, m->tok_dev + 1, nullptr, 0);
  PB_LAUNCHED(ctx, "k_step_end");
  if (logits_host) PB_TRY_CUDA(ctx, cudaMemcpyAsync(logits_host, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, ctx->stream));
  PB_TRY(pb_wait(ctx));
  // position after the prompt
  int io[2] = {0, start_pos + n};
  PB_TRY_CUDA(ctx, cudaMemcpy(io, m->tok_dev, 4, cudaMemcpyDeviceToHost));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->tok_dev + 1, &io[1], 4, cudaMemcpyHostToDevice, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_model_forward(pb_model* m, const int* tokens, int n, int start_pos, float* logits_host) {
  return pb_model_forward_ex(m, tokens, n, start_pos, 0, logits_host, nullptr);
}

extern "C" int pb_model_set_early_exit(pb_model* m, double threshold, int interval) {
  if (!m) return PB_ERR_ARG;
  m->exit_threshold = threshold > 0.0 ? threshold : 0.0;  // options.earlyExitThreshold || 0
  m->exit_interval = interval > 0 ? interval : 4;          // options.earlyExitInterval || 4
  return PB_OK;
}

extern "C" int pb_model_exit_stats(const pb_model* m, int* layers_used, int* last_exit_layer, int* early_exits) {
  if (!m) return PB_ERR_ARG;
  if (layers_used) *layers_used = m->layers_used;
  if (last_exit_layer) *last_exit_layer = m->last_exit_layer;
  if (early_exits) *early_exits = m->early_exits;
  return PB_OK;
}

// sample(logits, topK, temperature) over the logits of the model's last
// forward, on the device; the draw is pb_sample_uniform(seed, counter).
extern "C" int pb_model_sample(pb_model* m, int top_k, double temperature, uint64_t seed, uint64_t counter,
                               int* token_host) {
  if (!m || !token_host) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  PB_TRY(ensure_sample_buffers(m));
  PB_TRY(pb_launch_sample(ctx, m->logits, m->c.vocab, top_k, temperature, seed, counter, nullptr, m->samp_cand,
                          m->samp_tok, nullptr, nullptr, 0, nullptr));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->h_io_pinned + 3, m->samp_tok, 4, cudaMemcpyDeviceToHost, ctx->stream));
  PB_TRY(pb_wait(ctx));
  *token_host = m->h_io_pinned[3];
  return PB_OK;
}

// Decode step graph over the first L < n_layers layers (the draft of
// self-speculative decoding, forward(..., {maxLayers: L})).
static int ensure_graph_layers(pb_model* m, int L) {
  check_graph_mode(m);
  PB_TRY(ensure_head_rows(m));
  if ((int)m->lexec.size() < m->c.n_layers) {
    m->lexec.resize(m->c.n_layers, nullptr);
    m->lgraph.resize(m->c.n_layers, nullptr);
  }
  if (m->lexec[L]) return PB_OK;
  pb_ctx* ctx = m->ctx;
  PB_TRY(ensure_act(m, 1));
  if ((int)m->lexec.size() < m->c.n_layers) {  // ensure_act may have dropped every graph
    m->lexec.resize(m->c.n_layers, nullptr);
    m->lgraph.resize(m->c.n_layers, nullptr);
  }
  PB_TRY_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_decode_step(m, L);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (rc != PB_OK) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "draft graph capture");
  e = cudaGraphInstantiate(&m->lexec[L], g, 0);
  if (e != cudaSuccess) { cudaGraphDestroy(g); return pb_cuda_error(ctx, e, "draft graph instantiate"); }
  m->lgraph[L] = g;
  return PB_OK;
}

// One decode step with the early-exit check (llama-streaming.js:767-803):
// after every `exit_interval` layers (not after the last) the final norm and
// head run on the hidden state and k_exit_prob scores the top-8 confidence;
// at or above the threshold those logits are the step's.  The host reads the
// confidence at each check, so this step runs without a recorded graph.
static int decode_early_exit(pb_model* m, int L) {
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  PB_TRY(ensure_act(m, 1));
  PB_TRY(ensure_sample_buffers(m));
  PB_TRY(launch_embed(m, m->tok_dev, 1));
  int used = 0;
  bool exited = false;
  double* prob_host = reinterpret_cast<double*>(m->h_io_pinned + 6);
  for (int l = 0; l < L && !exited; ++l) {
    PB_TRY(run_layer(m, l, 1, 0, true));
    ++used;
    if (l < c.n_layers - 1 && (l + 1) % m->exit_interval == 0) {
      PB_TRY_CUDA(ctx, cudaMemsetAsync(m->key, 0, 8, ctx->stream));
      PB_TRY(launch_head(m, m->x));
      PB_TRY(pb_launch_exit_prob(ctx, m->logits, c.vocab, m->samp_cand, m->exit_prob));
      PB_TRY_CUDA(ctx, cudaMemcpyAsync(prob_host, m->exit_prob, 8, cudaMemcpyDeviceToHost, ctx->stream));
      PB_TRY(pb_wait(ctx));
      if (*prob_host >= m->exit_threshold) {
        exited = true;
        ++m->early_exits;
        m->last_exit_layer = l;
      }
    }
  }
  if (!exited) {
    PB_TRY_CUDA(ctx, cudaMemsetAsync(m->key, 0, 8, ctx->stream));
    PB_TRY(launch_head(m, m->x));
    m->last_exit_layer = used - 1;
  }
  m->layers_used = used;
  k_step_end<<<1, 32, 0, ctx->stream>>>(m->key, m->tok_dev, m->tok_dev + 1, m->hist, c.seq_len + 1);
  PB_LAUNCHED(ctx, "k_step_end");
  return PB_OK;
}

extern "C" int pb_model_decode_ex(pb_model* m, int token, int pos, int max_layers, int* next_host, float* logits_host,
                                  int* layers_used) {
  if (!m) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  if (pos < 0 || pos >= m->c.seq_len) return pb_set_error(ctx, PB_ERR_ARG, "position %d outside the cache", pos);
  if (token < 0 || token >= m->c.vocab) return pb_set_error(ctx, PB_ERR_ARG, "token %d out of range", token);
  const int n = m->c.n_layers;
  const int L = max_layers <= 0 || max_layers > n ? n : max_layers;  // Math.min(maxLayers, nLayers)
  if (m->exit_threshold <= 0.0) {
    if (L == n) PB_TRY(ensure_graph(m));
    else PB_TRY(ensure_graph_layers(m, L));
  }
  m->h_io_pinned[0] = token;
  m->h_io_pinned[1] = pos;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->tok_dev, m->h_io_pinned, 8, cudaMemcpyHostToDevice, ctx->stream));
  if (m->exit_threshold > 0.0) {
    PB_TRY(decode_early_exit(m, L));
  } else {
    PB_TRY_CUDA(ctx, cudaGraphLaunch(L == n ? m->exec : m->lexec[L], ctx->stream));
    m->layers_used = L;
    m->last_exit_layer = L - 1;
  }
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->h_io_pinned + 2, m->tok_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (logits_host)
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(logits_host, m->logits, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToHost, ctx->stream));
  PB_TRY(pb_wait(ctx));
  if (next_host) *next_host = m->h_io_pinned[2];
  if (layers_used) *layers_used = m->layers_used;
  return PB_OK;
}

extern "C" int pb_model_decode(pb_model* m, int token, int pos, int* next_host, float* logits_host) {
  return pb_model_decode_ex(m, token, pos, 0, next_host, logits_host, nullptr);
}

extern "C" int pb_model_set_token(pb_model* m, int token) {
  if (!m) return PB_ERR_ARG;
  if (token < 0 || token >= m->c.vocab) return pb_set_error(m->ctx, PB_ERR_ARG, "token %d out of range", token);
  m->h_io_pinned[0] = token;
  PB_TRY_CUDA(m->ctx, cudaMemcpyAsync(m->tok_dev, m->h_io_pinned, 4, cudaMemcpyHostToDevice, m->ctx->stream));
  return pb_wait(m->ctx);
}

extern "C" int pb_model_decode_loop(pb_model* m, int pos0, int steps, int* out_dev) {
  if (!m || steps < 0) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  if (pos0 < 0 || pos0 + steps > m->c.seq_len)
    return pb_set_error(ctx, PB_ERR_ARG, "positions [%d, %d) exceed the cache length", pos0, pos0 + steps);
  PB_TRY(ensure_graph(m));
  m->h_io_pinned[4] = pos0;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->tok_dev + 1, &m->h_io_pinned[4], 4, cudaMemcpyHostToDevice, ctx->stream));
  for (int s = 0; s < steps; ++s) PB_TRY_CUDA(ctx, cudaGraphLaunch(m->exec, ctx->stream));
  if (out_dev && steps)
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(out_dev, m->hist + pos0 + 1, (size_t)steps * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  return PB_OK;  // asynchronous: pb_sync() waits
}

extern "C" int pb_model_generate(pb_model* m, const int* prompt, int n_prompt, int max_tokens, int eos_id, int* out,
                                 int cap, int* n_out) {
  if (!m || !prompt || n_prompt <= 0 || !out || cap <= 0) return PB_ERR_ARG;
  if (n_out) *n_out = 0;
  PB_TRY(pb_model_reset_cache(m));
  int cnt = 0;
  for (int i = 0; i < n_prompt && cnt < cap; ++i) out[cnt++] = prompt[i];
  int next = 0;
  if (n_prompt == 1) {
    PB_TRY(pb_model_decode(m, prompt[0], 0, &next, nullptr));
  } else {
    PB_TRY(pb_model_forward(m, prompt, n_prompt, 0, nullptr));
    PB_TRY_CUDA(m->ctx, cudaMemcpy(&next, m->tok_dev, 4, cudaMemcpyDeviceToHost));
  }
  int pos = n_prompt;
  if (cnt < cap) out[cnt++] = next;
  for (int i = 1; i < max_tokens; ++i) {
    if (next == eos_id) break;
    if (pos >= m->c.seq_len) break;
    int nx;
    PB_TRY(pb_model_decode(m, next, pos, &nx, nullptr));
    pos++;
    next = nx;
    if (cnt < cap) out[cnt++] = next;
    if (next == eos_id) break;
  }
  if (n_out) *n_out = cnt;
  return PB_OK;
}

// Decode step with top-K sampling in place of the greedy step end: the head
// writes the logits, k_sample_cand / k_sample_pick draw the next token with
// the device counter, advance the position and record the token.

static int ensure_sample_graph(pb_model* m, int top_k, double temperature, uint64_t seed) {
  pb_ctx* ctx = m->ctx;
  PB_TRY(ensure_sample_buffers(m));
  check_graph_mode(m);
  PB_TRY(ensure_head_rows(m));
  if (m->sexec && m->s_topk == top_k && m->s_temp == temperature && m->s_seed == seed) return PB_OK;
  if (m->sexec) cudaGraphExecDestroy(m->sexec);
  if (m->sgraph) cudaGraphDestroy(m->sgraph);
  m->sexec = nullptr;
  m->sgraph = nullptr;
  PB_TRY(ensure_act(m, 1));
  PB_TRY_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  int rc = launch_embed(m, m->tok_dev, 1);
  for (int l = 0; l < m->c.n_layers && rc == PB_OK; ++l) rc = run_layer(m, l, 1, 0, true);
  if (rc == PB_OK) rc = launch_head(m, m->x);
  if (rc == PB_OK)
    rc = pb_launch_sample(ctx, m->logits, m->c.vocab, top_k, temperature, seed, 0, m->samp_ctr, m->samp_cand,
                          m->tok_dev, m->tok_dev + 1, m->hist, m->c.seq_len + 1, m->key);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
  if (rc != PB_OK) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return pb_cuda_error(ctx, e, "sampling graph capture");
  e = cudaGraphInstantiate(&m->sexec, g, 0);
  if (e != cudaSuccess) { cudaGraphDestroy(g); return pb_cuda_error(ctx, e, "sampling graph instantiate"); }
  m->sgraph = g;
  m->s_topk = top_k;
  m->s_temp = temperature;
  m->s_seed = seed;
  return PB_OK;
}

extern "C" int pb_model_generate_sampled(pb_model* m, const int* prompt, int n_prompt, int max_tokens, int eos_id,
                                         int top_k, double temperature, uint64_t seed, int* out, int cap, int* n_out) {
  if (!m || !prompt || n_prompt <= 0 || !out || cap <= 0) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  if (top_k <= 0 || top_k > 256 || !(temperature > 0.0))
    return pb_set_error(ctx, PB_ERR_ARG, "sampling needs 0 < topK <= 256 and temperature > 0");
  if (n_out) *n_out = 0;
  PB_TRY(ensure_sample_buffers(m));
  PB_TRY(pb_model_reset_cache(m));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(m->samp_ctr, 0, 8, ctx->stream));
  int cnt = 0;
  for (int i = 0; i < n_prompt && cnt < cap; ++i) out[cnt++] = prompt[i];
  // the prompt's logits (llama-streaming.js:925-930), then draw 0
  PB_TRY(pb_model_forward(m, prompt, n_prompt, 0, nullptr));
  PB_TRY(pb_launch_sample(ctx, m->logits, m->c.vocab, top_k, temperature, seed, 0, m->samp_ctr, m->samp_cand,
                          m->tok_dev, nullptr, nullptr, 0, nullptr));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->h_io_pinned + 2, m->tok_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
  PB_TRY(pb_wait(ctx));
  int next = m->h_io_pinned[2];
  int pos = n_prompt;
  if (cnt < cap) out[cnt++] = next;
  // recorded after the prefill, which may have regrown the activations
  if (max_tokens > 1) PB_TRY(ensure_sample_graph(m, top_k, temperature, seed));
  for (int i = 1; i < max_tokens; ++i) {
    if (next == eos_id || pos >= m->c.seq_len) break;
    m->h_io_pinned[0] = next;
    m->h_io_pinned[1] = pos;
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->tok_dev, m->h_io_pinned, 8, cudaMemcpyHostToDevice, ctx->stream));
    PB_TRY_CUDA(ctx, cudaGraphLaunch(m->sexec, ctx->stream));
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(m->h_io_pinned + 2, m->tok_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
    PB_TRY(pb_wait(ctx));
    next = m->h_io_pinned[2];
    ++pos;
    if (cnt < cap) out[cnt++] = next;
  }
  if (n_out) *n_out = cnt;
  return PB_OK;
}

extern "C" int pb_model_reset_cache(pb_model* m) {
  if (!m) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  PB_TRY_CUDA(ctx, cudaMemsetAsync(m->kc, 0, kv_floats(m) * 4, ctx->stream));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(m->vc, 0, kv_floats(m) * 4, ctx->stream));
  return pb_wait(ctx);
}

extern "C" int pb_model_rollback_cache(pb_model* m, int pos) {
  if (!m) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  if (pos < 0) pos = 0;
  if (pos >= m->c.seq_len) return PB_OK;
  size_t rowb = (size_t)m->kv_dim * 4;
  for (int l = 0; l < m->c.n_layers; ++l) {
    PB_TRY_CUDA(ctx, cudaMemsetAsync(kcache(m, l) + (size_t)pos * m->kv_dim, 0, (m->c.seq_len - pos) * rowb, ctx->stream));
    PB_TRY_CUDA(ctx, cudaMemsetAsync(vcache(m, l) + (size_t)pos * m->kv_dim, 0, (m->c.seq_len - pos) * rowb, ctx->stream));
  }
  return pb_wait(ctx);
}

// Llama-3 RoPE frequency scaling (pb_rope_freqs) on the model's rotation
// table; factor <= 0 restores the reference's unscaled table.  The table is
// rebuilt in place, so recorded decode graphs pick it up.
extern "C" int pb_rope_freqs(double theta, int hd, double factor, double low_freq_factor, double high_freq_factor,
                             int original_max_pos, double* freqs_out);
extern "C" int pb_model_set_rope_scaling(pb_model* m, double factor, double low_freq_factor, double high_freq_factor,
                                         int original_max_pos) {
  if (!m) return PB_ERR_ARG;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  std::vector<double> freqs((size_t)c.head_dim / 2);
  if (pb_rope_freqs(c.rope_theta, c.head_dim, factor, low_freq_factor, high_freq_factor, original_max_pos,
                    freqs.data()) != PB_OK)
    return pb_set_error(ctx, PB_ERR_ARG,
                        "RoPE scaling needs factor > 0, 0 < low_freq_factor < high_freq_factor and "
                        "original_max_pos > 0 (or factor <= 0 to turn it off)");
  std::vector<double2> tab((size_t)c.seq_len * (c.head_dim / 2));
  pb_rope_table_freqs(freqs.data(), c.head_dim, 0, c.seq_len, tab.data());
  PB_TRY(pb_wait(ctx));  // no replay may read the table while it changes
  PB_TRY_CUDA(ctx, cudaMemcpy(m->rope_tab, tab.data(), tab.size() * sizeof(double2), cudaMemcpyHostToDevice));
  if (factor > 0) {
    m->rope_scaling[0] = factor;
    m->rope_scaling[1] = low_freq_factor;
    m->rope_scaling[2] = high_freq_factor;
    m->rope_scaling[3] = original_max_pos;
  } else {
    m->rope_scaling[0] = m->rope_scaling[1] = m->rope_scaling[2] = m->rope_scaling[3] = 0;
  }
  return PB_OK;
}

extern "C" int pb_model_rope_scaling(const pb_model* m, double* factor_out) {
  if (!m || !factor_out) return PB_ERR_ARG;
  *factor_out = m->rope_scaling[0];
  return PB_OK;
}

extern "C" int pb_model_kv(pb_model* m, int layer, int which_v, float* host, size_t floats) {
  if (!m || !host || layer < 0 || layer >= m->c.n_layers) return PB_ERR_ARG;
  size_t n = (size_t)m->c.seq_len * m->kv_dim;
  if (floats != n) return pb_set_error(m->ctx, PB_ERR_ARG, "kv buffer needs %zu floats", n);
  return pb_download(m->ctx, host, which_v ? vcache(m, layer) : kcache(m, layer), n * 4);
}

extern "C" int64_t pb_model_decode_bytes(const pb_model* m, int pos) {
  if (!m) return 0;
  const pb_model_config& c = m->c;
  int64_t w = 0;
  for (int which = 1; which <= 7; ++which) {
    int r, k;
    mshape(c, which, &r, &k);
    int64_t n = (int64_t)r * k;
    w += c.kind == PB_MODEL_STREAMING_Q4 ? n / 32 * 18 : (n + 31) / 32 * 36;
  }
  w *= c.n_layers;
  int64_t ne = (int64_t)c.vocab * c.dim;
  int mode = 0;
  const int ht = head_table(m, &mode)->type;
  int64_t head = ht == PB_TYPE_F32 ? ne * 4 : ne / 32 * (ht == PB_TYPE_Q4_0 ? 18 : 34);
  int64_t kvb = (int64_t)2 * c.n_layers * (pos + 1) * m->kv_dim * 4;
  return w + head + kvb;
}

extern "C" int pb_model_decode_launches(const pb_model* m) { return m ? m->launches_per_step : 0; }

// ===========================================================================
// batched serving: n_seqs independent sequences over one streaming model's
// weights.  Every sequence has its own KV cache; all of them advance together
// (same prompt length, same position).  The projections and the LM head run
// as tensor-core GEMMs over the token rows of all sequences
// (pb_launch_q4_gemm: f16 operands, f32 accumulation, so the logits agree with
// the one-sequence path within a tolerance); RoPE, attention, SwiGLU and the
// residual adds are launched over all sequences at once.  The reference runs
// one sequence at a time (llama-streaming.js:738-815); this is the batched
// configuration's form of it.
//
// Row split over `world` ranks (thread-pool.js:165-246 splits one matvec's
// output rows over worker threads; here every projection and the LM head is
// split by output rows over GPUs).  Rank r holds
//   - the query heads [r*H/w, (r+1)*H/w) and kv heads [r*Hkv/w, ...) of every
//     layer: its rows of [wq; wk; wv] and its slice of the KV cache, so RoPE
//     and attention stay local;
//   - output rows [r*dim/w, ...) of wo and w2, rows [r*2F/w, ...) of the
//     interleaved gate|up matrix (hidden units [r*F/w, ...)), and a contiguous
//     range of vocab rows of the head.
// Activations that every rank reads whole are stored as column chunks,
// [w][rows][width/w], chunk r written by rank r, so one in-place all-gather
// per exchange completes them: the attention output (before wo), the
// residual x (after wo and after w2) and the SwiGLU output h (before w2).
// The GEMMs read chunked operands directly (pb_gemm_epi.x_chunk) and plan
// split K for the whole matrix (split_n), and the greedy token is the
// largest of the ranks' argmax keys, so every rank's tokens and logits have
// the same bits as one GPU's.  Across processes the all-gather is NCCL on
// the context stream (recorded into the decode graph); an emulated group
// runs all ranks' shards in one process on one device and copies the chunks.
// ===========================================================================

// One rank's weights, cache and activations.
struct pb_shard {
  int rank = 0;
  bool owns = false;  // row copies (world > 1) rather than the model's own matrices
  std::vector<pb_qmat*> qkv, wo, gu, w2;
  pb_qmat* head = nullptr;
  pb_split_plan p{};
  float *kc = nullptr, *vc = nullptr;  // [layer][seq][seq_len][n_kv_heads(rank) * head_dim]
  float* x = nullptr;     // residual, column chunks [world][rows][dim / world] (all ranks hold all)
  float* xn = nullptr;    // normed rows, row-major (f16 on the TMA path)
  float* qkvo = nullptr;  // the rank's q | k | v per token
  float* att = nullptr;   // attention output chunks [world][rows][dim / world]
  float* hb = nullptr;    // SwiGLU output chunks [world][rows][F / world] (f16 on the TMA path)
  float* xl = nullptr;    // last row of every sequence, row-major [B][dim]
  float* logits = nullptr;               // [world][B][vocab_chunk]; the rank's chunk is computed
  unsigned long long* keys = nullptr;    // [world][B] argmax keys of each rank's vocab rows
  // the prefill's K and V as hi/lo halves, [K, V][seq][prompt pos][kv head][hi 64 | lo 64]
  // (three-term prefill attention operands, written by k_rope_kv)
  __half* kvhl = nullptr;
  size_t kvhl_bytes = 0;
};

struct pb_batch {
  pb_model* m = nullptr;
  int B = 0;
  int world = 1;
  pb_comm* comm = nullptr;    // NCCL: this process holds one shard
  std::vector<pb_shard> sh;   // one shard, or all `world` of an emulated group
  int rows_cap = 0;           // activation rows allocated
  int P = 0;                  // prompt length of the current batch
  int* toks = nullptr;        // [rows] token ids (prefill)
  int* next = nullptr;        // [B] greedy tokens of the last step
  int* pos_dev = nullptr;     // position of the tokens the next decode step reads
  int* hist = nullptr;        // [seq_len + 1][B] greedy token produced at each position
  float* ws = nullptr;        // split-K partial tiles of the decode-step GEMMs (and attention partials)
  size_t ws_bytes = 0;
  int* attn_cnt = nullptr;    // [B][n_kv] split counters of the decode attention (reset by the kernel)
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // peer exchange (NCCL communicator with peer access on every rank): every
  // rank's copy of the exchanged buffers, by XG_* id, [id][rank]
  void* peer[5][PB_MAX_RANKS] = {};
  bool p2p_fixed = false;  // keys, logits shared
  bool p2p_rows = false;   // x, att, hb shared (re-shared when they grow)
  // low-latency exchange slots (pb_comm_ll_gather) for chunks up to ll_cap
  // units of 8 bytes: the decode step's exchanges
  pb_ll_slots ll{};
  size_t ll_cap = 0;
  bool p2p_ll = false;
  void* ll_mem = nullptr;  // this rank's slots, then its epoch and done counters
  bool decoding = false;   // the layer being enqueued is a decode step (one row per sequence)
  // GEMM precision: 3 = f16 hi/lo pairs of both operands, three tensor-core
  // products (the default); 1 = each operand rounded to f16 once
  int terms = 3;
};

// halves per value of an f16 GEMM operand the batch writes: hi and lo, or hi alone
static int op_halves(const pb_batch* b) { return b->terms == 3 ? 2 : 1; }

// the buffers the row split exchanges
enum { XG_X = 0, XG_ATT = 1, XG_HB = 2, XG_KEYS = 3, XG_LOGITS = 4 };
static void* xg_buf(pb_shard& s, int id) {
  switch (id) {
    case XG_X: return s.x;
    case XG_ATT: return s.att;
    case XG_HB: return s.hb;
    case XG_KEYS: return s.keys;
    default: return s.logits;
  }
}

// Share buffers ids[0..n) of this process's shard with the other ranks (peer
// exchange); false when some rank could not.
static int batch_share(pb_batch* b, const int* ids, int n, bool* ok) {
  *ok = false;
  if (!b->comm || !pb_comm_p2p(b->comm)) return PB_OK;
  void* local[5];
  void* table[5 * PB_MAX_RANKS] = {};
  for (int i = 0; i < n; ++i) local[i] = xg_buf(b->sh[0], ids[i]);
  PB_TRY(pb_comm_share_agreed(b->comm, local, n, table, true, ok));
  if (*ok)
    for (int i = 0; i < n; ++i)
      for (int q = 0; q < b->world; ++q) b->peer[ids[i]][q] = table[(size_t)i * b->world + q];
  return PB_OK;
}

static void batch_unshare(pb_batch* b, const int* ids, int n) {
  for (int i = 0; i < n; ++i) {
    void* table[PB_MAX_RANKS];
    for (int q = 0; q < b->world; ++q) table[q] = b->peer[ids[i]][q];
    pb_comm_unshare(b->comm, table, 1);
    for (int q = 0; q < PB_MAX_RANKS; ++q) b->peer[ids[i]][q] = nullptr;
  }
}

// The low-latency slots, sized for the decode step's largest chunk (the
// f32 SwiGLU output of all sequences); collective.
static int batch_share_ll(pb_batch* b) {
  if (!b->comm || !pb_comm_p2p(b->comm)) return PB_OK;
  pb_ctx* ctx = b->m->ctx;
  const pb_model_config& c = b->m->c;
  const int widest = c.hidden_dim > c.dim ? c.hidden_dim : c.dim;
  b->ll_cap = ((size_t)b->B * widest * 4 / b->world + 7) / 8;
  const size_t slot_bytes = 2 * (size_t)b->world * b->ll_cap * 16;
  PB_TRY_CUDA(ctx, cudaMalloc(&b->ll_mem, slot_bytes + 64));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(b->ll_mem, 0, slot_bytes + 64, ctx->stream));
  PB_TRY(pb_wait(ctx));
  void* table[PB_MAX_RANKS] = {};
  void* local = b->ll_mem;
  PB_TRY(pb_comm_share_agreed(b->comm, &local, 1, table, true, &b->p2p_ll));
  if (b->p2p_ll)
    for (int q = 0; q < b->world; ++q) b->ll.s[q] = static_cast<uint4*>(table[q]);
  return PB_OK;
}

static unsigned int* ll_counters(pb_batch* b) {
  return reinterpret_cast<unsigned int*>(static_cast<char*>(b->ll_mem) + 2 * (size_t)b->world * b->ll_cap * 16);
}

static const int XG_ROWS[3] = {XG_X, XG_ATT, XG_HB};
static const int XG_FIXED[2] = {XG_KEYS, XG_LOGITS};

extern "C" int pb_batch_split_plan(const pb_model_config* c, int world, int rank, pb_split_plan* out) {
  if (!c || !out || world < 1 || rank < 0 || rank >= world) return PB_ERR_ARG;
  if (c->n_heads <= 0 || c->n_kv_heads <= 0 || c->head_dim <= 0 || c->dim <= 0 || c->hidden_dim <= 0 || c->vocab <= 0)
    return PB_ERR_ARG;
  if (world > 1 && (c->n_kv_heads % world || c->dim % (64 * world) || c->hidden_dim % (64 * world)))
    return PB_ERR_ARG;
  pb_split_plan p{};
  const int hd = c->head_dim, kv = c->n_kv_heads * hd;
  p.world = world;
  p.rank = rank;
  p.n_heads = c->n_heads / world;
  p.n_kv_heads = c->n_kv_heads / world;
  p.q_row0 = rank * p.n_heads * hd;
  p.k_row0 = c->dim + rank * p.n_kv_heads * hd;
  p.v_row0 = c->dim + kv + rank * p.n_kv_heads * hd;
  p.qkv_rows = (p.n_heads + 2 * p.n_kv_heads) * hd;
  p.dim_chunk = c->dim / world;
  p.hidden_chunk = c->hidden_dim / world;
  // vocab rows in chunks of a multiple of 32 rows; the last rank takes the rest
  const int per = world == 1 ? c->vocab : (c->vocab + world - 1) / world;
  p.vocab_chunk = world == 1 ? c->vocab : (per + 31) / 32 * 32;
  p.vocab_row0 = rank * p.vocab_chunk;
  const int left = c->vocab - p.vocab_row0;
  p.vocab_rows = left < 0 ? 0 : left < p.vocab_chunk ? left : p.vocab_chunk;
  if (p.vocab_rows <= 0) return PB_ERR_ARG;  // more ranks than vocab chunks
  *out = p;
  return PB_OK;
}

// rows [src_row0, src_row0 + rows) of a row-layout matrix -> dst rows from dst_row0
static int copy_rows(pb_ctx* ctx, pb_qmat* dst, int dst_row0, const pb_qmat* src, int src_row0, int rows) {
  const size_t nb = (size_t)src->nb;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(dst->qs + (size_t)dst_row0 * nb * 16, src->qs + (size_t)src_row0 * nb * 16,
                                   (size_t)rows * nb * 16, cudaMemcpyDeviceToDevice, ctx->stream));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(dst->d + (size_t)dst_row0 * nb, src->d + (size_t)src_row0 * nb, (size_t)rows * nb * 2,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  return PB_OK;
}

static int slice_rows(pb_ctx* ctx, const pb_qmat* src, int row0, int rows, pb_qmat** out) {
  PB_TRY(pb_qmat_alloc(ctx, src->type, PB_LAYOUT_ROWS, rows, src->K, out));
  return copy_rows(ctx, *out, 0, src, row0, rows);
}

static void shard_free(pb_ctx* ctx, pb_shard& s) {
  if (s.owns) {
    for (auto* q : s.qkv) pb_qmat_free(ctx, q);
    for (auto* q : s.wo) pb_qmat_free(ctx, q);
    for (auto* q : s.gu) pb_qmat_free(ctx, q);
    for (auto* q : s.w2) pb_qmat_free(ctx, q);
    pb_qmat_free(ctx, s.head);
  }
  s.qkv.clear(); s.wo.clear(); s.gu.clear(); s.w2.clear();
  s.head = nullptr;
  cudaFree(s.kc); cudaFree(s.vc); cudaFree(s.x); cudaFree(s.xn); cudaFree(s.qkvo); cudaFree(s.att); cudaFree(s.hb);
  cudaFree(s.xl); cudaFree(s.logits); cudaFree(s.keys); cudaFree(s.kvhl);
  s.kc = s.vc = s.x = s.xn = s.qkvo = s.att = s.hb = s.xl = s.logits = nullptr;
  s.keys = nullptr;
}

// The rank's weights (row copies when split) and its fixed-size buffers.
static int shard_init(pb_batch* b, pb_shard& s, int rank) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  s.rank = rank;
  if (pb_batch_split_plan(&c, b->world, rank, &s.p) != PB_OK)
    return pb_set_error(ctx, PB_ERR_ARG, "a row split over %d ranks needs n_kv_heads, dim / 64 and hidden_dim / 64 "
                                         "divisible by it and a vocab of at least one row chunk per rank", b->world);
  const pb_split_plan& p = s.p;
  const int L = c.n_layers, hd = c.head_dim;
  if (b->world == 1) {
    s.qkv = m->qkv; s.wo = m->wo; s.gu = m->gu; s.w2 = m->w2;
    s.head = head_of(m);
  } else {
    s.owns = true;
    s.qkv.assign(L, nullptr); s.wo.assign(L, nullptr); s.gu.assign(L, nullptr); s.w2.assign(L, nullptr);
    for (int l = 0; l < L; ++l) {
      PB_TRY(pb_qmat_alloc(ctx, PB_TYPE_Q4_0, PB_LAYOUT_ROWS, p.qkv_rows, c.dim, &s.qkv[l]));
      PB_TRY(copy_rows(ctx, s.qkv[l], 0, m->qkv[l], p.q_row0, p.n_heads * hd));
      PB_TRY(copy_rows(ctx, s.qkv[l], p.n_heads * hd, m->qkv[l], p.k_row0, p.n_kv_heads * hd));
      PB_TRY(copy_rows(ctx, s.qkv[l], (p.n_heads + p.n_kv_heads) * hd, m->qkv[l], p.v_row0, p.n_kv_heads * hd));
      PB_TRY(slice_rows(ctx, m->wo[l], rank * p.dim_chunk, p.dim_chunk, &s.wo[l]));
      // 2F/world rows of the interleave-4 gate|up matrix: hidden units [rank*F/world, ...)
      PB_TRY(slice_rows(ctx, m->gu[l], rank * 2 * p.hidden_chunk, 2 * p.hidden_chunk, &s.gu[l]));
      PB_TRY(slice_rows(ctx, m->w2[l], rank * p.dim_chunk, p.dim_chunk, &s.w2[l]));
    }
    // head rows [vocab_row0, +vocab_rows) of the tiled table: whole 8-row tiles
    const pb_qmat* h = head_of(m);
    PB_TRY(pb_qmat_alloc(ctx, h->type, PB_LAYOUT_TILED8, p.vocab_rows, c.dim, &s.head));
    const size_t qb = h->type == PB_TYPE_Q8_0 ? 32 : 16, slots = (size_t)pb_cdiv(p.vocab_rows, 8) * 8 * h->nb;
    const size_t s0 = (size_t)pb_qslot(p.vocab_row0, 0, h->nb);
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(s.head->qs, h->qs + s0 * qb, slots * qb, cudaMemcpyDeviceToDevice, ctx->stream));
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(s.head->d, h->d + s0, slots * 2, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  const size_t kv = (size_t)L * b->B * c.seq_len * p.n_kv_heads * hd;
  PB_TRY_CUDA(ctx, cudaMalloc(&s.kc, kv * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&s.vc, kv * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&s.xl, (size_t)b->B * c.dim * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&s.logits, (size_t)b->world * b->B * p.vocab_chunk * 4));
  PB_TRY_CUDA(ctx, cudaMalloc(&s.keys, (size_t)b->world * b->B * 8));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(s.keys, 0, (size_t)b->world * b->B * 8, ctx->stream));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(s.kc, 0, kv * 4, ctx->stream));
  PB_TRY_CUDA(ctx, cudaMemsetAsync(s.vc, 0, kv * 4, ctx->stream));
  return PB_OK;
}

__global__ void k_gather_last(const float* __restrict__ x, int rows_per_seq, int dim, int xc, int rows,
                              float* __restrict__ out) {
  const int s = blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= dim) return;
  const size_t row = (size_t)s * rows_per_seq + rows_per_seq - 1;
  out[(size_t)s * dim + d] = x[(size_t)(d / xc) * rows * xc + row * xc + d % xc];
}

// Embedding rows of a tiled Q4_0 / Q8_0 table (gguf.js:239-286 values) into
// x's column chunks of width xc.
__global__ void k_batch_embed(int type, const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, int V,
                              int dim, const int* __restrict__ toks, float* __restrict__ x, int xc, int rows, int* err) {
  const int i = blockIdx.y, d = blockIdx.x * blockDim.x + threadIdx.x;
  const int tok = toks[i];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0) pb_raise(err, PB_DEVERR_TOKEN);
    return;
  }
  if (d >= dim) return;
  const int nb = dim / 32, b = d >> 5, j = d & 31;
  const size_t slot = (size_t)pb_qslot(tok, b, nb);
  const float sc = pb_f16_exact(dsc[slot]);
  float v;
  if (type == PB_TYPE_Q4_0) {
    const uint8_t byte = qs[slot * 16 + (j & 15)];
    v = __fmul_rn((float)((j < 16 ? (byte & 15) : (byte >> 4)) - 8), sc);
  } else {
    v = __fmul_rn((float)(int8_t)qs[slot * 32 + j], sc);
  }
  x[(size_t)(d / xc) * rows * xc + (size_t)i * xc + d % xc] = v;
}

// Greedy token (llama-streaming.js:899-909: the first strict maximum) as an
// ordered key per row over vocab chunks: CTA (row, chunk) folds its chunk
// into keys[row] with atomicMax (the largest value, the lowest index among
// equals, so the order of the atomics does not matter).  The key carries the
// global token index (v0 + i).
constexpr int AMX_CHUNK = 8192;
__global__ void __launch_bounds__(256)
k_argmax_chunks(const float* __restrict__ logits, int n, int ld, int v0, unsigned long long* __restrict__ keys) {
  pb_pdl_trigger();
  pb_pdl_wait();  // the logits come from the head
  __shared__ unsigned long long red[8];
  const int r = blockIdx.y, c0 = blockIdx.x * AMX_CHUNK, c1 = min(n, c0 + AMX_CHUNK);
  unsigned long long key = 0ull;
  for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const unsigned long long k = pb_argmax_key(logits[(size_t)r * ld + i], v0 + i);
    key = k > key ? k : key;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
    key = t > key ? t : key;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long best = 0ull;
    for (int w = 0; w < 8; ++w) best = red[w] > best ? red[w] : best;
    atomicMax(keys + r, best);
  }
}

// The largest of the ranks' keys [world][B] per row: the global first maximum.
// reset: clear this rank's keys for the next step's atomicMax.
__global__ void k_argmax_merge(unsigned long long* __restrict__ keys, int world, int B, int* __restrict__ next,
                               int* __restrict__ hist, const int* __restrict__ pos_dev, int hist_len,
                               unsigned long long* __restrict__ reset) {
  pb_pdl_trigger();
  pb_pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B) return;
  unsigned long long best = 0ull;
  for (int w = 0; w < world; ++w) best = keys[(size_t)w * B + r] > best ? keys[(size_t)w * B + r] : best;
  if (reset) reset[r] = 0ull;
  if (!next) return;
  const int tok = pb_argmax_index(best);
  next[r] = tok;
  if (hist && pos_dev) {
    const int p = *pos_dev;
    if (p >= 0 && p < hist_len) hist[(size_t)p * B + r] = tok;
  }
}

__global__ void k_batch_step_end(int* __restrict__ pos_dev) {
  pb_pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) *pos_dev += 1;
}

static void batch_free_graph(pb_batch* b) {
  if (b->exec) cudaGraphExecDestroy(b->exec);
  if (b->graph) cudaGraphDestroy(b->graph);
  b->exec = nullptr;
  b->graph = nullptr;
}

static int batch_ensure_rows(pb_batch* b, int rows) {
  if (rows <= b->rows_cap) return PB_OK;
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  PB_TRY(pb_wait(ctx));
  batch_free_graph(b);  // a recorded graph holds the old buffer addresses
  if (b->p2p_rows) batch_unshare(b, XG_ROWS, 3);
  b->p2p_rows = false;
  cudaFree(b->toks);
  b->toks = nullptr;
  b->rows_cap = 0;
  const pb_model_config& c = m->c;
  for (auto& s : b->sh) {
    cudaFree(s.x); cudaFree(s.xn); cudaFree(s.qkvo); cudaFree(s.att); cudaFree(s.hb);
    s.x = s.xn = s.qkvo = s.att = s.hb = nullptr;
  }
  for (auto& s : b->sh) {
    PB_TRY_CUDA(ctx, cudaMalloc(&s.x, (size_t)rows * c.dim * 4));
    PB_TRY_CUDA(ctx, cudaMalloc(&s.xn, (size_t)rows * c.dim * 4));
    PB_TRY_CUDA(ctx, cudaMalloc(&s.qkvo, (size_t)rows * s.p.qkv_rows * 4));
    PB_TRY_CUDA(ctx, cudaMalloc(&s.att, (size_t)rows * c.dim * 4));
    PB_TRY_CUDA(ctx, cudaMalloc(&s.hb, (size_t)rows * c.hidden_dim * 4));
  }
  PB_TRY_CUDA(ctx, cudaMalloc(&b->toks, (size_t)rows * 4));
  b->rows_cap = rows;
  // collective: every rank grows its buffers in the same call
  return batch_share(b, XG_ROWS, 3, &b->p2p_rows);
}

extern "C" int pb_batch_set_precision(pb_batch* b, int terms) {
  if (!b || (terms != 1 && terms != 3)) return PB_ERR_ARG;
  if (terms != b->terms) batch_free_graph(b);  // the recorded decode step holds the other kernels
  b->terms = terms;
  return PB_OK;
}

extern "C" int pb_batch_free(pb_batch* b) {
  if (!b) return PB_OK;
  pb_ctx* ctx = b->m ? b->m->ctx : nullptr;
  if (ctx) pb_wait(ctx);
  batch_free_graph(b);  // before the communicator its NCCL nodes use goes away
  if (b->p2p_rows) batch_unshare(b, XG_ROWS, 3);
  if (b->p2p_fixed) batch_unshare(b, XG_FIXED, 2);
  if (b->p2p_ll) {
    void* table[PB_MAX_RANKS];
    for (int q = 0; q < b->world; ++q) table[q] = b->ll.s[q];
    pb_comm_unshare(b->comm, table, 1);
  }
  cudaFree(b->ll_mem);
  for (auto& s : b->sh) shard_free(ctx, s);
  cudaFree(b->toks); cudaFree(b->next); cudaFree(b->pos_dev); cudaFree(b->hist); cudaFree(b->ws);
  cudaFree(b->attn_cnt);
  delete b;
  return PB_OK;
}

static int batch_create(pb_model* m, int n_seqs, int world, pb_comm* comm, pb_batch** out) {
  if (!m || !out || n_seqs <= 0 || world < 1) return PB_ERR_ARG;
  *out = nullptr;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  // decode steps run the fused-dequant GEMM, which needs no growable scratch
  // (the recorded decode graph relies on that)
  if (n_seqs > 256) return pb_set_error(ctx, PB_ERR_ARG, "at most 256 sequences per batch");
  if (c.kind != PB_MODEL_STREAMING_Q4 || !m->emb || m->emb->type != PB_TYPE_Q4_0 || !head_of(m) ||
      head_of(m)->type != PB_TYPE_Q4_0)
    return pb_set_error(ctx, PB_ERR_ARG, "batched serving needs a streaming model with a Q4_0 embedding and head");
  if (!pb_attn_decode_group_ok(c.n_heads / world, c.n_kv_heads / world, c.head_dim, c.seq_len))
    return pb_set_error(ctx, PB_ERR_ARG, "batched decode attention needs <= 8 query heads per kv head, head_dim %% 4 "
                                         "== 0, head_dim <= 256 and the scores of a kv head in shared memory");
  pb_batch* b = new pb_batch();
  b->m = m;
  b->B = n_seqs;
  b->world = world;
  b->comm = comm;
  auto fail = [&](int rc) { pb_batch_free(b); return rc; };
  const int nshards = comm ? 1 : world;
  b->sh.resize(nshards);
  for (int i = 0; i < nshards; ++i) {
    const int rc = shard_init(b, b->sh[i], comm ? pb_comm_rank(comm) : i);
    if (rc != PB_OK) return fail(rc);
  }
  const int widest = 2 * c.hidden_dim > c.dim + 2 * m->kv_dim ? 2 * c.hidden_dim : c.dim + 2 * m->kv_dim;
  b->ws_bytes = (size_t)8 * n_seqs * widest * 4;  // up to 8 K splits of the widest layer matrix
  cudaError_t e = cudaMalloc(&b->next, (size_t)n_seqs * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->pos_dev, 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->hist, (size_t)(c.seq_len + 1) * n_seqs * 4);
  if (e == cudaSuccess) e = cudaMalloc(&b->ws, b->ws_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&b->attn_cnt, (size_t)n_seqs * c.n_kv_heads * 4);
  if (e == cudaSuccess) e = cudaMemsetAsync(b->attn_cnt, 0, (size_t)n_seqs * c.n_kv_heads * 4, ctx->stream);
  if (e != cudaSuccess) return fail(pb_cuda_error(ctx, e, "batch allocation"));
  cudaMemsetAsync(b->hist, 0, (size_t)(c.seq_len + 1) * n_seqs * 4, ctx->stream);
  cudaMemsetAsync(b->pos_dev, 0, 4, ctx->stream);
  int rc = pb_wait(ctx);
  if (rc == PB_OK) rc = batch_share(b, XG_FIXED, 2, &b->p2p_fixed);
  if (rc == PB_OK) rc = batch_share_ll(b);
  if (rc != PB_OK) return fail(rc);
  *out = b;
  return PB_OK;
}

extern "C" int pb_batch_create(pb_model* m, int n_seqs, pb_batch** out) {
  return batch_create(m, n_seqs, 1, nullptr, out);
}

extern "C" int pb_batch_create_split(pb_model* m, int n_seqs, pb_comm* comm, pb_batch** out) {
  if (!m || !comm || pb_comm_ctx(comm) != m->ctx) return PB_ERR_ARG;
  const int world = pb_comm_world(comm);
  return batch_create(m, n_seqs, world, world > 1 ? comm : nullptr, out);
}

extern "C" int pb_batch_create_group(pb_model* m, int n_seqs, int world, pb_batch** out) {
  return batch_create(m, n_seqs, world, nullptr, out);
}

// In-place all-gather of chunk_bytes per rank: chunk r of buffer `id` is
// rank r's; afterwards every shard's buffer holds every chunk.  Across
// processes: the peer exchange kernel when every rank shared the buffer,
// else an NCCL all-gather; in an emulated group, device copies.
static int batch_gather(pb_batch* b, int id, size_t chunk_bytes) {
  if (b->world == 1) return PB_OK;
  pb_ctx* ctx = b->m->ctx;
  if (b->comm) {
    const bool p2p = (id == XG_KEYS || id == XG_LOGITS) ? b->p2p_fixed : b->p2p_rows;
    if (b->p2p_ll && chunk_bytes % 8 == 0 && chunk_bytes / 8 <= b->ll_cap) {
      unsigned int* cnt = ll_counters(b);
      return pb_comm_ll_gather(b->comm, b->ll, b->ll_cap, static_cast<char*>(xg_buf(b->sh[0], id)), chunk_bytes, cnt,
                               cnt + 1);
    }
    if (p2p) return pb_comm_peer_gather(b->comm, b->peer[id], chunk_bytes);
    return pb_comm_gather_inplace(b->comm, xg_buf(b->sh[0], id), chunk_bytes);
  }
  for (auto& dst : b->sh)
    for (auto& src : b->sh) {
      if (&dst == &src) continue;
      const size_t off = (size_t)src.rank * chunk_bytes;
      PB_TRY_CUDA(ctx, cudaMemcpyAsync(static_cast<char*>(xg_buf(dst, id)) + off,
                                       static_cast<char*>(xg_buf(src, id)) + off, chunk_bytes,
                                       cudaMemcpyDeviceToDevice, ctx->stream));
    }
  return PB_OK;
}

// The x_chunk of an operand stored in `width`-wide chunks (0 when unsplit).
static int chunk_of(const pb_batch* b, int width) { return b->world > 1 ? width : 0; }

// Whether this step's residual exchanges are fused into their producers and
// consumers: decode steps of a row split whose ranks exchange over peer
// memory, the residual chunk within the low-latency slots.  The GEMM that adds
// into this rank's chunk of x sends it (pb_xsend), the next RMSNorm receives
// the peers' chunks (k_rmsnorm_xrecv): no exchange kernel in between.
static bool fused_x(const pb_batch* b, int rows) {
  const size_t chunk = (size_t)rows * (b->m->c.dim / b->world) * 4;
  return b->decoding && b->comm && b->p2p_ll && b->world > 1 && chunk % 8 == 0 && chunk / 8 <= b->ll_cap &&
         (b->m->c.dim / b->world) % 2 == 0 && (size_t)b->m->c.dim * 4 <= 48 * 1024;
}
static pb_xsend xsend_of(pb_batch* b, int width) {
  pb_xsend xs;
  for (int q = 0; q < PB_MAX_RANKS; ++q) xs.slots[q] = q < b->world ? b->ll.s[q] : nullptr;
  xs.cap_units = b->ll_cap;
  xs.epoch = ll_counters(b);
  xs.rank = b->sh[0].rank;
  xs.world = b->world;
  xs.width = width;
  return xs;
}
static pb_xrecv xrecv_of(pb_batch* b) {
  pb_xrecv xr;
  xr.mine = b->ll.s[b->sh[0].rank];
  xr.cap_units = b->ll_cap;
  xr.epoch = ll_counters(b);
  xr.done = xr.epoch + 1;
  xr.rank = b->sh[0].rank;
  xr.world = b->world;
  return xr;
}

// Decode-size steps (<= 64 token rows, head_dim 64): every GEMM takes f16
// activations (the warp-specialised decode GEMM), which the norms, the split
// attention and the SwiGLU epilogue write directly.
static bool dec16(const pb_batch* b, const pb_shard& s, int l, int rows) {
  return b->decoding && rows <= 64 && b->m->c.head_dim == 64 && pb_gemm_uses_ws(s.qkv[l], rows) &&
         pb_gemm_uses_ws(s.wo[l], rows) &&
         pb_gemm_uses_ws(s.gu[l], rows) && pb_gemm_uses_ws(s.w2[l], rows);
}

// One process with the whole model, a three-term prefill whose wo GEMM takes
// f16 operands (the TMA path): the prefill attention writes its output as the
// GEMM's hi/lo pairs (the bits k_f32_to_f16 would make of the f32 rows).
static bool att_hl_prefill(const pb_batch* b, const pb_shard& s, int l, int rows) {
  return b->world == 1 && b->sh.size() == 1 && b->terms == 3 && !b->decoding && b->m->c.head_dim == 64 &&
         pb_gemm_uses_tma(s.wo[l], rows);
}

// norm -> this rank's q | k | v -> RoPE + KV append -> attention of its heads
// into its chunk of att.
static int shard_attention(pb_batch* b, pb_shard& s, int l, int rows, int rows_per_seq, int start_pos,
                           const int* pos_dev, bool recv_x = false, bool normed = false) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  const pb_split_plan& p = s.p;
  const int dim = c.dim, hd = c.head_dim, qw = p.qkv_rows, dc = p.dim_chunk, kvl = p.n_kv_heads * hd;
  const int64_t cache_seq = (int64_t)c.seq_len * kvl;
  float* kc = s.kc + (size_t)l * b->B * cache_seq;
  float* vc = s.vc + (size_t)l * b->B * cache_seq;
  pb_gemm_epi st;
  st.split_n = dim + 2 * m->kv_dim;
  st.terms = b->terms;
  // the norm writes the GEMM's f16 operand directly on the TMA and decode paths
  __half* xn16 = reinterpret_cast<__half*>(s.xn);
  const bool d16 = dec16(b, s, l, rows);
  if (recv_x) {  // x's other chunks arrive with the norm (fused exchange)
    const bool f16 = pb_gemm_uses_tma(s.qkv[l], rows) || d16;
    PB_TRY(pb_launch_rmsnorm_xrecv(ctx, s.x, rows, dim, m->rms_att + (size_t)l * dim, c.eps, f16 ? nullptr : s.xn,
                                   f16 ? xn16 : nullptr, dc, f16 && b->terms == 3, xrecv_of(b)));
    if (f16) PB_TRY(pb_launch_q4_gemm(ctx, s.qkv[l], nullptr, dim, rows, s.qkvo, qw, b->ws, b->ws_bytes, &st, xn16));
    else PB_TRY(pb_launch_q4_gemm(ctx, s.qkv[l], s.xn, dim, rows, s.qkvo, qw, b->ws, b->ws_bytes, &st));
  } else if (pb_gemm_uses_tma(s.qkv[l], rows) || d16) {  // (normed: the previous down GEMM ran this norm)
    if (!normed) PB_TRY(launch_norm(m, s.x, rows, m->rms_att + (size_t)l * dim, nullptr, xn16, dc, b->terms == 3));
    PB_TRY(pb_launch_q4_gemm(ctx, s.qkv[l], nullptr, dim, rows, s.qkvo, qw, b->ws, b->ws_bytes, &st, xn16));
  } else {
    if (!normed) PB_TRY(launch_norm(m, s.x, rows, m->rms_att + (size_t)l * dim, s.xn, nullptr, dc));
    PB_TRY(pb_launch_q4_gemm(ctx, s.qkv[l], s.xn, dim, rows, s.qkvo, qw, b->ws, b->ws_bytes, &st));
  }
  // the three-term prefill attention reads K and V as hi/lo halves converted once, here
  const bool kv_hl = b->terms == 3 && hd == 64 && !pos_dev && start_pos == 0 && rows_per_seq > 1;
  const int64_t hl_stride = (int64_t)rows_per_seq * 2 * kvl;  // halves per sequence
  __half *khl = nullptr, *vhl = nullptr;
  if (kv_hl) {
    const size_t need = (size_t)2 * b->B * hl_stride * sizeof(__half);
    if (s.kvhl_bytes < need) {
      PB_TRY(pb_wait(ctx));
      cudaFree(s.kvhl);
      s.kvhl = nullptr;
      s.kvhl_bytes = 0;
      PB_TRY_CUDA(ctx, cudaMalloc(&s.kvhl, need));
      s.kvhl_bytes = need;
    }
    khl = s.kvhl;
    vhl = s.kvhl + (size_t)b->B * hl_stride;
  }
  {
    const int tot = (p.n_heads + p.n_kv_heads) * (hd / 2) + kvl, rpc = rope_rows_per_cta(rows);
    PB_TRY(pb_launch(ctx, "k_rope_kv", true, k_rope_kv, dim3(pb_cdiv(tot, 128), pb_cdiv(rows, rpc)), dim3(128), 0,
                     s.qkvo, qw, (const float*)(s.qkvo + p.n_heads * hd), qw,
                     (const float*)(s.qkvo + (p.n_heads + p.n_kv_heads) * hd), qw, p.n_heads, p.n_kv_heads, hd,
                     (const double2*)m->rope_tab, start_pos, pos_dev, kc, vc, c.seq_len, rows_per_seq, cache_seq,
                     ctx->d_err, rows, rpc, khl, vhl, kv_hl ? hl_stride : (int64_t)0));
  }
  float* att = s.att + (size_t)s.rank * rows * dc;
  pb_seq_geo geo;
  geo.kv = cache_seq;
  if (rows_per_seq == 1 && pos_dev) {
    geo.q = qw;
    geo.out = dc;
    __half* att16 = d16 ? reinterpret_cast<__half*>(s.att) + (size_t)s.rank * rows * dc * op_halves(b) : nullptr;
    return pb_launch_attn_decode(ctx, s.qkvo, kc, vc, pos_dev, p.n_heads, p.n_kv_heads, hd, att, c.seq_len, b->B, geo,
                                 b->ws, b->ws_bytes / 4, b->attn_cnt, att16, b->terms == 3);
  }
  geo.q = (int64_t)rows_per_seq * qw;
  geo.out = (int64_t)rows_per_seq * dc;
  if (hd == 64 && !pos_dev)
    return pb_launch_attn_prefill(ctx, s.qkvo, qw, kc, vc, rows_per_seq, start_pos, p.n_heads, p.n_kv_heads, hd, att,
                                  b->B, geo, b->terms, khl, vhl, hl_stride,
                                  att_hl_prefill(b, s, l, rows) ? reinterpret_cast<__half*>(att) : nullptr);
  return pb_launch_attn_cached(ctx, s.qkvo, qw, kc, vc, rows_per_seq, start_pos, pos_dev, p.n_heads, p.n_kv_heads, hd,
                               att, c.seq_len, b->B, geo);
}

// this rank's rows of wo with the residual add into its chunk of x
// (llama-streaming.js:579-580)
// One process holding the whole model (no row split): a residual GEMM (wo,
// down) also runs the RMSNorm that comes next (pb_gemm_epi::norm_w), into
// the operand the next GEMM reads; its split-K reduce and the norm are then
// one kernel.  The same bits as the norm launched by the next phase.
static bool norm_in_gemm(const pb_batch* b) { return b->world == 1 && b->sh.size() == 1; }

static void set_norm(pb_batch* b, pb_shard& s, pb_gemm_epi& e, const float* w, bool f16) {
  e.norm_w = w;
  e.norm_eps = b->m->c.eps;
  e.norm_out = f16 ? nullptr : s.xn;
  e.norm_out16 = f16 ? reinterpret_cast<__half*>(s.xn) : nullptr;
  e.norm_hl = f16 && b->terms == 3;
}

static int shard_wo(pb_batch* b, pb_shard& s, int l, int rows, bool send_x = false, bool norm_next = false) {
  pb_model* m = b->m;
  const int dc = s.p.dim_chunk;
  pb_gemm_epi add;
  add.mode = PB_GEMM_ADD;
  add.x_chunk = chunk_of(b, dc);
  add.split_n = m->c.dim;
  add.terms = b->terms;
  if (send_x) add.xs = xsend_of(b, dc);
  if (norm_next)  // the FFN norm, into the gate|up GEMM's operand
    set_norm(b, s, add, m->rms_ffn + (size_t)l * m->c.dim, pb_gemm_uses_tma(s.gu[l], rows) || dec16(b, s, l, rows));
  if (dec16(b, s, l, rows) || att_hl_prefill(b, s, l, rows))  // the attention wrote hi/lo pairs
    return pb_launch_q4_gemm(m->ctx, s.wo[l], nullptr, m->c.dim, rows, s.x + (size_t)s.rank * rows * dc, dc, b->ws,
                             b->ws_bytes, &add, reinterpret_cast<const __half*>(s.att));
  return pb_launch_q4_gemm(m->ctx, s.wo[l], s.att, m->c.dim, rows, s.x + (size_t)s.rank * rows * dc, dc, b->ws,
                           b->ws_bytes, &add);
}

static bool hidden_f16(const pb_batch* b, const pb_shard& s, int l, int rows) {
  return pb_gemm_uses_tma(s.w2[l], rows) || dec16(b, s, l, rows);
}

// norm -> this rank's gate|up rows with SwiGLU in the epilogue, h into its
// chunk of hb (f16 for the TMA path of w2, f32 otherwise)
static int shard_gate_up(pb_batch* b, pb_shard& s, int l, int rows, bool recv_x = false, bool normed = false) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const int dim = m->c.dim, fc = s.p.hidden_chunk;
  const bool gu16 = pb_gemm_uses_tma(s.gu[l], rows) || dec16(b, s, l, rows);
  __half* xn16 = reinterpret_cast<__half*>(s.xn);
  if (recv_x)  // x's other chunks arrive with the norm (fused exchange)
    PB_TRY(pb_launch_rmsnorm_xrecv(ctx, s.x, rows, dim, m->rms_ffn + (size_t)l * dim, m->c.eps, gu16 ? nullptr : s.xn,
                                   gu16 ? xn16 : nullptr, s.p.dim_chunk, gu16 && b->terms == 3, xrecv_of(b)));
  else if (!normed)  // (normed: the wo GEMM ran this norm)
    PB_TRY(launch_norm(m, s.x, rows, m->rms_ffn + (size_t)l * dim, gu16 ? nullptr : s.xn, gu16 ? xn16 : nullptr,
                       s.p.dim_chunk, b->terms == 3));
  pb_gemm_epi glu;
  glu.mode = PB_GEMM_SWIGLU;
  glu.split_n = 2 * m->c.hidden_dim;
  glu.terms = b->terms;
  const size_t off = (size_t)s.rank * rows * fc * (hidden_f16(b, s, l, rows) ? op_halves(b) : 1);
  if (hidden_f16(b, s, l, rows)) glu.h16 = reinterpret_cast<__half*>(s.hb) + off;
  else glu.h32 = s.hb + off;
  if (gu16) return pb_launch_q4_gemm(ctx, s.gu[l], nullptr, dim, rows, nullptr, 2 * fc, b->ws, b->ws_bytes, &glu, xn16);
  return pb_launch_q4_gemm(ctx, s.gu[l], s.xn, dim, rows, nullptr, 2 * fc, b->ws, b->ws_bytes, &glu);
}

// this rank's rows of w2 with the residual add into its chunk of x (:601)
static int shard_down(pb_batch* b, pb_shard& s, int l, int rows, bool send_x = false, bool norm_next = false) {
  pb_model* m = b->m;
  const int F = m->c.hidden_dim, dc = s.p.dim_chunk;
  pb_gemm_epi add;
  add.mode = PB_GEMM_ADD;
  add.x_chunk = chunk_of(b, s.p.hidden_chunk);
  add.split_n = m->c.dim;
  add.terms = b->terms;
  if (send_x) add.xs = xsend_of(b, dc);
  if (norm_next)  // the next layer's attention norm, into its qkv GEMM's operand
    set_norm(b, s, add, m->rms_att + (size_t)(l + 1) * m->c.dim,
             pb_gemm_uses_tma(s.qkv[l + 1], rows) || dec16(b, s, l + 1, rows));
  float* C = s.x + (size_t)s.rank * rows * dc;
  if (hidden_f16(b, s, l, rows))
    return pb_launch_q4_gemm(m->ctx, s.w2[l], nullptr, F, rows, C, dc, b->ws, b->ws_bytes, &add,
                             reinterpret_cast<const __half*>(s.hb));
  return pb_launch_q4_gemm(m->ctx, s.w2[l], s.hb, F, rows, C, dc, b->ws, b->ws_bytes, &add);
}

// One layer over `rows` token rows: n_seqs sequences of rows_per_seq rows each,
// at positions start (or *pos_dev) + row-in-sequence.  Each phase runs on
// every shard of this process, then the all-gather that the next phase needs.
static int batch_layer(pb_batch* b, int l, int rows, int rows_per_seq, int start_pos, const int* pos_dev) {
  const pb_model_config& c = b->m->c;
  b->decoding = rows_per_seq == 1 && pos_dev != nullptr;
  const size_t dchunk = (size_t)rows * (c.dim / b->world) * 4;
  // f16 attention output (hi/lo pairs take the bytes of f32)
  const size_t achunk = dec16(b, b->sh[0], l, rows) ? dchunk / 2 * op_halves(b) : dchunk;
  // fused residual exchanges: the wo / down GEMMs send, the next norm receives
  const bool fx = fused_x(b, rows);
  // one process with the whole model: the residual GEMMs run the next norms
  const bool ng = !fx && norm_in_gemm(b);
  for (auto& s : b->sh)
    PB_TRY(shard_attention(b, s, l, rows, rows_per_seq, start_pos, pos_dev, fx && l > 0, ng && l > 0));
  PB_TRY(batch_gather(b, XG_ATT, achunk));
  for (auto& s : b->sh) PB_TRY(shard_wo(b, s, l, rows, fx, ng));
  if (!fx) PB_TRY(batch_gather(b, XG_X, dchunk));
  for (auto& s : b->sh) PB_TRY(shard_gate_up(b, s, l, rows, fx, ng));
  const size_t hchunk =
      (size_t)rows * (c.hidden_dim / b->world) * (hidden_f16(b, b->sh[0], l, rows) ? 2 * op_halves(b) : 4);
  PB_TRY(batch_gather(b, XG_HB, hchunk));
  for (auto& s : b->sh) PB_TRY(shard_down(b, s, l, rows, fx, ng && l + 1 < c.n_layers));
  return fx ? PB_OK : batch_gather(b, XG_X, dchunk);
}

// Final RMSNorm of each sequence's last row (xl, or x itself when every row
// is a last row), the LM head as one GEMM over this rank's vocab rows, the
// greedy token of every sequence.
static int batch_head(pb_batch* b, bool from_x, const int* pos_dev) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  for (auto& s : b->sh) {
    const bool h16 = pb_gemm_uses_ws(s.head, b->B);
    __half* xn16 = h16 ? reinterpret_cast<__half*>(s.xn) : nullptr;
    const int hl = b->terms == 3;
    if (from_x && fused_x(b, b->B))  // the last layer's down GEMM sent its residual chunk
      PB_TRY(pb_launch_rmsnorm_xrecv(ctx, s.x, b->B, c.dim, m->rms_final, c.eps, h16 ? nullptr : s.xn, xn16,
                                     s.p.dim_chunk, h16 && hl, xrecv_of(b)));
    else if (from_x) PB_TRY(launch_norm(m, s.x, b->B, m->rms_final, h16 ? nullptr : s.xn, xn16, s.p.dim_chunk, hl));
    else PB_TRY(launch_norm(m, s.xl, b->B, m->rms_final, h16 ? nullptr : s.xn, xn16, 0, hl));
    const int vc = s.p.vocab_chunk;
    float* lg = s.logits + (size_t)s.rank * b->B * vc;
    pb_gemm_epi he;
    he.terms = b->terms;
    if (h16) PB_TRY(pb_launch_q4_gemm(ctx, s.head, nullptr, c.dim, b->B, lg, vc, nullptr, 0, &he, xn16));
    else PB_TRY(pb_launch_q4_gemm(ctx, s.head, s.xn, c.dim, b->B, lg, vc, nullptr, 0, &he));
    // this rank's keys (zero: cleared by the previous merge or at creation)
    PB_TRY(pb_launch(ctx, "k_argmax_chunks", true, k_argmax_chunks, dim3(pb_cdiv(s.p.vocab_rows, AMX_CHUNK), b->B),
                     dim3(256), 0, (const float*)lg, s.p.vocab_rows, vc, s.p.vocab_row0,
                     s.keys + (size_t)s.rank * b->B));
  }
  PB_TRY(batch_gather(b, XG_KEYS, (size_t)b->B * 8));
  for (auto& s : b->sh) {  // every shard reads the gathered keys and clears its own for the next step
    const bool first = &s == &b->sh[0];
    k_argmax_merge<<<pb_cdiv(b->B, 128), 128, 0, ctx->stream>>>(
        s.keys, b->world, b->B, first ? b->next : nullptr, first ? b->hist : nullptr, pos_dev, c.seq_len + 1,
        s.keys + (size_t)s.rank * b->B);
    PB_LAUNCHED(ctx, "k_argmax_merge");
  }
  return PB_OK;
}

// Embedding of `rows` tokens into every shard's x.
static int batch_embed(pb_batch* b, const int* toks, int rows) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  for (auto& s : b->sh) {
    k_batch_embed<<<dim3(pb_cdiv(c.dim, 256), rows), 256, 0, ctx->stream>>>(
        m->emb->type, m->emb->qs, m->emb->d, c.vocab, c.dim, toks, s.x, s.p.dim_chunk, rows, ctx->d_err);
    PB_LAUNCHED(ctx, "k_batch_embed");
  }
  return PB_OK;
}

// Every rank's logits [B][vocab] to the host (an all-gather of the chunks
// first across processes).
static int batch_logits_to_host(pb_batch* b, float* host) {
  pb_ctx* ctx = b->m->ctx;
  const pb_model_config& c = b->m->c;
  const int vc = b->sh[0].p.vocab_chunk;
  if (b->comm) PB_TRY(batch_gather(b, XG_LOGITS, (size_t)b->B * vc * 4));
  for (int r = 0; r < b->world; ++r) {
    const pb_shard& s = b->comm ? b->sh[0] : b->sh[r];
    pb_split_plan p;
    PB_TRY(pb_batch_split_plan(&c, b->world, r, &p));
    PB_TRY_CUDA(ctx, cudaMemcpy2DAsync(host + p.vocab_row0, (size_t)c.vocab * 4, s.logits + (size_t)r * b->B * vc,
                                       (size_t)vc * 4, (size_t)p.vocab_rows * 4, b->B, cudaMemcpyDeviceToHost,
                                       ctx->stream));
  }
  return PB_OK;
}

extern "C" int pb_batch_prefill(pb_batch* b, const int* tokens_host, int n_prompt, int* next_host,
                                float* logits_host) {
  if (!b || !tokens_host || n_prompt <= 0) return PB_ERR_ARG;
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  if (n_prompt >= c.seq_len) return pb_set_error(ctx, PB_ERR_ARG, "prompt of %d tokens fills the cache", n_prompt);
  const int rows = b->B * n_prompt;
  PB_TRY(batch_ensure_rows(b, rows));
  b->P = n_prompt;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(b->toks, tokens_host, (size_t)rows * 4, cudaMemcpyHostToDevice, ctx->stream));
  PB_TRY(batch_embed(b, b->toks, rows));
  for (int l = 0; l < c.n_layers; ++l) PB_TRY(batch_layer(b, l, rows, n_prompt, 0, nullptr));
  for (auto& s : b->sh) {
    k_gather_last<<<dim3(pb_cdiv(c.dim, 256), b->B), 256, 0, ctx->stream>>>(s.x, n_prompt, c.dim, s.p.dim_chunk, rows,
                                                                            s.xl);
    PB_LAUNCHED(ctx, "k_gather_last");
  }
  // the greedy token after the prompt is recorded at position n_prompt - 1
  const int last = n_prompt - 1;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(b->pos_dev, &last, 4, cudaMemcpyHostToDevice, ctx->stream));
  PB_TRY(batch_head(b, false, b->pos_dev));
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(b->pos_dev, &n_prompt, 4, cudaMemcpyHostToDevice, ctx->stream));
  if (next_host)
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(next_host, b->next, (size_t)b->B * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (logits_host) PB_TRY(batch_logits_to_host(b, logits_host));
  return pb_wait(ctx);
}

// One decode step for every sequence: the tokens are the previous greedy
// tokens (b->next), the position is *pos_dev (advanced at the end).
static int batch_enqueue_step(pb_batch* b) {
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  PB_TRY(batch_embed(b, b->next, b->B));
  for (int l = 0; l < c.n_layers; ++l) PB_TRY(batch_layer(b, l, b->B, 1, 0, b->pos_dev));
  PB_TRY(batch_head(b, true, b->pos_dev));
  k_batch_step_end<<<1, 32, 0, ctx->stream>>>(b->pos_dev);
  PB_LAUNCHED(ctx, "k_batch_step_end");
  return PB_OK;
}

extern "C" int pb_batch_decode(pb_batch* b, int steps, int* tokens_host, float* logits_host) {
  if (!b || steps <= 0) return PB_ERR_ARG;
  pb_model* m = b->m;
  pb_ctx* ctx = m->ctx;
  const pb_model_config& c = m->c;
  if (b->P <= 0) return pb_set_error(ctx, PB_ERR_STATE, "pb_batch_decode before pb_batch_prefill");
  int pos = 0;
  PB_TRY_CUDA(ctx, cudaMemcpyAsync(&pos, b->pos_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
  PB_TRY(pb_wait(ctx));
  if (pos + steps > c.seq_len)
    return pb_set_error(ctx, PB_ERR_ARG, "%d steps from position %d overflow the cache", steps, pos);
  PB_TRY(batch_ensure_rows(b, b->B));
  if (!b->exec) {
    PB_TRY_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    int rc = batch_enqueue_step(b);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (rc != PB_OK) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return pb_cuda_error(ctx, e, "batch decode capture");
    e = cudaGraphInstantiate(&b->exec, g, 0);
    if (e != cudaSuccess) { cudaGraphDestroy(g); return pb_cuda_error(ctx, e, "batch decode instantiate"); }
    b->graph = g;
  }
  for (int i = 0; i < steps; ++i) PB_TRY_CUDA(ctx, cudaGraphLaunch(b->exec, ctx->stream));
  if (tokens_host)
    PB_TRY_CUDA(ctx, cudaMemcpyAsync(tokens_host, b->hist + (size_t)pos * b->B, (size_t)steps * b->B * 4,
                                     cudaMemcpyDeviceToHost, ctx->stream));
  if (logits_host) PB_TRY(batch_logits_to_host(b, logits_host));
  return pb_wait(ctx);
}
