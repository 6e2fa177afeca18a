// GGUF model files on the host: header, metadata, tensor index, raw tensor
// reads (gguf.js:76-194 GGUFParser, streaming-loader.js:35-87 parseHeader,
// :245-262 loadTensorRaw), config extraction (gguf.js:402-424 extractConfig)
// and the load of a whole model into device-resident packed weights
// (streaming-loader.js:119-162 caches every tensor's raw bytes once; here the
// bytes go straight to the device layout instead).
//
// Host code only; no kernels.  Errors are returned as PB_ERR_* codes with a
// message kept per thread (pb_gguf_last_error), since a file is parsed before
// any context exists.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "pb_internal.cuh"

namespace {

// GGUF metadata value types (gguf.js:24-27)
enum : uint32_t {
  GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7,
  GT_STRING = 8, GT_ARRAY = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};

// ggml tensor types and their block geometry (gguf.js:30-51)
struct TypeSize { uint32_t type, block, bytes; };
const TypeSize kTypeSizes[] = {{0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {8, 32, 34},
                               {9, 32, 36},   {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
                               {14, 256, 210}, {15, 256, 292}};

const TypeSize* type_size(uint32_t t) {
  for (const auto& s : kTypeSizes)
    if (s.type == t) return &s;
  return nullptr;
}

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

struct Meta {
  std::string key;
  uint32_t type = 0;      // GT_*
  uint32_t arr_type = 0;  // element type of an array
  int64_t i = 0;          // integer / bool scalar
  double d = 0.0;         // any numeric scalar as a double
  std::string s;          // string scalar
  std::vector<std::string> as;  // string array
  std::vector<double> an;       // numeric array
};

struct TensorInfo {
  std::string name;
  std::vector<int64_t> dims;
  uint32_t type = 0;
  uint64_t rel = 0;    // offset inside the data section
  uint64_t off = 0;    // absolute file offset
  uint64_t bytes = 0;  // tensorByteSize (gguf.js:204-211)
};

// Little-endian reader over a FILE with a bounds check against the file size.
struct Reader {
  FILE* f;
  uint64_t size, pos = 0;
  bool ok = true;
  bool read(void* dst, uint64_t n) {
    if (!ok || pos + n > size || (n && fread(dst, 1, n, f) != n)) return ok = false;
    pos += n;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    read(&v, sizeof v);
    return v;
  }
  bool str(std::string& s) {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > size - pos) return ok = false;
    s.resize(n);
    return read(&s[0], n);
  }
};

// Smallest encoded size of one array element of GGUF value type t (0: not
// an element type).
uint64_t elem_min_bytes(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: case GT_STRING: return 8;
    default: return 0;
  }
}

bool scalar(Reader& r, uint32_t t, Meta& m) {
  switch (t) {
    case GT_U8: m.i = r.get<uint8_t>(); break;
    case GT_I8: m.i = r.get<int8_t>(); break;
    case GT_U16: m.i = r.get<uint16_t>(); break;
    case GT_I16: m.i = r.get<int16_t>(); break;
    case GT_U32: m.i = r.get<uint32_t>(); break;
    case GT_I32: m.i = r.get<int32_t>(); break;
    case GT_BOOL: m.i = r.get<uint8_t>() != 0; break;
    case GT_U64: m.i = (int64_t)r.get<uint64_t>(); m.d = (double)(uint64_t)m.i; return r.ok;
    case GT_I64: m.i = r.get<int64_t>(); break;
    case GT_F32: m.d = r.get<float>(); m.i = (int64_t)m.d; return r.ok;
    case GT_F64: m.d = r.get<double>(); m.i = (int64_t)m.d; return r.ok;
    case GT_STRING: return r.str(m.s);
    default: return false;
  }
  m.d = (double)m.i;
  return r.ok;
}

}  // namespace

struct pb_gguf {
  FILE* f = nullptr;
  uint32_t version = 0;
  uint64_t size = 0, alignment = 32, data_start = 0;
  std::vector<Meta> meta;
  std::vector<TensorInfo> tensors;
  const Meta* find(const char* key) const {
    for (const auto& m : meta)
      if (m.key == key) return &m;
    return nullptr;
  }
};

extern "C" const char* pb_gguf_last_error(void) { return g_err.c_str(); }

static int gguf_open(const char* path, pb_gguf** out) {
  if (!path || !out) return fail(PB_ERR_ARG, "pb_gguf_open: null argument");
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) return fail(PB_ERR_ARG, "cannot open %s", path);
  pb_gguf* g = new pb_gguf();
  g->f = f;
  fseeko(f, 0, SEEK_END);
  g->size = (uint64_t)ftello(f);
  fseeko(f, 0, SEEK_SET);
  Reader r{f, g->size};
  auto bad = [&](int code, const char* what) {
    const int rc = fail(code, "%s: %s (at byte %llu)", path, what, (unsigned long long)r.pos);
    fclose(f);
    delete g;
    return rc;
  };
  // header (gguf.js:146-157)
  const uint32_t magic = r.get<uint32_t>();
  if (!r.ok || magic != 0x46554747u) return bad(PB_ERR_ARG, "not a GGUF file (bad magic)");
  g->version = r.get<uint32_t>();
  if (!r.ok || g->version < 2 || g->version > 3) return bad(PB_ERR_ARG, "unsupported GGUF version (supports v2-v3)");
  const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  // every metadata entry takes at least 13 bytes (key length, type, one value
  // byte) and every tensor entry 32, so the counts cannot exceed what is left
  if (!r.ok || n_tensors > (r.size - r.pos) / 32 || n_kv > (r.size - r.pos) / 13)
    return bad(PB_ERR_ARG, "bad tensor or metadata count");
  // metadata (gguf.js:159-167)
  g->meta.resize(n_kv);
  for (uint64_t i = 0; i < n_kv; ++i) {
    Meta& m = g->meta[i];
    if (!r.str(m.key)) return bad(PB_ERR_ARG, "truncated metadata key");
    m.type = r.get<uint32_t>();
    if (!r.ok) return bad(PB_ERR_ARG, "truncated metadata type");
    if (m.type == GT_ARRAY) {  // gguf.js:137-144
      m.arr_type = r.get<uint32_t>();
      const uint64_t n = r.get<uint64_t>();
      if (m.arr_type == GT_ARRAY) return bad(PB_ERR_ARG, "nested metadata arrays are not supported");
      // each element takes at least its encoded size (a string its 8-byte
      // length), so the count cannot exceed what is left of the file; this
      // keeps a corrupt count from asking for more host memory than the
      // file could describe
      const uint64_t esz = elem_min_bytes(m.arr_type);
      if (!r.ok || esz == 0 || n > (r.size - r.pos) / esz) return bad(PB_ERR_ARG, "bad metadata array");
      Meta e;
      if (m.arr_type == GT_STRING) {
        m.as.resize(n);
        for (uint64_t j = 0; j < n; ++j)
          if (!r.str(m.as[j])) return bad(PB_ERR_ARG, "truncated string array");
      } else {
        m.an.resize(n);
        for (uint64_t j = 0; j < n; ++j) {
          if (!scalar(r, m.arr_type, e)) return bad(PB_ERR_ARG, "bad metadata array element");
          m.an[j] = e.d;
        }
      }
    } else if (!scalar(r, m.type, m)) {
      return bad(PB_ERR_ARG, "unknown or truncated metadata value");
    }
  }
  // tensor index (gguf.js:169-183)
  g->tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    TensorInfo& t = g->tensors[i];
    if (!r.str(t.name)) return bad(PB_ERR_ARG, "truncated tensor name");
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd == 0 || nd > 4) return bad(PB_ERR_ARG, "bad tensor rank");
    t.dims.resize(nd);
    for (uint32_t d = 0; d < nd; ++d) t.dims[d] = (int64_t)r.get<uint64_t>();
    t.type = r.get<uint32_t>();
    t.rel = r.get<uint64_t>();
    if (!r.ok) return bad(PB_ERR_ARG, "truncated tensor info");
  }
  // data section start, aligned (streaming-loader.js:61-62)
  if (const Meta* a = g->find("general.alignment"))
    if (a->type != GT_STRING && a->type != GT_ARRAY && a->i > 0) {
      if (a->i > (1 << 20)) return bad(PB_ERR_ARG, "general.alignment out of range");
      g->alignment = (uint64_t)a->i;
    }
  g->data_start = (r.pos + g->alignment - 1) / g->alignment * g->alignment;
  for (auto& t : g->tensors) {
    int64_t n = 1;
    for (int64_t d : t.dims) {
      if (d <= 0) return bad(PB_ERR_ARG, "non-positive tensor dimension");
      if (__builtin_mul_overflow(n, d, &n) || n > ((int64_t)1 << 50))
        return bad(PB_ERR_ARG, "tensor element count out of range");
    }
    const TypeSize* ts = type_size(t.type);
    t.bytes = ts ? (ts->block == 1 ? (uint64_t)n * ts->bytes : (uint64_t)((n + ts->block - 1) / ts->block) * ts->bytes)
                 : 0;
    if (t.rel > g->size) {
      std::string what = "tensor " + t.name + " starts past the end of the file";
      return bad(PB_ERR_ARG, what.c_str());
    }
    t.off = g->data_start + t.rel;
    if (ts && (t.bytes > g->size || t.off > g->size - t.bytes)) {
      std::string what = "tensor " + t.name + " runs past the end of the file";
      return bad(PB_ERR_ARG, what.c_str());
    }
  }
  *out = g;
  return PB_OK;
}

// No C++ exception may cross the C ABI: a host allocation that fails while
// parsing becomes an error status.
extern "C" int pb_gguf_open(const char* path, pb_gguf** out) {
  try {
    return gguf_open(path, out);
  } catch (const std::bad_alloc&) {
    return fail(PB_ERR_OOM, "%s: out of host memory while parsing", path ? path : "(null)");
  } catch (const std::exception& e) {
    return fail(PB_ERR_ARG, "%s: %s", path ? path : "(null)", e.what());
  }
}

extern "C" int pb_gguf_close(pb_gguf* g) {
  if (!g) return PB_OK;
  if (g->f) fclose(g->f);
  delete g;
  return PB_OK;
}

extern "C" int pb_gguf_version(const pb_gguf* g) { return g ? (int)g->version : 0; }
extern "C" int64_t pb_gguf_data_start(const pb_gguf* g) { return g ? (int64_t)g->data_start : -1; }
extern "C" int64_t pb_gguf_alignment(const pb_gguf* g) { return g ? (int64_t)g->alignment : -1; }
extern "C" int pb_gguf_meta_count(const pb_gguf* g) { return g ? (int)g->meta.size() : 0; }

extern "C" int pb_gguf_meta_find(const pb_gguf* g, const char* key) {
  if (!g || !key) return -1;
  for (size_t i = 0; i < g->meta.size(); ++i)
    if (g->meta[i].key == key) return (int)i;
  return -1;
}

static const Meta* meta_at(const pb_gguf* g, int i) {
  return g && i >= 0 && (size_t)i < g->meta.size() ? &g->meta[i] : nullptr;
}

extern "C" int pb_gguf_meta_key(const pb_gguf* g, int i, const char** key) {
  const Meta* m = meta_at(g, i);
  if (!m || !key) return fail(PB_ERR_ARG, "metadata index %d out of range", i);
  *key = m->key.c_str();
  return PB_OK;
}

extern "C" int pb_gguf_meta_type(const pb_gguf* g, int i, int* type, int* arr_type, int64_t* arr_len) {
  const Meta* m = meta_at(g, i);
  if (!m) return fail(PB_ERR_ARG, "metadata index %d out of range", i);
  if (type) *type = (int)m->type;
  if (arr_type) *arr_type = (int)m->arr_type;
  if (arr_len) *arr_len = m->type == GT_ARRAY ? (int64_t)(m->arr_type == GT_STRING ? m->as.size() : m->an.size()) : 0;
  return PB_OK;
}

extern "C" int pb_gguf_meta_int(const pb_gguf* g, int i, int64_t* v) {
  const Meta* m = meta_at(g, i);
  if (!m || !v) return fail(PB_ERR_ARG, "metadata index %d out of range", i);
  if (m->type == GT_STRING || m->type == GT_ARRAY || m->type == GT_F32 || m->type == GT_F64)
    return fail(PB_ERR_ARG, "metadata %s is not an integer", m->key.c_str());
  *v = m->i;
  return PB_OK;
}

extern "C" int pb_gguf_meta_float(const pb_gguf* g, int i, double* v) {
  const Meta* m = meta_at(g, i);
  if (!m || !v) return fail(PB_ERR_ARG, "metadata index %d out of range", i);
  if (m->type == GT_STRING || m->type == GT_ARRAY) return fail(PB_ERR_ARG, "metadata %s is not a number", m->key.c_str());
  *v = m->d;
  return PB_OK;
}

extern "C" int pb_gguf_meta_string(const pb_gguf* g, int i, const char** s, int64_t* len) {
  const Meta* m = meta_at(g, i);
  if (!m || !s) return fail(PB_ERR_ARG, "metadata index %d out of range", i);
  if (m->type != GT_STRING) return fail(PB_ERR_ARG, "metadata %s is not a string", m->key.c_str());
  *s = m->s.data();
  if (len) *len = (int64_t)m->s.size();
  return PB_OK;
}

extern "C" int pb_gguf_meta_array_string(const pb_gguf* g, int i, int64_t j, const char** s, int64_t* len) {
  const Meta* m = meta_at(g, i);
  if (!m || !s || m->type != GT_ARRAY || m->arr_type != GT_STRING || j < 0 || (size_t)j >= m->as.size())
    return fail(PB_ERR_ARG, "no string element %lld in metadata %d", (long long)j, i);
  *s = m->as[j].data();
  if (len) *len = (int64_t)m->as[j].size();
  return PB_OK;
}

extern "C" int pb_gguf_meta_array_number(const pb_gguf* g, int i, int64_t j, double* v) {
  const Meta* m = meta_at(g, i);
  if (!m || !v || m->type != GT_ARRAY || m->arr_type == GT_STRING || j < 0 || (size_t)j >= m->an.size())
    return fail(PB_ERR_ARG, "no numeric element %lld in metadata %d", (long long)j, i);
  *v = m->an[j];
  return PB_OK;
}

extern "C" int pb_gguf_tensor_count(const pb_gguf* g) { return g ? (int)g->tensors.size() : 0; }

extern "C" int pb_gguf_tensor_find(const pb_gguf* g, const char* name) {
  if (!g || !name) return -1;
  for (size_t i = 0; i < g->tensors.size(); ++i)
    if (g->tensors[i].name == name) return (int)i;
  return -1;
}

extern "C" int pb_gguf_tensor_info(const pb_gguf* g, int i, const char** name, int* type, int* n_dims, int64_t* dims,
                                   int64_t* file_offset, int64_t* bytes) {
  if (!g || i < 0 || (size_t)i >= g->tensors.size()) return fail(PB_ERR_ARG, "tensor index %d out of range", i);
  const TensorInfo& t = g->tensors[i];
  if (name) *name = t.name.c_str();
  if (type) *type = (int)t.type;
  if (n_dims) *n_dims = (int)t.dims.size();
  if (dims)
    for (size_t d = 0; d < 4; ++d) dims[d] = d < t.dims.size() ? t.dims[d] : 1;
  if (file_offset) *file_offset = (int64_t)t.off;
  if (bytes) *bytes = (int64_t)t.bytes;
  return PB_OK;
}

// Raw bytes of tensor i (streaming-loader.js:245-262 loadTensorRaw).
extern "C" int pb_gguf_tensor_read(const pb_gguf* g, int i, void* host, size_t bytes) {
  if (!g || !host || i < 0 || (size_t)i >= g->tensors.size()) return fail(PB_ERR_ARG, "tensor index %d out of range", i);
  const TensorInfo& t = g->tensors[i];
  if (!type_size(t.type)) return fail(PB_ERR_ARG, "tensor %s has unsupported type %u", t.name.c_str(), t.type);
  if (bytes != t.bytes)
    return fail(PB_ERR_ARG, "tensor %s holds %llu bytes, got a buffer of %zu", t.name.c_str(),
                (unsigned long long)t.bytes, bytes);
  if (fseeko(g->f, (off_t)t.off, SEEK_SET) != 0 || fread(host, 1, bytes, g->f) != bytes)
    return fail(PB_ERR_ARG, "read of tensor %s failed", t.name.c_str());
  return PB_OK;
}

// extractConfig (gguf.js:402-424): `<arch>.<key>` with the reference's
// defaults (a missing or zero value takes the default, as JS `||` does),
// head_dim = floor(dim / heads), vocab = the tokenizer's token count
// (streaming-loader.js:57), else the embedding's row count.  kind and
// emb_type come from the tensor types: Q4_0 layer weights make a streaming
// model; its embedding is Q4_0 or Q8_0.
// Embedding / output tables of these ggml types are kept as a dequantized f32
// table (the reference dequantizes every table to f32 at load,
// streaming-loader.js:324-335); Q4_0 and Q8_0 stay quantized and are
// dequantized exactly inside the kernels.
static bool table_as_f32(uint32_t t) { return t == 0 || t == 1 || t == PB_TYPE_Q6_K; }

extern "C" int pb_gguf_config(const pb_gguf* g, pb_model_config* cfg) {
  if (!g || !cfg) return fail(PB_ERR_ARG, "pb_gguf_config: null argument");
  std::string arch = "llama";
  if (const Meta* a = g->find("general.architecture"))
    if (a->type == GT_STRING && !a->s.empty()) arch = a->s;
  auto num = [&](const char* key, double def) {
    const Meta* m = g->find((arch + "." + key).c_str());
    if (!m || m->type == GT_STRING || m->type == GT_ARRAY || m->d == 0.0) return def;
    return m->d;
  };
  memset(cfg, 0, sizeof *cfg);
  cfg->dim = (int)num("embedding_length", 0);
  cfg->hidden_dim = (int)num("feed_forward_length", 0);
  cfg->n_layers = (int)num("block_count", 0);
  cfg->n_heads = (int)num("attention.head_count", 0);
  cfg->n_kv_heads = (int)num("attention.head_count_kv", cfg->n_heads);
  cfg->seq_len = (int)num("context_length", 2048);
  cfg->eps = num("attention.layer_norm_rms_epsilon", 1e-5);
  cfg->rope_theta = num("rope.freq_base", 10000.0);
  if (cfg->dim <= 0 || cfg->hidden_dim <= 0 || cfg->n_layers <= 0 || cfg->n_heads <= 0)
    return fail(PB_ERR_ARG, "GGUF metadata lacks %s.embedding_length / feed_forward_length / block_count / "
                            "attention.head_count", arch.c_str());
  cfg->head_dim = cfg->dim / cfg->n_heads;
  const int emb = pb_gguf_tensor_find(g, "token_embd.weight");
  if (emb < 0) return fail(PB_ERR_ARG, "GGUF file has no token_embd.weight");
  const TensorInfo& e = g->tensors[emb];
  if (const Meta* tk = g->find("tokenizer.ggml.tokens"); tk && tk->type == GT_ARRAY && !tk->as.empty())
    cfg->vocab = (int)tk->as.size();
  else
    cfg->vocab = e.dims.size() > 1 ? (int)e.dims[1] : 0;
  cfg->kind = PB_MODEL_STREAMING_Q4;
  if (e.type == 2) cfg->emb_type = PB_TYPE_Q4_0;
  else if (e.type == 8) cfg->emb_type = PB_TYPE_Q8_0;
  else if (table_as_f32(e.type)) cfg->emb_type = PB_TYPE_F32;  // dequantized, as streaming-loader.js:324-335
  else
    return fail(PB_ERR_ARG, "token_embd.weight has ggml type %u; the device model takes Q4_0, Q8_0, Q6_K, F16 or F32",
                e.type);
  return PB_OK;
}

// ---------------------------------------------------------------------------
// whole-model load
// ---------------------------------------------------------------------------

// pb_model_set_tensor slot of a GGUF tensor name (gguf.js:376-404 mapTensorName).
static int tensor_slot(const std::string& n, int* layer) {
  *layer = 0;
  if (n == "token_embd.weight") return 0;
  if (n == "output_norm.weight") return 10;
  if (n == "output.weight") return 11;
  if (n.compare(0, 4, "blk.") != 0) return -1;
  const size_t dot = n.find('.', 4);
  if (dot == std::string::npos) return -1;
  *layer = atoi(n.substr(4, dot - 4).c_str());
  const std::string s = n.substr(dot + 1);
  static const char* names[] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                                "ffn_gate.weight", "ffn_down.weight", "ffn_up.weight", "attn_norm.weight",
                                "ffn_norm.weight"};
  for (int i = 0; i < 9; ++i)
    if (s == names[i]) return i + 1;
  return -1;
}

static void f16_to_f32(const uint16_t* src, float* dst, size_t n) {  // exact IEEE half decode (gguf.js:55-70)
  for (size_t i = 0; i < n; ++i) {
    const uint32_t h = src[i], s = (h >> 15) << 31, e = (h >> 10) & 31, f = h & 1023;
    uint32_t b;
    if (e == 0) {
      if (f == 0) {
        b = s;
      } else {  // subnormal: renormalise
        int ee = -1;
        uint32_t ff = f;
        do {
          ff <<= 1;
          ++ee;
        } while (!(ff & 1024));
        b = s | ((uint32_t)(127 - 15 - ee) << 23) | ((ff & 1023) << 13);
      }
    } else if (e == 31) {
      b = s | 0x7f800000u | (f << 13);
    } else {
      b = s | ((e + 112) << 23) | (f << 13);
    }
    memcpy(dst + i, &b, 4);
  }
}

extern "C" int pb_model_load_gguf(pb_ctx* ctx, const pb_gguf* g, int seq_len, pb_model** out) {
  if (!ctx || !g || !out) return PB_ERR_ARG;
  *out = nullptr;
  pb_model_config cfg;
  if (int rc = pb_gguf_config(g, &cfg)) return pb_set_error(ctx, rc, "%s", g_err.c_str());
  if (seq_len > 0) cfg.seq_len = seq_len;
  // every tensor the model needs, with the type and shape it must have
  const int nw = 1 + cfg.n_layers * 9 + 1;
  std::vector<int> found(nw, -1);
  int head = -1;
  for (size_t i = 0; i < g->tensors.size(); ++i) {
    int layer, w = tensor_slot(g->tensors[i].name, &layer);
    if (w < 0) continue;
    if (w == 11) { head = (int)i; continue; }
    if (w >= 1 && w <= 9 && (layer < 0 || layer >= cfg.n_layers)) continue;
    found[w == 0 ? 0 : w == 10 ? nw - 1 : 1 + layer * 9 + (w - 1)] = (int)i;
  }
  for (int k = 0; k < nw; ++k) {
    if (found[k] >= 0) continue;
    const int l = (k - 1) / 9, w = (k - 1) % 9 + 1;
    return pb_set_error(ctx, PB_ERR_ARG, "GGUF file lacks %s", k == 0 ? "token_embd.weight" : k == nw - 1 ?
                        "output_norm.weight" : (std::string("blk.") + std::to_string(l) + " tensor " +
                                                std::to_string(w)).c_str());
  }
  for (int k = 1; k < nw - 1; ++k) {
    const TensorInfo& t = g->tensors[found[k]];
    const int w = (k - 1) % 9 + 1;
    const bool norm = w >= 8;
    if (norm ? (t.type != 0 && t.type != 1) : t.type != 2)
      return pb_set_error(ctx, PB_ERR_ARG, "%s has ggml type %u; the device model takes Q4_0 weights and F32/F16 norms",
                          t.name.c_str(), t.type);
  }
  const uint32_t ht = head >= 0 ? g->tensors[head].type : 2;
  if (head >= 0 && ht != 2 && ht != 8 && !table_as_f32(ht))
    return pb_set_error(ctx, PB_ERR_ARG, "output.weight has ggml type %u; the head takes Q4_0, Q8_0, Q6_K, F16 or F32",
                        ht);
  const int64_t n_table = (int64_t)cfg.vocab * cfg.dim;
  for (int ti : {found[0], head}) {
    if (ti < 0) continue;
    int64_t n = 1;
    for (int64_t d : g->tensors[ti].dims) n *= d;
    if (n != n_table)
      return pb_set_error(ctx, PB_ERR_ARG, "%s holds %lld values; vocab x dim is %lld", g->tensors[ti].name.c_str(),
                          (long long)n, (long long)n_table);
  }
  pb_model* m = nullptr;
  PB_TRY(pb_model_create(ctx, &cfg, &m));
  int rc = PB_OK;
  if (head >= 0) rc = pb_model_attach_head(m, ht == 2 ? PB_TYPE_Q4_0 : ht == 8 ? PB_TYPE_Q8_0 : PB_TYPE_F32);
  std::vector<char> buf;
  std::vector<float> f32;
  // a table kept as f32: decoded on the device (pb_gguf_dequant, gguf.js:219-355)
  auto dequant_table = [&](const TensorInfo& t) -> int {
    void* raw_dev = nullptr;
    float* out_dev = nullptr;
    int r = PB_OK;
    if (cudaMalloc(&raw_dev, t.bytes) != cudaSuccess || cudaMalloc(&out_dev, (size_t)n_table * 4) != cudaSuccess)
      r = pb_set_error(ctx, PB_ERR_OOM, "decoding %s", t.name.c_str());
    if (r == PB_OK) r = pb_upload(ctx, raw_dev, buf.data(), t.bytes);
    if (r == PB_OK) r = pb_gguf_dequant(ctx, (int)t.type, raw_dev, n_table, out_dev);
    if (r == PB_OK) {
      f32.resize((size_t)n_table);
      r = pb_download(ctx, f32.data(), out_dev, (size_t)n_table * 4);
    }
    cudaFree(raw_dev);
    cudaFree(out_dev);
    return r;
  };
  auto load = [&](int ti, int layer, int w) -> int {
    const TensorInfo& t = g->tensors[ti];
    buf.resize(t.bytes);
    if (pb_gguf_tensor_read(g, ti, buf.data(), t.bytes)) return pb_set_error(ctx, PB_ERR_ARG, "%s", g_err.c_str());
    if ((w == 0 || w == 11) && table_as_f32(t.type)) {
      if (int r = dequant_table(t)) return r;
      return pb_model_set_tensor(m, layer, w, f32.data(), f32.size() * 4);
    }
    if (w >= 8 && w <= 10 && t.type == 1) {  // F16 norm gains -> f32
      f32.resize(t.bytes / 2);
      f16_to_f32(reinterpret_cast<const uint16_t*>(buf.data()), f32.data(), f32.size());
      return pb_model_set_tensor(m, layer, w, f32.data(), f32.size() * 4);
    }
    return pb_model_set_tensor(m, layer, w, buf.data(), t.bytes);
  };
  for (int k = 0; k < nw && rc == PB_OK; ++k) {
    const int w = k == 0 ? 0 : k == nw - 1 ? 10 : (k - 1) % 9 + 1;
    rc = load(found[k], k == 0 || k == nw - 1 ? 0 : (k - 1) / 9, w);
  }
  if (rc == PB_OK && head >= 0) rc = load(head, 0, 11);
  if (rc != PB_OK) {
    pb_model_free(m);
    return rc;
  }
  *out = m;
  return PB_OK;
}
