// Host side of the reference's resident server over the C ABI: the GGUF
// reader, the model loader and the server's request semantics.
//
//   gqa_gguf_*     reads a GGUF v2/v3 file: header, metadata (every value type
//                  of the format; integer keys, general.alignment and
//                  tokenizer.ggml.tokens kept), the tensor table and the data
//                  start -- the information qwen_server.c gets from
//                  parse_gguf_tensors (:113-178) and load_tokenizer_tokens
//                  (:203-266).  Every length is checked against the file size.
//   gqa_model_*    uploads one model's tensors the way the server lays them
//                  out (:525-588): per layer W_qkv = attn_q | attn_k | attn_v
//                  rows and b_qkv = the three biases, W_o, the FFN weights and
//                  both norms; token_embd.weight; output_norm.weight; and
//                  output.weight, laid out for the head by gqa_lm_head_pack
//                  (Q6_K) or gqa_lm_head_q8_0_pack (Q8_0, the 0.5B model of
//                  generate_stream_05b.c:553-615), at the context's sizes.
//                  Tensor types and shapes are checked (the server trusts them).
//   gqa_session_*  SET_BASE / QUERY / RAW_QUERY / STATUS of the server
//                  (:770-1054) without the socket: the same validation, the
//                  same token-by-token prompt walk through the layers, the
//                  head on the last prompt token, greedy generation with the
//                  end-of-generation stop.  Each step is one replay of a CUDA
//                  graph built from the public entry points.
#include <cerrno>
#include <cstdint>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include "gqa.h"

namespace gqa {
int set_error(int code, const char* fmt, ...);
int ctx_block_model(const gqa_ctx* c);
int block_d_model(int model);
int block_d_ffn(int model);
}

namespace {

using gqa::set_error;

constexpr int kQ4Block = 18;
constexpr int kEogDefault[2] = {151643, 151645};  // <|endoftext|>, <|im_end|> (:1007-1008)

enum GgufType : uint32_t { kF32 = 0, kQ4_0 = 2, kQ8_0 = 8, kQ6_K = 14 };

// Bytes of n elements of a GGUF tensor type; 0 for a type this reader does
// not size.
unsigned long long type_bytes(uint32_t type, unsigned long long n) {
  switch (type) {
    case 0: return 4 * n;                  // F32
    case 1: return 2 * n;                  // F16
    case 2: return n / 32 * 18;            // Q4_0
    case 3: return n / 32 * 20;            // Q4_1
    case 6: return n / 32 * 22;            // Q5_0
    case 7: return n / 32 * 24;            // Q5_1
    case 8: return n / 32 * 34;            // Q8_0
    case 9: return n / 32 * 36;            // Q8_1
    case 10: return n / 256 * 84;          // Q2_K
    case 11: return n / 256 * 110;         // Q3_K
    case 12: return n / 256 * 144;         // Q4_K
    case 13: return n / 256 * 176;         // Q5_K
    case 14: return n / 256 * 210;         // Q6_K
    case 15: return n / 256 * 292;         // Q8_K
    case 30: return 2 * n;                 // BF16
    default: return 0;
  }
}

struct Tensor {
  std::string name;
  int n_dims = 0;
  long long ne[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  unsigned long long rel = 0, abs = 0, bytes = 0;
};

// pread-based cursor with every read checked against the file size.
class Reader {
 public:
  Reader(int fd, unsigned long long size) : fd_(fd), size_(size) {}
  bool read(void* dst, unsigned long long n) {
    if (n > size_ || pos_ > size_ - n) return false;
    unsigned char* p = static_cast<unsigned char*>(dst);
    unsigned long long left = n, at = pos_;
    while (left > 0) {
      const ssize_t r = pread(fd_, p, left, (off_t)at);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) return false;
      p += r;
      at += (unsigned long long)r;
      left -= (unsigned long long)r;
    }
    pos_ += n;
    return true;
  }
  bool skip(unsigned long long n) {
    if (n > size_ || pos_ > size_ - n) return false;
    pos_ += n;
    return true;
  }
  template <typename T>
  bool get(T& v) { return read(&v, sizeof(T)); }
  bool str(std::string& s) {
    uint64_t len = 0;
    if (!get(len) || len > size_ - pos_) return false;
    s.resize(len);
    return len == 0 || read(&s[0], len);
  }
  unsigned long long pos() const { return pos_; }

 private:
  int fd_;
  unsigned long long size_, pos_ = 0;
};

// Size of a scalar metadata value type; 0 for strings, arrays, unknown types.
int scalar_bytes(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;       // u8, i8, bool
    case 2: case 3: return 2;               // u16, i16
    case 4: case 5: case 6: return 4;       // u32, i32, f32
    case 10: case 11: case 12: return 8;    // u64, i64, f64
    default: return 0;
  }
}

bool is_integer_type(uint32_t t) { return t <= 5 || t == 7 || t == 10 || t == 11; }

long long integer_value(const unsigned char* b, uint32_t t) {
  switch (t) {
    case 0: case 7: return b[0];
    case 1: return (int8_t)b[0];
    case 2: { uint16_t v; memcpy(&v, b, 2); return v; }
    case 3: { int16_t v; memcpy(&v, b, 2); return v; }
    case 4: { uint32_t v; memcpy(&v, b, 4); return v; }
    case 5: { int32_t v; memcpy(&v, b, 4); return v; }
    case 10: { uint64_t v; memcpy(&v, b, 8); return (long long)v; }
    case 11: { int64_t v; memcpy(&v, b, 8); return v; }
    default: return 0;
  }
}

}  // namespace

struct gqa_gguf {
  int fd = -1;
  uint32_t version = 0;
  unsigned long long file_size = 0, alignment = 32, data_start = 0;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, int> by_name;
  std::unordered_map<std::string, long long> ints;
  std::vector<std::string> tokens;
};

namespace {

int gguf_fail(gqa_gguf* g, const char* what) {
  delete g;
  return set_error(GQA_ERR_INVALID_ARG, "GGUF: %s", what);
}

void fill_tensor(const Tensor& t, gqa_gguf_tensor* out) {
  out->name = t.name.c_str();
  out->n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) out->ne[d] = t.ne[d];
  out->type = (int)t.type;
  out->offset = t.abs;
  out->bytes = t.bytes;
}

}  // namespace

// ---------------------------------------------------------------------------
// Model: device copies of one model's weights
// ---------------------------------------------------------------------------
struct gqa_model_weights {
  int device = 0;
  int n_layers = 0, vocab = 0;
  std::vector<void*> allocs;  // every device allocation, freed together
  std::vector<gqa_block_weights> attn;
  std::vector<gqa_ffn_weights> ffn;
  void* token_embd = nullptr;
  float* gamma_output = nullptr;
  void* lm_head = nullptr;
  int lm_head_type = GQA_HEAD_Q6_K;
};

// ---------------------------------------------------------------------------
// Session: the server's state machine
// ---------------------------------------------------------------------------
struct gqa_session {
  gqa_ctx* ctx = nullptr;
  int t_max = 0, vocab = 0;
  std::vector<gqa_block_weights> attn;
  std::vector<gqa_ffn_weights> ffn;
  std::vector<gqa_layer_kv> kv;
  gqa_model model{};
  std::vector<int> eog;
  cudaStream_t stream = nullptr;
  float* state = nullptr;        // device [d_model]
  int* d_tok = nullptr;          // device: token in, pick out
  int* d_pos = nullptr;          // device: next position
  int* h_buf = nullptr;          // pinned: prompt tokens (t_max) + pick + position
  cudaGraphExec_t prompt_step = nullptr;  // embedding + layers + position advance
  cudaGraphExec_t token_step = nullptr;   // the same + head + pick
  int base_pos = 0;
  unsigned long long base_hash = 0;
  int base_generation = 0;
  int ready = 0;                 // memory_state READY
};

extern "C" {

int gqa_gguf_open(const char* path, gqa_gguf** out) {
  if (!path || !out) return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_open: null argument");
  *out = nullptr;
  gqa_gguf* g = new gqa_gguf();
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    const int e = errno;
    delete g;
    return set_error(GQA_ERR_INVALID_ARG, "GGUF: cannot open %s: %s", path, strerror(e));
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0) return gguf_fail(g, "fstat failed");
  g->file_size = (unsigned long long)st.st_size;
  Reader r(g->fd, g->file_size);
  uint32_t magic = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!r.get(magic) || magic != 0x46554747u) return gguf_fail(g, "bad magic (not a GGUF file)");
  if (!r.get(g->version) || (g->version != 2 && g->version != 3))
    return gguf_fail(g, "unsupported version (2 and 3 are read)");
  if (!r.get(n_tensors) || !r.get(n_kv)) return gguf_fail(g, "truncated header");
  // Every tensor info takes at least 8 + 4 + 8 + 4 + 8 bytes, every key-value
  // at least 8 + 4: counts beyond that are a corrupt header.
  if (n_tensors > g->file_size / 32 || n_kv > g->file_size / 12)
    return gguf_fail(g, "tensor or key count larger than the file");

  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key;
    uint32_t vt = 0;
    if (!r.str(key) || !r.get(vt)) return gguf_fail(g, "truncated metadata");
    if (const int nb = scalar_bytes(vt)) {
      unsigned char b[8];
      if (!r.read(b, nb)) return gguf_fail(g, "truncated metadata value");
      if (is_integer_type(vt)) g->ints[key] = integer_value(b, vt);
    } else if (vt == 8) {
      std::string v;
      if (!r.str(v)) return gguf_fail(g, "truncated metadata string");
    } else if (vt == 9) {
      uint32_t at = 0;
      uint64_t n = 0;
      if (!r.get(at) || !r.get(n)) return gguf_fail(g, "truncated metadata array");
      const bool want_tokens = key == "tokenizer.ggml.tokens" && at == 8;
      if (at == 8) {
        if (n > g->file_size / 8) return gguf_fail(g, "array longer than the file");
        if (want_tokens) g->tokens.resize(n);
        for (uint64_t a = 0; a < n; ++a) {
          std::string v;
          if (!r.str(v)) return gguf_fail(g, "truncated string array");
          if (want_tokens) g->tokens[a].swap(v);
        }
      } else if (const int nb = scalar_bytes(at)) {
        if (n > g->file_size / (unsigned)nb || !r.skip(n * (unsigned)nb))
          return gguf_fail(g, "truncated metadata array");
      } else {
        return gguf_fail(g, "array of an unknown or nested value type");
      }
    } else {
      return gguf_fail(g, "unknown metadata value type");
    }
  }
  auto al = g->ints.find("general.alignment");
  if (al != g->ints.end()) {
    if (al->second <= 0 || (al->second & (al->second - 1)))
      return gguf_fail(g, "general.alignment is not a power of two");
    g->alignment = (unsigned long long)al->second;
  }

  g->tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    Tensor& t = g->tensors[i];
    uint32_t nd = 0;
    if (!r.str(t.name) || !r.get(nd) || nd < 1 || nd > 4) return gguf_fail(g, "bad tensor info");
    t.n_dims = (int)nd;
    unsigned long long n = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t v = 0;
      if (!r.get(v) || v == 0 || v > (1ull << 40)) return gguf_fail(g, "bad tensor dimension");
      t.ne[d] = (long long)v;
      if (n > (1ull << 48) / v) return gguf_fail(g, "tensor too large");
      n *= v;
    }
    if (!r.get(t.type) || !r.get(t.rel)) return gguf_fail(g, "truncated tensor info");
    t.bytes = type_bytes(t.type, n);
    if (!g->by_name.emplace(t.name, (int)i).second) return gguf_fail(g, "duplicate tensor name");
  }
  g->data_start = (r.pos() + g->alignment - 1) / g->alignment * g->alignment;
  for (Tensor& t : g->tensors) {
    t.abs = g->data_start + t.rel;
    if (t.rel > g->file_size || t.abs > g->file_size || t.bytes > g->file_size - t.abs)
      return gguf_fail(g, ("tensor data past the end of the file: " + t.name).c_str());
  }
  *out = g;
  return GQA_OK;
}

int gqa_gguf_close(gqa_gguf* g) {
  if (!g) return GQA_OK;
  if (g->fd >= 0) close(g->fd);
  delete g;
  return GQA_OK;
}

int gqa_gguf_tensor_count(const gqa_gguf* g) { return g ? (int)g->tensors.size() : -1; }

int gqa_gguf_tensor_at(const gqa_gguf* g, int i, gqa_gguf_tensor* out) {
  if (!g || !out || i < 0 || i >= (int)g->tensors.size())
    return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_tensor_at: bad index %d", i);
  fill_tensor(g->tensors[i], out);
  return GQA_OK;
}

int gqa_gguf_find(const gqa_gguf* g, const char* name, gqa_gguf_tensor* out) {
  if (!g || !name || !out) return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_find: null argument");
  auto it = g->by_name.find(name);
  if (it == g->by_name.end()) return set_error(GQA_ERR_INVALID_ARG, "GGUF: tensor '%s' not found", name);
  fill_tensor(g->tensors[it->second], out);
  return GQA_OK;
}

int gqa_gguf_read(const gqa_gguf* g, const gqa_gguf_tensor* t, void* dst) {
  if (!g || !t || !dst) return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_read: null argument");
  if (t->bytes == 0 || t->offset > g->file_size || t->bytes > g->file_size - t->offset)
    return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_read: bad tensor range");
  Reader r(g->fd, g->file_size);
  if (!r.skip(t->offset) || !r.read(dst, t->bytes))
    return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_read: read failed");
  return GQA_OK;
}

int gqa_gguf_meta_int(const gqa_gguf* g, const char* key, long long* out) {
  if (!g || !key || !out) return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_meta_int: null argument");
  auto it = g->ints.find(key);
  if (it == g->ints.end())
    return set_error(GQA_ERR_INVALID_ARG, "GGUF: no integer metadata '%s'", key);
  *out = it->second;
  return GQA_OK;
}

int gqa_gguf_vocab_size(const gqa_gguf* g) { return g ? (int)g->tokens.size() : -1; }

int gqa_gguf_token_string(const gqa_gguf* g, int id, char* out, int cap) {
  if (!g || !out || cap < 1 || id < 0 || id >= (int)g->tokens.size())
    return set_error(GQA_ERR_INVALID_ARG, "gqa_gguf_token_string: bad id %d", id);
  const std::string& s = g->tokens[id];
  const size_t n = s.size() < (size_t)cap - 1 ? s.size() : (size_t)cap - 1;
  memcpy(out, s.data(), n);
  out[n] = '\0';
  return (int)s.size();
}

}  // extern "C"

namespace {

#define MODEL_CUDA(call)                                                                  \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return set_error(GQA_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));    \
  } while (0)

// Checks one tensor's type and leading dimensions (ne[0] = columns).
int expect(const gqa_gguf* g, const std::string& name, uint32_t type, long long ne0, long long ne1,
           gqa_gguf_tensor* t) {
  int rc = gqa_gguf_find(g, name.c_str(), t);
  if (rc != GQA_OK) return rc;
  const bool dims_ok = t->ne[0] == ne0 && (ne1 < 0 ? true : t->ne[1] == ne1) &&
                       t->ne[2] == 1 && t->ne[3] == 1 && (ne1 != 1 || t->n_dims == 1);
  if ((uint32_t)t->type != type || !dims_ok)
    return set_error(GQA_ERR_UNSUPPORTED,
                     "GGUF: %s is type %d [%lld x %lld], expected type %u [%lld x %lld]",
                     name.c_str(), t->type, t->ne[0], t->ne[1], type, ne0, ne1);
  return GQA_OK;
}

// File -> pinned staging -> device, in pieces of at most the staging size.
int upload(const gqa_gguf* g, const gqa_gguf_tensor& t, void* dst, void* stage, size_t stage_bytes) {
  unsigned long long done = 0;
  while (done < t.bytes) {
    const unsigned long long n = t.bytes - done < stage_bytes ? t.bytes - done : stage_bytes;
    gqa_gguf_tensor piece = t;
    piece.offset = t.offset + done;
    piece.bytes = n;
    int rc = gqa_gguf_read(g, &piece, stage);
    if (rc != GQA_OK) return rc;
    MODEL_CUDA(cudaMemcpy(static_cast<char*>(dst) + done, stage, n, cudaMemcpyHostToDevice));
    done += n;
  }
  return GQA_OK;
}

int model_alloc(gqa_model_weights* m, void** p, size_t bytes) {
  MODEL_CUDA(cudaMalloc(p, bytes));
  m->allocs.push_back(*p);
  return GQA_OK;
}

int load_impl(gqa_ctx* ctx, const gqa_gguf* g, int n_layers, gqa_model_weights* m, void* stage,
              size_t stage_bytes) {
  gqa_gguf_tensor t;
  int rc;
  // The sizes of the context's shape: Qwen2.5-1.5B (qwen_server.c:525-588) or
  // Qwen2.5-0.5B (generate_stream_05b.c:553-615).
  const int model = gqa::ctx_block_model(ctx);
  if (model < 0)
    return set_error(GQA_ERR_UNSUPPORTED,
                     "gqa_model_load: the context's shape has no built decoder sizes");
  const long long d_model = gqa::block_d_model(model), d_ffn = gqa::block_d_ffn(model);
  const long long d_kv = d_model / (model == 0 ? 6 : 7);  // n_heads_kv * head_dim
  const long long d_qkv = d_model + 2 * d_kv;
  // token_embd.weight: Q4_0 [d_model][vocab]; output.weight: Q6_K (1.5B) or
  // Q8_0 (0.5B) [d_model][vocab]
  if ((rc = expect(g, "token_embd.weight", kQ4_0, d_model, -1, &t)) != GQA_OK) return rc;
  m->vocab = (int)t.ne[1];
  if ((rc = model_alloc(m, &m->token_embd, t.bytes)) != GQA_OK) return rc;
  if ((rc = upload(g, t, m->token_embd, stage, stage_bytes)) != GQA_OK) return rc;
  if ((rc = expect(g, "output_norm.weight", kF32, d_model, 1, &t)) != GQA_OK) return rc;
  if ((rc = model_alloc(m, (void**)&m->gamma_output, t.bytes)) != GQA_OK) return rc;
  if ((rc = upload(g, t, m->gamma_output, stage, stage_bytes)) != GQA_OK) return rc;
  const bool q8 = model == 1;
  m->lm_head_type = q8 ? GQA_HEAD_Q8_0 : GQA_HEAD_Q6_K;
  if ((rc = expect(g, "output.weight", q8 ? kQ8_0 : kQ6_K, d_model, m->vocab, &t)) != GQA_OK)
    return rc;
  {
    void* raw = nullptr;
    MODEL_CUDA(cudaMalloc(&raw, t.bytes));
    rc = upload(g, t, raw, stage, stage_bytes);
    const long long packed =
        q8 ? gqa_lm_head_q8_0_packed_bytes(m->vocab) : gqa_lm_head_packed_bytes(m->vocab);
    if (rc == GQA_OK) rc = model_alloc(m, &m->lm_head, (size_t)packed);
    if (rc == GQA_OK)
      rc = q8 ? gqa_lm_head_q8_0_pack(ctx, nullptr, raw, m->vocab, m->lm_head)
              : gqa_lm_head_pack(ctx, nullptr, raw, m->vocab, m->lm_head);
    if (rc == GQA_OK && cudaDeviceSynchronize() != cudaSuccess)
      rc = set_error(GQA_ERR_CUDA, "LM head pack failed");
    cudaFree(raw);
    if (rc != GQA_OK) return rc;
  }

  const size_t q4_row = (size_t)(d_model / 32) * kQ4Block;
  const size_t q4_row_ffn = (size_t)(d_ffn / 32) * kQ4Block;
  for (int l = 0; l < n_layers; ++l) {
    const std::string b = "blk." + std::to_string(l) + ".";
    void *w_qkv, *b_qkv, *w_o, *g_attn, *w_gate, *w_up, *w_down, *g_ffn;
    if ((rc = model_alloc(m, &w_qkv, d_qkv * q4_row)) != GQA_OK ||
        (rc = model_alloc(m, &b_qkv, sizeof(float) * d_qkv)) != GQA_OK ||
        (rc = model_alloc(m, &w_o, d_model * q4_row)) != GQA_OK ||
        (rc = model_alloc(m, &g_attn, sizeof(float) * d_model)) != GQA_OK ||
        (rc = model_alloc(m, &w_gate, d_ffn * q4_row)) != GQA_OK ||
        (rc = model_alloc(m, &w_up, d_ffn * q4_row)) != GQA_OK ||
        (rc = model_alloc(m, &w_down, d_model * q4_row_ffn)) != GQA_OK ||
        (rc = model_alloc(m, &g_ffn, sizeof(float) * d_model)) != GQA_OK)
      return rc;
    struct Piece {
      const char* name;
      uint32_t type;
      long long ne0, ne1;
      void* dst;
    };
    // W_qkv = attn_q | attn_k | attn_v rows, b_qkv likewise (qwen_server.c:551-567,
    // generate_stream_05b.c:583-596)
    const Piece pieces[] = {
        {"attn_norm.weight", kF32, d_model, 1, g_attn},
        {"ffn_norm.weight", kF32, d_model, 1, g_ffn},
        {"attn_q.bias", kF32, d_model, 1, b_qkv},
        {"attn_k.bias", kF32, d_kv, 1, static_cast<float*>(b_qkv) + d_model},
        {"attn_v.bias", kF32, d_kv, 1, static_cast<float*>(b_qkv) + d_model + d_kv},
        {"attn_q.weight", kQ4_0, d_model, d_model, w_qkv},
        {"attn_k.weight", kQ4_0, d_model, d_kv, static_cast<char*>(w_qkv) + d_model * q4_row},
        {"attn_v.weight", kQ4_0, d_model, d_kv,
         static_cast<char*>(w_qkv) + (d_model + d_kv) * q4_row},
        {"attn_output.weight", kQ4_0, d_model, d_model, w_o},
        {"ffn_gate.weight", kQ4_0, d_model, d_ffn, w_gate},
        {"ffn_up.weight", kQ4_0, d_model, d_ffn, w_up},
        {"ffn_down.weight", kQ4_0, d_ffn, d_model, w_down},
    };
    for (const Piece& p : pieces) {
      if ((rc = expect(g, b + p.name, p.type, p.ne0, p.ne1, &t)) != GQA_OK) return rc;
      if ((rc = upload(g, t, p.dst, stage, stage_bytes)) != GQA_OK) return rc;
    }
    m->attn.push_back(gqa_block_weights{w_qkv, static_cast<const float*>(b_qkv), w_o,
                                        static_cast<const float*>(g_attn)});
    m->ffn.push_back(gqa_ffn_weights{w_gate, w_up, w_down, static_cast<const float*>(g_ffn)});
  }
  m->n_layers = n_layers;
  return GQA_OK;
}

}  // namespace

extern "C" {

int gqa_model_load(gqa_ctx* ctx, const gqa_gguf* g, int n_layers, gqa_model_weights** out) {
  if (!ctx || !g || !out) return set_error(GQA_ERR_INVALID_ARG, "gqa_model_load: null argument");
  *out = nullptr;
  if (n_layers <= 0) {
    long long bc = 0;
    if (gqa_gguf_meta_int(g, "qwen2.block_count", &bc) != GQA_OK || bc < 1 || bc > 1024)
      return set_error(GQA_ERR_INVALID_ARG,
                       "gqa_model_load: n_layers not given and no qwen2.block_count in the file");
    n_layers = (int)bc;
  }
  int dev = 0;
  MODEL_CUDA(cudaGetDevice(&dev));
  gqa_model_weights* m = new gqa_model_weights();
  m->device = dev;
  const size_t stage_bytes = 64u << 20;
  void* stage = nullptr;
  int rc = GQA_OK;
  if (cudaMallocHost(&stage, stage_bytes) != cudaSuccess)
    rc = set_error(GQA_ERR_NO_MEMORY, "gqa_model_load: no pinned staging buffer");
  if (rc == GQA_OK) rc = load_impl(ctx, g, n_layers, m, stage, stage_bytes);
  if (stage) cudaFreeHost(stage);
  if (rc != GQA_OK) {
    gqa_model_free(m);
    return rc;
  }
  *out = m;
  return GQA_OK;
}

int gqa_model_view(const gqa_model_weights* m, const gqa_layer_kv* kv, gqa_model* out) {
  if (!m || !out) return set_error(GQA_ERR_INVALID_ARG, "gqa_model_view: null argument");
  out->n_layers = m->n_layers;
  out->attn = m->attn.data();
  out->ffn = m->ffn.data();
  out->kv = kv;
  out->token_embd = m->token_embd;
  out->gamma_output = m->gamma_output;
  out->lm_head = m->lm_head;
  out->vocab = m->vocab;
  out->lm_head_type = m->lm_head_type;
  return GQA_OK;
}

int gqa_model_free(gqa_model_weights* m) {
  if (!m) return GQA_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != m->device) cudaSetDevice(m->device);
  for (void* p : m->allocs) cudaFree(p);
  if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
  delete m;
  return GQA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Session
// ---------------------------------------------------------------------------
namespace {

void session_release(gqa_session* s) {
  if (s->prompt_step) cudaGraphExecDestroy(s->prompt_step);
  if (s->token_step) cudaGraphExecDestroy(s->token_step);
  if (s->state) cudaFree(s->state);
  if (s->d_tok) cudaFree(s->d_tok);
  if (s->d_pos) cudaFree(s->d_pos);
  if (s->h_buf) cudaFreeHost(s->h_buf);
  if (s->stream) cudaStreamDestroy(s->stream);
}

// Captures `body` on the session's stream into an executable graph.
template <typename F>
int capture(gqa_session* s, F body, cudaGraphExec_t* out) {
  MODEL_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = body();
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
  if (rc != GQA_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_error(GQA_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
  const cudaError_t ie = cudaGraphInstantiate(out, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) return set_error(GQA_ERR_CUDA, "instantiate: %s", cudaGetErrorString(ie));
  return GQA_OK;
}

int check_device(gqa_session* s) {
  int status = 0;
  int rc = gqa_device_status(s->ctx, &status, 1);
  if (rc != GQA_OK) return rc;
  if (status) return set_error(GQA_ERR_DEVICE, "ERR_GPU_FAILURE (device status 0x%x)", status);
  return GQA_OK;
}

// Prompt tokens [0, n) through the layers at positions pos .. pos + n - 1,
// the last one with the head (its pick lands in d_tok) when `head` is set.
int run_prompt(gqa_session* s, const int* tokens, int n, int pos, bool head) {
  memcpy(s->h_buf, tokens, sizeof(int) * n);
  s->h_buf[s->t_max + 1] = pos;
  MODEL_CUDA(cudaMemcpyAsync(s->d_pos, s->h_buf + s->t_max + 1, sizeof(int),
                             cudaMemcpyHostToDevice, s->stream));
  for (int p = 0; p < n; ++p) {
    MODEL_CUDA(cudaMemcpyAsync(s->d_tok, s->h_buf + p, sizeof(int), cudaMemcpyHostToDevice,
                               s->stream));
    const bool last = head && p == n - 1;
    MODEL_CUDA(cudaGraphLaunch(last ? s->token_step : s->prompt_step, s->stream));
  }
  MODEL_CUDA(cudaStreamSynchronize(s->stream));
  return check_device(s);
}

bool valid_ids(const gqa_session* s, const int* tokens, int n) {
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= s->vocab) return false;
  return true;
}

}  // namespace

extern "C" {

int gqa_session_create(gqa_ctx* ctx, const gqa_model* model, int t_max, const int* eog_ids,
                       int n_eog, gqa_session** out) {
  if (!ctx || !model || !out || !model->kv || !model->attn || !model->ffn || model->n_layers < 1 ||
      t_max < 2 || n_eog < 0 || (n_eog > 0 && !eog_ids))
    return set_error(GQA_ERR_INVALID_ARG, "gqa_session_create: bad arguments");
  *out = nullptr;
  gqa_session* s = new gqa_session();
  s->ctx = ctx;
  s->t_max = t_max;
  s->vocab = model->vocab;
  s->attn.assign(model->attn, model->attn + model->n_layers);
  s->ffn.assign(model->ffn, model->ffn + model->n_layers);
  s->kv.assign(model->kv, model->kv + model->n_layers);
  s->model = *model;
  s->model.attn = s->attn.data();
  s->model.ffn = s->ffn.data();
  s->model.kv = s->kv.data();
  if (eog_ids) s->eog.assign(eog_ids, eog_ids + n_eog);
  else s->eog.assign(kEogDefault, kEogDefault + 2);
  int rc = GQA_OK;
  auto cu = [&](cudaError_t e, const char* what) {
    if (rc == GQA_OK && e != cudaSuccess)
      rc = set_error(GQA_ERR_CUDA, "gqa_session_create: %s: %s", what, cudaGetErrorString(e));
  };
  cu(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "stream");
  const int model_sizes = gqa::ctx_block_model(ctx);
  if (model_sizes < 0)
    rc = set_error(GQA_ERR_UNSUPPORTED, "gqa_session_create: the context's shape has no built "
                   "decoder sizes");
  cu(cudaMalloc(&s->state, sizeof(float) * (model_sizes < 0 ? 1 : gqa::block_d_model(model_sizes))),
     "state");
  cu(cudaMalloc(&s->d_tok, sizeof(int)), "token");
  cu(cudaMalloc(&s->d_pos, sizeof(int)), "position");
  cu(cudaMallocHost(&s->h_buf, sizeof(int) * ((size_t)t_max + 2)), "pinned buffer");
  if (rc == GQA_OK) rc = gqa_reserve(ctx, 1, t_max);
  // One prompt token: embedding, layers (position advanced); one generated
  // token: the same with the head and the pick (gqa_decode_token).
  if (rc == GQA_OK)
    rc = capture(s, [&] {
      int r = gqa_token_embedding(ctx, s->stream, s->model.token_embd, s->vocab, s->d_tok,
                                  s->state);
      if (r == GQA_OK)
        r = gqa_decoder_layers(ctx, s->stream, s->model.n_layers, s->model.attn, s->model.ffn,
                               s->model.kv, s->state, s->d_pos, 1, 0, 0);
      return r;
    }, &s->prompt_step);
  if (rc == GQA_OK)
    rc = capture(s, [&] {
      return gqa_decode_token(ctx, s->stream, &s->model, s->state, s->d_tok, s->d_pos, nullptr, 0,
                              0);
    }, &s->token_step);
  if (rc != GQA_OK) {
    session_release(s);
    delete s;
    return rc;
  }
  *out = s;
  return GQA_OK;
}

int gqa_session_destroy(gqa_session* s) {
  if (!s) return GQA_OK;
  cudaStreamSynchronize(s->stream);
  session_release(s);
  delete s;
  return GQA_OK;
}

int gqa_session_set_base(gqa_session* s, const int* tokens, int n) {
  if (!s) return set_error(GQA_ERR_INVALID_ARG, "null session");
  // Validation before any state changes (qwen_server.c:790-814)
  if (!tokens || n <= 0) return set_error(GQA_ERR_INVALID_ARG, "ERR_BAD_REQUEST");
  if (!valid_ids(s, tokens, n)) return set_error(GQA_ERR_INVALID_ARG, "ERR_INVALID_TOKEN");
  if (n + 1 >= s->t_max) return set_error(GQA_ERR_INVALID_ARG, "ERR_CONTEXT_FULL");
  s->ready = 0;  // REBUILDING
  unsigned long long hash = 14695981039346656037ull;  // FNV-1a over the ids (:821-822)
  for (int p = 0; p < n; ++p) {
    hash ^= (unsigned long long)(unsigned)tokens[p];
    hash *= 1099511628211ull;
  }
  const int rc = run_prompt(s, tokens, n, 0, false);
  if (rc != GQA_OK) {  // :843-852
    s->base_pos = 0;
    s->base_hash = 0;
    return rc;
  }
  s->base_pos = n;
  s->base_hash = hash;
  s->base_generation += 1;
  s->ready = 1;
  return GQA_OK;
}

int gqa_session_query(gqa_session* s, const int* tokens, int n, int max_new, int raw,
                      int* out_tokens, int* n_out) {
  if (!s || !n_out) return set_error(GQA_ERR_INVALID_ARG, "null session or count");
  *n_out = 0;
  // qwen_server.c:872-950: state, token ids, then the capacity checks
  if (raw && s->base_pos > 0 && s->ready)
    return set_error(GQA_ERR_INVALID_ARG, "ERR_RAW_NOT_ALLOWED_WHEN_BASE_ACTIVE");
  if (!raw && !s->ready) return set_error(GQA_ERR_INVALID_ARG, "ERR_NOT_READY");
  if (max_new <= 0 || max_new > s->t_max || !tokens || n <= 0 || !valid_ids(s, tokens, n))
    return set_error(GQA_ERR_INVALID_ARG, "ERR_INVALID_TOKEN");
  const int cur_pos = raw ? 0 : s->base_pos;
  if (n >= s->t_max || cur_pos + n >= s->t_max || cur_pos + n + max_new >= s->t_max)
    return set_error(GQA_ERR_INVALID_ARG, "ERR_CONTEXT_FULL");
  if (!out_tokens) return set_error(GQA_ERR_INVALID_ARG, "null output buffer");

  int rc = run_prompt(s, tokens, n, cur_pos, true);
  if (rc != GQA_OK) return rc;
  int next_pos = cur_pos + n;
  int* h_pick = s->h_buf + s->t_max;
  for (int gen = 0; gen < max_new; ++gen) {  // :997-1049
    MODEL_CUDA(cudaMemcpyAsync(h_pick, s->d_tok, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
    MODEL_CUDA(cudaStreamSynchronize(s->stream));
    const int best = *h_pick;
    bool eog = false;
    for (int e : s->eog) eog = eog || best == e;
    if (eog) break;
    out_tokens[(*n_out)++] = best;
    if (gen + 1 >= max_new || next_pos >= s->t_max) break;
    MODEL_CUDA(cudaGraphLaunch(s->token_step, s->stream));  // picks into d_tok, advances pos
    ++next_pos;
  }
  MODEL_CUDA(cudaStreamSynchronize(s->stream));
  return check_device(s);
}

int gqa_session_status(const gqa_session* s, int* base_pos, unsigned long long* base_hash,
                       int* base_generation, int* ready) {
  if (!s) return set_error(GQA_ERR_INVALID_ARG, "null session");
  if (base_pos) *base_pos = s->base_pos;
  if (base_hash) *base_hash = s->base_hash;
  if (base_generation) *base_generation = s->base_generation;
  if (ready) *ready = s->ready;
  return GQA_OK;
}

}  // extern "C"
