// CPU ORACLE — test infrastructure only.
//
// A C++ restatement of the reference's CPU path for the LFM2.5-8B-A1B Q6_K
// token loop (`lfm2-greedy --cpu --tokens`). It is the checker the B200 path
// is compared against; nothing in the product links or calls it. Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
//
// Followed files (reference project paths):
//   engine/src/q6k.rs        Q6_K block layout and dequant (:74-146), f64 matvec (:167-183)
//   engine/src/lfm.rs        hyperparameters (:102-145), Engine::load (:148-190),
//                            mul_mat_weight (:205-228), rms_norm (:231-244),
//                            rope_neox (:248-267), norm_head_dim (:270-286),
//                            forward (:290-694), mul_mat_expert (:698-725)
//   engine/src/main.rs       argmax (:112-141), CPU token loop (:160-195)
//   engine/tests/dequant_mirror.rs  byte-addressed shader dequant (:10-46)
//
// Arithmetic contract: every f32 sum is accumulated in exactly the order the
// reference uses (compiled with -ffp-contract=off, no fast-math). Work is only
// parallelised (threads) and vectorised (SIMD lanes) ACROSS independent
// accumulators — output rows, tokens, heads — never inside one reduction, so
// results are bit-identical for any thread count. Rust's f32::exp / powf /
// sin / cos and f64::exp call the platform libm; this file calls glibc's
// expf / powf / sinf / cosf / exp. f32::powi lowers to __powisf2, which
// __builtin_powif also calls. half::f16 conversions are IEEE-754 binary16
// with round-to-nearest-even, restated below from the standard.
//
// Deviation that keeps bit-identity: the reference re-dequantises each routed
// expert row for every token (lfm.rs:698-725). For n > 1 this file groups the
// (token, rank) slots by expert and dequantises each row once for all slots
// of that expert; each dot product is still the same sequential f32 sum and
// the rank-order combine is unchanged.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <memory>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------- binary16
// IEEE-754 binary16 <-> binary32 (the `half` crate contract, q6k.rs:56-58,
// lfm.rs:95-98).
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mag = x & 0x7fffffffu;
  if (mag > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((mag >> 13) & 0x3ffu));  // NaN
  if (mag >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf (>= 65520)
  if (mag >= 0x38800000u) {  // normal half range
    uint32_t r = mag - 0x38000000u;  // rebias exponent (127-15)<<23
    uint32_t lsb = (r >> 13) & 1u;
    r += 0x0fffu + lsb;
    return (uint16_t)(sign | (r >> 13));
  }
  if (mag < 0x33000000u) return (uint16_t)sign;  // < 2^-25: rounds to zero
  // subnormal half: value = mant * 2^(e-150); half ulp = 2^-24
  uint32_t e = mag >> 23;
  uint32_t mant = (mag & 0x7fffffu) | 0x800000u;
  uint32_t shift = 126 - e;  // 14..24 (value / 2^-24 = mant >> shift)
  uint32_t base = mant >> shift;
  uint32_t rem = mant & ((1u << shift) - 1u);
  uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (base & 1u))) base++;
  return (uint16_t)(sign | base);
}

inline float f16_round(float x) { return f16_to_f32(f32_to_f16_rne(x)); }

// ------------------------------------------------------------------- Q6_K
constexpr int QK_K = 256;
constexpr int QK_K_BYTES = 210;

// q6k.rs:104-146 `dequant_half`
void dequant_half(float d, const uint8_t* ql, const uint8_t* qh, const uint8_t* sc, float* y) {
  for (int l = 0; l < 32; l++) {
    int is = l / 16;
    uint8_t qh_l = qh[l];
    int8_t q1 = (int8_t)((int8_t)(ql[l] & 0x0F) | (int8_t)((qh_l & 0x03) << 4)) - 32;
    int8_t q2 = (int8_t)((int8_t)(ql[l + 32] & 0x0F) | (int8_t)(((qh_l >> 2) & 0x03) << 4)) - 32;
    int8_t q3 = (int8_t)((int8_t)(ql[l] >> 4) | (int8_t)(((qh_l >> 4) & 0x03) << 4)) - 32;
    int8_t q4 = (int8_t)((int8_t)(ql[l + 32] >> 4) | (int8_t)(((qh_l >> 6) & 0x03) << 4)) - 32;
    float s0 = (float)(int8_t)sc[is];
    float s2 = (float)(int8_t)sc[is + 2];
    float s4 = (float)(int8_t)sc[is + 4];
    float s6 = (float)(int8_t)sc[is + 6];
    y[l] = d * s0 * (float)q1;
    y[l + 32] = d * s2 * (float)q2;
    y[l + 64] = d * s4 * (float)q3;
    y[l + 96] = d * s6 * (float)q4;
  }
}

// q6k.rs:74-101 `dequantize_q6k_block_mode` (signed scales)
void dequant_block(const uint8_t* block, float* out) {
  float d = f16_to_f32((uint16_t)(block[208] | (block[209] << 8)));
  dequant_half(d, block, block + 128, block + 192, out);
  dequant_half(d, block + 64, block + 160, block + 200, out + 128);
}

void dequant_row(const uint8_t* blocks, float* out, int n) {
  for (int b = 0; b < n / QK_K; b++) dequant_block(blocks + (size_t)b * QK_K_BYTES, out + b * QK_K);
}

// engine/tests/dequant_mirror.rs:10-46 (byte-granular shader formulation)
float shader_dequant(const uint8_t* block, uint32_t k) {
  uint32_t half = k >> 7, jj = k & 127, sub = jj >> 5, l = jj & 31, is = l >> 4;
  size_t ql_idx = half * 64 + (l + (sub & 1) * 32);
  size_t qh_idx = 128 + half * 32 + l;
  size_t sc_idx = 192 + half * 8 + (is + 2 * sub);
  uint8_t qlbyte = block[ql_idx];
  uint8_t nibble = (sub >> 1) != 0 ? (uint8_t)(qlbyte >> 4) : (uint8_t)(qlbyte & 0x0F);
  uint8_t field = (uint8_t)((block[qh_idx] >> (2 * sub)) & 3);
  int q = (int)(uint8_t)(nibble | (field << 4)) - 32;
  int scbyte = block[sc_idx];
  int sc = scbyte >= 128 ? scbyte - 256 : scbyte;
  float d = f16_to_f32((uint16_t)(block[208] | (block[209] << 8)));
  return d * (float)sc * (float)q;
}

// ------------------------------------------------------------- libm calls
// Called through volatile pointers so the compiler cannot fuse sinf+cosf into
// sincosf or constant-fold anything the reference evaluates at run time.
float (*volatile p_expf)(float) = expf;
float (*volatile p_sinf)(float) = sinf;
float (*volatile p_cosf)(float) = cosf;
float (*volatile p_powf)(float, float) = powf;
double (*volatile p_exp)(double) = exp;

// --------------------------------------------------------------- GGUF read
struct TInfo {
  std::string name;
  std::vector<uint64_t> ne;
  uint32_t type;
  uint64_t offset, nbytes;
  const uint8_t* data;
};

struct Gguf {
  int fd = -1;
  uint8_t* map = nullptr;
  size_t len = 0;
  std::map<std::string, uint64_t> u;      // integer scalars
  std::map<std::string, double> f;        // float scalars
  std::map<std::string, std::vector<uint64_t>> ua;  // integer arrays
  std::vector<TInfo> tensors;
  std::map<std::string, size_t> by_name;
  std::string err;
  ~Gguf() {
    if (map) munmap(map, len);
    if (fd >= 0) close(fd);
  }
};

struct Cur {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <class T> T get() {
    T v{};
    if ((size_t)(end - p) < sizeof(T)) { ok = false; return v; }
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (!ok || (uint64_t)(end - p) < n) { ok = false; return ""; }
    std::string s((const char*)p, n);
    p += n;
    return s;
  }
};

bool read_value(Cur& c, uint32_t t, const std::string& key, Gguf& g, bool in_array,
                std::vector<uint64_t>* arr) {
  auto put_u = [&](uint64_t v) {
    if (in_array) { if (arr) arr->push_back(v); } else g.u[key] = v;
  };
  auto put_f = [&](double v) { if (!in_array) g.f[key] = v; };
  switch (t) {
    case 0: put_u(c.get<uint8_t>()); break;
    case 1: put_u((uint64_t)(int64_t)c.get<int8_t>()); break;
    case 2: put_u(c.get<uint16_t>()); break;
    case 3: put_u((uint64_t)(int64_t)c.get<int16_t>()); break;
    case 4: put_u(c.get<uint32_t>()); break;
    case 5: put_u((uint64_t)(int64_t)c.get<int32_t>()); break;
    case 6: put_f(c.get<float>()); break;
    case 7: c.get<uint8_t>(); break;
    case 8: c.str(); break;
    case 9: {
      uint32_t et = c.get<uint32_t>();
      uint64_t n = c.get<uint64_t>();
      if (!c.ok || n > 10000000ull) return false;
      std::vector<uint64_t> v;
      for (uint64_t i = 0; i < n && c.ok; i++) read_value(c, et, key, g, true, &v);
      if (!in_array) g.ua[key] = v;
      break;
    }
    case 10: put_u(c.get<uint64_t>()); break;
    case 11: put_u((uint64_t)c.get<int64_t>()); break;
    case 12: put_f(c.get<double>()); break;
    default: return false;
  }
  return c.ok;
}

bool gguf_open(const char* path, Gguf& g) {
  g.fd = open(path, O_RDONLY);
  if (g.fd < 0) { g.err = std::string("open ") + path; return false; }
  struct stat st;
  fstat(g.fd, &st);
  g.len = (size_t)st.st_size;
  void* m = mmap(nullptr, g.len, PROT_READ, MAP_PRIVATE, g.fd, 0);
  if (m == MAP_FAILED) { g.err = "mmap"; return false; }
  g.map = (uint8_t*)m;
  Cur c{g.map, g.map + g.len};
  uint32_t magic = c.get<uint32_t>();
  uint32_t ver = c.get<uint32_t>();
  if (magic != 0x46554747u || ver != 3) { g.err = "not GGUF v3"; return false; }
  uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  for (uint64_t i = 0; i < nkv; i++) {
    std::string k = c.str();
    uint32_t t = c.get<uint32_t>();
    if (!read_value(c, t, k, g, false, nullptr)) { g.err = "bad kv " + k; return false; }
  }
  uint64_t align = g.u.count("general.alignment") ? g.u["general.alignment"] : 32;
  for (uint64_t i = 0; i < nt; i++) {
    TInfo t;
    t.name = c.str();
    uint32_t nd = c.get<uint32_t>();
    for (uint32_t d = 0; d < nd; d++) t.ne.push_back(c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    uint64_t n = 1;
    for (auto d : t.ne) n *= d;
    t.nbytes = t.type == 0 ? n * 4 : t.type == 14 ? n / 256 * 210 : 0;
    g.by_name[t.name] = g.tensors.size();
    g.tensors.push_back(t);
  }
  if (!c.ok) { g.err = "truncated header"; return false; }
  uint64_t pos = (uint64_t)(c.p - g.map);
  uint64_t data = (pos + align - 1) / align * align;
  for (auto& t : g.tensors) {
    if (data + t.offset + t.nbytes > g.len) { g.err = "tensor past EOF: " + t.name; return false; }
    t.data = g.map + data + t.offset;
  }
  return true;
}

// --------------------------------------------------------------- matrices
typedef float v16 __attribute__((vector_size(64)));
// Weight rows are read through an unaligned alias (std::vector storage is not
// 64-byte aligned).
typedef float v16u __attribute__((vector_size(64), aligned(4)));

// Row-blocked transpose of an f32 weight w[in,out] (element (k,o) at k+o*in):
// wt[(ob*in + k)*16 + r] = w[k + (ob*16+r)*in]. Lane r of a v16 accumulator
// then holds row ob*16+r and sums k in increasing order, like lfm.rs:218-227.
struct MatT {
  int in = 0, out = 0;
  std::vector<float> wt;
};

void make_matt(const float* w, int in, int out, MatT& m) {
  m.in = in;
  m.out = out;
  m.wt.resize((size_t)in * out);
#pragma omp parallel for schedule(static)
  for (int ob = 0; ob < out / 16; ob++)
    for (int r = 0; r < 16; r++) {
      const float* row = w + (size_t)(ob * 16 + r) * in;
      for (int k = 0; k < in; k++) m.wt[((size_t)ob * in + k) * 16 + r] = row[k];
    }
}

// out[o + j*out] = sum_k w[o,k] * x[k + j*in], k ascending (lfm.rs:205-228).
void mul_mat(const MatT& m, const float* x, int n, float* out) {
  const int in = m.in, nob = m.out / 16;
#pragma omp parallel for schedule(dynamic, 4)
  for (int ob = 0; ob < nob; ob++) {
    const v16u* w = (const v16u*)(m.wt.data() + (size_t)ob * in * 16);
    int j = 0;
    for (; j + 4 <= n; j += 4) {
      v16 a0 = {}, a1 = {}, a2 = {}, a3 = {};
      const float* x0 = x + (size_t)j * in;
      for (int k = 0; k < in; k++) {
        v16 wk = w[k];
        a0 += wk * x0[k];
        a1 += wk * x0[k + in];
        a2 += wk * x0[k + 2 * in];
        a3 += wk * x0[k + 3 * in];
      }
      for (int r = 0; r < 16; r++) {
        out[ob * 16 + r + (size_t)j * m.out] = a0[r];
        out[ob * 16 + r + (size_t)(j + 1) * m.out] = a1[r];
        out[ob * 16 + r + (size_t)(j + 2) * m.out] = a2[r];
        out[ob * 16 + r + (size_t)(j + 3) * m.out] = a3[r];
      }
    }
    for (; j < n; j++) {
      v16 a0 = {};
      const float* x0 = x + (size_t)j * in;
      for (int k = 0; k < in; k++) a0 += w[k] * x0[k];
      for (int r = 0; r < 16; r++) out[ob * 16 + r + (size_t)j * m.out] = a0[r];
    }
  }
}

// Dequantise 16 consecutive Q6_K rows (expert slice) into the transposed
// [in][16] layout used by mul_mat.
void dequant_rows16_t(const uint8_t* rows, size_t row_bytes, int in, float* wt16, float* tmp) {
  for (int r = 0; r < 16; r++) {
    dequant_row(rows + r * row_bytes, tmp, in);
    for (int k = 0; k < in; k++) wt16[k * 16 + r] = tmp[k];
  }
}

// --------------------------------------------------------------- engine
constexpr int DIM = 2048, HEADS = 32, HEAD_DIM = 64, N_LAYERS = 24, N_EXPERT = 32, N_USED = 4,
              EXPERT_FF = 1792;

struct Engine {
  Gguf g;
  // hyperparameters (lfm.rs:102-145)
  int dim, heads, head_dim, n_layers, vocab, n_expert, n_used, expert_ff, n_ff, dense_lead,
      conv_l_cache;
  std::vector<int> kv_heads;
  float eps, rope_theta;
  uint32_t eos;
  bool kv_f16 = false;
  size_t ctx = 4096;
  std::map<std::string, MatT> mats;                 // 2-D weights, pre-dequantised
  std::map<std::string, std::vector<float>> vecs;   // 1-D / small f32 tensors
  std::vector<std::vector<float>> conv_cache;       // [cache_len, dim] per layer (ne0=cache_len)
  std::vector<std::vector<float>> keys, values;     // lfm.rs:78-81 layouts
  std::vector<size_t> kv_ctx;                       // ctx each layer's cache was sized with
  std::string err;
  std::vector<float> last_logits;
  // session state saved by oracle_checkpoint (test/bench helper, no reference counterpart)
  std::vector<std::vector<float>> saved_conv, saved_keys, saved_values;
  std::vector<size_t> saved_kv_ctx;

  const TInfo* t(const std::string& n) const {
    auto it = g.by_name.find(n);
    return it == g.by_name.end() ? nullptr : &g.tensors[it->second];
  }
  const float* f32(const std::string& n) {
    auto it = vecs.find(n);
    if (it == vecs.end()) { fprintf(stderr, "missing tensor %s\n", n.c_str()); abort(); }
    return it->second.data();
  }
  const MatT& mat(const std::string& n) {
    auto it = mats.find(n);
    if (it == mats.end()) { fprintf(stderr, "weight %s not in f32 cache\n", n.c_str()); abort(); }
    return it->second;
  }
};

bool load_hyperparams(Engine& e) {
  auto& g = e.g;
  auto need = [&](const char* k, uint64_t& v) {
    if (!g.u.count(k)) { e.err = std::string("metadata ") + k + " not a u32"; return false; }
    v = g.u[k];
    return true;
  };
  uint64_t nl, dim, heads, vocab, ne, nu, eff, nff;
  if (!need("lfm2moe.block_count", nl) || !need("lfm2moe.embedding_length", dim) ||
      !need("lfm2moe.attention.head_count", heads) || !need("lfm2moe.vocab_size", vocab) ||
      !need("lfm2moe.expert_count", ne) || !need("lfm2moe.expert_used_count", nu) ||
      !need("lfm2moe.expert_feed_forward_length", eff) ||
      !need("lfm2moe.feed_forward_length", nff))
    return false;
  if (!g.ua.count("lfm2moe.attention.head_count_kv")) {
    e.err = "metadata lfm2moe.attention.head_count_kv not an array";
    return false;
  }
  if (dim != DIM || heads != HEADS || nl != N_LAYERS || vocab != 128000 || ne != N_EXPERT ||
      nu != N_USED || eff != EXPERT_FF) {
    char b[256];
    snprintf(b, sizeof b,
             "unsupported geometry: dim=%lu heads=%lu layers=%lu vocab=%lu n_expert=%lu "
             "n_used=%lu expert_ff=%lu",
             (unsigned long)dim, (unsigned long)heads, (unsigned long)nl, (unsigned long)vocab,
             (unsigned long)ne, (unsigned long)nu, (unsigned long)eff);
    e.err = b;
    return false;
  }
  e.dim = (int)dim;
  e.heads = (int)heads;
  e.head_dim = HEAD_DIM;
  e.n_layers = (int)nl;
  e.vocab = (int)vocab;
  e.n_expert = (int)ne;
  e.n_used = (int)nu;
  e.expert_ff = (int)eff;
  e.n_ff = (int)nff;
  e.dense_lead = g.u.count("lfm2moe.leading_dense_block_count")
                     ? (int)g.u["lfm2moe.leading_dense_block_count"] : 2;
  e.conv_l_cache = g.u.count("lfm2moe.shortconv.l_cache") ? (int)g.u["lfm2moe.shortconv.l_cache"] : 3;
  for (auto v : g.ua["lfm2moe.attention.head_count_kv"]) e.kv_heads.push_back((int)v);
  if (!g.f.count("lfm2moe.attention.layer_norm_rms_epsilon") || !g.f.count("lfm2moe.rope.freq_base")) {
    e.err = "metadata eps/rope not an f32";
    return false;
  }
  e.eps = (float)g.f["lfm2moe.attention.layer_norm_rms_epsilon"];
  e.rope_theta = (float)g.f["lfm2moe.rope.freq_base"];
  e.eos = g.u.count("tokenizer.ggml.eos_token_id") ? (uint32_t)g.u["tokenizer.ggml.eos_token_id"] : 124900;
  return true;
}

// lfm.rs:148-190: every non-3-D tensor is pre-dequantised to f32 once.
bool engine_load(Engine& e, const char* path) {
  if (!gguf_open(path, e.g)) { e.err = e.g.err; return false; }
  if (!load_hyperparams(e)) return false;
  std::vector<float> tmp;
  for (auto& ti : e.g.tensors) {
    if (ti.ne.size() == 3) continue;
    size_t n = 1;
    for (auto d : ti.ne) n *= d;
    const float* src = nullptr;
    if (ti.type == 0) {
      src = (const float*)ti.data;
    } else if (ti.type == 14) {
      tmp.resize(n);
      size_t nb = n / QK_K;
#pragma omp parallel for schedule(static)
      for (size_t b = 0; b < nb; b++) dequant_block(ti.data + b * QK_K_BYTES, tmp.data() + b * QK_K);
      src = tmp.data();
    } else {
      continue;
    }
    if (ti.ne.size() == 2 && ti.ne[1] % 16 == 0 && ti.ne[1] >= 16) {
      make_matt(src, (int)ti.ne[0], (int)ti.ne[1], e.mats[ti.name]);
    }
    if (ti.ne.size() == 1 || ti.type == 0) e.vecs[ti.name].assign(src, src + n);
  }
  e.conv_cache.assign(e.n_layers, {});
  e.keys.assign(e.n_layers, {});
  e.values.assign(e.n_layers, {});
  e.kv_ctx.assign(e.n_layers, 0);
  const char* kvf = getenv("LFM_KV_F16");
  e.kv_f16 = kvf && std::string(kvf) == "1";
  return true;
}

void rms_norm(const Engine& e, const float* x, const float* scale, int n, float* out) {
  const int dim = e.dim;
  for (int j = 0; j < n; j++) {
    float ss = 0.f;
    for (int k = 0; k < dim; k++) {
      float v = x[k + (size_t)j * dim];
      ss += v * v;
    }
    float inv = 1.0f / sqrtf(ss / (float)dim + e.eps);
    for (int k = 0; k < dim; k++) out[k + (size_t)j * dim] = x[k + (size_t)j * dim] * inv * scale[k];
  }
}

void rope_neox(const Engine& e, float* q, int heads, int n, const int64_t* positions) {
  const int hd = e.head_dim, dim_all = hd * heads;
  float tscale = p_powf(e.rope_theta, -2.0f / (float)hd);
  for (int j = 0; j < n; j++) {
    float pos = (float)positions[j];
    for (int p = 0; p < hd / 2; p++) {
      float theta = pos * __builtin_powif(tscale, p);
      float s = p_sinf(theta), c = p_cosf(theta);
      for (int h = 0; h < heads; h++) {
        size_t i0 = p + h * hd + (size_t)j * dim_all;
        size_t i1 = p + hd / 2 + h * hd + (size_t)j * dim_all;
        float x0 = q[i0], x1 = q[i1];
        q[i0] = x0 * c - x1 * s;
        q[i1] = x0 * s + x1 * c;
      }
    }
  }
}

void norm_head_dim(const Engine& e, float* q, const float* scale, int heads, int n) {
  const int hd = e.head_dim, dim_all = hd * heads;
  for (int h = 0; h < heads; h++)
    for (int j = 0; j < n; j++) {
      float ss = 0.f;
      for (int k = 0; k < hd; k++) {
        float v = q[k + h * hd + (size_t)j * dim_all];
        ss += v * v;
      }
      float inv = 1.0f / sqrtf(ss / (float)hd + e.eps);
      for (int k = 0; k < hd; k++) q[k + h * hd + (size_t)j * dim_all] *= inv * scale[k];
    }
}

// lfm.rs:613-637 — sigmoid, stable descending sort of (prob + bias), top n_used,
// renormalise with the 6.103515625e-5 clamp.
void route(const float* router, const float* bias, int n_expert, int n_used, int* sel, float* wsel) {
  std::vector<float> probs(n_expert), score(n_expert);
  for (int ex = 0; ex < n_expert; ex++) {
    float lg = router[ex];
    probs[ex] = 1.0f / (1.0f + p_expf(-lg));
    score[ex] = probs[ex] + bias[ex];
  }
  // A stable sort by descending score keeps the lower id first among equals;
  // selecting the running maximum with a strict '>' gives the same prefix.
  std::vector<bool> used(n_expert, false);
  for (int r = 0; r < n_used; r++) {
    int best = -1;
    for (int ex = 0; ex < n_expert; ex++) {
      if (used[ex]) continue;
      if (best < 0 || score[ex] > score[best]) best = ex;
    }
    used[best] = true;
    sel[r] = best;
  }
  float wsum = 0.f;
  for (int r = 0; r < n_used; r++) {
    wsel[r] = probs[sel[r]];
    wsum += probs[sel[r]];
  }
  if (wsum < 6.103515625e-5f) wsum = 6.103515625e-5f;
  for (int r = 0; r < n_used; r++) wsel[r] /= wsum;
}

inline float silu_mul(float g, float u) { return g / (1.0f + p_expf(-g)) * u; }

// Expert slice (lfm.rs:698-725) for a set of input columns: out[c*out_dim + o]
// = sum_k dequant(W_e)[o,k] * xs[c*in_dim + k] (k ascending, f32).
void expert_matmul(const Engine& e, const TInfo* t, int ex, int in_dim, int out_dim,
                   const float* xs, int ncols, float* out) {
  size_t row_bytes = (size_t)(in_dim / QK_K) * QK_K_BYTES;
  const uint8_t* base = t->data + (size_t)ex * out_dim * row_bytes;
  int nob = out_dim / 16;
#pragma omp parallel
  {
    std::vector<float> wt((size_t)in_dim * 16), tmp(in_dim);
#pragma omp for schedule(dynamic, 2)
    for (int ob = 0; ob < nob; ob++) {
      dequant_rows16_t(base + (size_t)ob * 16 * row_bytes, row_bytes, in_dim, wt.data(), tmp.data());
      const v16u* w = (const v16u*)wt.data();
      int c = 0;
      for (; c + 4 <= ncols; c += 4) {
        v16 a0 = {}, a1 = {}, a2 = {}, a3 = {};
        const float* x0 = xs + (size_t)c * in_dim;
        for (int k = 0; k < in_dim; k++) {
          v16 wk = w[k];
          a0 += wk * x0[k];
          a1 += wk * x0[k + in_dim];
          a2 += wk * x0[k + 2 * in_dim];
          a3 += wk * x0[k + 3 * in_dim];
        }
        for (int r = 0; r < 16; r++) {
          out[(size_t)c * out_dim + ob * 16 + r] = a0[r];
          out[(size_t)(c + 1) * out_dim + ob * 16 + r] = a1[r];
          out[(size_t)(c + 2) * out_dim + ob * 16 + r] = a2[r];
          out[(size_t)(c + 3) * out_dim + ob * 16 + r] = a3[r];
        }
      }
      for (; c < ncols; c++) {
        v16 a0 = {};
        const float* x0 = xs + (size_t)c * in_dim;
        for (int k = 0; k < in_dim; k++) a0 += w[k] * x0[k];
        for (int r = 0; r < 16; r++) out[(size_t)c * out_dim + ob * 16 + r] = a0[r];
      }
    }
  }
}

void dump_vec(const char* dir, const std::string& name, const float* v, size_t n) {
  std::string path = std::string(dir) + "/" + name + ".bin";
  FILE* f = fopen(path.c_str(), "wb");
  if (!f) { fprintf(stderr, "dump %s failed\n", path.c_str()); abort(); }
  fwrite(v, 4, n, f);
  fclose(f);
}

// lfm.rs:290-694
bool forward(Engine& e, const uint32_t* ids, int n, int64_t start_pos, float* logits_out) {
  const int dim = e.dim, hd = e.head_dim;
  const size_t ctx = e.ctx;
  if (n < 1 || start_pos < 0) { e.err = "forward range"; return false; }
  for (int j = 0; j < n; j++)
    if (ids[j] >= (uint32_t)e.vocab) { e.err = "token out of range"; return false; }
  const char* dump_dir = n > 1 ? getenv("LFM_LAYER_DUMP") : nullptr;

  std::vector<float> x((size_t)dim * n);
  {
    const MatT& emb = e.mat("token_embd.weight");
    // token_embd.weight is pre-dequantised [dim, vocab]; read row `tok`.
    for (int j = 0; j < n; j++) {
      size_t tok = ids[j];
      size_t ob = tok / 16, r = tok % 16;
      for (int k = 0; k < dim; k++) x[k + (size_t)j * dim] = emb.wt[(ob * dim + k) * 16 + r];
    }
  }
  if (dump_dir) dump_vec(dump_dir, "embd", &x[(size_t)(n - 1) * dim], dim);

  std::vector<float> h((size_t)dim * n);
  for (int l = 0; l < e.n_layers; l++) {
    std::string prefix = "blk." + std::to_string(l) + ".";
    int kv = e.kv_heads[l];
    rms_norm(e, x.data(), e.f32(prefix + "attn_norm.weight"), n, h.data());

    if (kv > 0) {
      const int hdkv = hd * kv;
      std::vector<float> q((size_t)dim * n), k((size_t)hdkv * n), v((size_t)hdkv * n);
      mul_mat(e.mat(prefix + "attn_q.weight"), h.data(), n, q.data());
      mul_mat(e.mat(prefix + "attn_k.weight"), h.data(), n, k.data());
      mul_mat(e.mat(prefix + "attn_v.weight"), h.data(), n, v.data());
      norm_head_dim(e, q.data(), e.f32(prefix + "attn_q_norm.weight"), e.heads, n);
      norm_head_dim(e, k.data(), e.f32(prefix + "attn_k_norm.weight"), kv, n);
      std::vector<int64_t> positions(n);
      for (int j = 0; j < n; j++) positions[j] = start_pos + j;
      rope_neox(e, q.data(), e.heads, n, positions.data());
      rope_neox(e, k.data(), kv, n, positions.data());

      // ensure_kv (lfm.rs:727-732) sizes the cache with the ctx of first use.
      if (e.keys[l].empty()) {
        e.keys[l].assign((size_t)hd * kv * ctx, 0.f);
        e.values[l].assign(ctx * hd * kv, 0.f);
        e.kv_ctx[l] = ctx;
      }
      const size_t lctx = e.kv_ctx[l];
      if ((size_t)start_pos + n > lctx) { e.err = "kv cache overflow"; return false; }
      float* keys = e.keys[l].data();
      float* values = e.values[l].data();
      for (int j = 0; j < n; j++) {
        size_t p = (size_t)(start_pos + j);
        for (int kh = 0; kh < kv; kh++)
          for (int d = 0; d < hd; d++) {
            float kk = k[(kh * hd + d) + (size_t)j * hdkv];
            float vv = v[(kh * hd + d) + (size_t)j * hdkv];
            keys[d + kh * hd + p * hdkv] = e.kv_f16 ? f16_round(kk) : kk;
            values[p + d * lctx + kh * (lctx * hd)] = e.kv_f16 ? f16_round(vv) : vv;
          }
      }
      const float scale = 1.0f / sqrtf((float)hd);
      std::vector<float> a((size_t)dim * n);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
      for (int j = 0; j < n; j++)
        for (int hh = 0; hh < e.heads; hh++) {
          size_t p = (size_t)(start_pos + j);
          int kh = hh * kv / e.heads;
          std::vector<float> s(p + 1);
          float m = -INFINITY;
          for (size_t t2 = 0; t2 <= p; t2++) {
            double acc = 0.0;
            for (int d = 0; d < hd; d++)
              acc += (double)q[(hh * hd + d) + (size_t)j * dim] * (double)keys[d + kh * hd + t2 * hdkv];
            float sc = (float)acc * scale;
            s[t2] = sc;
            if (sc > m) m = sc;
          }
          double sum = 0.0;
          for (size_t t2 = 0; t2 <= p; t2++) {
            double ev = p_exp((double)(s[t2] - m));
            s[t2] = (float)ev;
            sum += ev;
          }
          for (size_t t2 = 0; t2 <= p; t2++) s[t2] = (float)((double)s[t2] / sum);
          for (int d = 0; d < hd; d++) {
            double acc = 0.0;
            for (size_t t2 = 0; t2 <= p; t2++)
              acc += (double)s[t2] * (double)values[t2 + d * lctx + kh * (lctx * hd)];
            a[(hh * hd + d) + (size_t)j * dim] = (float)acc;
          }
        }
      std::vector<float> ax((size_t)dim * n);
      mul_mat(e.mat(prefix + "attn_output.weight"), a.data(), n, ax.data());
      for (size_t i = 0; i < (size_t)dim * n; i++) x[i] += ax[i];
    } else {
      const int conv_l = e.conv_l_cache, cache_len = conv_l - 1;
      std::vector<float> bcx((size_t)3 * dim * n);
      mul_mat(e.mat(prefix + "shortconv.in_proj.weight"), h.data(), n, bcx.data());
      std::vector<float> bx((size_t)n * dim);
      for (int t2 = 0; t2 < n; t2++)
        for (int ch = 0; ch < dim; ch++) {
          float b = bcx[ch + (size_t)t2 * (3 * dim)];
          float xx = bcx[2 * dim + ch + (size_t)t2 * (3 * dim)];
          bx[t2 + (size_t)ch * n] = b * xx;
        }
      std::vector<float> cache = e.conv_cache[l];
      if (cache.empty()) cache.assign((size_t)cache_len * dim, 0.f);
      const size_t cl = (size_t)cache_len + n;
      std::vector<float> ci(cl * dim);
      for (int ch = 0; ch < dim; ch++) {
        for (int t2 = 0; t2 < cache_len; t2++) ci[t2 + ch * cl] = cache[t2 + (size_t)ch * cache_len];
        for (int t2 = 0; t2 < n; t2++) ci[cache_len + t2 + ch * cl] = bx[t2 + (size_t)ch * n];
      }
      std::vector<float> newcache((size_t)cache_len * dim);
      for (int ch = 0; ch < dim; ch++)
        for (int t2 = 0; t2 < cache_len; t2++)
          newcache[t2 + (size_t)ch * cache_len] = ci[n + t2 + ch * cl];
      e.conv_cache[l] = newcache;
      const float* cw = e.f32(prefix + "shortconv.conv.weight");
      std::vector<float> co((size_t)dim * n);
      for (int t2 = 0; t2 < n; t2++)
        for (int ch = 0; ch < dim; ch++) {
          float acc = 0.f;
          for (int kk = 0; kk < conv_l; kk++) acc += ci[(t2 + kk) + ch * cl] * cw[kk + ch * conv_l];
          co[ch + (size_t)t2 * dim] = acc;
        }
      std::vector<float> gated((size_t)dim * n);
      for (int t2 = 0; t2 < n; t2++)
        for (int ch = 0; ch < dim; ch++) {
          float cc = bcx[dim + ch + (size_t)t2 * (3 * dim)];
          gated[ch + (size_t)t2 * dim] = cc * co[ch + (size_t)t2 * dim];
        }
      std::vector<float> projected((size_t)dim * n);
      mul_mat(e.mat(prefix + "shortconv.out_proj.weight"), gated.data(), n, projected.data());
      for (size_t i = 0; i < (size_t)dim * n; i++) x[i] += projected[i];
    }
    if (dump_dir) dump_vec(dump_dir, "ffn_inp-" + std::to_string(l), &x[(size_t)(n - 1) * dim], dim);

    // FFN: the last layer only runs on the last token (lfm.rs:540-541).
    const int nf = l == e.n_layers - 1 ? 1 : n;
    const int f_off = nf == 1 ? n - 1 : 0;
    std::vector<float> fnorm((size_t)dim * nf);
    rms_norm(e, &x[(size_t)f_off * dim], e.f32(prefix + "ffn_norm.weight"), nf, fnorm.data());
    if (l < e.dense_lead) {
      std::vector<float> gate((size_t)e.n_ff * nf), up((size_t)e.n_ff * nf), swig((size_t)e.n_ff * nf);
      mul_mat(e.mat(prefix + "ffn_gate.weight"), fnorm.data(), nf, gate.data());
      mul_mat(e.mat(prefix + "ffn_up.weight"), fnorm.data(), nf, up.data());
      for (size_t i = 0; i < (size_t)e.n_ff * nf; i++) swig[i] = silu_mul(gate[i], up[i]);
      std::vector<float> ffn_out((size_t)dim * nf);
      mul_mat(e.mat(prefix + "ffn_down.weight"), swig.data(), nf, ffn_out.data());
      for (int j = 0; j < nf; j++)
        for (int k = 0; k < dim; k++) x[k + (size_t)(f_off + j) * dim] += ffn_out[k + (size_t)j * dim];
    } else {
      const int ne = e.n_expert, nu = e.n_used, eff = e.expert_ff;
      std::vector<float> router((size_t)ne * nf);
      {
        // ffn_gate_inp.weight is [dim, 32] F32 (32 rows of 2048).
        const float* w = e.f32(prefix + "ffn_gate_inp.weight");
        for (int o = 0; o < ne; o++)
          for (int j = 0; j < nf; j++) {
            float acc = 0.f;
            for (int k = 0; k < dim; k++) acc += w[(size_t)o * dim + k] * fnorm[k + (size_t)j * dim];
            router[o + (size_t)j * ne] = acc;
          }
      }
      const float* bias = e.f32(prefix + "exp_probs_b.bias");
      std::vector<int> sel((size_t)nf * nu);
      std::vector<float> wsel((size_t)nf * nu);
      for (int j = 0; j < nf; j++) route(&router[(size_t)j * ne], bias, ne, nu, &sel[j * nu], &wsel[j * nu]);
      const TInfo* tg = e.t(prefix + "ffn_gate_exps.weight");
      const TInfo* tu = e.t(prefix + "ffn_up_exps.weight");
      const TInfo* td = e.t(prefix + "ffn_down_exps.weight");
      // down outputs per (token, rank), combined afterwards in rank order.
      std::vector<float> down_out((size_t)nf * nu * dim);
      for (int ex = 0; ex < ne; ex++) {
        std::vector<int> slots;
        for (int s = 0; s < nf * nu; s++)
          if (sel[s] == ex) slots.push_back(s);
        if (slots.empty()) continue;
        const int ns = (int)slots.size();
        std::vector<float> xs((size_t)ns * dim), gate((size_t)ns * eff), up((size_t)ns * eff),
            swig((size_t)ns * eff), dn((size_t)ns * dim);
        for (int c = 0; c < ns; c++)
          memcpy(&xs[(size_t)c * dim], &fnorm[(size_t)(slots[c] / nu) * dim], dim * 4);
        expert_matmul(e, tg, ex, dim, eff, xs.data(), ns, gate.data());
        expert_matmul(e, tu, ex, dim, eff, xs.data(), ns, up.data());
        for (size_t i = 0; i < (size_t)ns * eff; i++) swig[i] = silu_mul(gate[i], up[i]);
        expert_matmul(e, td, ex, eff, dim, swig.data(), ns, dn.data());
        for (int c = 0; c < ns; c++) memcpy(&down_out[(size_t)slots[c] * dim], &dn[(size_t)c * dim], dim * 4);
      }
      for (int j = 0; j < nf; j++) {
        std::vector<float> acc(dim, 0.f);
        for (int r = 0; r < nu; r++) {
          float wgt = wsel[j * nu + r];
          const float* d = &down_out[((size_t)j * nu + r) * dim];
          for (int k = 0; k < dim; k++) acc[k] += d[k] * wgt;
        }
        for (int k = 0; k < dim; k++) x[k + (size_t)(f_off + j) * dim] += acc[k];
      }
    }
    if (dump_dir) dump_vec(dump_dir, "l_out-" + std::to_string(l), &x[(size_t)(n - 1) * dim], dim);
  }

  // lfm.rs:676-693: logits = token_embd^T * norm(x_last)
  const float* onorm = e.f32("token_embd_norm.weight");
  std::vector<float> xnorm(dim);
  {
    const float* xl = &x[(size_t)(n - 1) * dim];
    float ss = 0.f;
    for (int k = 0; k < dim; k++) ss += xl[k] * xl[k];
    float inv = 1.0f / sqrtf(ss / (float)dim + e.eps);
    for (int k = 0; k < dim; k++) xnorm[k] = xl[k] * inv * onorm[k];
  }
  e.last_logits.resize(e.vocab);
  mul_mat(e.mat("token_embd.weight"), xnorm.data(), 1, e.last_logits.data());
  if (logits_out) memcpy(logits_out, e.last_logits.data(), (size_t)e.vocab * 4);
  return true;
}

// main.rs:112-141 — 8 independent lanes, then ties to the lowest index, then
// the tail; equivalent to "first maximum wins, NaN never wins".
uint32_t argmax(const float* logits, size_t len) {
  float values[8];
  size_t indices[8] = {0};
  for (int i = 0; i < 8; i++) values[i] = -INFINITY;
  size_t nchunks = len / 8;
  for (size_t block = 0; block < nchunks; block++)
    for (int lane = 0; lane < 8; lane++) {
      float v = logits[block * 8 + lane];
      if (v > values[lane]) {
        values[lane] = v;
        indices[lane] = block * 8 + lane;
      }
    }
  size_t best = 0;
  float value = -INFINITY;
  for (int lane = 0; lane < 8; lane++)
    if (values[lane] > value || (values[lane] == value && indices[lane] < best)) {
      best = indices[lane];
      value = values[lane];
    }
  size_t offset = nchunks * 8;
  for (size_t i = offset; i < len; i++)
    if (logits[i] > value) {
      best = i;
      value = logits[i];
    }
  return (uint32_t)best;
}

}  // namespace

// ===================================================================== C ABI
extern "C" {

float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t oracle_f32_to_f16(float x) { return f32_to_f16_rne(x); }
void oracle_dequant_block(const uint8_t* block, float* out) { dequant_block(block, out); }
float oracle_shader_dequant(const uint8_t* block, uint32_t k) { return shader_dequant(block, k); }
void oracle_dequant_rows(const uint8_t* blocks, size_t nblocks, float* out) {
#pragma omp parallel for schedule(static)
  for (size_t b = 0; b < nblocks; b++) dequant_block(blocks + b * QK_K_BYTES, out + b * QK_K);
}

// q6k.rs:167-183: dequantise each row, f64 dot, rounded to f32.
void oracle_q6k_matvec_f64(const uint8_t* weight, int in_dim, int out_dim, const float* x, float* out) {
  size_t row_bytes = (size_t)(in_dim / QK_K) * QK_K_BYTES;
#pragma omp parallel
  {
    std::vector<float> wrow(in_dim);
#pragma omp for schedule(static)
    for (int o = 0; o < out_dim; o++) {
      dequant_row(weight + o * row_bytes, wrow.data(), in_dim);
      double acc = 0.0;
      for (int k = 0; k < in_dim; k++) acc += (double)wrow[k] * (double)x[k];
      out[o] = (float)acc;
    }
  }
}

// lfm.rs:218-227 order (sequential f32) on Q6_K rows: the oracle's mul_mat_weight.
void oracle_q6k_matmul_f32(const uint8_t* weight, int in_dim, int out_dim, const float* x, int n, float* out) {
  size_t row_bytes = (size_t)(in_dim / QK_K) * QK_K_BYTES;
#pragma omp parallel
  {
    std::vector<float> wrow(in_dim);
#pragma omp for schedule(static)
    for (int o = 0; o < out_dim; o++) {
      dequant_row(weight + o * row_bytes, wrow.data(), in_dim);
      for (int j = 0; j < n; j++) {
        float acc = 0.f;
        for (int k = 0; k < in_dim; k++) acc += wrow[k] * x[k + (size_t)j * in_dim];
        out[o + (size_t)j * out_dim] = acc;
      }
    }
  }
}

uint32_t oracle_argmax(const float* logits, size_t len) { return argmax(logits, len); }

void oracle_route(const float* router, const float* bias, int n_expert, int n_used, int* sel, float* w) {
  route(router, bias, n_expert, n_used, sel, w);
}

float oracle_silu_mul(float g, float u) { return silu_mul(g, u); }

void* oracle_engine_create(const char* path, char* err, size_t errlen) {
  auto* e = new Engine();
  if (!engine_load(*e, path)) {
    if (err && errlen) snprintf(err, errlen, "%s", e->err.c_str());
    delete e;
    return nullptr;
  }
  return e;
}

void oracle_engine_destroy(void* h) { delete (Engine*)h; }
void oracle_engine_set_ctx(void* h, size_t ctx) { ((Engine*)h)->ctx = ctx; }
void oracle_engine_set_kv_f16(void* h, int on) { ((Engine*)h)->kv_f16 = on != 0; }
int oracle_engine_vocab(void* h) { return ((Engine*)h)->vocab; }
uint32_t oracle_engine_eos(void* h) { return ((Engine*)h)->eos; }
const char* oracle_engine_error(void* h) { return ((Engine*)h)->err.c_str(); }

int oracle_forward(void* h, const uint32_t* ids, int n, int64_t start_pos, float* logits) {
  return forward(*(Engine*)h, ids, n, start_pos, logits) ? 0 : 1;
}

// Session state in the byte layout of the reference's resident snapshot
// (gpu_lfm/resident_graph.rs:572-602): per layer in order, attention layers
// give K then V for the valid prefix as f32 words, position-major
// [p][kh*64+d]; conv layers give the 2-slot state as [ch][slot] f32.
size_t oracle_snapshot(void* h, size_t valid, float* out) {
  Engine& e = *(Engine*)h;
  size_t w = 0;
  for (int l = 0; l < e.n_layers; l++) {
    int kv = e.kv_heads[l];
    if (kv > 0) {
      size_t hdkv = (size_t)e.head_dim * kv, lctx = e.kv_ctx[l];
      for (size_t p = 0; p < valid; p++)
        for (size_t i = 0; i < hdkv; i++) {
          if (out) out[w] = e.keys[l].empty() ? 0.f : e.keys[l][i + p * hdkv];
          w++;
        }
      for (size_t p = 0; p < valid; p++)
        for (int kh = 0; kh < kv; kh++)
          for (int d = 0; d < e.head_dim; d++) {
            if (out)
              out[w] = e.values[l].empty() ? 0.f
                                           : e.values[l][p + d * lctx + kh * (lctx * e.head_dim)];
            w++;
          }
    } else {
      size_t cl = (size_t)e.conv_l_cache - 1;
      for (int ch = 0; ch < e.dim; ch++)
        for (size_t s = 0; s < cl; s++) {
          if (out) out[w] = e.conv_cache[l].empty() ? 0.f : e.conv_cache[l][s + ch * cl];
          w++;
        }
    }
  }
  return w;
}

// main.rs:174-195: prefill, then greedy decode until EOS or n tokens. Returns
// the number of generated tokens; logits of every forward (prompt first) are
// written to `step_logits` (capacity (n+1)*vocab floats) when not null.
int oracle_greedy(void* h, const uint32_t* prompt, int prompt_len, int n, uint32_t eos,
                  uint32_t* out_tokens, float* step_logits) {
  Engine& e = *(Engine*)h;
  std::vector<float> logits(e.vocab);
  if (!forward(e, prompt, prompt_len, 0, logits.data())) return -1;
  if (step_logits) memcpy(step_logits, logits.data(), (size_t)e.vocab * 4);
  int count = 0;
  for (int step = 0; step < n; step++) {
    uint32_t token = argmax(logits.data(), logits.size());
    if (token == eos) break;
    out_tokens[count++] = token;
    if (!forward(e, &token, 1, prompt_len + step, logits.data())) return -1;
    if (step_logits) memcpy(step_logits + (size_t)(step + 1) * e.vocab, logits.data(), (size_t)e.vocab * 4);
  }
  return count;
}

// Save / put back the session state (K/V caches, conv states): lets a
// caller re-run the same decode steps, e.g. on a different thread count to
// check that the results are bit-identical. Not part of the reference.
void oracle_checkpoint(void* h) {
  Engine& e = *(Engine*)h;
  e.saved_conv = e.conv_cache;
  e.saved_keys = e.keys;
  e.saved_values = e.values;
  e.saved_kv_ctx = e.kv_ctx;
}

void oracle_rollback(void* h) {
  Engine& e = *(Engine*)h;
  e.conv_cache = e.saved_conv;
  e.keys = e.saved_keys;
  e.values = e.saved_values;
  e.kv_ctx = e.saved_kv_ctx;
}

int oracle_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// Thread count of the parallel loops (output rows / experts). Set explicitly
// because a host process may have initialised the OpenMP runtime with
// OMP_NUM_THREADS=1 (torchrun does) before this library was loaded.
void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"

// ===================================================================== CLI
// `lfm2_greedy_cpu --model M --tokens 1,2,3 [--n 64] [--eos E]`, printing the
// JSON line of main.rs:190-193.
#ifdef ORACLE_MAIN
int main(int argc, char** argv) {
  std::string model, tokens;
  int n = 64;
  long eos = 124900;
  for (int i = 1; i < argc; i++) {
    std::string a = argv[i];
    if (a == "--cpu") continue;
    if (i + 1 >= argc) { fprintf(stderr, "%s needs a value\n", a.c_str()); return 2; }
    if (a == "--model") model = argv[++i];
    else if (a == "--tokens") tokens = argv[++i];
    else if (a == "--n") n = atoi(argv[++i]);
    else if (a == "--eos") eos = atol(argv[++i]);
    else { fprintf(stderr, "unknown arg %s\n", a.c_str()); return 2; }
  }
  std::vector<uint32_t> prompt;
  size_t p = 0;
  while (p < tokens.size()) {
    size_t c = tokens.find(',', p);
    std::string s = tokens.substr(p, c == std::string::npos ? std::string::npos : c - p);
    size_t b = s.find_first_not_of(" \t"), en = s.find_last_not_of(" \t");
    if (b != std::string::npos) prompt.push_back((uint32_t)strtoul(s.substr(b, en - b + 1).c_str(), nullptr, 10));
    if (c == std::string::npos) break;
    p = c + 1;
  }
  if (prompt.empty() || model.empty()) { fprintf(stderr, "need --model and --tokens\n"); return 2; }
  char err[512];
  void* h = oracle_engine_create(model.c_str(), err, sizeof err);
  if (!h) { fprintf(stderr, "%s\n", err); return 1; }
  Engine& e = *(Engine*)h;
  uint32_t eos_u = (uint32_t)eos;
  if (eos == 124900) eos_u = e.eos;
  e.ctx = prompt.size() + n + 16;
  std::vector<uint32_t> out(n);
  int cnt = oracle_greedy(h, prompt.data(), (int)prompt.size(), n, eos_u, out.data(), nullptr);
  if (cnt < 0) { fprintf(stderr, "%s\n", e.err.c_str()); return 1; }
  printf("{\"greedy\":true,\"device\":\"cpu-reference\",\"eos\":%u,\"n_vocab\":%d,\"tokens\":[", eos_u, e.vocab);
  for (int i = 0; i < cnt; i++) printf("%s%u", i ? "," : "", out[i]);
  printf("]}\n");
  oracle_engine_destroy(h);
  return 0;
}
#endif
