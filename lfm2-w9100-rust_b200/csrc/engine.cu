// The B200 engine behind include/lfm_cuda.h — the replacement of the
// reference's GpuEngine (engine/src/gpu_lfm.rs:23-245) and its resident graph
// (engine/src/gpu_lfm/resident_graph.rs:4-602).
//
// Device data layout (HBM):
//   * every Q6_K tensor in the unit-plane layout of q6k.cuh (same byte count
//     as the GGUF payload); experts [in, out, 32] are one matrix of 32*out rows;
//   * F32 tensors (norms, router, bias, conv taps) as in the GGUF;
//   * K and V caches fp16 [attn layer][kv head][ctx][64] (the reference rounds
//     K/V through f16, gpu_lfm.rs:8-11, so fp16 storage holds the same values);
//   * short-conv state f32 [conv layer][channel][2] (resident_graph.rs:75);
//   * RoPE (cos, sin) table [ctx][32] computed once on the host with the same
//     libm calls and operation order as the CPU path (lfm.rs:248-267).
// A decode step (n == 1) is one CUDA graph: a 8-byte H2D copy of (token,
// position), the step itself, and a 16-byte D2H copy of the argmax and the
// status words — the analogue of the reference's immutable decode replay with
// a device-side position (vulkan/reusable.rs:4-173). The step is one
// persistent cooperative kernel (step.cu) when it fits one CTA per SM, else
// (or with LFM_STEP=0) a chain of 126 kernels (mvt.cu / decode.cu).
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <stdexcept>
#include <memory>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/lfm_cuda.h"
#include "gguf.h"
#include "kernels.h"
#include "step.h"
#include "ep.h"
#include "tc_gemm.h"

namespace lfm {

void gemm_q6_ld(const Q6Mat& W, const float* X, int n, float* out, int ldo, bool resid, cudaStream_t s);

namespace {

thread_local std::string g_error;

struct LayerW {
  bool attn = false;
  int attn_idx = -1, conv_idx = -1, moe_idx = -1;
  const float *attn_norm = nullptr, *ffn_norm = nullptr;
  Q6Mat q{}, k{}, v{}, o{};
  const float *q_norm = nullptr, *k_norm = nullptr;
  Q6Mat in_proj{}, out_proj{};
  const float* conv_w = nullptr;
  bool dense = false;
  Q6Mat gate{}, up{}, down{};
  const float *router = nullptr, *bias = nullptr;
  Q6Mat gate_x{}, up_x{}, down_x{};
};

struct CudaError {
  cudaError_t e;
};

#define CK(call)                                  \
  do {                                            \
    cudaError_t _e = (call);                      \
    if (_e != cudaSuccess) throw ::lfm::CudaError{_e}; \
  } while (0)

// Per-token session map of a batched decode step: token j is at position
// pos[j] of session sess[j]; sessions' caches and conv states lie kv_stride /
// conv_stride elements apart, starting at session 0's.
struct TokBatch {
  const int* pos = nullptr;
  const int* sess = nullptr;
  __half* kc = nullptr;
  __half* vc = nullptr;
  float* conv = nullptr;
  size_t kv_stride = 0, conv_stride = 0;
  float* part = nullptr;  // attention split partials
};

// Device state of the independent sessions (lfm_batch_*).
struct BatchState {
  uint32_t nsess = 0, ctx = 0;
  __half *kc = nullptr, *vc = nullptr;  // [session][attn layer][kv head][ctx][64]
  float* conv = nullptr;                // [session][conv layer][2048][2]
  size_t kv_stride = 0, conv_stride = 0;
  int* map = nullptr;                   // per step: tokens | positions | sessions
  int* next = nullptr;
  float* logits = nullptr;              // [session][vocab]
  float* attn_part = nullptr;           // attention split partials of one step
  uint32_t last_count = 0;              // entries of the last lfm_batch_decode step
  std::vector<int> h_map;
  std::vector<void*> allocs;
};

}  // namespace

// Several sessions' fresh prompts in one pass of the layer stack: session
// sess[i]'s tokens are rows off[i] .. off[i] + len[i] - 1 (host arrays).
struct SessRuns {
  int count = 0;
  const uint32_t* sess = nullptr;
  const int* off = nullptr;
  const int* len = nullptr;
};

struct EngineImpl {
  int device = 0;
  int sms = 148;
  std::string name;
  cudaStream_t stream = nullptr;
  lfm_hparams hp{};
  std::vector<LayerW> layers;
  Q6Mat embd{};
  const float* out_norm = nullptr;
  std::vector<void*> weight_allocs;
  size_t weight_bytes = 0;
  int n_attn = 0, n_conv = 0, n_moe = 0;
  bool pdl = false;  // programmatic dependent launch between decode kernels (LFM_PDL=1)
  bool use_graph = true;
  bool use_mvt = true;  // TMA-staged decode matvecs
  bool use_step = true;  // persistent decode step (LFM_STEP=0 selects the kernel chain)
  bool use_tc = true;    // tensor-core Q6_K prompt GEMMs (LFM_PREFILL=fp32 selects the CUDA-core GEMMs)
  // prompt GEMMs read load-time expanded fp16 weights (LFM_PREFILL_X16=0: dequantise on chip)
  bool use_x16 = true;
  std::unordered_map<const void*, const __half*> x16_of;  // Q6Mat::q -> its fp16 A operand
  const __half* x16(const Q6Mat& W) const {
    auto it = x16_of.find(W.q);
    return it == x16_of.end() ? nullptr : it->second;
  }
  int tc_min = 1;        // token batches of at least this many tokens use them (LFM_TC_MIN_TOKENS)
  TcScratch tcs;
  std::string step_reason;  // why the persistent step is not in use
  StepCtl* ctl = nullptr;
  StepStage* d_stages = nullptr;
  int nstages = 0;
  unsigned long long* trace = nullptr;  // [stage][cta][4] globaltimer stamps
  bool trace_on = false;
  uint64_t step_epochs = 0;  // steps since the control block was zeroed
  std::string info;

  // resident state
  uint32_t ctx = 4096;
  bool state_ready = false;
  uint32_t state_ctx = 0;
  __half *kc = nullptr, *vc = nullptr;
  float* conv_state = nullptr;
  float2* rope = nullptr;
  // decode buffers
  float *x = nullptr, *qkv = nullptr, *a = nullptr, *gated = nullptr, *sw = nullptr, *down = nullptr,
        *logits = nullptr, *attn_part = nullptr, *selw = nullptr, *router_lg = nullptr;
  int* sel = nullptr;
  int* io = nullptr;  // [0] token, [1] position, [2] next token, [3] loop index, [4] device error word
  unsigned* counters = nullptr;
  float2* am_part = nullptr;
  int* h_io = nullptr;  // pinned
  // prefill buffers (capacity ncap tokens)
  int ncap = 0;
  float *px = nullptr, *ph = nullptr, *pqkv = nullptr, *pa = nullptr, *pbcx = nullptr, *pgated = nullptr,
        *pgate = nullptr, *pup = nullptr, *psw = nullptr, *pdown = nullptr, *prlog = nullptr, *pselw = nullptr;
  int *psel = nullptr, *pgroups = nullptr;
  uint32_t* pids = nullptr;
  std::vector<void*> state_allocs, prefill_allocs;

  cudaGraphExec_t graph = nullptr;
  cudaGraphExec_t loop_graph = nullptr;  // advance + decode step, token fed back on device
  // the batched decode step (lfm_batch_decode) of one session count as a CUDA
  // graph: captured at the second step with that count, replayed after
  cudaGraphExec_t bgraph = nullptr;
  int bgraph_n = 0, bgraph_nl = 0, beager_n = 0;
  // a prompt chunk of n <= LFM_PREFILL_CHUNK tokens of the engine's own
  // session as a CUDA graph per n (its first position is read from io[1]):
  // captured at the second chunk with that n, replayed after
  struct PGraph {
    int n = 0, nl = 0;
    cudaGraphExec_t exec = nullptr;
  };
  static constexpr int PGRAPH_MAX = 8;
  std::vector<PGraph> pgraphs;   // at most PGRAPH_MAX, oldest first
  std::vector<int> pgraph_seen;  // chunk lengths run once eagerly
  bool session_swap = false;     // kc / vc / conv_state point into a session slot
  uint32_t* loop_tokens = nullptr;       // device record of loop tokens
  uint32_t loop_cap = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  lfm_counters ctr{};
  std::string err;
  int launches_per_decode = 0;

  // expert-parallel prompt path (ep.h): communicator and exchange buffers
  EpComm ep;
  bool ep_on = false;
  bool ep_now = false;  // the prompt being run uses the expert-parallel MoE layers
  int ep_cap_send = 0, ep_cap_recv = 0;  // slots
  int ep_total = 0;  // tokens of all ranks in the current expert-parallel prompt
  float *ep_send = nullptr, *ep_recv = nullptr, *ep_back = nullptr, *ep_local = nullptr;
  int32_t *ep_send_tag = nullptr, *ep_recv_tag = nullptr, *ep_order = nullptr, *ep_sel4 = nullptr,
          *ep_counts = nullptr, *ep_all = nullptr;
  std::vector<void*> ep_allocs;
  std::vector<int32_t> h_sel, h_order, h_counts, h_all;

  ~EngineImpl() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    // free_state() destroys the graph execs (each exactly once)
    if (loop_tokens) cudaFree(loop_tokens);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    free_prefill();
    free_state();
    batch_free();
    for (auto& kv : x16_of) cudaFree((void*)kv.second);
    for (void* p : ep_allocs) cudaFree(p);
    ep_comm_destroy(ep);
    for (void* p : weight_allocs) cudaFree(p);
    if (h_io) cudaFreeHost(h_io);
    if (stream) cudaStreamDestroy(stream);
  }

  template <class T>
  T* dalloc(std::vector<void*>& list, size_t count) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 16)));
    list.push_back(p);
    return (T*)p;
  }
  void free_state() {
    drop_bgraph();  // both hold the status word's and the session state's addresses
    drop_pgraphs();
    for (void* p : state_allocs) cudaFree(p);
    state_allocs.clear();
    state_ready = false;
    ctl = nullptr;
    d_stages = nullptr;
    trace = nullptr;
    if (graph) {
      cudaGraphExecDestroy(graph);
      graph = nullptr;
    }
    if (loop_graph) {
      cudaGraphExecDestroy(loop_graph);
      loop_graph = nullptr;
    }
  }
  void free_prefill() {
    drop_bgraph();  // both hold the prompt buffers' addresses
    drop_pgraphs();
    for (void* p : prefill_allocs) cudaFree(p);
    prefill_allocs.clear();
    ncap = 0;
  }
  void drop_bgraph() {
    if (bgraph) {
      cudaGraphExecDestroy(bgraph);
      bgraph = nullptr;
    }
    bgraph_n = bgraph_nl = beager_n = 0;
  }
  void drop_pgraphs() {
    for (PGraph& g : pgraphs) cudaGraphExecDestroy(g.exec);
    pgraphs.clear();
    pgraph_seen.clear();
  }

  // ------------------------------------------------------------- loading
  bool load(const char* path);
  void upload_q6(const GgufFile& f, const GgufTensor& t, int rows, int nb, Q6Mat& out,
                 std::vector<uint8_t>& src, std::vector<uint8_t>& dst);
  const float* upload_f32(const GgufFile& f, const GgufTensor& t);

  // --------------------------------------------------------------- state
  void ensure_state();
  void ensure_prefill(int n);
  void build_step();
  bool step_active() const { return use_step && ctl != nullptr; }
  void drop_graphs();
  void step_epoch_guard(uint64_t steps);

  // ------------------------------------------------------------- forward
  void enqueue_decode(cudaStream_t s, bool pdl_on);
  void enqueue_ffn(const LayerW& L, float* xr, const LaunchCfg& c, unsigned* err);
  void check_device_error();
  void run_decode(uint32_t token, uint32_t pos);
  void run_prefill(const uint32_t* ids, int n, uint32_t start, bool ep_mode = false);
  void ep_moe(const LayerW& L, const float* rows, int n, float* xres);
  void ep_reserve(int send_slots, int recv_slots);
  void enqueue_layers(int n, uint32_t start, const TokBatch* tb, int& nl, const SessRuns* runs = nullptr,
                      const int* start_dev = nullptr);
  void batch_prefill_many(const uint32_t* sess, const uint32_t* ids, const uint32_t* lens, int count,
                          uint32_t* next);
  BatchState batch;
  void batch_create(uint32_t nsess);
  void batch_free();
  uint32_t batch_prefill(uint32_t sess, const uint32_t* ids, int n, bool ep_mode = false);
  void run_batch_decode(uint32_t count, const uint32_t* tokens, const uint32_t* pos, const uint32_t* sess,
                        uint32_t* next);
  void run_loop(uint32_t steps, uint32_t* out_tokens);
  std::vector<uint8_t> snapshot(uint32_t valid);
  void restore(uint32_t valid, const uint8_t* buf, size_t len);
};

namespace {

void set_err(EngineImpl* e, const std::string& m) {
  if (e) e->err = m;
  g_error = m;
}

}  // namespace

void EngineImpl::upload_q6(const GgufFile& f, const GgufTensor& t, int rows, int nb, Q6Mat& out,
                           std::vector<uint8_t>& src, std::vector<uint8_t>& dst) {
  const size_t bytes = q6_total_bytes(rows, nb);
  if (t.nbytes != bytes) throw std::runtime_error("tensor " + t.name + " has unexpected size");
  src.resize(bytes);
  dst.resize(bytes);
  if (!f.read(t, 0, bytes, src.data())) throw std::runtime_error("read tensor " + t.name);
  const int nthreads = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  const size_t per = (rows + nthreads - 1) / nthreads;
  for (int i = 0; i < nthreads; i++) {
    const size_t r0 = i * per;
    if (r0 >= (size_t)rows) break;
    const size_t r1 = std::min<size_t>(rows, r0 + per);
    th.emplace_back([&, r0, r1] {
      q6_repack_rows(src.data() + r0 * nb * QB, r0, r1 - r0, nb, rows, dst.data());
    });
  }
  for (auto& x : th) x.join();
  void* d = nullptr;
  CK(cudaMalloc(&d, bytes));
  weight_allocs.push_back(d);
  CK(cudaMemcpy(d, dst.data(), bytes, cudaMemcpyHostToDevice));
  weight_bytes += bytes;
  out = q6_view(d, rows, nb);
  if (use_x16 && use_tc) {
    // the prompt GEMMs' fp16 A operand of this matrix (2 bytes per weight);
    // without room for it the prompt GEMMs dequantise on chip instead
    void* x = nullptr;
    if (cudaMalloc(&x, (size_t)rows * nb * QK * 2) != cudaSuccess) {
      cudaGetLastError();
      use_x16 = false;
      for (auto& kv : x16_of) cudaFree((void*)kv.second);
      x16_of.clear();
      return;
    }
    CK(q6_expand_f16(out, (__half*)x, stream));
    CK(cudaStreamSynchronize(stream));
    x16_of[out.q] = (const __half*)x;
  }
}

const float* EngineImpl::upload_f32(const GgufFile& f, const GgufTensor& t) {
  std::vector<uint8_t> buf(t.nbytes);
  if (!f.read(t, 0, t.nbytes, buf.data())) throw std::runtime_error("read tensor " + t.name);
  void* d = nullptr;
  CK(cudaMalloc(&d, t.nbytes));
  weight_allocs.push_back(d);
  CK(cudaMemcpy(d, buf.data(), t.nbytes, cudaMemcpyHostToDevice));
  weight_bytes += t.nbytes;
  return (const float*)d;
}

// load_hyperparams (lfm.rs:102-145): the metadata keys, the reference's
// hard-coded geometry check and its message, plus the limits of this engine
// (short-conv L_cache 3, dense n_ff 7168, 8 KV heads per attention layer).
// Needs no device.
static bool read_hparams(const GgufFile& f, lfm_hparams& hp, std::string& err) {
  uint32_t nl, dim, heads, vocab, ne, nu, eff, nff;
  std::vector<uint32_t> kvh;
  const char* keys[] = {"lfm2moe.block_count", "lfm2moe.embedding_length", "lfm2moe.attention.head_count",
                        "lfm2moe.vocab_size", "lfm2moe.expert_count", "lfm2moe.expert_used_count",
                        "lfm2moe.expert_feed_forward_length", "lfm2moe.feed_forward_length"};
  uint32_t* outs[] = {&nl, &dim, &heads, &vocab, &ne, &nu, &eff, &nff};
  for (int i = 0; i < 8; i++)
    if (!f.meta_u32(keys[i], *outs[i])) {
      err = std::string("metadata ") + keys[i] + " not a u32";
      return false;
    }
  if (!f.meta_u32_array("lfm2moe.attention.head_count_kv", kvh)) {
    err = "metadata lfm2moe.attention.head_count_kv not an array";
    return false;
  }
  if (dim != DIM || heads != HEADS || nl != 24 || vocab != 128000 || ne != N_EXPERT || nu != N_USED ||
      eff != EXPERT_FF) {
    char b[256];
    snprintf(b, sizeof b,
             "unsupported geometry: dim=%u heads=%u layers=%u vocab=%u n_expert=%u n_used=%u expert_ff=%u", dim,
             heads, nl, vocab, ne, nu, eff);
    err = b;
    return false;
  }
  if (kvh.size() != nl) {
    err = "head_count_kv length differs from block_count";
    return false;
  }
  hp = lfm_hparams{};
  hp.dim = dim;
  hp.heads = heads;
  hp.head_dim = HEAD_DIM;
  hp.n_layers = nl;
  hp.vocab = vocab;
  hp.n_expert = ne;
  hp.n_used = nu;
  hp.expert_ff = eff;
  hp.n_ff = nff;
  hp.dense_lead = f.meta_u32_default("lfm2moe.leading_dense_block_count", 2);
  hp.conv_l_cache = f.meta_u32_default("lfm2moe.shortconv.l_cache", 3);
  hp.eos = f.meta_u32_default("tokenizer.ggml.eos_token_id", 124900);
  if (!f.meta_f32("lfm2moe.attention.layer_norm_rms_epsilon", hp.eps)) {
    err = "metadata lfm2moe.attention.layer_norm_rms_epsilon not an f32";
    return false;
  }
  if (!f.meta_f32("lfm2moe.rope.freq_base", hp.rope_theta)) {
    err = "metadata lfm2moe.rope.freq_base not an f32";
    return false;
  }
  for (uint32_t l = 0; l < nl; l++) hp.kv_heads[l] = kvh[l];
  if (hp.conv_l_cache != 3 || nff != N_FF || hp.dense_lead > nl) {
    err = "unsupported short-conv / dense FFN geometry";
    return false;
  }
  for (uint32_t l = 0; l < nl; l++)
    if (kvh[l] != 0 && kvh[l] != KV_HEADS) {
      err = "attention layers must have 8 KV heads";
      return false;
    }
  return true;
}

// Every tensor the engine uploads, with its GGML type and dimensions (the
// names and shapes of the reference's loader, lfm.rs:147-190 and
// gpu_lfm.rs:51-115). Reads no payload and needs no device.
static bool check_tensors(const GgufFile& f, const lfm_hparams& hp, std::string& err) {
  auto need = [&](const std::string& name, uint32_t type, std::vector<uint64_t> ne_) {
    const GgufTensor* t = f.tensor(name);
    if (!t) {
      err = "missing tensor " + name;
      return false;
    }
    if (t->type != type || t->ne != ne_) {
      err = "tensor " + name + " has unexpected type/shape";
      return false;
    }
    return true;
  };
  if (!need("token_embd.weight", 14, {DIM, hp.vocab}) || !need("token_embd_norm.weight", 0, {DIM})) return false;
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const std::string p = "blk." + std::to_string(l) + ".";
    if (!need(p + "attn_norm.weight", 0, {DIM}) || !need(p + "ffn_norm.weight", 0, {DIM})) return false;
    bool ok = hp.kv_heads[l] > 0
                  ? need(p + "attn_q.weight", 14, {DIM, DIM}) && need(p + "attn_k.weight", 14, {DIM, 512}) &&
                        need(p + "attn_v.weight", 14, {DIM, 512}) && need(p + "attn_output.weight", 14, {DIM, DIM}) &&
                        need(p + "attn_q_norm.weight", 0, {HEAD_DIM}) && need(p + "attn_k_norm.weight", 0, {HEAD_DIM})
                  : need(p + "shortconv.in_proj.weight", 14, {DIM, 3 * DIM}) &&
                        need(p + "shortconv.out_proj.weight", 14, {DIM, DIM}) &&
                        need(p + "shortconv.conv.weight", 0, {3, DIM});
    if (!ok) return false;
    ok = l < hp.dense_lead
             ? need(p + "ffn_gate.weight", 14, {DIM, N_FF}) && need(p + "ffn_up.weight", 14, {DIM, N_FF}) &&
                   need(p + "ffn_down.weight", 14, {N_FF, DIM})
             : need(p + "ffn_gate_inp.weight", 0, {DIM, N_EXPERT}) && need(p + "exp_probs_b.bias", 0, {N_EXPERT}) &&
                   need(p + "ffn_gate_exps.weight", 14, {DIM, EXPERT_FF, N_EXPERT}) &&
                   need(p + "ffn_up_exps.weight", 14, {DIM, EXPERT_FF, N_EXPERT}) &&
                   need(p + "ffn_down_exps.weight", 14, {EXPERT_FF, DIM, N_EXPERT});
    if (!ok) return false;
  }
  return true;
}

bool EngineImpl::load(const char* path) {
  GgufFile f;
  if (!f.open(path)) {
    set_err(this, "parse GGUF header: " + f.err());
    return false;
  }
  std::string verr;
  if (!read_hparams(f, hp, verr) || !check_tensors(f, hp, verr)) {
    set_err(this, verr);
    return false;
  }
  const uint32_t nl = hp.n_layers, vocab = hp.vocab;
  std::vector<uint32_t> kvh(hp.kv_heads, hp.kv_heads + nl);

  auto need = [&](const std::string& name, uint32_t type, std::vector<uint64_t> ne_) -> const GgufTensor& {
    const GgufTensor* t = f.tensor(name);
    if (!t) throw std::runtime_error("missing tensor " + name);
    if (t->type != type || t->ne != ne_) throw std::runtime_error("tensor " + name + " has unexpected type/shape");
    return *t;
  };
  std::vector<uint8_t> src, dst;
  try {
    CK(cudaSetDevice(device));
    const GgufTensor& te = need("token_embd.weight", 14, {DIM, vocab});
    upload_q6(f, te, vocab, DIM / QK, embd, src, dst);
    out_norm = upload_f32(f, need("token_embd_norm.weight", 0, {DIM}));
    layers.resize(nl);
    for (uint32_t l = 0; l < nl; l++) {
      LayerW& L = layers[l];
      const std::string p = "blk." + std::to_string(l) + ".";
      L.attn_norm = upload_f32(f, need(p + "attn_norm.weight", 0, {DIM}));
      L.ffn_norm = upload_f32(f, need(p + "ffn_norm.weight", 0, {DIM}));
      if (kvh[l] > 0) {
        L.attn = true;
        L.attn_idx = n_attn++;
        upload_q6(f, need(p + "attn_q.weight", 14, {DIM, DIM}), DIM, DIM / QK, L.q, src, dst);
        upload_q6(f, need(p + "attn_k.weight", 14, {DIM, 512}), 512, DIM / QK, L.k, src, dst);
        upload_q6(f, need(p + "attn_v.weight", 14, {DIM, 512}), 512, DIM / QK, L.v, src, dst);
        upload_q6(f, need(p + "attn_output.weight", 14, {DIM, DIM}), DIM, DIM / QK, L.o, src, dst);
        L.q_norm = upload_f32(f, need(p + "attn_q_norm.weight", 0, {HEAD_DIM}));
        L.k_norm = upload_f32(f, need(p + "attn_k_norm.weight", 0, {HEAD_DIM}));
      } else {
        L.conv_idx = n_conv++;
        upload_q6(f, need(p + "shortconv.in_proj.weight", 14, {DIM, 3 * DIM}), 3 * DIM, DIM / QK, L.in_proj, src,
                  dst);
        upload_q6(f, need(p + "shortconv.out_proj.weight", 14, {DIM, DIM}), DIM, DIM / QK, L.out_proj, src, dst);
        L.conv_w = upload_f32(f, need(p + "shortconv.conv.weight", 0, {3, DIM}));
      }
      if (l < hp.dense_lead) {
        L.dense = true;
        upload_q6(f, need(p + "ffn_gate.weight", 14, {DIM, N_FF}), N_FF, DIM / QK, L.gate, src, dst);
        upload_q6(f, need(p + "ffn_up.weight", 14, {DIM, N_FF}), N_FF, DIM / QK, L.up, src, dst);
        upload_q6(f, need(p + "ffn_down.weight", 14, {N_FF, DIM}), DIM, N_FF / QK, L.down, src, dst);
      } else {
        L.moe_idx = n_moe++;
        L.router = upload_f32(f, need(p + "ffn_gate_inp.weight", 0, {DIM, N_EXPERT}));
        L.bias = upload_f32(f, need(p + "exp_probs_b.bias", 0, {N_EXPERT}));
        upload_q6(f, need(p + "ffn_gate_exps.weight", 14, {DIM, EXPERT_FF, N_EXPERT}), N_EXPERT * EXPERT_FF,
                  DIM / QK, L.gate_x, src, dst);
        upload_q6(f, need(p + "ffn_up_exps.weight", 14, {DIM, EXPERT_FF, N_EXPERT}), N_EXPERT * EXPERT_FF,
                  DIM / QK, L.up_x, src, dst);
        upload_q6(f, need(p + "ffn_down_exps.weight", 14, {EXPERT_FF, DIM, N_EXPERT}), N_EXPERT * DIM,
                  EXPERT_FF / QK, L.down_x, src, dst);
      }
    }
  } catch (const std::exception& ex) {
    set_err(this, ex.what());
    return false;
  } catch (const CudaError& ce) {
    set_err(this, std::string("CUDA: ") + cudaGetErrorString(ce.e));
    return false;
  }
  return true;
}

void EngineImpl::ensure_state() {
  if (state_ready && state_ctx == ctx) return;
  free_state();
  const size_t kvsz = (size_t)std::max(n_attn, 1) * KV_HEADS * ctx * HEAD_DIM;
  kc = dalloc<__half>(state_allocs, kvsz);
  vc = dalloc<__half>(state_allocs, kvsz);
  CK(cudaMemsetAsync(kc, 0, kvsz * 2, stream));
  CK(cudaMemsetAsync(vc, 0, kvsz * 2, stream));
  conv_state = dalloc<float>(state_allocs, (size_t)std::max(n_conv, 1) * DIM * 2);
  CK(cudaMemsetAsync(conv_state, 0, (size_t)std::max(n_conv, 1) * DIM * 2 * 4, stream));
  // RoPE table: theta = pos * tscale^p, tscale = theta_base^(-2/64) (lfm.rs:251-256).
  {
    std::vector<float2> t((size_t)ctx * 32);
    float (*volatile p_powf)(float, float) = powf;
    float (*volatile p_sinf)(float) = sinf;
    float (*volatile p_cosf)(float) = cosf;
    const float tscale = p_powf(hp.rope_theta, -2.0f / (float)HEAD_DIM);
    for (uint32_t pos = 0; pos < ctx; pos++)
      for (int p = 0; p < 32; p++) {
        const float theta = (float)pos * __builtin_powif(tscale, p);
        t[(size_t)pos * 32 + p] = make_float2(p_cosf(theta), p_sinf(theta));
      }
    rope = dalloc<float2>(state_allocs, t.size());
    CK(cudaMemcpy(rope, t.data(), t.size() * sizeof(float2), cudaMemcpyHostToDevice));
  }
  x = dalloc<float>(state_allocs, DIM);
  qkv = dalloc<float>(state_allocs, DIM + 2 * KV_HEADS * HEAD_DIM);
  a = dalloc<float>(state_allocs, DIM);
  gated = dalloc<float>(state_allocs, DIM);
  sw = dalloc<float>(state_allocs, std::max(N_FF, N_USED * EXPERT_FF));
  down = dalloc<float>(state_allocs, N_USED * DIM);
  logits = dalloc<float>(state_allocs, hp.vocab);
  const int nsplit = (ctx + ATTN_SPLIT - 1) / ATTN_SPLIT;
  attn_part = dalloc<float>(state_allocs, (size_t)KV_HEADS * nsplit * 4 * (HEAD_DIM + 2));
  sel = dalloc<int>(state_allocs, 8);
  router_lg = dalloc<float>(state_allocs, N_EXPERT);
  selw = dalloc<float>(state_allocs, 8);
  io = dalloc<int>(state_allocs, 8);
  CK(cudaMemsetAsync(io, 0, 8 * 4, stream));
  counters = dalloc<unsigned>(state_allocs, 1024);
  CK(cudaMemsetAsync(counters, 0, 1024 * 4, stream));
  am_part = dalloc<float2>(state_allocs, 4096);
  ctl = nullptr;
  d_stages = nullptr;
  trace = nullptr;
  if (use_step) build_step();
  CK(cudaStreamSynchronize(stream));
  state_ready = true;
  state_ctx = ctx;
}

// The step's barrier counters grow by one grid per step; zero the control
// block long before they could wrap (2^32 / 148 steps), between launches.
void EngineImpl::step_epoch_guard(uint64_t steps) {
  if (!step_active()) return;
  if (step_epochs + steps > (1ull << 24)) {
    CK(cudaMemsetAsync(ctl, 0, sizeof(StepCtl), stream));
    step_epochs = 0;
  }
  step_epochs += steps;
}

void EngineImpl::drop_graphs() {
  if (graph) {
    cudaGraphExecDestroy(graph);
    graph = nullptr;
  }
  if (loop_graph) {
    cudaGraphExecDestroy(loop_graph);
    loop_graph = nullptr;
  }
}

// Stage list of the persistent decode step: the reference's resident decode
// graph (resident_graph.rs:226-546) in dependency order.
void EngineImpl::build_step() {
  cudaError_t e = step_prepare();
  if (e != cudaSuccess) {
    step_reason = std::string("persistent step unavailable: ") + cudaGetErrorString(e) + " (" +
                  step_occupancy_report() + ")";
    cudaGetLastError();
    return;
  }
  if (sms > STEP_MAX_CTAS) {
    step_reason = "persistent step unavailable: more SMs than the control block holds";
    return;
  }
  std::vector<StepStage> st;
  auto add = [&](int type) -> StepStage& {
    st.push_back(StepStage{});
    st.back().type = type;
    return st.back();
  };
  add(ST_EMBED);
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const LayerW& L = layers[l];
    if (L.attn) {
      StepStage& q = add(ST_QKV);
      q.W = L.q, q.W2 = L.k, q.W3 = L.v;
      q.xin = x, q.norm = L.attn_norm, q.out = qkv;
      q.ntiles = (L.q.rows + L.k.rows + L.v.rows) / 16;
      StepStage& at = add(ST_ATTN);
      at.xin = qkv, at.q_norm = L.q_norm, at.k_norm = L.k_norm, at.out = a;
      at.kc = kc + (size_t)L.attn_idx * KV_HEADS * ctx * HEAD_DIM;
      at.vc = vc + (size_t)L.attn_idx * KV_HEADS * ctx * HEAD_DIM;
      StepStage& o = add(ST_RESID);
      o.W = L.o, o.xin = a, o.resid = x, o.ntiles = L.o.rows / 16;
    } else {
      StepStage& c = add(ST_CONV);
      c.W = L.in_proj, c.xin = x, c.norm = L.attn_norm, c.conv_w = L.conv_w;
      c.state = conv_state + (size_t)L.conv_idx * DIM * 2, c.out = gated, c.ntiles = DIM / 8;
      StepStage& o = add(ST_RESID);
      o.W = L.out_proj, o.xin = gated, o.resid = x, o.ntiles = L.out_proj.rows / 16;
    }
    if (L.dense) {
      StepStage& g = add(ST_SWIGLU);
      g.W = L.gate, g.W2 = L.up, g.xin = x, g.norm = L.ffn_norm, g.out = sw, g.ntiles = L.gate.rows / 8;
      StepStage& d = add(ST_DOWN28);
      d.W = L.down, d.xin = sw, d.resid = x, d.ntiles = L.down.rows / 4;
    } else {
      // the residual stage just added publishes this layer's router partials
      const int dep = (int)st.size() - 1;
      st[dep].rw = L.router, st[dep].bias = L.bias, st[dep].norm = L.ffn_norm;
      StepStage& g = add(ST_XSWIGLU);
      g.W = L.gate_x, g.W2 = L.up_x, g.xin = x, g.norm = L.ffn_norm, g.out = sw, g.ff = EXPERT_FF;
      g.ntiles = N_USED * EXPERT_FF / 8, g.dep = dep;
      StepStage& d = add(ST_XDOWN);
      d.W = L.down_x, d.xin = sw, d.resid = x, d.ff = EXPERT_FF, d.ntiles = DIM / 4, d.dep = dep;
    }
  }
  StepStage& h = add(ST_LMHEAD);
  h.W = embd, h.xin = x, h.norm = out_norm, h.out = logits, h.ntiles = embd.rows / 16;
  for (const StepStage& q : st) {
    const bool partial = q.type == ST_CONV || q.type == ST_SWIGLU || q.type == ST_XSWIGLU || q.type == ST_XDOWN ||
                         q.type == ST_DOWN28;
    if (partial && (q.ntiles + sms - 1) / sms > STEP_PART_TILES) {
      step_reason = "persistent step unavailable: too few SMs for the per-CTA partial buffer";
      return;
    }
    if (q.type == ST_XSWIGLU && q.ntiles / sms < STEP_PRODUCERS) {
      step_reason = "persistent step unavailable: more SMs than the routed stages have tiles for every producer";
      return;
    }
  }
  if ((int)st.size() > STEP_MAX_STAGES || embd.rows % 16 != 0) {
    step_reason = "persistent step unavailable: model shape outside the step kernel's tiling";
    return;
  }
  nstages = (int)st.size();
  d_stages = dalloc<StepStage>(state_allocs, st.size());
  CK(cudaMemcpy(d_stages, st.data(), st.size() * sizeof(StepStage), cudaMemcpyHostToDevice));
  ctl = dalloc<StepCtl>(state_allocs, 1);
  CK(cudaMemsetAsync(ctl, 0, sizeof(StepCtl), stream));
  step_epochs = 0;
  trace = dalloc<unsigned long long>(state_allocs, (size_t)STEP_MAX_STAGES * STEP_MAX_CTAS * STEP_TRACE_FIELDS);
  CK(cudaMemsetAsync(trace, 0, (size_t)STEP_MAX_STAGES * STEP_MAX_CTAS * STEP_TRACE_FIELDS * 8, stream));
  step_reason.clear();
}

void EngineImpl::ensure_prefill(int n) {
  if (n <= ncap) return;
  free_prefill();
  const int cap = std::max(n, (int)LFM_PREFILL_CHUNK);
  const size_t N = cap;
  px = dalloc<float>(prefill_allocs, N * DIM);
  ph = dalloc<float>(prefill_allocs, N * DIM);
  pqkv = dalloc<float>(prefill_allocs, N * (DIM + 2 * KV_HEADS * HEAD_DIM));
  pa = dalloc<float>(prefill_allocs, N * DIM);
  pbcx = dalloc<float>(prefill_allocs, N * 3 * DIM);
  pgated = dalloc<float>(prefill_allocs, N * DIM);
  const size_t wide = std::max<size_t>(N * N_FF, N * N_USED * EXPERT_FF);
  pgate = dalloc<float>(prefill_allocs, wide);
  pup = dalloc<float>(prefill_allocs, wide);
  psw = dalloc<float>(prefill_allocs, wide);
  pdown = dalloc<float>(prefill_allocs, N * N_USED * DIM);
  prlog = dalloc<float>(prefill_allocs, N * N_EXPERT);
  psel = dalloc<int>(prefill_allocs, N * N_USED);
  pselw = dalloc<float>(prefill_allocs, N * N_USED);
  pgroups = dalloc<int>(prefill_allocs, (size_t)N_EXPERT * (N + 1));
  pids = dalloc<uint32_t>(prefill_allocs, N);
  // operand of the tensor-core prompt GEMMs: dense (K up to 7168) or grouped (K up to 2048)
  tcs.rows = tc_scratch_rows(cap);
  tcs.halves = std::max<size_t>(2 * ((N + 127) / 128 * 128) * N_FF, 2 * tcs.rows * DIM);
  tcs.xg = dalloc<__half>(prefill_allocs, tcs.halves);
  tcs.inv = dalloc<float>(prefill_allocs, tcs.rows);
  tcs.tiles = dalloc<int>(prefill_allocs, 1 + 2 * (size_t)tc_max_tiles_cap(cap));
  tcs.slots = dalloc<int>(prefill_allocs, tcs.rows);
  tcs.rowof = dalloc<int>(prefill_allocs, N * N_USED);
  tcs.part_cap = (size_t)16 * std::min<size_t>(N, 128) * N_FF;  // split-K partials of one token tile
  tcs.part = dalloc<float>(prefill_allocs, tcs.part_cap);
  ncap = cap;
}

// One decode step for the token/position in io[0], io[1]; next token -> io[2].
void EngineImpl::enqueue_decode(cudaStream_t s, bool pdl_on) {
  LaunchCfg c;
  c.stream = s;
  c.pdl = pdl_on;
  c.sms = sms;
  int n = 0;
  const float eps = hp.eps;
  unsigned* err = (unsigned*)(io + 4);
  if (step_active()) {
    StepParams p = {};
    p.stages = d_stages;
    p.nstages = nstages;
    p.ctl = ctl;
    p.io = io;
    p.rope = rope;
    p.attn_part = attn_part;
    p.ctx = (int)ctx;
    p.eps = eps;
    p.embd = embd;
    p.x = x;
    p.trace = trace_on ? trace : nullptr;
    CK(step_launch(p, sms, s));
    launches_per_decode = 1;
    return;
  }
  embed_token(embd, io + 0, x, err, c);
  n++;
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const LayerW& L = layers[l];
    const XSrc xa{x, L.attn_norm, eps};
    if (L.attn) {
      if (use_mvt) {
        mvt_qkv(L.q, L.k, L.v, xa, qkv, err, c);
        n -= 2;
      } else {
        mv_plain(L.q, xa, qkv, c);
        mv_plain(L.k, xa, qkv + DIM, c);
        mv_plain(L.v, xa, qkv + DIM + KV_HEADS * HEAD_DIM, c);
      }
      AttnDecodeArgs aa;
      aa.qkv = qkv;
      aa.q_norm = L.q_norm;
      aa.k_norm = L.k_norm;
      aa.rope = rope;
      aa.pos = io + 1;
      aa.kc = kc + (size_t)L.attn_idx * KV_HEADS * ctx * HEAD_DIM;
      aa.vc = vc + (size_t)L.attn_idx * KV_HEADS * ctx * HEAD_DIM;
      aa.part = attn_part;
      aa.counters = counters + 8 * L.attn_idx;
      aa.out = a;
      aa.ctx = (int)ctx;
      aa.eps = eps;
      attn_decode(aa, c);
      if (use_mvt) mvt_resid(L.o, XSrc{a, nullptr, 0.f}, x, err, c);
      else mv_resid(L.o, XSrc{a, nullptr, 0.f}, x, c);
      n += 5;
    } else {
      float* st = conv_state + (size_t)L.conv_idx * DIM * 2;
      if (use_mvt) {
        mvt_conv(L.in_proj, xa, L.conv_w, st, gated, err, c);
        mvt_resid(L.out_proj, XSrc{gated, nullptr, 0.f}, x, err, c);
      } else {
        mv_conv(L.in_proj, xa, L.conv_w, st, gated, c);
        mv_resid(L.out_proj, XSrc{gated, nullptr, 0.f}, x, c);
      }
      n += 2;
    }
    enqueue_ffn(L, x, c, err);
    n += L.dense ? 2 : 3;
  }
  if (use_mvt) mvt_lmhead(embd, XSrc{x, out_norm, eps}, logits, am_part, counters + 128, io + 2, err, c);
  else mv_lmhead(embd, XSrc{x, out_norm, eps}, logits, am_part, counters + 128, io + 2, c);
  n++;
  launches_per_decode = n;
}

// FFN of one token whose residual row is `xr` (decode, and the last token of a
// prefill: lfm.rs:540-541).
void EngineImpl::enqueue_ffn(const LayerW& L, float* xr, const LaunchCfg& c, unsigned* err) {
  const XSrc xf{xr, L.ffn_norm, hp.eps};
  if (L.dense) {
    if (use_mvt) mvt_swiglu(L.gate, L.up, xf, sw, err, c);
    else mv_swiglu(L.gate, L.up, xf, sw, c);
    mv_down7168_resid(L.down, sw, xr, c);
  } else {
    router_top4_mc(L.router, L.bias, xf, router_lg, counters + 160, sel, selw, c);
    if (use_mvt) {
      mvt_expert_swiglu(L.gate_x, L.up_x, EXPERT_FF, xf, sel, sw, err, c);
      mvt_expert_down(L.down_x, EXPERT_FF, sw, sel, selw, down, xr, counters + 64 + L.moe_idx, err, c);
    } else {
      mv_expert_swiglu(L.gate_x, L.up_x, EXPERT_FF, xf, sel, sw, c);
      mv_expert_down(L.down_x, EXPERT_FF, sw, sel, selw, down, xr, counters + 64 + L.moe_idx, c);
    }
  }
}

void EngineImpl::run_decode(uint32_t token, uint32_t pos) {
  h_io[0] = (int)token;
  h_io[1] = (int)pos;
  step_epoch_guard(1);
  CK(cudaEventRecord(ev0, stream));
  if (use_graph) {
    if (!graph) {
      cudaGraph_t g;
      CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      cudaMemcpyAsync(io, h_io, 8, cudaMemcpyHostToDevice, stream);
      enqueue_decode(stream, pdl);
      cudaMemcpyAsync(h_io + 2, io + 2, 12, cudaMemcpyDeviceToHost, stream);
      if (step_active()) cudaMemcpyAsync(h_io + 5, &ctl->err, 4, cudaMemcpyDeviceToHost, stream);
      CK(cudaStreamEndCapture(stream, &g));
      cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
      cudaGraphDestroy(g);
      CK(e);
      ctr.graph_captures++;
    } else {
      ctr.graph_replays++;
    }
    CK(cudaGraphLaunch(graph, stream));
  } else {
    CK(cudaMemcpyAsync(io, h_io, 8, cudaMemcpyHostToDevice, stream));
    enqueue_decode(stream, pdl);
    CK(cudaMemcpyAsync(h_io + 2, io + 2, 12, cudaMemcpyDeviceToHost, stream));
    if (step_active()) CK(cudaMemcpyAsync(h_io + 5, &ctl->err, 4, cudaMemcpyDeviceToHost, stream));
  }
  CK(cudaEventRecord(ev1, stream));
  CK(cudaStreamSynchronize(stream));
  CK(cudaGetLastError());
  CK(cudaEventElapsedTime(&last_ms, ev0, ev1));
  ctr.kernel_launches += launches_per_decode;
  ctr.gpu_argmax++;
  check_device_error();
}

// The device status words (io[4] for the kernel chain, ctl->err for the
// persistent step) are raised by a bounded wait that timed out (codes 1-3) or
// by an embedding lookup of an out-of-range device-side token id (4). After a
// timeout the step's barrier counters are inconsistent, so the control block
// is zeroed (epoch 0) before the next step.
void EngineImpl::check_device_error() {
  const int chain = h_io[4], step = h_io[5];
  if (chain != 0 || step != 0) {
    h_io[4] = h_io[5] = 0;
    cudaMemsetAsync(io + 4, 0, 4, stream);
    if (ctl) cudaMemsetAsync(ctl, 0, sizeof(StepCtl), stream);
    step_epochs = 0;
    cudaStreamSynchronize(stream);
    const int code = step ? step : chain;
    throw std::runtime_error(std::string("device status word raised (") + (step ? "persistent step" : "kernel chain") +
                             " code " + std::to_string(code) + "): " +
                             (code == 4 ? "a device-side token id was outside the vocabulary"
                                        : "a bounded wait in a kernel timed out"));
  }
}

namespace {
// Feed the previous step's argmax back as the next input token (the
// device-side position scalar of the reference's replayed decode,
// kernels.rs:648-652) and record it.
__global__ void k_advance(int* io, uint32_t* rec) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int next = io[2];
  rec[io[3]] = (uint32_t)next;
  io[3] += 1;
  io[0] = next;
  io[1] += 1;
}
}  // namespace

// `steps` decode steps, each consuming the previous step's argmax, with no host
// round trip in between; out_tokens receives the argmax of every step.
// k_advance records each step's INPUT token (the previous step's argmax), so
// the argmax of step i is record i + 1, and the last step's is io[2].
void EngineImpl::run_loop(uint32_t steps, uint32_t* out_tokens) {
  if (steps > loop_cap) {
    if (loop_tokens) cudaFree(loop_tokens);
    CK(cudaMalloc(&loop_tokens, (size_t)steps * 4));
    loop_cap = steps;
    if (loop_graph) {
      cudaGraphExecDestroy(loop_graph);
      loop_graph = nullptr;
    }
  }
  if (!loop_graph) {
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    k_advance<<<1, 1, 0, stream>>>(io, loop_tokens);
    enqueue_decode(stream, pdl);
    CK(cudaStreamEndCapture(stream, &g));
    cudaError_t e = cudaGraphInstantiate(&loop_graph, g, 0);
    cudaGraphDestroy(g);
    CK(e);
    ctr.graph_captures++;
  }
  // io[0..2] hold the last decode step (token, position, next); io[3] = 0.
  CK(cudaMemsetAsync(io + 3, 0, 4, stream));
  step_epoch_guard(steps);
  CK(cudaEventRecord(ev0, stream));
  for (uint32_t i = 0; i < steps; i++) CK(cudaGraphLaunch(loop_graph, stream));
  CK(cudaEventRecord(ev1, stream));
  if (steps > 1)
    CK(cudaMemcpyAsync(out_tokens, loop_tokens + 1, (size_t)(steps - 1) * 4, cudaMemcpyDeviceToHost, stream));
  CK(cudaMemcpyAsync(out_tokens + steps - 1, io + 2, 4, cudaMemcpyDeviceToHost, stream));
  CK(cudaMemcpyAsync(h_io + 4, io + 4, 4, cudaMemcpyDeviceToHost, stream));
  if (step_active()) CK(cudaMemcpyAsync(h_io + 5, &ctl->err, 4, cudaMemcpyDeviceToHost, stream));
  CK(cudaStreamSynchronize(stream));
  CK(cudaGetLastError());
  CK(cudaEventElapsedTime(&last_ms, ev0, ev1));
  check_device_error();
  ctr.graph_replays += steps;
  ctr.kernel_launches += (uint64_t)steps * (launches_per_decode + 1);
  ctr.gpu_argmax += steps;
}

// n > 1 tokens starting at `start` (resident_graph.rs:226-551 with n columns).
// The layer stack over n token rows in px (embedded), leaving the final
// residual stream in px. tb == nullptr: consecutive prompt tokens of the
// current session at positions start..start+n-1 (its caches kc/vc and conv
// state), with the last layer's FFN on the last token only (lfm.rs:540-541).
// tb != nullptr: one token from each of n independent sessions (batched
// decode): positions, sessions and per-session caches come from tb, and every
// token runs every layer.
void EngineImpl::enqueue_layers(int n, uint32_t start, const TokBatch* tb, int& nl, const SessRuns* runs,
                                const int* start_dev) {
  cudaStream_t s = stream;
  const float eps = hp.eps;
  LaunchCfg c;
  c.stream = s;
  c.pdl = false;
  c.sms = sms;
  const bool tc = use_tc && n >= tc_min;
  tcs.err = (unsigned*)(io + 4);
  // x (n rows of K, stride K) -> activation operand of the tensor-core GEMMs
  auto split = [&](const float* X, int K) {
    CK(tc_split(X, K, K, n, tcs, s));
    nl++;
  };
  // out[t * ldo + o] (+)= W x_t
  auto mm = [&](const Q6Mat& W, const float* X, float* out, int ldo, bool resid) {
    if (tc) CK(tc_gemm_q6(W, n, out, ldo, resid, tcs, s, x16(W)));
    else gemm_q6_ld(W, X, n, out, ldo, resid, s);
    nl++;
  };
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const LayerW& L = layers[l];
    if (tc) CK(tc_split_norm(px, L.attn_norm, eps, n, ph, tcs, s));  // RMSNorm + operand split
    else rmsnorm_n(px, L.attn_norm, eps, n, ph, s);
    nl++;
    if (L.attn) {
      const int ld = DIM + 2 * KV_HEADS * HEAD_DIM;
      mm(L.q, ph, pqkv, ld, false);
      mm(L.k, ph, pqkv + DIM, ld, false);
      mm(L.v, ph, pqkv + DIM + KV_HEADS * HEAD_DIM, ld, false);
      const size_t loff = (size_t)L.attn_idx * KV_HEADS * ctx * HEAD_DIM;
      if (tb) {
        qk_prep_batch(pqkv, L.q_norm, L.k_norm, rope, n, ctx, eps, tb->kc + loff, tb->vc + loff, tb->pos, tb->sess,
                      tb->kv_stride, s);
        attn_batch(pqkv, tb->kc + loff, tb->vc + loff, n, ctx, pa, tb->pos, tb->sess, tb->kv_stride, tb->part, s);
      } else if (runs) {
        // each session's prompt attends to itself only (its own cache)
        for (int i = 0; i < runs->count; i++) {
          const int o = runs->off[i], m = runs->len[i];
          __half* skc = batch.kc + (size_t)runs->sess[i] * batch.kv_stride + loff;
          __half* svc = batch.vc + (size_t)runs->sess[i] * batch.kv_stride + loff;
          qk_prep_n(pqkv + (size_t)o * ld, L.q_norm, L.k_norm, rope, 0, m, ctx, eps, skc, svc, s);
          if (tc) CK(attn_prefill_tc(pqkv + (size_t)o * ld, ld, skc, svc, 0, m, (int)ctx, pa + (size_t)o * DIM, DIM,
                                     tcs.err, s));
          else attn_prefill(pqkv + (size_t)o * ld, skc, svc, 0, m, ctx, pa + (size_t)o * DIM, s);
          nl += 2;
        }
      } else {
        qk_prep_n(pqkv, L.q_norm, L.k_norm, rope, start, n, ctx, eps, kc + loff, vc + loff, s, start_dev);
        if (tc)
          CK(attn_prefill_tc(pqkv, ld, kc + loff, vc + loff, (int)start, n, (int)ctx, pa, DIM, tcs.err, s,
                             start_dev));
        else attn_prefill(pqkv, kc + loff, vc + loff, start, n, ctx, pa, s);
      }
      if (tc) split(pa, DIM);
      mm(L.o, pa, px, DIM, true);
      nl += 2;
    } else {
      mm(L.in_proj, ph, pbcx, 3 * DIM, false);
      const size_t coff = (size_t)L.conv_idx * DIM * 2;
      if (tb) {
        conv_batch(pbcx, L.conv_w, tb->conv + coff, tb->conv_stride, tb->sess, n, pgated, s);
      } else if (runs) {
        for (int i = 0; i < runs->count; i++) {
          const int o = runs->off[i];
          conv_prefill(pbcx + (size_t)o * 3 * DIM, L.conv_w,
                       batch.conv + (size_t)runs->sess[i] * batch.conv_stride + coff, runs->len[i],
                       pgated + (size_t)o * DIM, s);
          nl++;
        }
      } else {
        conv_prefill(pbcx, L.conv_w, conv_state + coff, n, pgated, s);
      }
      if (tc) split(pgated, DIM);
      mm(L.out_proj, pgated, px, DIM, true);
      nl += tb ? 1 : 2;
    }
    const bool last = l == hp.n_layers - 1;
    if (last && !tb && !runs) {
      // The last layer's FFN only runs on the last token (lfm.rs:540-541).
      float* xl = px + (size_t)(n - 1) * DIM;
      if (ep_now && !L.dense) {
        rmsnorm_n(xl, L.ffn_norm, eps, 1, ph, s);
        ep_moe(L, ph, 1, xl);
        nl += 8;
      } else {
        enqueue_ffn(L, xl, c, (unsigned*)(io + 4));
        nl += L.dense ? 2 : 3;
      }
      continue;
    }
    if (tc && L.dense) CK(tc_split_norm(px, L.ffn_norm, eps, n, ph, tcs, s));
    else rmsnorm_n(px, L.ffn_norm, eps, n, ph, s);
    nl++;
    if (L.dense) {
      mm(L.gate, ph, pgate, N_FF, false);
      mm(L.up, ph, pup, N_FF, false);
      if (tc) {
        CK(tc_split(pgate, N_FF, N_FF, n, tcs, s, pup));  // SwiGLU fused into the operand split
      } else {
        swiglu_n(pgate, pup, (size_t)n * N_FF, psw, s);
      }
      mm(L.down, psw, px, DIM, true);
      nl += 1;
    } else if (ep_now && !tb) {
      ep_moe(L, ph, n, px);
      nl += 8;
    } else {
      router_logits_n(L.router, ph, n, prlog, s);
      route_n(prlog, L.bias, N_EXPERT, n, psel, pselw, s);
      expert_groups(psel, n, pgroups, n, s);
      if (tc) {
        CK(tc_group(pgroups, n, n, tcs, s));
        CK(tc_split_grouped(ph, DIM, N_USED, n, tcs, s));
        CK(tc_gemm_q6_grouped(L.gate_x, EXPERT_FF, n, pgate, tcs, s, x16(L.gate_x)));
        CK(tc_gemm_q6_grouped(L.up_x, EXPERT_FF, n, pup, tcs, s, x16(L.up_x)));
        CK(tc_split_grouped(pgate, EXPERT_FF, 1, n, tcs, s, pup));  // SwiGLU fused into the operand split
        CK(tc_gemm_q6_grouped(L.down_x, DIM, n, pdown, tcs, s, x16(L.down_x)));
        nl += 2;  // group layout, first split (the fused split stands in for SwiGLU)
      } else {
        gemm_q6_grouped(L.gate_x, EXPERT_FF, ph, N_USED, pgroups, n, n, pgate, s);
        gemm_q6_grouped(L.up_x, EXPERT_FF, ph, N_USED, pgroups, n, n, pup, s);
        swiglu_n(pgate, pup, (size_t)n * N_USED * EXPERT_FF, psw, s);
        gemm_q6_grouped(L.down_x, DIM, psw, 1, pgroups, n, n, pdown, s);
      }
      combine_n(pdown, pselw, n, px, s);
      nl += 8;
      ctr.expert_grouped_launches += 3;
    }
  }
}

// Exchange buffers of the expert-parallel MoE layers (grown, never shrunk).
void EngineImpl::ep_reserve(int send_slots, int recv_slots) {
  if (!ep_counts) {
    ep_counts = dalloc<int32_t>(ep_allocs, 64);
    ep_all = dalloc<int32_t>(ep_allocs, 64 * 64);
  }
  if (send_slots > ep_cap_send) {
    ep_send = dalloc<float>(ep_allocs, (size_t)send_slots * DIM);
    ep_back = dalloc<float>(ep_allocs, (size_t)send_slots * DIM);
    ep_local = dalloc<float>(ep_allocs, (size_t)send_slots * DIM);
    ep_send_tag = dalloc<int32_t>(ep_allocs, send_slots);
    ep_order = dalloc<int32_t>(ep_allocs, send_slots);
    ep_cap_send = send_slots;
  }
  if (recv_slots > ep_cap_recv) {
    ep_recv = dalloc<float>(ep_allocs, (size_t)recv_slots * DIM);
    CK(cudaMemsetAsync(ep_recv, 0, (size_t)recv_slots * DIM * 4, stream));  // padding slots read finite rows
    ep_recv_tag = dalloc<int32_t>(ep_allocs, recv_slots);
    ep_sel4 = dalloc<int32_t>(ep_allocs, recv_slots + N_USED);
    ep_cap_recv = recv_slots;
  }
}

// Expert-parallel routed FFN of `n` token rows (`rows`: the FFN inputs after
// ffn_norm; `xres`: their residual rows): route locally, send each
// (token, rank) slot's row to the owner of its expert, run this rank's experts
// on the slots it received (grouped tensor-core GEMMs), send the down rows
// back and combine them in rank order (kernels/resident.rs:101-117). Every
// rank of the communicator runs this for the same layer at the same time.
void EngineImpl::ep_moe(const LayerW& L, const float* rows, int n, float* xres) {
  cudaStream_t s = stream;
  const int G = ep.world, me = ep.rank, per = N_EXPERT / G;
  const int nslots = N_USED * n;
  std::string e;
  router_logits_n(L.router, rows, n, prlog, s);
  route_n(prlog, L.bias, N_EXPERT, n, psel, pselw, s);
  // send plan on the host (ep_plan), from the routing read back
  h_sel.resize(nslots);
  CK(cudaMemcpyAsync(h_sel.data(), psel, (size_t)nslots * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  h_order.resize(nslots);
  h_counts.assign(G, 0);
  ep_plan(h_sel.data(), nslots, G, h_counts.data(), h_order.data());
  CK(cudaMemcpyAsync(ep_order, h_order.data(), (size_t)nslots * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(ep_counts, h_counts.data(), (size_t)G * 4, cudaMemcpyHostToDevice, s));
  ep_pack(rows, psel, ep_order, nslots, ep_send, ep_send_tag, s);
  if (!ep_allgather_i32(ep, ep_counts, ep_all, G, s, e)) throw std::runtime_error(e);
  h_all.resize((size_t)G * G);
  CK(cudaMemcpyAsync(h_all.data(), ep_all, (size_t)G * G * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  std::vector<int> scnt(G), soff(G), rcnt(G), roff(G);
  int st = 0, rt = 0;
  for (int p = 0; p < G; p++) {
    scnt[p] = h_counts[p];
    soff[p] = st;
    st += scnt[p];
    rcnt[p] = h_all[(size_t)p * G + me];  // rank p's count for this rank
    roff[p] = rt;
    rt += rcnt[p];
  }
  if (rt + N_USED > ep_cap_recv) throw std::runtime_error("expert-parallel receive buffer too small");
  if (!ep_exchange(ep, ep_send, ep_send_tag, scnt.data(), soff.data(), ep_recv, ep_recv_tag, rcnt.data(),
                   roff.data(), DIM, s, e))
    throw std::runtime_error(e);
  if (rt > 0) {
    // the received slots as routing rows of 4 ranks (padding slots: a local
    // expert over zero rows), then the grouped gate/up -> SwiGLU -> down
    // the received slots as nf rows of 4 (padding slots: distinct local
    // experts over zero-or-stale finite rows). Unlike a real token's four
    // experts, four received slots may share an expert, so an expert's slot
    // list can be longer than nf: its capacity is every rank's token count
    // (one slot per token at most) plus one padding slot.
    const int nf = (rt + N_USED - 1) / N_USED;
    const int cap = ep_total + 1;
    ep_fake_sel(ep_recv_tag, rt, me * per, ep_sel4, s);
    expert_groups(ep_sel4, nf, pgroups, cap, s);
    CK(tc_group(pgroups, cap, nf, tcs, s));
    CK(tc_split_grouped(ep_recv, DIM, 1, nf, tcs, s));
    CK(tc_gemm_q6_grouped(L.gate_x, EXPERT_FF, nf, pgate, tcs, s, x16(L.gate_x)));
    CK(tc_gemm_q6_grouped(L.up_x, EXPERT_FF, nf, pup, tcs, s, x16(L.up_x)));
    CK(tc_split_grouped(pgate, EXPERT_FF, 1, nf, tcs, s, pup));  // SwiGLU fused into the operand split
    CK(tc_gemm_q6_grouped(L.down_x, DIM, nf, pdown, tcs, s, x16(L.down_x)));
    ctr.expert_grouped_launches += 3;
  }
  // down rows back to the ranks that sent the slots, in the order they came
  if (!ep_exchange(ep, pdown, nullptr, rcnt.data(), roff.data(), ep_back, nullptr, scnt.data(), soff.data(), DIM, s,
                   e))
    throw std::runtime_error(e);
  ep_unpack(ep_back, ep_order, nslots, ep_local, s);
  combine_n(ep_local, pselw, n, xres, s);
}

void EngineImpl::run_prefill(const uint32_t* ids, int n, uint32_t start, bool ep_mode) {
  cudaStream_t s = stream;
  const float eps = hp.eps;
  int nl = 0;
  if (ep_mode) {
    // every rank learns every rank's token count: a rank may receive up to
    // 4 slots of each of them in one MoE layer
    ep_reserve(0, 0);
    h_counts.assign(ep.world, 0);
    int32_t mine = n;
    CK(cudaMemcpyAsync(ep_counts, &mine, 4, cudaMemcpyHostToDevice, s));
    std::string e;
    if (!ep_allgather_i32(ep, ep_counts, ep_all, 1, s, e)) throw std::runtime_error(e);
    h_all.assign(ep.world, 0);
    CK(cudaMemcpyAsync(h_all.data(), ep_all, (size_t)ep.world * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    int total = 0;
    for (int v : h_all) total += v;
    // an expert receives at most one slot per token of any rank, plus one
    // padding slot: its slot list needs total + 1 entries (ep_moe)
    ep_total = total;
    ensure_prefill(std::max(n, total + N_USED));
    ep_reserve(N_USED * n, N_USED * total + N_USED);
  } else {
    ensure_prefill(n);
  }
  ep_now = ep_mode;
  CK(cudaEventRecord(ev0, s));
  // the chunk's ids and its first position (pinned h_io[1] -> io[1], read by
  // the attention launches): copies outside any graph
  CK(cudaMemcpyAsync(pids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  h_io[1] = (int)start;
  CK(cudaMemcpyAsync(io + 1, h_io + 1, 4, cudaMemcpyHostToDevice, s));
  // embedding .. lm_head argmax: for a given n the same launches serve every
  // start position of the engine's own session
  auto body = [&](int& cnt) {
    embed_n(embd, pids, n, px, s);
    cnt++;
    enqueue_layers(n, start, nullptr, cnt, nullptr, io + 1);
    LaunchCfg c;
    c.stream = s;
    c.pdl = false;
    c.sms = sms;
    if (use_mvt)
      mvt_lmhead(embd, XSrc{px + (size_t)(n - 1) * DIM, out_norm, eps}, logits, am_part, counters + 128, io + 2,
                 (unsigned*)(io + 4), c);
    else
      mv_lmhead(embd, XSrc{px + (size_t)(n - 1) * DIM, out_norm, eps}, logits, am_part, counters + 128, io + 2, c);
    cnt++;
  };
  // chunks of up to LFM_PREFILL_CHUNK tokens (the api_stream prompt chunks,
  // short turns) replay a graph per n; longer prompts and other sessions'
  // slots launch one by one
  const bool graphable =
      use_graph && use_tc && !ep_mode && !session_swap && n >= tc_min && n <= (int)LFM_PREFILL_CHUNK;
  PGraph* hit = nullptr;
  bool seen = false;
  if (graphable) {
    for (PGraph& g : pgraphs)
      if (g.n == n) hit = &g;
    for (int v : pgraph_seen) seen = seen || v == n;
  }
  try {
    if (hit) {
      CK(cudaGraphLaunch(hit->exec, s));
      nl = hit->nl;
      ctr.graph_replays++;
    } else if (graphable && seen) {
      // the second chunk of this length: capture it (the first, eager chunk
      // has made every one-time kernel attribute call)
      cudaGraph_t g = nullptr;
      CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        body(nl);
      } catch (...) {
        cudaStreamEndCapture(s, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      CK(cudaStreamEndCapture(s, &g));
      PGraph pg;
      pg.n = n;
      pg.nl = nl;
      const cudaError_t e = cudaGraphInstantiate(&pg.exec, g, 0);
      cudaGraphDestroy(g);
      CK(e);
      if ((int)pgraphs.size() >= PGRAPH_MAX) {
        cudaGraphExecDestroy(pgraphs.front().exec);
        pgraphs.erase(pgraphs.begin());
      }
      pgraphs.push_back(pg);
      ctr.graph_captures++;
      CK(cudaGraphLaunch(pg.exec, s));
    } else {
      body(nl);
      if (graphable && pgraph_seen.size() < 2 * LFM_PREFILL_CHUNK) pgraph_seen.push_back(n);
    }
  } catch (...) {
    ep_now = false;
    throw;
  }
  ep_now = false;
  CK(cudaMemcpyAsync(h_io + 2, io + 2, 12, cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(ev1, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaGetLastError());
  CK(cudaEventElapsedTime(&last_ms, ev0, ev1));
  ctr.kernel_launches += nl;
  ctr.gpu_argmax++;
  ctr.prefill_tokens += n;
  check_device_error();
}

// ---------------------------------------------------------------- sessions
// Independent sessions with their own KV caches and conv states, prefilled one
// at a time and decoded together, one token per session per step (the
// reference time-multiplexes sessions by snapshot/restore through one set of
// buffers, persistent.rs:164-176).
void EngineImpl::batch_create(uint32_t nsess) {
  ensure_state();
  batch_free();
  BatchState& B = batch;
  B.nsess = nsess;
  B.ctx = ctx;
  B.kv_stride = (size_t)std::max(n_attn, 1) * KV_HEADS * ctx * HEAD_DIM;
  B.conv_stride = (size_t)std::max(n_conv, 1) * DIM * 2;
  B.kc = dalloc<__half>(B.allocs, B.kv_stride * nsess);
  B.vc = dalloc<__half>(B.allocs, B.kv_stride * nsess);
  B.conv = dalloc<float>(B.allocs, B.conv_stride * nsess);
  CK(cudaMemsetAsync(B.kc, 0, B.kv_stride * nsess * 2, stream));
  CK(cudaMemsetAsync(B.vc, 0, B.kv_stride * nsess * 2, stream));
  CK(cudaMemsetAsync(B.conv, 0, B.conv_stride * nsess * 4, stream));
  B.map = dalloc<int>(B.allocs, 3 * (size_t)nsess);  // tokens | positions | sessions
  B.next = dalloc<int>(B.allocs, nsess);
  B.logits = dalloc<float>(B.allocs, (size_t)nsess * hp.vocab);
  B.attn_part = dalloc<float>(B.allocs, attn_batch_part_floats((int)nsess, (int)ctx));
  B.h_map.resize(3 * (size_t)nsess);
  CK(cudaStreamSynchronize(stream));
}

void EngineImpl::batch_free() {
  drop_bgraph();  // it holds the session buffers' addresses
  for (void* p : batch.allocs) cudaFree(p);
  batch = BatchState();
}

// Prefill session `sess` with its prompt (positions 0..n-1): the single-session
// prompt path with the session's caches in place of the engine's own.
uint32_t EngineImpl::batch_prefill(uint32_t sess, const uint32_t* ids, int n, bool ep_mode) {
  BatchState& B = batch;
  __half* k0 = kc;
  __half* v0 = vc;
  float* c0 = conv_state;
  kc = B.kc + (size_t)sess * B.kv_stride;
  vc = B.vc + (size_t)sess * B.kv_stride;
  conv_state = B.conv + (size_t)sess * B.conv_stride;
  CK(cudaMemsetAsync(conv_state, 0, B.conv_stride * 4, stream));  // a fresh session (reset_session)
  session_swap = true;
  try {
    run_prefill(ids, n, 0, ep_mode);
  } catch (...) {
    kc = k0, vc = v0, conv_state = c0;
    session_swap = false;
    throw;
  }
  kc = k0, vc = v0, conv_state = c0;
  session_swap = false;
  return (uint32_t)h_io[2];
}

// Fresh prompts of `count` distinct sessions in one pass (every projection is
// one GEMM over all their tokens, so each weight is read once per pass):
// session sess[i] gets ids[off_i .. off_i + lens[i]) at positions 0.. (off_i =
// sum of the earlier lens); attention and the short conv run per session on
// its own cache and state. The last layer's FFN runs on every token (the
// single-session path trims it to the last token; the rows it feeds are the
// same). next[i] = greedy next token of session sess[i].
void EngineImpl::batch_prefill_many(const uint32_t* sess, const uint32_t* ids, const uint32_t* lens, int count,
                                   uint32_t* next) {
  BatchState& B = batch;
  std::vector<int> off(count), len(count);
  int n = 0;
  for (int i = 0; i < count; i++) {
    off[i] = n;
    len[i] = (int)lens[i];
    n += len[i];
  }
  ensure_prefill(std::max(n, count));
  cudaStream_t s = stream;
  const float eps = hp.eps;
  int nl = 0;
  CK(cudaEventRecord(ev0, s));
  for (int i = 0; i < count; i++)  // fresh sessions (reset_session)
    CK(cudaMemsetAsync(B.conv + (size_t)sess[i] * B.conv_stride, 0, B.conv_stride * 4, s));
  CK(cudaMemcpyAsync(pids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  embed_n(embd, pids, n, px, s);
  nl++;
  SessRuns runs;
  runs.count = count;
  runs.sess = sess;
  runs.off = off.data();
  runs.len = len.data();
  enqueue_layers(n, 0, nullptr, nl, &runs);
  // the last token of each session: final norm, tied lm_head, row argmax
  for (int i = 0; i < count; i++)
    CK(cudaMemcpyAsync(ph + (size_t)i * DIM, px + (size_t)(off[i] + len[i] - 1) * DIM, DIM * 4,
                       cudaMemcpyDeviceToDevice, s));
  if (use_tc && count >= tc_min) {
    CK(tc_split_norm(ph, out_norm, eps, count, pa, tcs, s));
    CK(tc_gemm_q6(embd, count, B.logits, (int)hp.vocab, false, tcs, s, x16(embd)));
  } else {
    rmsnorm_n(ph, out_norm, eps, count, pa, s);
    gemm_q6_ld(embd, pa, count, B.logits, (int)hp.vocab, false, s);
  }
  argmax_rows(B.logits, count, (int)hp.vocab, B.next, s);
  nl += 3 + count;
  B.last_count = 0;  // the logits rows no longer belong to a decode step
  std::vector<int> h(count);
  CK(cudaMemcpyAsync(h.data(), B.next, (size_t)count * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(h_io + 4, io + 4, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(ev1, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaGetLastError());
  CK(cudaEventElapsedTime(&last_ms, ev0, ev1));
  for (int i = 0; i < count; i++) next[i] = (uint32_t)h[i];
  ctr.kernel_launches += nl;
  ctr.prefill_tokens += n;
  check_device_error();
}

// One decode step of `count` sessions: token tokens[i] at position pos[i] of
// session sess[i] (distinct sessions); next[i] = greedy next token.
void EngineImpl::run_batch_decode(uint32_t count, const uint32_t* tokens, const uint32_t* pos, const uint32_t* sess,
                                  uint32_t* next) {
  BatchState& B = batch;
  const int n = (int)count;
  ensure_prefill(n);
  cudaStream_t s = stream;
  const float eps = hp.eps;
  int nl = 0;
  for (int i = 0; i < n; i++) {
    B.h_map[i] = (int)tokens[i];
    B.h_map[n + i] = (int)pos[i];
    B.h_map[2 * n + i] = (int)sess[i];
  }
  // embedding .. row argmax: every launch reads the step's inputs from B.map
  // and device buffers that stay in place, so the same launches serve every
  // step with n sessions
  auto body = [&](int& cnt) {
    embed_n(embd, (const uint32_t*)B.map, n, px, s);
    cnt++;
    TokBatch tb;
    tb.pos = B.map + n;
    tb.sess = B.map + 2 * n;
    tb.kc = B.kc;
    tb.vc = B.vc;
    tb.conv = B.conv;
    tb.kv_stride = B.kv_stride;
    tb.conv_stride = B.conv_stride;
    tb.part = B.attn_part;
    enqueue_layers(n, 0, &tb, cnt);
    // final norm + tied lm_head for every token, then the row argmax
    if (use_tc && n >= tc_min) {
      CK(tc_split_norm(px, out_norm, eps, n, ph, tcs, s));
      CK(tc_gemm_q6(embd, n, B.logits, (int)hp.vocab, false, tcs, s, x16(embd)));
    } else {
      rmsnorm_n(px, out_norm, eps, n, ph, s);
      gemm_q6_ld(embd, ph, n, B.logits, (int)hp.vocab, false, s);
    }
    argmax_rows(B.logits, n, (int)hp.vocab, B.next, s);
    cnt += 3;
  };
  CK(cudaEventRecord(ev0, s));
  // the step's inputs (pageable host memory: a copy outside any graph)
  CK(cudaMemcpyAsync(B.map, B.h_map.data(), (size_t)3 * n * 4, cudaMemcpyHostToDevice, s));
  if (bgraph && bgraph_n == n) {
    CK(cudaGraphLaunch(bgraph, s));
    nl = bgraph_nl;
    ctr.graph_replays++;
  } else if (use_graph && beager_n == n) {
    // the second step with this session count: capture it (the first, eager
    // step has made every one-time kernel attribute call)
    drop_bgraph();
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      body(nl);
    } catch (...) {
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CK(cudaStreamEndCapture(s, &g));
    const cudaError_t e = cudaGraphInstantiate(&bgraph, g, 0);
    cudaGraphDestroy(g);
    CK(e);
    bgraph_n = n;
    bgraph_nl = nl;
    ctr.graph_captures++;
    CK(cudaGraphLaunch(bgraph, s));
  } else {
    body(nl);
    beager_n = n;
  }
  CK(cudaMemcpyAsync(next, B.next, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(h_io + 4, io + 4, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(ev1, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaGetLastError());
  CK(cudaEventElapsedTime(&last_ms, ev0, ev1));
  ctr.kernel_launches += nl;
  check_device_error();
}

std::vector<uint8_t> EngineImpl::snapshot(uint32_t valid) {
  std::vector<uint8_t> out;
  std::vector<__half> hk, hv;
  std::vector<float> conv(DIM * 2);
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const LayerW& L = layers[l];
    if (L.attn) {
      const size_t width = KV_HEADS * HEAD_DIM;
      hk.resize((size_t)KV_HEADS * valid * HEAD_DIM);
      hv.resize(hk.size());
      for (int kh = 0; kh < KV_HEADS; kh++) {
        const size_t off = ((size_t)L.attn_idx * KV_HEADS + kh) * ctx * HEAD_DIM;
        CK(cudaMemcpy(hk.data() + (size_t)kh * valid * HEAD_DIM, kc + off, (size_t)valid * HEAD_DIM * 2,
                      cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(hv.data() + (size_t)kh * valid * HEAD_DIM, vc + off, (size_t)valid * HEAD_DIM * 2,
                      cudaMemcpyDeviceToHost));
      }
      for (int which = 0; which < 2; which++) {
        const std::vector<__half>& h = which ? hv : hk;
        const size_t base = out.size();
        out.resize(base + (size_t)valid * width * 4);
        float* o = (float*)(out.data() + base);
        for (uint32_t p = 0; p < valid; p++)
          for (int kh = 0; kh < KV_HEADS; kh++)
            for (int d = 0; d < HEAD_DIM; d++)
              o[(size_t)p * width + kh * HEAD_DIM + d] = __half2float(h[((size_t)kh * valid + p) * HEAD_DIM + d]);
      }
    } else {
      CK(cudaMemcpy(conv.data(), conv_state + (size_t)L.conv_idx * DIM * 2, DIM * 2 * 4, cudaMemcpyDeviceToHost));
      const size_t base = out.size();
      out.resize(base + DIM * 2 * 4);
      memcpy(out.data() + base, conv.data(), DIM * 2 * 4);
    }
  }
  return out;
}

void EngineImpl::restore(uint32_t valid, const uint8_t* buf, size_t len) {
  size_t off = 0;
  std::vector<__half> hk;
  for (uint32_t l = 0; l < hp.n_layers; l++) {
    const LayerW& L = layers[l];
    if (L.attn) {
      const size_t width = KV_HEADS * HEAD_DIM;
      const size_t size = (size_t)valid * width * 4;
      for (int which = 0; which < 2; which++) {
        if (off + size > len) throw std::runtime_error("truncated snapshot");
        const float* src = (const float*)(buf + off);
        hk.resize((size_t)KV_HEADS * valid * HEAD_DIM);
        for (uint32_t p = 0; p < valid; p++)
          for (int kh = 0; kh < KV_HEADS; kh++)
            for (int d = 0; d < HEAD_DIM; d++)
              hk[((size_t)kh * valid + p) * HEAD_DIM + d] = __float2half_rn(src[(size_t)p * width + kh * HEAD_DIM + d]);
        __half* dst = which ? vc : kc;
        for (int kh = 0; kh < KV_HEADS; kh++) {
          const size_t doff = ((size_t)L.attn_idx * KV_HEADS + kh) * ctx * HEAD_DIM;
          if (valid)
            CK(cudaMemcpy(dst + doff, hk.data() + (size_t)kh * valid * HEAD_DIM, (size_t)valid * HEAD_DIM * 2,
                          cudaMemcpyHostToDevice));
        }
        off += size;
      }
    } else {
      const size_t size = DIM * 2 * 4;
      if (off + size > len) throw std::runtime_error("truncated snapshot");
      CK(cudaMemcpy(conv_state + (size_t)L.conv_idx * DIM * 2, buf + off, size, cudaMemcpyHostToDevice));
      off += size;
    }
  }
  if (off != len) throw std::runtime_error("extra snapshot data");
}

}  // namespace lfm

// =========================================================== C ABI
using lfm::EngineImpl;

struct lfm_engine {
  EngineImpl impl;
};

namespace {

template <class F>
lfm_status guarded(lfm_engine* e, F&& f) {
  if (!e) {
    lfm::g_error = "null engine";
    return LFM_ERR_ARG;
  }
  try {
    cudaSetDevice(e->impl.device);
    return f();
  } catch (const lfm::CudaError& ce) {
    lfm::set_err(&e->impl, std::string("CUDA: ") + cudaGetErrorString(ce.e));
    return LFM_ERR_CUDA;
  } catch (const std::exception& ex) {
    lfm::set_err(&e->impl, ex.what());
    return LFM_ERR_ARG;
  }
}

lfm_status check_ids(lfm_engine* e, const uint32_t* ids, uint32_t n, int64_t start) {
  EngineImpl& I = e->impl;
  if (!ids || n == 0 || start < 0 || (uint64_t)start + n > I.ctx) {
    lfm::set_err(&I, "forward context range");
    return LFM_ERR_ARG;
  }
  for (uint32_t i = 0; i < n; i++)
    if (ids[i] >= I.hp.vocab) {
      lfm::set_err(&I, "token out of range");
      return LFM_ERR_ARG;
    }
  return LFM_OK;
}

}  // namespace

extern "C" {

lfm_status lfm_model_inspect(const char* gguf_path, lfm_hparams* out) {
  if (!gguf_path) {
    lfm::g_error = "null argument";
    return LFM_ERR_ARG;
  }
  lfm::GgufFile f;
  if (!f.open(gguf_path)) {
    lfm::g_error = "parse GGUF header: " + f.err();
    return LFM_ERR_MODEL;
  }
  lfm_hparams hp;
  std::string err;
  if (!lfm::read_hparams(f, hp, err) || !lfm::check_tensors(f, hp, err)) {
    lfm::g_error = err;
    return LFM_ERR_MODEL;
  }
  if (out) *out = hp;
  return LFM_OK;
}

lfm_status lfm_engine_create(const char* gguf_path, int device, lfm_engine** out) {
  if (!gguf_path || !out) {
    lfm::g_error = "null argument";
    return LFM_ERR_ARG;
  }
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    lfm::g_error = "no CUDA device " + std::to_string(device);
    return LFM_ERR_CUDA;
  }
  auto* e = new lfm_engine();
  EngineImpl& I = e->impl;
  I.device = device;
  if (cudaSetDevice(device) != cudaSuccess) {
    lfm::g_error = "cudaSetDevice failed";
    delete e;
    return LFM_ERR_CUDA;
  }
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, device);
  if (prop.major != 10) {
    lfm::g_error = std::string("device ") + prop.name + " is not sm_100 (B200)";
    delete e;
    return LFM_ERR_CUDA;
  }
  I.name = prop.name;
  I.sms = prop.multiProcessorCount;
  if (const char* v = getenv("LFM_PDL")) I.pdl = std::string(v) != "0";
  if (const char* v = getenv("LFM_GRAPH")) I.use_graph = std::string(v) != "0";
  if (const char* v = getenv("LFM_MVT")) I.use_mvt = std::string(v) != "0";
  if (const char* v = getenv("LFM_STEP")) I.use_step = std::string(v) != "0";
  if (const char* v = getenv("LFM_PREFILL")) I.use_tc = std::string(v) != "fp32";
  if (const char* v = getenv("LFM_PREFILL_X16")) I.use_x16 = std::string(v) != "0";
  if (const char* v = getenv("LFM_TC_MIN_TOKENS")) I.tc_min = std::max(1, atoi(v));
  if (!I.use_step) I.step_reason = "persistent step disabled (LFM_STEP=0)";
  if (cudaStreamCreateWithFlags(&I.stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMallocHost(&I.h_io, 64) != cudaSuccess || cudaEventCreate(&I.ev0) != cudaSuccess ||
      cudaEventCreate(&I.ev1) != cudaSuccess) {
    lfm::g_error = "stream / pinned allocation failed";
    delete e;
    return LFM_ERR_CUDA;
  }
  if (!I.load(gguf_path)) {
    lfm::g_error = I.err;
    delete e;
    return LFM_ERR_MODEL;
  }
  *out = e;
  return LFM_OK;
}

void lfm_engine_destroy(lfm_engine* e) { delete e; }

lfm_status lfm_engine_set_ctx(lfm_engine* e, uint32_t ctx) {
  return guarded(e, [&]() -> lfm_status {
    if (ctx == 0 || ctx > LFM_MAX_CTX) {
      lfm::set_err(&e->impl, "context must be 1..4096");
      return LFM_ERR_ARG;
    }
    e->impl.ctx = ctx;
    return LFM_OK;
  });
}

lfm_status lfm_hparams_get(lfm_engine* e, lfm_hparams* out) {
  if (!e || !out) return LFM_ERR_ARG;
  *out = e->impl.hp;
  return LFM_OK;
}

lfm_status lfm_forward_token(lfm_engine* e, const uint32_t* ids, uint32_t n, uint32_t position,
                             uint32_t* next_token) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (n == 0 || n > LFM_PREFILL_CHUNK) {
      lfm::set_err(&I, "token batch must be 1..64");
      return LFM_ERR_ARG;
    }
    lfm_status st = check_ids(e, ids, n, position);
    if (st) return st;
    I.ensure_state();
    if (n == 1) I.run_decode(ids[0], position);
    else I.run_prefill(ids, (int)n, position);
    if (next_token) *next_token = (uint32_t)I.h_io[2];
    return LFM_OK;
  });
}

lfm_status lfm_forward_logits(lfm_engine* e, const uint32_t* ids, uint32_t n, int64_t start_pos, float* logits) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    lfm_status st = check_ids(e, ids, n, start_pos);
    if (st) return st;
    I.ensure_state();
    if (n == 1) I.run_decode(ids[0], (uint32_t)start_pos);
    else I.run_prefill(ids, (int)n, (uint32_t)start_pos);
    if (logits) CK(cudaMemcpy(logits, I.logits, (size_t)I.hp.vocab * 4, cudaMemcpyDeviceToHost));
    return LFM_OK;
  });
}

lfm_status lfm_generate(lfm_engine* e, const uint32_t* prompt, uint32_t prompt_len, uint32_t n, uint32_t eos,
                        uint32_t* out_tokens, uint32_t* n_out) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!prompt || prompt_len == 0 || (uint64_t)prompt_len + n > I.ctx || (n && !out_tokens)) {
      lfm::set_err(&I, "empty prompt or context exceeded");
      return LFM_ERR_ARG;
    }
    lfm_status st = check_ids(e, prompt, prompt_len, 0);
    if (st) return st;
    I.ensure_state();
    uint32_t pos = 0, next = 0;
    for (uint32_t off = 0; off < prompt_len; off += LFM_PREFILL_CHUNK) {
      const uint32_t c = std::min(LFM_PREFILL_CHUNK, prompt_len - off);
      if (c == 1) I.run_decode(prompt[off], pos);
      else I.run_prefill(prompt + off, (int)c, pos);
      next = (uint32_t)I.h_io[2];
      pos += c;
    }
    uint32_t cnt = 0;
    for (uint32_t i = 0; i < n; i++) {
      if (next == eos) break;
      out_tokens[cnt++] = next;
      I.run_decode(next, pos);
      next = (uint32_t)I.h_io[2];
      pos++;
    }
    if (n_out) *n_out = cnt;
    return LFM_OK;
  });
}

lfm_status lfm_decode_loop(lfm_engine* e, uint32_t first_token, uint32_t start_pos, uint32_t steps,
                           uint32_t* out_tokens, float* device_ms) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!out_tokens || steps == 0 || (uint64_t)start_pos + steps > I.ctx) {
      lfm::set_err(&I, "forward context range");
      return LFM_ERR_ARG;
    }
    lfm_status st = check_ids(e, &first_token, 1, start_pos);
    if (st) return st;
    I.ensure_state();
    I.run_decode(first_token, start_pos);
    out_tokens[0] = (uint32_t)I.h_io[2];
    float first_ms = I.last_ms;
    if (steps > 1) I.run_loop(steps - 1, out_tokens + 1);
    if (device_ms) *device_ms = steps > 1 ? I.last_ms : first_ms;
    return LFM_OK;
  });
}

lfm_status lfm_batch_create(lfm_engine* e, uint32_t n_sessions) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (n_sessions == 0 || n_sessions > 4096) {
      lfm::set_err(&I, "n_sessions must be 1..4096");
      return LFM_ERR_ARG;
    }
    I.batch_create(n_sessions);
    return LFM_OK;
  });
}

lfm_status lfm_batch_prefill(lfm_engine* e, uint32_t session, const uint32_t* ids, uint32_t n,
                             uint32_t* next_token) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (I.batch.nsess == 0 || I.batch.ctx != I.ctx) {
      lfm::set_err(&I, "no session slots for the current context length (lfm_batch_create)");
      return LFM_ERR_ARG;
    }
    if (session >= I.batch.nsess) {
      lfm::set_err(&I, "session out of range");
      return LFM_ERR_ARG;
    }
    lfm_status st = check_ids(e, ids, n, 0);
    if (st) return st;
    const uint32_t t = I.batch_prefill(session, ids, (int)n);
    if (next_token) *next_token = t;
    return LFM_OK;
  });
}

// ---------------------------------------------------------- expert parallel
lfm_status lfm_ep_unique_id(uint8_t* out) {
  if (!out) {
    lfm::g_error = "null argument";
    return LFM_ERR_ARG;
  }
  std::string err;
  if (!lfm::ep_unique_id(out, err)) {
    lfm::g_error = err;
    return LFM_ERR_STATE;
  }
  return LFM_OK;
}

lfm_status lfm_ep_init(lfm_engine* e, const uint8_t* id, int rank, int world) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!id || world < 1 || world > (int)lfm::N_EXPERT || lfm::N_EXPERT % world != 0 || rank < 0 || rank >= world) {
      lfm::set_err(&I, "expert-parallel group: world must divide 32 and 0 <= rank < world");
      return LFM_ERR_ARG;
    }
    if (!I.use_tc) {
      lfm::set_err(&I, "the expert-parallel prompt path runs on the tensor-core GEMMs (unset LFM_PREFILL=fp32)");
      return LFM_ERR_STATE;
    }
    lfm::ep_comm_destroy(I.ep);
    I.ep_on = false;
    std::string err;
    if (!lfm::ep_comm_init(I.ep, id, rank, world, err)) {
      lfm::set_err(&I, err);
      return LFM_ERR_STATE;
    }
    I.ep_on = true;
    return LFM_OK;
  });
}

lfm_status lfm_ep_prefill(lfm_engine* e, uint32_t session, const uint32_t* ids, uint32_t n, uint32_t* next_token) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!I.ep_on) {
      lfm::set_err(&I, "no expert-parallel group (lfm_ep_init)");
      return LFM_ERR_STATE;
    }
    lfm_status st = check_ids(e, ids, n, 0);
    if (st) return st;
    uint32_t t;
    if (session == LFM_EP_OWN_SESSION) {
      I.ensure_state();
      CK(cudaMemsetAsync(I.conv_state, 0, (size_t)std::max(I.n_conv, 1) * lfm::DIM * 2 * 4, I.stream));
      I.run_prefill(ids, (int)n, 0, true);
      t = (uint32_t)I.h_io[2];
    } else {
      if (I.batch.nsess == 0 || I.batch.ctx != I.ctx || session >= I.batch.nsess) {
        lfm::set_err(&I, "session out of range (lfm_batch_create)");
        return LFM_ERR_ARG;
      }
      t = I.batch_prefill(session, ids, (int)n, true);
    }
    if (next_token) *next_token = t;
    return LFM_OK;
  });
}

lfm_status lfm_ep_plan(const int32_t* sel, uint32_t nslots, uint32_t world, int32_t* counts, int32_t* order) {
  if ((!sel && nslots) || !counts || (!order && nslots) || world < 1 || world > lfm::N_EXPERT ||
      lfm::N_EXPERT % world != 0) {
    lfm::g_error = "lfm_ep_plan: bad argument";
    return LFM_ERR_ARG;
  }
  for (uint32_t j = 0; j < nslots; j++)
    if (sel[j] < 0 || sel[j] >= (int32_t)lfm::N_EXPERT) {
      lfm::g_error = "lfm_ep_plan: expert id out of range";
      return LFM_ERR_ARG;
    }
  lfm::ep_plan(sel, (int)nslots, (int)world, counts, order);
  return LFM_OK;
}

lfm_status lfm_ep_finalize(lfm_engine* e) {
  return guarded(e, [&]() -> lfm_status {
    lfm::ep_comm_destroy(e->impl.ep);
    e->impl.ep_on = false;
    return LFM_OK;
  });
}

lfm_status lfm_batch_prefill_many(lfm_engine* e, const uint32_t* sessions, const uint32_t* ids,
                                  const uint32_t* lens, uint32_t count, uint32_t* next_tokens) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (I.batch.nsess == 0 || I.batch.ctx != I.ctx) {
      lfm::set_err(&I, "no session slots for the current context length (lfm_batch_create)");
      return LFM_ERR_ARG;
    }
    if (!sessions || !ids || !lens || !next_tokens || count == 0 || count > I.batch.nsess) {
      lfm::set_err(&I, "batch prefill: bad arguments");
      return LFM_ERR_ARG;
    }
    std::vector<uint8_t> seen(I.batch.nsess, 0);
    uint64_t total = 0;
    for (uint32_t i = 0; i < count; i++) {
      if (sessions[i] >= I.batch.nsess || seen[sessions[i]]) {
        lfm::set_err(&I, "batch prefill: sessions must be distinct and in range");
        return LFM_ERR_ARG;
      }
      seen[sessions[i]] = 1;
      if (lens[i] == 0 || lens[i] > I.ctx) {
        lfm::set_err(&I, "batch prefill: every prompt needs 1..ctx tokens");
        return LFM_ERR_ARG;
      }
      total += lens[i];
    }
    if (total > (1u << 20)) {
      lfm::set_err(&I, "batch prefill: more than 2^20 tokens in one call");
      return LFM_ERR_ARG;
    }
    for (uint64_t i = 0; i < total; i++)
      if (ids[i] >= I.hp.vocab) {
        lfm::set_err(&I, "token out of range");
        return LFM_ERR_ARG;
      }
    I.batch_prefill_many(sessions, ids, lens, (int)count, next_tokens);
    return LFM_OK;
  });
}

lfm_status lfm_batch_decode(lfm_engine* e, const uint32_t* sessions, const uint32_t* tokens,
                            const uint32_t* positions, uint32_t count, uint32_t* next_tokens) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (I.batch.nsess == 0 || I.batch.ctx != I.ctx) {
      lfm::set_err(&I, "no session slots for the current context length (lfm_batch_create)");
      return LFM_ERR_ARG;
    }
    if (!sessions || !tokens || !positions || !next_tokens || count == 0 || count > I.batch.nsess) {
      lfm::set_err(&I, "batch decode: bad arguments");
      return LFM_ERR_ARG;
    }
    std::vector<uint8_t> seen(I.batch.nsess, 0);
    for (uint32_t i = 0; i < count; i++) {
      if (sessions[i] >= I.batch.nsess || seen[sessions[i]]) {
        lfm::set_err(&I, "batch decode: sessions must be distinct and in range");
        return LFM_ERR_ARG;
      }
      seen[sessions[i]] = 1;
      if (tokens[i] >= I.hp.vocab || positions[i] >= I.ctx) {
        lfm::set_err(&I, "batch decode: token or position out of range");
        return LFM_ERR_ARG;
      }
    }
    I.batch.last_count = 0;
    I.run_batch_decode(count, tokens, positions, sessions, next_tokens);
    I.batch.last_count = count;
    return LFM_OK;
  });
}

lfm_status lfm_batch_logits(lfm_engine* e, uint32_t index, float* logits) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!logits || I.batch.nsess == 0 || index >= I.batch.last_count) {
      lfm::set_err(&I, "batch logits: index " + std::to_string(index) + " is not an entry of the last batch decode step (" +
                           std::to_string(I.batch.last_count) + " entries)");
      return LFM_ERR_ARG;
    }
    CK(cudaMemcpy(logits, I.batch.logits + (size_t)index * I.hp.vocab, (size_t)I.hp.vocab * 4,
                  cudaMemcpyDeviceToHost));
    return LFM_OK;
  });
}

float lfm_last_device_ms(lfm_engine* e) { return e ? e->impl.last_ms : 0.f; }

lfm_status lfm_step_trace(lfm_engine* e, int enable, uint64_t* out, size_t cap, uint32_t* n_stages,
                          uint32_t* n_ctas) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    I.ensure_state();
    if (n_stages) *n_stages = I.step_active() ? (uint32_t)I.nstages : 0;
    if (n_ctas) *n_ctas = I.step_active() ? (uint32_t)I.sms : 0;
    if (out && I.step_active()) {
      const size_t need = (size_t)I.nstages * I.sms * lfm::STEP_TRACE_FIELDS;
      if (cap < need) {
        lfm::set_err(&I, "trace buffer too small");
        return LFM_ERR_ARG;
      }
      std::vector<unsigned long long> all((size_t)lfm::STEP_MAX_STAGES * lfm::STEP_MAX_CTAS * lfm::STEP_TRACE_FIELDS);
      CK(cudaMemcpy(all.data(), I.trace, need * 8, cudaMemcpyDeviceToHost));
      memcpy(out, all.data(), need * 8);
    }
    const bool on = enable != 0;
    if (on != I.trace_on) {
      I.trace_on = on;
      I.drop_graphs();  // the captured launches carry the trace pointer
    }
    return LFM_OK;
  });
}

const char* lfm_engine_info(lfm_engine* e) {
  if (!e) return "{}";
  EngineImpl& I = e->impl;
  std::string path = I.step_active() ? "persistent-step" : (I.use_mvt ? "kernel-chain-tma" : "kernel-chain-simt");
  if (!I.state_ready) path = I.use_step ? "persistent-step (pending first decode)" : path;
  std::string reason = I.step_reason;
  for (char& ch : reason)
    if (ch == '"' || ch == '\\') ch = '\'';
  I.info = "{\"decode_path\": \"" + path + "\", \"step_reason\": \"" + reason + "\", \"sms\": " +
           std::to_string(I.sms) + ", \"weight_bytes\": " + std::to_string(I.weight_bytes) + ", \"pdl\": " +
           (I.pdl ? "true" : "false") + ", \"graph\": " + (I.use_graph ? "true" : "false") +
           ", \"step_stages\": " + std::to_string(I.nstages) + ", \"launches_per_decode\": " +
           std::to_string(I.launches_per_decode) + ", \"prefill_path\": \"" +
           (I.use_tc ? "tcgen05 Q6_K GEMM (n >= " + std::to_string(I.tc_min) + ")" : std::string("fp32 CUDA-core")) +
           "\"}";
  return I.info.c_str();
}

lfm_status lfm_reset_session(lfm_engine* e) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (I.state_ready) {
      CK(cudaMemsetAsync(I.conv_state, 0, (size_t)std::max(I.n_conv, 1) * lfm::DIM * 2 * 4, I.stream));
      CK(cudaStreamSynchronize(I.stream));
    }
    return LFM_OK;
  });
}

lfm_status lfm_snapshot_cache(lfm_engine* e, uint32_t valid, uint8_t* buf, size_t cap, size_t* len) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!I.state_ready) {
      lfm::set_err(&I, "no resident state");
      return LFM_ERR_STATE;
    }
    if (valid > I.ctx) {
      lfm::set_err(&I, "snapshot range");
      return LFM_ERR_ARG;
    }
    const size_t need = (size_t)I.n_attn * 2 * valid * lfm::KV_HEADS * lfm::HEAD_DIM * 4 +
                        (size_t)I.n_conv * lfm::DIM * 2 * 4;
    if (len) *len = need;
    if (!buf) return LFM_OK;
    if (cap < need) {
      lfm::set_err(&I, "snapshot buffer too small");
      return LFM_ERR_ARG;
    }
    std::vector<uint8_t> v = I.snapshot(valid);
    memcpy(buf, v.data(), v.size());
    return LFM_OK;
  });
}

lfm_status lfm_restore_cache(lfm_engine* e, uint32_t valid, const uint8_t* buf, size_t len) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (valid > I.ctx || (!buf && len)) {
      lfm::set_err(&I, "restore context");
      return LFM_ERR_ARG;
    }
    I.ensure_state();
    I.restore(valid, buf, len);
    return LFM_OK;
  });
}

lfm_status lfm_snapshot_logits(lfm_engine* e, float* logits) {
  return guarded(e, [&]() -> lfm_status {
    EngineImpl& I = e->impl;
    if (!I.state_ready || !logits) {
      lfm::set_err(&I, "no resident state");
      return LFM_ERR_STATE;
    }
    CK(cudaMemcpy(logits, I.logits, (size_t)I.hp.vocab * 4, cudaMemcpyDeviceToHost));
    return LFM_OK;
  });
}

lfm_status lfm_counters_get(lfm_engine* e, lfm_counters* out) {
  if (!e || !out) return LFM_ERR_ARG;
  *out = e->impl.ctr;
  return LFM_OK;
}

const char* lfm_device_name(lfm_engine* e) { return e ? e->impl.name.c_str() : ""; }
const char* lfm_last_error(lfm_engine* e) { return e ? e->impl.err.c_str() : lfm::g_error.c_str(); }
const char* lfm_global_error(void) { return lfm::g_error.c_str(); }

}  // extern "C"
