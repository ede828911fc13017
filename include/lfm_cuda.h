/*
 * lfm_cuda.h — C ABI of the B200 (sm_100a) LFM2.5-8B-A1B Q6_K token-loop engine.
 *
 * This is the drop-in boundary that replaces the reference's
 * `lfm2_engine::gpu_lfm::GpuEngine` (engine/src/gpu_lfm.rs:23-245 and
 * engine/src/gpu_lfm/resident_graph.rs:90-602) for its callers
 * (`lfm2-greedy`, engine/src/main.rs:196-281; `api_stream`,
 * engine/src/bin/api_stream.rs:47-77; `persistent`). Each entry point cites
 * the reference method it stands in for.
 *
 * Conventions
 *  - Plain C types only; no CUDA or torch types cross the boundary.
 *  - Every call returns an lfm_status; on failure lfm_last_error() (engine
 *    calls) or lfm_global_error() (creation) holds a message. No C++
 *    exception crosses the boundary.
 *  - Calls are synchronous and blocking: they return after the device work
 *    they issued has completed, like the reference's fence-waited submits
 *    (engine/src/vulkan.rs:435-545). One engine per GPU per host thread; an
 *    engine is not thread-safe (the reference's GpuOps is !Sync).
 *  - The engine owns all device memory; callers own host buffers.
 *  - Input validation follows the reference: ids < vocab, n >= 1,
 *    start_pos + n <= ctx, ctx <= 4096 (resident_graph.rs:161-172,
 *    ops.rs:488-491), 1..=64 ids for lfm_forward_token
 *    (resident_graph.rs:95-98).
 */
#ifndef LFM_CUDA_H
#define LFM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t lfm_status;
#define LFM_OK 0
#define LFM_ERR_ARG 1        /* invalid argument (range, size, null) */
#define LFM_ERR_MODEL 2      /* GGUF parse / geometry / missing tensor */
#define LFM_ERR_CUDA 3       /* CUDA runtime error */
#define LFM_ERR_STATE 4      /* call not valid in the current engine state */
#define LFM_ERR_DEVICE 5     /* device-side status word reported a failure */

#define LFM_MAX_CTX 4096u
#define LFM_PREFILL_CHUNK 64u /* work_bound.rs:6 PREFILL_CHUNK */

typedef struct lfm_engine lfm_engine;

/* Hyperparams (engine/src/lfm.rs:31-49, load_hyperparams :102-145). */
typedef struct lfm_hparams {
  uint32_t dim, heads, head_dim, n_layers, vocab;
  uint32_t n_expert, n_used, expert_ff, n_ff, dense_lead, conv_l_cache;
  uint32_t eos;
  float eps, rope_theta;
  uint32_t kv_heads[64]; /* per layer: 0 = short-conv, 8 = attention */
} lfm_hparams;

/* Counters reported by the reference's result lines (main.rs:273-280,
 * persistent.rs:230-242): dispatches, GPU argmax, decode-plan reuse. */
typedef struct lfm_counters {
  uint64_t kernel_launches;       /* gpu_dispatch_count */
  uint64_t gpu_argmax;            /* gpu_argmax_dispatches */
  uint64_t graph_replays;         /* decode_command_buffer_reuses */
  uint64_t graph_captures;
  uint64_t prefill_tokens;        /* prefill_weight_reuse_tokens */
  uint64_t expert_grouped_launches; /* expert_grouped_dispatches */
} lfm_counters;

/* ---- engine lifetime ------------------------------------------------- */

/* The model check of GpuEngine::load without a device: parse the GGUF header
 * with the reference parser's rules (parser::gguf::parse,
 * parser/src/gguf.rs:304-440), read and validate the hyperparameters
 * (load_hyperparams, lfm.rs:102-145) and check that every tensor the engine
 * loads exists with its GGML type and shape. Reads no tensor payload.
 * LFM_ERR_MODEL with the message in lfm_global_error on any violation;
 * `out` (may be null) receives the hyperparameters. */
lfm_status lfm_model_inspect(const char* gguf_path, lfm_hparams* out);

/* GpuEngine::load(&ModelFile) (gpu_lfm.rs:51-115): parse the GGUF, validate
 * geometry (lfm.rs:115-126), repack every Q6_K tensor into the device layout
 * and upload it. `device` is the CUDA ordinal. */
lfm_status lfm_engine_create(const char* gguf_path, int device, lfm_engine** out);
void lfm_engine_destroy(lfm_engine* e);

/* GpuEngine::set_ctx (gpu_lfm.rs:117-119). ctx <= 4096. Takes effect before
 * the first forward (resident state is sized on first use, like
 * resident_graph.rs:173-181). */
lfm_status lfm_engine_set_ctx(lfm_engine* e, uint32_t ctx);

/* GpuEngine.hp (lfm.rs:31-49). */
lfm_status lfm_hparams_get(lfm_engine* e, lfm_hparams* out);

/* ---- token loop ------------------------------------------------------ */

/* GpuEngine::forward(ids, start_pos) -> Vec<f32> (gpu_lfm.rs:243-245 ->
 * resident_graph.rs:160-557): run n tokens starting at start_pos, write the
 * last token's full-vocabulary logits (vocab floats) into `logits`. */
lfm_status lfm_forward_logits(lfm_engine* e, const uint32_t* ids, uint32_t n,
                              int64_t start_pos, float* logits);

/* GpuEngine::forward_token(ids, position) -> u32 (resident_graph.rs:90-101):
 * 1..=64 ids, device-side argmax of the last token's logits (ties -> lowest
 * id, NaN never wins; kernels/persistent.rs:12-53). n == 1 replays the
 * resident CUDA graph of the decode step. */
lfm_status lfm_forward_token(lfm_engine* e, const uint32_t* ids, uint32_t n,
                             uint32_t position, uint32_t* next_token);

/* Device-resident greedy loop (main.rs:174-195 / api_stream.rs:56-77 with the
 * host only reading results): prefill `prompt` in <=64-token chunks, then
 * decode up to n tokens, stopping at `eos`. Tokens go to out_tokens (cap n);
 * *n_out receives the count. Equivalent to calling lfm_forward_token in a
 * loop (the api_stream request loop). */
lfm_status lfm_generate(lfm_engine* e, const uint32_t* prompt, uint32_t prompt_len,
                        uint32_t n, uint32_t eos, uint32_t* out_tokens, uint32_t* n_out);

/* Device-resident greedy decode: `steps` decode steps starting with
 * first_token at start_pos, each step consuming the previous step's device
 * argmax with no host round trip (the reference's replayed decode plan with a
 * device-side position, vulkan/reusable.rs:135-173, without its per-step
 * fence wait). out_tokens receives every step's argmax (no EOS stop);
 * *device_ms the CUDA-event time of steps 2..steps (of step 1 if steps == 1). */
lfm_status lfm_decode_loop(lfm_engine* e, uint32_t first_token, uint32_t start_pos, uint32_t steps,
                           uint32_t* out_tokens, float* device_ms);

/* CUDA-event device time (ms) of the last forward / decode call. */
float lfm_last_device_ms(lfm_engine* e);

/* Independent sessions decoded together (multi-session throughput). The
 * reference serves one session at a time and switches sessions by
 * snapshot/restore of its single buffer set (persistent.rs:164-176,
 * resident_graph.rs:572-602); here each session slot owns a KV cache and a
 * conv state at the engine's current context length, and one batched step
 * advances many sessions at once (every weight is read once per step).
 * lfm_batch_create: n_sessions slots (1..4096), replacing earlier ones. */
lfm_status lfm_batch_create(lfm_engine* e, uint32_t n_sessions);
/* Fresh prompt of session `session` at positions 0..n-1 (its conv state is
 * reset first, like reset_session); *next_token = greedy next token. */
lfm_status lfm_batch_prefill(lfm_engine* e, uint32_t session, const uint32_t* ids, uint32_t n,
                             uint32_t* next_token);
/* Fresh prompts of `count` distinct sessions prefilled together (no
 * reference counterpart: the reference prefills one session at a time):
 * session sessions[i] gets the lens[i] ids that follow the earlier sessions'
 * in `ids`, at positions 0..lens[i]-1. Every projection runs as one GEMM over
 * all the prompts' tokens; attention and the short conv stay per session.
 * next_tokens[i] = greedy next token of session sessions[i] (as
 * lfm_batch_prefill). At most 2^20 tokens per call. */
lfm_status lfm_batch_prefill_many(lfm_engine* e, const uint32_t* sessions, const uint32_t* ids,
                                  const uint32_t* lens, uint32_t count, uint32_t* next_tokens);
/* One decode step of `count` distinct sessions: token tokens[i] at position
 * positions[i] of session sessions[i]; next_tokens[i] = greedy next token
 * (forward_token semantics per session, resident_graph.rs:90-101). */
lfm_status lfm_batch_decode(lfm_engine* e, const uint32_t* sessions, const uint32_t* tokens,
                            const uint32_t* positions, uint32_t count, uint32_t* next_tokens);
/* ---- expert-parallel prompt path (one process per GPU) ---------------
 * New capability (the reference is single-GPU): the routed-expert FFN of
 * every MoE layer of a prompt runs on the GPU that owns each expert (expert e
 * on rank e / (32 / world)); routed (token, rank) activation rows go to the
 * owner and the down rows come back over NCCL point-to-point transfers, then
 * they are combined in rank order as the reference's combine does
 * (kernels/resident.rs:101-117). Attention, short conv, dense FFNs and the
 * lm_head stay on each rank's own tokens. */

/* A fresh NCCL id (128 bytes) that rank 0 creates and shares with the other
 * ranks (for example through torch.distributed). */
lfm_status lfm_ep_unique_id(uint8_t* id_out);
/* Join the expert-parallel group: world divides 32, 0 <= rank < world. Every
 * rank calls it with the same id. A group of one runs the same exchange
 * through NCCL with itself (all 32 experts local). */
lfm_status lfm_ep_init(lfm_engine* e, const uint8_t* id, int rank, int world);
#define LFM_EP_OWN_SESSION 0xFFFFFFFFu
/* Prefill a fresh prompt of n tokens at position 0, expert-parallel: into
 * session slot `session` (as lfm_batch_prefill) or, with LFM_EP_OWN_SESSION,
 * into the engine's own session (as reset_session + forward). Collective:
 * every rank of the group calls it at the same time (any n >= 1 per rank).
 * next_token = greedy next token of this rank's prompt. */
lfm_status lfm_ep_prefill(lfm_engine* e, uint32_t session, const uint32_t* ids, uint32_t n, uint32_t* next_token);
/* The send plan of one MoE layer (host only, no device): slot j = token * 4 +
 * rank with expert sel[j] goes to rank sel[j] / (32 / world); counts[world] =
 * slots per destination, order[nslots] = slot of each send position
 * (destinations ascending, slots ascending within one). */
lfm_status lfm_ep_plan(const int32_t* sel, uint32_t nslots, uint32_t world, int32_t* counts, int32_t* order);
/* Leave the expert-parallel group (before the process group is torn down). */
lfm_status lfm_ep_finalize(lfm_engine* e);

/* ---- streaming text of sessions decoded together (host only) ---------
 * The text path that runs beside the GPU loop: per session, token pieces
 * (raw bytes, possibly ending inside a UTF-8 sequence) are assembled as the
 * reference's StreamDecoder / Utf8Stream does (tokenizer/src/stream.rs:48-189:
 * complete text emitted, an incomplete tail kept, invalid bytes an error or
 * one U+FFFD per maximal invalid subsequence) and cleaned as its DecodedText
 * does (engine/src/text_output.rs:9-106: the decoder's clean_spaces over the
 * text so far, the last 16 bytes withheld until more text or the end). The
 * pieces are the caller's: the tokenizer's token_to_piece(id, render_special)
 * of every id, concatenated, with piece t at bytes [off[t], off[t+1]). */
typedef struct lfm_text lfm_text;
lfm_status lfm_text_create(const uint8_t* piece_bytes, const uint64_t* piece_off, uint32_t n_tokens,
                           uint32_t n_sessions, int clean_spaces, int replace_invalid, lfm_text** out);
void lfm_text_destroy(lfm_text* t);
/* One token for each of `count` entries (sessions may repeat; entries are
 * applied in order). The text each entry completes is appended to `out`
 * (capacity `cap` bytes): entry i's text is out[out_off[i], out_off[i+1]).
 * LFM_ERR_STATE if a session's bytes can never become valid UTF-8 under the
 * error policy (that session keeps its buffer; call lfm_text_reset). */
lfm_status lfm_text_push(lfm_text* t, const uint32_t* sessions, const uint32_t* tokens, uint32_t count, char* out,
                         size_t cap, uint64_t* out_off);
/* End of a session's stream: its remaining text (withheld suffix, and the
 * incomplete tail as U+FFFD under the replace policy); the session is empty
 * afterwards. LFM_ERR_STATE for an incomplete or invalid tail under the
 * error policy. */
lfm_status lfm_text_finish(lfm_text* t, uint32_t session, char* out, size_t cap, size_t* len);
lfm_status lfm_text_reset(lfm_text* t, uint32_t session);
const char* lfm_text_error(void);

/* Full logits (vocab floats) of entry `index` of the last lfm_batch_decode
 * step (snapshot_resident_logits, resident_graph.rs:561-568, for one batch entry). */
lfm_status lfm_batch_logits(lfm_engine* e, uint32_t index, float* logits);

/* Per-stage timeline of the persistent decode step, for profiling (the
 * reference's per-dispatch GPU timestamp queries, vulkan/profile.rs:18-45,
 * enabled by LFM_PROFILE_DISPATCH). `enable`
 * switches %globaltimer stamps on for later decode steps; when `out` is
 * non-null the last step's record is copied out as [n_stages][n_ctas][8]
 * u64: stage start, activations staged, first weight tile ready, stage done
 * (%globaltimer ns), then SM clock cycles waiting for weight tiles, tiles,
 * cycles of tile compute, cycles of epilogues. n_stages = n_ctas = 0 when the
 * kernel chain runs. */
lfm_status lfm_step_trace(lfm_engine* e, int enable, uint64_t* out, size_t cap, uint32_t* n_stages,
                          uint32_t* n_ctas);

/* JSON description of the engine's decode path (persistent step or kernel
 * chain, and why), SM count, resident weight bytes and launches per decode
 * step (the reference reports its device and profile header at load,
 * vulkan.rs:280-286, main.rs:198). The string stays valid until the next
 * call on this engine. */
const char* lfm_engine_info(lfm_engine* e);

/* GpuEngine::reset_session (resident_graph.rs:105-115): zero the short-conv
 * state; stale KV beyond the valid prefix is never attended. */
lfm_status lfm_reset_session(lfm_engine* e);

/* GpuEngine::snapshot_resident_cache(valid) (resident_graph.rs:572-602):
 * per layer in order, attention layers write K then V for positions
 * [0,valid) as f32 words laid out [p][kv_head*64+d]; short-conv layers write
 * their state as [channel][slot] f32. Pass buf = NULL to query *len. */
lfm_status lfm_snapshot_cache(lfm_engine* e, uint32_t valid, uint8_t* buf, size_t cap,
                              size_t* len);

/* GpuEngine::restore_session(valid, bytes) (resident_graph.rs:119-158): the
 * inverse of lfm_snapshot_cache; K/V words are rounded to fp16 storage. */
lfm_status lfm_restore_cache(lfm_engine* e, uint32_t valid, const uint8_t* buf, size_t len);

/* GpuEngine::snapshot_resident_logits (resident_graph.rs:561-568): the last
 * full-vocabulary logits left on the device (vocab floats). */
lfm_status lfm_snapshot_logits(lfm_engine* e, float* logits);

lfm_status lfm_counters_get(lfm_engine* e, lfm_counters* out);
const char* lfm_device_name(lfm_engine* e);      /* GpuEngine::device_name */
const char* lfm_last_error(lfm_engine* e);
const char* lfm_global_error(void);              /* failures before an engine exists */

/* ---- kernel-level entry points (device pointers, for parity tests and
 * the Q6_K microbench; stream = cudaStream_t or NULL) ------------------- */

/* Size in bytes of the device layout of a [in_dim, rows] Q6_K matrix (equal
 * to the GGUF size: every byte kept, no padding). */
size_t lfm_q6k_device_bytes(uint32_t in_dim, uint32_t rows);

/* Repack GGUF Q6_K rows (210-byte super-blocks, q6k.rs:8-17) held in HOST
 * memory into the device layout at `dst_dev` (the reference's load-time
 * repack, q6k.rs:25-39 / gpu_lfm.rs:83-87). */
lfm_status lfm_q6k_upload(const uint8_t* gguf_rows, uint32_t in_dim, uint32_t rows, void* dst_dev);

/* Dequantise rows [row0, row0+nrows) of a device-layout matrix to f32
 * (bit-exact with q6k.rs:74-146). out_dev: nrows*in_dim floats. */
lfm_status lfm_q6k_dequant(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t row0,
                           uint32_t nrows, float* out_dev, void* stream);

/* y[o + j*rows] = sum_k W[o,k] x[k + j*in_dim] for n columns (q6k_matmul,
 * ops.rs:340-374). */
lfm_status lfm_q6k_matmul(const void* w_dev, uint32_t in_dim, uint32_t rows, const float* x_dev,
                          uint32_t n, float* y_dev, void* stream);

/* Routed-expert matvec (q6k_routed, resident_graph.rs:446-495): for slot
 * s < 4, y[s*rows + o] = sum_k W[expert_ids[s]][o,k] x[s*x_stride + k].
 * `w_dev` holds all experts ([in_dim, rows, n_expert]); expert_ids_dev is a
 * device int32[4]. */
lfm_status lfm_q6k_routed(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t n_expert,
                          const int32_t* expert_ids_dev, const float* x_dev, uint32_t x_stride,
                          float* y_dev, void* stream);

/* Sigmoid router + top-k (kernels/resident.rs:58-99, lfm.rs:613-637) for n
 * tokens: logits [n][n_expert] -> sel_ids [n][4] int32, sel_w [n][4] f32. */
lfm_status lfm_route(const float* logits_dev, const float* bias_dev, uint32_t n_expert, uint32_t n,
                     int32_t* sel_ids_dev, float* sel_w_dev, void* stream);

/* Deterministic argmax (kernels/persistent.rs:12-53): first maximum, NaN
 * never wins. */
lfm_status lfm_argmax(const float* x_dev, uint32_t n, uint32_t* out_dev, void* stream);

/* lfm_argmax without any device allocation. It has no counterpart in the
 * reference. lfm_argmax allocates 2 KiB of scratch per call with
 * cudaMallocAsync; callers that may not allocate device memory at call time
 * (a host that has handed the whole device to its own memory pool, or code
 * running where the CUDA allocator must not be entered) call this instead.
 * Its scratch is a fixed 2 KiB device array inside this library, present on
 * every device that loads it until the process exits. Same result as
 * lfm_argmax; n must be 1..2^30 (larger n returns LFM_ERR_ARG with a message
 * in lfm_ops_error). The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress), so make that first call before any stream
 * capture. The address is cached per device together with the context it
 * belongs to; after a device reset the next call looks it up again. All
 * calls on a device share the one array: calls that overlap on the GPU
 * (different streams, no ordering between them) race and may return wrong
 * indices. */
lfm_status lfm_argmax_noalloc(const float* x_dev, uint32_t n, uint32_t* out_dev, void* stream);

/* Tensor-core GEMM core of the prompt path (tcgen05 MMA, fp32 accumulation in
 * tensor memory): c[i][j] = sum_k a[i][k] * b[j][k] for fp16 a [m][k] and
 * b [n][k] (both row-major), fp32 c [m][n]. m % 128 == 0, n % 256 == 0,
 * k % 64 == 0. Synchronous; LFM_ERR_DEVICE if a bounded wait timed out.
 * Stands in for the reference's f32_matmul dispatch (kernels.rs:552-574)
 * at the GEMM level; the Q6_K prompt GEMMs are built on it. */
lfm_status lfm_tc_gemm_f16(const void* a_dev, const void* b_dev, uint32_t m, uint32_t n, uint32_t k, float* c_dev,
                           void* stream);

/* The same core with an MN-major second operand, the layout of the V cache
 * (positions x 64 contiguous values): c[i][j] = sum_k a[i][k] * b[k][j] for
 * fp16 a [m][k], b [k][64], fp32 c [m][64]; m % 128 == 0, k % 64 == 0.
 * Synchronous. The P*V product of prompt attention (lfm.rs:425-437). */
lfm_status lfm_tc_gemm_f16_bmn(const void* a_dev, const void* b_dev, uint32_t m, uint32_t k, float* c_dev,
                               void* stream);

/* Causal GQA prompt attention on the tensor cores (the reference's prompt
 * attention, lfm.rs:395-437 / kernels.rs:672-763): for token j < n at
 * position start + j and query head h < 32 (KV head h / 4),
 * out[j*out_stride + h*64 + d] = sum_t softmax_t(q.k_t / 8) v_t[d] over
 * positions t <= start + j, with q at q_dev[j*q_stride + h*64 ..] (fp32) and
 * the fp16 caches laid out [8][ctx][64]. Synchronous. */
lfm_status lfm_attention_prefill(const float* q_dev, uint32_t q_stride, const void* k_cache, const void* v_cache,
                                 uint32_t ctx, uint32_t start, uint32_t n, float* out_dev, uint32_t out_stride,
                                 void* stream);

/* Tensor-core (tcgen05 / TMEM) Q6_K prompt GEMM, the prefill counterpart of
 * lfm_q6k_matmul with the same contract: y[o + j*rows] = sum_k W[o,k]
 * x[k + j*in_dim] for n columns (q6k_prompt, ops.rs:340-374). Weights enter
 * the tensor cores as the integers sc*(q-32) with d applied per super-block,
 * activations as an fp16 hi/lo pair; fp32 accumulation. rows % 128 == 0.
 * Synchronous (scratch is allocated per call); LFM_ERR_DEVICE if a bounded
 * wait timed out. */
lfm_status lfm_q6k_prompt_gemm(const void* w_dev, uint32_t in_dim, uint32_t rows, const float* x_dev,
                               uint32_t n, float* y_dev, void* stream);

/* Grouped routed-expert form (q6k_grouped over expert_groups lists,
 * resident_graph.rs:450-495): for token t < n and rank r < 4 with
 * e = expert_ids[t*4 + r] and slot q = t*4 + r,
 * y[q*rows + o] = sum_k W[e][o,k] x[(q / x_div)*in_dim + k]; x_div is 4 (one
 * activation row per token, the gate/up input) or 1 (one per slot, the down
 * input). n_expert == 32, rows % 128 == 0. The four ids of a token must be
 * distinct, as the router's top 4 are (LFM_ERR_ARG otherwise; ids outside
 * 0..31 select no expert and leave their slot's rows unwritten).
 * Synchronous. */
lfm_status lfm_q6k_prompt_grouped(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t n_expert,
                                  const int32_t* expert_ids_dev, const float* x_dev, uint32_t x_div,
                                  uint32_t n, float* y_dev, void* stream);

/* The prompt GEMMs' weight operand expanded ahead of time: out_dev (fp16,
 * [rows][in_dim], 2 bytes per weight, 16-byte aligned) receives the exact
 * integers sc*(q-32) of every weight (q6k.rs:74-146 without the super-block
 * scale d, which the GEMM applies per super-block). The engine builds this
 * operand for every Q6_K matrix when it loads a model (unless
 * LFM_PREFILL_X16=0 or the device lacks the room). No counterpart in the
 * reference, whose prompt kernels dequantise on the fly. Asynchronous on
 * `stream`. */
lfm_status lfm_q6k_expand_f16(const void* w_dev, uint32_t in_dim, uint32_t rows, void* out_dev, void* stream);

/* lfm_q6k_prompt_gemm and lfm_q6k_prompt_grouped reading their weight
 * operand from w16_dev (lfm_q6k_expand_f16 of w_dev; w_dev still supplies the
 * super-block scales d). Same contracts and results, bit for bit. */
lfm_status lfm_q6k_prompt_gemm_x16(const void* w_dev, const void* w16_dev, uint32_t in_dim, uint32_t rows,
                                   const float* x_dev, uint32_t n, float* y_dev, void* stream);
lfm_status lfm_q6k_prompt_grouped_x16(const void* w_dev, const void* w16_dev, uint32_t in_dim, uint32_t rows,
                                      uint32_t n_expert, const int32_t* expert_ids_dev, const float* x_dev,
                                      uint32_t x_div, uint32_t n, float* y_dev, void* stream);

/* Failure-detection self-test (no counterpart in the reference, whose
 * watchdog handling is vulkan/fence_stop.rs): one thread waits on an
 * mbarrier that nothing completes, through the library's bounded wait (about
 * one second of SM cycles). On return *status holds the device status word
 * the wait raised (1 = timed out; 0 or 99 would mean the bound failed) and
 * *cycles the SM cycles the wait took. Synchronous; the context stays usable. */
lfm_status lfm_selftest_wait_timeout(uint32_t* status, uint64_t* cycles);

/* Message of the last failing kernel-level call on this thread. */
const char* lfm_ops_error(void);

#ifdef __cplusplus
}
#endif
#endif /* LFM_CUDA_H */
