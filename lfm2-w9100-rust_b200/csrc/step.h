// Persistent decode step: one cooperative launch runs a whole batch-1 decode
// token (embedding, 24 layers, lm_head + argmax). See step.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "kernels.h"

namespace lfm {

enum StepStageType {
  ST_EMBED = 0,   // x = dequant(token_embd row token)
  ST_QKV,         // q|k|v = W (rmsnorm x)
  ST_ATTN,        // head norm + rope + fp16 KV write + split attention + merge -> a
  ST_RESID,       // x += W in (o-proj, out_proj)
  ST_CONV,        // in_proj + short conv -> gated, rolls conv state
  ST_ROUTER,      // (unused: routing is folded into the residual stage before each MoE FFN)
  ST_XSWIGLU,     // routed gate/up + SwiGLU -> sw[4][ff]
  ST_XDOWN,       // routed down + rank-ordered combine -> x += ...
  ST_SWIGLU,      // dense gate/up + SwiGLU -> sw
  ST_DOWN28,      // dense down (in = 7168) + residual
  ST_LMHEAD,      // tied lm_head -> logits, two-stage argmax -> io[2]
};

struct StepStage {
  int type;
  int ntiles;        // weight tiles of the stage (ring stages)
  Q6Mat W, W2, W3;
  const float* xin;  // activation input
  const float* norm; // RMSNorm weights (nullptr: none)
  float* out;
  float* resid;
  const float* conv_w;
  float* state;
  const float* rw;   // ST_RESID before an MoE FFN: that layer's router [32][2048] (norm = its ffn_norm)
  const float* bias; // ... and expert bias
  const float* q_norm;
  const float* k_norm;
  __half* kc;
  __half* vc;
  int ff;            // expert ff / x stride
  int dep;           // ST_XSWIGLU / ST_XDOWN: index of the residual stage that publishes the routing
};

constexpr int STEP_MAX_STAGES = 192;
constexpr int STEP_MAX_CTAS = 160;
// producer warps of the step kernel (one per weight-ring slot); every CTA
// needs at least this many tiles in each routed gate/up stage
constexpr int STEP_PRODUCERS = 4;
// Most tiles one CTA may own in a stage whose rows are finished at stage end
// (short conv, SwiGLU, expert and dense down projections).
constexpr int STEP_PART_TILES = 16;
// Trace record per (stage, CTA): %globaltimer ns stamps [0] stage start, [1]
// activations staged, [2] first weight tile ready, [3] arrival at the stage
// barrier; SM clock cycles of consumer warp 0: [4] total wait for weight
// tiles, [6] total tile compute and epilogue; [5] tiles; [7] unused.
constexpr int STEP_TRACE_FIELDS = 8;

// Device-resident control block (zeroed once; barrier counters only grow).
struct StepCtl {
  unsigned bar[STEP_MAX_STAGES];
  unsigned epoch;     // decode steps completed
  unsigned err;       // device status word: a bounded wait timed out
  unsigned abort;     // raised with err; every later wait returns at once
  unsigned attn_cnt[KV_HEADS];
  float2 am_part[STEP_MAX_CTAS];
  // per-CTA router partials of the current MoE layer: 32 expert logits (before
  // the 1/rms factor) and the sum of squares of the CTA's residual rows
  float rpart[STEP_MAX_CTAS][N_EXPERT + 1];
};

struct StepParams {
  const StepStage* stages;
  int nstages;
  StepCtl* ctl;
  int* io;           // [0] token, [1] position, [2] next token
  const float2* rope;
  float* attn_part;  // [8][ceil(ctx/32)][4][66]
  int ctx;
  float eps;
  Q6Mat embd;
  float* x;
  unsigned long long* trace;  // optional [stage][cta][STEP_TRACE_FIELDS]
};

// Dynamic shared memory of the step kernel (weight ring + stage table).
size_t step_smem_bytes();
// Set the kernel attributes and check that one CTA fits per SM (required by
// the cooperative launch); returns the reason when it does not.
cudaError_t step_prepare();
// Registers, shared memory and blocks/SM of the step kernel, for diagnostics.
std::string step_occupancy_report();
// Enqueue one decode step (cooperative launch, one CTA per SM).
cudaError_t step_launch(const StepParams& p, int sms, cudaStream_t s);

}  // namespace lfm
