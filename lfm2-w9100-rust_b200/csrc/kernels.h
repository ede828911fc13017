// Launchers of the B200 kernels. Each launcher names the reference kernel(s)
// it replaces (engine/src/kernels.rs, engine/src/kernels/*.rs).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q6k.cuh"

namespace lfm {

constexpr int DIM = 2048;
constexpr int HEADS = 32;
constexpr int HEAD_DIM = 64;
constexpr int KV_HEADS = 8;
constexpr int N_EXPERT = 32;
constexpr int N_USED = 4;
constexpr int EXPERT_FF = 1792;
constexpr int N_FF = 7168;
constexpr int ATTN_SPLIT = 32;  // positions per decode-attention split (one per lane)

// Activation source of a matvec: x, optionally RMS-normalised with `norm`
// (kernels.rs:576-634 fused as a prologue).
struct XSrc {
  const float* x;
  const float* norm;  // nullptr: use x as is
  float eps;
};

// Per-launch knobs shared by the decode kernels.
struct LaunchCfg {
  cudaStream_t stream = 0;
  bool pdl = false;  // programmatic dependent launch
  int sms = 148;
};

// ---------------------------------------------------------------- decode
// y[r] = W x (q6k_matmul, kernels.rs:832-1025, n == 1)
void mv_plain(const Q6Mat& W, XSrc xs, float* y, const LaunchCfg& c);
// resid[r] += W x (q6k_matmul + residual, kernels/resident.rs:20-31)
void mv_resid(const Q6Mat& W, XSrc xs, float* resid, const LaunchCfg& c);
// Short-conv in_proj + conv (kernels/resident.rs:33-56): gated[ch] from rows
// ch, dim+ch, 2dim+ch of W; rolls state[ch*2 + {0,1}].
void mv_conv(const Q6Mat& W, XSrc xs, const float* conv_w, float* state, float* gated,
             const LaunchCfg& c);
// Dense gate/up + SwiGLU (kernels.rs:543-550): sw[i] = silu(g_i) * u_i.
void mv_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, XSrc xs, float* sw, const LaunchCfg& c);
// Dense down (in = 7168) + residual.
void mv_down7168_resid(const Q6Mat& W, const float* sw, float* resid, const LaunchCfg& c);
// Routed gate/up + SwiGLU for the 4 selected experts (q6k_routed,
// resident_graph.rs:446-473): sw[s*ff + i].
void mv_expert_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, int ff, XSrc xs, const int* sel, float* sw,
                      const LaunchCfg& c);
// Routed down for the 4 selected experts (resident_graph.rs:474-495), then the
// rank-ordered combine into the residual (kernels/resident.rs:101-117).
void mv_expert_down(const Q6Mat& Wd, int ff, const float* sw, const int* sel, const float* selw,
                    float* down, float* resid, unsigned* counter, const LaunchCfg& c);
// Plain routed matvec for the 4 slots (no combine): y[s*orows + o] =
// W[sel[s]] x[s*x_stride ..] (q6k_routed, resident_graph.rs:446-495).
void mv_routed(const Q6Mat& W, int orows, const float* x, int x_stride, const int* sel, float* y,
               const LaunchCfg& c);
// Tied lm_head + two-stage argmax (resident_graph.rs:522-546,
// kernels/persistent.rs:12-53). Writes logits and *token.
void mv_lmhead(const Q6Mat& W, XSrc xs, float* logits, float2* partials, unsigned* counter,
               int* token, const LaunchCfg& c);
// Router logits + sigmoid top-4 (kernels.rs:552-574 + kernels/resident.rs:58-99).
void router_top4(const float* Wr, const float* bias, XSrc xs, int* sel, float* selw,
                 const LaunchCfg& c);
// Same over 32 CTAs (one expert logit each, last CTA selects); lg_scratch
// holds 32 floats, counter one zeroed word.
void router_top4_mc(const float* Wr, const float* bias, XSrc xs, float* lg_scratch, unsigned* counter, int* sel,
                    float* selw, const LaunchCfg& c);
// Embedding row dequant (kernels/resident.rs:4-18) for a device-resident token;
// an id outside the table raises *err (code 4) and reads row 0.
void embed_token(const Q6Mat& E, const int* token, float* x, unsigned* err, const LaunchCfg& c);
// GQA decode attention: head RMSNorm + NEOX RoPE of q/k (kernels.rs:576-670),
// fp16 KV write at *pos (kernels/resident.rs:119-169), split attention and
// merge (kernels/attention_split.rs:3-33).
struct AttnDecodeArgs {
  const float* qkv;      // q[2048] k[512] v[512]
  const float* q_norm;   // [64]
  const float* k_norm;   // [64]
  const float2* rope;    // [ctx][32] (cos, sin)
  const int* pos;        // device position
  __half* kc;            // [8][ctx][64]
  __half* vc;            // [8][ctx][64]
  float* part;           // [8][nsplit][4][66], nsplit = ceil(ctx / ATTN_SPLIT)
  unsigned* counters;    // [8]
  float* out;            // a[2048]
  int ctx;
  float eps;
};
void attn_decode(const AttnDecodeArgs& a, const LaunchCfg& c);

// TMA-staged variants (mvt.cu) for the engine's decode step: 1 CTA per SM,
// bulk-copy weight pipeline issued before the PDL wait. `err` is the engine's
// device error word (raised if a bounded mbarrier wait times out).
bool mvt_supported(const Q6Mat& W);
void mvt_plain(const Q6Mat& W, XSrc xs, float* y, unsigned* err, const LaunchCfg& c);
void mvt_resid(const Q6Mat& W, XSrc xs, float* resid, unsigned* err, const LaunchCfg& c);
// q, k, v projections in one launch: y = [q | k | v] (rows of 16-row tiles).
void mvt_qkv(const Q6Mat& Wq, const Q6Mat& Wk, const Q6Mat& Wv, XSrc xs, float* y, unsigned* err,
             const LaunchCfg& c);
void mvt_conv(const Q6Mat& W, XSrc xs, const float* conv_w, float* state, float* gated, unsigned* err,
              const LaunchCfg& c);
void mvt_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, XSrc xs, float* sw, unsigned* err, const LaunchCfg& c);
void mvt_expert_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, int ff, XSrc xs, const int* sel, float* sw, unsigned* err,
                       const LaunchCfg& c);
void mvt_expert_down(const Q6Mat& Wd, int ff, const float* sw, const int* sel, const float* selw, float* down,
                     float* resid, unsigned* counter, unsigned* err, const LaunchCfg& c);
void mvt_lmhead(const Q6Mat& W, XSrc xs, float* logits, float2* partials, unsigned* counter, int* token,
                unsigned* err, const LaunchCfg& c);

// ------------------------------------------------------------- generic ops
void q6_dequant_rows(const Q6Mat& W, int row0, int nrows, float* out, cudaStream_t s);
void argmax_f32(const float* x, int n, float2* partials, unsigned* counter, int* out,
                cudaStream_t s);
void route_n(const float* logits, const float* bias, int n_expert, int n, int* sel, float* selw,
             cudaStream_t s);

// ---------------------------------------------------------------- prefill
// out[j*rows + r] (+)= sum_k W[r,k] * X[j*in + k] for n tokens (ggml layout
// [in, n] with in fastest). RESID adds into `out`.
void gemm_q6(const Q6Mat& W, const float* X, int n, float* out, bool resid, cudaStream_t s);
// Same with an output row stride `ldo` (out[j*ldo + r]).
void gemm_q6_ld(const Q6Mat& W, const float* X, int n, float* out, int ldo, bool resid, cudaStream_t s);
// Grouped expert GEMM over device-side slot lists (q6k_grouped_compact,
// kernels/persistent.rs:58-76 grouping): for expert e, list slots
// groups[e*(cap+1)+1 ..], count groups[e*(cap+1)]; X row of slot = slot/x_div.
void gemm_q6_grouped(const Q6Mat& W, int out_rows, const float* X, int x_div, const int* groups,
                     int cap, int max_count, float* out, cudaStream_t s);
void embed_n(const Q6Mat& E, const uint32_t* ids, int n, float* x, cudaStream_t s);
void rmsnorm_n(const float* x, const float* w, float eps, int n, float* out, cudaStream_t s);
void conv_prefill(const float* bcx, const float* conv_w, float* state, int n, float* gated,
                  cudaStream_t s);
// (with start_dev the first position is read from device memory; it must equal `start`)
void qk_prep_n(float* qkv, const float* q_norm, const float* k_norm, const float2* rope,
               int start, int n, int ctx, float eps, __half* kc, __half* vc, cudaStream_t s,
               const int* start_dev = nullptr);
void attn_prefill(const float* qkv, const __half* kc, const __half* vc, int start, int n, int ctx,
                  float* out, cudaStream_t s);
// Batched decode of independent sessions: token j is at position tpos[j] of
// session tsess[j]; per-session caches / conv states lie sstride elements apart.
void qk_prep_batch(float* qkv, const float* q_norm, const float* k_norm, const float2* rope, int n, int ctx,
                   float eps, __half* kc, __half* vc, const int* tpos, const int* tsess, size_t sstride,
                   cudaStream_t s);
// (split over 64-position blocks; `part` holds attn_batch_part_floats(n, ctx) floats)
size_t attn_batch_part_floats(int n, int ctx);
void attn_batch(const float* qkv, const __half* kc, const __half* vc, int n, int ctx, float* out, const int* tpos,
                const int* tsess, size_t sstride, float* part, cudaStream_t s);
void conv_batch(const float* bcx, const float* conv_w, float* state, size_t sstride, const int* tsess, int n,
                float* gated, cudaStream_t s);
// out[i] = argmax of row i of x [n][len].
void argmax_rows(const float* x, int n, int len, int* out, cudaStream_t s);
// Router logits [n][32] of normalised tokens (f32_matmul, kernels.rs:552-574).
void router_logits_n(const float* Wr, const float* xnorm, int n, float* logits, cudaStream_t s);
// Per-expert slot lists: groups[e*(cap+1)] = count, then the slots routed to
// e in slot order. A list longer than cap (a token naming one expert twice)
// is cut at cap and raises GROUP_OVERFLOW in *overflow when given.
constexpr unsigned GROUP_OVERFLOW = 4u;
void expert_groups(const int* sel, int n, int* groups, int cap, cudaStream_t s, unsigned* overflow = nullptr);
void swiglu_n(const float* gate, const float* up, size_t count, float* out, cudaStream_t s);
void combine_n(const float* down, const float* selw, int n, float* x, cudaStream_t s);
void add_n(float* x, const float* y, size_t count, cudaStream_t s);

}  // namespace lfm
