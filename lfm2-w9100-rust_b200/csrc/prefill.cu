// Prompt (n > 1) kernels: the reference's batched graph
// (gpu_lfm/resident_graph.rs:226-551 with n tokens) on B200.
//
// gemm_q6 / gemm_q6_grouped are the exact-arithmetic (FP32 CUDA-core) Q6_K
// GEMMs: a CTA dequantises a 64-row x 256-k weight tile (one super-block per
// row) into shared memory once and reuses it for 64 tokens, the role of the
// reference's q6k_prompt tiles (kernels.rs:1039-1044) and of the grouped
// expert tiles over device-built slot lists (q6k_grouped_compact,
// kernels/persistent.rs:58-76).
#include <math.h>

#include "host_once.h"
#include "kernels.h"

namespace lfm {
namespace {

constexpr int GM = 64, GN = 64, GK = 256;
constexpr int GPAD = 4;  // Xs row padding (floats)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// argmax order: larger value, then smaller index (NaN never wins)
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// GROUPED = false: columns are tokens 0..n-1, X row j, output row j.
// GROUPED = true : blockIdx.z = expert; columns are that expert's slots.
template <bool GROUPED>
__global__ void __launch_bounds__(256) k_gemm_q6(Q6Mat W, int out_rows, const float* X, int n,
                                                 int ldx, int x_div, const int* groups, int cap,
                                                 float* out, int ldo, bool resid) {
  extern __shared__ float smem[];
  float* Ws = smem;                    // [GK][GM]
  float* Xs = smem + GK * GM;          // [GK][GN + GPAD]
  __shared__ int s_slot[GN];
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * GM;
  const int c0 = blockIdx.y * GN;
  int ncols = n;
  int wrow0 = 0;
  if (GROUPED) {
    const int e = blockIdx.z;
    const int* g = groups + (size_t)e * (cap + 1);
    ncols = g[0];
    if (c0 >= ncols) return;
    wrow0 = e * out_rows;
    if (tid < GN) s_slot[tid] = (c0 + tid < ncols) ? g[1 + c0 + tid] : -1;
  } else {
    if (tid < GN) s_slot[tid] = (c0 + tid < ncols) ? c0 + tid : -1;
  }
  __syncthreads();
  const int U = 4 * W.nb;
  const int in = W.nb * QK;
  const int tx = tid & 15, ty = tid >> 4;
  float acc[4][4] = {};
  for (int b = 0; b < W.nb; b++) {
    // dequantise 64 rows x 4 units of block b
    {
      const int r = tid & 63, uu = tid >> 6;  // 4 units
      const int row = r0 + r;
      const int u = 4 * b + uu;
      float w[64];
      if (row < out_rows) {
        const size_t grow = (size_t)wrow0 + row;
        const uint4* qp = W.q + grow * 3 * U + u;
        q6_unit_dequant(qp[0], qp[U], qp[2 * U], W.sc[grow * U + u],
                        __half2float(W.d[grow * W.nb + b]), w);
      } else {
#pragma unroll
        for (int i = 0; i < 64; i++) w[i] = 0.f;
      }
      const int kb = q6_unit_base(u) - 256 * b;  // offset within the block
#pragma unroll
      for (int m = 0; m < 4; m++)
#pragma unroll
        for (int i = 0; i < 16; i++) Ws[(kb + 32 * m + i) * GM + r] = w[m * 16 + i];
    }
    // activations: column c, 64 k per thread
    {
      const int c = tid & 63, kq = tid >> 6;
      const int slot = s_slot[c];
      const float* xrow = slot >= 0 ? X + (size_t)(slot / x_div) * ldx + 256 * b + kq * 64 : nullptr;
#pragma unroll 4
      for (int k = 0; k < 64; k += 4) {
        float4 v = xrow ? *(const float4*)(xrow + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        Xs[(kq * 64 + k + 0) * (GN + GPAD) + c] = v.x;
        Xs[(kq * 64 + k + 1) * (GN + GPAD) + c] = v.y;
        Xs[(kq * 64 + k + 2) * (GN + GPAD) + c] = v.z;
        Xs[(kq * 64 + k + 3) * (GN + GPAD) + c] = v.w;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < GK; k++) {
      const float4 a = *(const float4*)(Ws + k * GM + ty * 4);
      const float4 x = *(const float4*)(Xs + k * (GN + GPAD) + tx * 4);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], xv[j], acc[i][j]);
    }
    __syncthreads();
  }
  (void)in;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int slot = s_slot[tx * 4 + j];
    if (slot < 0) continue;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int row = r0 + ty * 4 + i;
      if (row >= out_rows) continue;
      float* o = out + (size_t)slot * ldo + row;
      if (resid) *o += acc[i][j];
      else *o = acc[i][j];
    }
  }
}

constexpr size_t GEMM_SMEM = (size_t)GK * GM * 4 + (size_t)GK * (GN + GPAD) * 4;

__global__ void k_embed_n(Q6Mat E, const uint32_t* ids, float* x) {
  const int j = blockIdx.x, u = threadIdx.x;
  const int U = 4 * E.nb;
  if (u >= U) return;
  const size_t tok = ids[j];
  const uint4* qp = E.q + tok * 3 * U + u;
  float w[64];
  q6_unit_dequant(qp[0], qp[U], qp[2 * U], E.sc[tok * U + u], __half2float(E.d[tok * E.nb + (u >> 2)]), w);
  float* xo = x + (size_t)j * DIM + q6_unit_base(u);
#pragma unroll
  for (int m = 0; m < 4; m++)
#pragma unroll
    for (int i = 0; i < 16; i++) xo[32 * m + i] = w[m * 16 + i];
}

// RMSNorm of each token row (kernels.rs:576-634; lfm.rs:231-244).
__global__ void __launch_bounds__(256) k_rmsnorm_n(const float* x, const float* w, float eps, float* out) {
  static_assert(DIM == 2 * 4 * 256, "two float4 per thread");
  __shared__ float red[8];
  const float4* xr = (const float4*)(x + (size_t)blockIdx.x * DIM);
  const float4 a = xr[threadIdx.x], b = xr[threadIdx.x + 256];
  float ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, a.w * a.w)));
  ss = fmaf(b.x, b.x, fmaf(b.y, b.y, fmaf(b.z, b.z, fmaf(b.w, b.w, ss))));
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < 8; i++) t += red[i];
  const float inv = 1.0f / sqrtf(t / (float)DIM + eps);
  const float4 wa = __ldg((const float4*)w + threadIdx.x), wb = __ldg((const float4*)w + threadIdx.x + 256);
  float4* o = (float4*)(out + (size_t)blockIdx.x * DIM);
  o[threadIdx.x] = make_float4(a.x * inv * wa.x, a.y * inv * wa.y, a.z * inv * wa.z, a.w * inv * wa.w);
  o[threadIdx.x + 256] = make_float4(b.x * inv * wb.x, b.y * inv * wb.y, b.z * inv * wb.z, b.w * inv * wb.w);
}

// Short conv over n tokens (kernels/resident.rs:33-56: three taps over
// [state0, state1, b*x], the state rolling by one token per step). The taps
// of token j are b*x of tokens j-2, j-1 (or the incoming state) and j, so
// tokens are independent: thread (channel, run of CONV_RUN tokens) slides the
// two older taps along its run, reading b, c and x of each token once (all
// of the run's loads issued before the first product), with the same
// operations per token as the serial form. The new state is written by
// k_conv_state afterwards.
constexpr int CONV_RUN = 8;
__global__ void __launch_bounds__(256) k_conv_prefill(const float* __restrict__ bcx, const float* __restrict__ conv_w,
                                                      const float* __restrict__ state, int n,
                                                      float* __restrict__ gated) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  const int j0 = blockIdx.y * CONV_RUN;
  if (ch >= DIM || j0 >= n) return;
  auto bx_of = [&](int t) {
    const float* r = bcx + (size_t)t * 3 * DIM;
    return r[ch] * r[2 * DIM + ch];
  };
  float b[CONV_RUN], c[CONV_RUN], x[CONV_RUN];
#pragma unroll
  for (int i = 0; i < CONV_RUN; i++) {
    const float* r = bcx + (size_t)min(j0 + i, n - 1) * 3 * DIM;
    b[i] = r[ch];
    c[i] = r[DIM + ch];
    x[i] = r[2 * DIM + ch];
  }
  // taps of token j0 (j0 is a multiple of CONV_RUN: 0 or >= 2)
  float s0 = j0 >= 2 ? bx_of(j0 - 2) : state[2 * ch];
  float s1 = j0 >= 1 ? bx_of(j0 - 1) : state[2 * ch + 1];
  const float w0 = conv_w[3 * ch], w1 = conv_w[3 * ch + 1], w2 = conv_w[3 * ch + 2];
#pragma unroll
  for (int i = 0; i < CONV_RUN; i++) {
    if (j0 + i >= n) break;
    const float bx = b[i] * x[i];
    float conv = 0.f;
    conv += s0 * w0;
    conv += s1 * w1;
    conv += bx * w2;
    gated[(size_t)(j0 + i) * DIM + ch] = c[i] * conv;
    s0 = s1;
    s1 = bx;
  }
}

// Conv state after n tokens: (b*x of tokens n-2, n-1), or (old state1, b*x of
// token 0) when n == 1.
__global__ void k_conv_state(const float* bcx, float* state, int n) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= DIM) return;
  auto bx_of = [&](int t) {
    const float* r = bcx + (size_t)t * 3 * DIM;
    return r[ch] * r[2 * DIM + ch];
  };
  const float s0 = n >= 2 ? bx_of(n - 2) : state[2 * ch + 1];
  const float s1 = bx_of(n - 1);
  state[2 * ch] = s0;
  state[2 * ch + 1] = s1;
}

// Head RMSNorm + NEOX RoPE of q (32 heads) and k (8 heads) in place, then the
// fp16 K/V cache write at positions start..start+n-1 (lfm.rs:368-393). With a
// token map (batched decode of independent sessions), token j is at position
// tpos[j] of session tsess[j], whose caches start sstride elements apart.
__global__ void k_qk_prep_n(float* qkv, const float* q_norm, const float* k_norm, const float2* rope,
                            int start, int ctx, float eps, __half* kc, __half* vc, const int* tpos,
                            const int* tsess, size_t sstride, const int* start_dev) {
  const int j = blockIdx.x;
  const int hh = blockIdx.y * 8 + (threadIdx.x >> 5);  // 0..47
  const int lane = threadIdx.x & 31;
  const int pos = tpos ? tpos[j] : (start_dev ? *start_dev : start) + j;
  if (tsess) {
    kc += (size_t)tsess[j] * sstride;
    vc += (size_t)tsess[j] * sstride;
  }
  float* row = qkv + (size_t)j * (DIM + 2 * KV_HEADS * HEAD_DIM);
  if (hh < HEADS + KV_HEADS) {
    const bool isq = hh < HEADS;
    float* v = isq ? row + hh * HEAD_DIM : row + DIM + (hh - HEADS) * HEAD_DIM;
    const float* nw = isq ? q_norm : k_norm;
    float a0 = v[lane], a1 = v[lane + 32];
    const float ss = warp_sum(a0 * a0 + a1 * a1);
    const float inv = 1.0f / sqrtf(ss / (float)HEAD_DIM + eps);
    a0 *= inv * nw[lane];
    a1 *= inv * nw[lane + 32];
    const float2 cs = rope[(size_t)pos * 32 + lane];
    const float r0 = a0 * cs.x - a1 * cs.y, r1 = a0 * cs.y + a1 * cs.x;
    v[lane] = r0;
    v[lane + 32] = r1;
    if (!isq) {
      const int kh = hh - HEADS;
      const size_t off = ((size_t)kh * ctx + pos) * HEAD_DIM;
      kc[off + lane] = __float2half_rn(r0);
      kc[off + lane + 32] = __float2half_rn(r1);
    }
  } else {
    const int kh = hh - HEADS - KV_HEADS;
    const float* v = row + DIM + KV_HEADS * HEAD_DIM + kh * HEAD_DIM;
    const size_t off = ((size_t)kh * ctx + pos) * HEAD_DIM;
    vc[off + lane] = __float2half_rn(v[lane]);
    vc[off + lane + 32] = __float2half_rn(v[lane + 32]);
  }
}

// Causal GQA attention for n new tokens over the fp16 cache (lfm.rs:395-437):
// one warp per (token, head), online softmax over 32-position chunks.
__global__ void __launch_bounds__(256) k_attn_prefill(const float* qkv, const __half* kc, const __half* vc,
                                                      int start, int n, int ctx, float* out, const int* tpos,
                                                      const int* tsess, size_t sstride) {
  __shared__ float sq[8][HEAD_DIM];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + warp;
  if (gw >= n * HEADS) return;
  const int j = gw / HEADS, h = gw % HEADS;
  const int kh = h / (HEADS / KV_HEADS);
  const int p = tpos ? tpos[j] : start + j;
  if (tsess) {
    kc += (size_t)tsess[j] * sstride;
    vc += (size_t)tsess[j] * sstride;
  }
  const float* q = qkv + (size_t)j * (DIM + 2 * KV_HEADS * HEAD_DIM) + h * HEAD_DIM;
  sq[warp][lane] = q[lane];
  sq[warp][lane + 32] = q[lane + 32];
  __syncwarp();
  const __half* kb = kc + (size_t)kh * ctx * HEAD_DIM;
  const __half* vb = vc + (size_t)kh * ctx * HEAD_DIM;
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
  for (int t0 = 0; t0 <= p; t0 += 32) {
    const int t = t0 + lane;
    float s = -INFINITY;
    if (t <= p) {
      const uint4* kp = (const uint4*)(kb + (size_t)t * HEAD_DIM);
      float acc = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; c8++) {
        const uint4 v = kp[c8];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const float2 f = __half22float2(*(const __half2*)&w[jj]);
          acc = fmaf(f.x, sq[warp][c8 * 8 + 2 * jj], acc);
          acc = fmaf(f.y, sq[warp][c8 * 8 + 2 * jj + 1], acc);
        }
      }
      s = acc * 0.125f;
    }
    const float cm = warp_max(s);
    const float nm = fmaxf(m, cm);
    const float scale = expf(m - nm);
    const float pv = t <= p ? expf(s - nm) : 0.f;
    l = l * scale + warp_sum(pv);
    o0 *= scale;
    o1 *= scale;
    const int cnt = min(32, p - t0 + 1);
    for (int i = 0; i < cnt; i++) {
      const float pi = __shfl_sync(0xffffffffu, pv, i);
      const __half* vr = vb + (size_t)(t0 + i) * HEAD_DIM;
      o0 = fmaf(pi, __half2float(vr[lane]), o0);
      o1 = fmaf(pi, __half2float(vr[lane + 32]), o1);
    }
    m = nm;
  }
  float* o = out + (size_t)j * DIM + h * HEAD_DIM;
  o[lane] = o0 / l;
  o[lane + 32] = o1 / l;
}

// Decode attention of one token per session (batched decode; lfm.rs:395-437
// for one query): block (kv head, split, token) scores the 64 cached
// positions of its split for the 4 query heads of the KV head (one warp each,
// two positions per lane) and leaves a partial (max, sum, weighted V) that
// k_attn_batch_merge combines over the token's splits in order. q is already
// head-normalised and rotated (k_qk_prep_n); the split holding the token's
// own position reads the K/V row that k_qk_prep_n wrote.
constexpr int ABS = 64;  // positions per split
__global__ void __launch_bounds__(128) k_attn_batch(const float* qkv, const __half* kc, const __half* vc, int ctx,
                                                    const int* tpos, const int* tsess, size_t sstride, float* part,
                                                    int nsplit_max) {
  constexpr int KP = HEAD_DIM + 8;
  __shared__ float sq[4][HEAD_DIM];
  __shared__ __align__(16) __half sk[ABS][KP];
  __shared__ __align__(16) __half sv[ABS][HEAD_DIM];
  const int kh = blockIdx.x, split = blockIdx.y, j = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = tpos[j];
  const int t0 = split * ABS;
  if (t0 > pos) return;
  const size_t sbase = (size_t)tsess[j] * sstride;
  const int h = kh * (HEADS / KV_HEADS) + warp;
  const float* q = qkv + (size_t)j * (DIM + 2 * KV_HEADS * HEAD_DIM) + h * HEAD_DIM;
  sq[warp][lane] = q[lane];
  sq[warp][lane + 32] = q[lane + 32];
  const int cnt = min(ABS, pos + 1 - t0);
  {
    const uint4* kg = (const uint4*)(kc + sbase + ((size_t)kh * ctx + t0) * HEAD_DIM);
    const uint4* vg = (const uint4*)(vc + sbase + ((size_t)kh * ctx + t0) * HEAD_DIM);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int idx = threadIdx.x + i * 128;  // 0..511 = 64 rows x 8 pieces
      const int r = idx >> 3, c = idx & 7;
      if (r < cnt) {
        *(uint4*)&sk[r][c * 8] = kg[idx];
        *(uint4*)&sv[r][c * 8] = vg[idx];
      }
    }
  }
  __syncthreads();
  float sc[2];
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    const int r = lane + 32 * hf;
    sc[hf] = -INFINITY;
    if (r < cnt) {
      float acc = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; c8++) {
        const uint4 v = *(const uint4*)&sk[r][c8 * 8];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const float2 f = __half22float2(*(const __half2*)&w[jj]);
          acc = fmaf(f.x, sq[warp][c8 * 8 + 2 * jj], acc);
          acc = fmaf(f.y, sq[warp][c8 * 8 + 2 * jj + 1], acc);
        }
      }
      sc[hf] = acc * 0.125f;
    }
  }
  const float m = warp_max(fmaxf(sc[0], sc[1]));
  const float p0 = lane < cnt ? expf(sc[0] - m) : 0.f;
  const float p1 = lane + 32 < cnt ? expf(sc[1] - m) : 0.f;
  const float l = warp_sum(p0 + p1);
  float o0 = 0.f, o1 = 0.f;
  for (int t = 0; t < cnt; t++) {
    const float pt = __shfl_sync(0xffffffffu, t < 32 ? p0 : p1, t & 31);
    o0 = fmaf(pt, __half2float(sv[t][lane]), o0);
    o1 = fmaf(pt, __half2float(sv[t][lane + 32]), o1);
  }
  float* pp = part + ((((size_t)j * KV_HEADS + kh) * nsplit_max + split) * 4 + warp) * (HEAD_DIM + 2);
  pp[lane] = o0;
  pp[lane + 32] = o1;
  if (lane == 0) {
    pp[HEAD_DIM] = m;
    pp[HEAD_DIM + 1] = l;
  }
}

// out[j][h*64 + d] = sum_s exp(m_s - M) o_s[d] / sum_s exp(m_s - M) l_s over
// token j's splits in order; block per token, warp per query head.
__global__ void __launch_bounds__(1024) k_attn_batch_merge(const float* part, const int* tpos, int nsplit_max,
                                                           float* out) {
  const int j = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kh = h / (HEADS / KV_HEADS), w = h % (HEADS / KV_HEADS);
  const int nact = tpos[j] / ABS + 1;
  const float* pb = part + (((size_t)j * KV_HEADS + kh) * nsplit_max * 4 + w) * (HEAD_DIM + 2);
  float M = -INFINITY;
  for (int s = 0; s < nact; s++) M = fmaxf(M, pb[(size_t)s * 4 * (HEAD_DIM + 2) + HEAD_DIM]);
  float L = 0.f, o0 = 0.f, o1 = 0.f;
  for (int s = 0; s < nact; s++) {
    const float* ps = pb + (size_t)s * 4 * (HEAD_DIM + 2);
    const float f = expf(ps[HEAD_DIM] - M);
    L = fmaf(ps[HEAD_DIM + 1], f, L);
    o0 = fmaf(ps[lane], f, o0);
    o1 = fmaf(ps[lane + 32], f, o1);
  }
  float* o = out + (size_t)j * DIM + h * HEAD_DIM;
  o[lane] = o0 / L;
  o[lane + 32] = o1 / L;
}

// Short conv of one token per session (batched decode): token j advances the
// conv state of its session tsess[j] by one step (kernels/resident.rs:33-56).
__global__ void k_conv_batch(const float* bcx, const float* conv_w, float* state, size_t sstride, const int* tsess,
                             int n, float* gated) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  const int j = blockIdx.y;
  if (ch >= DIM || j >= n) return;
  float* st = state + (size_t)tsess[j] * sstride;
  const float* r = bcx + (size_t)j * 3 * DIM;
  const float bx = r[ch] * r[2 * DIM + ch];
  const float s0 = st[2 * ch], s1 = st[2 * ch + 1];
  float conv = 0.f;
  conv += s0 * conv_w[3 * ch];
  conv += s1 * conv_w[3 * ch + 1];
  conv += bx * conv_w[3 * ch + 2];
  gated[(size_t)j * DIM + ch] = r[DIM + ch] * conv;
  st[2 * ch] = s1;
  st[2 * ch + 1] = bx;
}

// Row-wise argmax of [n][len] logits (the reference's GPU argmax semantics:
// largest value, first index on ties, NaN never selected; main.rs:287-317).
__global__ void __launch_bounds__(1024) k_argmax_rows(const float* x, int len, int* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* r = x + (size_t)blockIdx.x * len;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < len; i += blockDim.x)
    if (am_better(r[i], i, bv, bi)) {
      bv = r[i];
      bi = i;
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    bv = threadIdx.x < blockDim.x / 32 ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < blockDim.x / 32 ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

// Router logits for n normalised tokens (f32_matmul, kernels.rs:552-574),
// then route_n picks the top 4. A block of 4 warps takes 32 tokens; lane
// (p, h) of warp w computes experts p and p + 16 for tokens 8w + 4h .. +3,
// each logit one fmaf chain in K order (eight chains per lane). 64-wide K
// chunks of the 32 router rows and the 32 token rows are staged in shared
// memory by cp.async through a ring of RL_STAGES buffers (a chunk's
// multiply, ~700 cycles, is shorter than a load's latency, so three chunks
// are in flight); per K step a lane reads two router float4 (16 distinct rows
// a warp, two wavefronts) and four token float4 (two distinct rows, one
// wavefront) for 32 FMAs.
constexpr int RL_KC = 64, RL_TOK = 32, RL_RS = RL_KC + 4;  // RL_RS: row stride, conflict-free float4 reads
constexpr int RL_STAGES = 4;
constexpr int RL_STAGE_FLOATS = (N_EXPERT + RL_TOK) * RL_RS;
constexpr int RL_SMEM = RL_STAGES * RL_STAGE_FLOATS * 4;  // 69632 bytes
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__global__ void __launch_bounds__(128) k_router_logits_n(const float* Wr, const float* xn, int n, float* logits) {
  static_assert(N_EXPERT == 32 && DIM % RL_KC == 0 && DIM / RL_KC >= RL_STAGES, "router tiling");
  extern __shared__ __align__(16) float rl_smem[];  // stage b: router rows [32][RL_RS], then token rows [32][RL_RS]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int j0 = blockIdx.x * RL_TOK;
  const int p = lane & 15, h = lane >> 4;
  const int tr = warp * 8 + h * 4;  // this lane's first token row in the block
  constexpr int NC = DIM / RL_KC;
  // chunk c into its stage: 512 float4 of router rows and 512 of token rows,
  // four of each per thread; one commit group per chunk (empty past the end,
  // so that the group count stays uniform)
  auto fetch = [&](int c) {
    if (c < NC) {
      float* ws = rl_smem + (c % RL_STAGES) * RL_STAGE_FLOATS;
      float* xs = ws + N_EXPERT * RL_RS;
      const int k0 = c * RL_KC;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int f = t + 128 * i, r = f >> 4, c4 = f & 15;
        cp_async16(ws + r * RL_RS + 4 * c4, Wr + (size_t)r * DIM + k0 + 4 * c4);
        cp_async16(xs + r * RL_RS + 4 * c4, xn + (size_t)min(j0 + r, n - 1) * DIM + k0 + 4 * c4);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; i++) acc[i][0] = acc[i][1] = 0.f;
#pragma unroll
  for (int c = 0; c < RL_STAGES - 1; c++) fetch(c);
  for (int c = 0; c < NC; c++) {
    // the stage refilled here was read in iteration c - 1, before its
    // closing barrier
    fetch(c + RL_STAGES - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(RL_STAGES - 1) : "memory");  // chunk c has landed
    __syncthreads();
    const float* ws = rl_smem + (c % RL_STAGES) * RL_STAGE_FLOATS;
    const float* xs = ws + N_EXPERT * RL_RS;
#pragma unroll 4
    for (int k4 = 0; k4 < RL_KC / 4; k4++) {
      const float4 wa = *(const float4*)&ws[p * RL_RS + 4 * k4];
      const float4 wb = *(const float4*)&ws[(p + 16) * RL_RS + 4 * k4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 xv = *(const float4*)&xs[(tr + i) * RL_RS + 4 * k4];
        acc[i][0] = fmaf(wa.x, xv.x, acc[i][0]);
        acc[i][0] = fmaf(wa.y, xv.y, acc[i][0]);
        acc[i][0] = fmaf(wa.z, xv.z, acc[i][0]);
        acc[i][0] = fmaf(wa.w, xv.w, acc[i][0]);
        acc[i][1] = fmaf(wb.x, xv.x, acc[i][1]);
        acc[i][1] = fmaf(wb.y, xv.y, acc[i][1]);
        acc[i][1] = fmaf(wb.z, xv.z, acc[i][1]);
        acc[i][1] = fmaf(wb.w, xv.w, acc[i][1]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int j = j0 + tr + i;
    if (j < n) {
      logits[(size_t)j * N_EXPERT + p] = acc[i][0];
      logits[(size_t)j * N_EXPERT + p + 16] = acc[i][1];
    }
  }
}

// Router logits for few tokens (batched decode, short prompts): block
// (group of RT_TOK tokens, group of 8 experts); the group's x rows are staged
// in shared memory and warp w computes expert 8 * blockIdx.y + w for all of
// them, each router row read once per block. Per (token, expert) the sum is
// lane-strided over K (lane l takes float4 l, l + 32, ...) and closed by a
// warp butterfly.
constexpr int RT_TOK = 4;
__global__ void __launch_bounds__(256) k_router_logits_tok(const float* Wr, const float* xn, int n, float* logits) {
  __shared__ float4 xs[RT_TOK][DIM / 4];
  const int j0 = blockIdx.x * RT_TOK, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.y * 8 + warp;
#pragma unroll
  for (int i = 0; i < RT_TOK * DIM / 4 / 256; i++) {
    const int f = threadIdx.x + 256 * i, t = f / (DIM / 4), c = f % (DIM / 4);
    xs[t][c] = *((const float4*)(xn + (size_t)min(j0 + t, n - 1) * DIM) + c);
  }
  __syncthreads();
  const float4* w = (const float4*)(Wr + (size_t)e * DIM);
  float a[RT_TOK];
#pragma unroll
  for (int t = 0; t < RT_TOK; t++) a[t] = 0.f;
#pragma unroll 4
  for (int i = lane; i < DIM / 4; i += 32) {
    const float4 v = __ldg(w + i);
#pragma unroll
    for (int t = 0; t < RT_TOK; t++) {
      const float4 xv = xs[t][i];
      a[t] = fmaf(v.x, xv.x, a[t]);
      a[t] = fmaf(v.y, xv.y, a[t]);
      a[t] = fmaf(v.z, xv.z, a[t]);
      a[t] = fmaf(v.w, xv.w, a[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < RT_TOK; t++) {
    const float r = warp_sum(a[t]);
    if (lane == 0 && j0 + t < n) logits[(size_t)(j0 + t) * N_EXPERT + e] = r;
  }
}

// Stable per-expert slot lists (kernels/persistent.rs:58-76): block e scans
// the slots (token*4 + rank) in order and appends those routed to e. Each
// thread takes GROUP_SPT consecutive slots a pass (16384 slots, 4096 tokens,
// per pass), and a block-wide exclusive scan of the threads' hit counts gives
// each hit its place, so every list is in slot order. A list never grows past
// `cap` entries: a hit beyond it (only possible when a token names one expert
// twice) is dropped, the count stops at cap and `overflow` (if given) gets
// GROUP_OVERFLOW.
constexpr int GROUP_SPT = 16;
__global__ void __launch_bounds__(1024) k_expert_groups(const int* sel, int n, int* groups, int cap,
                                                        unsigned* overflow) {
  __shared__ int wpre[32];
  __shared__ int wtot;
  const int e = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  int* g = groups + (size_t)e * (cap + 1);
  int count = 0;
  const int total = n * N_USED;
  const bool vec = ((uintptr_t)sel & 15) == 0;
  for (int s0 = 0; s0 < total; s0 += 1024 * GROUP_SPT) {
    const int base = s0 + t * GROUP_SPT;
    unsigned m = 0;  // bit i: slot base + i is routed to e
    if (vec && base + GROUP_SPT <= total) {
#pragma unroll
      for (int q = 0; q < GROUP_SPT / 4; q++) {
        const int4 v = *((const int4*)(sel + base) + q);
        m |= (unsigned)(v.x == e) << (4 * q) | (unsigned)(v.y == e) << (4 * q + 1) |
             (unsigned)(v.z == e) << (4 * q + 2) | (unsigned)(v.w == e) << (4 * q + 3);
      }
    } else {
      for (int i = 0; i < GROUP_SPT; i++)
        if (base + i < total && sel[base + i] == e) m |= 1u << i;
    }
    const int c = __popc(m);
    int inc = c;  // inclusive scan over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    if (lane == 31) wpre[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const int own = wpre[lane];
      int winc = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, winc, o);
        if (lane >= o) winc += v;
      }
      wpre[lane] = winc - own;
      if (lane == 31) wtot = winc;
    }
    __syncthreads();
    int pos = count + wpre[warp] + inc - c;
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1;
      if (pos < cap) g[1 + pos] = base + i;
      pos++;
    }
    count += wtot;
    __syncthreads();  // wpre / wtot are rewritten by the next pass
  }
  if (t == 0) {
    g[0] = min(count, cap);
    if (count > cap && overflow) atomicOr(overflow, GROUP_OVERFLOW);
  }
}

__global__ void k_swiglu_n(const float* gate, const float* up, size_t count, float* out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) {
    const float g = gate[i];
    out[i] = g / (1.0f + expf(-g)) * up[i];
  }
}

// x[j] += sum_r w[j,r] * down[j*4 + r] in rank order (kernels/resident.rs:101-117).
__global__ void k_combine_n(const float* down, const float* selw, int n, float* x) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)n * DIM) return;
  const size_t j = i / DIM, k = i % DIM;
  float a = 0.f;
#pragma unroll
  for (int r = 0; r < N_USED; r++) a += down[(j * N_USED + r) * DIM + k] * selw[j * N_USED + r];
  x[i] += a;
}

__global__ void k_add_n(float* x, const float* y, size_t count) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) x[i] += y[i];
}

}  // namespace

void gemm_q6_ld(const Q6Mat& W, const float* X, int n, float* out, int ldo, bool resid, cudaStream_t s) {
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu, [] {
    cudaFuncSetAttribute(k_gemm_q6<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM);
    cudaFuncSetAttribute(k_gemm_q6<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM);
  });
  dim3 grid((W.rows + GM - 1) / GM, (n + GN - 1) / GN);
  k_gemm_q6<false><<<grid, 256, GEMM_SMEM, s>>>(W, W.rows, X, n, W.nb * QK, 1, nullptr, 0, out, ldo, resid);
}

void gemm_q6(const Q6Mat& W, const float* X, int n, float* out, bool resid, cudaStream_t s) {
  gemm_q6_ld(W, X, n, out, W.rows, resid, s);
}

void gemm_q6_grouped(const Q6Mat& W, int out_rows, const float* X, int x_div, const int* groups, int cap,
                     int max_count, float* out, cudaStream_t s) {
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu,
                  [] { cudaFuncSetAttribute(k_gemm_q6<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM); });
  dim3 grid((out_rows + GM - 1) / GM, (max_count + GN - 1) / GN, N_EXPERT);
  k_gemm_q6<true><<<grid, 256, GEMM_SMEM, s>>>(W, out_rows, X, 0, W.nb * QK, x_div, groups, cap, out,
                                               out_rows, false);
}

void embed_n(const Q6Mat& E, const uint32_t* ids, int n, float* x, cudaStream_t s) {
  k_embed_n<<<n, 32, 0, s>>>(E, ids, x);
}

void rmsnorm_n(const float* x, const float* w, float eps, int n, float* out, cudaStream_t s) {
  k_rmsnorm_n<<<n, 256, 0, s>>>(x, w, eps, out);
}

void conv_prefill(const float* bcx, const float* conv_w, float* state, int n, float* gated, cudaStream_t s) {
  k_conv_prefill<<<dim3(DIM / 256, (n + CONV_RUN - 1) / CONV_RUN), 256, 0, s>>>(bcx, conv_w, state, n, gated);
  k_conv_state<<<DIM / 256, 256, 0, s>>>(bcx, state, n);
}

void qk_prep_n(float* qkv, const float* q_norm, const float* k_norm, const float2* rope, int start, int n,
               int ctx, float eps, __half* kc, __half* vc, cudaStream_t s, const int* start_dev) {
  k_qk_prep_n<<<dim3(n, 6), 256, 0, s>>>(qkv, q_norm, k_norm, rope, start, ctx, eps, kc, vc, nullptr, nullptr, 0,
                                         start_dev);
}

void attn_prefill(const float* qkv, const __half* kc, const __half* vc, int start, int n, int ctx, float* out,
                  cudaStream_t s) {
  k_attn_prefill<<<(n * HEADS + 7) / 8, 256, 0, s>>>(qkv, kc, vc, start, n, ctx, out, nullptr, nullptr, 0);
}

void qk_prep_batch(float* qkv, const float* q_norm, const float* k_norm, const float2* rope, int n, int ctx,
                   float eps, __half* kc, __half* vc, const int* tpos, const int* tsess, size_t sstride,
                   cudaStream_t s) {
  k_qk_prep_n<<<dim3(n, 6), 256, 0, s>>>(qkv, q_norm, k_norm, rope, 0, ctx, eps, kc, vc, tpos, tsess, sstride,
                                         nullptr);
}

size_t attn_batch_part_floats(int n, int ctx) {
  return (size_t)n * KV_HEADS * ((ctx + ABS - 1) / ABS) * 4 * (HEAD_DIM + 2);
}

void attn_batch(const float* qkv, const __half* kc, const __half* vc, int n, int ctx, float* out, const int* tpos,
                const int* tsess, size_t sstride, float* part, cudaStream_t s) {
  const int nsplit = (ctx + ABS - 1) / ABS;
  k_attn_batch<<<dim3(KV_HEADS, nsplit, n), 128, 0, s>>>(qkv, kc, vc, ctx, tpos, tsess, sstride, part, nsplit);
  k_attn_batch_merge<<<n, HEADS * 32, 0, s>>>(part, tpos, nsplit, out);
}

void conv_batch(const float* bcx, const float* conv_w, float* state, size_t sstride, const int* tsess, int n,
                float* gated, cudaStream_t s) {
  k_conv_batch<<<dim3(DIM / 256, n), 256, 0, s>>>(bcx, conv_w, state, sstride, tsess, n, gated);
}

void argmax_rows(const float* x, int n, int len, int* out, cudaStream_t s) {
  k_argmax_rows<<<n, 1024, 0, s>>>(x, len, out);
}

void router_logits_n(const float* Wr, const float* xnorm, int n, float* logits, cudaStream_t s) {
  static_assert(N_EXPERT == 32, "router tiling assumes 32 experts");
  if (n < 256) k_router_logits_tok<<<dim3((n + RT_TOK - 1) / RT_TOK, N_EXPERT / 8), 256, 0, s>>>(Wr, xnorm, n, logits);
  else {
    static unsigned long long done = 0;
    static std::mutex mu;
    once_per_device(done, mu,
                    [] { cudaFuncSetAttribute(k_router_logits_n, cudaFuncAttributeMaxDynamicSharedMemorySize, RL_SMEM); });
    k_router_logits_n<<<(n + RL_TOK - 1) / RL_TOK, 128, RL_SMEM, s>>>(Wr, xnorm, n, logits);
  }
}

void expert_groups(const int* sel, int n, int* groups, int cap, cudaStream_t s, unsigned* overflow) {
  k_expert_groups<<<N_EXPERT, 1024, 0, s>>>(sel, n, groups, cap, overflow);
}

void swiglu_n(const float* gate, const float* up, size_t count, float* out, cudaStream_t s) {
  k_swiglu_n<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(gate, up, count, out);
}

void combine_n(const float* down, const float* selw, int n, float* x, cudaStream_t s) {
  const size_t count = (size_t)n * DIM;
  k_combine_n<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(down, selw, n, x);
}

void add_n(float* x, const float* y, size_t count, cudaStream_t s) {
  k_add_n<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(x, y, count);
}

}  // namespace lfm
