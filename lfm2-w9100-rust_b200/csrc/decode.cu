// Batch-1 decode kernels for sm_100a.
//
// Decode is HBM-bound weight streaming (~1.38 GB of Q6_K per token), so every
// matrix product here is a warp-per-row matvec over the device layout of
// q6k.cuh: one lane owns one 64-weight unit of the row, reads it with three
// coalesced 16-byte streaming loads (L1 no-allocate), and keeps the 64
// matching activations in registers for the whole kernel, so no shared-memory
// traffic is spent on x. A warp works on RPW rows at once to keep enough bytes
// in flight. The neighbouring element-wise work of the reference graph
// (resident_graph.rs:240-546) is fused into prologues (RMSNorm) and epilogues
// (residual, short-conv, SwiGLU, expert combine, argmax), which removes the
// reference's separate norm/residual/swiglu/combine/argmax dispatches.
//
// All kernels call griddepcontrol.wait before touching activations, so they
// can be launched with programmatic dependent launch inside the decode graph.
#include <math.h>

#include "kernels.h"

namespace lfm {

namespace {

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_half(const __half* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

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

// Deterministic block sum (fixed warp order).
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

// RMS normalisation factor of x[0..DIM) (kernels.rs:576-634; lfm.rs:231-244).
__device__ float rms_inv(const float* x, float eps, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < DIM; i += blockDim.x) {
    float v = x[i];
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  return 1.0f / sqrtf(ss / (float)DIM + eps);
}

// The 64 activations of unit u (x-register order), optionally normalised.
__device__ __forceinline__ void load_xr(const float* x, const float* norm, float inv, int u,
                                        float* xr) {
  if (u < 0) return;
  const int base = q6_unit_base(u);
#pragma unroll
  for (int m = 0; m < 4; m++)
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const float4 v = *(const float4*)(x + base + 32 * m + 4 * t);
      if (norm) {
        const float4 g = *(const float4*)(norm + base + 32 * m + 4 * t);
        xr[m * 16 + 4 * t + 0] = v.x * inv * g.x;
        xr[m * 16 + 4 * t + 1] = v.y * inv * g.y;
        xr[m * 16 + 4 * t + 2] = v.z * inv * g.z;
        xr[m * 16 + 4 * t + 3] = v.w * inv * g.w;
      } else {
        xr[m * 16 + 4 * t + 0] = v.x;
        xr[m * 16 + 4 * t + 1] = v.y;
        xr[m * 16 + 4 * t + 2] = v.z;
        xr[m * 16 + 4 * t + 3] = v.w;
      }
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Candidate (v, i) beats (bv, bi): larger value, ties to the lower index,
// NaN never wins (kernels/persistent.rs:12-53, main.rs:112-141).
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

enum MvMode { MV_PLAIN, MV_RESID, MV_CONV, MV_SWIGLU, MV_XSWIGLU, MV_XDOWN, MV_LMHEAD, MV_DOWN_SLICED };

struct MvParams {
  Q6Mat W, W2;
  XSrc xs;
  float* y;
  float* resid;
  const float* conv_w;
  float* state;
  const int* sel;
  const float* selw;
  int ff;
  float2* partials;
  unsigned* counter;
  int* token;
  int ntasks;
  int orows;  // MV_XDOWN: output rows per expert
};

constexpr int WPB = 4;  // warps per CTA

template <int MODE, int RPW, int NS>
__global__ void __launch_bounds__(WPB * 32) k_mv(MvParams p) {
  constexpr bool TWO = MODE == MV_SWIGLU || MODE == MV_XSWIGLU;
  constexpr int RG = WPB / NS;  // row groups per CTA iteration
  __shared__ float red[32];
  __shared__ float spart[WPB][RPW];
  __shared__ float s_bv[WPB];
  __shared__ int s_bi[WPB];
  __shared__ bool s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = warp % NS, rg = warp / NS;
  const int U = 4 * p.W.nb;
  const int S = U / NS;
  const int u = lane < S ? slice * S + lane : -1;
  const int slot = MODE == MV_XDOWN ? (int)blockIdx.y : 0;

  pdl_trigger();
  pdl_wait();

  float xr[64];
  {
    const float* x = p.xs.x;
    if (MODE == MV_XDOWN) x += (size_t)slot * p.ff;
    float inv = 1.f;
    if (p.xs.norm) inv = rms_inv(x, p.xs.eps, red);
    load_xr(x, p.xs.norm, inv, u, xr);
  }
  int ebase = 0;
  if (MODE == MV_XDOWN) ebase = p.sel[slot] * p.orows;

  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int ngroups = (p.ntasks + RG - 1) / RG;
  for (int g = blockIdx.x; g < ngroups; g += gridDim.x) {
    const int task = g * RG + rg;
    const bool valid = task < p.ntasks;
    int rows[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) {
      int row = -1;
      if (valid) {
        if (MODE == MV_PLAIN || MODE == MV_RESID || MODE == MV_LMHEAD || MODE == MV_DOWN_SLICED) {
          row = task * RPW + r;
          if (row >= p.W.rows) row = -1;
        } else if (MODE == MV_CONV) {
          row = task + r * DIM;  // b, c, x rows of channel `task`
        } else if (MODE == MV_SWIGLU) {
          row = task * (RPW / 2) + r / 2;
        } else if (MODE == MV_XSWIGLU) {
          const int t = task * (RPW / 2) + r / 2;  // (slot, i) pair index
          const int s = t / p.ff, i = t - s * p.ff;
          row = p.sel[s] * p.ff + i;
        } else if (MODE == MV_XDOWN) {
          row = task * RPW + r;
          row = row < p.orows ? ebase + row : -1;
        }
      }
      rows[r] = row;
    }
    uint4 A[RPW], B[RPW], Q[RPW];
    uint32_t SC[RPW];
    float D[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++) {
      const Q6Mat& M = (TWO && (r & 1)) ? p.W2 : p.W;
      if (u >= 0 && rows[r] >= 0) {
        const uint4* qp = M.q + (size_t)rows[r] * 3 * U + u;
        A[r] = ld_stream(qp);
        B[r] = ld_stream(qp + U);
        Q[r] = ld_stream(qp + 2 * U);
        SC[r] = ld_stream32(M.sc + (size_t)rows[r] * U + u);
        D[r] = ld_half(M.d + (size_t)rows[r] * M.nb + (u >> 2));
      }
    }
    float acc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++)
      acc[r] = (u >= 0 && rows[r] >= 0) ? q6_unit_dot(A[r], B[r], Q[r], SC[r], D[r], xr) : 0.f;
#pragma unroll
    for (int r = 0; r < RPW; r++) acc[r] = warp_sum(acc[r]);
    if (NS > 1) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < RPW; r++) spart[warp][r] = acc[r];
      __syncthreads();
      if (slice == 0)
#pragma unroll
        for (int r = 0; r < RPW; r++) {
          float t = 0.f;
          for (int s = 0; s < NS; s++) t += spart[rg * NS + s][r];
          acc[r] = t;
        }
      __syncthreads();
    }
    if (slice != 0 || lane != 0 || !valid) continue;
    // ------------------------------------------------------------ epilogue
    if (MODE == MV_PLAIN) {
#pragma unroll
      for (int r = 0; r < RPW; r++)
        if (rows[r] >= 0) p.y[rows[r]] = acc[r];
    } else if (MODE == MV_RESID || MODE == MV_DOWN_SLICED) {
#pragma unroll
      for (int r = 0; r < RPW; r++)
        if (rows[r] >= 0) p.y[rows[r]] += acc[r];
    } else if (MODE == MV_LMHEAD) {
#pragma unroll
      for (int r = 0; r < RPW; r++)
        if (rows[r] >= 0) {
          p.y[rows[r]] = acc[r];
          if (am_better(acc[r], rows[r], bv, bi)) {
            bv = acc[r];
            bi = rows[r];
          }
        }
    } else if (MODE == MV_CONV) {
      // kernels/resident.rs:33-56; lfm.rs:464-520 for one token.
      const int ch = task;
      const float b = acc[0], c = acc[1], xx = acc[2];
      const float bx = b * xx;
      const float s0 = p.state[2 * ch], s1 = p.state[2 * ch + 1];
      float conv = 0.f;
      conv += s0 * p.conv_w[3 * ch + 0];
      conv += s1 * p.conv_w[3 * ch + 1];
      conv += bx * p.conv_w[3 * ch + 2];
      p.y[ch] = c * conv;
      p.state[2 * ch] = s1;
      p.state[2 * ch + 1] = bx;
    } else if (MODE == MV_SWIGLU || MODE == MV_XSWIGLU) {
#pragma unroll
      for (int r = 0; r < RPW; r += 2) {
        const int t = task * (RPW / 2) + r / 2;
        if (rows[r] >= 0) p.y[t] = silu_mul(acc[r], acc[r + 1]);
      }
    } else if (MODE == MV_XDOWN) {
#pragma unroll
      for (int r = 0; r < RPW; r++)
        if (rows[r] >= 0) p.y[(size_t)slot * p.orows + rows[r] - ebase] = acc[r];
    }
  }

  if (MODE == MV_LMHEAD || (MODE == MV_XDOWN && p.resid != nullptr)) {
    if (MODE == MV_LMHEAD) {
      // warp 0..WPB-1 lane 0 hold their best; reduce in the CTA.
      if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        float cv = s_bv[0];
        int ci = s_bi[0];
        for (int w = 1; w < WPB; w++)
          if (am_better(s_bv[w], s_bi[w], cv, ci)) {
            cv = s_bv[w];
            ci = s_bi[w];
          }
        p.partials[blockIdx.x] = make_float2(cv, __int_as_float(ci));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned total = gridDim.x * gridDim.y;
      s_last = atomicAdd(p.counter, 1u) == total - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (MODE == MV_XDOWN) {
      // Rank-ordered combine (kernels/resident.rs:101-117; lfm.rs:645-668).
      for (int k = threadIdx.x; k < DIM; k += blockDim.x) {
        float a = 0.f;
#pragma unroll
        for (int s = 0; s < N_USED; s++) a += __ldcg(p.y + (size_t)s * DIM + k) * p.selw[s];
        p.resid[k] += a;
      }
    } else {
      float cv = -INFINITY;
      int ci = 0x7fffffff;
      for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
        const float2 q = __ldcg(p.partials + i);
        if (am_better(q.x, __float_as_int(q.y), cv, ci)) {
          cv = q.x;
          ci = __float_as_int(q.y);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, cv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ci, o);
        if (am_better(ov, oi, cv, ci)) {
          cv = ov;
          ci = oi;
        }
      }
      if (lane == 0) {
        s_bv[warp] = cv;
        s_bi[warp] = ci;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < WPB; w++)
          if (am_better(s_bv[w], s_bi[w], cv, ci)) {
            cv = s_bv[w];
            ci = s_bi[w];
          }
        *p.token = ci == 0x7fffffff ? 0 : ci;
      }
    }
    if (threadIdx.x == 0) *p.counter = 0;
  }
}

template <int MODE, int RPW, int NS>
void launch_mv(MvParams p, dim3 grid, const LaunchCfg& c) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(WPB * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = c.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_mv<MODE, RPW, NS>, p);
}

int grid_for(int ntasks, int tasks_per_cta, const LaunchCfg& c, int ctas_per_sm) {
  int g = (ntasks + tasks_per_cta - 1) / tasks_per_cta;
  int cap = c.sms * ctas_per_sm;
  return g < cap ? (g < 1 ? 1 : g) : cap;
}

MvParams mvp(const Q6Mat& W, XSrc xs) {
  MvParams p = {};
  p.W = W;
  p.W2 = W;
  p.xs = xs;
  return p;
}

}  // namespace

void mv_plain(const Q6Mat& W, XSrc xs, float* y, const LaunchCfg& c) {
  constexpr int RPW = 4;
  MvParams p = mvp(W, xs);
  p.y = y;
  p.ntasks = (W.rows + RPW - 1) / RPW;
  launch_mv<MV_PLAIN, RPW, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

void mv_resid(const Q6Mat& W, XSrc xs, float* resid, const LaunchCfg& c) {
  constexpr int RPW = 2;
  MvParams p = mvp(W, xs);
  p.y = resid;
  p.ntasks = (W.rows + RPW - 1) / RPW;
  launch_mv<MV_RESID, RPW, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

void mv_conv(const Q6Mat& W, XSrc xs, const float* conv_w, float* state, float* gated,
             const LaunchCfg& c) {
  MvParams p = mvp(W, xs);
  p.y = gated;
  p.conv_w = conv_w;
  p.state = state;
  p.ntasks = DIM;
  launch_mv<MV_CONV, 3, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

void mv_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, XSrc xs, float* sw, const LaunchCfg& c) {
  constexpr int RPW = 4;
  MvParams p = mvp(Wg, xs);
  p.W2 = Wu;
  p.y = sw;
  p.ntasks = Wg.rows / (RPW / 2);
  launch_mv<MV_SWIGLU, RPW, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

void mv_down7168_resid(const Q6Mat& W, const float* sw, float* resid, const LaunchCfg& c) {
  constexpr int RPW = 2;
  MvParams p = mvp(W, XSrc{sw, nullptr, 0.f});
  p.y = resid;
  p.ntasks = (W.rows + RPW - 1) / RPW;
  launch_mv<MV_DOWN_SLICED, RPW, 4>(p, dim3(grid_for(p.ntasks, 1, c, 4)), c);
}

void mv_expert_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, int ff, XSrc xs, const int* sel, float* sw,
                      const LaunchCfg& c) {
  constexpr int RPW = 4;
  MvParams p = mvp(Wg, xs);
  p.W2 = Wu;
  p.y = sw;
  p.sel = sel;
  p.ff = ff;
  p.ntasks = N_USED * ff / (RPW / 2);
  launch_mv<MV_XSWIGLU, RPW, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

void mv_expert_down(const Q6Mat& Wd, int ff, const float* sw, const int* sel, const float* selw,
                    float* down, float* resid, unsigned* counter, const LaunchCfg& c) {
  constexpr int RPW = 2;
  MvParams p = mvp(Wd, XSrc{sw, nullptr, 0.f});
  p.y = down;
  p.resid = resid;
  p.sel = sel;
  p.selw = selw;
  p.ff = ff;
  p.counter = counter;
  p.orows = DIM;
  p.ntasks = DIM / RPW;
  int gx = grid_for(p.ntasks, WPB, c, 1);
  launch_mv<MV_XDOWN, RPW, 1>(p, dim3(gx, N_USED), c);
}

void mv_routed(const Q6Mat& W, int orows, const float* x, int x_stride, const int* sel, float* y,
               const LaunchCfg& c) {
  constexpr int RPW = 2;
  MvParams p = mvp(W, XSrc{x, nullptr, 0.f});
  p.y = y;
  p.resid = nullptr;
  p.sel = sel;
  p.ff = x_stride;
  p.orows = orows;
  p.ntasks = (orows + RPW - 1) / RPW;
  int gx = grid_for(p.ntasks, WPB, c, 1);
  launch_mv<MV_XDOWN, RPW, 1>(p, dim3(gx, N_USED), c);
}

void mv_lmhead(const Q6Mat& W, XSrc xs, float* logits, float2* partials, unsigned* counter,
               int* token, const LaunchCfg& c) {
  constexpr int RPW = 4;
  MvParams p = mvp(W, xs);
  p.y = logits;
  p.partials = partials;
  p.counter = counter;
  p.token = token;
  p.ntasks = (W.rows + RPW - 1) / RPW;
  launch_mv<MV_LMHEAD, RPW, 1>(p, dim3(grid_for(p.ntasks, WPB, c, 4)), c);
}

// --------------------------------------------------------------- router
namespace {

// One CTA of 32 warps: warp e computes router logit e over the normalised x,
// warp 0 then selects the top 4 like kernels/resident.rs:58-99: sigmoid,
// + bias, four rounds of max with the lowest id on ties, weights
// p / max(sum p, 6.103515625e-5).
__device__ void route_warp(float lg, const float* bias, int n_expert, int lane, int* sel,
                           float* selw) {
  float prob = 0.f, score = -INFINITY;
  if (lane < n_expert) {
    prob = 1.0f / (1.0f + expf(-lg));
    score = prob + bias[lane];
  }
  float ps[N_USED];
  int ids[N_USED];
#pragma unroll
  for (int r = 0; r < N_USED; r++) {
    const float best = warp_max(score);
    const unsigned m = __ballot_sync(0xffffffffu, score == best && lane < n_expert);
    const int id = m ? __ffs(m) - 1 : 0;
    ps[r] = __shfl_sync(0xffffffffu, prob, id);
    ids[r] = id;
    if (lane == id) score = -INFINITY;
  }
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < N_USED; r++) sum += ps[r];
  sum = fmaxf(sum, 6.103515625e-5f);
  if (lane == 0)
#pragma unroll
    for (int r = 0; r < N_USED; r++) {
      sel[r] = ids[r];
      selw[r] = ps[r] / sum;
    }
}

__global__ void __launch_bounds__(1024) k_router(const float* Wr, const float* bias, XSrc xs,
                                                 int* sel, float* selw) {
  __shared__ float fx[DIM];
  __shared__ float red[32];
  __shared__ float lg[N_EXPERT];
  pdl_trigger();
  pdl_wait();
  float inv = 1.f;
  if (xs.norm) inv = rms_inv(xs.x, xs.eps, red);
  for (int k = threadIdx.x; k < DIM; k += blockDim.x)
    fx[k] = xs.norm ? xs.x[k] * inv * xs.norm[k] : xs.x[k];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const float4* w = (const float4*)(Wr + (size_t)warp * DIM);
    float a = 0.f;
#pragma unroll 4
    for (int i = lane; i < DIM / 4; i += 32) {
      const float4 v = __ldg(w + i);
      a = fmaf(v.x, fx[4 * i + 0], a);
      a = fmaf(v.y, fx[4 * i + 1], a);
      a = fmaf(v.z, fx[4 * i + 2], a);
      a = fmaf(v.w, fx[4 * i + 3], a);
    }
    a = warp_sum(a);
    if (lane == 0) lg[warp] = a;
  }
  __syncthreads();
  if (warp == 0) route_warp(lg[lane], bias, N_EXPERT, lane, sel, selw);
}

// Router over 32 CTAs (one expert logit each) with the top-4 selection done
// by the last CTA to finish (deterministic: logits are reduced in a fixed
// order, the selection reads them back in expert order).
__global__ void __launch_bounds__(256) k_router_mc(const float* Wr, const float* bias, XSrc xs, float* lg,
                                                   unsigned* counter, int* sel, float* selw) {
  __shared__ float red[32];
  __shared__ bool s_last;
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x;
  const float inv = xs.norm ? rms_inv(xs.x, xs.eps, red) : 1.f;
  const float* w = Wr + (size_t)e * DIM;
  float a = 0.f;
  for (int i = threadIdx.x; i < DIM; i += blockDim.x) {
    const float xv = xs.norm ? xs.x[i] * inv * xs.norm[i] : xs.x[i];
    a = fmaf(__ldg(w + i), xv, a);
  }
  a = block_sum(a, red);
  if (threadIdx.x == 0) {
    lg[e] = a;
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x < 32) route_warp(__ldcg(lg + threadIdx.x), bias, (int)gridDim.x, threadIdx.x, sel, selw);
  if (threadIdx.x == 0) *counter = 0;
}

__global__ void k_route_n(const float* logits, const float* bias, int n_expert, int n, int* sel,
                          float* selw) {
  const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= n) return;
  const float lg = lane < n_expert ? logits[(size_t)j * n_expert + lane] : 0.f;
  route_warp(lg, bias, n_expert, lane, sel + (size_t)j * N_USED, selw + (size_t)j * N_USED);
}

// Embedding: one warp dequantises row `tok` (32 units of 64 weights).
__global__ void k_embed(Q6Mat E, const int* token, float* x, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  int tok = *token;
  const int u = threadIdx.x;
  // the id comes from device memory (the previous step's argmax): a value
  // outside the table raises the status word and reads row 0 instead
  if ((unsigned)tok >= (unsigned)E.rows) {
    if (u == 0 && err) atomicExch(err, 4u);
    tok = 0;
  }
  const int U = 4 * E.nb;
  if (u >= U) return;
  const uint4* qp = E.q + (size_t)tok * 3 * U + u;
  float w[64];
  q6_unit_dequant(qp[0], qp[U], qp[2 * U], E.sc[(size_t)tok * U + u],
                  __half2float(E.d[(size_t)tok * E.nb + (u >> 2)]), w);
  const int base = q6_unit_base(u);
#pragma unroll
  for (int m = 0; m < 4; m++)
#pragma unroll
    for (int i = 0; i < 16; i++) x[base + 32 * m + i] = w[m * 16 + i];
}

// ---------------------------------------------------------- attention
__global__ void __launch_bounds__(128) k_attn_decode(AttnDecodeArgs a) {
  const int kh = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int S = ATTN_SPLIT;   // positions per split (== 32: one per lane)
  constexpr int KP = HEAD_DIM + 8; // padded fp16 row (conflict-free 16-byte reads)
  __shared__ float sq[4][HEAD_DIM];
  __shared__ __align__(16) __half sk[S][KP];
  __shared__ __align__(16) __half sv[S][HEAD_DIM];
  __shared__ bool s_last;
  pdl_trigger();
  pdl_wait();
  const int pos = *a.pos;
  const int t0 = split * S;
  if (t0 > pos) return;
  const int nact = pos / S + 1;
  const int nsplit = (a.ctx + S - 1) / S;
  const int h = kh * (HEADS / KV_HEADS) + warp;  // GQA: kh = h * kv / heads
  const float2 cs = a.rope[(size_t)pos * 32 + lane];
  {
    // head RMSNorm (lfm.rs:270-286) then NEOX RoPE (lfm.rs:248-267); lane owns
    // the rotation pair (lane, lane + 32).
    float q0 = a.qkv[h * HEAD_DIM + lane], q1 = a.qkv[h * HEAD_DIM + lane + 32];
    const float ss = warp_sum(q0 * q0 + q1 * q1);
    const float inv = 1.0f / sqrtf(ss / (float)HEAD_DIM + a.eps);
    q0 *= inv * a.q_norm[lane];
    q1 *= inv * a.q_norm[lane + 32];
    sq[warp][lane] = q0 * cs.x - q1 * cs.y;
    sq[warp][lane + 32] = q0 * cs.y + q1 * cs.x;
  }
  if (pos < t0 + S) {
    // This split holds `pos`: write the new K/V (fp16, RNE) before reading.
    const size_t off = ((size_t)kh * a.ctx + pos) * HEAD_DIM;
    if (warp == 0) {
      float k0 = a.qkv[DIM + kh * HEAD_DIM + lane], k1 = a.qkv[DIM + kh * HEAD_DIM + lane + 32];
      const float ss = warp_sum(k0 * k0 + k1 * k1);
      const float inv = 1.0f / sqrtf(ss / (float)HEAD_DIM + a.eps);
      k0 *= inv * a.k_norm[lane];
      k1 *= inv * a.k_norm[lane + 32];
      a.kc[off + lane] = __float2half_rn(k0 * cs.x - k1 * cs.y);
      a.kc[off + lane + 32] = __float2half_rn(k0 * cs.y + k1 * cs.x);
    } else if (warp == 1) {
      const float* v = a.qkv + DIM + KV_HEADS * HEAD_DIM + kh * HEAD_DIM;
      a.vc[off + lane] = __float2half_rn(v[lane]);
      a.vc[off + lane + 32] = __float2half_rn(v[lane + 32]);
    }
    __syncthreads();
  }
  const int tend = min(t0 + S, pos + 1);
  const int cnt = tend - t0;
  {
    // stage the K and V tiles (S x 64 fp16 each): 128 threads x 2 x 16 B
    const uint4* kg = (const uint4*)(a.kc + ((size_t)kh * a.ctx + t0) * HEAD_DIM);
    const uint4* vg = (const uint4*)(a.vc + ((size_t)kh * a.ctx + t0) * HEAD_DIM);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int idx = threadIdx.x + i * 128;  // 0..255 = 32 rows x 8 chunks
      const int r = idx >> 3, c = idx & 7;
      if (r < cnt) {
        *(uint4*)&sk[r][c * 8] = kg[idx];
        *(uint4*)&sv[r][c * 8] = vg[idx];
      }
    }
  }
  __syncthreads();
  // scores: lane = position
  float sc = -INFINITY;
  if (lane < cnt) {
    float acc = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < 8; c8++) {
      const uint4 v = *(const uint4*)&sk[lane][c8 * 8];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(*(const __half2*)&w[j]);
        acc = fmaf(f.x, sq[warp][c8 * 8 + 2 * j], acc);
        acc = fmaf(f.y, sq[warp][c8 * 8 + 2 * j + 1], acc);
      }
    }
    sc = acc * 0.125f;  // 1/sqrt(head_dim)
  }
  const float m = warp_max(sc);
  const float pl = lane < cnt ? expf(sc - m) : 0.f;
  const float l = warp_sum(pl);
  float o0 = 0.f, o1 = 0.f;
#pragma unroll 8
  for (int t = 0; t < cnt; t++) {
    const float pt = __shfl_sync(0xffffffffu, pl, t);
    o0 = fmaf(pt, __half2float(sv[t][lane]), o0);
    o1 = fmaf(pt, __half2float(sv[t][lane + 32]), o1);
  }
  float* pp = a.part + (((size_t)kh * nsplit + split) * 4 + warp) * (HEAD_DIM + 2);
  pp[lane] = o0;
  pp[lane + 32] = o1;
  if (lane == 0) {
    pp[64] = m;
    pp[65] = l;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&a.counters[kh], 1u) == (unsigned)(nact - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Merge the splits in index order (attention_split.rs:18-33).
  const float* base = a.part + ((size_t)kh * nsplit * 4 + warp) * (HEAD_DIM + 2);
  float M = -INFINITY;
  for (int sidx = lane; sidx < nact; sidx += 32) M = fmaxf(M, __ldcg(base + (size_t)sidx * 4 * (HEAD_DIM + 2) + 64));
  M = warp_max(M);
  float L = 0.f, O0 = 0.f, O1 = 0.f;
  for (int sidx = 0; sidx < nact; sidx++) {
    const float* q = base + (size_t)sidx * 4 * (HEAD_DIM + 2);
    const float w = expf(__ldcg(q + 64) - M);
    L = fmaf(__ldcg(q + 65), w, L);
    O0 = fmaf(__ldcg(q + lane), w, O0);
    O1 = fmaf(__ldcg(q + lane + 32), w, O1);
  }
  a.out[h * HEAD_DIM + lane] = O0 / L;
  a.out[h * HEAD_DIM + lane + 32] = O1 / L;
  if (threadIdx.x == 0) a.counters[kh] = 0;
}

template <typename K, typename... Args>
void launch_pdl(K kernel, dim3 grid, dim3 block, const LaunchCfg& c, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = c.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

void router_top4(const float* Wr, const float* bias, XSrc xs, int* sel, float* selw,
                 const LaunchCfg& c) {
  launch_pdl(k_router, dim3(1), dim3(1024), c, Wr, bias, xs, sel, selw);
}

void router_top4_mc(const float* Wr, const float* bias, XSrc xs, float* lg_scratch, unsigned* counter, int* sel,
                    float* selw, const LaunchCfg& c) {
  launch_pdl(k_router_mc, dim3(N_EXPERT), dim3(256), c, Wr, bias, xs, lg_scratch, counter, sel, selw);
}

void route_n(const float* logits, const float* bias, int n_expert, int n, int* sel, float* selw,
             cudaStream_t s) {
  k_route_n<<<(n + 7) / 8, 256, 0, s>>>(logits, bias, n_expert, n, sel, selw);
}

void embed_token(const Q6Mat& E, const int* token, float* x, unsigned* err, const LaunchCfg& c) {
  launch_pdl(k_embed, dim3(1), dim3(32), c, E, token, x, err);
}

void attn_decode(const AttnDecodeArgs& a, const LaunchCfg& c) {
  const int nsplit = (a.ctx + ATTN_SPLIT - 1) / ATTN_SPLIT;
  launch_pdl(k_attn_decode, dim3(KV_HEADS, nsplit), dim3(128), c, a);
}

// ------------------------------------------------------------ generic ops
namespace {
__global__ void k_dequant_rows(Q6Mat W, int row0, int nrows, float* out) {
  const int U = 4 * W.nb;
  const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (size_t)nrows * U) return;
  const int r = (int)(gid / U), u = (int)(gid % U);
  const size_t row = (size_t)row0 + r;
  const uint4* qp = W.q + row * 3 * U + u;
  float w[64];
  q6_unit_dequant(qp[0], qp[U], qp[2 * U], W.sc[row * U + u], __half2float(W.d[row * W.nb + (u >> 2)]), w);
  float* o = out + (size_t)r * W.nb * QK + q6_unit_base(u);
#pragma unroll
  for (int m = 0; m < 4; m++)
#pragma unroll
    for (int i = 0; i < 16; i++) o[32 * m + i] = w[m * 16 + i];
}

__global__ void k_argmax_partial(const float* x, int n, float2* partials, unsigned* counter, int* out) {
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  __shared__ bool s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (am_better(x[i], i, bv, bi)) {
      bv = x[i];
      bi = i;
    }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_bv[warp] = bv;
    s_bi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; w++)
      if (am_better(s_bv[w], s_bi[w], bv, bi)) {
        bv = s_bv[w];
        bi = s_bi[w];
      }
    partials[blockIdx.x] = make_float2(bv, __int_as_float(bi));
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  float cv = -INFINITY;
  int ci = 0x7fffffff;
  for (int i = 0; i < (int)gridDim.x; i++) {
    const float2 q = __ldcg(partials + i);
    if (am_better(q.x, __float_as_int(q.y), cv, ci)) {
      cv = q.x;
      ci = __float_as_int(q.y);
    }
  }
  *out = ci == 0x7fffffff ? 0 : ci;
  *counter = 0;
}
}  // namespace

void q6_dequant_rows(const Q6Mat& W, int row0, int nrows, float* out, cudaStream_t s) {
  const size_t total = (size_t)nrows * 4 * W.nb;
  k_dequant_rows<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(W, row0, nrows, out);
}

void argmax_f32(const float* x, int n, float2* partials, unsigned* counter, int* out, cudaStream_t s) {
  int g = (n + 1023) / 1024;
  if (g > 256) g = 256;
  if (g < 1) g = 1;
  k_argmax_partial<<<g, 1024, 0, s>>>(x, n, partials, counter, out);
}

}  // namespace lfm
