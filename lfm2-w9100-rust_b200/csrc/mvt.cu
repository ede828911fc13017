// TMA-staged Q6_K decode matvecs (sm_100a).
//
// One CTA per SM streams a contiguous range of row tiles from HBM into shared
// memory with bulk asynchronous copies (cp.async.bulk, each CTA loading its own tiles) issued by
// a dedicated producer warp and completed on mbarriers; eight consumer warps
// compute from shared memory with the activations held in registers (one
// 64-weight unit per lane, layout of q6k.cuh). Because weights do not depend
// on the previous kernel, the producer issues its first tiles BEFORE
// griddepcontrol.wait, so under programmatic dependent launch the weight
// stream of a kernel overlaps the tail of the one before it.
//
// Tiles (a stage holds up to 24 rows):
//   PLAIN / RESID / LMHEAD : 16 consecutive rows, warp w -> rows 2w, 2w+1
//   CONV                   : 8 channels x (b, c, x) rows, warp w -> channel w
//   SWIGLU / XSWIGLU       : 8 (gate, up) row pairs, warp w -> pair w
//   XDOWN                  : 16 rows of the slot's expert, warp w -> rows 2w, 2w+1
// Every wait on an mbarrier is bounded (1 s of %globaltimer); on timeout the
// kernel raises the engine's device error word, drains its own copies and
// returns instead of hanging.
#include <math.h>

#include <stdlib.h>

#include "dev_common.cuh"
#include "host_once.h"

namespace lfm {
namespace {

constexpr int NCW = 8;                // consumer warps
constexpr int NTHREADS = (NCW + 1) * 32;

enum Mode { M_PLAIN, M_RESID, M_LMHEAD, M_CONV, M_SWIGLU, M_XSWIGLU, M_XDOWN, M_QKV };

struct MvtParams {
  Q6Mat W, W2;
  XSrc xs;
  float* y;
  float* resid;
  const float* conv_w;
  float* state;
  const int* sel;
  const float* selw;
  float2* partials;
  unsigned* counter;
  int* token;
  unsigned* err;
  int ntiles;
  int ff;  // expert ff (XSWIGLU rows per expert, XDOWN x stride)
  Q6Mat W3;       // M_QKV: W = q, W2 = k, W3 = v (outputs y, y + q.rows, ...)
};

using namespace dev;

template <int MODE>
struct TileDef {
  static constexpr int NSEG = MODE == M_CONV ? 3 : (MODE == M_SWIGLU || MODE == M_XSWIGLU) ? 2 : 1;
  static constexpr int SEGROWS = (MODE == M_CONV || MODE == M_SWIGLU || MODE == M_XSWIGLU) ? 8 : 16;
  static constexpr bool ROUTED = MODE == M_XSWIGLU || MODE == M_XDOWN;
  static constexpr int ROWS = NSEG * SEGROWS;        // rows per stage
  static constexpr int STAGES = ROWS > 16 ? 3 : 4;   // <= ~121 KB of shared memory
};

// QKV tiles: 0..127 -> q rows, then k, then v (16 rows each).
__device__ __forceinline__ const Q6Mat& qkv_mat(const MvtParams& p, int t, int& row0, int& obase) {
  const int tq = p.W.rows / 16, tk = p.W2.rows / 16;
  if (t < tq) {
    row0 = t * 16;
    obase = 0;
    return p.W;
  }
  if (t < tq + tk) {
    row0 = (t - tq) * 16;
    obase = p.W.rows;
    return p.W2;
  }
  row0 = (t - tq - tk) * 16;
  obase = p.W.rows + p.W2.rows;
  return p.W3;
}

// Row (in its matrix) of segment s of tile t, and the slot for routed tiles.
template <int MODE>
__device__ __forceinline__ int seg_row0(const MvtParams& p, int t, int s, int& slot) {
  slot = 0;
  if (MODE == M_CONV) return t * 8 + s * DIM;
  if (MODE == M_SWIGLU) return t * 8;
  if (MODE == M_XSWIGLU) {
    const int per = p.ff / 8;
    slot = t / per;
    return p.sel[slot] * p.ff + (t - slot * per) * 8;
  }
  if (MODE == M_XDOWN) {
    const int per = DIM / 16;
    slot = t / per;
    return p.sel[slot] * DIM + (t - slot * per) * 16;
  }
  return t * 16;
}

template <int MODE>
__global__ void __launch_bounds__(NTHREADS, 2) k_mvt(MvtParams p) {
  using TD = TileDef<MODE>;
  constexpr int STAGES = TD::STAGES;
  constexpr int MAX_ROWS = TD::ROWS;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[STAGES], empty[STAGES];
  __shared__ float red[NCW + 1];
  __shared__ float s_bv[NCW];
  __shared__ int s_bi[NCW];
  __shared__ bool s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Q6Mat& W = p.W;
  const int nb = W.nb, U = 4 * nb;
  const uint32_t row_q = 48u * U, row_sc = 4u * U, row_d = 2u * nb;
  const uint32_t q_off = 0, sc_off = MAX_ROWS * row_q, d_off = sc_off + MAX_ROWS * row_sc;
  const uint32_t stage_bytes = (d_off + MAX_ROWS * row_d + 127) & ~127u;
  const int t_begin = (int)((long long)blockIdx.x * p.ntiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * p.ntiles / gridDim.x);
  const int ntl = t_end - t_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (ntl == 0 && threadIdx.x == 0) pdl_trigger();

  if (warp == NCW) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      if (TD::ROUTED) pdl_wait();  // expert ids come from the previous kernel
      bool ok = true;
      int issued = 0;
      for (int k = 0; k < ntl && ok; k++) {
        const int st = k % STAGES, round = k / STAGES;
        if (round > 0) ok = mbar_wait(&empty[st], (round - 1) & 1, p.err);
        if (!ok) break;
        const int t = t_begin + k;
        uint8_t* base = smem + st * stage_bytes;
        int rows_in[TD::NSEG], r0[TD::NSEG];
        uint32_t tx = 0;
        int ob_unused = 0;
        int qkv_r0 = 0;
        const Q6Mat& MQ = MODE == M_QKV ? qkv_mat(p, t, qkv_r0, ob_unused) : W;
#pragma unroll
        for (int s = 0; s < TD::NSEG; s++) {
          int slot;
          r0[s] = MODE == M_QKV ? qkv_r0 : seg_row0<MODE>(p, t, s, slot);
          const Q6Mat& M = (TD::NSEG == 2 && s == 1) ? p.W2 : MQ;
          int n = M.rows - r0[s];
          rows_in[s] = n < TD::SEGROWS ? n : TD::SEGROWS;
          tx += rows_in[s] * (row_q + row_sc + row_d);
        }
        mbar_expect_tx(&full[st], tx);
#pragma unroll
        for (int s = 0; s < TD::NSEG; s++) {
          const Q6Mat& M = (TD::NSEG == 2 && s == 1) ? p.W2 : MQ;
          const int sr = s * TD::SEGROWS;  // stage row of the segment
          const size_t row = (size_t)r0[s];
          bulk_g2s(base + q_off + sr * row_q, (const uint8_t*)M.q + row * row_q, rows_in[s] * row_q, &full[st]);
          bulk_g2s(base + sc_off + sr * row_sc, (const uint8_t*)M.sc + row * row_sc, rows_in[s] * row_sc,
                   &full[st]);
          bulk_g2s(base + d_off + sr * row_d, (const uint8_t*)M.d + row * row_d, rows_in[s] * row_d, &full[st]);
        }
        issued = k + 1;
        if (issued == ntl) pdl_trigger();  // dependents may launch once our weights are in flight
      }
      if (issued < ntl) pdl_trigger();
      // Drain: every issued stage must have landed before the CTA may exit.
      for (int k = (issued > STAGES ? issued - STAGES : 0); k < issued; k++)
        mbar_wait(&full[k % STAGES], (k / STAGES) & 1, p.err);
    }
    // the producer warp takes no part in the epilogue reductions below
    if (MODE != M_LMHEAD && MODE != M_XDOWN) return;
  }

  // -------------------------------------------------------------- consumers
  float xr[64];
  const int u = lane < U ? lane : -1;  // U <= 32 for this kernel
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if (warp < NCW) {
    pdl_wait();
    // activations (RMS-normalised when xs.norm is set)
    float inv = 1.f;
    if (p.xs.norm && MODE != M_XDOWN) {
      float ss = 0.f;
      for (int i = threadIdx.x; i < DIM; i += NCW * 32) ss = fmaf(p.xs.x[i], p.xs.x[i], ss);
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
      float t = 0.f;
      for (int i = 0; i < NCW; i++) t += red[i];
      inv = 1.0f / sqrtf(t / (float)DIM + p.xs.eps);
    }
    int cur_slot = -1;
    auto load_x = [&](const float* x, const float* norm) {
      if (u < 0) return;
      const int base = q6_unit_base(u);
#pragma unroll
      for (int m = 0; m < 4; m++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 v = *(const float4*)(x + base + 32 * m + 4 * q);
          if (norm) {
            const float4 g = *(const float4*)(norm + base + 32 * m + 4 * q);
            xr[m * 16 + 4 * q + 0] = v.x * inv * g.x;
            xr[m * 16 + 4 * q + 1] = v.y * inv * g.y;
            xr[m * 16 + 4 * q + 2] = v.z * inv * g.z;
            xr[m * 16 + 4 * q + 3] = v.w * inv * g.w;
          } else {
            xr[m * 16 + 4 * q + 0] = v.x;
            xr[m * 16 + 4 * q + 1] = v.y;
            xr[m * 16 + 4 * q + 2] = v.z;
            xr[m * 16 + 4 * q + 3] = v.w;
          }
        }
    };
    if (MODE != M_XDOWN) load_x(p.xs.x, p.xs.norm);

    for (int k = 0; k < ntl; k++) {
      const int st = k % STAGES;
      const int t = t_begin + k;
      int slot = 0;
      int row0 = 0, obase = 0, mrows = W.rows;
      if (MODE == M_QKV) {
        mrows = qkv_mat(p, t, row0, obase).rows;
      } else {
        row0 = seg_row0<MODE>(p, t, 0, slot);
      }
      if (MODE == M_XDOWN && slot != cur_slot) {
        load_x(p.xs.x + (size_t)slot * p.ff, nullptr);
        cur_slot = slot;
      }
      if (!mbar_wait(&full[st], (k / STAGES) & 1, p.err)) break;
      const uint8_t* base = smem + st * stage_bytes;
      // stage rows of this warp
      constexpr int RPW = MODE == M_CONV ? 3 : 2;
      int srow[RPW];
#pragma unroll
      for (int r = 0; r < RPW; r++) {
        if (MODE == M_CONV) srow[r] = warp + 8 * r;
        else if (MODE == M_SWIGLU || MODE == M_XSWIGLU) srow[r] = warp + 8 * r;
        else srow[r] = 2 * warp + r;
      }
      // validity (partial last tile of a plain matrix)
      const int seg_rows = (MODE == M_PLAIN || MODE == M_RESID || MODE == M_LMHEAD || MODE == M_QKV)
                               ? min(16, mrows - row0)
                               : TD::SEGROWS;
      float acc[RPW];
#pragma unroll
      for (int r = 0; r < RPW; r++) {
        const int rr = srow[r] % TD::SEGROWS;
        const bool valid = rr < seg_rows;
        float a = 0.f;
        if (valid && u >= 0) {
          const uint4* qp = (const uint4*)(base + q_off + srow[r] * row_q) + u;
          const uint4 A = qp[0], B = qp[U], Q = qp[2 * U];
          const uint32_t scw = *(const uint32_t*)(base + sc_off + srow[r] * row_sc + 4 * u);
          const float d = __half2float(*(const __half*)(base + d_off + srow[r] * row_d + 2 * (u >> 2)));
          a = q6_unit_dot(A, B, Q, scw, d, xr);
        }
        acc[r] = a;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
      for (int r = 0; r < RPW; r++) acc[r] = warp_sum(acc[r]);
      if (lane != 0) continue;
      // -------------------------------------------------------- epilogue
      if (MODE == M_PLAIN || MODE == M_RESID || MODE == M_LMHEAD || MODE == M_QKV) {
#pragma unroll
        for (int r = 0; r < RPW; r++) {
          if (srow[r] >= seg_rows) continue;
          const int row = row0 + srow[r];
          if (MODE == M_QKV) p.y[obase + row] = acc[r];
          else if (MODE == M_PLAIN) p.y[row] = acc[r];
          else if (MODE == M_RESID) p.y[row] += acc[r];
          else {
            p.y[row] = acc[r];
            if (am_better(acc[r], row, bv, bi)) {
              bv = acc[r];
              bi = row;
            }
          }
        }
      } else if (MODE == M_CONV) {
        const int ch = t * 8 + warp;
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
      } else if (MODE == M_SWIGLU) {
        p.y[t * 8 + warp] = silu_mul(acc[0], acc[1]);
      } else if (MODE == M_XSWIGLU) {
        const int per = p.ff / 8;
        const int s = t / per;
        p.y[(size_t)s * p.ff + (t - s * per) * 8 + warp] = silu_mul(acc[0], acc[1]);
      } else if (MODE == M_XDOWN) {
        const int per = DIM / 16;
        const int s = t / per;
        const int o = (t - s * per) * 16 + srow[0];
        p.y[(size_t)s * DIM + o] = acc[0];
        p.y[(size_t)s * DIM + o + 1] = acc[1];
      }
    }
  }

  if (MODE == M_LMHEAD || MODE == M_XDOWN) {
    if (MODE == M_LMHEAD) {
      if (warp < NCW && lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        float cv = s_bv[0];
        int ci = s_bi[0];
        for (int w = 1; w < NCW; w++)
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
      s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (MODE == M_XDOWN) {
      for (int kk = threadIdx.x; kk < DIM; kk += NTHREADS) {
        float a = 0.f;
#pragma unroll
        for (int s = 0; s < N_USED; s++) a += __ldcg(p.y + (size_t)s * DIM + kk) * p.selw[s];
        p.resid[kk] += a;
      }
    } else if (warp == 0) {
      float cv = -INFINITY;
      int ci = 0x7fffffff;
      for (int i = lane; i < (int)gridDim.x; i += 32) {
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
      if (lane == 0) *p.token = ci == 0x7fffffff ? 0 : ci;
    }
    if (threadIdx.x == 0) *p.counter = 0;
  }
}

size_t stage_bytes_for(int nb, int rows) {
  const size_t U = 4 * nb;
  const size_t b = rows * (48 * U + 4 * U + 2 * nb);
  return (b + 127) & ~(size_t)127;
}

template <int MODE>
void launch_mvt(const MvtParams& p, const LaunchCfg& c) {
  using TD = TileDef<MODE>;
  const size_t smem = TD::STAGES * stage_bytes_for(p.W.nb, TD::ROWS);
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu, [] {
    cudaFuncSetAttribute(k_mvt<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)(TD::STAGES * stage_bytes_for(8, TD::ROWS)));
    // all of the unified L1/shared array as shared memory, so two CTAs (this
    // kernel and the next one under PDL) fit on an SM
    cudaFuncSetAttribute(k_mvt<MODE>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  });
  // One or two CTAs per SM. Two hide more dependent-instruction latency (each
  // CTA keeps its own 3-4 stage weight ring) and pay off when every CTA has
  // many tiles (lm_head); for the short per-layer matrices one CTA per SM
  // measured faster (fewer ring fills per tile).
  static int env_per_sm = -1;
  if (env_per_sm < 0) {
    const char* v = getenv("LFM_MVT_CTAS_PER_SM");
    env_per_sm = v ? atoi(v) : 0;
    if (env_per_sm < 0 || env_per_sm > 2) env_per_sm = 0;
  }
  const int per_sm = env_per_sm ? env_per_sm : (p.ntiles >= 16 * c.sms ? 2 : 1);
  const int cap = c.sms * per_sm;
  int g = p.ntiles < cap ? p.ntiles : cap;
  if (g < 1) g = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr_[1];
  attr_[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_;
  cfg.numAttrs = c.pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, k_mvt<MODE>, p);
}

MvtParams base_params(const Q6Mat& W, XSrc xs, unsigned* err) {
  MvtParams p = {};
  p.W = W;
  p.W2 = W;
  p.xs = xs;
  p.err = err;
  return p;
}

}  // namespace

bool mvt_supported(const Q6Mat& W) { return (W.nb == 8 || W.nb == 7) && W.rows % 16 == 0; }

void mvt_plain(const Q6Mat& W, XSrc xs, float* y, unsigned* err, const LaunchCfg& c) {
  MvtParams p = base_params(W, xs, err);
  p.y = y;
  p.ntiles = (W.rows + 15) / 16;
  launch_mvt<M_PLAIN>(p, c);
}

void mvt_qkv(const Q6Mat& Wq, const Q6Mat& Wk, const Q6Mat& Wv, XSrc xs, float* y, unsigned* err,
             const LaunchCfg& c) {
  MvtParams p = base_params(Wq, xs, err);
  p.W2 = Wk;
  p.W3 = Wv;
  p.y = y;
  p.ntiles = (Wq.rows + Wk.rows + Wv.rows) / 16;
  launch_mvt<M_QKV>(p, c);
}

void mvt_resid(const Q6Mat& W, XSrc xs, float* resid, unsigned* err, const LaunchCfg& c) {
  MvtParams p = base_params(W, xs, err);
  p.y = resid;
  p.ntiles = (W.rows + 15) / 16;
  launch_mvt<M_RESID>(p, c);
}

void mvt_conv(const Q6Mat& W, XSrc xs, const float* conv_w, float* state, float* gated, unsigned* err,
              const LaunchCfg& c) {
  MvtParams p = base_params(W, xs, err);
  p.y = gated;
  p.conv_w = conv_w;
  p.state = state;
  p.ntiles = DIM / 8;
  launch_mvt<M_CONV>(p, c);
}

void mvt_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, XSrc xs, float* sw, unsigned* err, const LaunchCfg& c) {
  MvtParams p = base_params(Wg, xs, err);
  p.W2 = Wu;
  p.y = sw;
  p.ntiles = Wg.rows / 8;
  launch_mvt<M_SWIGLU>(p, c);
}

void mvt_expert_swiglu(const Q6Mat& Wg, const Q6Mat& Wu, int ff, XSrc xs, const int* sel, float* sw, unsigned* err,
                       const LaunchCfg& c) {
  MvtParams p = base_params(Wg, xs, err);
  p.W2 = Wu;
  p.y = sw;
  p.sel = sel;
  p.ff = ff;
  p.ntiles = N_USED * ff / 8;
  launch_mvt<M_XSWIGLU>(p, c);
}

void mvt_expert_down(const Q6Mat& Wd, int ff, const float* sw, const int* sel, const float* selw, float* down,
                     float* resid, unsigned* counter, unsigned* err, const LaunchCfg& c) {
  MvtParams p = base_params(Wd, XSrc{sw, nullptr, 0.f}, err);
  p.y = down;
  p.resid = resid;
  p.sel = sel;
  p.selw = selw;
  p.ff = ff;
  p.counter = counter;
  p.ntiles = N_USED * DIM / 16;
  launch_mvt<M_XDOWN>(p, c);
}

void mvt_lmhead(const Q6Mat& W, XSrc xs, float* logits, float2* partials, unsigned* counter, int* token,
                unsigned* err, const LaunchCfg& c) {
  MvtParams p = base_params(W, xs, err);
  p.y = logits;
  p.partials = partials;
  p.counter = counter;
  p.token = token;
  p.ntiles = (W.rows + 15) / 16;
  launch_mvt<M_LMHEAD>(p, c);
}

}  // namespace lfm
