// Persistent batch-1 decode step (sm_100a).
//
// One cooperative launch, one CTA per SM, runs the whole decode token: the
// ~126 dependent stages of the reference's resident graph
// (gpu_lfm/resident_graph.rs:226-546) become a stage list walked in order by
// every CTA. Between dependent stages the CTAs meet at a grid barrier
// (monotonic arrival counters in global memory, acquire/release ordering,
// bounded polling). Thread 0 of each CTA doubles as the producer: a
// non-blocking state machine, advanced whenever thread 0 would otherwise wait,
// streams this CTA's weight tiles of ALL stages, in order, through a 4-slot
// shared-memory ring with bulk async copies (cp.async.bulk, no multicast)
// completed on mbarriers. It waits on no grid barrier except before
// routed-expert tiles (the expert ids come from the router stage), so the
// weight stream of stage s+1.. is in flight while stage s computes, and HBM
// streaming continues across the dependency chain instead of restarting at
// every kernel boundary. (A separate producer warp would make 17 warps, and
// the register file is split over four SM sub-partitions: 17 warps cap every
// thread at 96 registers, 16 warps allow 128.)
//
// All 16 warps compute: they hold the stage's activation vector in registers
// (one 64-weight unit per lane, q6k.cuh layout), dequantise weight tiles from
// the ring, and run the stage epilogues (residual, short conv, SwiGLU,
// rank-ordered expert combine, argmax). Activations written by other CTAs are
// read with L2-coherent loads (ld.global.cg). Every wait is bounded (1 s); a
// timeout raises the status word, sets an abort flag that releases all other
// waits, and the kernel drains its copies and returns.
#include <math.h>

#include <string>

#include "dev_common.cuh"
#include "step.h"

namespace lfm {
namespace {
using namespace dev;

constexpr int NCW = 16;                // warps; all compute, thread 0 also produces
constexpr int NT = NCW * 32;           // 16 warps x 128 registers fill the register file
constexpr int RING = 4;
constexpr int SLOT = 40320;            // 24 rows x (1536 + 128 + 16): the largest tile
constexpr int KP = HEAD_DIM + 8;       // padded fp16 K row in shared memory

struct AttnSmem {
  float sq[4][HEAD_DIM];
  __align__(16) __half sk[ATTN_SPLIT][KP];
  __align__(16) __half sv[ATTN_SPLIT][HEAD_DIM];
  int last;
};

// Activation vector(s) of a ring stage staged once per CTA, in x-register
// order: element (unit u, slot m*16+i) at xs[((m*4 + i/4) * U + u) * 4 + i%4],
// so lane u's 16 float4 reads are consecutive across lanes (conflict-free).
constexpr int XS_FLOATS = N_USED * EXPERT_FF;  // 7168: 4 expert vectors or one 7168 vector
union StageSmem {
  AttnSmem attn[2];
  __align__(16) float xs[XS_FLOATS];
};

__device__ __forceinline__ int xs_index(int k, int U) {
  const int b = k >> 8, e = k & 255, h = e >> 7, r = e & 127;
  const int m = r >> 5, l = r & 31, qq = l >> 4, i = l & 15;
  const int u = 4 * b + 2 * h + qq;
  return ((m * 4 + (i >> 2)) * U + u) * 4 + (i & 3);
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_vol(const unsigned* p) { return *(volatile const unsigned*)p; }
// Stage descriptors live in shared memory, after the weight ring: an acquire
// at gpu scope invalidates L1, so descriptors read from global memory would
// turn every producer step into a chain of L2 round trips.
__device__ __forceinline__ StepStage* stage_table(uint8_t* ring) { return (StepStage*)(ring + RING * SLOT); }
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
// CTA barriers in the non-aligned form: thread 0 may reach them from its own
// producer/poll path while the rest of warp 0 is already waiting.
__device__ __forceinline__ void cons_sync() { asm volatile("barrier.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }
// named barriers 2..3: the two 4-warp attention groups
__device__ __forceinline__ void group_sync(int g) {
  if (g == 0)
    asm volatile("barrier.sync 2, 128;" ::: "memory");
  else
    asm volatile("barrier.sync 3, 128;" ::: "memory");
}

__device__ void raise_abort(StepCtl* ctl, unsigned code) {
  atomicExch(&ctl->err, code);
  atomicExch(&ctl->abort, 1u);
}

// mbarrier wait that also gives up once another CTA aborted.
__device__ bool ring_wait(uint64_t* b, uint32_t parity, StepCtl* ctl) {
  WaitBudget wb;
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 15u) == 15u) {
      if (ld_vol(&ctl->abort)) return false;
      if (wb.spent()) {
        raise_abort(ctl, 3u);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool is_ring(int t) {
  return t == ST_QKV || t == ST_RESID || t == ST_CONV || t == ST_XSWIGLU || t == ST_XDOWN || t == ST_SWIGLU ||
         t == ST_DOWN28 || t == ST_LMHEAD;
}
__device__ __forceinline__ int tile_nseg(int t) {
  return t == ST_CONV ? 3 : (t == ST_SWIGLU || t == ST_XSWIGLU) ? 2 : t == ST_XDOWN ? 4 : 1;
}
__device__ __forceinline__ int tile_segrows(int t) {
  return (t == ST_CONV || t == ST_SWIGLU || t == ST_XSWIGLU) ? 8 : (t == ST_XDOWN || t == ST_DOWN28) ? 4 : 16;
}

// Matrix and first row of segment `seg` of tile `t`; obase = output offset (QKV).
__device__ __forceinline__ const Q6Mat& seg_src(const StepStage& S, const int* sel, int t, int seg, int& row0,
                                                int& obase) {
  obase = 0;
  switch (S.type) {
    case ST_QKV: {
      const int tq = S.W.rows / 16, tk = S.W2.rows / 16;
      if (t < tq) {
        row0 = t * 16;
        return S.W;
      }
      if (t < tq + tk) {
        row0 = (t - tq) * 16;
        obase = S.W.rows;
        return S.W2;
      }
      row0 = (t - tq - tk) * 16;
      obase = S.W.rows + S.W2.rows;
      return S.W3;
    }
    case ST_CONV:
      row0 = t * 8 + seg * DIM;
      return S.W;
    case ST_SWIGLU:
      row0 = t * 8;
      return seg ? S.W2 : S.W;
    case ST_XSWIGLU: {
      const int per = S.ff / 8, slot = t / per;
      row0 = sel[slot] * S.ff + (t - slot * per) * 8;
      return seg ? S.W2 : S.W;
    }
    case ST_XDOWN:
      row0 = sel[seg] * DIM + t * 4;
      return S.W;
    case ST_DOWN28:
      row0 = t * 4;
      return S.W;
    default:
      row0 = t * 16;
      return S.W;
  }
}

__device__ __forceinline__ void tile_range(int ntiles, int& t0, int& t1) {
  t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x);
  t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
}

// --------------------------------------------------------------- producer
// Thread 0 is also the producer: a non-blocking state machine walks this CTA's
// weight tiles of all stages in order and issues each one as soon as its ring
// slot is free (and, for expert tiles, once the router stage has published the
// expert ids). Thread 0 advances it whenever it would otherwise wait. Its state
// lives in shared memory between polls; a poll copies it and the stage fields
// it needs into registers first, because every mbarrier / bulk-copy asm
// statement is a compiler memory barrier that would otherwise turn each field
// access into a fresh shared-memory round trip on the critical path.
struct Cursor {
  int s, t, t1, k;  // stage, tile, end tile, tiles issued so far
  int ready;        // tile range (and expert ids) of stage s loaded
  int sel[N_USED];
};

__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Producer-side forms of the mbarrier / bulk-copy instructions without a
// compiler memory clobber: the producer reads no data that these order (the
// consumers' view of a tile is ordered by their own waits on the full
// barrier), so the compiler may keep descriptor fields in registers across them.
__device__ __forceinline__ void p_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes));
}
__device__ __forceinline__ void p_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar)));
}
__device__ __forceinline__ bool p_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity));
  return ok != 0;
}

// Copy tile t of stage S into the ring slot at `base`.
__device__ __forceinline__ void issue_tile(const StepStage& S, const int (&sel)[N_USED], int t, uint8_t* base,
                                           uint64_t* bar) {
  const int type = S.type;
  const int nseg = tile_nseg(type), segrows = tile_segrows(type);
  const int nb = S.W.nb, U = 4 * nb;
  const uint32_t row_q = 48u * U, row_sc = 4u * U, row_d = 2u * nb;
  const bool d_bulk = type != ST_XDOWN;
  const uint32_t R = nseg * segrows;
  const uint32_t sc_off = R * row_q, d_off = sc_off + R * row_sc;
  p_expect_tx(bar, R * (row_q + row_sc + (d_bulk ? row_d : 0)));
  for (int g = 0; g < nseg; g++) {
    int row0, ob;
    const Q6Mat& M = seg_src(S, sel, t, g, row0, ob);
    const uint32_t sr = g * segrows;
    const size_t row = (size_t)row0;
    p_bulk(base + sr * row_q, (const uint8_t*)M.q + row * row_q, segrows * row_q, bar);
    p_bulk(base + sc_off + sr * row_sc, (const uint8_t*)M.sc + row * row_sc, segrows * row_sc, bar);
    if (d_bulk) p_bulk(base + d_off + sr * row_d, (const uint8_t*)M.d + row * row_d, segrows * row_d, bar);
  }
}

// Move cursor c to its next tile; false when it must wait (expert ids not
// published yet) or the stage list is exhausted.
__device__ __forceinline__ bool cursor_next(const StepParams& P, const StepStage* stg, Cursor& c, unsigned target) {
  const int nst = P.nstages;
  while (c.s < nst) {
    if (!c.ready) {
      const int type = stg[c.s].type;
      if (!is_ring(type)) {
        c.s++;
        continue;
      }
      if (type == ST_XSWIGLU || type == ST_XDOWN) {
        const unsigned* b = &P.ctl->bar[stg[c.s].dep];
        // relaxed poll (no L1 invalidation), one acquire once it is reached
        if (ld_relaxed(b) < target || ld_acquire(b) < target) return false;
#pragma unroll
        for (int i = 0; i < N_USED; i++) c.sel[i] = __ldcg(&P.ctl->sel[i]);
      }
      tile_range(stg[c.s].ntiles, c.t, c.t1);
      c.ready = 1;
    }
    if (c.t < c.t1) return true;
    c.s++;
    c.ready = 0;
  }
  return false;
}

// Issue every tile the ring and the dependencies allow; never blocks.
__device__ __forceinline__ void prod_poll(const StepParams& P, Cursor& shared_c, uint8_t* ring, uint64_t* full,
                                          uint64_t* empty, unsigned target) {
  const StepStage* stg = stage_table(ring);
  Cursor c = shared_c;  // registers for the duration of the poll
  bool moved = false;
  while (cursor_next(P, stg, c, target)) {
    const int st = c.k % RING, round = c.k / RING;
    if (round > 0 && !p_test(&empty[st], (round - 1) & 1)) break;  // slot still being read
    issue_tile(stg[c.s], c.sel, c.t, ring + st * SLOT, &full[st]);
    c.t++;
    c.k++;
    moved = true;
  }
  if (moved || c.s != shared_c.s || c.ready != shared_c.ready) shared_c = c;
}

// Before an aborting CTA returns, thread 0 waits (time-bounded, ignoring the
// abort flag) for the copies it issued but nobody consumed: the shared memory
// they write must stay allocated until they land.
__device__ void drain(const Cursor& pr, int k, uint64_t* full) {
  for (int j = k; j < pr.k; j++) mbar_wait(&full[j % RING], (j / RING) & 1, nullptr);
}

// Thread 0's waits keep the producer going.
__device__ bool t0_wait_bar(const StepParams& P, Cursor& pr, uint8_t* ring, uint64_t* full, uint64_t* empty, int s,
                            unsigned target) {
  WaitBudget wb;
  for (uint32_t i = 0;; i++) {
    prod_poll(P, pr, ring, full, empty, target);
    if (ld_relaxed(&P.ctl->bar[s]) >= target && ld_acquire(&P.ctl->bar[s]) >= target) return true;
    if ((i & 63u) == 63u && ld_vol(&P.ctl->abort)) return false;
    if ((i & 63u) == 63u && wb.spent()) {
      raise_abort(P.ctl, 2u);
      return false;
    }
  }
}

// Warp 0 waits for a full slot as one converged warp: lane 0 keeps producing,
// and no lane sleeps in a suspending try_wait while the copy it waits for may
// still have to be issued by lane 0 of the same warp.
__device__ bool w0_wait_full(const StepParams& P, Cursor& pr, uint8_t* ring, uint64_t* full, uint64_t* empty,
                             int kk, unsigned target) {
  WaitBudget wb;
  const bool lead = threadIdx.x == 0;
  for (uint32_t i = 0;; i++) {
    if (lead) prod_poll(P, pr, ring, full, empty, target);
    __syncwarp();
    if (__all_sync(0xffffffffu, mbar_test(&full[kk % RING], (kk / RING) & 1))) return true;
    if ((i & 63u) == 63u) {
      int stop = 0;
      if (lead) {
        if (ld_vol(&P.ctl->abort)) stop = 1;
        else if (wb.spent()) {
          raise_abort(P.ctl, 3u);
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

// ------------------------------------------------------------- consumers
// RMS factor of x over DIM (all warps).
__device__ float cons_rms(const float* x, float eps, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < DIM; i += NCW * 32) {
    const float v = ldcg(x + i);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  cons_sync();
  float t = 0.f;
  for (int i = 0; i < NCW; i++) t += red[i];
  cons_sync();
  return 1.0f / sqrtf(t / (float)DIM + eps);
}

// Per-CTA shared state of the consumers. Values that live across a stage's
// tile loop are kept here rather than in registers: the tile loop already
// holds the 64-float activation unit per lane, and 16 warps leave 128
// registers per thread.
struct ConsShared {
  float red[NCW];
  float res[2][24];  // per-tile row results (double-buffered by tile parity)
  float bv[16];      // LMHEAD running argmax of epilogue thread r
  int bi[16];
  int sel[N_USED];   // expert ids / weights of the current routed stage
  float selw[N_USED];
  unsigned long long tw, tc, te, ts;  // trace sums (thread 0)
  int flag;
};

// One weight-ring stage. Returns false on abort.
__device__ bool ring_stage(const StepParams& P, const StepStage& S, int sidx, uint8_t* ring, uint64_t* full,
                           uint64_t* empty, int& k, ConsShared& cs, float* xsm, Cursor& pr, unsigned target) {
  StepCtl* ctl = P.ctl;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nseg = tile_nseg(S.type), segrows = tile_segrows(S.type);
  const int nb = S.W.nb, U = 4 * nb;
  const uint32_t row_q = 48u * U, row_sc = 4u * U, row_d = 2u * nb;
  const uint32_t R = nseg * segrows;
  const uint32_t sc_off = R * row_q, d_off = sc_off + R * row_sc;
  if ((S.type == ST_XSWIGLU || S.type == ST_XDOWN) && threadIdx.x < N_USED) {
    cs.sel[threadIdx.x] = __ldcg(&ctl->sel[threadIdx.x]);
    cs.selw[threadIdx.x] = __ldcg(&ctl->selw[threadIdx.x]);
  }
  if (S.type == ST_LMHEAD && threadIdx.x >= 32 && threadIdx.x < 48) {
    cs.bv[threadIdx.x - 32] = -INFINITY;
    cs.bi[threadIdx.x - 32] = 0x7fffffff;
  }
  // unit owned by this lane and the stage's activation registers
  int u = lane < U ? lane : -1;
  if (S.type == ST_DOWN28) u = lane < 28 ? (warp & 3) * 28 + lane : -1;
  float xr[64];
  {
    // Stage the activations once per CTA (one L2 read of the vector instead of
    // one per warp), RMS-normalising on the way when the stage has a norm.
    const int nvec = S.type == ST_XDOWN ? N_USED : 1;
    const int len = (S.type == ST_XDOWN) ? S.ff : (S.type == ST_DOWN28 ? N_FF : DIM);
    const int Uv = len / 64;
    const int nf4 = nvec * len / 4;
    constexpr int PER = (XS_FLOATS / 4 + NCW * 32 - 1) / (NCW * 32);
    float4 v[PER];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int f = threadIdx.x + i * NCW * 32;
      if (f < nf4) {
        v[i] = __ldcg((const float4*)S.xin + f);
        ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
      }
    }
    float inv = 1.f;
    if (S.norm) {
      ss = warp_sum(ss);
      if (lane == 0) cs.red[warp] = ss;
      cons_sync();
      float t = 0.f;
      for (int i = 0; i < NCW; i++) t += cs.red[i];
      inv = 1.0f / sqrtf(t / (float)DIM + P.eps);
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int f = threadIdx.x + i * NCW * 32;
      if (f < nf4) {
        float4 o = v[i];
        if (S.norm) {
          const float4 g = __ldg((const float4*)S.norm + f);
          o = make_float4(o.x * inv * g.x, o.y * inv * g.y, o.z * inv * g.z, o.w * inv * g.w);
        }
        const int vec = (4 * f) / len, kk = 4 * f - vec * len;
        *(float4*)&xsm[vec * len + xs_index(kk, Uv)] = o;
      }
    }
    cons_sync();
    if (u >= 0) {
      const float* src = xsm + (S.type == ST_XDOWN ? (warp >> 2) * len : 0);
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const float4 q = *(const float4*)&src[(j * Uv + u) * 4];
        xr[4 * j + 0] = q.x;
        xr[4 * j + 1] = q.y;
        xr[4 * j + 2] = q.z;
        xr[4 * j + 3] = q.w;
      }
    }
    cons_sync();  // xsm may be overwritten by the next stage's staging
  }
  if (P.trace && threadIdx.x == 0) P.trace[((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 1] = gtime();
  int t0, t1;
  tile_range(S.ntiles, t0, t1);
  const bool tr = P.trace && threadIdx.x == 0;
  if (tr) cs.tw = cs.tc = cs.te = 0;
  for (int t = t0; t < t1; t++, k++) {
    const int st = k % RING;
    float* res = cs.res[k & 1];
    // residual values this tile adds to, fetched before the compute
    // epilogue thread r = threadIdx.x - 32 (warp 1): warp 0 also produces and
    // should go straight on to the next tile
    const int r = (int)threadIdx.x - 32;
    float rold = 0.f;
    if (S.type == ST_RESID && r >= 0 && r < 16)
      rold = __ldcg(S.resid + t * 16 + r);
    else if ((S.type == ST_XDOWN || S.type == ST_DOWN28) && r >= 0 && r < 4)
      rold = __ldcg(S.resid + t * 4 + r);
    if (tr) cs.ts = clock64();
    const bool ok = warp == 0 ? w0_wait_full(P, pr, ring, full, empty, k, target)
                              : ring_wait(&full[st], (k / RING) & 1, ctl);
    if (tr) {
      const unsigned long long now = clock64();
      cs.tw += now - cs.ts;
      cs.ts = now;
      if (t == t0) P.trace[((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 2] = gtime();
    }
    const uint8_t* base = ring + st * SLOT;
    // this warp's stage rows: one per tile (two for the 24-row conv tile)
    const int srow0 = S.type == ST_DOWN28 ? (warp >> 2) : warp;
    const int nrow = (R > 16 && warp + 16 < (int)R) ? 2 : 1;
    float acc[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; r++) {
      if (!ok || r >= nrow || u < 0) continue;
      const int srow = srow0 + 16 * r;
      const uint4* qp = (const uint4*)(base + srow * row_q) + u;
      const uint4 A = qp[0], B = qp[U], Q = qp[2 * U];
      const uint32_t scw = *(const uint32_t*)(base + sc_off + srow * row_sc + 4 * u);
      float d;
      if (S.type == ST_XDOWN) {
        const size_t row = (size_t)cs.sel[srow >> 2] * DIM + t * 4 + (srow & 3);
        d = __half2float(__ldg(S.W.d + row * nb + (u >> 2)));
      } else {
        d = __half2float(*(const __half*)(base + d_off + srow * row_d + 2 * (u >> 2)));
      }
      acc[r] = q6_unit_dot(A, B, Q, scw, d, xr);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    acc[0] = warp_sum(acc[0]);
    if (R > 16) acc[1] = warp_sum(acc[1]);
    if (lane == 0) {
      res[S.type == ST_DOWN28 ? warp : srow0] = acc[0];
      if (nrow == 2) res[srow0 + 16] = acc[1];
    }
    // CTA-wide barrier that also agrees on an abort, so no thread is left
    // waiting at a later barrier for threads that already returned
    if (__syncthreads_or(!ok)) return false;
    if (tr) {
      const unsigned long long now = clock64();
      cs.tc += now - cs.ts;
      cs.ts = now;
    }
    // ------------------------------------------------------------ epilogues
    if (r >= 0 && r < 16) switch (S.type) {
      case ST_QKV: {
        int row0, ob;
        seg_src(S, cs.sel, t, 0, row0, ob);
        if (r < 16) S.out[ob + row0 + r] = res[r];
        break;
      }
      case ST_RESID:
        if (r < 16) S.resid[t * 16 + r] = rold + res[r];
        break;
      case ST_LMHEAD:
        if (r < 16) {
          const int row = t * 16 + r;
          const float v = res[r];
          S.out[row] = v;
          if (v > cs.bv[r] || (v == cs.bv[r] && row < cs.bi[r])) {
            cs.bv[r] = v;
            cs.bi[r] = row;
          }
        }
        break;
      case ST_CONV:
        if (r < 8) {
          // kernels/resident.rs:33-56; lfm.rs:464-520 for one token
          const int ch = t * 8 + r;
          const float bx = res[r] * res[16 + r];
          const float s0 = S.state[2 * ch], s1 = S.state[2 * ch + 1];
          float conv = 0.f;
          conv += s0 * S.conv_w[3 * ch + 0];
          conv += s1 * S.conv_w[3 * ch + 1];
          conv += bx * S.conv_w[3 * ch + 2];
          S.out[ch] = res[8 + r] * conv;
          S.state[2 * ch] = s1;
          S.state[2 * ch + 1] = bx;
        }
        break;
      case ST_SWIGLU:
        if (r < 8) S.out[t * 8 + r] = res[r] / (1.0f + expf(-res[r])) * res[8 + r];
        break;
      case ST_XSWIGLU:
        if (r < 8) {
          const int per = S.ff / 8, slot = t / per;
          S.out[(size_t)slot * S.ff + (t - slot * per) * 8 + r] = res[r] / (1.0f + expf(-res[r])) * res[8 + r];
        }
        break;
      case ST_XDOWN:
        // rank-ordered combine of the 4 slots (kernels/resident.rs:101-117)
        if (r < 4) {
          float a = 0.f;
#pragma unroll
          for (int s2 = 0; s2 < N_USED; s2++) a += res[s2 * 4 + r] * cs.selw[s2];
          S.resid[t * 4 + r] = rold + a;
        }
        break;
      case ST_DOWN28:
        if (r < 4) S.resid[t * 4 + r] = rold + (((res[4 * r] + res[4 * r + 1]) + res[4 * r + 2]) + res[4 * r + 3]);
        break;
      default:
        break;
    }
    if (tr) cs.te += clock64() - cs.ts;
  }
  if (tr) {
    unsigned long long* rec = P.trace + ((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS;
    rec[4] = cs.tw;
    rec[5] = (unsigned long long)(t1 - t0);
    rec[6] = cs.tc;
    rec[7] = cs.te;
  }
  return true;
}

// Attention task (kv head kh, split) for a 4-warp group g (head = warp & 3).
__device__ void attn_task(const StepParams& P, const StepStage& S, AttnSmem& sm, int g, int kh, int split, int pos,
                          int nact) {
  const int w4 = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31, gt = threadIdx.x & 127;
  constexpr int SPL = ATTN_SPLIT;
  const int t0 = split * SPL;
  const int nsplit = (P.ctx + SPL - 1) / SPL;
  const int h = kh * (HEADS / KV_HEADS) + w4;
  const float2 cs = P.rope[(size_t)pos * 32 + lane];
  const float* qkv = S.xin;
  {
    float q0 = ldcg(qkv + h * HEAD_DIM + lane), q1 = ldcg(qkv + h * HEAD_DIM + lane + 32);
    const float ss = warp_sum(q0 * q0 + q1 * q1);
    const float inv = 1.0f / sqrtf(ss / (float)HEAD_DIM + P.eps);
    q0 *= inv * S.q_norm[lane];
    q1 *= inv * S.q_norm[lane + 32];
    sm.sq[w4][lane] = q0 * cs.x - q1 * cs.y;
    sm.sq[w4][lane + 32] = q0 * cs.y + q1 * cs.x;
  }
  if (pos < t0 + SPL) {
    const size_t off = ((size_t)kh * P.ctx + pos) * HEAD_DIM;
    if (w4 == 0) {
      float k0 = ldcg(qkv + DIM + kh * HEAD_DIM + lane), k1 = ldcg(qkv + DIM + kh * HEAD_DIM + lane + 32);
      const float ss = warp_sum(k0 * k0 + k1 * k1);
      const float inv = 1.0f / sqrtf(ss / (float)HEAD_DIM + P.eps);
      k0 *= inv * S.k_norm[lane];
      k1 *= inv * S.k_norm[lane + 32];
      S.kc[off + lane] = __float2half_rn(k0 * cs.x - k1 * cs.y);
      S.kc[off + lane + 32] = __float2half_rn(k0 * cs.y + k1 * cs.x);
    } else if (w4 == 1) {
      const float* v = qkv + DIM + KV_HEADS * HEAD_DIM + kh * HEAD_DIM;
      S.vc[off + lane] = __float2half_rn(ldcg(v + lane));
      S.vc[off + lane + 32] = __float2half_rn(ldcg(v + lane + 32));
    }
    __threadfence();
  }
  group_sync(g);
  const int tend = min(t0 + SPL, pos + 1), cnt = tend - t0;
  {
    const uint4* kg = (const uint4*)(S.kc + ((size_t)kh * P.ctx + t0) * HEAD_DIM);
    const uint4* vg = (const uint4*)(S.vc + ((size_t)kh * P.ctx + t0) * HEAD_DIM);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int idx = gt + i * 128, r = idx >> 3, c = idx & 7;
      if (r < cnt) {
        *(uint4*)&sm.sk[r][c * 8] = __ldcg(kg + idx);
        *(uint4*)&sm.sv[r][c * 8] = __ldcg(vg + idx);
      }
    }
  }
  group_sync(g);
  float sc = -INFINITY;
  if (lane < cnt) {
    float acc = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < 8; c8++) {
      const uint4 v = *(const uint4*)&sm.sk[lane][c8 * 8];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 f = __half22float2(*(const __half2*)&w[j]);
        acc = fmaf(f.x, sm.sq[w4][c8 * 8 + 2 * j], acc);
        acc = fmaf(f.y, sm.sq[w4][c8 * 8 + 2 * j + 1], acc);
      }
    }
    sc = acc * 0.125f;
  }
  float m = sc;
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float pl = lane < cnt ? expf(sc - m) : 0.f;
  const float l = warp_sum(pl);
  float o0 = 0.f, o1 = 0.f;
  for (int t = 0; t < cnt; t++) {
    const float pt = __shfl_sync(0xffffffffu, pl, t);
    o0 = fmaf(pt, __half2float(sm.sv[t][lane]), o0);
    o1 = fmaf(pt, __half2float(sm.sv[t][lane + 32]), o1);
  }
  float* pp = P.attn_part + (((size_t)kh * nsplit + split) * 4 + w4) * (HEAD_DIM + 2);
  pp[lane] = o0;
  pp[lane + 32] = o1;
  if (lane == 0) {
    pp[64] = m;
    pp[65] = l;
  }
  __threadfence();
  group_sync(g);
  if (gt == 0) {
    __threadfence();
    sm.last = atomicAdd(&P.ctl->attn_cnt[kh], 1u) == (unsigned)(nact - 1);
  }
  group_sync(g);
  if (!sm.last) return;
  __threadfence();
  const float* base = P.attn_part + ((size_t)kh * nsplit * 4 + w4) * (HEAD_DIM + 2);
  float M = -INFINITY;
  for (int sidx = lane; sidx < nact; sidx += 32) M = fmaxf(M, ldcg(base + (size_t)sidx * 4 * (HEAD_DIM + 2) + 64));
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f, O0 = 0.f, O1 = 0.f;
  for (int sidx = 0; sidx < nact; sidx++) {
    const float* q = base + (size_t)sidx * 4 * (HEAD_DIM + 2);
    const float w = expf(ldcg(q + 64) - M);
    L = fmaf(ldcg(q + 65), w, L);
    O0 = fmaf(ldcg(q + lane), w, O0);
    O1 = fmaf(ldcg(q + lane + 32), w, O1);
  }
  S.out[h * HEAD_DIM + lane] = O0 / L;
  S.out[h * HEAD_DIM + lane + 32] = O1 / L;
  __threadfence();
  group_sync(g);
  if (gt == 0) P.ctl->attn_cnt[kh] = 0;
}

// sigmoid top-4 of the 32 router logits (kernels/resident.rs:58-99)
__device__ void route_top4(const float* lg, const float* bias, StepCtl* ctl) {
  const int lane = threadIdx.x & 31;
  const float prob = 1.0f / (1.0f + expf(-lg[lane]));
  float score = prob + bias[lane];
  float ps[N_USED];
  int ids[N_USED];
#pragma unroll
  for (int r = 0; r < N_USED; r++) {
    float best = score;
#pragma unroll
    for (int o = 16; o; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
    const unsigned mk = __ballot_sync(0xffffffffu, score == best);
    const int id = mk ? __ffs(mk) - 1 : 0;
    ps[r] = __shfl_sync(0xffffffffu, prob, id);
    ids[r] = id;
    if (lane == id) score = -INFINITY;
  }
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < N_USED; r++) sum += ps[r];
  sum = fmaxf(sum, 6.103515625e-5f);
  if (lane < N_USED) {
    ctl->sel[lane] = ids[lane];
    ctl->selw[lane] = ps[lane] / sum;
  }
}

__global__ void __launch_bounds__(NT, 1) k_step(StepParams P) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[RING], empty[RING];
  __shared__ StageSmem stsm;
  __shared__ ConsShared cs;
  __shared__ Cursor prod;
  __shared__ float lgs[N_EXPERT];
  StepCtl* ctl = P.ctl;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned G = gridDim.x;
  const unsigned target = (ld_vol(&ctl->epoch) + 1u) * G;

  StepStage* stg = stage_table(ring);
  {
    const unsigned long long* src = (const unsigned long long*)P.stages;
    unsigned long long* dst = (unsigned long long*)stg;
    const int words = P.nstages * (int)(sizeof(StepStage) / 8);
    for (int i = threadIdx.x; i < words; i += NT) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < RING; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prod.s = 0, prod.t = 0, prod.t1 = 0, prod.k = 0, prod.ready = 0;
    prod_poll(P, prod, ring, full, empty, target);  // fill the ring
  }
  __syncthreads();

  const int pos = P.io[1];
  int k = 0;
  for (int s = 0; s < P.nstages; s++) {
    const StepStage& S = stg[s];
    if (s > 0) {
      if (threadIdx.x == 0) cs.flag = t0_wait_bar(P, prod, ring, full, empty, s - 1, target) ? 1 : 0;
      cons_sync();
      if (!cs.flag) {
        if (threadIdx.x == 0) drain(prod, k, full);
        return;
      }
      cons_sync();
    }
    if (P.trace && threadIdx.x == 0) P.trace[((size_t)s * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS] = gtime();
    switch (S.type) {
      case ST_EMBED:
        if (blockIdx.x == 0 && warp == 0) {
          const int tok = P.io[0];
          const int U = 4 * P.embd.nb;
          if (lane < U) {
            // kernels/resident.rs:4-18: one 64-weight unit per lane, written
            // out four values at a time (no 64-float temporary)
            const uint4* qp = P.embd.q + (size_t)tok * 3 * U + lane;
            const uint4 A = qp[0], B = qp[U], Q = qp[2 * U];
            const uint32_t scw = P.embd.sc[(size_t)tok * U + lane];
            const float d = __half2float(P.embd.d[(size_t)tok * P.embd.nb + (lane >> 2)]);
            const uint32_t a[4] = {A.x, A.y, A.z, A.w}, b[4] = {B.x, B.y, B.z, B.w}, q[4] = {Q.x, Q.y, Q.z, Q.w};
            float* xo = P.x + q6_unit_base(lane);
#pragma unroll
            for (int t4 = 0; t4 < 4; t4++) {
              uint32_t w0, w1, w2, w3;
              q6_words(a[t4], b[t4], q[t4], w0, w1, w2, w3);
              const uint32_t wm[4] = {w0, w1, w2, w3};
#pragma unroll
              for (int m = 0; m < 4; m++) {
                const float sm = d * sc_val(scw, m);
                *(float4*)(xo + 32 * m + 4 * t4) = make_float4(sm * q6_val(wm[m], 0), sm * q6_val(wm[m], 1),
                                                               sm * q6_val(wm[m], 2), sm * q6_val(wm[m], 3));
              }
            }
          }
        }
        break;
      case ST_ATTN: {
        const int nact = pos / ATTN_SPLIT + 1;
        const int ntask = KV_HEADS * nact;
        int a0, a1;
        tile_range(ntask, a0, a1);
        // two 4-warp groups (shared memory budget); the other warps idle here
        const int g = warp >> 2;
        if (g < 2)
          for (int a = a0 + g; a < a1; a += 2) attn_task(P, S, stsm.attn[g], g, a / nact, a % nact, pos, nact);
        break;
      }
      case ST_ROUTER:
        if (blockIdx.x < N_EXPERT) {
          const int e = blockIdx.x;
          const float inv = cons_rms(S.xin, P.eps, cs.red);
          const float* w = S.rw + (size_t)e * DIM;
          float a = 0.f;
          for (int i = threadIdx.x; i < DIM; i += NCW * 32)
            a = fmaf(__ldg(w + i), ldcg(S.xin + i) * inv * S.norm[i], a);
          a = warp_sum(a);
          if (lane == 0) cs.red[warp] = a;
          cons_sync();
          if (threadIdx.x == 0) {
            float t = 0.f;
            for (int i = 0; i < NCW; i++) t += cs.red[i];
            ctl->router_lg[e] = t;
            __threadfence();
            cs.flag = atomicAdd(&ctl->router_cnt, 1u) == (unsigned)(N_EXPERT - 1);
          }
          cons_sync();
          if (cs.flag && warp == 0) {
            __threadfence();
            lgs[lane] = ldcg(&ctl->router_lg[lane]);
            __syncwarp();
            route_top4(lgs, S.bias, ctl);
            if (lane == 0) ctl->router_cnt = 0;
          }
        }
        break;
      default:
        if (!ring_stage(P, S, s, ring, full, empty, k, cs, stsm.xs, prod, target)) {
          if (threadIdx.x == 0) drain(prod, k, full);
          return;
        }
    }
    // arrive at this stage's barrier: after the CTA barrier (which orders every
    // thread's global writes before thread 0), thread 0 fences at gpu scope
    // and publishes the CTA's arrival.
    cons_sync();
    if (threadIdx.x == 0) {
      if (S.type == ST_LMHEAD) {
        float cv = cs.bv[0];
        int ci = cs.bi[0];
        for (int w = 1; w < 16; w++)
          if (cs.bv[w] > cv || (cs.bv[w] == cv && cs.bi[w] < ci)) {
            cv = cs.bv[w];
            ci = cs.bi[w];
          }
        ctl->am_part[blockIdx.x] = make_float2(cv, __int_as_float(ci));
      }
      __threadfence();
      if (P.trace) P.trace[((size_t)s * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 3] = gtime();
      const unsigned prev = atomicAdd(&ctl->bar[s], 1u);
      if (s == P.nstages - 1 && prev == target - 1) {
        // last CTA of the step: final argmax (kernels/persistent.rs:12-53)
        __threadfence();
        float cv = -INFINITY;
        int ci = 0x7fffffff;
        for (unsigned c = 0; c < G; c++) {
          const float2 q = __ldcg(&ctl->am_part[c]);
          const int qi = __float_as_int(q.y);
          if (q.x > cv || (q.x == cv && qi < ci)) {
            cv = q.x;
            ci = qi;
          }
        }
        P.io[2] = ci == 0x7fffffff ? 0 : ci;
        __threadfence();
        atomicAdd(&ctl->epoch, 1u);
      }
    }
  }
}

}  // namespace

size_t step_smem_bytes() { return (size_t)RING * SLOT + (size_t)STEP_MAX_STAGES * sizeof(StepStage); }

cudaError_t step_prepare() {
  static cudaError_t status = cudaErrorNotReady;
  if (status == cudaErrorNotReady) {
    cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes());
    cudaFuncSetAttribute(k_step, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    int blocks = 0;
    status = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k_step, NT, step_smem_bytes());
    if (status == cudaSuccess && blocks < 1) status = cudaErrorCooperativeLaunchTooLarge;
  }
  return status;
}

std::string step_occupancy_report() {
  cudaFuncAttributes a = {};
  cudaFuncGetAttributes(&a, k_step);
  int blocks = -1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k_step, NT, step_smem_bytes());
  return "regs " + std::to_string(a.numRegs) + ", static smem " + std::to_string(a.sharedSizeBytes) +
         ", dynamic smem " + std::to_string(step_smem_bytes()) + ", max dynamic " +
         std::to_string(a.maxDynamicSharedSizeBytes) + ", threads " + std::to_string(NT) + ", blocks/SM " +
         std::to_string(blocks);
}

cudaError_t step_launch(const StepParams& p, int sms, cudaStream_t s) {
  cudaError_t e = step_prepare();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = step_smem_bytes();
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_step, p);
}

}  // namespace lfm
