// Persistent batch-1 decode step (sm_100a).
//
// One cooperative launch, one CTA per SM, runs the whole decode token: the
// ~126 dependent stages of the reference's resident graph
// (gpu_lfm/resident_graph.rs:226-546) become a stage list walked in order by
// every CTA. Between dependent stages the CTAs meet at a grid barrier
// (monotonic arrival counters in global memory, acquire/release ordering,
// bounded polling).
//
// Warps 16-19 of each CTA are producers: together they walk this CTA's weight
// tiles of ALL stages in order and stream them through a 4-slot shared-memory
// ring with bulk async copies (cp.async.bulk into this CTA only) completed on
// mbarriers; producer p issues the tiles that land in slot p. A producer
// waits only for its free slot and, before routed-expert tiles, for the
// layer's top-4 experts, which the consumers compute at the start of the
// gate/up stage from the router partials the residual stage publishes (there
// is no router stage). The weight stream of later stages is in flight while
// earlier stages compute and the grid barriers never drain the HBM pipeline.
// One producer per slot, not one for all: issuing a bulk copy whose source
// page misses the address-translation caches holds the issuing thread for
// several hundred cycles, and a decode tile is six copies from six different
// weight pages, so a single issuing thread held the stream near 2 TB/s;
// four issuers overlap those stalls.
//
// Warps 0-15 consume. Each holds the stage's activation unit in registers (one
// 64-weight unit per lane, q6k.cuh layout) and computes one dot row of every
// tile on its own: wait for the tile, dequantise and reduce, release the slot,
// and either finish the row (projection output, residual add, logits and
// argmax) or park the dot in a shared-memory partial buffer, with no CTA-wide
// barrier per tile. Rows that combine several dots (short conv b/c/x, SwiGLU
// gate/up, the rank-ordered expert combine, the dense down projection split in
// quarters) are finished at the end of the stage by the CTA that owns them.
//
// Every wait is bounded (~1 s of SM cycles). A timeout raises the status word
// and an abort flag that releases all other waits; the consumers agree on it
// at the next stage boundary, the producer drains its copies, and the kernel
// returns.
#include <math.h>

#include <mutex>
#include <string>

#include "dev_common.cuh"
#include "step.h"

namespace lfm {
namespace {
using namespace dev;

constexpr int NCW = 16;                // consumer warps
constexpr int NPROD = STEP_PRODUCERS;  // producer warps, one per ring slot
constexpr int NT = (NCW + NPROD) * 32;  // 20 warps x 96 registers fit one SM
constexpr int MAXREG = 96;             // 20 warps: 5 per SM sub-partition x 32 lanes x 96 registers
constexpr int PART_TILES = STEP_PART_TILES;
constexpr int PRODUCER = NCW;          // warp index of the first producer
constexpr int RING = 4;
static_assert(NPROD == RING, "one producer warp per ring slot");
constexpr int SLOT = 40320;            // 24 rows x (1536 + 128 + 16): the largest tile
constexpr int KP = HEAD_DIM + 8;       // padded fp16 K row in shared memory
// 32-position chunks per attention task: at most 32 tasks per kv head, so a
// 4096-token context needs 4 (the loop is unrolled to this bound; a loop
// carrying the group barriers cost the tile loops registers)
constexpr int ATTN_MAX_CPT = 4;
static_assert(ATTN_MAX_CPT * 32 * ATTN_SPLIT >= 4096, "context limit needs more chunks per task");

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
// the routed gate/up stage stages its 2048-float input here, above the router
// partials (G x 33 floats + 33 sums fit below it for G <= 154 CTAs)
constexpr int ROUTE_XOFF = XS_FLOATS - DIM;
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
__device__ __forceinline__ unsigned ld_vol(const unsigned* p) { return *(volatile const unsigned*)p; }
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
// Stage descriptors live in shared memory, after the weight ring.
__device__ __forceinline__ StepStage* stage_table(uint8_t* ring) { return (StepStage*)(ring + RING * SLOT); }

// Barriers among the 256 consumer threads (named barrier 1; the producer warp
// never takes part). Non-aligned form: thread 0 reaches it from its own poll.
__device__ __forceinline__ void cons_sync() { asm volatile("barrier.sync 1, %0;" ::"n"(NCW * 32) : "memory"); }
// ... and the same barrier reducing a predicate: true if any consumer passed true
__device__ __forceinline__ bool cons_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n barrier.red.or.pred po, 1, %2, pi;\n selp.u32 %0, 1, 0, po;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCW * 32)
      : "memory");
  return r != 0;
}
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

// Bounded wait for a grid barrier counter (acquire polls: the load that sees
// the target already orders everything after it).
__device__ bool counter_wait(const unsigned* c, unsigned target, StepCtl* ctl, unsigned code) {
  WaitBudget wb;
  for (uint32_t i = 0;; i++) {
    if (ld_acquire(c) >= target) return true;
    if ((i & 15u) == 15u) {
      if (ld_vol(&ctl->abort)) return false;
      if (wb.spent()) {
        raise_abort(ctl, code);
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
// Producer-side forms of the mbarrier / bulk-copy instructions without a
// compiler memory clobber: the producer reads nothing these order.
__device__ __forceinline__ void p_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes));
}
__device__ __forceinline__ void p_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar)));
}

// Copy tile t of stage S into the ring slot at `base`.
__device__ __forceinline__ void issue_tile(const StepStage& S, const int* sel, int t, uint8_t* base, uint64_t* bar) {
  const int type = S.type;
  const int nseg = tile_nseg(type), segrows = tile_segrows(type);
  const int nb = S.W.nb, U = 4 * nb;
  const uint32_t row_q = 48u * U, row_sc = 4u * U, row_d = 2u * nb;
  const bool d_bulk = type != ST_XDOWN;  // 7-block rows: 14-byte d rows are read by the consumers
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

// Shared state of the consumers (and the producer's routing hand-off).
struct ConsShared {
  uint64_t route_bar;  // consumers -> producer: the current MoE layer's routing is in psel/pselw
  float red[NCW];
  float bv[NCW];     // LMHEAD argmax per consumer warp
  int bi[NCW];
  int psel[N_USED];  // expert ids / weights of the current MoE layer (producer -> consumers)
  float pselw[N_USED];
  int flag;
  unsigned long long tw, tc, ts;  // trace sums of consumer warp 0 (thread 0 only)
  float part[PART_TILES * 24];  // dot results [local tile][tile row] finished at stage end
};

// Routing of one MoE layer from the per-CTA router partials that the
// preceding residual stage published (see ring_stage<ST_RESID>): logit_e =
// (1/rms(x)) * sum_c part[c][e], summed over CTAs in a fixed order so that
// every CTA selects the same experts; then the sigmoid top-4 of
// kernels/resident.rs:58-99 (prob + bias ranks, first index wins ties,
// weights renormalised with the 6.103515625e-5 clamp). Run by the 16 consumer
// warps at the start of the expert gate/up stage; `buf` is scratch shared
// memory of at least G * 33 floats. The result goes to cs.psel / cs.pselw and
// the producer is released through cs.route_bar.
// Returns, to every consumer thread, the layer input's sum of squares (the
// 1/rms of both the router and the FFN input).
__device__ float route_layer(const StepParams& P, const float* bias, ConsShared& cs, float* buf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the expert bias is read long before the selection needs it (a global
  // load issued at the selection put its latency on the routing's path)
  const float bias_l = warp == 0 ? __ldg(bias + lane) : 0.f;
  const StepCtl* ctl = P.ctl;
  const int G = gridDim.x;
  constexpr int W = N_EXPERT + 1;
  // one round of loads: the G x 33 partials into shared memory (all of a
  // thread's loads issued before the first store)
  const float* src = &ctl->rpart[0][0];
  constexpr int RP = (STEP_MAX_CTAS * W + NCW * 32 - 1) / (NCW * 32);
  float rv[RP];
#pragma unroll
  for (int i = 0; i < RP; i++) {
    const int f = threadIdx.x + i * NCW * 32;
    rv[i] = f < G * W ? __ldcg(src + f) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < RP; i++) {
    const int f = threadIdx.x + i * NCW * 32;
    if (f < G * W) buf[f] = rv[i];
  }
  cons_sync();
  // column sums in a fixed order: lane l adds CTAs l, l+32, ... then a fixed
  // butterfly across the warp; warp w handles columns w, w+16 (and warp 0
  // column 32), the columns' chains interleaved
  static_assert(W == 2 * NCW + 1, "33 columns over 16 warps");
  {
    const bool third = warp == 0;
    float v0 = 0.f, v1 = 0.f, v2 = 0.f;
    for (int c = lane; c < G; c += 32) {
      v0 += buf[c * W + warp];
      v1 += buf[c * W + warp + NCW];
      if (third) v2 += buf[c * W + 2 * NCW];
    }
    v0 = warp_sum(v0);
    v1 = warp_sum(v1);
    if (third) v2 = warp_sum(v2);
    if (lane == 0) {
      buf[G * W + warp] = v0;
      buf[G * W + warp + NCW] = v1;
      if (third) buf[G * W + 2 * NCW] = v2;
    }
  }
  cons_sync();
  if (warp == 0) {
    const float ss = buf[G * W + N_EXPERT];
    const float inv = 1.0f / sqrtf(ss / (float)DIM + P.eps);
    const float prob = 1.0f / (1.0f + expf(-(buf[G * W + lane] * inv)));
    // rank of this expert among the 32 (higher score first, lower index first
    // among equal scores; a NaN score ranks last): the same order as picking
    // the maximum four times, in one round of independent shuffles
    const float s0 = prob + bias_l;
    const float score = s0 == s0 ? s0 : -INFINITY;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const float o = __shfl_sync(0xffffffffu, score, j);
      rank += (o > score || (o == score && j < lane)) ? 1 : 0;
    }
    float ps[N_USED];
    int ids[N_USED];
#pragma unroll
    for (int r = 0; r < N_USED; r++) {
      const unsigned mk = __ballot_sync(0xffffffffu, rank == r);  // the ranks are a permutation
      ids[r] = __ffs(mk) - 1;
      ps[r] = __shfl_sync(0xffffffffu, prob, ids[r]);
    }
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < N_USED; r++) sum += ps[r];
    sum = fmaxf(sum, 6.103515625e-5f);
#pragma unroll
    for (int r = 0; r < N_USED; r++)
      if (lane == r) {
        cs.psel[r] = ids[r];
        cs.pselw[r] = ps[r] / sum;
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&cs.route_bar);  // release: psel/pselw are written
  }
  // read by every consumer after the column-sum barrier; warp 0 may still be
  // selecting experts from buf[G * W ...] when the caller stages its
  // activation (above ROUTE_XOFF, clear of the partials)
  return buf[G * W + N_EXPERT];
}

// Producer warp p: walks all ring tiles of this CTA in stage order and issues
// those that land in ring slot p (global tile index k with k % RING == p;
// lane 0 issues). Returns the global index of the last tile it issued (-1
// if none); on abort it stops early.
//
// Every producer waits for each MoE layer's routing (one phase of
// cs.route_bar per layer, observed by parity). That stays in step because
// every producer has a tile in every routed gate/up stage (at least RING
// consecutive tiles per CTA, checked when the stage list is built), so the
// consumers cannot publish the next layer's routing before each producer has
// passed this one.
__device__ int producer(const StepParams& P, const StepStage* stg, uint8_t* ring, uint64_t* full, uint64_t* empty,
                        ConsShared& cs, int p) {
  StepCtl* ctl = P.ctl;
  const int lane = threadIdx.x & 31;
  int k = 0, last = -1;
  int sel[N_USED] = {0, 0, 0, 0};
  int routed = -1;  // residual stage whose routing `sel` holds
  uint32_t rphase = 0;
  for (int s = 0; s < P.nstages; s++) {
    const StepStage& S = stg[s];
    const int type = S.type;
    if (!is_ring(type)) continue;
    if ((type == ST_XSWIGLU || type == ST_XDOWN) && S.dep != routed) {
      // the consumers compute this layer's routing at the start of its gate/up
      // stage and release cs.route_bar (one phase per MoE layer)
      int ok = 1;
      if (lane == 0) ok = ring_wait(&cs.route_bar, rphase, ctl) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) return last;
#pragma unroll
      for (int i = 0; i < N_USED; i++) sel[i] = cs.psel[i];
      rphase ^= 1u;
      routed = S.dep;
    }
    int t0, t1;
    tile_range(S.ntiles, t0, t1);
    for (int t = t0; t < t1; t++, k++) {
      const int st = k % RING, round = k / RING;
      if (st != p) continue;
      int ok = 1;
      if (lane == 0 && round > 0) ok = ring_wait(&empty[st], (round - 1) & 1, ctl) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) return last;
      if (lane == 0) issue_tile(S, sel, t, ring + st * SLOT, &full[st]);
      last = k;
      __syncwarp();
    }
  }
  return last;
}

// ------------------------------------------------------------- consumers
// Stage the activation vector(s) of a ring stage into shared memory (RMS
// normalised when the stage has a norm) and load this lane's unit into xr.
template <int TYPE>
__device__ __forceinline__ void stage_x(const StepParams& P, const StepStage& S, ConsShared& cs, float* xsm, float* xr,
                                        int u, int vec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NVEC = TYPE == ST_XDOWN ? N_USED : 1;
  constexpr int LEN = TYPE == ST_XDOWN ? EXPERT_FF : (TYPE == ST_DOWN28 ? N_FF : DIM);
  constexpr int UV = LEN / 64;
  constexpr int NF4 = NVEC * LEN / 4;
  constexpr int PER = (NF4 + NCW * 32 - 1) / (NCW * 32);
  // stages whose input is RMS-normalised (the others read a gated / SwiGLU /
  // attention vector as it is)
  constexpr bool NORM = TYPE == ST_QKV || TYPE == ST_CONV || TYPE == ST_SWIGLU || TYPE == ST_XSWIGLU ||
                        TYPE == ST_LMHEAD;
  if (NORM) {
    static_assert(!NORM || PER == 1, "normalised inputs are DIM long");
    const int f = threadIdx.x;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f), g = v;
    if (f < NF4) {
      // both loads in flight together: one L2 round trip, not two
      v = __ldcg((const float4*)S.xin + f);
      g = __ldg((const float4*)S.norm + f);
    }
    float ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, v.w * v.w)));
    ss = warp_sum(ss);
    if (lane == 0) cs.red[warp] = ss;
    cons_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; i++) t += cs.red[i];
    const float inv = 1.0f / sqrtf(t / (float)DIM + P.eps);
    if (f < NF4) {
      v = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
      *(float4*)&xsm[xs_index(4 * f, UV)] = v;
    }
  } else {
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int f = threadIdx.x + i * NCW * 32;
      if (f < NF4) {
        const float4 v = __ldcg((const float4*)S.xin + f);
        const int vv = (4 * f) / LEN, kk = 4 * f - vv * LEN;
        *(float4*)&xsm[vv * LEN + xs_index(kk, UV)] = v;
      }
    }
  }
  cons_sync();
  {
    const float* src = xsm + vec * LEN;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float4 q = *(const float4*)&src[(j * UV + u) * 4];
      xr[4 * j + 0] = q.x;
      xr[4 * j + 1] = q.y;
      xr[4 * j + 2] = q.z;
      xr[4 * j + 3] = q.w;
    }
  }
  // no barrier here: xsm is next written after the barrier that closes the
  // stage's tile loop (cons_sync_or) or the next stage's opening barrier
}

// One weight-ring stage on the consumer side. Returns false on abort (agreed
// by all consumer threads). Warp w computes tile row(s):
//   QKV / RESID / LMHEAD : 16-row tiles, row w (finished at once)
//   CONV                 : 8 channels x (b, c, x) = 24 rows, rows w and w+16 (w < 8)
//   SWIGLU / XSWIGLU     : 8 gate rows then 8 up rows, row w
//   XDOWN                : 4 experts x 4 output rows, row w (expert w/4)
//   DOWN28               : 4 rows x 7168 = 4 quarters of 28 units; quarter w%4 of row w/4
// Not inlined: one kernel body holding all eight instantiations needs more
// registers than a thread has with 20 warps per SM; as separate functions
// each tile loop is allocated on its own.
template <int TYPE>
__device__ __noinline__ bool ring_stage(const StepParams& P, const StepStage& S, int sidx, uint8_t* ring,
                                        uint64_t* full, uint64_t* empty, int& k, ConsShared& cs, float* xsm) {
  StepCtl* ctl = P.ctl;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NSEG = TYPE == ST_CONV ? 3 : (TYPE == ST_SWIGLU || TYPE == ST_XSWIGLU) ? 2 : TYPE == ST_XDOWN ? 4 : 1;
  constexpr int SEGROWS = (TYPE == ST_CONV || TYPE == ST_SWIGLU || TYPE == ST_XSWIGLU) ? 8
                          : (TYPE == ST_XDOWN || TYPE == ST_DOWN28)                 ? 4
                                                                                    : 16;
  constexpr int R = NSEG * SEGROWS;
  constexpr int NB = TYPE == ST_XDOWN ? 7 : TYPE == ST_DOWN28 ? 28 : 8;
  constexpr int U = 4 * NB;
  constexpr uint32_t ROW_Q = 48u * U, ROW_SC = 4u * U, ROW_D = 2u * NB;
  constexpr uint32_t SC_OFF = R * ROW_Q, D_OFF = SC_OFF + R * ROW_SC;
  constexpr bool PARTIAL = TYPE == ST_CONV || TYPE == ST_SWIGLU || TYPE == ST_XSWIGLU || TYPE == ST_XDOWN ||
                           TYPE == ST_DOWN28;
  // this lane's unit and the warp's x vector. Rows of 28 units leave lanes
  // 28-31 idle: they compute a duplicate unit whose dot is dropped (branch-free
  // code keeps the tile loop within the register budget)
  constexpr int UL = TYPE == ST_DOWN28 ? 28 : (U < 32 ? U : 32);
  const bool live = lane < UL;
  const int u = (TYPE == ST_DOWN28 ? (warp & 3) * 28 : 0) + (live ? lane : lane - UL);
  const int vec = TYPE == ST_XDOWN ? warp >> 2 : 0;
  float xr[64];
  if (TYPE == ST_XSWIGLU) {
    // The FFN input's loads go out before the routing (one L2 round trip for
    // both), and its RMS factor is the routing's sum of squares (the same
    // vector), so the staging needs no reduction of its own.
    const float4 v = __ldcg((const float4*)S.xin + threadIdx.x);
    const float4 g = __ldg((const float4*)S.norm + threadIdx.x);
    const float ss = route_layer(P, stage_table(ring)[S.dep].bias, cs, xsm);
    const float inv = 1.0f / sqrtf(ss / (float)DIM + P.eps);
    if ((int)gridDim.x * (N_EXPERT + 1) + N_EXPERT + 1 > ROUTE_XOFF) cons_sync();  // partials reach the staging
    float* xst = xsm + ROUTE_XOFF;
    *(float4*)&xst[xs_index(4 * threadIdx.x, DIM / 64)] =
        make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
    cons_sync();
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float4 q = *(const float4*)&xst[(j * (DIM / 64) + u) * 4];
      xr[4 * j + 0] = q.x;
      xr[4 * j + 1] = q.y;
      xr[4 * j + 2] = q.z;
      xr[4 * j + 3] = q.w;
    }
    // no barrier here: xsm is next written after the stage's closing barrier
  } else {
    stage_x<TYPE>(P, S, cs, xsm, xr, u, vec);
  }
  const bool tr = P.trace && threadIdx.x == 0;
  if (tr) P.trace[((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 1] = gtime();
  // tile rows of this warp (DOWN28: row w/4 of the tile in the smem row order)
  const int nrow = (TYPE == ST_CONV && warp < 8) ? 2 : 1;
  const int srow0 = TYPE == ST_DOWN28 ? (warp >> 2) : warp;
  int t0, t1;
  tile_range(S.ntiles, t0, t1);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  bool ok = true;
  if (tr) cs.tw = cs.tc = 0;
  for (int t = t0; t < t1; t++, k++) {
    const int st = k % RING;
    // the residual row this warp adds its dot to, loaded before the tile wait
    const float rold = (TYPE == ST_RESID && lane == 0) ? S.resid[t * 16 + warp] : 0.f;
    if (tr) cs.ts = clock64();
    if (!ring_wait(&full[st], (k / RING) & 1, ctl)) {
      ok = false;
      break;
    }
    if (tr) {
      const unsigned long long now = clock64();
      cs.tw += now - cs.ts;
      cs.ts = now;
      if (t == t0) P.trace[((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 2] = gtime();
    }
    const uint8_t* base = ring + st * SLOT;
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1
    for (int r = 0; r < nrow; r++) {
      const int sr = srow0 + 16 * r;
      float a;
      {
        const uint4* qp = (const uint4*)(base + sr * ROW_Q) + u;
        const uint4 A = qp[0], B = qp[U], Q = qp[2 * U];
        const uint32_t scw = *(const uint32_t*)(base + SC_OFF + sr * ROW_SC + 4 * u);
        float d;
        if (TYPE == ST_XDOWN) {
          const size_t row = (size_t)cs.psel[sr >> 2] * DIM + t * 4 + (sr & 3);
          d = __half2float(__ldg(S.W.d + row * NB + (u >> 2)));
        } else {
          d = __half2float(*(const __half*)(base + D_OFF + sr * ROW_D + 2 * (u >> 2)));
        }
        a = q6_unit_dot(A, B, Q, scw, d, xr);
        if (!live) a = 0.f;
      }
      if (r == 0) acc0 = a;
      else acc1 = a;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    acc0 = warp_sum(acc0);
    if (TYPE == ST_CONV) acc1 = warp_sum(acc1);
    if (lane == 0) {
      if (TYPE == ST_QKV) {
        int row0, ob;
        seg_src(S, cs.psel, t, 0, row0, ob);
        S.out[ob + row0 + warp] = acc0;
      } else if (TYPE == ST_RESID) {
        S.resid[t * 16 + warp] = rold + acc0;  // this warp owns the row
      } else if (TYPE == ST_LMHEAD) {
        const int row = t * 16 + warp;
        S.out[row] = acc0;
        if (am_better(acc0, row, bv, bi)) {
          bv = acc0;
          bi = row;
        }
      } else if (TYPE == ST_DOWN28) {
        cs.part[(t - t0) * 16 + (warp & 3) * 4 + (warp >> 2)] = acc0;  // [quarter][row]
      } else if (PARTIAL) {
        cs.part[(t - t0) * R + srow0] = acc0;
        if (TYPE == ST_CONV && nrow == 2) cs.part[(t - t0) * R + srow0 + 16] = acc1;
      }
    }
    if (tr) cs.tc += clock64() - cs.ts;
  }
  if (TYPE == ST_LMHEAD && lane == 0) {
    cs.bv[warp] = bv;
    cs.bi[warp] = bi;
  }
  // all consumers agree on an abort (and see each other's partials) before
  // the stage is finished
  if (cons_sync_or(!ok)) return false;
  if (TYPE == ST_RESID && S.rw != nullptr) {
    // Router partials of the MoE layer that follows (its rmsnorm input is the
    // residual this stage just finished): for the rows this CTA owns,
    // sum_r W_router[e][r] * g[r] * x[r] per expert e and sum_r x[r]^2. The
    // 1/rms factor is applied when the partials are reduced (route_layer).
    // S.norm / S.rw / S.bias hold the FFN norm and router of that layer.
    float a = 0.f, ss = 0.f;
    for (int r = t0 * 16 + warp; r < t1 * 16; r += NCW) {
      const float xv = __ldcg(S.resid + r);
      a = fmaf(__ldg(S.rw + (size_t)lane * DIM + r), xv * __ldg(S.norm + r), a);
      ss = fmaf(xv, xv, ss);
    }
    xsm[warp * (N_EXPERT + 1) + lane] = a;
    if (lane == 0) xsm[warp * (N_EXPERT + 1) + N_EXPERT] = ss;
    cons_sync();
    if (threadIdx.x <= N_EXPERT) {
      float t = 0.f;
      for (int w = 0; w < NCW; w++) t += xsm[w * (N_EXPERT + 1) + threadIdx.x];
      ctl->rpart[blockIdx.x][threadIdx.x] = t;
    }
  }
  if (PARTIAL) {
    const int nt = t1 - t0;
    if (TYPE == ST_CONV) {
      // kernels/resident.rs:33-56; lfm.rs:464-520 for one token
      for (int i = threadIdx.x; i < nt * 8; i += NCW * 32) {
        const int lt = i >> 3, r = i & 7, ch = (t0 + lt) * 8 + r;
        const float* pp = cs.part + lt * R;
        const float bx = pp[r] * pp[16 + r];
        const float s0 = S.state[2 * ch], s1 = S.state[2 * ch + 1];
        float conv = 0.f;
        conv += s0 * S.conv_w[3 * ch + 0];
        conv += s1 * S.conv_w[3 * ch + 1];
        conv += bx * S.conv_w[3 * ch + 2];
        S.out[ch] = pp[8 + r] * conv;
        S.state[2 * ch] = s1;
        S.state[2 * ch + 1] = bx;
      }
    } else if (TYPE == ST_SWIGLU || TYPE == ST_XSWIGLU) {
      for (int i = threadIdx.x; i < nt * 8; i += NCW * 32) {
        const int lt = i >> 3, r = i & 7, t = t0 + lt;
        const float v = silu_mul(cs.part[lt * R + r], cs.part[lt * R + 8 + r]);
        if (TYPE == ST_SWIGLU) {
          S.out[t * 8 + r] = v;
        } else {
          const int per = S.ff / 8, slot = t / per;
          S.out[(size_t)slot * S.ff + (t - slot * per) * 8 + r] = v;
        }
      }
    } else {
      // XDOWN: rank-ordered expert combine (kernels/resident.rs:101-117);
      // DOWN28: the four quarters of the 7168-wide row in order
      for (int i = threadIdx.x; i < nt * 4; i += NCW * 32) {
        const int lt = i >> 2, r = i & 3;
        const float* pp = cs.part + lt * 16;
        float a;
        if (TYPE == ST_XDOWN) {
          a = 0.f;
#pragma unroll
          for (int s2 = 0; s2 < N_USED; s2++) a += pp[s2 * 4 + r] * cs.pselw[s2];
        } else {
          a = ((pp[r] + pp[4 + r]) + pp[8 + r]) + pp[12 + r];
        }
        S.resid[(t0 + lt) * 4 + r] += a;
      }
    }
  }
  if (tr) {
    unsigned long long* rec = P.trace + ((size_t)sidx * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS;
    rec[4] = cs.tw;
    rec[5] = (unsigned long long)(t1 - t0);
    rec[6] = cs.tc;
    rec[7] = 0;
  }
  return true;
}

// Attention task (kv head kh, task j of ntask) for a 4-warp group g (head =
// warp & 3): chunks [c0, c1) of 32 positions with an online softmax, the next
// chunk's K/V rows loaded into registers while this one is computed. The
// partial (unnormalised o, running max m, sum l) goes to attn_part; the last
// task of the kv head to finish merges the head's ntask partials (lane-parallel
// statistics, batched loads). Same math as engine/src/lfm.rs:396-433 (scores
// * 1/sqrt(64), softmax over positions 0..=pos, weighted V) with fp32 sums in
// chunk order instead of f64 sums in position order.
__device__ __noinline__ void attn_task(const StepParams& P, const StepStage& S, AttnSmem& sm, int g, int kh, int j,
                                       int ntask, int cpt, int pos) {
  const int w4 = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31, gt = threadIdx.x & 127;
  constexpr int SPL = ATTN_SPLIT;
  constexpr int PSTR = 4 * (HEAD_DIM + 2);  // floats between one head's partials of consecutive tasks
  const int nchunk = pos / SPL + 1;
  const int c0 = j * cpt, c1 = min(c0 + cpt, nchunk);
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
  if (c1 == nchunk) {
    // this task reads the current position: write its K (normed, roped) and V
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
  const uint4* kg = (const uint4*)(S.kc + (size_t)kh * P.ctx * HEAD_DIM);
  const uint4* vg = (const uint4*)(S.vc + (size_t)kh * P.ctx * HEAD_DIM);
  // K/V rows of a chunk: 32 rows x 8 uint4 each, two per thread
  uint4 kr[2], vr[2];
  auto fetch = [&](int c) {
    const int cnt = min(SPL, pos + 1 - c * SPL);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int idx = gt + i * 128, r = idx >> 3;
      if (r < cnt) {
        kr[i] = __ldcg(kg + (size_t)c * SPL * 8 + idx);
        vr[i] = __ldcg(vg + (size_t)c * SPL * 8 + idx);
      }
    }
  };
  fetch(c0);
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
  for (int ci = 0; ci < ATTN_MAX_CPT; ci++) {
    const int c = c0 + ci;
    if (c >= c1) break;
    const int cnt = min(SPL, pos + 1 - c * SPL);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int idx = gt + i * 128, r = idx >> 3, cc = idx & 7;
      if (r < cnt) {
        *(uint4*)&sm.sk[r][cc * 8] = kr[i];
        *(uint4*)&sm.sv[r][cc * 8] = vr[i];
      }
    }
    if (c + 1 < c1) fetch(c + 1);
    group_sync(g);
    float sc = -INFINITY;
    if (lane < cnt) {
      float acc = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; c8++) {
        const uint4 v = *(const uint4*)&sm.sk[lane][c8 * 8];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float2 f = __half22float2(*(const __half2*)&w[q]);
          acc = fmaf(f.x, sm.sq[w4][c8 * 8 + 2 * q], acc);
          acc = fmaf(f.y, sm.sq[w4][c8 * 8 + 2 * q + 1], acc);
        }
      }
      sc = acc * 0.125f;
    }
    float cm = sc;
#pragma unroll
    for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float mn = fmaxf(m, cm);
    const float scale = expf(m - mn);  // 0 on the first chunk (m = -inf, mn finite)
    const float pl = lane < cnt ? expf(sc - mn) : 0.f;
    l = fmaf(l, scale, warp_sum(pl));
    o0 *= scale;
    o1 *= scale;
    for (int t = 0; t < cnt; t++) {
      const float pt = __shfl_sync(0xffffffffu, pl, t);
      o0 = fmaf(pt, __half2float(sm.sv[t][lane]), o0);
      o1 = fmaf(pt, __half2float(sm.sv[t][lane + 32]), o1);
    }
    m = mn;
    group_sync(g);  // the chunk's rows are read before the next chunk overwrites them
  }
  float* pp = P.attn_part + (((size_t)kh * nsplit + j) * 4 + w4) * (HEAD_DIM + 2);
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
    sm.last = atomicAdd(&P.ctl->attn_cnt[kh], 1u) == (unsigned)(ntask - 1);
  }
  group_sync(g);
  if (!sm.last) return;
  __threadfence();
  // merge: lane s holds task s's statistics (ntask <= 32)
  const float* base = P.attn_part + ((size_t)kh * nsplit * 4 + w4) * (HEAD_DIM + 2);
  float ms = -INFINITY, ls = 0.f;
  if (lane < ntask) {
    ms = ldcg(base + (size_t)lane * PSTR + 64);
    ls = ldcg(base + (size_t)lane * PSTR + 65);
  }
  float M = ms;
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float ws = lane < ntask ? expf(ms - M) : 0.f;
  const float L = warp_sum(ls * ws);
  float O0 = 0.f, O1 = 0.f;
  for (int s0 = 0; s0 < ntask; s0 += 8) {
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const bool in = s0 + i < ntask;
      a[i] = in ? ldcg(base + (size_t)(s0 + i) * PSTR + lane) : 0.f;
      b[i] = in ? ldcg(base + (size_t)(s0 + i) * PSTR + lane + 32) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float w = __shfl_sync(0xffffffffu, ws, (s0 + i) & 31);
      O0 = fmaf(a[i], w, O0);
      O1 = fmaf(b[i], w, O1);
    }
  }
  S.out[h * HEAD_DIM + lane] = O0 / L;
  S.out[h * HEAD_DIM + lane + 32] = O1 / L;
  __threadfence();
  group_sync(g);
  if (gt == 0) P.ctl->attn_cnt[kh] = 0;
}

__global__ void __maxnreg__(MAXREG) k_step(StepParams P) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[RING], empty[RING];
  __shared__ StageSmem stsm;
  __shared__ ConsShared cs;
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
  if (threadIdx.x == 0) {
    for (int s = 0; s < RING; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    mbar_init(&cs.route_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp >= PRODUCER) {
    const int last = producer(P, stg, ring, full, empty, cs, warp - PRODUCER);
    // every issued copy must land before the CTA may exit (bounded waits,
    // regardless of the abort flag): the slot's earlier tiles were consumed
    // before it was reused, so only the last one can be in flight
    if (lane == 0 && last >= 0) mbar_wait(&full[last % RING], (last / RING) & 1, nullptr);
    return;
  }

  const int pos = P.io[1];
  int k = 0;
  for (int s = 0; s < P.nstages; s++) {
    const StepStage& S = stg[s];
    if (s > 0) {
      if (threadIdx.x == 0) cs.flag = counter_wait(&ctl->bar[s - 1], target, ctl, 2u) ? 1 : 0;
      cons_sync();
      if (!cs.flag) return;
    }
    if (P.trace && threadIdx.x == 0) P.trace[((size_t)s * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS] = gtime();
    bool ok = true;
    switch (S.type) {
      case ST_EMBED:
        if (blockIdx.x == 0 && warp == 0) {
          int tok = P.io[0];
          // a device-side id outside the table raises the status word and
          // reads row 0 instead
          if ((unsigned)tok >= (unsigned)P.embd.rows) {
            if (lane == 0) atomicExch(&ctl->err, 4u);
            tok = 0;
          }
          const int U = 4 * P.embd.nb;
          if (lane < U) {
            // kernels/resident.rs:4-18: one 64-weight unit per lane, written
            // out four values at a time
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
        // at most 32 tasks per kv head (one merge statistic per lane), each
        // covering cpt consecutive 32-position chunks
        const int nchunk = pos / ATTN_SPLIT + 1;
        const int cpt = (nchunk + 31) / 32;
        const int nth = (nchunk + cpt - 1) / cpt;
        const int ntask = KV_HEADS * nth;
        int a0, a1;
        tile_range(ntask, a0, a1);
        // two 4-warp groups (shared memory budget); the other warps idle here
        const int g = warp >> 2;
        if (g < 2)
          for (int a = a0 + g; a < a1; a += 2) attn_task(P, S, stsm.attn[g], g, a / nth, a % nth, nth, cpt, pos);
        break;
      }
      case ST_QKV: ok = ring_stage<ST_QKV>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_RESID: ok = ring_stage<ST_RESID>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_CONV: ok = ring_stage<ST_CONV>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_SWIGLU: ok = ring_stage<ST_SWIGLU>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_DOWN28: ok = ring_stage<ST_DOWN28>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_XSWIGLU: ok = ring_stage<ST_XSWIGLU>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_XDOWN: ok = ring_stage<ST_XDOWN>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      case ST_LMHEAD: ok = ring_stage<ST_LMHEAD>(P, S, s, ring, full, empty, k, cs, stsm.xs); break;
      default: break;
    }
    if (!ok) return;
    // arrive at this stage's barrier: after the consumer barrier (which orders
    // every consumer's global writes before thread 0), thread 0 fences at gpu
    // scope and publishes the CTA's arrival.
    cons_sync();
    if (threadIdx.x == 0) {
      if (S.type == ST_LMHEAD) {
        float cv = cs.bv[0];
        int ci = cs.bi[0];
        for (int w = 1; w < NCW; w++)
          if (am_better(cs.bv[w], cs.bi[w], cv, ci)) {
            cv = cs.bv[w];
            ci = cs.bi[w];
          }
        ctl->am_part[blockIdx.x] = make_float2(cv, __int_as_float(ci));
      }
      if (P.trace) P.trace[((size_t)s * gridDim.x + blockIdx.x) * STEP_TRACE_FIELDS + 3] = gtime();
      // release at gpu scope: every consumer's writes are ordered before this
      // thread by the consumer barrier above
      unsigned prev;
      asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&ctl->bar[s]) : "memory");
      if (s == P.nstages - 1 && prev == target - 1) {
        // last CTA of the step: final argmax (kernels/persistent.rs:12-53)
        __threadfence();
        float cv = -INFINITY;
        int ci = 0x7fffffff;
        for (unsigned c = 0; c < G; c++) {
          const float2 q = __ldcg(&ctl->am_part[c]);
          const int qi = __float_as_int(q.y);
          if (am_better(q.x, qi, cv, ci)) {
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
  // kernel attributes and the residency check, once per device
  static std::mutex mu;
  static cudaError_t status[64];
  static unsigned long long known = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!((known >> dev) & 1ull)) {
    cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes());
    cudaFuncSetAttribute(k_step, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    int blocks = 0;
    cudaError_t st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k_step, NT, step_smem_bytes());
    if (st == cudaSuccess && blocks < 1) st = cudaErrorCooperativeLaunchTooLarge;
    status[dev] = st;
    known |= 1ull << dev;
  }
  return status[dev];
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
