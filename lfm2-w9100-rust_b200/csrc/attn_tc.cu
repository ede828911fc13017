// Causal GQA prompt attention on the tensor cores (tcgen05 / TMEM, sm_100a).
//
// Same contract as the reference's prompt attention (lfm.rs:395-437; GPU
// kernel kernels.rs:672-763): for token j at position start + j and query
// head h (KV head h / 4), out = softmax(q . K[0..pos] / 8) . V[0..pos] over
// the fp16 K/V cache. One CTA takes 32 consecutive tokens of the 4 query heads
// that share one KV head: 128 rows, row r = 32 * (head % 4) + token, so the
// rows of one head are one TMEM lane quarter. It walks the key positions in
// tiles of 128:
//   warp 0     TMA: K and V tiles (128 positions x 64 values, 128-byte
//              swizzle) into a 2-slot ring
//   warp 1     TMEM (512 columns) and the MMAs:
//              S = Qhi K^T + Qlo K^T      (M=128, N=128, two S buffers)
//              O_t = Phi V + Plo V       (M=128, N=64, V MN-major, two buffers)
//   warps 2-9  softmax: each row is shared by two warps of the same TMEM lane
//              quarter, one per half of the S tile's 64-column halves (and
//              of the output's 32-column halves): q -> fp16 hi/lo operand
//              (scaled by 1/8); per tile two passes over the thread's 64 S
//              values in TMEM (max, combined with the partner warp through
//              shared memory; then p = exp(s - m) written as an fp16 hi/lo
//              pair, the A operand of P.V, into one of two P buffers); the
//              running output (32 registers) is rescaled and added to the
//              previous tile's O_t (online softmax).
// The hi/lo pairs carry about 22 significant bits of q and p, the K/V cache
// values are exact in fp16, and every product accumulates in fp32, so the
// result matches the fp32 formulation to a few units of 2^-22.
// Every mbarrier wait is bounded; a timeout raises *err and the CTA releases
// its tensor memory after its MMAs and copies have finished.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "dev_common.cuh"
#include "host_once.h"
#include "kernels.h"
#include "tc_common.cuh"
#include "tc_gemm.h"

namespace lfm {
namespace {
using namespace dev;
using namespace tc;

constexpr int AQ = 32;                  // query tokens per CTA (x 4 heads = 128 rows)
constexpr int KT = 128;                 // key positions per tile
constexpr int ATHREADS = 10 * 32;
constexpr int NSOFT = 8;                // softmax warps
constexpr int Q_BYTES = 128 * 128;      // 128 rows x 64 fp16
constexpr int KV_BYTES = KT * 128;      // 128 positions x 64 fp16
constexpr int P_BYTES = 128 * 256;      // 128 rows x 128 fp16 (two 64-wide chunks)
// P buffer b: hi rows at OFF_P + 2 b P_BYTES, lo rows P_BYTES after them
constexpr int OFF_QH = 0, OFF_QL = Q_BYTES, OFF_K = 2 * Q_BYTES, OFF_V = OFF_K + 2 * KV_BYTES,
              OFF_P = OFF_V + 2 * KV_BYTES;
constexpr int ASMEM = OFF_P + 4 * P_BYTES + 1024;
static_assert(ASMEM + 2048 <= 232448, "attention shared memory");
constexpr uint32_t ATMEM_COLS = 512;    // S: [0, 256), O_t: [256, 384)
constexpr uint32_t IDESC_S = idesc_f16(128, KT, false);
constexpr uint32_t IDESC_PV = idesc_f16(128, HEAD_DIM, true);
constexpr float LOG2E = 1.4426950408889634f;

struct AttnParams {
  const float* q;  // q of token j, head h: q + j * q_stride + h * 64
  int q_stride;
  float* out;      // out + j * out_stride + h * 64
  int out_stride;
  int start, n, ctx;
  const int* start_dev;  // when set, the first position is read here (a replayed graph's launches keep their arguments)
  unsigned* err;
};

// Row r's 8 consecutive fp16 values (16 bytes) at column block `piece` of a
// 64-wide, 128-byte-swizzled K-major chunk.
__device__ __forceinline__ void st_piece(uint8_t* chunk, int r, int piece, uint4 v) {
  *(uint4*)(chunk + r * 128 + ((piece ^ (r & 7)) << 4)) = v;
}

__device__ __forceinline__ void split8(const float (&f)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __half2 hh = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    const float2 back = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(f[2 * i] - back.x, f[2 * i + 1] - back.y);
    h[i] = *(const uint32_t*)&hh;
    l[i] = *(const uint32_t*)&ll;
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// the two softmax warps of a row quarter meet on named barrier 1 + quarter
__device__ __forceinline__ void pair_sync(int quarter) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}

__global__ void __launch_bounds__(ATHREADS, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapV, AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full[2], p_empty[2], o_full[2],
      o_empty[2], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float s_red[2][128];  // per row: the two halves' maxima, at the end their sums
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (p.n + AQ - 1) / AQ;
  const int kh = blockIdx.x;
  const int qb = nqb - 1 - (int)blockIdx.y;  // longest rows first
  const int j0 = qb * AQ;
  const int last_tok = min(j0 + AQ, p.n) - 1;
  const int start = p.start_dev ? *p.start_dev : p.start;
  const int ntiles = (start + last_tok) / KT + 1;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, NSOFT);
    for (int b = 0; b < 2; b++) {
      mbar_init(&kv_full[b], 1);
      mbar_init(&kv_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], NSOFT);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], NSOFT);
      mbar_init(&p_full[b], NSOFT);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_base, ATMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ----------------------------------------------------------- producer
      int issued = 0;
      for (int i = 0; i < ntiles; i++) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&kv_empty[b], ((i >> 1) - 1) & 1, p.err)) break;
        mbar_expect_tx(&kv_full[b], 2 * KV_BYTES);
        tma_load_2d(smem + OFF_K + b * KV_BYTES, &mapK, 0, kh * p.ctx + i * KT, &kv_full[b]);
        tma_load_2d(smem + OFF_V + b * KV_BYTES, &mapV, 0, kh * p.ctx + i * KT, &kv_full[b]);
        issued = i + 1;
      }
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; i++) mbar_wait(&kv_full[i & 1], (i >> 1) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------------- MMA
      const uint32_t qh = smem_u32(smem + OFF_QH), ql = smem_u32(smem + OFF_QL);
      bool ok = mbar_wait(&q_full, 0, p.err);
      auto issue_s = [&](int i) -> bool {
        const int b = i & 1;
        if (!mbar_wait(&kv_full[b], (i >> 1) & 1, p.err)) return false;
        if (i >= 2 && !mbar_wait(&s_empty[b], ((i >> 1) - 1) & 1, p.err)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * KT);
        const uint32_t kb = smem_u32(smem + OFF_K + b * KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          mma_f16(d, smem_desc_sw128(qh + kk * 32), smem_desc_sw128(kb + kk * 32), IDESC_S, kk ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          mma_f16(d, smem_desc_sw128(ql + kk * 32), smem_desc_sw128(kb + kk * 32), IDESC_S, 1u);
        mma_commit(&s_full[b]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int i = 0; i < ntiles && ok; i++) {
        if (i + 1 < ntiles && !(ok = issue_s(i + 1))) break;
        const int b = i & 1;
        if (!(ok = mbar_wait(&p_full[b], (i >> 1) & 1, p.err))) break;
        if (i >= 2 && !(ok = mbar_wait(&o_empty[b], ((i >> 1) - 1) & 1, p.err))) break;
        tc_fence_after();
        const uint32_t ph = smem_u32(smem + OFF_P + b * 2 * P_BYTES), pl = ph + P_BYTES;
        const uint32_t d = tmem + 256u + (uint32_t)(b * HEAD_DIM);
        const uint32_t vb = smem_u32(smem + OFF_V + b * KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < KT / 16; ks++)
          mma_f16(d, smem_desc_sw128(ph + (ks >> 2) * 16384 + (ks & 3) * 32), smem_desc_mn_sw128(vb + ks * 2048),
                  IDESC_PV, ks ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < KT / 16; ks++)
          mma_f16(d, smem_desc_sw128(pl + (ks >> 2) * 16384 + (ks & 3) * 32), smem_desc_mn_sw128(vb + ks * 2048),
                  IDESC_PV, 1u);
        mma_commit(&o_full[b]);
        mma_commit(&p_empty[b]);
        mma_commit(&kv_empty[b]);
      }
      // tensor memory and the operand buffers stay in use until every issued MMA has finished
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0, nullptr);
    }
  } else {
    // ---------------------------------------------------------- softmax rows
    const int quarter = warp & 3;        // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;    // S / P columns [64 half, 64 half + 64), O columns [32 half, +32)
    const int r = quarter * 32 + lane;
    const int h = kh * 4 + quarter;
    const int j = j0 + lane;
    const bool valid = j < p.n;
    const int pr = start + j;  // last key position of this row
    {
      const float* qr = p.q + (size_t)(valid ? j : 0) * p.q_stride + h * HEAD_DIM;
#pragma unroll
      for (int pc = 4 * half; pc < 4 * half + 4; pc++) {
        float f[8];
        const float4 a = valid ? *(const float4*)(qr + 8 * pc) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 b = valid ? *(const float4*)(qr + 8 * pc + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
        f[0] = a.x * 0.125f, f[1] = a.y * 0.125f, f[2] = a.z * 0.125f, f[3] = a.w * 0.125f;
        f[4] = b.x * 0.125f, f[5] = b.y * 0.125f, f[6] = b.z * 0.125f, f[7] = b.w * 0.125f;
        uint4 hi, lo;
        split8(f, hi, lo);
        st_piece(smem + OFF_QH, r, pc, hi);
        st_piece(smem + OFF_QL, r, pc, lo);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full);
    }
    float o[HEAD_DIM / 2];
#pragma unroll
    for (int d = 0; d < HEAD_DIM / 2; d++) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;  // l: this half's share of the row sum
    bool ok = true;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    for (int i = 0; i < ntiles; i++) {
      const int b = i & 1;
      // every softmax warp walks every tile (also after a wait gave up) so
      // that the pair barriers always meet
      if (ok) ok = mbar_wait(&s_full[b], (i >> 1) & 1, p.err);
      tc_fence_after();
      const uint32_t sbase = lane_base + (uint32_t)(b * KT + 64 * half);
      const int col0 = i * KT + 64 * half;  // key position of this thread's first column
      const bool need_mask = col0 + 63 > pr;
      // pass 1: maximum over this half's visible positions, then over the row
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[16];
        tmem_ld16_nowait(sbase + 16 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e++) {
          const float s = __uint_as_float(v[e]);
          mx = fmaxf(mx, (!need_mask || col0 + 16 * c + e <= pr) ? s : -INFINITY);
        }
      }
      s_red[half][r] = mx;
      pair_sync(quarter);
      const float m_new = fmaxf(m, fmaxf(s_red[0][r], s_red[1][r]));  // finite: position 0 is visible to every row
      pair_sync(quarter);  // both reads done before the next tile's writes
      const float alpha = exp2f((m - m_new) * LOG2E);
      // pass 2: probabilities -> fp16 hi/lo operand in P buffer b (after the
      // P.V of tile i - 2 has read it)
      if (ok && i >= 2) ok = mbar_wait(&p_empty[b], ((i >> 1) - 1) & 1, p.err);
      uint8_t* pbuf = smem + OFF_P + b * 2 * P_BYTES + half * 16384;
      const float mlog = m_new * LOG2E;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[16];
        tmem_ld16_nowait(sbase + 16 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 2; g++) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const int col = col0 + 16 * c + 8 * g + e;
            const float pe = exp2f(fmaf(__uint_as_float(v[8 * g + e]), LOG2E, -mlog));
            f[e] = (!need_mask || col <= pr) ? pe : 0.f;
            sum += f[e];
          }
          uint4 hi, lo;
          split8(f, hi, lo);
          st_piece(pbuf, r, 2 * c + g, hi);
          st_piece(pbuf + P_BYTES, r, 2 * c + g, lo);
        }
      }
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[b]);
        mbar_arrive(&p_full[b]);
      }
      l = l * alpha + sum;
      m = m_new;
      // fold the previous tile's P.V into the running output
      if (i >= 1) {
        const int pb = (i - 1) & 1;
        if (ok) ok = mbar_wait(&o_full[pb], ((i - 1) >> 1) & 1, p.err);
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(lane_base + 256u + (uint32_t)(pb * HEAD_DIM + 32 * half), v);
#pragma unroll
        for (int e = 0; e < 32; e++) o[e] = fmaf(o[e], alpha_prev, __uint_as_float(v[e]));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[pb]);
      }
      alpha_prev = alpha;
    }
    const int pb = (ntiles - 1) & 1;
    if (ok) ok = mbar_wait(&o_full[pb], ((ntiles - 1) >> 1) & 1, p.err);
    tc_fence_after();
    {
      uint32_t v[32];
      tmem_ld32(lane_base + 256u + (uint32_t)(pb * HEAD_DIM + 32 * half), v);
#pragma unroll
      for (int e = 0; e < 32; e++) o[e] = fmaf(o[e], alpha_prev, __uint_as_float(v[e]));
    }
    s_red[half][r] = l;
    pair_sync(quarter);
    const float lsum = s_red[0][r] + s_red[1][r];
    if (ok && valid) {
      const float inv = 1.0f / lsum;
      float* dst = p.out + (size_t)j * p.out_stride + h * HEAD_DIM + 32 * half;
#pragma unroll
      for (int d = 0; d < 32; d += 4)
        *(float4*)(dst + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ATMEM_COLS);
  }
}

}  // namespace

cudaError_t attn_prefill_tc(const float* q, int q_stride, const __half* kc, const __half* vc, int start, int n,
                            int ctx, float* out, int out_stride, unsigned* err, cudaStream_t s, const int* start_dev) {
  if (n <= 0 || start < 0 || start + n > ctx || q_stride % 4 || out_stride % 4 || ((uintptr_t)q & 15) ||
      ((uintptr_t)out & 15))
    return cudaErrorInvalidValue;
  CUtensorMap mk, mv;
  cudaError_t e = tc_map_f16(&mk, kc, KV_HEADS * ctx, HEAD_DIM, KT);
  if (e != cudaSuccess) return e;
  e = tc_map_f16(&mv, vc, KV_HEADS * ctx, HEAD_DIM, KT);
  if (e != cudaSuccess) return e;
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu, [] { cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, ASMEM); });
  AttnParams p;
  p.q = q;
  p.q_stride = q_stride;
  p.out = out;
  p.out_stride = out_stride;
  p.start = start;
  p.start_dev = start_dev;
  p.n = n;
  p.ctx = ctx;
  p.err = err;
  k_attn_tc<<<dim3(KV_HEADS, (n + AQ - 1) / AQ), ATHREADS, ASMEM, s>>>(mk, mv, p);
  return cudaGetLastError();
}

}  // namespace lfm
