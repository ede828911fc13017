// Tensor-core (tcgen05 / TMEM) GEMM core for the prompt path (sm_100a).
//
// C[m][n] = sum_k A[m][k] * B[n][k] with fp16 A and B (both K-major) and fp32
// accumulation in tensor memory. One CTA computes a 128 x 256 tile:
//   warp 0        TMA producer: 64-wide K chunks of A (128 rows) and B (256
//                 rows) into a 4-stage shared-memory ring, 128-byte swizzle
//   warp 1        allocates TMEM (256 columns) and issues tcgen05.mma
//                 (M=128, N=256, K=16, kind::f16) from one lane; each stage
//                 is released by tcgen05.commit when its MMAs have read it
//   warps 2-5     epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//                 lanes 32*(w%4)..+31, i.e. rows of the tile) and the store
// Every mbarrier wait is bounded (~1 s of SM cycles); a timeout raises *err
// and the CTA still releases its tensor memory before returning.
//
// Shared-memory operand layout (what tcgen05 calls the K-major canonical
// layout with 128-byte swizzle, and what TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B): a chunk of R rows x 64 fp16 is R consecutive
// 128-byte rows; inside each 1024-byte group of 8 rows the 16-byte pieces of
// row r are permuted by (piece ^ (r % 8)). The matrix descriptor names the
// chunk's start address, an 8-row group stride (SBO) of 1024 bytes and the
// swizzle mode; K steps of 16 elements advance the start address by 32 bytes.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "dev_common.cuh"
#include "host_once.h"
#include "tc_common.cuh"
#include "tc_gemm.h"

namespace lfm {
namespace {
using namespace dev;
using namespace tc;

constexpr int TM = 128, TN = 256, TK = 64;  // tile and K chunk
constexpr int STAGES = 4;
constexpr int A_BYTES = TM * TK * 2;        // 16 KB
constexpr int B_BYTES = TN * TK * 2;        // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 6 * 32;
constexpr uint32_t TMEM_COLS = 256;

// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, both K-major.
constexpr uint32_t IDESC = idesc_f16(TM, TN, false);

__global__ void __launch_bounds__(THREADS, 1)
    k_tc_f16(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, float* C, int M,
             int N, int K, unsigned* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // operand ring at a 1024-byte aligned offset (the swizzle pattern follows address bits)
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * TM, n0 = blockIdx.y * TN;
  const int nk = K / TK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0 && lane == 0) {
    // ----------------------------------------------------------- producer
    for (int kc = 0; kc < nk; kc++) {
      const int s = kc % STAGES, round = kc / STAGES;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, err)) break;
      uint8_t* a = smem + s * STAGE_BYTES;
      uint8_t* b = a + A_BYTES;
      mbar_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(a, &mapA, kc * TK, m0, &full[s]);
      tma_load_2d(b, &mapB, kc * TK, n0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer
    bool ok = true;
    for (int kc = 0; kc < nk && ok; kc++) {
      const int s = kc % STAGES;
      ok = mbar_wait(&full[s], (kc / STAGES) & 1, err);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = smem_u32(smem + s * STAGE_BYTES), b = a + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < TK / 16; kk++)
        mma_f16(tmem, smem_desc_sw128(a + kk * 32), smem_desc_sw128(b + kk * 32), IDESC, (kc | kk) ? 1u : 0u);
      mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    mma_commit(&acc_full);  // the accumulator is complete (or the loop gave up)
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const bool ok = mbar_wait(&acc_full, 0, err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int row = m0 + quarter * 32 + lane;
    for (int c0 = 0; c0 < TN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, r);
      if (ok && row < M)
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (n0 + c0 + j < N) C[(size_t)row * N + n0 + c0 + j] = __uint_as_float(r[j]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ======================================================================
// MN-major B operand (the V tile of prompt attention, stored position-major:
// B[k][n] with n contiguous): C[m][n] = sum_k A[m][k] B[k][n] for N = 64.
// A 64-wide row of B is one 128-byte swizzle atom; a K chunk of 64 rows is
// 8 groups of 8 rows at a 1024-byte stride (SBO), and the MMA's K steps of 16
// rows advance the start address by 2048 bytes. The instruction descriptor
// marks B as MN-major (bit 16).
namespace {
constexpr int BN_N = 64;
constexpr uint32_t IDESC_BMN = idesc_f16(TM, BN_N, true);
constexpr int BMN_A = TM * TK * 2, BMN_B = TK * BN_N * 2, BMN_STAGE = BMN_A + BMN_B;
// the ring is followed by 32 KB that no operand uses
constexpr int BMN_SMEM = STAGES * BMN_STAGE + 32768 + 1024;

__global__ void __launch_bounds__(THREADS, 1)
    k_tc_f16_bmn(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, float* C,
                 int M, int K, unsigned* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * TM;
  const int nk = K / TK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(64));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int kc = 0; kc < nk; kc++) {
      const int s = kc % STAGES, round = kc / STAGES;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1, err)) break;
      uint8_t* a = smem + s * BMN_STAGE;
      mbar_expect_tx(&full[s], BMN_STAGE);
      tma_load_2d(a, &mapA, kc * TK, m0, &full[s]);
      tma_load_2d(a + BMN_A, &mapB, 0, kc * TK, &full[s]);
      issued = kc + 1;
    }
    for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; j++)
      mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr);
  } else if (warp == 1 && lane == 0) {
    bool ok = true;
    for (int kc = 0; kc < nk && ok; kc++) {
      const int s = kc % STAGES;
      ok = mbar_wait(&full[s], (kc / STAGES) & 1, err);
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = smem_u32(smem + s * BMN_STAGE), b = a + BMN_A;
#pragma unroll
      for (int kk = 0; kk < TK / 16; kk++)
        mma_f16(tmem, smem_desc_sw128(a + kk * 32), smem_desc_mn_sw128(b + kk * 2048), IDESC_BMN,
                     (kc | kk) ? 1u : 0u);
      mma_commit(&empty[s]);
    }
    mma_commit(&acc_full);
    mbar_wait(&acc_full, 0, nullptr);
  } else if (warp >= 2) {
    const bool ok = mbar_wait(&acc_full, 0, err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    for (int c0 = 0; c0 < BN_N; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, r);
      if (ok && row < M)
#pragma unroll
        for (int j = 0; j < 32; j++) C[(size_t)row * BN_N + c0 + j] = __uint_as_float(r[j]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64));
  }
}
}  // namespace

// ======================================================================
// Q6_K prompt GEMM: out[t][o] (+)= sum_k W[o][k] x[t][k] for n tokens.
//
// Precision: the tensor cores multiply fp16 operands into fp32 sums, and an
// fp16 copy of a Q6_K weight d*sc*(q-32) is not exact. The super-block scale
// d is therefore kept out of the operand: A holds the integers sc*(q-32),
// which fp16 holds exactly when |sc*(q-32)| <= 2048 or the product is even
// (every weight with |sc| <= 64; above that, odd products round to the
// nearest even integer, a relative error below 2^-11 on those weights only),
// and each 256-wide super-block accumulates into its own TMEM accumulator
// which the epilogue scales by d. The activations are split into an fp16 pair
// hi + lo (about 22 significant bits) after a per-row power-of-two scaling
// into fp16 range; hi and lo of 128 tokens form the 256 B-rows of one N=256
// MMA, and the epilogue adds the two halves of the accumulator.
//
// Roles (10 warps), for a tile of 128 weight rows x TT tokens (TT = 16, 32,
// 64 or 128; the MMA is M=128, N=2*TT):
//   warp 0        TMA, two lanes with independent rings: lane 0 streams the
//                 64-wide K chunks of the hi/lo activations (5 to 16 deep),
//                 lane 1 the raw Q6_K planes of the weight tile, half a
//                 super-block at a time (3-D box over the quant plane, the
//                 2-D scale box with the first half; 2 to 6 buffers)
//   warp 1        TMEM allocation (2 or 4 super-block accumulators of 2*TT
//                 columns) and the MMA issue: 4 x (M=128, N=2*TT, K=16) per
//                 chunk
//   warps 2-9     workers, two per tile row: each reads its row's raw
//                 pieces once per half super-block into registers and writes
//                 half of every chunk's fp16 sc*(q-32) values into a ring of
//                 swizzled K-major A chunks; one chunk into a super-block it
//                 folds an earlier super-block's finished accumulator into
//                 its TT/2 running sums, y += d * (hi + lo), and at the end
//                 it stores them
// The ring depths (activation, A, raw) and the number of accumulators depend
// on TT: narrow tiles have small activation chunks and little tensor work per
// chunk, so they keep more chunks of everything in flight.
// Grouped (routed experts): the activations of each expert are gathered into
// a contiguous, 128-padded run of hi/lo rows (tc_group, tc_split_grouped), a tile
// table lists (expert, first row) per token tile, and the epilogue writes
// each row to its selection slot.
namespace {
// Ring depths per token tile: A = dequantised weight chunks (made on chip),
// B = activation chunks (TMA from L2/HBM, ~1-2 us away: the deep ring), raw =
// half super-blocks of Q6_K planes. Narrow tiles have small B chunks and run
// through chunks quickly, so they keep more of everything in flight.
// The 16-token tile (routed experts of small batches) is bound by the latency
// of its per-chunk hand-offs, not by any pipe, so it is sized for two CTAs
// per SM (~106 KB of shared memory each) to overlap two such chains.
__host__ __device__ constexpr int q_ctas_per_sm(int tt) { return tt <= 16 ? 2 : 1; }
__host__ __device__ constexpr int q_astages(int tt) { return tt >= 128 ? 2 : (tt >= 64 ? 3 : (tt >= 32 ? 4 : 3)); }
__host__ __device__ constexpr int q_bstages(int tt) { return tt >= 128 ? 5 : (tt >= 64 ? 8 : (tt >= 32 ? 12 : 6)); }
constexpr int QA_BYTES = 128 * 128;           // A chunk: 128 rows x 64 fp16
constexpr int RAWH_Q = 128 * 3 * 32;          // half super-block: 3 pieces x 2 units x 128 rows
constexpr int RAWH_S = 128 * 16;              // scales of the super-block (with the first half)
constexpr int RAWH_BYTES = RAWH_Q + RAWH_S;   // 14 KB
__host__ __device__ constexpr int q_off_b(int tt) { return q_astages(tt) * QA_BYTES; }
constexpr int RAWN_MAX = 16;
// Shared memory of the TT-token kernel: A ring, B ring of 2*TT-row chunks, and
// as many raw half super-block buffers as fit (2 at TT = 128 and at TT = 16,
// which runs two CTAs per SM; 3 at TT = 64; 4 at TT = 32). The ring depths
// were chosen by measurement: at TT = 128, A/B = 2/5 beat 3/4, 4/3, 3/3 and
// 2/4 (the last three with deeper raw rings).
__host__ __device__ constexpr int q_off_raw(int tt) { return q_off_b(tt) + q_bstages(tt) * 2 * tt * 128; }
__host__ __device__ constexpr int q_smem_budget(int tt) { return q_ctas_per_sm(tt) == 2 ? 110 * 1024 : 232448 - 2048; }
__host__ __device__ constexpr int q_rawn(int tt) {
  return (q_smem_budget(tt) - q_off_raw(tt)) / RAWH_BYTES < RAWN_MAX ? (q_smem_budget(tt) - q_off_raw(tt)) / RAWH_BYTES
                                                                      : RAWN_MAX;
}
__host__ __device__ constexpr int q_smem(int tt) { return q_off_raw(tt) + q_rawn(tt) * RAWH_BYTES + 1024; }
constexpr int QTHREADS = 10 * 32;
// Super-block accumulators in TMEM (2 * TT columns each): two at TT = 128
// (all 512 columns), four for narrower tiles, which lets the workers fold a
// super-block three super-blocks after it was issued instead of waiting for
// the tensor core.
__host__ __device__ constexpr int q_nacc(int tt) { return tt >= 128 ? 2 : 4; }
__host__ __device__ constexpr uint32_t q_tmem_cols(int tt) { return (uint32_t)(q_nacc(tt) * 2 * tt); }

struct TcQ6Params {
  Q6Mat W;
  int out_rows;        // rows per expert (grouped) or W.rows
  int rpad;            // hi rows of the activation operand (lo rows follow)
  const float* inv;    // [rpad] inverse activation scale per operand row
  float* out;
  int ldo;
  int resid;
  int ntok;            // dense: valid operand rows
  const int* tiles;    // grouped: [0] = count, then (expert, first row) pairs
  const int* slots;    // grouped: operand row -> output slot (-1: padding)
  int grouped;
  int tiles_y;         // dense: token tiles (the expanded-weight kernel's tile space)
  int ksplit;          // dense, one token tile: super-blocks split over blockIdx.z
  float* part;         // ... partial sums [ksplit][ntok][W.rows], reduced by k_tc_reduce
  unsigned* err;
};

// 4 codes (bytes of `code`) -> two half2 of sc*(code-32), exact.
__device__ __forceinline__ void codes_to_h2(uint32_t code, __half2 sc2, uint32_t& lo, uint32_t& hi) {
  const __half2 bias = __halves2half2(__float2half_rn(1056.f), __float2half_rn(1056.f));
  // 0x64XX is the fp16 value 1024 + XX for XX < 256
  uint32_t a = __byte_perm(code, 0x64646464u, 0x4140), b = __byte_perm(code, 0x64646464u, 0x4342);
  __half2 ha = __hmul2(__hsub2(*(__half2*)&a, bias), sc2);
  __half2 hb = __hmul2(__hsub2(*(__half2*)&b, bias), sc2);
  lo = *(uint32_t*)&ha;
  hi = *(uint32_t*)&hb;
}

// TT: tokens per tile (16, 32, 64 or 128); the MMA is M=128, N=2*TT.
template <int TT>
__global__ void __launch_bounds__(QTHREADS, q_ctas_per_sm(TT))
    k_tc_q6(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapS,
            const __grid_constant__ CUtensorMap mapX, TcQ6Params p) {
  constexpr int QB_BYTES = 2 * TT * 128;
  constexpr uint32_t QTMEM_COLS = q_tmem_cols(TT);
  constexpr uint32_t IDESC_Q = idesc_f16(128, 2 * TT, false);
  constexpr int TH = TT / 2;  // tokens of one worker thread
  constexpr int ASTAGES = q_astages(TT), BSTAGES = q_bstages(TT);
  constexpr int NACC = q_nacc(TT), LAG = NACC - 1;  // a super-block is folded LAG super-blocks later
  constexpr int OFF_B = q_off_b(TT);
  constexpr int OFF_RAW = q_off_raw(TT);
  constexpr int RAWN = q_rawn(TT);
  static_assert(RAWN >= 2, "raw ring");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* raw = smem + OFF_RAW;
  __shared__ uint64_t bfull[BSTAGES], bempty[BSTAGES], afull[ASTAGES], aempty[ASTAGES], raw_full[RAWN],
      raw_empty[RAWN], acc_full[NACC], acc_empty[NACC], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float s_inv[TT];  // row scale of each operand row of the tile
  __shared__ int s_slot[TT];   // grouped: output slot of each operand row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.W.nb;
  // this CTA's super-blocks [kb0, kb0 + nbl) (all of them unless split over K)
  const int kb0 = (int)((long long)blockIdx.z * nb / p.ksplit);
  const int nbl = (int)((long long)(blockIdx.z + 1) * nb / p.ksplit) - kb0;
  const int o0 = blockIdx.x * 128;
  int brow0, wrow0;
  if (p.grouped) {
    if ((int)blockIdx.y >= p.tiles[0]) return;  // whole CTA leaves before any barrier or TMEM use
    wrow0 = p.tiles[1 + 2 * blockIdx.y] * p.out_rows;
    brow0 = p.tiles[2 + 2 * blockIdx.y];
  } else {
    wrow0 = 0;
    brow0 = blockIdx.y * TT;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < BSTAGES; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < ASTAGES; s++) {
      mbar_init(&afull[s], 8);
      mbar_init(&aempty[s], 1);
    }
    for (int r = 0; r < RAWN; r++) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], 8);
    }
    for (int r = 0; r < NACC; r++) {
      mbar_init(&acc_full[r], 1);
      mbar_init(&acc_empty[r], 8);
    }
    mbar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_base, QTMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int nchunks = 4 * nbl;

  if (warp == 0) {
    if (lane == 0) {
      // ----------------------------------------------------------- producer
      // lane 0: activation chunks j (5-deep ring)
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nchunks && ok; j++) {
        const int s = j % BSTAGES, round = j / BSTAGES;
        if (round > 0 && !(ok = mbar_wait(&bempty[s], (round - 1) & 1, p.err))) break;
        uint8_t* bs = smem + OFF_B + s * QB_BYTES;
        mbar_expect_tx(&bfull[s], QB_BYTES);
        tma_load_3d(bs, &mapX, 64 * (4 * kb0 + j), brow0, 0, &bfull[s]);  // hi and lo rows
        issued = j + 1;
      }
      // every issued copy must land before the CTA may exit
      for (int j = issued > BSTAGES ? issued - BSTAGES : 0; j < issued; j++)
        mbar_wait(&bfull[j % BSTAGES], (j / BSTAGES) & 1, nullptr);
    } else if (lane == 1) {
      // lane 1: raw weight pieces, half super-block k = 2 * (b - kb0) + h into
      // buffer k % RAWN (runs ahead of the activations by up to RAWN halves)
      int issued = 0;
      bool ok = true;
      for (int k = 0; k < 2 * nbl && ok; k++) {
        const int b = kb0 + (k >> 1), h = k & 1, rb = k % RAWN;
        if (k >= RAWN && !(ok = mbar_wait(&raw_empty[rb], ((k / RAWN) - 1) & 1, p.err))) break;
        uint8_t* rq = raw + rb * RAWH_BYTES;
        mbar_expect_tx(&raw_full[rb], RAWH_Q + (h == 0 ? RAWH_S : 0));
        tma_load_3d(rq, &mapQ, 64 * b + 32 * h, 0, wrow0 + o0, &raw_full[rb]);
        if (h == 0) tma_load_2d(rq + RAWH_Q, &mapS, 16 * b, wrow0 + o0, &raw_full[rb]);
        issued = k + 1;
      }
      for (int k = issued > RAWN ? issued - RAWN : 0; k < issued; k++)
        mbar_wait(&raw_full[k % RAWN], (k / RAWN) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------------- MMA
      // One thread issues everything, so its per-chunk overhead bounds the
      // tensor pipe: ring positions and phases advance incrementally and the
      // descriptors are offsets of two precomputed bases (the start address
      // field counts 16-byte units; shared addresses stay below 2^18).
      bool ok = true;
      int sb = 0, sa = 0;
      uint32_t pb = 0, pa = 0;
      const uint64_t dA0 = smem_desc_sw128(smem_u32(smem)), dB0 = smem_desc_sw128(smem_u32(smem + OFF_B));
      for (int b = 0; b < nbl && ok; b++) {
        const int a = b % NACC;
        if (b >= NACC && !(ok = mbar_wait(&acc_empty[a], ((b / NACC) - 1) & 1, p.err))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * 2 * TT);
        for (int c = 0; c < 4 && ok; c++) {
          ok = mbar_wait(&bfull[sb], pb, p.err) && mbar_wait(&afull[sa], pa, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint64_t da = dA0 + (uint64_t)((sa * QA_BYTES) >> 4), db = dB0 + (uint64_t)((sb * QB_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; kk++) mma_f16(d, da + 2 * kk, db + 2 * kk, IDESC_Q, (c | kk) ? 1u : 0u);
          mma_commit(&bempty[sb]);
          mma_commit(&aempty[sa]);
          if (++sb == BSTAGES) sb = 0, pb ^= 1u;
          if (++sa == ASTAGES) sa = 0, pa ^= 1u;
        }
        mma_commit(&acc_full[a]);
      }
      // tensor memory and the operand stages stay in use until every issued MMA has finished
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0, nullptr);
    }
  } else {
    // --------------------------------------------------------------- workers
    // Thread (row, g): dequantises element pair m = 2 * (c & 1) + g of its
    // tile row for every chunk c, and owns tokens 64g..64g+63 of that row in
    // the epilogue (TMEM lanes of quarter warp % 4).
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const size_t wrow = (size_t)wrow0 + o0 + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(TH * g);
    // the tile's row scales and slots, staged while the first operands load
    // (the store phase then reads them from shared memory)
    const int wt = threadIdx.x - 64;  // 0..255
    if (wt < TT) {
      s_inv[wt] = __ldg(p.inv + brow0 + wt);
      s_slot[wt] = p.grouped ? __ldg(p.slots + brow0 + wt) : -1;
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight worker warps
    float y[TH];
#pragma unroll
    for (int j = 0; j < TH; j++) y[j] = 0.f;
    bool ok = true;
    // y += d_b * (hi + lo) for super-block b's accumulator
    auto epilogue = [&](int b, float d) {
      const int a = b % NACC;
      ok = ok && mbar_wait(&acc_full[a], (b / NACC) & 1, p.err);
      tc_fence_after();
      const uint32_t base = lane_base + (uint32_t)(a * 2 * TT);
      if constexpr (TH >= 16) {
#pragma unroll
        for (int h = 0; h < TH / 16; h++) {
          uint32_t hi[16], lo[16];
          tmem_ld16_nowait(base + 16 * h, hi);
          tmem_ld16_nowait(base + TT + 16 * h, lo);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j++)
            y[16 * h + j] = fmaf(d, __uint_as_float(hi[j]) + __uint_as_float(lo[j]), y[16 * h + j]);
        }
      } else {
        uint32_t hi[8], lo[8];
        tmem_ld8_nowait(base, hi);
        tmem_ld8_nowait(base + TT, lo);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; j++) y[j] = fmaf(d, __uint_as_float(hi[j]) + __uint_as_float(lo[j]), y[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    };
    // dd[i] = d of super-block b - i (loaded when b starts, used LAG super-blocks later)
    float dd[NACC];
#pragma unroll
    for (int i = 0; i < NACC; i++) dd[i] = 0.f;
    for (int b = 0; b < nbl && ok; b++) {
#pragma unroll
      for (int i = NACC - 1; i > 0; i--) dd[i] = dd[i - 1];
      dd[0] = __half2float(p.W.d[wrow * nb + kb0 + b]);
      uint4 ql[2], qh[2];
      uint32_t scw[4];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int j = 4 * b + c, s = j % ASTAGES, round = j / ASTAGES;
        const int h = c >> 1, m = 2 * (c & 1) + g;
        if ((c & 1) == 0) {
          // this half's pieces (low nibbles: piece g; high bits: piece 2) of units 2h, 2h+1
          const int k = 2 * b + h, rb = k % RAWN;
          if (!(ok = mbar_wait(&raw_full[rb], (k / RAWN) & 1, p.err))) break;
          const uint8_t* rq = raw + rb * RAWH_BYTES + row * 96;
#pragma unroll
          for (int qq = 0; qq < 2; qq++) {
            ql[qq] = *(const uint4*)(rq + g * 32 + qq * 16);
            qh[qq] = *(const uint4*)(rq + 64 + qq * 16);
          }
          if (c == 0) {
            const uint4 sv = *(const uint4*)(raw + rb * RAWH_BYTES + RAWH_Q + row * 16);
            scw[0] = sv.x, scw[1] = sv.y, scw[2] = sv.z, scw[3] = sv.w;
          }
        }
        if (round > 0 && !(ok = mbar_wait(&aempty[s], (round - 1) & 1, p.err))) break;
        uint8_t* arow = smem + s * QA_BYTES + row * 128;
#pragma unroll
        for (int qq = 0; qq < 2; qq++) {
          const int uu = 2 * h + qq;
          const float scf = (float)(int8_t)(uint8_t)(scw[uu] >> (8 * m));
          const __half2 sc2 = __float2half2_rn(scf);
          const uint32_t lw[4] = {ql[qq].x, ql[qq].y, ql[qq].z, ql[qq].w};
          const uint32_t hw[4] = {qh[qq].x, qh[qq].y, qh[qq].z, qh[qq].w};
          uint32_t o[8];
#pragma unroll
          for (int w = 0; w < 4; w++) {
            const uint32_t code =
                ((lw[w] >> (4 * (m >> 1))) & 0x0F0F0F0Fu) | (((hw[w] >> (2 * m)) & 0x03030303u) << 4);
            codes_to_h2(code, sc2, o[2 * w], o[2 * w + 1]);
          }
          // 16 fp16 = two 16-byte pieces at chunk offset 32*g + 16*qq elements
          const int p0 = 4 * g + 2 * qq;
          *(uint4*)(arow + ((p0 ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *(uint4*)(arow + (((p0 + 1) ^ (row & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        // The A writes go to the tensor core (async proxy), and for c = 0, 2
        // the raw half just consumed is refilled by TMA (async proxy) once
        // released: order this thread's shared-memory accesses first. The raw
        // loads are complete here (their values fed the A writes).
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[s]);
          if ((c & 1) == 0) mbar_arrive(&raw_empty[(2 * b + h) % RAWN]);  // this half is in registers
        }
        // super-block b - LAG's accumulator is complete by now: fold it in
        if (c == 1 && b >= LAG) epilogue(b - LAG, dd[LAG]);
      }
    }
    // the last LAG super-blocks, in order (dd[i] holds super-block nbl - 1 - i)
#pragma unroll
    for (int i = LAG - 1; i >= 0; i--)
      if (ok && nbl - 1 - i >= 0) epilogue(nbl - 1 - i, dd[i]);
    if (ok) {
      // Output rows of this thread's tokens, JC at a time: a residual chunk's
      // loads are all issued before its first store, so the chunk costs one
      // memory round trip, not one per token.
      const int o = o0 + row;
      const int bq = brow0 + TH * g;
      constexpr int JC = TH < 16 ? TH : 16;
#pragma unroll
      for (int j0 = 0; j0 < TH; j0 += JC) {
        float v[JC];
#pragma unroll
        for (int j = 0; j < JC; j++) v[j] = __fmul_rn(y[j0 + j], s_inv[TH * g + j0 + j]);
        if (p.grouped) {
#pragma unroll
          for (int j = 0; j < JC; j++) {
            const int slot = s_slot[TH * g + j0 + j];
            if (slot >= 0) p.out[(size_t)slot * p.ldo + o] = v[j];
          }
        } else if (p.part) {
#pragma unroll
          for (int j = 0; j < JC; j++)
            if (bq + j0 + j < p.ntok) p.part[((size_t)blockIdx.z * p.ntok + bq + j0 + j) * p.W.rows + o] = v[j];
        } else if (p.resid) {
          float old[JC];
#pragma unroll
          for (int j = 0; j < JC; j++) old[j] = bq + j0 + j < p.ntok ? p.out[(size_t)(bq + j0 + j) * p.ldo + o] : 0.f;
#pragma unroll
          for (int j = 0; j < JC; j++)
            if (bq + j0 + j < p.ntok) p.out[(size_t)(bq + j0 + j) * p.ldo + o] = __fadd_rn(old[j], v[j]);
        } else {
#pragma unroll
          for (int j = 0; j < JC; j++)
            if (bq + j0 + j < p.ntok) p.out[(size_t)(bq + j0 + j) * p.ldo + o] = v[j];
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QTMEM_COLS));
  }
}

// ======================================================================
// Q6_K prompt GEMM over load-time expanded weights (the default when the
// engine holds them): the A operand is the same fp16 integers sc*(q-32) that
// k_tc_q6's workers make on chip, written once at load time into an fp16
// matrix [rows][K] (q6_expand_f16), so the tile's A chunks arrive by TMA like
// its activation chunks and no warp dequantises. Same MMAs, same
// per-super-block TMEM accumulators, same fold y += d * (hi + lo) and the same
// stores, so the results are bit-identical to k_tc_q6's.
//   warp 0        TMA: the activation chunks (as k_tc_q6)
//   warp 1        TMEM allocation and the MMA issue (as k_tc_q6)
//   warps 2-9     fold each super-block's accumulator as soon as it is complete,
//                 then store
//   warp 10       TMA: the A chunks (64-wide K x 128 rows, 128-byte swizzle)
#ifndef LFM_X_A128
#define LFM_X_A128 4
#endif
#ifndef LFM_X_B128
#define LFM_X_B128 5
#endif
__host__ __device__ constexpr int x_astages(int tt) {
  return tt >= 128 ? LFM_X_A128 : (tt >= 64 ? 4 : (tt >= 32 ? 4 : 3));
}
__host__ __device__ constexpr int x_bstages(int tt) {
  return tt >= 128 ? LFM_X_B128 : (tt >= 64 ? 8 : (tt >= 32 ? 12 : 6));
}
__host__ __device__ constexpr int x_off_b(int tt) { return x_astages(tt) * QA_BYTES; }
__host__ __device__ constexpr int x_smem(int tt) { return x_off_b(tt) + x_bstages(tt) * 2 * tt * 128 + 1024; }
static_assert(x_smem(128) <= 232448 - 2048 && x_smem(64) <= 232448 - 2048 && x_smem(32) <= 232448 - 2048 &&
                  x_smem(16) <= 110 * 1024,
              "expanded-weight GEMM shared memory");

// warps of k_tc_q6x: 0 activation loads, 1 MMA, 2-9 fold and store, 10 weight
// loads. Each TMA load holds its issuing thread for a few hundred cycles and
// the lanes of one warp issue one after another, so the two operand streams
// have a warp each.
constexpr int XTHREADS = 11 * 32;
constexpr int XA_WARP = 10;

template <int TT>
__global__ void __launch_bounds__(XTHREADS, q_ctas_per_sm(TT))
    k_tc_q6x(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapX, TcQ6Params p) {
  constexpr int QB_BYTES = 2 * TT * 128;
  constexpr uint32_t QTMEM_COLS = q_tmem_cols(TT);
  constexpr uint32_t IDESC_Q = idesc_f16(128, 2 * TT, false);
  constexpr int TH = TT / 2;  // tokens of one worker thread
  constexpr int ASTAGES = x_astages(TT), BSTAGES = x_bstages(TT);
  constexpr int NACC = q_nacc(TT);
  constexpr int OFF_B = x_off_b(TT);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t bfull[BSTAGES], bempty[BSTAGES], afull[ASTAGES], aempty[ASTAGES], acc_full[NACC],
      acc_empty[NACC], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float s_inv[TT];
  __shared__ int s_slot[TT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.W.nb;
  // Persistent: this CTA takes tiles blockIdx.x, + gridDim.x, ... of the
  // (weight tile, token tile, K split) space, weight tiles fastest. Every ring
  // and accumulator counter runs on across its tiles, so the next tile's
  // loads and first MMAs proceed while the workers fold and store this one.
  const int tiles_x = p.out_rows / 128;
  const int tiles_y = p.grouped ? p.tiles[0] : p.tiles_y;
  const int ntile = tiles_x * tiles_y * p.ksplit;
  auto tile_of = [&](int t, int& o0, int& brow0, int& wrow0, int& kb0, int& nbl, int& z) {
    const int x = t % tiles_x, r = t / tiles_x, y = r % tiles_y;
    z = r / tiles_y;
    o0 = x * 128;
    if (p.grouped) {
      wrow0 = p.tiles[1 + 2 * y] * p.out_rows;
      brow0 = p.tiles[2 + 2 * y];
    } else {
      wrow0 = 0;
      brow0 = y * TT;
    }
    kb0 = (int)((long long)z * nb / p.ksplit);
    nbl = (int)((long long)(z + 1) * nb / p.ksplit) - kb0;
  };
  if ((int)blockIdx.x >= ntile) return;  // whole CTA leaves before any barrier or TMEM use
  if (threadIdx.x == 0) {
    for (int s = 0; s < BSTAGES; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < ASTAGES; s++) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int r = 0; r < NACC; r++) {
      mbar_init(&acc_full[r], 1);
      mbar_init(&acc_empty[r], 8);
    }
    mbar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_base, QTMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0 || warp == XA_WARP) {
    if (lane == 0) {
      // warp 0: activation chunks (hi and lo rows); warp XA_WARP: A chunks
      const bool act = warp == 0;
      const int NS = act ? BSTAGES : ASTAGES;
      uint64_t* full = act ? bfull : afull;
      uint64_t* empty = act ? bempty : aempty;
      int j = 0;  // chunks issued (all tiles)
      bool ok = true;
      for (int t = blockIdx.x; t < ntile && ok; t += gridDim.x) {
        int o0, brow0, wrow0, kb0, nbl, z;
        tile_of(t, o0, brow0, wrow0, kb0, nbl, z);
        for (int c = 0; c < 4 * nbl; c++, j++) {
          const int s = j % NS, round = j / NS;
          if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1, p.err))) break;
          const int kx = 64 * (4 * kb0 + c);
          if (act) {
            uint8_t* bs = smem + OFF_B + s * QB_BYTES;
            mbar_expect_tx(&full[s], QB_BYTES);
            tma_load_3d(bs, &mapX, kx, brow0, 0, &full[s]);  // hi and lo rows
          } else {
            mbar_expect_tx(&full[s], QA_BYTES);
            tma_load_2d(smem + s * QA_BYTES, &mapA, kx, wrow0 + o0, &full[s]);
          }
        }
      }
      // every issued copy must land before the CTA may exit
      for (int k = j > NS ? j - NS : 0; k < j; k++) mbar_wait(&full[k % NS], (k / NS) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // -------------------------------------------------------------- MMA
      bool ok = true;
      int sb = 0, sa = 0, bg = 0;  // bg: super-blocks issued (all tiles)
      uint32_t pb = 0, pa = 0;
      const uint64_t dA0 = smem_desc_sw128(smem_u32(smem)), dB0 = smem_desc_sw128(smem_u32(smem + OFF_B));
      for (int t = blockIdx.x; t < ntile && ok; t += gridDim.x) {
        int o0, brow0, wrow0, kb0, nbl, z;
        tile_of(t, o0, brow0, wrow0, kb0, nbl, z);
        for (int b = 0; b < nbl && ok; b++, bg++) {
          const int a = bg % NACC;
          if (bg >= NACC && !(ok = mbar_wait(&acc_empty[a], ((bg / NACC) - 1) & 1, p.err))) break;
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(a * 2 * TT);
          for (int c = 0; c < 4 && ok; c++) {
            ok = mbar_wait(&bfull[sb], pb, p.err) && mbar_wait(&afull[sa], pa, p.err);
            if (!ok) break;
            tc_fence_after();
            const uint64_t da = dA0 + (uint64_t)((sa * QA_BYTES) >> 4), db = dB0 + (uint64_t)((sb * QB_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) mma_f16(d, da + 2 * kk, db + 2 * kk, IDESC_Q, (c | kk) ? 1u : 0u);
            mma_commit(&bempty[sb]);
            mma_commit(&aempty[sa]);
            if (++sb == BSTAGES) sb = 0, pb ^= 1u;
            if (++sa == ASTAGES) sa = 0, pa ^= 1u;
          }
          mma_commit(&acc_full[a]);
        }
      }
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0, nullptr);
    }
  } else if (warp < XA_WARP) {
    // --------------------------------------------------------------- workers
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(TH * g);
    const int wt = threadIdx.x - 64;  // 0..255
    bool ok = true;
    int bg = 0;  // super-blocks folded (all tiles)
    // Every worker warp walks every tile, also after a wait gave up, so that
    // all of them meet the same named barriers.
    for (int t = blockIdx.x; t < ntile; t += gridDim.x) {
      int o0, brow0, wrow0, kb0, nbl, zk;  // zk: this tile's K split
      tile_of(t, o0, brow0, wrow0, kb0, nbl, zk);
      const size_t wrow = (size_t)wrow0 + o0 + row;
      // the tile's row scales and slots (the previous tile's stores are done:
      // every worker has passed this barrier after them)
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (wt < TT) {
        s_inv[wt] = __ldg(p.inv + brow0 + wt);
        s_slot[wt] = p.grouped ? __ldg(p.slots + brow0 + wt) : -1;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      float y[TH];
#pragma unroll
      for (int jj = 0; jj < TH; jj++) y[jj] = 0.f;
      float dnext = __half2float(p.W.d[wrow * nb + kb0]);
      for (int b = 0; b < nbl && ok; b++, bg++) {
        // y += d_b * (hi + lo) for super-block b's accumulator, as soon as it is complete
        const float d = dnext;
        if (b + 1 < nbl) dnext = __half2float(p.W.d[wrow * nb + kb0 + b + 1]);
        const int a = bg % NACC;
        ok = mbar_wait(&acc_full[a], (bg / NACC) & 1, p.err);
        tc_fence_after();
        const uint32_t base = lane_base + (uint32_t)(a * 2 * TT);
        if constexpr (TH >= 16) {
#pragma unroll
          for (int h = 0; h < TH / 16; h++) {
            uint32_t hi[16], lo[16];
            tmem_ld16_nowait(base + 16 * h, hi);
            tmem_ld16_nowait(base + TT + 16 * h, lo);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 16; jj++)
              y[16 * h + jj] = fmaf(d, __uint_as_float(hi[jj]) + __uint_as_float(lo[jj]), y[16 * h + jj]);
          }
        } else {
          uint32_t hi[8], lo[8];
          tmem_ld8_nowait(base, hi);
          tmem_ld8_nowait(base + TT, lo);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 8; jj++) y[jj] = fmaf(d, __uint_as_float(hi[jj]) + __uint_as_float(lo[jj]), y[jj]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
      }
      if (!ok) continue;
      const int o = o0 + row;
      const int bq = brow0 + TH * g;
      constexpr int JC = TH < 16 ? TH : 16;
#pragma unroll
      for (int j0 = 0; j0 < TH; j0 += JC) {
        float v[JC];
#pragma unroll
        for (int jj = 0; jj < JC; jj++) v[jj] = __fmul_rn(y[j0 + jj], s_inv[TH * g + j0 + jj]);
        if (p.grouped) {
#pragma unroll
          for (int jj = 0; jj < JC; jj++) {
            const int slot = s_slot[TH * g + j0 + jj];
            if (slot >= 0) p.out[(size_t)slot * p.ldo + o] = v[jj];
          }
        } else if (p.part) {
#pragma unroll
          for (int jj = 0; jj < JC; jj++)
            if (bq + j0 + jj < p.ntok) p.part[((size_t)zk * p.ntok + bq + j0 + jj) * p.W.rows + o] = v[jj];
        } else if (p.resid) {
          float old[JC];
#pragma unroll
          for (int jj = 0; jj < JC; jj++)
            old[jj] = bq + j0 + jj < p.ntok ? p.out[(size_t)(bq + j0 + jj) * p.ldo + o] : 0.f;
#pragma unroll
          for (int jj = 0; jj < JC; jj++)
            if (bq + j0 + jj < p.ntok) p.out[(size_t)(bq + j0 + jj) * p.ldo + o] = __fadd_rn(old[jj], v[jj]);
        } else {
#pragma unroll
          for (int jj = 0; jj < JC; jj++)
            if (bq + j0 + jj < p.ntok) p.out[(size_t)(bq + j0 + jj) * p.ldo + o] = v[jj];
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QTMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// 2-SM form of k_tc_q6x for 128-token tiles: a cluster of two CTAs (one per SM)
// computes 256 weight rows x 128 tokens with tcgen05.mma.cta_group::2 (M=256,
// N=256). CTA r of the pair holds weight rows [128 r, 128 r + 128) of the tile
// (A) and one half of the activation operand (B): CTA 0 the hi rows, CTA 1 the
// lo rows; its TMEM receives its 128 rows x all 256 columns (hi then lo), so
// each CTA's workers fold and store exactly as k_tc_q6x's do. Per 64-wide K
// chunk each SM loads 32 KB (16 KB of A, 16 KB of B) instead of 48 KB, which
// buys a deeper ring in the same shared memory.
//   Barriers: the leader (rank 0) owns the operand-full barriers; both CTAs'
//   TMA loads complete their bytes on the leader's barrier (the .cta_group::2
//   load form with the leader's barrier mapped by mapa), the leader's producer
//   arms it for both. The leader's warp 1 issues the MMAs; its commits arrive
//   on both CTAs' slot-empty and accumulator-full barriers (multicast commit).
//   Both CTAs' workers release an accumulator on the leader's barrier (16
//   arrivals). Every wait is bounded; a cluster barrier before teardown keeps
//   each CTA alive while its peer may still signal it.
constexpr int X2_ASTAGES = 7, X2_BSTAGES = 6;
constexpr int X2_STAGE = 128 * 128;  // 128 rows x 64 fp16, either operand
constexpr int X2_OFF_B = X2_ASTAGES * X2_STAGE;
constexpr int X2_SMEM = X2_OFF_B + X2_BSTAGES * X2_STAGE + 1024;
static_assert(X2_SMEM <= 232448 - 2048, "2-SM expanded-weight GEMM shared memory");

__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared variable `p` in CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}
// TMA load into this CTA's shared memory completing on an mbarrier that may be
// the peer CTA's (shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// arrive on `bar` (same offset) in both CTAs of the pair once this thread's MMAs completed
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(XTHREADS, 1)
    k_tc_q6x2(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapX, TcQ6Params p) {
  constexpr int TT = 128, TH = TT / 2;
  constexpr uint32_t IDESC2 = idesc_f16(256, 2 * TT, false);
  constexpr int NACC = 2;  // two 256-column accumulators: all 512 TMEM columns
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t bfull[X2_BSTAGES], bempty[X2_BSTAGES], afull[X2_ASTAGES], aempty[X2_ASTAGES], acc_full[NACC],
      acc_empty[NACC], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float s_inv[TT];
  __shared__ int s_slot[TT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank_in_cluster();
  const bool leader = rank == 0;
  const int nb = p.W.nb;
  // pairs walk the (256-row weight tile, token tile, K split) space, weight tiles fastest
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_x = p.out_rows / 256;
  const int tiles_y = p.grouped ? p.tiles[0] : p.tiles_y;
  const int ntile = tiles_x * tiles_y * p.ksplit;
  auto tile_of = [&](int t, int& o0, int& brow0, int& wrow0, int& kb0, int& nbl, int& z) {
    const int x = t % tiles_x, r = t / tiles_x, y = r % tiles_y;
    z = r / tiles_y;
    o0 = x * 256 + 128 * (int)rank;  // this CTA's 128 rows
    if (p.grouped) {
      wrow0 = p.tiles[1 + 2 * y] * p.out_rows;
      brow0 = p.tiles[2 + 2 * y];
    } else {
      wrow0 = 0;
      brow0 = y * TT;
    }
    kb0 = (int)((long long)z * nb / p.ksplit);
    nbl = (int)((long long)(z + 1) * nb / p.ksplit) - kb0;
  };
  // both CTAs of a pair see the same tile count, so a pair leaves together
  if (pair >= ntile) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < X2_BSTAGES; s++) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < X2_ASTAGES; s++) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int r = 0; r < NACC; r++) {
      mbar_init(&acc_full[r], 1);
      mbar_init(&acc_empty[r], 16);  // 8 worker warps in each CTA
    }
    mbar_init(&mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before anything signals them
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0 || warp == XA_WARP) {
    if (lane == 0) {
      // warp 0: this CTA's half of the activation chunk; warp XA_WARP: its A chunk
      const bool act = warp == 0;
      const int NS = act ? X2_BSTAGES : X2_ASTAGES;
      uint64_t* full = act ? bfull : afull;
      uint64_t* empty = act ? bempty : aempty;
      uint8_t* ring = smem + (act ? X2_OFF_B : 0);
      int j = 0;
      bool ok = true;
      for (int t = pair; t < ntile && ok; t += npairs) {
        int o0, brow0, wrow0, kb0, nbl, z;
        tile_of(t, o0, brow0, wrow0, kb0, nbl, z);
        for (int c = 0; c < 4 * nbl; c++, j++) {
          const int s = j % NS, round = j / NS;
          if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1, p.err))) break;
          const int kx = 64 * (4 * kb0 + c);
          if (leader) mbar_expect_tx(&full[s], 2 * X2_STAGE);  // both CTAs' bytes
          const uint32_t bar = cluster_addr(&full[s], 0);
          if (act)
            tma_load_2d_pair(ring + s * X2_STAGE, &mapX, kx, (rank ? p.rpad : 0) + brow0, bar);
          else
            tma_load_2d_pair(ring + s * X2_STAGE, &mapA, kx, wrow0 + o0, bar);
        }
      }
      // the leader's copies (and the peer's, which complete on the same
      // barriers) land before the CTA may exit
      if (leader)
        for (int k = j > NS ? j - NS : 0; k < j; k++) mbar_wait(&full[k % NS], (k / NS) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      if (leader) {
        // ------------------------------------------------------------ MMA
        bool ok = true;
        int sb = 0, sa = 0, bg = 0;
        uint32_t pb = 0, pa = 0;
        const uint64_t dA0 = smem_desc_sw128(smem_u32(smem)), dB0 = smem_desc_sw128(smem_u32(smem + X2_OFF_B));
        for (int t = pair; t < ntile && ok; t += npairs) {
          int o0, brow0, wrow0, kb0, nbl, z;
          tile_of(t, o0, brow0, wrow0, kb0, nbl, z);
          for (int b = 0; b < nbl && ok; b++, bg++) {
            const int a = bg % NACC;
            if (bg >= NACC && !(ok = mbar_wait(&acc_empty[a], ((bg / NACC) - 1) & 1, p.err))) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(a * 2 * TT);
            for (int c = 0; c < 4 && ok; c++) {
              ok = mbar_wait(&bfull[sb], pb, p.err) && mbar_wait(&afull[sa], pa, p.err);
              if (!ok) break;
              tc_fence_after();
              const uint64_t da = dA0 + (uint64_t)((sa * X2_STAGE) >> 4), db = dB0 + (uint64_t)((sb * X2_STAGE) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; kk++) mma_f16_pair(d, da + 2 * kk, db + 2 * kk, IDESC2, (c | kk) ? 1u : 0u);
              mma_commit_pair(&bempty[sb]);
              mma_commit_pair(&aempty[sa]);
              if (++sb == X2_BSTAGES) sb = 0, pb ^= 1u;
              if (++sa == X2_ASTAGES) sa = 0, pa ^= 1u;
            }
            mma_commit_pair(&acc_full[a]);
          }
        }
        mma_commit_pair(&mma_done);
      }
      // both CTAs: the leader's MMAs (which read this CTA's operands) are done
      mbar_wait(&mma_done, 0, nullptr);
    }
  } else if (warp < XA_WARP) {
    // --------------------------------------------------------------- workers
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(TH * g);
    const int wt = threadIdx.x - 64;
    bool ok = true;
    int bg = 0;
    for (int t = pair; t < ntile; t += npairs) {
      int o0, brow0, wrow0, kb0, nbl, zk;
      tile_of(t, o0, brow0, wrow0, kb0, nbl, zk);
      const size_t wrow = (size_t)wrow0 + o0 + row;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (wt < TT) {
        s_inv[wt] = __ldg(p.inv + brow0 + wt);
        s_slot[wt] = p.grouped ? __ldg(p.slots + brow0 + wt) : -1;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      float y[TH];
#pragma unroll
      for (int jj = 0; jj < TH; jj++) y[jj] = 0.f;
      float dnext = __half2float(p.W.d[wrow * nb + kb0]);
      for (int b = 0; b < nbl && ok; b++, bg++) {
        const float d = dnext;
        if (b + 1 < nbl) dnext = __half2float(p.W.d[wrow * nb + kb0 + b + 1]);
        const int a = bg % NACC;
        ok = mbar_wait(&acc_full[a], (bg / NACC) & 1, p.err);
        tc_fence_after();
        const uint32_t base = lane_base + (uint32_t)(a * 2 * TT);
#pragma unroll
        for (int h = 0; h < TH / 16; h++) {
          uint32_t hi[16], lo[16];
          tmem_ld16_nowait(base + 16 * h, hi);
          tmem_ld16_nowait(base + TT + 16 * h, lo);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; jj++)
            y[16 * h + jj] = fmaf(d, __uint_as_float(hi[jj]) + __uint_as_float(lo[jj]), y[16 * h + jj]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&acc_empty[a], 0));
      }
      if (!ok) continue;
      const int o = o0 + row;
      const int bq = brow0 + TH * g;
#pragma unroll
      for (int j0 = 0; j0 < TH; j0 += 16) {
        float v[16];
#pragma unroll
        for (int jj = 0; jj < 16; jj++) v[jj] = __fmul_rn(y[j0 + jj], s_inv[TH * g + j0 + jj]);
        if (p.grouped) {
#pragma unroll
          for (int jj = 0; jj < 16; jj++) {
            const int slot = s_slot[TH * g + j0 + jj];
            if (slot >= 0) p.out[(size_t)slot * p.ldo + o] = v[jj];
          }
        } else if (p.part) {
#pragma unroll
          for (int jj = 0; jj < 16; jj++)
            if (bq + j0 + jj < p.ntok) p.part[((size_t)zk * p.ntok + bq + j0 + jj) * p.W.rows + o] = v[jj];
        } else if (p.resid) {
          float old[16];
#pragma unroll
          for (int jj = 0; jj < 16; jj++)
            old[jj] = bq + j0 + jj < p.ntok ? p.out[(size_t)(bq + j0 + jj) * p.ldo + o] : 0.f;
#pragma unroll
          for (int jj = 0; jj < 16; jj++)
            if (bq + j0 + jj < p.ntok) p.out[(size_t)(bq + j0 + jj) * p.ldo + o] = __fadd_rn(old[jj], v[jj]);
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; jj++)
            if (bq + j0 + jj < p.ntok) p.out[(size_t)(bq + j0 + jj) * p.ldo + o] = v[jj];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// Load-time expansion of a Q6_K matrix into the fp16 A operand of k_tc_q6x:
// out[row][k] = fp16(sc * (q - 32)), rounded to nearest even like k_tc_q6's
// on-chip __hmul2 (exact whenever |sc * (q - 32)| <= 2048 or even). One thread
// per 64-weight unit.
__global__ void k_q6_expand_f16(Q6Mat W, __half* out) {
  const int U = 4 * W.nb;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)W.rows * U) return;
  const size_t row = i / U;
  const int u = (int)(i % U);
  const uint4* qp = W.q + row * 3 * U + u;
  const uint4 A = qp[0], B = qp[U], Q = qp[2 * U];
  const uint32_t scw = W.sc[row * U + u];
  const uint32_t a[4] = {A.x, A.y, A.z, A.w}, b[4] = {B.x, B.y, B.z, B.w}, q[4] = {Q.x, Q.y, Q.z, Q.w};
  __half* dst = out + row * (size_t)(W.nb * QK) + q6_unit_base(u);
#pragma unroll
  for (int t = 0; t < 4; t++) {
    uint32_t w[4];
    q6_words(a[t], b[t], q[t], w[0], w[1], w[2], w[3]);
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const float sc = sc_val(scw, m);
#pragma unroll
      for (int j = 0; j < 4; j++) dst[32 * m + 4 * t + j] = __float2half_rn(sc * q6_val(w[m], j));
    }
  }
}

// Activation operand. Block i handles source row i / x_div of X and writes
// operand row r = rowof[i] (dense: r = i, x_div = 1) of the hi half and row
// rpad + r of the lo half, after scaling the row by a power of two that
// brings its largest magnitude into [2^13, 2^14); inv[r] undoes the scaling.
// With `up`, the row is first the SwiGLU product silu(X) * up (the
// reference's swiglu kernel, kernels.rs:543-550, same float operations).
// Operand rows that no block writes (tile padding) feed only output columns
// that are never stored.
__global__ void __launch_bounds__(256) k_tc_split(const float* X, const float* up, int ldx, int K, int x_div,
                                                  const int* rowof, int rpad, __half* xg, float* inv, int per) {
  // slots [i0, i0 + per) share one source row (per == x_div or 1): it is read,
  // its scale found and its hi/lo pair computed once, then written per slot
  extern __shared__ float4 srow[];  // the row (K floats)
  const int i0 = blockIdx.x * per;
  const size_t src = (size_t)(i0 / x_div) * ldx;
  const float4* xr = (const float4*)(X + src);
  const float4* ur = up ? (const float4*)(up + src) : nullptr;
  __shared__ float red[8];
  float mx = 0.f;
  for (int k = threadIdx.x; k < K / 4; k += 256) {
    float4 v = xr[k];
    if (ur) {
      const float4 u = ur[k];
      v = make_float4(silu_mul(v.x, u.x), silu_mul(v.y, u.y), silu_mul(v.z, u.z), silu_mul(v.w, u.w));
    }
    srow[k] = v;
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
  int ex = 0;
  if (mx > 0.f && mx < 3.0e38f) {
    frexpf(mx, &ex);  // mx < 2^ex
    ex = min(max(14 - ex, -100), 100);
  } else {
    ex = 0;
  }
  const float sc = ldexpf(1.f, ex);
  for (int k = threadIdx.x; k < K / 4; k += 256) {
    const float4 v = srow[k];
    const float f[4] = {v.x * sc, v.y * sc, v.z * sc, v.w * sc};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      h[j] = __float2half_rn(f[j]);
      l[j] = __float2half_rn(f[j] - __half2float(h[j]));
    }
    const __half2 h01 = __halves2half2(h[0], h[1]), h23 = __halves2half2(h[2], h[3]);
    const __half2 l01 = __halves2half2(l[0], l[1]), l23 = __halves2half2(l[2], l[3]);
    const uint2 hv = make_uint2(*(const uint32_t*)&h01, *(const uint32_t*)&h23);
    const uint2 lv = make_uint2(*(const uint32_t*)&l01, *(const uint32_t*)&l23);
    for (int q = 0; q < per; q++) {
      const int r = rowof ? rowof[i0 + q] : i0 + q;
      if (r < 0 || r >= rpad) continue;  // a slot whose expert id was out of range has no row
      *(uint2*)(xg + (size_t)r * K + 4 * k) = hv;
      *(uint2*)(xg + ((size_t)rpad + r) * K + 4 * k) = lv;
    }
  }
  if (threadIdx.x < per) {
    const int r = rowof ? rowof[i0 + threadIdx.x] : i0 + threadIdx.x;
    if (r >= 0 && r < rpad) inv[r] = ldexpf(1.f, -ex);
  }
}

// RMSNorm fused with the dense operand split (rows of DIM): the normalised
// row x * (1 / sqrt(mean(x^2) + eps)) * w is written to `normed` (fp32) and
// split into the hi/lo operand like k_tc_split. Thread t holds elements
// t + 256 i (i < 8) in registers from the first load to the last store; the
// sum of squares runs over them in that order, then over the warps.
__global__ void __launch_bounds__(256) k_tc_split_norm(const float* __restrict__ X, const float* __restrict__ w,
                                                       float eps, float* __restrict__ normed, int rpad,
                                                       __half* __restrict__ xg, float* __restrict__ inv) {
  constexpr int PER = DIM / 256;
  __shared__ float red[8], redm[8];
  const int r = blockIdx.x, t = threadIdx.x;
  const float* xr = X + (size_t)r * DIM;
  float v[PER], g[PER];
#pragma unroll
  for (int i = 0; i < PER; i++) {
    v[i] = xr[t + 256 * i];
    g[i] = __ldg(w + t + 256 * i);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; i++) tot += red[i];
  const float rinv = 1.0f / sqrtf(tot / (float)DIM + eps);
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    v[i] = v[i] * rinv * g[i];
    normed[(size_t)r * DIM + t + 256 * i] = v[i];
    mx = fmaxf(mx, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((t & 31) == 0) redm[t >> 5] = mx;
  __syncthreads();
  mx = redm[0];
#pragma unroll
  for (int i = 1; i < 8; i++) mx = fmaxf(mx, redm[i]);
  int ex = 0;
  if (mx > 0.f && mx < 3.0e38f) {
    frexpf(mx, &ex);
    ex = min(max(14 - ex, -100), 100);
  } else {
    ex = 0;
  }
  const float sc = ldexpf(1.f, ex);
  __half* hi = xg + (size_t)r * DIM;
  __half* lo = xg + ((size_t)rpad + r) * DIM;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const float f = v[i] * sc;
    const __half h = __float2half_rn(f);
    hi[t + 256 * i] = h;
    lo[t + 256 * i] = __float2half_rn(f - __half2float(h));
  }
  if (t == 0) inv[r] = ldexpf(1.f, -ex);
}

// Split-K partials -> output, the splits summed in order (deterministic):
// out[t * ldo + o] (+)= sum_s part[s][t][o].
__global__ void k_tc_reduce(const float* part, int ksplit, int n, int rows, float* out, int ldo, int resid) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)n * rows) return;
  const int t = (int)(i / rows), o = (int)(i % rows);
  float v = part[i];
  for (int s = 1; s < ksplit; s++) v += part[(size_t)s * n * rows + i];
  float* dst = out + (size_t)t * ldo + o;
  *dst = resid ? *dst + v : v;
}

// Grouped layout from the expert lists (groups[e * (cap + 1)] = count, then
// the selection slots): experts' rows start at tt-aligned bases; tiles =
// {count, (expert, first row) ...}; slots[row] = selection slot or -1;
// rowof[slot] = operand row (the caller clears rowof to -1 first). Every
// block scans the 32 counts in warp 0, then the grid places the rows: row r
// belongs to the expert whose padded range holds it and is either that
// expert's entry r - base or padding. Each output word has one writer, so the
// blocks need no ordering.
__global__ void __launch_bounds__(256) k_tc_group_tiles(const int* groups, int cap, int* tiles, int* slots,
                                                        int* rowof, int rpad, int tt) {
  __shared__ int base[N_EXPERT + 1], first[N_EXPERT + 1], tile0[N_EXPERT + 1];
  const int t = threadIdx.x, lane = t & 31;
  if (t < 32) {
    const int cnt = lane < N_EXPERT ? groups[(size_t)lane * (cap + 1)] : 0;
    const int nt = (cnt + tt - 1) / tt;
    // inclusive scans of the padded rows, the entries and the tiles
    int rows = nt * tt, ent = cnt, til = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int r2 = __shfl_up_sync(0xffffffffu, rows, o), e2 = __shfl_up_sync(0xffffffffu, ent, o),
                t2 = __shfl_up_sync(0xffffffffu, til, o);
      if (lane >= o) rows += r2, ent += e2, til += t2;
    }
    if (lane < N_EXPERT) {
      base[lane + 1] = rows;
      first[lane + 1] = ent;
      tile0[lane + 1] = til;
    }
    if (lane == 0) base[0] = first[0] = tile0[0] = 0;
  }
  __syncthreads();
  const int gt = blockIdx.x * blockDim.x + t, gs = gridDim.x * blockDim.x;
  const int ntiles = tile0[N_EXPERT], nrows = base[N_EXPERT];
  if (gt == 0) tiles[0] = ntiles;
  for (int i = gt; i < ntiles; i += gs) {
    int e = 0;
    while (tile0[e + 1] <= i) e++;
    tiles[1 + 2 * i] = e;
    tiles[2 + 2 * i] = base[e] + tt * (i - tile0[e]);
  }
  for (int r = gt; r < rpad; r += gs) {
    int v = -1;
    if (r < nrows) {
      int lo = 0, hi = N_EXPERT - 1;  // the last expert e with base[e] <= r (empty experts share a base)
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (base[mid] <= r) lo = mid;
        else hi = mid - 1;
      }
      const int i = r - base[lo];
      if (i < first[lo + 1] - first[lo]) {
        v = groups[(size_t)lo * (cap + 1) + 1 + i];
        rowof[v] = r;
      }
    }
    slots[r] = v;
  }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeFn)p;
  });
  return fn;
}

}  // namespace

// K-major fp16 matrix [rows][K] as a TMA tensor map with a (64 x box_rows) box.
cudaError_t tc_map_f16(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (((uintptr_t)base & 15) || (K * 2) % 16) return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)TK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The hi/lo activation operand (hi rows [0, rpad), lo rows [rpad, 2 rpad), K
// fp16 each) as a 3-D map (K, row, hi|lo) whose (64 x box_rows x 2) box brings a
// chunk's hi rows and lo rows in one load, laid out in shared memory exactly as
// two 2-D loads would (hi rows, then lo rows; box_rows a multiple of 8 keeps
// the 128-byte swizzle pattern of the lo half the same).
cudaError_t tc_map_hilo(CUtensorMap* map, const void* base, int rpad, int K, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (((uintptr_t)base & 15) || (K * 2) % 16 || box_rows % 8) return cudaErrorInvalidValue;
  const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rpad, 2};
  const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)rpad * K * 2};
  const cuuint32_t box[3] = {(cuuint32_t)TK, (cuuint32_t)box_rows, 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t tc_gemm_f16(const __half* A, const __half* B, int M, int N, int K, float* C, unsigned* err,
                        cudaStream_t s) {
  if (M % TM || N % TN || K % TK || K <= 0) return cudaErrorInvalidValue;
  CUtensorMap ma, mb;
  cudaError_t e = tc_map_f16(&ma, A, M, K, TM);
  if (e != cudaSuccess) return e;
  e = tc_map_f16(&mb, B, N, K, TN);
  if (e != cudaSuccess) return e;
  const int smem = STAGES * STAGE_BYTES + 1024;
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu, [smem] { cudaFuncSetAttribute(k_tc_f16, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
  k_tc_f16<<<dim3(M / TM, N / TN), THREADS, smem, s>>>(ma, mb, C, M, N, K, err);
  return cudaGetLastError();
}

cudaError_t tc_gemm_f16_bmn(const __half* A, const __half* B, int M, int K, float* C, unsigned* err,
                            cudaStream_t s) {
  if (M % TM || K % TK || K <= 0) return cudaErrorInvalidValue;
  CUtensorMap ma, mb;
  cudaError_t e = tc_map_f16(&ma, A, M, K, TM);
  if (e != cudaSuccess) return e;
  e = tc_map_f16(&mb, B, K, BN_N, TK);  // B [K][64]: 64-wide rows, 64-row boxes
  if (e != cudaSuccess) return e;
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu,
                  [] { cudaFuncSetAttribute(k_tc_f16_bmn, cudaFuncAttributeMaxDynamicSharedMemorySize, BMN_SMEM); });
  k_tc_f16_bmn<<<M / TM, THREADS, BMN_SMEM, s>>>(ma, mb, C, M, K, err);
  return cudaGetLastError();
}


namespace {
cudaError_t map_raw(CUtensorMap* mq, CUtensorMap* ms, const Q6Mat& W) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const int U = 4 * W.nb;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)U * 16, 3, (cuuint64_t)W.rows};
    const cuuint64_t strides[2] = {(cuuint64_t)U * 16, (cuuint64_t)U * 48};
    const cuuint32_t box[3] = {32, 3, 128};  // half a super-block: 2 units x 3 pieces x 128 rows
    const cuuint32_t estr[3] = {1, 1, 1};
    if (fn(mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)W.q, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)U * 4, (cuuint64_t)W.rows};
    const cuuint64_t strides[1] = {(cuuint64_t)U * 4};
    const cuuint32_t box[2] = {16, 128};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)W.sc, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

// Token tile of a GEMM over n tokens: the smallest of 16/32/64/128 that holds
// them (dense) or the average expert's share of them (grouped); every
// activation row a tile loads is streamed once per 128 weight rows, so small
// batches use narrow tiles.
int tile_tokens(int per_tile) { return per_tile <= 16 ? 16 : (per_tile <= 32 ? 32 : (per_tile <= 64 ? 64 : 128)); }
int dense_tt(int n) { return tile_tokens(n); }
int grouped_tt(int n) { return tile_tokens((n * N_USED + N_EXPERT - 1) / N_EXPERT); }
int dense_rpad(int n) { const int tt = dense_tt(n); return (n + tt - 1) / tt * tt; }
int grouped_rpad(int n) { return (int)tc_scratch_rows(n); }

bool fits(const TcScratch& sc, int rpad, int K) {
  return sc.xg && (size_t)rpad <= sc.rows && 2 * (size_t)rpad * (size_t)K <= sc.halves;
}

template <int TT>
cudaError_t launch_q6_tt(const CUtensorMap& mq, const CUtensorMap& ms, const CUtensorMap& mx, dim3 grid,
                         const TcQ6Params& p, cudaStream_t s) {
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu,
                  [] { cudaFuncSetAttribute(k_tc_q6<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, q_smem(TT)); });
  k_tc_q6<TT><<<grid, QTHREADS, q_smem(TT), s>>>(mq, ms, mx, p);
  return cudaGetLastError();
}

template <int TT>
cudaError_t launch_q6x_tt(const CUtensorMap& ma, const CUtensorMap& mx, dim3 grid, const TcQ6Params& p,
                          cudaStream_t s) {
  static unsigned long long done = 0;
  static std::mutex mu;
  once_per_device(done, mu,
                  [] { cudaFuncSetAttribute(k_tc_q6x<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, x_smem(TT)); });
  k_tc_q6x<TT><<<grid, XTHREADS, x_smem(TT), s>>>(ma, mx, p);
  return cudaGetLastError();
}

// Pairs of the 2-SM kernel that fit on the device at once (per device, once).
int x2_max_pairs() {
  static int cached[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  if (cudaFuncSetAttribute(k_tc_q6x2, cudaFuncAttributeMaxDynamicSharedMemorySize, X2_SMEM) == cudaSuccess &&
      cudaFuncSetAttribute(k_tc_q6x2, cudaFuncAttributeNonPortableClusterSizeAllowed, 0) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(XTHREADS, 1, 1);
    cfg.dynamicSmemBytes = X2_SMEM;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, k_tc_q6x2, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  n = n > 0 ? n : -1;  // -1: the 2-SM kernel cannot run here
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

// LFM_PREFILL_2SM=1 moves 128-token tiles to the 2-SM kernel. Off by default:
// measured on the prompt path it is bit-identical and slower (3840 tokens
// 31.4-31.9 vs 29.8-30.5 ms, 1024 tokens 12.1 vs 11.2 ms, both kernels with
// their weight loads in a warp of their own).
bool x2_enabled() {
  static const bool on = [] {
    const char* v = getenv("LFM_PREFILL_2SM");
    return v && std::string(v) == "1";
  }();
  return on;
}

cudaError_t launch_q6x2(const CUtensorMap& ma, const CUtensorMap& mx, int pairs, const TcQ6Params& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(XTHREADS, 1, 1);
  cfg.dynamicSmemBytes = X2_SMEM;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_tc_q6x2, ma, mx, p);
}

// the expanded-weight kernel when x16 (the load-time fp16 A operand of W) is given
cudaError_t launch_q6(const Q6Mat& W, int rpad, int tt, int ntiles_y, const TcQ6Params& p, const TcScratch& sc,
                      cudaStream_t s, const __half* x16 = nullptr) {
  if (x16 && tt == 128 && p.out_rows % 256 == 0 && x2_enabled() && x2_max_pairs() > 0) {
    CUtensorMap ma, mx;
    cudaError_t e = tc_map_f16(&ma, x16, W.rows, W.nb * QK, 128);
    if (e != cudaSuccess) return e;
    e = tc_map_f16(&mx, sc.xg, 2 * rpad, W.nb * QK, 128);
    if (e != cudaSuccess) return e;
    TcQ6Params q = p;
    q.tiles_y = ntiles_y;
    const long long ntile = (long long)(p.out_rows / 256) * ntiles_y * p.ksplit;
    const int pairs = (int)std::min<long long>(ntile, x2_max_pairs());
    return launch_q6x2(ma, mx, pairs, q, s);
  }
  if (x16) {
    CUtensorMap ma, mx;
    cudaError_t e = tc_map_f16(&ma, x16, W.rows, W.nb * QK, 128);
    if (e != cudaSuccess) return e;
    e = tc_map_hilo(&mx, sc.xg, rpad, W.nb * QK, tt);
    if (e != cudaSuccess) return e;
    // persistent: at most one wave of CTAs walks every tile
    TcQ6Params q = p;
    q.tiles_y = ntiles_y;
    const long long ntile = (long long)(p.out_rows / 128) * ntiles_y * p.ksplit;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const dim3 grid((unsigned)std::min<long long>(ntile, (long long)sms * q_ctas_per_sm(tt)));
    switch (tt) {
      case 16: return launch_q6x_tt<16>(ma, mx, grid, q, s);
      case 32: return launch_q6x_tt<32>(ma, mx, grid, q, s);
      case 64: return launch_q6x_tt<64>(ma, mx, grid, q, s);
      case 128: return launch_q6x_tt<128>(ma, mx, grid, q, s);
      default: return cudaErrorInvalidValue;
    }
  }
  CUtensorMap mq, ms, mx;
  cudaError_t e = map_raw(&mq, &ms, W);
  if (e != cudaSuccess) return e;
  e = tc_map_hilo(&mx, sc.xg, rpad, W.nb * QK, tt);
  if (e != cudaSuccess) return e;
  const dim3 grid(p.out_rows / 128, ntiles_y, p.ksplit);
  switch (tt) {
    case 16: return launch_q6_tt<16>(mq, ms, mx, grid, p, s);
    case 32: return launch_q6_tt<32>(mq, ms, mx, grid, p, s);
    case 64: return launch_q6_tt<64>(mq, ms, mx, grid, p, s);
    case 128: return launch_q6_tt<128>(mq, ms, mx, grid, p, s);
    default: return cudaErrorInvalidValue;
  }
}
}  // namespace

bool tc_q6_supported(const Q6Mat& W, int out_rows) {
  return out_rows > 0 && out_rows % 128 == 0 && W.rows % out_rows == 0 && W.nb > 0 && encode_fn() != nullptr;
}

size_t tc_scratch_rows(int n) { return (size_t)n * N_USED + (size_t)N_EXPERT * 128 + 128; }

cudaError_t tc_split(const float* X, int ldx, int K, int n, const TcScratch& sc, cudaStream_t s, const float* up) {
  const int rpad = dense_rpad(n);
  if (n <= 0 || K % 64 || K > TC_SPLIT_KMAX || ldx % 4 || !fits(sc, rpad, K)) return cudaErrorInvalidValue;
  k_tc_split<<<n, 256, K * 4, s>>>(X, up, ldx, K, 1, nullptr, rpad, sc.xg, sc.inv, 1);
  return cudaGetLastError();
}

cudaError_t tc_split_norm(const float* X, const float* w, float eps, int n, float* normed, const TcScratch& sc,
                          cudaStream_t s) {
  const int rpad = dense_rpad(n);
  if (n <= 0 || !fits(sc, rpad, DIM)) return cudaErrorInvalidValue;
  k_tc_split_norm<<<n, 256, 0, s>>>(X, w, eps, normed, rpad, sc.xg, sc.inv);
  return cudaGetLastError();
}

cudaError_t q6_expand_f16(const Q6Mat& W, __half* out, cudaStream_t s) {
  const size_t units = (size_t)W.rows * 4 * W.nb;
  if (!out || units == 0) return cudaErrorInvalidValue;
  k_q6_expand_f16<<<(unsigned)((units + 255) / 256), 256, 0, s>>>(W, out);
  return cudaGetLastError();
}

cudaError_t tc_gemm_q6(const Q6Mat& W, int n, float* out, int ldo, bool resid, const TcScratch& sc,
                       cudaStream_t s, const __half* x16) {
  const int rpad = dense_rpad(n);
  if (n <= 0 || !fits(sc, rpad, W.nb * QK) || !tc_q6_supported(W, W.rows)) return cudaErrorInvalidValue;
  TcQ6Params p = {};
  p.W = W;
  p.out_rows = W.rows;
  p.rpad = rpad;
  p.inv = sc.inv;
  p.out = out;
  p.ldo = ldo;
  p.resid = resid ? 1 : 0;
  p.ntok = n;
  p.err = sc.err;
  p.ksplit = 1;
  // A single token tile leaves most SMs idle on the narrow matrices: split the
  // super-blocks over up to ~2 CTAs per SM and reduce the partials in order.
  const int tt = dense_tt(n);
  const int ctas = (W.rows / 128) * (rpad / tt);
  if (rpad == tt && sc.part && ctas < 148) {
    int ks = std::min(std::min(W.nb, 16), (296 + ctas - 1) / ctas);
    while (ks > 1 && (size_t)ks * n * W.rows > sc.part_cap) ks--;
    if (ks > 1) {
      p.ksplit = ks;
      p.part = sc.part;
      cudaError_t e = launch_q6(W, rpad, tt, 1, p, sc, s, x16);
      if (e != cudaSuccess) return e;
      const size_t cnt = (size_t)n * W.rows;
      k_tc_reduce<<<(unsigned)((cnt + 255) / 256), 256, 0, s>>>(sc.part, ks, n, W.rows, out, ldo, resid ? 1 : 0);
      return cudaGetLastError();
    }
  }
  return launch_q6(W, rpad, tt, rpad / tt, p, sc, s, x16);
}

cudaError_t tc_group(const int* groups, int cap, int n, const TcScratch& sc, cudaStream_t s) {
  const int rpad = grouped_rpad(n);
  if (n <= 0 || (size_t)rpad > sc.rows || !sc.tiles || !sc.slots || !sc.rowof) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(sc.rowof, 0xFF, (size_t)n * N_USED * sizeof(int), s);  // rowof = -1
  if (e != cudaSuccess) return e;
  const int grid = std::min((rpad + 255) / 256, 148);
  k_tc_group_tiles<<<grid, 256, 0, s>>>(groups, cap, sc.tiles, sc.slots, sc.rowof, rpad, grouped_tt(n));
  return cudaGetLastError();
}

cudaError_t tc_split_grouped(const float* X, int K, int x_div, int n, const TcScratch& sc, cudaStream_t s,
                             const float* up) {
  const int rpad = grouped_rpad(n);
  if (n <= 0 || K % 64 || K > TC_SPLIT_KMAX || x_div <= 0 || !fits(sc, rpad, K)) return cudaErrorInvalidValue;
  // one CTA per source row: the N_USED slots of a token share it when x_div == N_USED
  const int per = x_div == N_USED ? N_USED : 1;
  k_tc_split<<<n * N_USED / per, 256, K * 4, s>>>(X, up, K, K, x_div, sc.rowof, rpad, sc.xg, sc.inv, per);
  return cudaGetLastError();
}

cudaError_t tc_gemm_q6_grouped(const Q6Mat& W, int out_rows, int n, float* out, const TcScratch& sc,
                               cudaStream_t s, const __half* x16) {
  const int rpad = grouped_rpad(n);
  if (n <= 0 || !fits(sc, rpad, W.nb * QK) || !tc_q6_supported(W, out_rows) || W.rows / out_rows > N_EXPERT)
    return cudaErrorInvalidValue;
  TcQ6Params p = {};
  p.W = W;
  p.out_rows = out_rows;
  p.rpad = rpad;
  p.inv = sc.inv;
  p.out = out;
  p.ldo = out_rows;
  p.tiles = sc.tiles;
  p.slots = sc.slots;
  p.grouped = 1;
  p.err = sc.err;
  p.ksplit = 1;
  return launch_q6(W, rpad, grouped_tt(n), tc_max_tiles(n), p, sc, s, x16);
}

int tc_max_tiles(int n) {
  const int tt = grouped_tt(n);
  return (n * N_USED + tt - 1) / tt + N_EXPERT;
}

int tc_max_tiles_cap(int n) { return std::max(2 * N_EXPERT, (n * N_USED + 127) / 128 + N_EXPERT); }

}  // namespace lfm
