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

#include <mutex>

#include "dev_common.cuh"
#include "tc_gemm.h"

namespace lfm {
namespace {
using namespace dev;

constexpr int TM = 128, TN = 256, TK = 64;  // tile and K chunk
constexpr int STAGES = 4;
constexpr int A_BYTES = TM * TK * 2;        // 16 KB
constexpr int B_BYTES = TN * TK * 2;        // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 6 * 32;
constexpr uint32_t TMEM_COLS = 256;

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);          // start address
  d |= (uint64_t)1 << 16;                           // leading byte offset (unused with swizzle): 16 B
  d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: 8-row group = 1024 B
  d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                           // layout: 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, both K-major.
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(IDESC), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

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
        mma_f16(tmem, smem_desc_sw128(a + kk * 32), smem_desc_sw128(b + kk * 32), (kc | kk) ? 1u : 0u);
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

cudaError_t tc_gemm_f16(const __half* A, const __half* B, int M, int N, int K, float* C, unsigned* err,
                        cudaStream_t s) {
  if (M % TM || N % TN || K % TK || K <= 0) return cudaErrorInvalidValue;
  CUtensorMap ma, mb;
  cudaError_t e = tc_map_f16(&ma, A, M, K, TM);
  if (e != cudaSuccess) return e;
  e = tc_map_f16(&mb, B, N, K, TN);
  if (e != cudaSuccess) return e;
  const int smem = STAGES * STAGE_BYTES + 1024;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_tc_f16, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  k_tc_f16<<<dim3(M / TM, N / TN), THREADS, smem, s>>>(ma, mb, C, M, N, K, err);
  return cudaGetLastError();
}

}  // namespace lfm
