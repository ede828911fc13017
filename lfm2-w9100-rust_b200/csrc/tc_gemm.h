// Tensor-core (tcgen05) GEMM pieces of the prompt path. See tc_gemm.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace lfm {

// K-major fp16 matrix [rows][K] as a TMA tensor map (64-wide K box, 128-byte swizzle).
cudaError_t tc_map_f16(CUtensorMap* map, const void* base, int rows, int K, int box_rows);
// C[m][n] = sum_k A[m][k] B[n][k]; fp16 A [M][K], B [N][K], fp32 C [M][N].
// M % 128 == 0, N % 256 == 0, K % 64 == 0. *err is raised if a wait timed out.
cudaError_t tc_gemm_f16(const __half* A, const __half* B, int M, int N, int K, float* C, unsigned* err,
                        cudaStream_t s);

}  // namespace lfm
