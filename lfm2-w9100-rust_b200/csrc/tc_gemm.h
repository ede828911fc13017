// Tensor-core (tcgen05) GEMM pieces of the prompt path. See tc_gemm.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"

namespace lfm {

// K-major fp16 matrix [rows][K] as a TMA tensor map (64-wide K box, 128-byte swizzle).
cudaError_t tc_map_f16(CUtensorMap* map, const void* base, int rows, int K, int box_rows);
// C[m][n] = sum_k A[m][k] B[n][k]; fp16 A [M][K], B [N][K], fp32 C [M][N].
// M % 128 == 0, N % 256 == 0, K % 64 == 0. *err is raised if a wait timed out.
cudaError_t tc_gemm_f16(const __half* A, const __half* B, int M, int N, int K, float* C, unsigned* err,
                        cudaStream_t s);
// C[m][n] = sum_k A[m][k] B[k][n] for fp16 A [M][K] and B [K][64] (B
// MN-major: rows of 64 contiguous values), fp32 C [M][64]. M % 128 == 0,
// K % 64 == 0.
cudaError_t tc_gemm_f16_bmn(const __half* A, const __half* B, int M, int K, float* C, unsigned* err,
                            cudaStream_t s);

// Causal GQA prompt attention on the tensor cores for tokens [0, n) at
// positions start.. (q of token j, head h at q + j*q_stride + h*64; K/V cache
// [8][ctx][64] fp16 already holding positions 0..start+n-1); output at
// out + j*out_stride + h*64. With start_dev the kernel reads the first
// position from device memory (it must equal `start`, which the host checks).
cudaError_t attn_prefill_tc(const float* q, int q_stride, const __half* kc, const __half* vc, int start, int n,
                            int ctx, float* out, int out_stride, unsigned* err, cudaStream_t s,
                            const int* start_dev = nullptr);

// Scratch of the Q6_K prompt GEMMs (engine-owned device memory): the hi/lo
// activation operand, per-row inverse scales, and the grouped tile table,
// row -> slot and slot -> row maps.
struct TcScratch {
  __half* xg = nullptr;  // hi rows [0, rpad) then lo rows [rpad, 2 rpad), K halves each
  float* inv = nullptr;  // [rows]
  int* tiles = nullptr;  // [1 + 2 * tc_max_tiles_cap(n)]
  int* slots = nullptr;  // [rows]
  int* rowof = nullptr;  // [n * N_USED]
  unsigned* err = nullptr;
  float* part = nullptr; // split-K partial sums of single-tile GEMMs (optional)
  size_t part_cap = 0;   // floats
  size_t rows = 0;       // operand rows (tc_scratch_rows of the largest n)
  size_t halves = 0;     // capacity of xg
};
// Operand rows needed for n tokens in the grouped case (n * 4 selection slots
// plus 128-row padding per expert); the dense case needs n rounded up to 128.
size_t tc_scratch_rows(int n);
// Most token tiles a grouped GEMM of n tokens can have, and the most of any
// GEMM of at most n tokens (the tile table's capacity).
int tc_max_tiles(int n);
int tc_max_tiles_cap(int n);
// The tensor-core path serves this matrix: 128-row output tiles.
bool tc_q6_supported(const Q6Mat& W, int out_rows);

// Dense: split rows [0, n) of X (row stride ldx, K columns) into the operand,
// then out[t * ldo + o] (+)= sum_k W[o][k] X[t][k] for t < n, o < W.rows. One
// split serves every GEMM on the same activations (q, k and v; gate and up).
// With `up` (same layout as X), the rows are the SwiGLU products silu(X) * up.
constexpr int TC_SPLIT_KMAX = 12288;  // row length held in shared memory
cudaError_t tc_split(const float* X, int ldx, int K, int n, const TcScratch& sc, cudaStream_t s,
                     const float* up = nullptr);
// RMSNorm of rows [0, n) of X [n][2048] with weights w into `normed` (fp32),
// fused with the split of the normalised rows into the operand.
cudaError_t tc_split_norm(const float* X, const float* w, float eps, int n, float* normed, const TcScratch& sc,
                          cudaStream_t s);
// x16 (optional): W expanded at load time into its fp16 A operand
// (q6_expand_f16); the GEMM then loads A by TMA instead of dequantising on chip.
cudaError_t tc_gemm_q6(const Q6Mat& W, int n, float* out, int ldo, bool resid, const TcScratch& sc,
                       cudaStream_t s, const __half* x16 = nullptr);
// The fp16 A operand of W's prompt GEMMs: out[row][k] = fp16(sc * (q - 32))
// ([W.rows][W.nb * 256], 2 bytes per weight).
cudaError_t q6_expand_f16(const Q6Mat& W, __half* out, cudaStream_t s);

// Routed experts: tc_group lays out the expert lists (groups[e * (cap + 1)] =
// count, then selection slots t * 4 + rank), tc_split_grouped fills operand
// row of slot q with X[q / x_div], and the GEMM writes, for expert e and each
// of its slots, out[slot * out_rows + o] = sum_k W[e * out_rows + o][k] X[..][k].
cudaError_t tc_group(const int* groups, int cap, int n, const TcScratch& sc, cudaStream_t s);
cudaError_t tc_split_grouped(const float* X, int K, int x_div, int n, const TcScratch& sc, cudaStream_t s,
                             const float* up = nullptr);
cudaError_t tc_gemm_q6_grouped(const Q6Mat& W, int out_rows, int n, float* out, const TcScratch& sc,
                               cudaStream_t s, const __half* x16 = nullptr);

}  // namespace lfm
