// Q6_K device layout and the device-side dequant arithmetic.
//
// GGUF stores a Q6_K matrix [in, rows] as rows of in/256 super-blocks of 210
// bytes: ql[128] qh[64] int8 scales[16] fp16 d (engine/src/q6k.rs:8-17).
// 210 is not a multiple of 16, so rows cannot be read with aligned 128-bit
// loads. At load time every block is split into "units" of 64 weights, and the
// bytes of a unit are stored so that one warp lane reads one unit with three
// coalesced 16-byte loads. Every original byte is kept and nothing is padded:
// the device copy is exactly rows * in/256 * 210 bytes, like the reference's
// own load-time repack (q6k.rs:25-39) but without its two pad bytes.
//
// Unit u = 4*b + 2*h + qq of a row covers block b, half h (elements
// h*128..h*128+127) and l in [16*qq, 16*qq+16). Element l + 32*m (m = 0..3)
// of that half is (q6k.rs:104-146):
//   m=0: low  nibble of ql[h*64 + l],      qh[h*32 + l] bits 0-1, scale sc[h*8 + qq + 0]
//   m=1: low  nibble of ql[h*64 + 32 + l], qh bits 2-3,           scale sc[h*8 + qq + 2]
//   m=2: high nibble of ql[h*64 + l],      qh bits 4-5,           scale sc[h*8 + qq + 4]
//   m=3: high nibble of ql[h*64 + 32 + l], qh bits 6-7,           scale sc[h*8 + qq + 6]
// Planes of one matrix (row-major, U = 4*nb units per row):
//   Q : [rows][3][U] x 16 B   piece 0 = ql[h*64+16qq .. +16], piece 1 = ql[h*64+32+16qq .. +16],
//                             piece 2 = qh[h*32+16qq .. +16]
//   SC: [rows][U]    x 4 B    the unit's four int8 scales, m = 0..3
//   D : [rows][nb]   x 2 B    fp16 d
// The weight value is d * sc_m * (q6 - 32), which is exact in f32 for every
// input (11 + 7 + 5 significant bits), so any evaluation order reproduces the
// reference's `d * s * q` bit for bit.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace lfm {

constexpr int QK = 256;
constexpr int QB = 210;

struct Q6Mat {
  const uint4* q;      // [rows][3][U]
  const uint32_t* sc;  // [rows][U]
  const __half* d;     // [rows][nb]
  int rows;
  int nb;
};

// Plane offsets inside one contiguous allocation of a [nb*256, rows] matrix.
__host__ __device__ inline size_t q6_q_bytes(size_t rows, int nb) { return rows * (size_t)nb * 192; }
__host__ __device__ inline size_t q6_sc_bytes(size_t rows, int nb) { return rows * (size_t)nb * 16; }
__host__ __device__ inline size_t q6_total_bytes(size_t rows, int nb) { return rows * (size_t)nb * QB; }

inline Q6Mat q6_view(const void* base, int rows, int nb) {
  const uint8_t* p = (const uint8_t*)base;
  Q6Mat m;
  m.q = (const uint4*)p;
  m.sc = (const uint32_t*)(p + q6_q_bytes(rows, nb));
  m.d = (const __half*)(p + q6_q_bytes(rows, nb) + q6_sc_bytes(rows, nb));
  m.rows = rows;
  m.nb = nb;
  return m;
}

// Host repack of GGUF rows [row0, row0 + nrows) (src points at row0's first
// block) into the planes of a matrix with `rows` rows starting at `dst`.
inline void q6_repack_rows(const uint8_t* src, size_t row0, size_t nrows, int nb, size_t rows,
                           uint8_t* dst) {
  const int U = 4 * nb;
  uint8_t* Q = dst;
  uint8_t* SC = dst + q6_q_bytes(rows, nb);
  uint8_t* D = SC + q6_sc_bytes(rows, nb);
  for (size_t r = 0; r < nrows; r++) {
    const size_t row = row0 + r;
    uint8_t* q = Q + row * (size_t)U * 48;
    uint8_t* sc = SC + row * (size_t)U * 4;
    uint8_t* d = D + row * (size_t)nb * 2;
    for (int b = 0; b < nb; b++) {
      const uint8_t* blk = src + (r * nb + b) * (size_t)QB;
      for (int h = 0; h < 2; h++)
        for (int qq = 0; qq < 2; qq++) {
          const int u = 4 * b + 2 * h + qq;
          for (int i = 0; i < 16; i++) {
            q[(0 * U + u) * 16 + i] = blk[h * 64 + 16 * qq + i];
            q[(1 * U + u) * 16 + i] = blk[h * 64 + 32 + 16 * qq + i];
            q[(2 * U + u) * 16 + i] = blk[128 + h * 32 + 16 * qq + i];
          }
          for (int m = 0; m < 4; m++) sc[u * 4 + m] = blk[192 + h * 8 + qq + 2 * m];
        }
      d[2 * b] = blk[208];
      d[2 * b + 1] = blk[209];
    }
  }
}

#ifdef __CUDACC__
// The four words of 6-bit codes (one byte per element, elements 4t..4t+3 of
// the unit's 16-l run) for m = 0..3.
__device__ __forceinline__ void q6_words(uint32_t a, uint32_t b, uint32_t q, uint32_t& w0,
                                         uint32_t& w1, uint32_t& w2, uint32_t& w3) {
  w0 = (a & 0x0F0F0F0Fu) | ((q << 4) & 0x30303030u);
  w1 = (b & 0x0F0F0F0Fu) | ((q << 2) & 0x30303030u);
  w2 = ((a >> 4) & 0x0F0F0F0Fu) | (q & 0x30303030u);
  w3 = ((b >> 4) & 0x0F0F0F0Fu) | ((q >> 2) & 0x30303030u);
}

// Byte j of w (a 6-bit code c) as the float c - 32, exactly: the byte is
// placed in the mantissa of 2^23 (0x4B000000) and 2^23 + 32 is subtracted.
__device__ __forceinline__ float q6_val(uint32_t w, int j) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)j)) - 8388640.0f;
}

__device__ __forceinline__ float sc_val(uint32_t scw, int m) {
  return (float)(int8_t)(uint8_t)(scw >> (8 * m));
}

// Packed fp32x2 arithmetic of sm_100 (two IEEE fp32 lanes per instruction,
// same rounding as the scalar forms).
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rr;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rr, ra, rb;\n mov.b64 {%0, %1}, rr;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rc, rr;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rr, ra, rb, rc;\n mov.b64 {%0, %1}, rr;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}
// Bytes j, j+1 of w as the exact floats (c - 32) (magic 2^23 mantissa trick).
__device__ __forceinline__ float2 q6_val2(uint32_t w, int j) {
  const float2 m = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)j)),
                               __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)(j + 1))));
  return f2_add(m, make_float2(-8388640.0f, -8388640.0f));
}

// Dot of one unit with the 64 activations x[m*16 + i] (element l0+i+32m of the
// unit's half). Returns sum_m (d*sc_m) * sum_i (q6-32)*x, with the inner sums
// in fp32x2 pairs (even / odd i) added at the end.
__device__ __forceinline__ float q6_unit_dot(const uint4& A, const uint4& B, const uint4& Q,
                                             uint32_t scw, float d, const float* x) {
  const uint32_t a[4] = {A.x, A.y, A.z, A.w};
  const uint32_t b[4] = {B.x, B.y, B.z, B.w};
  const uint32_t q[4] = {Q.x, Q.y, Q.z, Q.w};
  const float2* x2 = reinterpret_cast<const float2*>(x);
  float2 p0 = make_float2(0.f, 0.f), p1 = p0, p2 = p0, p3 = p0;
#pragma unroll
  for (int t = 0; t < 4; t++) {
    uint32_t w0, w1, w2, w3;
    q6_words(a[t], b[t], q[t], w0, w1, w2, w3);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      p0 = f2_fma(q6_val2(w0, j), x2[(0 * 16 + 4 * t + j) / 2], p0);
      p1 = f2_fma(q6_val2(w1, j), x2[(1 * 16 + 4 * t + j) / 2], p1);
      p2 = f2_fma(q6_val2(w2, j), x2[(2 * 16 + 4 * t + j) / 2], p2);
      p3 = f2_fma(q6_val2(w3, j), x2[(3 * 16 + 4 * t + j) / 2], p3);
    }
  }
  float r = (d * sc_val(scw, 0)) * (p0.x + p0.y);
  r = fmaf(d * sc_val(scw, 1), p1.x + p1.y, r);
  r = fmaf(d * sc_val(scw, 2), p2.x + p2.y, r);
  r = fmaf(d * sc_val(scw, 3), p3.x + p3.y, r);
  return r;
}

// The 64 dequantised weights of a unit, in x-register order out[m*16 + i].
__device__ __forceinline__ void q6_unit_dequant(const uint4& A, const uint4& B, const uint4& Q,
                                                uint32_t scw, float d, float* out) {
  const uint32_t a[4] = {A.x, A.y, A.z, A.w};
  const uint32_t b[4] = {B.x, B.y, B.z, B.w};
  const uint32_t q[4] = {Q.x, Q.y, Q.z, Q.w};
  const float s0 = d * sc_val(scw, 0), s1 = d * sc_val(scw, 1), s2 = d * sc_val(scw, 2),
              s3 = d * sc_val(scw, 3);
#pragma unroll
  for (int t = 0; t < 4; t++) {
    uint32_t w0, w1, w2, w3;
    q6_words(a[t], b[t], q[t], w0, w1, w2, w3);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      out[0 * 16 + 4 * t + j] = s0 * q6_val(w0, j);
      out[1 * 16 + 4 * t + j] = s1 * q6_val(w1, j);
      out[2 * 16 + 4 * t + j] = s2 * q6_val(w2, j);
      out[3 * 16 + 4 * t + j] = s3 * q6_val(w3, j);
    }
  }
}

// Element offset (within the row) of x-register slot m*16+i of unit u.
__device__ __forceinline__ int q6_unit_base(int u) {
  return 256 * (u >> 2) + 128 * ((u >> 1) & 1) + 16 * (u & 1);
}
#endif

}  // namespace lfm
