// Kernel-level C ABI (include/lfm_cuda.h, "kernel-level entry points"): the
// per-kernel surface of the reference's GpuOps (engine/src/ops.rs:56-575),
// on caller-owned device pointers. Used by the parity tests and the Q6_K
// matvec microbench.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/lfm_cuda.h"
#include "dev_common.cuh"
#include "kernels.h"
#include "tc_gemm.h"

namespace {
thread_local std::string t_err;

lfm_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return LFM_OK;
  t_err = std::string("CUDA: ") + cudaGetErrorString(e);
  return LFM_ERR_CUDA;
}

bool shape_ok(uint32_t in_dim, uint32_t rows) { return in_dim >= 256 && in_dim % 256 == 0 && rows > 0; }

// status word of lfm_tc_gemm_f16 (raised by a bounded wait that timed out)
__device__ unsigned g_tc_err;

// Failure-detection self-test: thread 0 waits on an mbarrier that nothing
// arrives at, through the same bounded wait every kernel of the library uses
// (lfm::dev::mbar_wait, about one second of SM cycles). It must give up,
// raise the status word and return; the kernel then exits normally and the
// context stays usable. No fault, trap or unbounded spin is involved.
__global__ void k_selftest_wait_timeout(unsigned* err, unsigned long long* cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    lfm::dev::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const long long t0 = clock64();
    const bool ok = lfm::dev::mbar_wait(&bar, 0, err);  // phase 0 never completes
    *cycles = (unsigned long long)(clock64() - t0);
    if (ok) atomicExch(err, 99u);  // a wait that returned success would be a bug
  }
}
}  // namespace

extern "C" {

size_t lfm_q6k_device_bytes(uint32_t in_dim, uint32_t rows) {
  if (!shape_ok(in_dim, rows)) return 0;
  return lfm::q6_total_bytes(rows, (int)(in_dim / 256));
}

lfm_status lfm_q6k_upload(const uint8_t* gguf_rows, uint32_t in_dim, uint32_t rows, void* dst_dev) {
  if (!gguf_rows || !dst_dev || !shape_ok(in_dim, rows)) {
    t_err = "lfm_q6k_upload: bad argument";
    return LFM_ERR_ARG;
  }
  const int nb = (int)(in_dim / 256);
  const size_t bytes = lfm::q6_total_bytes(rows, nb);
  std::vector<uint8_t> dst(bytes);
  const unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  std::vector<std::thread> th;
  const size_t per = (rows + nt - 1) / nt;
  for (unsigned i = 0; i < nt; i++) {
    const size_t r0 = i * per;
    if (r0 >= rows) break;
    const size_t r1 = std::min<size_t>(rows, r0 + per);
    th.emplace_back([&, r0, r1] { lfm::q6_repack_rows(gguf_rows + r0 * nb * lfm::QB, r0, r1 - r0, nb, rows, dst.data()); });
  }
  for (auto& t : th) t.join();
  return cuda_status(cudaMemcpy(dst_dev, dst.data(), bytes, cudaMemcpyHostToDevice));
}

lfm_status lfm_q6k_dequant(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t row0, uint32_t nrows,
                           float* out_dev, void* stream) {
  if (!w_dev || !out_dev || !shape_ok(in_dim, rows) || row0 + nrows > rows) {
    t_err = "lfm_q6k_dequant: bad argument";
    return LFM_ERR_ARG;
  }
  if (nrows == 0) return LFM_OK;
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)rows, (int)(in_dim / 256));
  lfm::q6_dequant_rows(W, (int)row0, (int)nrows, out_dev, (cudaStream_t)stream);
  return cuda_status(cudaGetLastError());
}

lfm_status lfm_q6k_matmul(const void* w_dev, uint32_t in_dim, uint32_t rows, const float* x_dev, uint32_t n,
                          float* y_dev, void* stream) {
  if (!w_dev || !x_dev || !y_dev || !shape_ok(in_dim, rows) || n == 0) {
    t_err = "lfm_q6k_matmul: bad argument";
    return LFM_ERR_ARG;
  }
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)rows, (int)(in_dim / 256));
  if (n == 1 && lfm::mvt_supported(W)) {
    // the engine's TMA-staged decode matvec (no device error word here)
    lfm::LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, dev);
    lfm::mvt_plain(W, lfm::XSrc{x_dev, nullptr, 0.f}, y_dev, nullptr, c);
  } else if (n == 1 && in_dim <= 2048) {
    lfm::LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    lfm::mv_plain(W, lfm::XSrc{x_dev, nullptr, 0.f}, y_dev, c);
  } else if (n == 1 && in_dim == (uint32_t)lfm::N_FF) {
    // the decode kernel of the dense down projection (7168-wide rows), which
    // adds to its output: y = 0 + W x, the same values as a plain store
    lfm::LaunchCfg c;
    c.stream = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(y_dev, 0, (size_t)rows * 4, c.stream);
    if (e != cudaSuccess) return cuda_status(e);
    lfm::mv_down7168_resid(W, x_dev, y_dev, c);
  } else {
    lfm::gemm_q6(W, x_dev, (int)n, y_dev, false, (cudaStream_t)stream);
  }
  return cuda_status(cudaGetLastError());
}

lfm_status lfm_q6k_routed(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t n_expert,
                          const int32_t* expert_ids_dev, const float* x_dev, uint32_t x_stride, float* y_dev,
                          void* stream) {
  if (!w_dev || !x_dev || !y_dev || !expert_ids_dev || !shape_ok(in_dim, rows) || in_dim > 2048 ||
      n_expert == 0 || x_stride < in_dim) {
    t_err = "lfm_q6k_routed: bad argument (in_dim must be <= 2048)";
    return LFM_ERR_ARG;
  }
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)(rows * n_expert), (int)(in_dim / 256));
  lfm::LaunchCfg c;
  c.stream = (cudaStream_t)stream;
  lfm::mv_routed(W, (int)rows, x_dev, (int)x_stride, expert_ids_dev, y_dev, c);
  return cuda_status(cudaGetLastError());
}

lfm_status lfm_route(const float* logits_dev, const float* bias_dev, uint32_t n_expert, uint32_t n,
                     int32_t* sel_ids_dev, float* sel_w_dev, void* stream) {
  if (!logits_dev || !bias_dev || !sel_ids_dev || !sel_w_dev || n_expert < 4 || n_expert > 32 || n == 0) {
    t_err = "lfm_route: bad argument (4 <= n_expert <= 32)";
    return LFM_ERR_ARG;
  }
  lfm::route_n(logits_dev, bias_dev, (int)n_expert, (int)n, sel_ids_dev, sel_w_dev, (cudaStream_t)stream);
  return cuda_status(cudaGetLastError());
}

lfm_status lfm_argmax(const float* x_dev, uint32_t n, uint32_t* out_dev, void* stream) {
  if (!x_dev || !out_dev || n == 0) {
    t_err = "lfm_argmax: bad argument";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  // Scratch: up to 256 per-CTA partial maxima and the last-CTA counter.
  void* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(&scratch, 256 * sizeof(float2) + 16, s);
  if (e != cudaSuccess) return cuda_status(e);
  unsigned* counter = (unsigned*)((char*)scratch + 256 * sizeof(float2));
  cudaMemsetAsync(counter, 0, 4, s);
  lfm::argmax_f32(x_dev, (int)n, (float2*)scratch, counter, (int*)out_dev, s);
  e = cudaGetLastError();
  cudaFreeAsync(scratch, s);
  return cuda_status(e);
}

// Scratch of one synchronous prompt-GEMM call (stream-ordered allocations).
struct CallScratch {
  lfm::TcScratch sc;
  void* mem = nullptr;
  cudaStream_t s;
  explicit CallScratch(cudaStream_t st) : s(st) {}
  cudaError_t alloc(size_t rows, size_t K, size_t slots) {
    sc.rows = rows;
    sc.halves = 2 * rows * K;
    const size_t tiles = 1 + 2 * (rows / 128 + 64);
    sc.part_cap = rows <= 128 ? (size_t)16 * 128 * 8192 : 0;  // split-K partials (one token tile)
    const size_t bytes = sc.halves * 2 + rows * 4 + tiles * 4 + rows * 4 + slots * 4 + sc.part_cap * 4 + 256 * 6;
    cudaError_t e = cudaMallocAsync(&mem, bytes, s);
    if (e != cudaSuccess) return e;
    char* p = (char*)mem;
    auto take = [&](size_t b) {
      char* r = p;
      p += (b + 255) / 256 * 256;
      return r;
    };
    sc.xg = (__half*)take(sc.halves * 2);
    sc.inv = (float*)take(rows * 4);
    sc.tiles = (int*)take(tiles * 4);
    sc.slots = (int*)take(rows * 4);
    sc.rowof = (int*)take(slots * 4);
    sc.part = sc.part_cap ? (float*)take(sc.part_cap * 4) : nullptr;
    return cudaGetSymbolAddress((void**)&sc.err, g_tc_err);
  }
  // zero the status word, run, read it back; frees the scratch
  lfm_status finish(cudaError_t e, const char* who) {
    if (e == cudaSuccess) {
      unsigned h = 0;
      e = cudaMemcpyAsync(&h, sc.err, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e == cudaSuccess && h) {
        if (mem) cudaFreeAsync(mem, s);
        if (h == lfm::GROUP_OVERFLOW) {
          t_err = std::string(who) + ": the four expert ids of a token must be distinct";
          return LFM_ERR_ARG;
        }
        t_err = std::string(who) + ": a bounded wait in the kernel timed out";
        return LFM_ERR_DEVICE;
      }
    }
    if (mem) cudaFreeAsync(mem, s);
    return cuda_status(e);
  }
};

lfm_status lfm_q6k_prompt_gemm(const void* w_dev, uint32_t in_dim, uint32_t rows, const float* x_dev, uint32_t n,
                               float* y_dev, void* stream) {
  if (!w_dev || !x_dev || !y_dev || !shape_ok(in_dim, rows) || rows % 128 || n == 0 || n > (1u << 20)) {
    t_err = "lfm_q6k_prompt_gemm: bad argument (rows % 128 == 0, 1 <= n <= 2^20)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)rows, (int)(in_dim / 256));
  CallScratch cs(s);
  cudaError_t e = cs.alloc((n + 127) / 128 * 128, in_dim, 1);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = lfm::tc_split(x_dev, (int)in_dim, (int)in_dim, (int)n, cs.sc, s);
  if (e == cudaSuccess) e = lfm::tc_gemm_q6(W, (int)n, y_dev, (int)rows, false, cs.sc, s);
  return cs.finish(e, "lfm_q6k_prompt_gemm");
}

lfm_status lfm_q6k_prompt_grouped(const void* w_dev, uint32_t in_dim, uint32_t rows, uint32_t n_expert,
                                  const int32_t* expert_ids_dev, const float* x_dev, uint32_t x_div, uint32_t n,
                                  float* y_dev, void* stream) {
  if (!w_dev || !x_dev || !y_dev || !expert_ids_dev || !shape_ok(in_dim, rows) || rows % 128 ||
      n_expert != (uint32_t)lfm::N_EXPERT || (x_div != 1 && x_div != (uint32_t)lfm::N_USED) || n == 0 ||
      n > (1u << 16)) {
    t_err = "lfm_q6k_prompt_grouped: bad argument (rows % 128 == 0, n_expert == 32, x_div 1 or 4, 1 <= n <= 65536)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)(rows * n_expert), (int)(in_dim / 256));
  CallScratch cs(s);
  int* groups = nullptr;
  cudaError_t e = cs.alloc(lfm::tc_scratch_rows((int)n), in_dim, (size_t)n * lfm::N_USED);
  if (e == cudaSuccess) e = cudaMallocAsync(&groups, sizeof(int) * (size_t)lfm::N_EXPERT * (n + 1), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) {
    lfm::expert_groups(expert_ids_dev, (int)n, groups, (int)n, s, cs.sc.err);
    e = lfm::tc_group(groups, (int)n, (int)n, cs.sc, s);
  }
  if (e == cudaSuccess) e = lfm::tc_split_grouped(x_dev, (int)in_dim, (int)x_div, (int)n, cs.sc, s);
  if (e == cudaSuccess) e = lfm::tc_gemm_q6_grouped(W, (int)rows, (int)n, y_dev, cs.sc, s);
  if (groups) cudaFreeAsync(groups, s);
  return cs.finish(e, "lfm_q6k_prompt_grouped");
}

lfm_status lfm_q6k_expand_f16(const void* w_dev, uint32_t in_dim, uint32_t rows, void* out_dev, void* stream) {
  if (!w_dev || !out_dev || !shape_ok(in_dim, rows) || (uintptr_t)out_dev % 16) {
    t_err = "lfm_q6k_expand_f16: bad argument (out_dev 16-byte aligned)";
    return LFM_ERR_ARG;
  }
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)rows, (int)(in_dim / 256));
  return cuda_status(lfm::q6_expand_f16(W, (__half*)out_dev, (cudaStream_t)stream));
}

lfm_status lfm_q6k_prompt_gemm_x16(const void* w_dev, const void* w16_dev, uint32_t in_dim, uint32_t rows,
                                   const float* x_dev, uint32_t n, float* y_dev, void* stream) {
  if (!w_dev || !w16_dev || !x_dev || !y_dev || !shape_ok(in_dim, rows) || rows % 128 || n == 0 ||
      n > (1u << 20) || (uintptr_t)w16_dev % 16) {
    t_err = "lfm_q6k_prompt_gemm_x16: bad argument (rows % 128 == 0, 1 <= n <= 2^20, w16_dev 16-byte aligned)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)rows, (int)(in_dim / 256));
  CallScratch cs(s);
  cudaError_t e = cs.alloc((n + 127) / 128 * 128, in_dim, 1);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = lfm::tc_split(x_dev, (int)in_dim, (int)in_dim, (int)n, cs.sc, s);
  if (e == cudaSuccess) e = lfm::tc_gemm_q6(W, (int)n, y_dev, (int)rows, false, cs.sc, s, (const __half*)w16_dev);
  return cs.finish(e, "lfm_q6k_prompt_gemm_x16");
}

lfm_status lfm_q6k_prompt_grouped_x16(const void* w_dev, const void* w16_dev, uint32_t in_dim, uint32_t rows,
                                      uint32_t n_expert, const int32_t* expert_ids_dev, const float* x_dev,
                                      uint32_t x_div, uint32_t n, float* y_dev, void* stream) {
  if (!w_dev || !w16_dev || !x_dev || !y_dev || !expert_ids_dev || !shape_ok(in_dim, rows) || rows % 128 ||
      n_expert != (uint32_t)lfm::N_EXPERT || (x_div != 1 && x_div != (uint32_t)lfm::N_USED) || n == 0 ||
      n > (1u << 16) || (uintptr_t)w16_dev % 16) {
    t_err = "lfm_q6k_prompt_grouped_x16: bad argument (rows % 128 == 0, n_expert == 32, x_div 1 or 4, "
            "1 <= n <= 65536, w16_dev 16-byte aligned)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  lfm::Q6Mat W = lfm::q6_view(w_dev, (int)(rows * n_expert), (int)(in_dim / 256));
  CallScratch cs(s);
  int* groups = nullptr;
  cudaError_t e = cs.alloc(lfm::tc_scratch_rows((int)n), in_dim, (size_t)n * lfm::N_USED);
  if (e == cudaSuccess) e = cudaMallocAsync(&groups, sizeof(int) * (size_t)lfm::N_EXPERT * (n + 1), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) {
    lfm::expert_groups(expert_ids_dev, (int)n, groups, (int)n, s, cs.sc.err);
    e = lfm::tc_group(groups, (int)n, (int)n, cs.sc, s);
  }
  if (e == cudaSuccess) e = lfm::tc_split_grouped(x_dev, (int)in_dim, (int)x_div, (int)n, cs.sc, s);
  if (e == cudaSuccess)
    e = lfm::tc_gemm_q6_grouped(W, (int)rows, (int)n, y_dev, cs.sc, s, (const __half*)w16_dev);
  if (groups) cudaFreeAsync(groups, s);
  return cs.finish(e, "lfm_q6k_prompt_grouped_x16");
}

lfm_status lfm_attention_prefill(const float* q_dev, uint32_t q_stride, const void* k_cache, const void* v_cache,
                                 uint32_t ctx, uint32_t start, uint32_t n, float* out_dev, uint32_t out_stride,
                                 void* stream) {
  if (!q_dev || !k_cache || !v_cache || !out_dev || n == 0 || ctx == 0 || (uint64_t)start + n > ctx ||
      q_stride < (uint32_t)lfm::DIM || out_stride < (uint32_t)lfm::DIM || q_stride % 4 || out_stride % 4 ||
      ctx > 65536) {
    t_err = "lfm_attention_prefill: bad argument (start + n <= ctx <= 65536, strides >= 2048 and % 4 == 0)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  CallScratch cs(s);
  cudaError_t e = cudaGetSymbolAddress((void**)&cs.sc.err, g_tc_err);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess)
    e = lfm::attn_prefill_tc(q_dev, (int)q_stride, (const __half*)k_cache, (const __half*)v_cache, (int)start,
                             (int)n, (int)ctx, out_dev, (int)out_stride, cs.sc.err, s);
  return cs.finish(e, "lfm_attention_prefill");
}

lfm_status lfm_selftest_wait_timeout(uint32_t* status, uint64_t* cycles) {
  if (!status || !cycles) {
    t_err = "lfm_selftest_wait_timeout: bad argument";
    return LFM_ERR_ARG;
  }
  unsigned* err = nullptr;
  unsigned long long* cyc = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&err, g_tc_err);
  if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMalloc(&cyc, sizeof(unsigned long long));
  if (e == cudaSuccess) {
    k_selftest_wait_timeout<<<1, 32>>>(err, cyc);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  unsigned h = 0;
  unsigned long long hc = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h, err, sizeof h, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(&hc, cyc, sizeof hc, cudaMemcpyDeviceToHost);
  if (cyc) cudaFree(cyc);
  if (e != cudaSuccess) return cuda_status(e);
  *status = h;
  *cycles = hc;
  return LFM_OK;
}

lfm_status lfm_tc_gemm_f16_bmn(const void* a_dev, const void* b_dev, uint32_t m, uint32_t k, float* c_dev,
                               void* stream) {
  if (!a_dev || !b_dev || !c_dev || m == 0 || k == 0 || m % 128 || k % 64) {
    t_err = "lfm_tc_gemm_f16_bmn: bad argument (m % 128, k % 64 must be 0)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  CallScratch cs(s);
  cudaError_t e = cudaGetSymbolAddress((void**)&cs.sc.err, g_tc_err);
  if (e == cudaSuccess) e = cudaMemsetAsync(cs.sc.err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess)
    e = lfm::tc_gemm_f16_bmn((const __half*)a_dev, (const __half*)b_dev, (int)m, (int)k, c_dev, cs.sc.err, s);
  return cs.finish(e, "lfm_tc_gemm_f16_bmn");
}

lfm_status lfm_tc_gemm_f16(const void* a_dev, const void* b_dev, uint32_t m, uint32_t n, uint32_t k, float* c_dev,
                           void* stream) {
  if (!a_dev || !b_dev || !c_dev || m == 0 || n == 0 || k == 0 || m % 128 || n % 256 || k % 64) {
    t_err = "lfm_tc_gemm_f16: bad argument (m % 128, n % 256, k % 64 must be 0)";
    return LFM_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  unsigned* err = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&err, g_tc_err);
  if (e != cudaSuccess) return cuda_status(e);
  e = cudaMemsetAsync(err, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return cuda_status(e);
  e = lfm::tc_gemm_f16((const __half*)a_dev, (const __half*)b_dev, (int)m, (int)n, (int)k, c_dev, err, s);
  if (e != cudaSuccess) return cuda_status(e);
  unsigned h = 0;
  e = cudaMemcpyAsync(&h, err, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  if (h) {
    t_err = "lfm_tc_gemm_f16: a bounded wait in the kernel timed out";
    return LFM_ERR_DEVICE;
  }
  return LFM_OK;
}

const char* lfm_ops_error(void) { return t_err.c_str(); }

}  // extern "C"

// ---------------------------------------------------------------------------
// lfm_argmax_noalloc: lfm_argmax with its scratch in a fixed device array.
//
// Some callers of this library cannot allocate device memory at call time: a
// host that runs under a fixed memory budget and has already handed every byte
// of the device to its own pool, an allocator that must not be re-entered from
// inside its own callbacks, or a caller that may not touch the CUDA allocator
// on that thread. lfm_argmax needs 2 KiB of scratch (one partial maximum per
// CTA plus an arrival counter) and gets it with cudaMallocAsync; this variant
// takes it from a file-scope device array instead, so it calls no allocating
// routine at all.
namespace {
// The launcher (lfm::argmax_f32) runs at most 256 CTAs, each writing one
// partial, so 256 slots suffice for every n. The kernel's grid-stride index is
// a signed 32-bit int, so n is capped at 2^30 elements (4 GiB of fp32), well
// clear of overflow.
constexpr int kNoAllocPartials = 256;
constexpr uint32_t kNoAllocMaxN = 1u << 30;

// Slots 0..255: per-CTA partial maxima. Slot 256: its first word is the
// last-CTA arrival counter, which must be 0 when the kernel starts.
// One copy per device that loads this library (2 KiB + 8 B), held until the
// process exits.
static __device__ __align__(256) float2 g_argmax_scratch[kNoAllocPartials + 1];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float2* g_scratch_ptr[kMaxDevices] = {};
void* g_scratch_ctx[kMaxDevices] = {};  // the context each cached address belongs to

// cuCtxGetCurrent through the runtime's driver entry point (no link against
// libcuda); null if the driver does not offer it.
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (CtxGetCurrentFn)p;
  });
  return fn;
}

// Device address of g_argmax_scratch on the current device. In host code the
// array's name is only a host-side stand-in, not a device address, so the
// address is looked up once per device, with that device current, and cached
// together with the context it was looked up in. A device reset
// (cudaDeviceReset) replaces the primary context and unloads the module; the
// next call sees a different context and looks the address up again instead
// of handing the kernel a stale pointer.
cudaError_t argmax_scratch(float2** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  auto current_ctx = [] {
    void* c = nullptr;
    if (CtxGetCurrentFn f = ctx_get_current_fn())
      if (f(&c) != 0) c = nullptr;
    return c;
  };
  void* ctx = current_ctx();  // null before the runtime has made a context current
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev] || !ctx || g_scratch_ctx[dev] != ctx) {
    float2* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_argmax_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = current_ctx();  // the lookup made the device's primary context current
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}
}  // namespace

extern "C" lfm_status lfm_argmax_noalloc(const float* x_dev, uint32_t n, uint32_t* out_dev, void* stream) {
  if (!x_dev || !out_dev || n == 0) {
    t_err = "lfm_argmax_noalloc: bad argument";
    return LFM_ERR_ARG;
  }
  if (n > kNoAllocMaxN) {
    t_err = "lfm_argmax_noalloc: n = " + std::to_string(n) + " exceeds the maximum " +
            std::to_string(kNoAllocMaxN) + " elements";
    return LFM_ERR_ARG;
  }
  float2* sc = nullptr;
  cudaError_t e = argmax_scratch(&sc);
  if (e != cudaSuccess) return cuda_status(e);
  cudaStream_t s = (cudaStream_t)stream;
  unsigned* counter = (unsigned*)&sc[kNoAllocPartials];
  // The array keeps whatever the previous call left: zero the counter first.
  e = cudaMemsetAsync(counter, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return cuda_status(e);
  lfm::argmax_f32(x_dev, (int)n, sc, counter, (int*)out_dev, s);
  return cuda_status(cudaGetLastError());
}
