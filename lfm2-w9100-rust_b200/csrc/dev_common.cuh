// Device helpers shared by the TMA-staged kernels (mvt.cu, step.cu): mbarrier
// and bulk-copy wrappers, bounded waits, warp reductions.
#pragma once
#include <math.h>
#include <stdint.h>

#include "kernels.h"

namespace lfm {
namespace dev {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or ~10 us pass, instead of spinning on the issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(10000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bound of every wait, in SM clock cycles: about one second at B200 clocks
// (longer if the clock is throttled, never unbounded). Waits count cycles with
// clock64(), which is cheap, and only after a run of failed polls: reading
// %globaltimer costs on the order of 100 ns, too much for the critical path
// of a wait that usually succeeds within a few polls.
constexpr long long WAIT_CYCLES = 2000000000ll;
struct WaitBudget {
  long long t0 = 0;
  // Call every few dozen failed polls; true once the budget is spent.
  __device__ __forceinline__ bool spent() {
    const long long now = clock64();
    if (t0 == 0) {
      t0 = now;
      return false;
    }
    return now - t0 > WAIT_CYCLES;
  }
};
// Non-blocking probe of a phase (no suspend): the cheap path when the phase
// has usually completed already.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after ~1 s without completion (error word raised).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, unsigned* err) {
  if (mbar_test_wait(b, parity)) return true;
  WaitBudget wb;
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 15u) == 15u && wb.spent()) {
      if (err) atomicExch(err, 1u);
      return false;
    }
  }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

}  // namespace dev
}  // namespace lfm
