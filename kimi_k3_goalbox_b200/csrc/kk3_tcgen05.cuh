// kk3_tcgen05.cuh - PTX wrappers for the 5th-generation tensor cores (sm_100a): mbarriers, the async-proxy
// fence, TMEM allocation and loads, MMA completion, shared-memory matrix descriptors. Shared by the step
// kernel's tensor-core projection engine (kk3_tc_gemv.cuh) and the tensor-core expert engine
// (kk3_tc_experts.cuh). Every wait is bounded.
#pragma once
#include "kk3_common.cuh"

namespace kk3 {

KK3_DEV void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
KK3_DEV void mbar_inval(unsigned bar) { asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory"); }
KK3_DEV void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
KK3_DEV void mbar_arrive_tx(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
KK3_DEV bool mbar_test(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait for the phase of parity `parity` to complete; false (error raised) on timeout or error.
KK3_DEV bool mbar_wait(const StepArgs& a, unsigned bar, unsigned parity) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (unsigned spin = 0;; ++spin) {
    if (mbar_test(bar, parity)) return true;
    if ((spin & 15) == 15 && (failed(a) || globaltimer() - t0 > (unsigned long long)a.g.timeout_ns)) {
      set_error(a, kErrTimeout);
      return false;
    }
  }
}

// Bounded wait that ignores the error word (cleanup after a failure): true if the phase completed in time.
KK3_DEV bool mbar_wait_for(unsigned bar, unsigned parity, unsigned long long ns) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_test(bar, parity))
    if (globaltimer() - t0 > ns) return false;
  return true;
}

KK3_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
KK3_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

KK3_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KK3_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
KK3_DEV void tmem_alloc(unsigned dst_smem, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
KK3_DEV void tmem_dealloc(unsigned taddr, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
KK3_DEV void umma_commit(unsigned bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
KK3_DEV float tmem_ld1(unsigned taddr) {
  unsigned v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr) : "memory");
  return __uint_as_float(v);
}
KK3_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptors (tcgen05): K-major, 128-byte swizzle, 8-row atoms of 1024 bytes
KK3_DEV unsigned long long sdesc_sw128(unsigned addr) {
  return (unsigned long long)((addr & 0x3ffffu) >> 4) | (1ull << 16) | ((unsigned long long)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

}  // namespace kk3
