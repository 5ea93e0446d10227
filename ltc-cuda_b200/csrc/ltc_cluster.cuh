// Per-unfold exchange of per-neuron vectors between the CTAs of a cluster.
//
// Each CTA owns a slice of the neurons; after an unfold every CTA needs every
// neuron's new value.  Instead of generic DSMEM stores followed by a cluster
// barrier (whose release half waits for all of the CTA's outstanding memory
// operations), each value goes out as one `st.async` per destination CTA that
// also signals `complete_tx` on the destination's mbarrier for that buffer slot.
// A CTA starts the next unfold once its own mbarrier has seen the expected
// number of bytes: no cluster-wide barrier and no fence per unfold.
//
// Protocol for a double-buffered vector (slots 0/1; the kernels keep one mbarrier
// per (slot, 4-sample block), so each block is its own instance of this protocol):
//   * init (thread 0): mbarrier.init(count 1) for every slot, fence, arm each with
//     expect_tx(bytes of one phase); then one cluster barrier before the first
//     remote store.
//   * producer: every (neuron, sample) item of the cluster's sample group is sent
//     by exactly one lane to every CTA (zeros for padding), so each phase
//     receives exactly the armed byte count.
//   * consumer: all threads wait on the slot's parity; thread 0 then re-arms the
//     slot for its next phase.  Bytes of the next phase can arrive before the
//     re-arm (the tx-count goes negative while the pending arrival of thread 0
//     keeps the phase open), never before the current phase completed: a CTA
//     sends data of phase k+1 only after it received all of phase k+1's inputs,
//     which every CTA produces only after having waited phase k.
//   * every wait is bounded (about 2 s of SM clock); on expiry the kernel counts a
//     timeout in a device counter (read by ltc_wait_timeouts()), stops waiting for
//     the rest of the launch (its results are then invalid) and still exits.
// The streamed backward reuses mbar_* for its TMA chunk arrivals (local bytes only).
#pragma once

#include <stdint.h>

namespace ltc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arm(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// cluster address of `local_addr` in the shared memory of CTA `rank`
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_async(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
               : "memory");
}

// Store v at the same shared-memory offset in every CTA of the cluster,
// completing tx bytes on each destination's copy of the mbarrier `bar`.
template <int CL>
__device__ __forceinline__ void st_async_all(const float* local, float v, uint32_t bar) {
  const uint32_t a = smem_addr(local);
#pragma unroll
  for (int r = 0; r < CL; ++r) st_async(cluster_map(a, r), v, cluster_map(bar, r));
}

// Bounded parity wait.  `aborted` (shared) turns every later wait of the CTA into
// a no-op once one wait expired, so that a failed launch still ends quickly.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity, volatile int* aborted, int* timeouts) {
  if (*aborted) return;
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return;
    if (*aborted) return;
    if (clock64() - t0 > (4LL << 30)) {
      atomicAdd(timeouts, 1);
      *aborted = 1;
      return;
    }
  }
}

}  // namespace ltc
