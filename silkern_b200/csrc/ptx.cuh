// Thin inline-PTX wrappers for the sm_90+/sm_100a features the kernels use:
// programmatic dependent launch, thread-block cluster barriers, distributed
// shared memory stores signalled on transaction barriers, the bulk L2
// prefetch and 256-bit global accesses.
#pragma once

#include <cstdint>

namespace silkern {

// Programmatic dependent launch: block until the previous grid in the stream
// has completed and its memory is visible (no-op when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next grid in the stream to start launching its CTAs.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Cluster barrier phases. Every thread of every CTA in the cluster executes
// each arrive and each wait exactly once, in the same order (".aligned").
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The address of the copy of the shared variable at `local` that lives in
// CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
  return remote;
}

// Transaction barrier in shared memory, initialised with `count` arrivals
// and made visible to the other CTAs of the cluster (their first access must
// still follow a cluster barrier phase that this thread arrived at after the
// initialisation).
__device__ __forceinline__ void mbar_init_cluster(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival on `bar` that also expects `bytes` more bytes of transactions
// in the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Store v into CTA `rank`'s copy of `local` and count its 4 bytes as a
// completed transaction on that CTA's copy of `bar`. No fence: the barrier's
// phase completion is what publishes the value.
__device__ __forceinline__ void st_async_cluster(int32_t* local, uint64_t* bar, uint32_t rank, int32_t v) {
  const uint32_t dst = cluster_addr(local, rank);
  const uint32_t rbar = cluster_addr(bar, rank);
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst), "r"(v),
               "r"(rbar)
               : "memory");
}

// Wait, with acquire semantics at cluster scope, until phase `parity` of
// `bar` completes; give up after `tries` polls (each poll may suspend the
// thread for a hardware-chosen time). Returns whether the phase completed.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t tries) {
  uint32_t done = 0;
  for (uint32_t i = 0; i < tries && done == 0; ++i) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
  }
  return done != 0;
}

// Hint: bring [ptr, ptr + bytes) into L2. ptr 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* ptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

// Hint: bring the 128-byte line holding ptr into L2.
__device__ __forceinline__ void prefetch_l2_line(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr) : "memory");
}

// Index of this cluster in the grid (x) and of this CTA inside its cluster.
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t v;
  asm("mov.u32 %0, %%clusterid.x;" : "=r"(v));
  return v;
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t v;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(v));
  return v;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// 256-bit global load through the non-coherent (read-only) path; ptr 32-byte
// aligned. Volatile so that it stays after griddepcontrol.wait.
__device__ __forceinline__ void ld_nc_v8(const int32_t* ptr, int32_t (&v)[8]) {
  asm volatile("ld.global.nc.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                 "=r"(v[7])
               : "l"(ptr));
}

// 256-bit global store; ptr 32-byte aligned.
__device__ __forceinline__ void st_v8(int32_t* ptr, const int32_t (&v)[8]) {
  asm volatile("st.global.v8.u32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

}  // namespace silkern
