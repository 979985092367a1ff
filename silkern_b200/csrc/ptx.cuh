// Thin inline-PTX wrappers for the sm_90+/sm_100a features the kernels use:
// programmatic dependent launch, thread-block cluster barriers, distributed
// shared memory stores, the bulk L2 prefetch and 256-bit global accesses.
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
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Store v into the copy of `local` that lives in CTA `rank` of this cluster.
__device__ __forceinline__ void st_shared_cluster(int32_t* local, uint32_t rank, int32_t v) {
  const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(v) : "memory");
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
