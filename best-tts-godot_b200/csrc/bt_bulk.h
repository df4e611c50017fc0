// bt_bulk.h -- bulk copies (the Blackwell / Hopper tensor memory accelerator's
// untiled form, cp.async.bulk) between global and shared memory, completion
// tracked by a shared-memory mbarrier (loads) or a bulk group (stores).
//
// No multicast: every load moves this GPU's own global memory into the
// issuing CTA's own shared memory, and every store the reverse, so these
// copies are safe in code that runs on any number of GPUs.  Addresses must be
// 16-byte aligned and sizes multiples of 16 bytes; callers copy the aligned
// interior of a row this way and its few edge elements with plain loads.
//
// Waits on an mbarrier are bounded: a wait that gives up counts itself in
// g_bulk_timeouts and returns, so a copy that never completes shows as an
// error instead of a hung kernel.  The counter has internal linkage (the
// library is built without relocatable device code): each translation unit
// that waits on bulk copies exports a reader of its own (bt_wait_timeouts).
#pragma once
#include <stdint.h>

namespace bt {
namespace {
__device__ unsigned int g_bulk_timeouts = 0;
}  // namespace

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  // the initialised barrier, visible to the async proxy that completes it
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

// One arrival that also announces `bytes` of bulk copies to come.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> this CTA's shared memory, `bytes` (a multiple of 16, both
// addresses 16-byte aligned), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* sdst, const void* gsrc, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Waits until phase `parity` of `bar` completes, polling at most `limit`
// times (each poll may suspend the thread briefly); false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned limit = 1u << 22) {
  const unsigned a = smem_u32(bar);
  for (unsigned i = 0; i < limit; ++i) {
    unsigned done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicAdd(&g_bulk_timeouts, 1u);
  return false;
}

// The address of the same shared-memory location in CTA `rank` of this
// cluster (a shared::cluster address).
__device__ __forceinline__ unsigned cluster_addr(unsigned local, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// Stores v at the shared::cluster address `addr` (any CTA of the cluster,
// this one included) and completes 4 bytes of the transaction count of the
// mbarrier at shared::cluster address `bar` (in that same CTA): a receiver
// that waits on its own mbarrier for the bytes it expects needs no cluster
// barrier.
__device__ __forceinline__ void st_async_f32(unsigned addr, float v, unsigned bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];\n" ::"r"(addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}

// Orders this thread's earlier (generic) shared-memory writes before later
// reads of the same bytes by bulk copies (the async proxy).
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// This CTA's shared memory -> global, `bytes` (a multiple of 16, both
// addresses 16-byte aligned), in the issuing thread's current bulk group.
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Waits until every bulk group this thread committed has completed (the
// issuing thread calls it before its CTA's shared memory goes away).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

}  // namespace bt
