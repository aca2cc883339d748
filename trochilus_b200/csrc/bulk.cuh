// bulk.cuh: the 1-D TMA bulk copy (cp.async.bulk, global -> shared, completing on an mbarrier) and the
// mbarrier operations the weight pipelines use. No multicast form is used anywhere: each CTA fetches its
// own bytes from this GPU's memory.
#pragma once
#include <cstdint>

__device__ __forceinline__ uint32_t trx_smem(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void trx_mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(trx_smem(bar)), "r"(count) : "memory");
}

// make initialised barriers visible to the async proxy (the TMA unit) before any copy names them
__device__ __forceinline__ void trx_fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// order this thread's earlier shared-memory accesses before later async-proxy (bulk copy) accesses
__device__ __forceinline__ void trx_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void trx_mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(trx_smem(bar)), "r"(bytes)
                 : "memory");
}

// bytes (a multiple of 16) from 16-byte aligned global src to 16-byte aligned shared dst
__device__ __forceinline__ void trx_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     trx_smem(dst)),
                 "l"(src), "r"(bytes), "r"(trx_smem(bar))
                 : "memory");
}

// An L2 policy for data a call reads once (the expert weights): its lines are the first the L2 evicts, so the
// stream of a layer's weights does not push out what every call reuses (the kernels' code, the routing arrays, the
// activations, the routers).
__device__ __forceinline__ uint64_t trx_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// trx_bulk_g2s with an L2 cache policy (trx_policy_evict_first)
__device__ __forceinline__ void trx_bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                  uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
                 "%4;" ::"r"(trx_smem(dst)),
                 "l"(src), "r"(bytes), "r"(trx_smem(bar)), "l"(policy)
                 : "memory");
}

// A 3-D tiled TMA load (no multicast) with an L2 cache policy: the box at element (x, y, z) of the tensor map (a
// CUtensorMap in kernel parameter, constant or global memory) into shared memory (128-byte aligned), completing on
// bar. x times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void trx_tma_load_3d_hint(void *dst, const void *map, int x, int y, int z, uint64_t *bar,
                                                     uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
                 "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(trx_smem(dst)),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(trx_smem(bar)), "l"(policy)
                 : "memory");
}

// Bring [src, src + bytes) into L2 without waiting for it (src and bytes multiples of 16)
__device__ __forceinline__ void trx_bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool trx_mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok)
                 : "r"(trx_smem(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Programmatic dependent launch: let the next kernel of the stream be scheduled (it still waits for this grid's end
// in its own trx_griddep_wait), and wait for the previous kernel's end and memory (a no-op without one)
__device__ __forceinline__ void trx_griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void trx_griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint64_t trx_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the barrier's phase `parity` to complete, at most limit_ns; false when it gave up.
__device__ __forceinline__ bool trx_mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
    if (trx_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = trx_globaltimer();
    while (!trx_mbar_try_wait(bar, parity))
        if (trx_globaltimer() - t0 > limit_ns) return false;
    return true;
}
