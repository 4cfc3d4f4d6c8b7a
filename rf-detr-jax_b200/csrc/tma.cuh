// Tensor-memory-accelerator (TMA) tile loads and shared-memory mbarriers for sm_100a.
//
// Tiles are described by CUtensorMap objects built on the host with cuTensorMapEncodeTiled
// (fetched through cudaGetDriverEntryPoint, so the library needs no link against libcuda) and
// passed to kernels as __grid_constant__ parameters.  One elected thread arms an mbarrier with
// the tile's byte count and issues cp.async.bulk.tensor loads into this CTA's shared memory;
// every consumer thread waits on the barrier's phase.  No load here uses cluster multicast, and
// the source is always this GPU's global memory.
//
// Waits are bounded: a wait that has not completed after kWaitLimit polls (each poll of
// mbarrier.try_wait suspends for a hardware-defined interval) raises the device fault word and
// returns false; a shared abort flag makes the CTA's other waiters give up at once, so the
// kernel runs to completion with undefined outputs instead of hanging.  A CTA that gave up arms no
// further barriers and, before it exits, drains (again bounded) the phases it armed, so no copy
// is still writing its shared memory when it leaves.  The host reads and
// clears the fault word with rfdetr_take_device_fault().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rfdetr {

// Set (bit 0) when a bounded device wait gave up.  The library compiles each .cu file as its
// own device module, so this word is per translation unit; the waits live in msda.cu, whose
// copy rfdetr_take_device_fault() reads.
static __device__ unsigned int g_device_fault = 0;

constexpr int kWaitLimit = 1 << 22;

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy before first use.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the barrier phase with the given parity; see the file comment.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, volatile int *abort_flag,
                                          int limit = kWaitLimit) {
    for (int i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    atomicOr(&g_device_fault, 1u);
    return false;
}

// After a CTA gave up waiting: waits (bounded, ignoring the abort flag) for a phase this CTA armed
// and whose copies may still be in flight, so that no bulk copy lands in shared memory after the
// CTA has exited.  A drain that gives up too raises bit 1 of the fault word.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, unsigned parity, int limit = kWaitLimit) {
    for (int i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return;
    atomicOr(&g_device_fault, 2u);
}

// 4-D tiled load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile whose rows are `rowbytes` (32, 64
// or 128) long and which TMA wrote with the matching CU_TENSOR_MAP_SWIZZLE_{32,64,128}B mode into
// a 1024-byte-aligned buffer: the chunk index is XORed with bits 7.. of the row's byte offset.
__device__ __forceinline__ unsigned swizzled_chunk(unsigned row, unsigned chunk, unsigned rowbytes) {
    const unsigned base = row * rowbytes;
    const unsigned mask = rowbytes / 16u - 1u;
    return base + (((chunk ^ (base >> 7)) & mask) << 4);
}

// Host side: builds a tiled tensor map; returns false when the driver entry point is missing
// or the encoder rejects the description (alignment, strides, box).
bool encode_tensor_map(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                       const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                       CUtensorMapSwizzle swizzle);

}  // namespace rfdetr
