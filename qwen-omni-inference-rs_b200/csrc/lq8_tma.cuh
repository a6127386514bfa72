// lq8_tma.cuh -- 2-D TMA tensor maps (encoded through the driver entry point, no -lcuda
// link) and the tiled load. Loads only: no multicast, this GPU's memory only.
#pragma once

#include <cuda.h>

#include "lq8_async.cuh"
#include "lq8_internal.cuh"

namespace lq {

// [outer][inner] tensor of 1- or 2-byte elements, row pitch row_bytes (a multiple of 16),
// box {box_inner, box_outer}; base 16-byte aligned
int make_tensor_map_2d(lq_ctx* ctx, CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                       uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                       CUtensorMapSwizzle swz);

// box at element coordinates (x, y) into shared memory, completion counted on bar (bytes);
// x * element size must be a multiple of 16
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// fetch a tensor map (kernel parameter) into the TMA unit's cache ahead of its first use
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace lq
