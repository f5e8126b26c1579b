// kg_async.cuh — mbarrier, TMA and bulk-copy helpers shared by the tcgen05
// GEMM (kg_umma.cu) and the decode-attention scores kernel (kg_tqattn.cu).
//
// Every wait is bounded: mbar_wait gives up after `KG_WAIT_CYCLES` clock
// cycles (about 2 s), raises the CTA's abort flag and writes KG_ERR_TIMEOUT to
// the device error word, so a lost arrival ends the kernel with an error
// status instead of a hang.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/kg_abi.h"

namespace kg {
namespace as {

constexpr long long KG_WAIT_CYCLES = 4ll << 30;

__device__ __forceinline__ uint32_t sa(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(sa(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of `parity` to complete; false when the clock limit
// passed (the abort flag and *err are set) or another thread already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *b, uint32_t parity, volatile int *abort_flag, int *err,
                                              long long limit_cycles) {
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(b, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > limit_cycles) {
            *abort_flag = 1;
            if (err) atomicExch(err, (int)KG_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag, int *err) {
    return mbar_wait_for(b, parity, abort_flag, err, KG_WAIT_CYCLES);
}

// 2-D tiled TMA load of one box into shared memory, completion on `bar`
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(sa(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(sa(bar))
        : "memory");
}
// Prefetch one box of a 2-D tiled tensor map into L2 (no shared memory, no
// barrier): a producer issues it a few stages ahead of its ring so that the
// stage's own TMA load finds the bytes in L2 instead of waiting on HBM.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *tm, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];\n" ::"l"(tm), "r"(x), "r"(y)
                 : "memory");
}
// contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(sa(dst)),
        "l"(src), "r"(bytes), "r"(sa(bar))
        : "memory");
}

}  // namespace as

// Host: the driver's tensor-map encoder (null when unavailable) and a 2-D map
// over a row-major [rows x cols] matrix of `elem`-byte elements with leading
// dimension ld (elements), box = box_cols x box_rows.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
bool make_tensor_map(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int64_t ld, int elem,
                     int box_cols, int box_rows, CUtensorMapSwizzle swizzle);

}  // namespace kg
