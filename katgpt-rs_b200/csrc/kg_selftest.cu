// kg_selftest.cu — a check of the bounded-wait path every pipelined kernel
// relies on (no reference counterpart: the reference has no device code).
//
// The tcgen05 GEMM and attention kernels wait on mbarriers with a clock
// limit; when it runs out the CTA raises its abort flag, writes
// KG_ERR_TIMEOUT to the context's error word and returns, so a lost arrival
// ends the call with an error status and the context stays usable. This
// kernel exercises exactly that path on purpose with a short limit: one
// thread waits on a barrier that nothing arrives on.
#include <cuda_runtime.h>

#include <string>

#include "kg_async.cuh"
#include "kg_internal.h"

namespace {

__global__ void wait_timeout_kernel(long long limit_cycles, int *err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        kg::as::mbar_init(&bar, 1);  // one arrival expected, none made
        abort_flag = 0;
        kg::as::mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) kg::as::mbar_wait_for(&bar, 0, &abort_flag, err, limit_cycles);
}

}  // namespace

extern "C" int kg_selftest_wait_timeout(kg_ctx *ctx, int64_t limit_cycles) {
    if (!ctx || limit_cycles < 1 || limit_cycles > ((int64_t)1 << 32)) return KG_ERR_INVALID_ARG;
    cudaError_t e = cudaSetDevice(ctx->device);
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_err, 0, 4, ctx->stream);
    if (e == cudaSuccess) {
        wait_timeout_kernel<<<1, 32, 0, ctx->stream>>>((long long)limit_cycles, ctx->d_err);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, ctx->d_err, 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_err, 0, 4, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        ctx->err = std::string("wait self-test: ") + cudaGetErrorString(e);
        return KG_ERR_CUDA;
    }
    if (herr == KG_ERR_TIMEOUT) {
        ctx->err = "a device-side wait exceeded its limit";
        return KG_ERR_TIMEOUT;
    }
    return herr ? KG_ERR_CUDA : KG_OK;
}
