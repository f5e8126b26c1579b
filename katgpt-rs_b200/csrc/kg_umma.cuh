// kg_umma.cuh — tcgen05 / TMA GEMM for prefill shapes (kg_umma.cu).
#pragma once
#include "kg_bf16.cuh"

namespace kg {
namespace umma {

// The operand / epilogue forms the kernel takes (one batch, K a multiple of
// 64, 16-byte aligned rows and bases); false also when the driver's tensor
// map encoder is unavailable.
bool supported(const bf::Gemm &g);
// C = A * B^T through tcgen05.mma with the bf::Gemm epilogues. A device wait
// that exceeds its clock limit writes KG_ERR_TIMEOUT to *err (if err).
cudaError_t gemm(const bf::Gemm &g, cudaStream_t s, int *err);

}  // namespace umma
}  // namespace kg
