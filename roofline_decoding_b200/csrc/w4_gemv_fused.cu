// w4_gemv_fused.cu - instances of the fused W4A16 GEMV for the operation
// combinations of a decode step (bf16 activations, up to 8 batch rows):
// RMSNorm + bias (q|k|v), RMSNorm (gate|up), RMSNorm + SwiGLU (gate|up with
// gate and up interleaved), residual (o), SwiGLU + residual (down). Each
// contains only its own prologue and epilogue code.
#include "w4_gemv_kernel.cuh"

namespace w4 {

void* gemv_kernel_fused(int ops, int sw, int rg) {
  switch (ops) {
    case kOpsRmsBias: return gemv_pick_tile<true, 1, kOpsRmsBias>(sw, rg);
    case kOpsRms: return gemv_pick_tile<true, 1, kOpsRms>(sw, rg);
    case kOpsResidual: return gemv_pick_tile<true, 1, kOpsResidual>(sw, rg);
    case kOpsSwigluResidual: return gemv_pick_tile<true, 1, kOpsSwigluResidual>(sw, rg);
    case kOpsRmsSwiglu: return gemv_pick_tile<true, 1, kOpsRmsSwiglu>(sw, rg);
    default: return nullptr;
  }
}

}  // namespace w4
