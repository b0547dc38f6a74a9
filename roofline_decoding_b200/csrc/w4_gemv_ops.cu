// w4_gemv_ops.cu - generic instances of the fused W4A16 GEMV (prologue,
// epilogue and gathered (peer) output chosen at run time; used for every
// combination without an instance of its own, and for the column-parallel
// gather) and the plain instances whose CTA columns stream several column
// tiles (large N), including the 16-warp tiles only they have.
#include "w4_gemv_kernel.cuh"

namespace w4 {

void* gemv_kernel_generic(int bf16, int mb, int sw, int rg) {
  if (bf16)
    return mb == 1 ? gemv_pick_tile<true, 1, kOpsGeneric>(sw, rg)
                   : gemv_pick_tile<true, 2, kOpsGeneric>(sw, rg);
  return mb == 1 ? gemv_pick_tile<false, 1, kOpsGeneric>(sw, rg)
                 : gemv_pick_tile<false, 2, kOpsGeneric>(sw, rg);
}

void* gemv_kernel_plain_tiles(int bf16, int mb, int sw, int rg) {
  if (bf16)
    return mb == 1 ? gemv_pick_stream_tile<true, 1>(sw, rg) : gemv_pick_stream_tile<true, 2>(sw, rg);
  return mb == 1 ? gemv_pick_stream_tile<false, 1>(sw, rg) : gemv_pick_stream_tile<false, 2>(sw, rg);
}

// The plain GEMV whose output is gathered into every rank's buffer
// (w4_gemv_allgather): without the generic instance's run-time prologue and
// epilogue it keeps the plain instance's register count, hence its CTAs per SM.
void* gemv_kernel_peer(int bf16, int mb, int sw, int rg) {
  if (bf16)
    return mb == 1 ? gemv_pick_tile<true, 1, kOpsPeer>(sw, rg) : gemv_pick_tile<true, 2, kOpsPeer>(sw, rg);
  return mb == 1 ? gemv_pick_tile<false, 1, kOpsPeer>(sw, rg) : gemv_pick_tile<false, 2, kOpsPeer>(sw, rg);
}

}  // namespace w4
