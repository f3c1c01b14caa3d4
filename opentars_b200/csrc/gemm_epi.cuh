// The W8A8 GEMM epilogue of the descriptor path (golden.py:326-349), shared by the SIMT GEMV
// kernels and the tensor-core GEMM: y = i2f(acc); [y = fmul(y, srow[m])]; y = fmul(y, scale[n or 0]);
// [y = fadd(y, bias[n])]; y = act(y); stored in the output format.
#pragma once
#include "fp32.cuh"
#include "ops.h"

namespace tc {

__device__ __forceinline__ void gemm_epilogue(const GemmArgs& g, int m, int n, int acc) {
  float y = i2f(acc);
  if (g.srow) y = fmul(y, ld_f32(g.srow + 4 * (uint64_t)m));
  y = fmul(y, ld_f32(g.scale + (g.per_channel ? 4 * (uint64_t)n : 0)));
  if (g.bias) y = fadd(y, ld_f32(g.bias + 4 * (uint64_t)n));
  y = act_fn(y, g.act);
  store_out(g.Y + (uint64_t)m * g.ldy, n, y, g.out, g.out_scale);
}

}  // namespace tc
