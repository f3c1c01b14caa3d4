// The W8A8 GEMM epilogue of the descriptor path (golden.py:326-349), shared by the SIMT GEMV
// kernels and the tensor-core GEMM: y = i2f(acc); [y = fmul(y, srow[m])]; y = fmul(y, scale[n or 0]);
// [y = fadd(y, bias[n])]; y = act(y); stored in the output format.
#pragma once
#include "fp32.cuh"
#include "ops.h"

namespace tc {

// With the column's scale `sc` and bias `bi` already loaded (bi is unused without a bias).
__device__ __forceinline__ void gemm_epilogue_v(const GemmArgs& g, int m, int n, int acc, float sc, float bi) {
  float y = i2f(acc);
  if (g.srow) y = fmul(y, ld_f32(g.srow + 4 * (uint64_t)m));
  y = fmul(y, sc);
  if (g.bias) y = fadd(y, bi);
  y = act_fn(y, g.act);
  store_out(g.Y + (uint64_t)m * g.ldy, n, y, g.out, g.out_scale);
}

__device__ __forceinline__ void gemm_epilogue(const GemmArgs& g, int m, int n, int acc) {
  const float sc = ld_f32(g.scale + (g.per_channel ? 4 * (uint64_t)n : 0));
  const float bi = g.bias ? ld_f32(g.bias + 4 * (uint64_t)n) : 0.0f;
  gemm_epilogue_v(g, m, n, acc, sc, bi);
}

}  // namespace tc
