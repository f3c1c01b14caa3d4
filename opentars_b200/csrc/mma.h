// The tensor-core (tcgen05, kind::i8) W8A8 GEMM of k_mma.cu: entry points for the decode engine
// and for the descriptor path. Each *_ok check says whether the operands meet the TMA rules
// (16-byte aligned bases and row strides, K a multiple of 16) so the caller can pick the kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "engine.h"
#include "ops.h"

namespace tc {

bool mma_engine_ok(const EngGemvArgs& g);
cudaError_t eng_gemm_mma(const EngGemvArgs& g, cudaStream_t st);
bool mma_machine_ok(const GemmArgs& g);
cudaError_t gemm_mma(const GemmArgs& g, cudaStream_t st);
// Smallest token-row count routed to the tensor-core kernel (TARSCUDA_MMA_MIN_M, default 16).
int mma_min_rows();
// Nonzero when a bounded wait of the tensor-core kernel gave up (1 producer, 2 MMA, 3 epilogue).
int mma_error_code();
// The device word every streaming kernel records a given-up bounded wait in (codes: tensor-core
// GEMM 1-5, grouped GEMV 21-22, streamed W4A16 GEMV 11-12); read by tc_wait_error.
int* wait_error_flag();
// The poll limit of the bounded waits for work (tc_set_spin_limit).
uint32_t spin_limit();
// A TMA map of a uint8 matrix [rows, cols] (row stride ld) in boxes of box_cols x box_rows, with the
// 128-byte swizzle or dense rows; false when the driver entry point is missing or an alignment rule
// fails.
bool make_map_u8(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows, bool swizzle = true);

}  // namespace tc
