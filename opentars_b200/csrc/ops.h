// Kernel launch interfaces of libtarscuda (device pointers + sizes; no torch types).
//
// Each launcher enqueues the work of one descriptor (or of one fused engine step) on `st`.
// Pointers are device addresses inside the HBM copy of the DDR image unless noted.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "codes.h"

namespace tc {

// W8A8 GEMM / GEMV, golden.py:326-349 (and the conv's implicit GEMM, golden.py:282-293)
struct GemmArgs {
  const uint8_t* A;  uint64_t lda;   // int8 [M, K] rows
  const uint8_t* W;                  // int8 [N, K] dense
  const uint8_t* scale;              // fp32 [N] (per channel) or [1] (per tensor)
  int per_channel;
  const uint8_t* srow;               // fp32 [M] row scales (QM_ROWCOL) or nullptr
  const uint8_t* bias;               // fp32 [N] or nullptr
  uint8_t* Y;  uint64_t ldy;
  int M, N, K, act, out;
  float out_scale;
};
cudaError_t launch_gemm_w8a8(const GemmArgs& g, cudaStream_t st);

// Independent descriptors of one dependency level batched into one launch (queue capture).
// Every entry is computed exactly as its own launch would compute it.
constexpr int kGroupMax = 64;

// Decode GEMVs of one kernel class (token rows per pass MB, K <= 512 * KU), streamed in chunks of
// 16 output columns: entry j owns chunks [c0[j], c0[j + 1]), ncx[j] = N / 16 chunks per pass of
// MB token rows.
struct GemvGroup {
  int n, mb, ku;
  int c0[kGroupMax + 1];
  int ncx[kGroupMax];
  GemmArgs g[kGroupMax];
  int* err;                          // device word for a bounded wait that gave up (set by the launcher)
  uint32_t spin;                     // poll limit of the bounded waits (set by the launcher)
};
// The class of a GEMM that the grouped decode GEMV computes (MB * 16 + KU), or -1.
int gemv8_class(const GemmArgs& g);
// Fills grp.c0 / grp.ncx and launches.
cudaError_t launch_gemv8_group(GemvGroup& grp, cudaStream_t st);

// W4A16 GEMM / GEMV, golden.py:295-324
struct W4Args {
  const uint8_t* A;  uint64_t lda;   // fp32 or bf16 [M, K] rows
  int a_bf16;
  const uint8_t* W;                  // packed int4 [N, K/2] (low nibble = even k)
  const uint8_t* scale;              // fp16 bits [N, K/128]
  const uint8_t* bias;               // fp32 [N] or nullptr
  uint8_t* Y;  uint64_t ldy;
  int M, N, K, act, out;
  float out_scale;
  int* err;                          // device word for a bounded wait that gave up (set by the launcher)
  uint32_t spin;                     // poll limit of the bounded waits (set by the launcher)
  uint8_t* scratch;                  // w4_scratch_bytes(M, K) of device memory for the aligned rows,
                                     // or nullptr (then the kernels align in every block)
};
cudaError_t launch_gemm_w4a16(const W4Args& g, cudaStream_t st);
// Scratch the tiled W4A16 GEMV needs for M rows of K (16-byte aligned).
uint64_t w4_scratch_bytes(int M, int K);
// Up to kW4GroupMax independent W4A16 GEMVs as one pre-pass and one tiled launch; `w4_group_class`
// is the key of GEMVs that may share a launch (the same row block and K), or -1 when the tiled
// kernel does not take the GEMV (each entry then needs a launch of its own).
constexpr int kW4GroupMax = 8;
int w4_group_class(const W4Args& g);
cudaError_t launch_w4_group(const W4Args* gs, int n, cudaStream_t st);

// conv: the NHWC int8 image gathered into [OH*OW, KH*KW*Cin] rows (zero padding), golden.py:282-293
struct Im2colArgs {
  const uint8_t* img;  uint64_t ld;  // H*W pixel rows of Cin bytes, row stride ld
  uint8_t* out;                      // [OH*OW, K] dense
  int H, W, KH, KW, S, P, Cin, OH, OW;
};
cudaError_t launch_im2col(const Im2colArgs& a, cudaStream_t st);

// Row ops (OPCODE 0x04), golden.py:358-380 and the RELU op (0x03), golden.py:351-356
struct RowArgs {
  const uint8_t* X;  uint64_t lda;   // fp32 [M, N]
  uint8_t* Y;  uint64_t ldy;
  const uint8_t* gamma;              // fp32 [N] (norms)
  const uint8_t* beta;               // fp32 [N] or nullptr
  uint8_t* scale_out;                // ROW_QUANT: fp32 [M]
  int M, N, fn, out, K;              // K: causal softmax start (0 = plain)
  float eps, out_scale;
};
cudaError_t launch_rowop(const RowArgs& a, cudaStream_t st);

// Row ops of one dependency level: entry j owns blocks (rows) [row0[j], row0[j + 1]); nmax is the
// longest row (floats) of the group.
struct RowGroup {
  int n, nmax;
  int row0[kGroupMax + 1];
  RowArgs a[kGroupMax];
};
bool rowop_groupable(const RowArgs& a);
cudaError_t launch_rowop_group(const RowGroup& g, cudaStream_t st);

struct ActArgs {
  const uint8_t* X;  uint64_t lda;
  uint8_t* Y;  uint64_t ldy;
  int M, N, act, out;
  float out_scale;
};
cudaError_t launch_act(const ActArgs& a, cudaStream_t st);

// ELT (0x06), golden.py:393-418
struct EltArgs {
  const uint8_t* A;  uint64_t lda;   // lda = 0: one row broadcast
  int a_fp16;
  const uint8_t* B;  uint64_t ldb;  int bmode;
  const uint8_t* C;                  // MULADD addend (output format, stride ldy) or nullptr
  uint8_t* Y;  uint64_t ldy;
  int M, N, op, act, out;
  float out_scale;
};
cudaError_t launch_elt(const EltArgs& a, cudaStream_t st);

// ROPE (0x07), golden.py:420-424
struct RopeArgs {
  const uint8_t* X;  uint64_t lda;
  const uint8_t* tab;                // fp32 [rows, R]: cos[0:R/2], sin[0:R/2]
  uint8_t* Y;  uint64_t ldy;
  int M, N, R, G, out;
  float out_scale;
};
cudaError_t launch_rope(const RopeArgs& a, cudaStream_t st);

// FDOT (0x08), golden.py:426-435
struct FdotArgs {
  const uint8_t* A;  uint64_t lda;   // fp32 [M, K]
  const uint8_t* B;  uint64_t ldb;   // NT: fp32 [N, K]; NN: fp32 or fp16 [K, N]
  int nn, b_fp16;
  uint8_t* Y;  uint64_t ldy;
  int M, N, K, out;
  float out_scale;
  int vec;                           // set by the launcher: A and B rows 16-byte aligned
};
cudaError_t launch_fdot(const FdotArgs& a, cudaStream_t st);

}  // namespace tc
