// The fused decode step (k_step.cu): one cooperative launch runs a whole decode step - every
// layer, the final norm and the head - for B <= 64 sequences of one token each.
//
// One CTA per SM, grid-wide barriers between the step's dependent phases (per layer: norm +
// quant, q|k|v GEMM, attention, o GEMM, norm + quant, gate|up GEMM, gated quant, down GEMM). The
// weights do not depend on the step's data, so a producer thread per CTA streams the weight
// slices of the CTA's coming GEMM work into a shared-memory ring as soon as slots free up, ahead
// of the barriers: the GEMM phases start with their weights on chip. A GEMM phase writes int32
// partial sums per K chunk (exact in any order); the phase after it adds them up and runs the
// GEMM's epilogue fused with its own work (residual add, norm, attention prologue, gating).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace tc {

constexpr int kStepSegs = 8;
constexpr int kStepMaxTok = 64;     // token rows per step (sequences of one token each)
constexpr int kStepSliceBytes = 128 * 128;

// Operand layout in HBM. Every operand slice the step's MMAs read is one contiguous block that a
// single 1-D bulk copy brings on chip, already in the shared-memory layout of the MMA's K-major
// operand with the 128-byte swizzle: row r of a slice (128 bytes of K) at byte 128 r, its 16-byte
// chunk c at chunk c ^ (r mod 8). The weights are re-laid out once per engine as [tile][slice]
// blocks of 128 rows (rows past the matrix zero); the step's int8 rows are written by the row
// phases as [slice][ntok rows].
__host__ __device__ inline uint32_t step_swz(uint32_t row, uint32_t byte) {
  return row * 128u + ((((byte >> 4) ^ (row & 7u)) << 4) | (byte & 15u));
}

// One GEMM of the step: weight segments (row tiles of 128 rows) concatenated along the output
// columns. The K slices (128 bytes each) form ksplit chunks of KC slices; CTA c takes chunk
// c % ksplit of the row tiles t = c / ksplit, + groups, ... and writes the int32 partial sums
// part[chunk][m][col] (the head, ksplit 1: the fp32 logits through the GEMM epilogue).
struct StepGemm {
  const uint8_t* wt;                // the weights re-laid out: [tile][slice] blocks of 16 KB
  int nseg;
  int tile0[kStepSegs + 1];         // row tiles of segment s: [tile0[s], tile0[s + 1])
  int col0[kStepSegs + 1];          // output columns of segment s: [col0[s], col0[s + 1])
  const float* scale[kStepSegs];    // per-row fp32 scales of segment s
  int nslices, kb;                  // K / 128; K slices of the first K block
  int KC, ksplit, groups;
};

struct StepLayer {
  StepGemm qkv, o, gu, down;
  const float *ln_in, *ln_post, *attn_norm, *mlp_norm, *qn, *kn, *tab;
  float *kc, *vc;                   // [B][Tp][n_kv][hd] fp32
};

struct StepArgs {
  const StepLayer* layers;          // [L], device memory
  StepGemm head;
  int L, B, ntok, H, I, nh, nkv, hd, rot, Tp, vocab, gemma, act, ldq;
  int tile, agroups;                // attention: keys per staged tile; concurrent units per CTA
  int gchunks;                      // gated MLP: units per row
  float eps, embed_scale;
  const float* E;                   // fp32 embedding table [vocab][H]
  const int* tok;                   // the step's token ids [B]
  const int* pos;                   // each sequence's position [B]
  const float* final_norm;
  float *x, *x1;                    // residual stream [B][H] (after attention: x1)
  uint8_t* q8t;                     // the step's int8 rows: [slice][ntok][128] in the operand layout
  float *qsa, *qsb;                 // their row scales, two alternating buffers [B]
  int* part;                        // int32 partial sums
  float* att;                       // attention output rows [B][nh * hd]
  float* amax;                      // per (sequence, kv head) absmax of the attention output
  float* gv;                        // the gated MLP's rows act(gate) * up [B][I]
  float* gmax;                      // their absmax per (row, unit)
  float* logits;                    // [B][vocab]
  unsigned* sync;                   // [0] grid barrier count, [1 + b] arrivals of sequence b's
                                    // attention units, [1 + B + m] of row m's gated units; zeroed
                                    // before every launch
  int* err;                         // the device word of bounded waits that gave up
  int* diag;                        // the first give-up: code, CTA, barrier count, detail
  uint64_t wait_ns, drain_ns;       // time limits of the waits for work / for copies in flight
  int lead;                         // the producer streams a GEMM's weights from `lead` barriers
                                    // before its phase on (large: as soon as ring slots free up)
  unsigned long long* trace;        // [0, 1024): CTA 0 leaving every barrier (0: the kernel's
                                    // start); from 1024: per barrier every CTA's arrival; or null
};

// Shared memory a CTA of the step kernel uses, and its staging region for rows / attention.
size_t step_smem_bytes();
int step_region_bytes();
// Plans one GEMM (KC, ksplit, groups) for `grid` CTAs; false when it does not fit.
bool step_plan_gemm(StepGemm& g, int ntok, int grid, bool fused);
// The attention's K / V tile (keys per staged tile) for a head dim, query heads per kv head and
// concurrent units per CTA; 0 when they do not fit.
int step_attn_tile(int hd, int G, int ngroups);
cudaError_t step_launch(const StepArgs& a, int grid, cudaStream_t st);
// CTAs of the step kernel that fit one SM (1 when it fits at all).
cudaError_t step_occupancy(int* per_sm);
// Writes rows [0, n) of an int8 weight (first K block w: [n][kb], second w2: [n][K - kb], or kb ==
// K) as slices of 128 rows into out (step_swz layout, [tile][slice]).
cudaError_t step_retile(const int8_t* w, const int8_t* w2, int n, int K, int kb, uint8_t* out, cudaStream_t st);

}  // namespace tc
