// The batched decode engine's kernel interfaces (see k_engine.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace tc {

enum { kEpiStore = 0, kEpiResid = 1, kEpiGated = 2, kEpiKSplit = 3 };
constexpr int kMaxSegs = 8;

// One block of weight rows [n, K] int8 (or two K blocks of one weight, the lowering's lin_k) with
// its per-row fp32 scales; its outputs are columns
// [n0, n0 + n) of the concatenated result, stored at out[m * ldo + c].
struct EngSeg {
  const int8_t* W;                 // rows of the first K block ([n, kb])
  const int8_t* W2;                // rows of the second K block ([n, K - kb]) when kb < K
  const float* scale;
  float* out;
  uint64_t ldo;
  int n0, n;
};

struct EngGemvArgs {
  const int8_t* A;  uint64_t lda;  // int8 rows [M, K]
  const float* srow;               // their row scales [M]
  int M, K, kb;                    // kb < K: two K blocks [0, kb) and [kb, K) sharing the scales
  int nseg, ncols;
  EngSeg seg[kMaxSegs];
  int mode, act;
  const float* res;  uint64_t ldres;   // residual rows (kEpiResid, or kEpiKSplit when given)
};

struct NormQuantArgs {
  const float* in;  uint64_t ld_in;
  const float* res;  float* x_out;     // mode 1, 2: x = res + (in or norm(in)), written to x_out
  const float* pre_gamma;              // mode 2
  const float* gamma;
  float eps;
  int8_t* q;  uint64_t ldq;
  float* qs;
  int H, rows, mode;
};

struct QkRopeArgs {
  const float* q;  const float* k;  const float* v;
  float* qr;  float* kc;  float* vc;
  const float* qn;  const float* kn;
  const float* tab;
  const int* pos;                      // each sequence's position [batch]
  int rows, n, nh, nkv, hd, rot, Tp;
  float eps;
};

struct AttnArgs {
  const float* qr;  const float* kc;  const float* vc;
  float* att;
  const int* pos;                      // each sequence's position [batch]
  int n, nh, nkv, hd, Tp;
};

cudaError_t eng_embed(const float* E, const int* tok, float* x, int H, int scale_on, float scale, int rows, cudaStream_t st);
cudaError_t eng_norm_quant(const NormQuantArgs& a, cudaStream_t st);
cudaError_t eng_quant(const float* x, int ldx, int N, int8_t* q, int ldq, float* qs, int rows, cudaStream_t st);
// rows of ftz(fmul(ftz(act(gate)), up)) quantised per row (the gated MLP's product and ROW_QUANT)
cudaError_t eng_quant_gated(const float* gate, const float* up, int ld, int N, int act, int8_t* q, int ldq, float* qs,
                            int rows, cudaStream_t st);
cudaError_t eng_gemv(const EngGemvArgs& g, cudaStream_t st);
cudaError_t eng_qk_rope(const QkRopeArgs& a, cudaStream_t st);
cudaError_t eng_attention(const AttnArgs& a, int batch, cudaStream_t st);
// q / k RMSNorm + RoPE (and the K / V cache writes), attention and the ROW_QUANT of the attention
// output rows in one launch: one block per (sequence, kv head), the kv heads of a sequence one
// thread-block cluster (n_kv <= 8) that shares the row absmax. Same bits as eng_qk_rope +
// eng_attention + eng_quant; r.qr and a.qr / a.att are not used.
struct AttnQuantArgs {
  QkRopeArgs r;
  int8_t* q8;  uint64_t ldq;
  float* qs;
};
cudaError_t eng_attention_quant(const AttnArgs& a, const AttnQuantArgs& f, int batch, cudaStream_t st);
cudaError_t eng_argmax(const float* logits, int vocab, int batch, int* tok_out, int tok_stride, cudaStream_t st);
cudaError_t eng_advance(int* pos, int n, int batch, cudaStream_t st);

}  // namespace tc
