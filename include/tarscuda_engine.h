/* libtarscuda decode engine: B independent sequences of a Qwen3 / Gemma 3 model decoded together
 * on one B200, bit-exact per sequence with the descriptor path (and so with the reference's golden
 * model).
 *
 * Replaces, for a whole batch, the per-token loop of the reference's QwenLowering.generate
 * (tars_mini/llm.py:815-836: host embedding lookup, run(ddr, q, n) of the chunk's queue, argmax of
 * the logits) and of the board runtime's Qwen.step / prefill (deploy/kv260/sw/tars_board.py:
 * 400-435). The weights are the DDR image that the lowering built (QwenLowering, llm.py:213-476),
 * opened with tc_open/tc_upload; the model description gives the image offsets of every layer's
 * tensors (the lowering's QLin / V records).
 */
#ifndef TARSCUDA_ENGINE_H
#define TARSCUDA_ENGINE_H
#include <stdint.h>

#include "tarscuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct tc_engine tc_engine;

/* One W8A8 linear in the image: int8 rows [n, k] at w_off, fp32 per-row scales at s_off (llm.py:181-188). */
typedef struct { uint64_t w_off, s_off; int32_t n, k; } tc_lin;

/* One full-attention layer (llm.py:365-418): norm gammas (0 = absent: Gemma 3 has attn_norm and
 * mlp_norm, Qwen3 not), q/k head-norm gammas (q's with the attention scaling folded in), the RoPE
 * table of the layer's type, the linears; down in n_down K blocks sharing one scale (llm.py:303-321). */
typedef struct {
  uint64_t ln_in, ln_post, attn_norm, mlp_norm, qn, kn, rope_tab;
  tc_lin q, k, v, o, gate, up;
  tc_lin down[4];
  int32_t n_down;
} tc_layer_desc;

typedef struct {
  int32_t n_layers, hidden, inter, n_heads, n_kv, head_dim, rot, vocab, max_tokens;
  int32_t act;            /* the gate's activation code: 4 SiLU (Qwen3), 3 tanh GELU (Gemma 3) */
  int32_t gemma;          /* Gemma 3: scaled embedding, attn_norm / mlp_norm */
  float eps, embed_scale;  /* the RMSNorm epsilon as fp32; Gemma's embedding scale fp32(sqrt(hidden)) */
  uint64_t final_norm;
  int32_t n_head_blocks;
  tc_lin head[8];         /* the tied head in row blocks of <= 65535 (qwen_ref.py:371-378) */
} tc_model_desc;

/* A decode engine over the weights in `image` for `batch` sequences; uploads the fp32 embedding
 * table [vocab][hidden] from embed_host; KV caches zeroed, position 0. TC_ERR_ARG (and *out = NULL)
 * for a missing argument or a model the engine does not serve. */
int tc_engine_create(tc_machine* image, const tc_model_desc* md, const tc_layer_desc* layers,
                     const float* embed_host, int32_t batch, tc_engine** out);
int tc_engine_destroy(tc_engine* e);
const char* tc_engine_error(tc_engine* e);
void* tc_engine_stream(tc_engine* e);
/* Zeroes every KV cache and the position (a new batch of conversations). */
int tc_engine_reset(tc_engine* e);
/* One chunk of n (1..4) tokens per sequence: tokens_host [batch][n] ids, or NULL to feed each
 * sequence's greedy pick of the previous chunk (n = 1). Enqueued on the engine's stream. */
int tc_engine_step(tc_engine* e, const int32_t* tokens_host, int32_t n);
/* The next token of each sequence (np.argmax of its last logits row) into / from the host. */
int tc_engine_tokens(tc_engine* e, int32_t* tokens_host);
int tc_engine_set_tokens(tc_engine* e, const int32_t* tokens_host);
/* Each sequence's logits of its last token [batch][vocab]. */
int tc_engine_logits(tc_engine* e, float* logits_host);
int tc_engine_sync(tc_engine* e);
/* Runs one decode step (n = 1, the previous picks as input) kernel by kernel, not captured, with
 * events around each launch: ms[i], kind[i] (0 embed, 1 norm+quant, 2 GEMV, 3 q/k norm+RoPE,
 * 4 attention, 5 quant, 6 argmax, 7 position) and the kernel's algorithmic bytes[i]. Returns the
 * number of kernels (the step counts as a decode step: the position advances). */
int tc_engine_profile(tc_engine* e, float* ms, int32_t* kind, uint64_t* bytes, uint32_t cap);
/* Starts sequence b afresh (a new conversation in that slot of a running batch): zeroes its KV
 * cache rows in every layer and sets its position to 0; the other sequences keep theirs. Sequences
 * at different positions step together: every step advances each sequence by the chunk's n tokens
 * (the continuous batching of a server; the reference decodes one sequence at a time). A step that
 * would take any sequence past max_tokens, or a host token id outside the vocabulary, is refused
 * (TC_ERR_ARG) before anything runs. */
int tc_engine_reset_seq(tc_engine* e, int32_t b);
/* Each sequence's position (its next token's index) [batch] into the host. */
int tc_engine_positions(tc_engine* e, int32_t* pos_host);
/* The fused decode step: one-token steps run as one cooperative kernel over every SM (all layers,
 * the final norm and the head; then the greedy pick) when the model and batch fit it (batch <= 64,
 * every K a multiple of 128, head dim 64 / 128 / 256); otherwise, and for chunks of more tokens, as
 * the per-kernel graph. enable 1 / 0 turns it on / off (on only where it was set up), -1 only asks;
 * returns whether it was on. tc_engine_fused_why says why it is not available. No counterpart in
 * the reference. */
int tc_engine_fused(tc_engine* e, int32_t enable);
const char* tc_engine_fused_why(tc_engine* e);
/* Where the fused step's first bounded wait gave up, if one did (tc_wait_error then reads its
 * code): out4 = {code (31 grid barrier, 41 weight slot, 42 rows copy, 43 accumulator free, 44
 * weight slice, 45 accumulator ready), CTA, grid barriers passed, detail}; zeros when none did.
 * Synchronous. */
int tc_engine_fused_diag(tc_engine* e, int32_t* out4);
/* Runs one fused decode step (the previous picks as input) with a globaltimer stamp (ns) at the
 * kernel's grid barriers, taken by its first CTA: per layer 8 phases (norm + quant, q|k|v GEMM,
 * attention, o GEMM, norm + quant, gate|up GEMM, gated quant, down GEMM), then the final norm and
 * the head; stamps[0] is the kernel's start. Returns the number of stamps (TC_ERR_ARG when the
 * fused step is off). The step counts as a decode step. */
int tc_engine_phase_times(tc_engine* e, uint64_t* stamps, uint32_t cap);
/* The engine's greedy pick on its own: tok_out[r] = np.argmax(logits[r]) for rows r < rows of
 * device logits [rows][vocab] (the first maximum; the first NaN wins over numbers): the
 * np.argmax of llm.py:834 and of tars_board.py:355. Device pointers; enqueued on `stream` (NULL:
 * the default stream). TC_ERR_ARG for null pointers, vocab or rows <= 0, or rows > 2^24. */
int tc_argmax(const float* logits, int32_t vocab, int32_t rows, int32_t* tok_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
