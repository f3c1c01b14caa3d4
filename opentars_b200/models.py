"""Host model data for the model images: configs, seeded random weights, weight quantisers.

Restates, for the model families on the hot path (Qwen3, Gemma 3 / 4 and Qwen3.5 text models):
  * make_config          tars_mini/qwen_ref.py:109-146 (transformers config objects)
  * random_weights       qwen_ref.py:165-198 (same generator, same draw order: the model's state_dict)
  * head_rows            qwen_ref.py:371-378 (the vocabulary in the fewest equal blocks <= 65535 rows)
  * quantize_weight      tars_mini/compiler.py:51-57 (per-channel symmetric INT8, float64 then fp32)
  * quantize_weight4     compiler.py:69-85 (group-128 INT4 with binary16 scales)
  * input_embedding, ple_embedding   tars_mini/llm.py:198-211
The host quantisers define data, not device arithmetic: they run once when an image is built.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32
W4_GROUP = 128

VOCAB_Q3_06B = 151936
CFG_Q3_06B = dict(model_type="qwen3", hidden_size=1024, intermediate_size=3072, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, vocab_size=16,
                  max_position_embeddings=40960, num_hidden_layers=28,
                  rope_parameters=dict(rope_type="default", rope_theta=1000000.0))
CFG_Q3_SMALL = dict(CFG_Q3_06B, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=64)
VOCAB_G3_1B = 262144
LAYERS_G3_1B = (["sliding_attention"] * 5 + ["full_attention"]) * 4 + ["sliding_attention"] * 2
CFG_G3_1B = dict(model_type="gemma3_text", hidden_size=1152, intermediate_size=6912, num_attention_heads=4,
                 num_key_value_heads=1, head_dim=256, query_pre_attn_scalar=256, rms_norm_eps=1e-6, vocab_size=16,
                 sliding_window=512, hidden_activation="gelu_pytorch_tanh", max_position_embeddings=32768,
                 attn_logit_softcapping=None, final_logit_softcapping=None,
                 rope_parameters={"full_attention": dict(rope_type="default", rope_theta=1000000.0),
                                  "sliding_attention": dict(rope_type="default", rope_theta=10000.0)})
CFG_G3_SMALL = dict(CFG_G3_1B, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, head_dim=64, query_pre_attn_scalar=64, sliding_window=64)

# Gemma 4 E2B's text model (qwen_ref.py:59-81): 4 sliding layers to 1 full layer, head_dim 256 /
# 512 (full), proportional 25 % RoPE on full layers, KV sharing over the last layers, double-wide
# MLP on them, per-layer embeddings, V-norm without scale, layer_scalar, softcapped tied head
VOCAB_G4_E2B = 262144
LAYERS_G4_E2B = (["sliding_attention"] * 4 + ["full_attention"]) * 7
CFG_G4_E2B = dict(model_type="gemma4_text", hidden_size=1536, intermediate_size=6144, num_attention_heads=8,
                  num_key_value_heads=1, head_dim=256, global_head_dim=512, hidden_size_per_layer_input=256,
                  vocab_size_per_layer_input=262144, num_kv_shared_layers=20, use_double_wide_mlp=True,
                  enable_moe_block=False, attention_k_eq_v=False, rms_norm_eps=1e-6, vocab_size=16,
                  sliding_window=512, hidden_activation="gelu_pytorch_tanh", max_position_embeddings=131072,
                  final_logit_softcapping=30.0,
                  rope_parameters={"full_attention": dict(rope_type="proportional", rope_theta=1000000.0,
                                                          partial_rotary_factor=0.25),
                                   "sliding_attention": dict(rope_type="default", rope_theta=10000.0)})
CFG_G4_SMALL = dict(CFG_G4_E2B, hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=1,
                    head_dim=64, global_head_dim=128, hidden_size_per_layer_input=128, vocab_size_per_layer_input=16,
                    num_kv_shared_layers=2, sliding_window=64)

# Qwen3.5-0.8B's text model (qwen_ref.py:20-33): 3 gated-DeltaNet layers to 1 gated full-attention
# layer, partial rotary 0.25 (text positions: plain RoPE), tied embeddings; the small variant of the
# block tests (qwen_ref.py:86-88)
VOCAB_08B = 248320
LAYERS_08B = (["linear_attention"] * 3 + ["full_attention"]) * 6
CFG_08B = dict(model_type="qwen3_5_text", hidden_size=1024, intermediate_size=3584, num_attention_heads=8,
               num_key_value_heads=2, head_dim=256, linear_conv_kernel_dim=4, linear_key_head_dim=128,
               linear_value_head_dim=128, linear_num_key_heads=16, linear_num_value_heads=16, rms_norm_eps=1e-6,
               vocab_size=16, max_position_embeddings=262144, attn_output_gate=True,
               rope_parameters=dict(rope_type="default", rope_theta=10000000.0, partial_rotary_factor=0.25,
                                    mrope_section=[11, 11, 10], mrope_interleaved=True))
CFG_Q35_SMALL = dict(CFG_08B, hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                     head_dim=128, linear_key_head_dim=16, linear_value_head_dim=16, linear_num_key_heads=16,
                     linear_num_value_heads=16)


def make_config(base: dict, layer_types: list[str] | None = None, vocab: int | None = None):
    """A transformers config for a Qwen3, Gemma 3, Gemma 4 or Qwen3.5 text model (tied embeddings,
    eager attention)."""
    b = {k: v for k, v in base.items() if k != "model_type"}
    if base.get("model_type") == "gemma4_text":
        from transformers.models.gemma4 import Gemma4TextConfig
        lt = list(layer_types or ["sliding_attention", "full_attention", "sliding_attention", "full_attention"])
        vs = vocab or b["vocab_size"]
        # the per-layer table follows the vocabulary unless the base gives a distinct one
        vs_ple = vs if vocab is not None or b.get("vocab_size_per_layer_input") == b["vocab_size"] \
            else b["vocab_size_per_layer_input"]
        n_shared = min(b.get("num_kv_shared_layers", 0), max(0, len(lt) - 2))
        cfg = Gemma4TextConfig(**dict(b, vocab_size=vs, vocab_size_per_layer_input=vs_ple,
                                      num_kv_shared_layers=n_shared, tie_word_embeddings=True),
                               num_hidden_layers=len(lt), layer_types=lt)
    elif base.get("model_type") == "gemma3_text":
        from transformers.models.gemma3.configuration_gemma3 import Gemma3TextConfig
        lt = list(layer_types or ["sliding_attention", "full_attention"])
        cfg = Gemma3TextConfig(**dict(b, vocab_size=vocab or b["vocab_size"], tie_word_embeddings=True),
                               num_hidden_layers=len(lt), layer_types=lt)
    elif base.get("model_type") == "qwen3":
        from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
        n = len(layer_types) if layer_types else b.pop("num_hidden_layers")
        b.pop("num_hidden_layers", None)
        cfg = Qwen3Config(**dict(b, vocab_size=vocab or b["vocab_size"], tie_word_embeddings=True),
                          num_hidden_layers=n, layer_types=["full_attention"] * n)
    elif base.get("model_type") == "qwen3_5_text":
        from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
        lt = list(layer_types or ["linear_attention", "full_attention"])
        cfg = Qwen3_5TextConfig(**dict(b, vocab_size=vocab or b["vocab_size"], tie_word_embeddings=True),
                                num_hidden_layers=len(lt), layer_types=lt)
    else:
        raise ValueError(f"model type {base.get('model_type')!r} is not on this path (Qwen3, Gemma 3 / 4, Qwen3.5)")
    cfg._attn_implementation = "eager"
    return cfg


def param_shapes(cfg) -> list[tuple[str, tuple[int, ...]]]:
    """The model's parameters (name, shape) in state_dict order, built on the meta device."""
    import torch
    if cfg.model_type == "qwen3":
        from transformers.models.qwen3.modeling_qwen3 import Qwen3Model as Model
    elif cfg.model_type == "qwen3_5_text":
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel as Model
    elif cfg.model_type == "gemma4_text":
        from transformers.models.gemma4 import Gemma4TextModel as Model
    else:
        from transformers.models.gemma3.modeling_gemma3 import Gemma3TextModel as Model
    with torch.device("meta"):
        m = Model(cfg)
    return [(n, tuple(p.shape)) for n, p in m.state_dict().items()]


def _linear_rows(rng, shape) -> np.ndarray:
    """N(0, 0.02), then 2 % of the output rows (one uniform draw per row) times 4."""
    a = rng.normal(0.0, 0.02, shape)
    a[rng.random(shape[0]) < 0.02] *= 4.0
    return a


def _drawer(cfg, name: str, shape: tuple[int, ...]):
    """How one non-embedding parameter is drawn: a function of the generator."""
    if len(shape) == 2:
        return lambda rng: _linear_rows(rng, shape)
    if "conv1d" in name:
        return lambda rng: rng.normal(0.0, 0.3, shape)
    if name.endswith("A_log"):
        return lambda rng: np.log(rng.uniform(1.0, 16.0, shape))
    if name.endswith(("dt_bias", ".layer_scalar")):
        return lambda rng: rng.uniform(0.5, 1.5, shape)
    # norm gains: around 1, except the zero-centred ones (gains applied as 1 + w)
    centred = cfg.model_type not in ("qwen3", "gemma4_text") and not name.endswith("linear_attn.norm.weight")
    return lambda rng: rng.normal(0.0 if centred else 1.0, 0.1, shape)


def _table(rng, shape, std: float, block: int = 8192) -> np.ndarray:
    """An embedding table drawn `block` rows at a time (bounded float64 temporaries)."""
    out = np.empty(shape, F32)
    for r0 in range(0, shape[0], block):
        r1 = min(shape[0], r0 + block)
        out[r0:r1] = rng.normal(0.0, std, (r1 - r0,) + tuple(shape[1:]))
    return out


def random_weights(cfg, seed: int = 0, embed: bool = False) -> dict[str, np.ndarray]:
    """Linears N(0, 0.02) with 2 % of the output rows x4; Qwen3.5's conv taps N(0, 0.3), A_log =
    log U(1, 16), dt_bias (and Gemma 4's layer_scalar) U(0.5, 1.5), the gated norm 1 + N(0, 0.1);
    norms 1 + N(0, 0.1) (Qwen3, Gemma 4) or N(0, 0.1) (Gemma 3 and Qwen3.5, zero-centred); with
    `embed` the embedding tables (the tied one, Gemma 4's per-layer one) N(0, 0.02), drawn 8192
    rows at a time. One generator, parameters in state_dict order."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in param_shapes(cfg):
        if not name.startswith("embed_tokens"):
            out[name] = _drawer(cfg, name, shape)(rng).astype(F32)
        elif embed:
            out[name] = _table(rng, shape, 0.02)
    return out


def random_mtp(cfg, seed: int = 5) -> dict[str, np.ndarray]:
    """Random Qwen3.5 MTP-head weights (qwen_ref.py:258-270): the linears N(0, 0.02) and the norms
    N(0, 0.1), drawn in this order, under the checkpoint's names (mtp.*)."""
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nq, nkv = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd
    attn, mlp = "layers.0.self_attn.", "layers.0.mlp."
    linears = [("fc", (H, 2 * H))]
    linears += [(attn + f"{p}_proj", s) for p, s in (("q", (2 * nq, H)), ("k", (nkv, H)), ("v", (nkv, H)),
                                                     ("o", (H, nq)))]
    linears += [(mlp + f"{p}_proj", s) for p, s in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I)))]
    gains = [(k, H) for k in ("norm", "pre_fc_norm_embedding", "pre_fc_norm_hidden", "layers.0.input_layernorm",
                              "layers.0.post_attention_layernorm")]
    gains += [(attn + "q_norm", hd), (attn + "k_norm", hd)]
    rng = np.random.default_rng(seed)
    out = {}
    for group, std in ((linears, 0.02), (gains, 0.1)):
        for key, shape in group:
            out[f"mtp.{key}.weight"] = rng.normal(0.0, std, shape).astype(F32)
    return out


def head_rows(vocab: int) -> int:
    """Rows of one block when the vocabulary is cut into the fewest equal blocks of at most 65535
    rows, each a multiple of 16: the largest such divisor."""
    fits = [r for r in range(16, min(vocab, 65535) + 1, 16) if vocab % r == 0]
    if not fits:
        raise ValueError(f"vocabulary {vocab}: no block split")
    return fits[-1]


def input_embedding(cfg, rows: np.ndarray) -> np.ndarray:
    """Gemma 3 / 4 scale embedding rows by fp32(sqrt(hidden)), one fp32 rounding (llm.py:198-204)."""
    out = np.asarray(rows, F32)
    if getattr(cfg, "model_type", "") in ("gemma3_text", "gemma4_text"):
        out = np.multiply(out, F32(np.sqrt(cfg.hidden_size)), dtype=F32)
    return out


def ple_embedding(cfg, rows: np.ndarray) -> np.ndarray:
    """Gemma 4's per-layer token embedding rows [n, L * ple_dim] times fp32(sqrt(ple_dim))
    (llm.py:207-211)."""
    rows = np.asarray(rows, F32)
    return (rows * F32(cfg.hidden_size_per_layer_input ** 0.5)).astype(F32)


@dataclass
class QWeight:
    q: np.ndarray            # int8 [N, K]
    scale: np.ndarray        # fp32 [N] or [1]
    n: int
    k: int


def quantize_weight(w: np.ndarray, per_channel: bool = True) -> QWeight:
    """Symmetric int8 weights (compiler.py:50-57): scale = absmax / 127 per output row (or one for
    the whole matrix), 1 where the absmax is 0; q = round half to even of w / scale, clipped to
    +-127; all in float64, the scales stored as fp32."""
    w64 = np.asarray(w, np.float64)
    amax = np.abs(w64).max(axis=1, keepdims=True)
    if not per_channel:
        amax = amax.max(keepdims=True)
    scale = amax / 127.0
    scale[amax == 0] = 1.0
    q = np.rint(w64 / scale).clip(-127, 127).astype(np.int8)
    return QWeight(q=q, scale=scale.reshape(-1).astype(np.float32), n=w64.shape[0], k=w64.shape[1])


@dataclass
class QWeight4:
    q: np.ndarray            # uint8 [N, K / 2], low nibble = even k
    scale: np.ndarray        # uint16 [N, K / 128], binary16 bits
    n: int
    k: int


def quantize_weight4(w: np.ndarray) -> QWeight4:
    w = np.asarray(w, dtype=np.float64)
    if w.ndim != 2 or w.shape[1] == 0 or w.shape[1] % W4_GROUP:
        raise ValueError("W4A16 weights need [N, K], K a nonzero multiple of 128")
    n, k = w.shape
    groups = w.reshape(n, k // W4_GROUP, W4_GROUP)
    amax = np.abs(groups).max(axis=2)
    sb = np.where(amax > 0, amax / 7.0, 1.0).astype(np.float32).astype(np.float16)
    s = sb.astype(np.float32).astype(np.float64)
    q = np.clip(np.rint(groups / s[:, :, None]), -7, 7).astype(np.int16)
    packed = ((q[:, :, 0::2] & 15) | ((q[:, :, 1::2] & 15) << 4)).astype(np.uint8)
    return QWeight4(packed.reshape(n, k // 2), sb.view(np.uint16), n, k)
