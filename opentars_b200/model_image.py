"""A text model as one DDR image plus per-chunk descriptor queues (Qwen3, Gemma 3 / 4, Qwen3.5).

    mi = ModelImage(cfg, weights, max_tokens=256, head=True, queue_cap=4096)
    ids, logits, counts = mi.generate(run, prompt, n_new)     # run(ddr, q, n) -> ddr

This is the caller above the drop-in boundary: it produces the images and queues that the golden
executor (and so libtarscuda's Machine, board backend and engine) runs. The image and the queues it
records are byte-identical to those of the reference's lowering for the same configuration and
weights (tars_mini/llm.py:213-836; pinned by tests/golden/models.json, full_models.json, mtp.json,
context.json): the same tensors in the same order on the contract's 128-byte boundaries, the same
descriptors in the same order.

Design: the weights of a layer are placed by interpreting a per-family layout table (FIELD_TABLES)
- entry order is placement order, each entry names its source parameter and how it is stored
(int8 per-row linear or group-128 int4, the same in K blocks, a norm gain, a derived constant);
the state (residual rows, KV caches, DeltaNet conv inputs and states, the logits) is placed by
place_state(); a chunk is recorded by block recorders that draw their temporaries from a scratch
region reset per layer.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import contract as C
from .models import head_rows, input_embedding, ple_embedding, quantize_weight, quantize_weight4
from .program import Buf, Image, Linear

F32 = np.float32
K_BLOCK = 4096                   # the executor's longest GEMM K: wider linears run as equal K blocks


def pad16(n: int) -> int:
    return (n + 15) // 16 * 16


# ------------------------------------------------------------------------------ model dimensions
@dataclass
class Dims:
    family: str                  # "qwen3", "gemma3", "gemma4", "qwen35"
    H: int
    I: int
    nh: int
    nkv: int
    hd: int                      # head dim (Gemma 4: of sliding layers)
    ghd: int                     # Gemma 4: head dim of full layers
    rot: int
    qmul: float                  # the attention scaling folded into q_norm
    eps: float
    types: list
    T: int
    Tp: int
    nk: int = 0                  # Qwen3.5 DeltaNet: key / value heads and head dims
    nv: int = 0
    dk: int = 0
    dv: int = 0
    taps: int = 4
    ple_dim: int = 0             # Gemma 4 per-layer inputs
    first_shared: int = 0        # Gemma 4: layers from here reuse an earlier layer's KV cache
    softcap: float | None = None

    @property
    def zero_centred(self) -> bool:
        """Norm weights stored as offsets from 1 (Gemma 3, Qwen3.5)."""
        return self.family in ("gemma3", "qwen35")

    def head_dim_of(self, layer_type: str) -> int:
        return self.ghd if (self.family == "gemma4" and layer_type == "full_attention") else self.hd


FAMILY = {"qwen3": "qwen3", "gemma3_text": "gemma3", "gemma4_text": "gemma4", "qwen3_5_text": "qwen35"}


def dims_of(cfg, max_tokens: int) -> Dims:
    fam = FAMILY.get(getattr(cfg, "model_type", ""))
    if fam is None:
        raise ValueError(f"model type {getattr(cfg, 'model_type', '')!r}: Qwen3, Gemma 3 / 4 and Qwen3.5 text only")
    types = list(cfg.layer_types)
    if fam in ("gemma3", "gemma4"):
        if not set(types) <= {"sliding_attention", "full_attention"}:
            raise ValueError("Gemma layers are sliding or full attention")
        if max_tokens > cfg.sliding_window:
            raise ValueError("the context must fit the sliding window")
        if cfg.hidden_activation != "gelu_pytorch_tanh" or getattr(cfg, "attn_logit_softcapping", None) is not None:
            raise ValueError("Gemma: tanh GELU and no attention softcapping")
    if fam == "gemma3" and cfg.final_logit_softcapping is not None:
        raise ValueError("Gemma 3 without a logit softcap")
    if fam == "gemma4" and (getattr(cfg, "enable_moe_block", False) or getattr(cfg, "attention_k_eq_v", False)
                            or getattr(cfg, "num_global_key_value_heads", None) not in (None, cfg.num_key_value_heads)):
        raise ValueError("Gemma 4 without MoE blocks, K = V or distinct global kv heads")
    if fam == "qwen3" and set(types) != {"full_attention"}:
        raise ValueError("Qwen3 layers are full attention")
    if fam == "qwen35" and not set(types) <= {"linear_attention", "full_attention"}:
        raise ValueError("Qwen3.5 layers are linear or full attention")
    hd = ghd = cfg.head_dim
    if fam == "gemma4":
        per = getattr(cfg, "per_layer_config", None)
        want = [per[i].head_dim if per else (getattr(cfg, "global_head_dim", None) or cfg.head_dim)
                if t == "full_attention" else cfg.head_dim for i, t in enumerate(types)]
        by = {}
        for t, d in zip(types, want):
            if by.setdefault(t, d) != d:
                raise ValueError("one head dim per Gemma 4 layer type")
        if per and any(p.num_key_value_heads != cfg.num_key_value_heads for p in per):
            raise ValueError("one kv head count")
        hd = by.get("sliding_attention", by.get("full_attention"))
        ghd = by.get("full_attention", hd)
    if fam in ("gemma3", "gemma4"):
        rot = hd
    else:
        rot = int(hd * cfg.rope_parameters.get("partial_rotary_factor", 1.0))
    qmul = 1.0 if fam == "gemma4" else (cfg.query_pre_attn_scalar ** -0.5 if fam == "gemma3" else hd ** -0.5)
    d = Dims(fam, cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.num_key_value_heads, hd, ghd,
             rot, qmul, cfg.rms_norm_eps, types, max_tokens, pad16(max_tokens))
    if fam == "qwen35":
        d.nk, d.nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        d.dk, d.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        d.taps = getattr(cfg, "linear_conv_kernel_dim", 4)
        if d.nk != d.nv:
            raise ValueError("the DeltaNet GQA repeat is not lowered")
    if fam == "gemma4":
        d.ple_dim = getattr(cfg, "hidden_size_per_layer_input", 0) or 0
        d.first_shared = len(types) - getattr(cfg, "num_kv_shared_layers", 0)
        d.softcap = getattr(cfg, "final_logit_softcapping", None)
    else:
        d.first_shared = len(types)
    return d


# ------------------------------------------------------------------------------ weight layout tables
# An entry: (key, kind, source, option). Kinds: "lin" an int8 / int4 linear (option: the name of a
# bias parameter), "kblocks" a linear in equal K blocks, "gain" a norm weight (option: "q" folds
# the attention scaling in), "ones" a fp32 vector of ones of the head dim, "table" a derived fp32
# constant (source: a function of the parameters), "no" an absent entry. Sources name parameters
# under the layer's prefix; callables derive arrays from (parameters, prefix, dims).
def _q_half(which: int):
    """Qwen3.5 full attention: q_proj holds, per head, the query's rows then the gate's."""
    def pick(W, pre, d):
        qp = W[pre + "self_attn.q_proj.weight"].reshape(d.nh, 2, d.hd, d.H)
        return qp[:, which].reshape(-1, d.H)
    return pick


def _qkv_rows(part: int):
    """Qwen3.5 DeltaNet: in_proj_qkv's q, k, v row blocks."""
    def pick(W, pre, d):
        kd = d.nk * d.dk
        rows = W[pre + "linear_attn.in_proj_qkv.weight"]
        return rows[(0, kd, 2 * kd)[part]:(kd, 2 * kd, None)[part]]
    return pick


FIELD_TABLES = {
    "qwen3": [("q", "lin", "self_attn.q_proj", None), ("g", "no", None, None),
              ("ln_in", "gain", "input_layernorm", None), ("ln_post", "gain", "post_attention_layernorm", None),
              ("k", "lin", "self_attn.k_proj", None), ("v", "lin", "self_attn.v_proj", None),
              ("qn", "gain", "self_attn.q_norm", "q"), ("kn", "gain", "self_attn.k_norm", None),
              ("o", "lin", "self_attn.o_proj", None), ("gate", "lin", "mlp.gate_proj", None),
              ("up", "lin", "mlp.up_proj", None), ("down", "lin", "mlp.down_proj", None)],
    "qwen35_full": [("q", "lin", _q_half(0), None), ("g", "lin", _q_half(1), None),
                    ("ln_in", "gain", "input_layernorm", None), ("ln_post", "gain", "post_attention_layernorm", None),
                    ("k", "lin", "self_attn.k_proj", None), ("v", "lin", "self_attn.v_proj", None),
                    ("qn", "gain", "self_attn.q_norm", "q"), ("kn", "gain", "self_attn.k_norm", None),
                    ("o", "lin", "self_attn.o_proj", None), ("gate", "lin", "mlp.gate_proj", None),
                    ("up", "lin", "mlp.up_proj", None), ("down", "lin", "mlp.down_proj", None)],
    "gemma3": [("ln_in", "gain", "input_layernorm", None), ("attn_norm", "gain", "post_attention_layernorm", None),
               ("ln_post", "gain", "pre_feedforward_layernorm", None),
               ("mlp_norm", "gain", "post_feedforward_layernorm", None),
               ("q", "lin", "self_attn.q_proj", None), ("g", "no", None, None),
               ("k", "lin", "self_attn.k_proj", None), ("v", "lin", "self_attn.v_proj", None),
               ("qn", "gain", "self_attn.q_norm", "q"), ("kn", "gain", "self_attn.k_norm", None),
               ("o", "lin", "self_attn.o_proj", None), ("gate", "lin", "mlp.gate_proj", None),
               ("up", "lin", "mlp.up_proj", None), ("down", "kblocks", "mlp.down_proj", None)],
    # Gemma 4; on KV-shared layers k, v, kn and vn are absent (see _place_layer)
    "gemma4": [("ln_in", "gain", "input_layernorm", None), ("attn_norm", "gain", "post_attention_layernorm", None),
               ("ln_post", "gain", "pre_feedforward_layernorm", None),
               ("mlp_norm", "gain", "post_feedforward_layernorm", None),
               ("q", "lin", "self_attn.q_proj", None), ("g", "no", None, None),
               ("k", "lin", "self_attn.k_proj", None), ("v", "lin", "self_attn.v_proj", None),
               ("qn", "gain", "self_attn.q_norm", "q"), ("kn", "gain", "self_attn.k_norm", None),
               ("vn", "ones", None, None),
               ("o", "kblocks", "self_attn.o_proj", None), ("gate", "lin", "mlp.gate_proj", None),
               ("up", "lin", "mlp.up_proj", None), ("down", "kblocks", "mlp.down_proj", None),
               ("layer_scalar", "table", lambda W, pre, d: W[pre + "layer_scalar"], None)],
    "gemma4_ple": [("ple_gate", "lin", "per_layer_input_gate", None), ("ple_proj", "lin", "per_layer_projection", None),
                   ("ple_norm", "gain", "post_per_layer_input_norm", None)],
    "qwen35_delta": [("ln_in", "gain", "input_layernorm", None), ("ln_post", "gain", "post_attention_layernorm", None),
                     ("q", "lin", _qkv_rows(0), None), ("k", "lin", _qkv_rows(1), None),
                     ("v", "lin", _qkv_rows(2), None), ("z", "lin", "linear_attn.in_proj_z", None),
                     ("b", "lin", "linear_attn.in_proj_b", None),
                     ("a", "lin", "linear_attn.in_proj_a", "linear_attn.dt_bias"),
                     ("negA", "table", lambda W, pre, d: -np.exp(W[pre + "linear_attn.A_log"].astype(F32)), None),
                     ("out", "lin", "linear_attn.out_proj", None),
                     ("gnorm", "table", lambda W, pre, d: W[pre + "linear_attn.norm.weight"], None),
                     ("qscale", "table", lambda W, pre, d: np.full(d.dk, F32(d.dk ** -0.5)), None),
                     ("kscale", "table", lambda W, pre, d: np.ones(d.dk, F32), None),
                     ("gate", "lin", "mlp.gate_proj", None), ("up", "lin", "mlp.up_proj", None),
                     ("down", "lin", "mlp.down_proj", None)],
}


# ------------------------------------------------------------------------------ the model image
class ModelImage:
    """A Qwen3 / Gemma 3 / Gemma 4 / Qwen3.5 text model laid out in one image, and the recording of
    its chunks. wbits 8: every linear W8A8 (ROW_QUANT, then QM_ROWCOL); 4: W4A16 (QM_GROUP on fp32
    rows). state_dtype fp16: the DeltaNet states in fp16. mtp: Qwen3.5's MTP head (two DeltaNet
    state copies, the MTP layer's own KV cache)."""

    def __init__(self, cfg, weights: dict, max_tokens: int, ddr_bytes: int = 1 << 27, head: bool = False,
                 queue_cap: int = 0, scratch_bytes: int = 1 << 22, verify_rows: int = 1, keep_layers: bool = True,
                 wbits: int = 8, state_dtype: str = "fp32", mtp: bool = False):
        if wbits not in (4, 8):
            raise ValueError("wbits: 8 (W8A8) or 4 (W4A16)")
        if state_dtype not in ("fp32", "fp16"):
            raise ValueError("state_dtype: fp32 or fp16")
        self.cfg, self.w = cfg, weights
        self.d = d = dims_of(cfg, max_tokens)
        self.wbits, self.keep_layers, self.verify_rows, self.mtp = wbits, keep_layers, verify_rows, mtp
        self.state_fmt = C.OUT_FP16 if state_dtype == "fp16" else C.OUT_FP32
        self.head = head
        self.vocab = weights["embed_tokens.weight"].shape[0] if head else 0
        self.parity, self.spec = 0, False
        self.p = Image(ddr_bytes)
        self._place_state()
        self.queue_cap = queue_cap
        self.qbase = self.p.reserve(64 * queue_cap) if queue_cap else None
        self.scratch0 = self.p.top
        self.scratch_end = self.p.reserve(scratch_bytes) + scratch_bytes
        self._place_weights()
        self.end = self.p.top

    # the dimensions under the names callers use
    T = property(lambda s: s.d.T)
    H = property(lambda s: s.d.H)
    eps = property(lambda s: s.d.eps)
    types = property(lambda s: s.d.types)
    nh = property(lambda s: s.d.nh)
    nkv = property(lambda s: s.d.nkv)
    hd = property(lambda s: s.d.hd)
    rot = property(lambda s: s.d.rot)
    ple_dim = property(lambda s: s.d.ple_dim)
    gemma = property(lambda s: s.d.family == "gemma3")
    gemma4 = property(lambda s: s.d.family == "gemma4")

    # -------------------------------------------------------------- placement: state
    def _place_state(self) -> None:
        d, p = self.d, self.p
        L = len(d.types)
        if self.keep_layers:
            self.xs = [p.matrix(d.T, d.H) for _ in range(L + 1)]
        else:                                    # the input rows, then two alternating layer outputs
            first, even, odd = p.matrix(d.T, d.H), p.matrix(d.T, d.H), p.matrix(d.T, d.H)
            self.xs = [first] + [even if i % 2 == 0 else odd for i in range(L)]
        self.x0 = self.xs[0]
        self.ple0 = self.ple = None
        if d.ple_dim:
            self.ple0 = p.matrix(d.T, L * d.ple_dim)          # the host's per-layer token rows
            self.ple = p.matrix(d.T, L * d.ple_dim)           # after the projection
        self.y = p.matrix(d.T, d.H)
        hist = d.taps - 1
        self.st, newest = [], {}
        for i, t in enumerate(d.types):
            if t == "linear_attention":
                kd, vd = d.nk * d.dk, d.nv * d.dv
                cin = {name: p.matrix(d.T + hist, width) for name, width in (("q", kd), ("k", kd), ("v", vd))}
                copies = [[p.matrix(d.dk, d.dv, self.state_fmt) for _ in range(d.nv)]
                          for _ in range(2 if self.mtp else 1)]
                self.st.append(dict(cin=cin, S=copies))
            elif i < d.first_shared:
                width = d.nkv * d.head_dim_of(t)
                kv = dict(kc=p.matrix(d.Tp, width), vc=p.matrix(d.Tp, width))
                newest[t] = kv
                self.st.append(kv)
            else:
                self.st.append(newest[t])
        if self.mtp:
            self.mst = dict(kc=p.matrix(d.Tp, d.nkv * d.hd), vc=p.matrix(d.Tp, d.nkv * d.hd))
        self.logits = p.matrix(self.verify_rows, self.vocab) if self.head else None

    # -------------------------------------------------------------- placement: weights
    def _linear(self, w, bias=None) -> Linear:
        b_off = self.p.store(np.asarray(bias, F32)) if bias is not None else None
        if self.wbits == 4:
            q4 = quantize_weight4(w)
            return Linear(self.p.store(q4.q, "u1"), self.p.store(q4.scale, "<u2"), b_off, q4.n, q4.k, 4)
        q8 = quantize_weight(np.asarray(w, np.float64), per_channel=True)
        if q8.n % 16 or q8.k % 16:
            raise ValueError("W8A8 linears need N and K multiples of 16")
        return Linear(self.p.store(q8.q, "i1"), self.p.store(q8.scale), b_off, q8.n, q8.k)

    def _k_blocks(self, w, parts: int = 0) -> list[Linear]:
        """Equal K blocks of one weight: W8 blocks share one per-row scale vector (placed first),
        W4 blocks have their own group scales."""
        if self.wbits == 4:
            q4 = quantize_weight4(w)
            parts = parts or -(-q4.k // K_BLOCK)
            kb = q4.k // parts
            if kb * parts != q4.k or kb % C.W4_GROUP:
                raise ValueError("K blocks of whole 128-groups")
            out = []
            for c in range(0, q4.k, kb):
                w_off = self.p.store(np.ascontiguousarray(q4.q[:, c // 2:(c + kb) // 2]), "u1")
                s_off = self.p.store(np.ascontiguousarray(q4.scale[:, c // C.W4_GROUP:(c + kb) // C.W4_GROUP]), "<u2")
                out.append(Linear(w_off, s_off, None, q4.n, kb, 4))
            return out
        q8 = quantize_weight(np.asarray(w, np.float64), per_channel=True)
        parts = parts or -(-q8.k // K_BLOCK)
        kb = q8.k // parts
        if kb * parts != q8.k or kb % 16 or q8.n % 16:
            raise ValueError("K blocks of multiples of 16")
        s_off = self.p.store(q8.scale)
        return [Linear(self.p.store(np.ascontiguousarray(q8.q[:, c:c + kb]), "i1"), s_off, None, q8.n, kb)
                for c in range(0, q8.k, kb)]

    def _gain(self, w, scale: float = 1.0) -> Buf:
        """A norm weight as the kernels apply it: fp32(1 + w) for zero-centred families, times the
        folded scaling."""
        g = np.asarray(w, F32)
        if self.d.zero_centred:
            g = (F32(1.0) + g).astype(F32)
        return self.p.constant((g * F32(scale)).astype(F32))

    def _place_table(self, table, pre: str, skip=()) -> dict:
        W, d, out = self.w, self.d, {}
        for key, kind, src, opt in table:
            if kind == "no" or key in skip:
                out[key] = None
                continue
            arr = src(W, pre, d) if callable(src) else None
            if kind == "lin":
                out[key] = self._linear(arr if arr is not None else W[pre + src + ".weight"],
                                        W[pre + opt] if opt else None)
            elif kind == "kblocks":
                out[key] = self._k_blocks(W[pre + src + ".weight"])
            elif kind == "gain":
                out[key] = self._gain(W[pre + src + ".weight"], d.qmul if opt == "q" else 1.0)
            elif kind == "ones":
                out[key] = self.p.constant(np.ones(self._lhd, F32))
            else:
                out[key] = self.p.constant(arr)
        return out

    def _place_layer(self, pre: str, i: int | None) -> dict:
        d = self.d
        t = d.types[i] if i is not None else "full_attention"
        if t == "linear_attention":
            lw = self._place_table(FIELD_TABLES["qwen35_delta"], pre)
            taps = self.w[pre + "linear_attn.conv1d.weight"][:, 0, :]          # [channels, taps]
            d.taps = taps.shape[1]
            kd, vd = d.nk * d.dk, d.nv * d.dv
            lw["conv"] = {name: [self.p.constant(taps[lo:lo + width, j]) for j in range(d.taps)]
                          for name, lo, width in (("q", 0, kd), ("k", kd, kd), ("v", 2 * kd, vd))}
            return lw
        if d.family == "gemma4":
            shared = i >= d.first_shared
            self._lhd = d.head_dim_of(t)
            lw = self._place_table(FIELD_TABLES["gemma4"], pre, skip=("k", "v", "kn", "vn") if shared else ())
            lw.update(hd=self._lhd, rot=self._lhd, rope=t, kv_shared=shared)
            if d.ple_dim:
                lw.update(self._place_table(FIELD_TABLES["gemma4_ple"], pre))
            return lw
        fam = {"qwen3": "qwen3", "gemma3": "gemma3", "qwen35": "qwen35_full"}[d.family]
        lw = self._place_table(FIELD_TABLES[fam], pre)
        if d.family == "gemma3":
            lw["rope"] = t
        return lw

    def _rope_rows(self, theta: float, width: int, angles: int | None = None) -> Buf:
        """Rows t = cos(t w), sin(t w) (fp32, as torch computes them) for the first `angles` of the
        width / 2 inverse frequencies; the rest stay 0 (proportional RoPE)."""
        d = self.d
        th = F32(theta)
        inv = np.zeros(width // 2, F32)
        n = width // 2 if angles is None else angles
        inv[:n] = (1.0 / (th ** (np.arange(0, 2 * n, 2, dtype=F32) / F32(width)))).astype(F32)
        ang = (np.arange(d.T, dtype=F32)[:, None] * inv[None, :]).astype(F32)
        return self.p.constant(np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(F32))

    def _place_weights(self) -> None:
        d, p, W = self.d, self.p, self.w
        d.taps = 4
        self.lw = [self._place_layer(f"layers.{i}.", i) for i in range(len(d.types))]
        if d.ple_dim:
            self.ple_w = dict(model_proj=self._linear(W["per_layer_model_projection.weight"]),
                              proj_scale=p.constant(np.array([F32(d.H ** -0.5)], F32)),
                              proj_norm=self._gain(W["per_layer_projection_norm.weight"]),
                              in_scale=p.constant(np.array([F32(2.0 ** -0.5)], F32)))
        self.final_norm = self._gain(W["norm.weight"])
        if self.mtp:
            mw = self._place_layer("mtp.layers.0.", None)
            mw.update(fc=self._linear(W["mtp.fc.weight"]), ge=self._gain(W["mtp.pre_fc_norm_embedding.weight"]),
                      gh=self._gain(W["mtp.pre_fc_norm_hidden.weight"]), norm=self._gain(W["mtp.norm.weight"]))
            self.mw = mw
        if d.family == "gemma4":
            self.rope_tabs = {}
            for t in sorted(set(d.types)):
                rp = self.cfg.rope_parameters[t]
                kind = rp.get("rope_type", "default")
                if kind not in ("default", "proportional"):
                    raise ValueError(f"RoPE type {kind!r}")
                width = d.head_dim_of(t)
                frac = rp.get("partial_rotary_factor", 1.0) if kind == "proportional" else 1.0
                self.rope_tabs[t] = self._rope_rows(rp["rope_theta"], width, int(frac * width // 2))
        elif d.family == "gemma3":
            self.rope_tabs = {t: self._rope_rows(self.cfg.rope_parameters[t]["rope_theta"], d.rot)
                              for t in sorted(set(d.types))}
        else:
            self.rope_tab = self._rope_rows(self.cfg.rope_parameters["rope_theta"], d.rot)
        if d.softcap is not None:
            cap = float(d.softcap)
            self.sc_inv2, self.sc_two, self.sc_val = (p.constant(np.array([F32(v)], F32))
                                                      for v in (2.0 / cap, 2.0 * cap, cap))
        self.head_lins = []
        if self.head:
            e = W["embed_tokens.weight"]
            rows = head_rows(e.shape[0])
            self.head_lins = [self._linear(e[r:r + rows]) for r in range(0, e.shape[0], rows)]

    # -------------------------------------------------------------- host-side rows
    def embed(self, ids) -> np.ndarray:
        return input_embedding(self.cfg, self.w["embed_tokens.weight"][np.asarray(ids)])

    def embed_ple(self, ids) -> np.ndarray:
        """Gemma 4's per-layer token rows [len(ids), L * ple_dim] (the host's lookup)."""
        return ple_embedding(self.cfg, self.w["embed_tokens_per_layer.weight"][np.asarray(ids)])

    def put_input(self, ddr, t0: int, x: np.ndarray, ple: np.ndarray | None = None) -> None:
        for buf, rows in ((self.x0, x), (self.ple0, ple)):
            if rows is None:
                continue
            at = self.p.base + buf.off + t0 * buf.ld
            ddr[at:at + rows.size * 4] = np.asarray(rows, F32).tobytes()

    def input(self, x: np.ndarray, t0: int = 0, ple: np.ndarray | None = None) -> None:
        self.put_input(self.p.ddr, t0, x, ple)

    # -------------------------------------------------------------- recording helpers
    def _proj(self, x: Buf, w: Linear, y: Buf, act: int = C.ACT_NONE, q=None) -> None:
        """One linear: W4A16 straight on x; W8A8 on x's int8 rows (q, quantised here when None)."""
        if self.wbits == 4:
            self.p.mm4(x, w, y, act)
            return
        xq, srow = self.p.quantize(x) if q is None else q
        self.p.mm8(xq, srow, w, y, act)

    def _proj_blocks(self, x: Buf, blocks, q, out: Buf) -> None:
        """A linear in K blocks: each block on its columns of x, partial results added in order."""
        blocks = blocks if isinstance(blocks, list) else [blocks]
        c0 = 0
        for i, blk in enumerate(blocks):
            dst = out if i == 0 else self.p.matrix(x.rows, self.d.H)
            xi = x.cols_at(c0, blk.k)
            self._proj(xi, blk, dst, q=None if q is None else (q[0].cols_at(c0, blk.k), q[1]))
            if i:
                self.p.elt(C.ELT_ADD, out, dst, out)
            c0 += blk.k

    def _q8(self, x: Buf):
        return self.p.quantize(x) if self.wbits == 8 else None

    # -------------------------------------------------------------- blocks
    def _feedforward(self, lw: dict, x: Buf, out: Buf) -> None:
        d, p, n = self.d, self.p, x.rows
        h = p.matrix(n, d.H)
        p.rms_norm(x, lw["ln_post"], d.eps, h)
        hq = self._q8(h)
        gate, up = p.matrix(n, lw["gate"].n), p.matrix(n, lw["up"].n)
        self._proj(h, lw["gate"], gate, C.ACT_GELU if d.family in ("gemma3", "gemma4") else C.ACT_SILU, q=hq)
        self._proj(h, lw["up"], up, q=hq)
        p.elt(C.ELT_MUL, gate, up, gate)
        mq = self._q8(gate)
        res = p.matrix(n, d.H)
        self._proj_blocks(gate, lw["down"], mq, res)
        if lw.get("mlp_norm") is not None:
            normed = p.matrix(n, d.H)
            p.rms_norm(res, lw["mlp_norm"], d.eps, normed)
            res = normed
        p.elt(C.ELT_ADD, x, res, out)

    def _attention(self, lw: dict, st: dict, x: Buf, out: Buf, t0: int, n: int, li: int | None = None) -> None:
        """A full-attention layer (llm.py:705-782) for tokens t0 .. t0 + n - 1."""
        d, p = self.d, self.p
        hd, rot = lw.get("hd", d.hd), lw.get("rot", d.rot)
        nh, nkv = d.nh, d.nkv
        kc, vc = st["kc"], st["vc"]
        h = p.matrix(n, d.H)
        p.rms_norm(x, lw["ln_in"], d.eps, h)
        hq = self._q8(h)
        q = p.matrix(n, nh * hd)
        self._proj(h, lw["q"], q, q=hq)
        gate = None
        if lw["g"] is not None:                        # Qwen3.5's attention output gate
            gate = p.matrix(n, nh * hd)
            self._proj(h, lw["g"], gate, q=hq)
        qn = p.matrix(n, nh * hd)
        p.rms_norm(q.as_heads(hd), lw["qn"], d.eps, qn.as_heads(hd))
        qr = p.matrix(n, nh * hd)
        tab = (self.rope_tabs[lw["rope"]] if "rope" in lw else self.rope_tab).rows_at(t0, n)
        p.rotary(qn.as_heads(hd), tab, nh, rot, qr.as_heads(hd))
        if not lw.get("kv_shared", False):
            k = p.matrix(n, nkv * hd)
            self._proj(h, lw["k"], k, q=hq)
            vrows = vc.rows_at(t0, n)
            if lw.get("vn") is not None:               # Gemma 4: V through an unscaled RMSNorm
                v = p.matrix(n, nkv * hd)
                self._proj(h, lw["v"], v, q=hq)
                p.rms_norm(v.as_heads(hd), lw["vn"], d.eps, vrows.as_heads(hd))
            else:
                self._proj(h, lw["v"], vrows, q=hq)
            kn = p.matrix(n, nkv * hd)
            p.rms_norm(k.as_heads(hd), lw["kn"], d.eps, kn.as_heads(hd))
            p.rotary(kn.as_heads(hd), tab, nkv, rot, kc.rows_at(t0, n).as_heads(hd))
        keys = pad16(t0 + n)
        att = p.matrix(n, nh * hd)
        scores, probs = p.matrix(n, keys), p.matrix(n, keys)
        group = nh // nkv
        for head in range(nh):
            kvh = head // group
            p.fdot(qr.column_of(head, hd), kc.column_of(kvh, hd)._replace(rows=keys), scores, nn=False)
            p.row_op(C.ROW_SOFTMAX, scores, probs, start=t0 + 1)
            p.fdot(probs, vc.column_of(kvh, hd)._replace(rows=keys), att.column_of(head, hd), nn=True)
        if gate is not None:
            gated = p.matrix(n, nh * hd)
            p.elt(C.ELT_MUL, gate, att, gated, act=C.ACT_SIGMOID)
            att = gated
        aq = self._q8(att)
        o = p.matrix(n, d.H)
        self._proj_blocks(att, lw["o"], aq, o)
        if lw.get("attn_norm") is not None:
            normed = p.matrix(n, d.H)
            p.rms_norm(o, lw["attn_norm"], d.eps, normed)
            o = normed
        x1 = p.matrix(n, d.H)
        p.elt(C.ELT_ADD, x, o, x1)
        ple = "ple_gate" in lw
        x2 = p.matrix(n, d.H) if ple else out
        self._feedforward(lw, x1, x2)
        if ple:                                        # Gemma 4: the layer's per-layer input, gated
            P = d.ple_dim
            pg = p.matrix(n, P)
            self._proj(x2, lw["ple_gate"], pg, C.ACT_GELU)
            p.elt(C.ELT_MUL, pg, self.ple.rows_at(t0, n).cols_at(li * P, P), pg)
            pp = p.matrix(n, d.H)
            self._proj(pg, lw["ple_proj"], pp)
            ppn = p.matrix(n, d.H)
            p.rms_norm(pp, lw["ple_norm"], d.eps, ppn)
            p.elt(C.ELT_ADD, x2, ppn, out)
        if lw.get("layer_scalar") is not None:
            p.elt(C.ELT_MUL, out, lw["layer_scalar"], out, bmode=C.BM_SCALAR)

    def _delta(self, li: int, t0: int, n: int) -> None:
        """A gated DeltaNet layer (llm.py:642-700): the causal conv over the last taps rows, the
        state recurrence token by token and head by head, the gated RMSNorm, out_proj, the MLP."""
        d, p, lw, st = self.d, self.p, self.lw[li], self.st[li]
        kd, vd, hist = d.nk * d.dk, d.nv * d.dv, d.taps - 1
        x = self.xs[li].rows_at(t0, n)
        h = p.matrix(n, d.H)
        p.rms_norm(x, lw["ln_in"], d.eps, h)
        hq = self._q8(h)
        for name in ("q", "k", "v"):
            self._proj(h, lw[name], st["cin"][name].rows_at(hist + t0, n), q=hq)
        z = p.matrix(n, vd)
        self._proj(h, lw["z"], z, q=hq)
        beta, soft = p.matrix(n, d.nv), p.matrix(n, d.nv)
        self._proj(h, lw["b"], beta, C.ACT_SIGMOID, q=hq)
        self._proj(h, lw["a"], soft, C.ACT_SOFTPLUS, q=hq)
        gexp = p.matrix(n, d.nv)
        p.elt(C.ELT_MUL, soft, lw["negA"], gexp, bmode=C.BM_ROW)
        decay = p.matrix(n, d.nv)
        p.activation(gexp, C.ACT_EXP, decay)
        conv = {}
        for name, width in (("q", kd), ("k", kd), ("v", vd)):
            src, acc = st["cin"][name], p.matrix(n, width)
            taps = lw["conv"][name]
            p.elt(C.ELT_MUL, src.rows_at(t0, n), taps[0], acc, bmode=C.BM_ROW)
            for j in range(1, d.taps):
                p.elt(C.ELT_MULADD, src.rows_at(t0 + j, n), taps[j], acc, bmode=C.BM_ROW, c=acc)
            act = p.matrix(n, width)
            p.activation(acc, C.ACT_SILU, act)
            conv[name] = act
        qn, kn = p.matrix(n, kd), p.matrix(n, kd)
        p.rms_norm(conv["q"].as_heads(d.dk), lw["qscale"], 1e-6, qn.as_heads(d.dk), l2=True)
        p.rms_norm(conv["k"].as_heads(d.dk), lw["kscale"], 1e-6, kn.as_heads(d.dk), l2=True)
        qh, kh, vh = qn.as_heads(d.dk), kn.as_heads(d.dk), conv["v"].as_heads(d.dv)
        o = p.matrix(n, vd)
        oh = o.as_heads(d.dv)
        kvmem, delta = p.matrix(1, d.dv), p.matrix(1, d.dv)
        for t in range(n):
            last = self.spec and t == n - 1
            for hh in range(d.nv):
                r = t * d.nv + hh
                s_in = st["S"][self.parity][hh]
                s_out = st["S"][1 - self.parity][hh] if last else s_in
                p.elt(C.ELT_MUL, s_in, decay.rows_at(t, 1).cols_at(hh, 1), s_out, bmode=C.BM_SCALAR)
                p.fdot(kh.rows_at(r, 1), s_out, kvmem, nn=True)
                p.elt(C.ELT_SUB, vh.rows_at(r, 1), kvmem, delta)
                p.elt(C.ELT_MUL, delta, beta.rows_at(t, 1).cols_at(hh, 1), delta, bmode=C.BM_SCALAR)
                p.elt(C.ELT_MULADD, delta, kh.rows_at(r, 1), s_out, bmode=C.BM_COL, arow=True, c=s_out)
                p.fdot(qh.rows_at(r, 1), s_out, oh.rows_at(r, 1), nn=True)
        on, og = p.matrix(n, vd), p.matrix(n, vd)
        p.rms_norm(oh, lw["gnorm"], d.eps, on.as_heads(d.dv))
        p.elt(C.ELT_MUL, z, on, og, act=C.ACT_SILU)
        a = p.matrix(n, d.H)
        self._proj(og, lw["out"], a)
        x1 = p.matrix(n, d.H)
        p.elt(C.ELT_ADD, x, a, x1)
        self._feedforward(lw, x1, self.xs[li + 1].rows_at(t0, n))

    def _per_layer_inputs(self, t0: int, n: int) -> None:
        """Gemma 4: the rows' per-layer projection times H^-0.5, RMSNorm per layer block, plus the
        host's per-layer token rows, times 2^-0.5."""
        d, p, pw = self.d, self.p, self.ple_w
        width = len(d.types) * d.ple_dim
        proj = p.matrix(n, width)
        self._proj(self.x0.rows_at(t0, n), pw["model_proj"], proj)
        p.elt(C.ELT_MUL, proj, pw["proj_scale"], proj, bmode=C.BM_SCALAR)
        normed = p.matrix(n, width)
        p.rms_norm(proj.as_heads(d.ple_dim), pw["proj_norm"], d.eps, normed.as_heads(d.ple_dim))
        dst = self.ple.rows_at(t0, n)
        p.elt(C.ELT_ADD, normed, self.ple0.rows_at(t0, n), dst)
        p.elt(C.ELT_MUL, dst, pw["in_scale"], dst, bmode=C.BM_SCALAR)

    def _logits_of(self, y: Buf) -> None:
        """The tied head in row blocks; each block's rows written densely, block after block."""
        p, r, c0 = self.p, y.rows, 0
        yq = self._q8(y)
        for blk in self.head_lins:
            dst = Buf(self.logits.off + 4 * c0 * r, r, blk.n, 4 * blk.n)
            self._proj(y, blk, dst, q=yq)
            if self.d.softcap is not None:             # cap tanh(x / cap) = 2 cap sigmoid(2 x / cap) - cap
                p.elt(C.ELT_MUL, dst, self.sc_inv2, dst, bmode=C.BM_SCALAR)
                p.elt(C.ELT_MUL, dst, self.sc_two, dst, bmode=C.BM_SCALAR, act=C.ACT_SIGMOID)
                p.elt(C.ELT_SUB, dst, self.sc_val, dst, bmode=C.BM_SCALAR)
            c0 += blk.n

    def _scratch(self) -> None:
        if self.p.top > self.scratch_end:
            raise MemoryError("scratch_bytes too small for this chunk")
        self.p.top = self.scratch0

    # -------------------------------------------------------------- chunks
    def chunk(self, t0: int, n: int, all_rows: bool = False, parity: int = 0, spec: bool = False) -> None:
        """Records tokens t0 .. t0 + n - 1 through every layer, the final norm and (head) the last
        row's logits (all_rows: every row's, for a speculative verify). parity selects the DeltaNet
        state copy; spec: the last token updates the other copy, so a rejected draft leaves this one
        as it was after token n - 2."""
        if all_rows and n > self.verify_rows:
            raise ValueError("all_rows needs n <= verify_rows")
        self.parity, self.spec = parity, spec
        d, p = self.d, self.p
        p.top = self.scratch0
        if d.ple_dim:
            self._per_layer_inputs(t0, n)
            self._scratch()
        for i, t in enumerate(d.types):
            p.top = self.scratch0
            if t == "linear_attention":
                self._delta(i, t0, n)
            else:
                self._attention(self.lw[i], self.st[i], self.xs[i].rows_at(t0, n), self.xs[i + 1].rows_at(t0, n),
                                t0, n, i)
            self._scratch()
        p.rms_norm(self.xs[-1].rows_at(t0, n), self.final_norm, d.eps, self.y.rows_at(t0, n))
        if self.head:
            r = n if all_rows else 1
            self._logits_of(self.y.rows_at(t0 + n - r, r))
        if p.top > self.scratch_end:
            raise MemoryError("scratch_bytes too small for this chunk")
        p.top = self.end

    def swap_state(self) -> None:
        """The second DeltaNet state copy into the first (ELT MUL by an exact 1.0), so that plain
        queues (parity 0) can follow a speculative run."""
        for st, lw in zip(self.st, self.lw):
            if "S" in st:
                one = lw["kscale"]._replace(rows=1, cols=1, ld=4)
                for src, dst in zip(st["S"][1], st["S"][0]):
                    self.p.elt(C.ELT_MUL, src, one, dst, bmode=C.BM_SCALAR)

    def mtp_chunk(self, r0: int, n: int, head: bool = True) -> None:
        """MTP rows r0 .. r0 + n - 1 (row r: the embedding of token r + 1 with the hidden state of
        position r, predicting token r + 2): fc over the two norms, one gated attention layer with
        its own KV cache, the norm and (head) the last row's logits."""
        d, p, mw = self.d, self.p, self.mw
        p.top = self.scratch0
        cat = p.matrix(n, 2 * d.H)
        p.rms_norm(self.x0.rows_at(r0 + 1, n), mw["ge"], d.eps, cat.cols_at(0, d.H))
        p.rms_norm(self.y.rows_at(r0, n), mw["gh"], d.eps, cat.cols_at(d.H, d.H))
        x, out = p.matrix(n, d.H), p.matrix(n, d.H)
        self._proj(cat, mw["fc"], x)
        self._attention(mw, self.mst, x, out, r0, n)
        if head:
            y = p.matrix(1, d.H)
            p.rms_norm(out.rows_at(n - 1, 1), mw["norm"], d.eps, y)
            self._logits_of(y)
        if p.top > self.scratch_end:
            raise MemoryError("scratch_bytes too small for this chunk")
        p.top = self.end

    # -------------------------------------------------------------- running chunk by chunk
    def stage(self, ddr, a: int, b: int) -> tuple[int, int]:
        """Descriptors [a, b) into the queue region; returns (queue address, count)."""
        if self.qbase is None or b - a > self.queue_cap:
            raise ValueError("the queue region is too small")
        at = self.p.base + self.qbase
        ddr[at:at + 64 * (b - a)] = b"".join(bytes(x) for x in self.p.descs[a:b])
        return at, b - a

    def logits_of(self, ddr) -> np.ndarray:
        at = self.p.base + self.logits.off
        return np.frombuffer(bytes(ddr[at:at + 4 * self.vocab]), "<f4").copy()

    def logits_rows(self, ddr, n: int) -> np.ndarray:
        """n rows of logits, reassembled from the head's block-major layout."""
        at = self.p.base + self.logits.off
        flat = np.frombuffer(bytes(ddr[at:at + 4 * self.vocab * n]), "<f4")
        out, c0 = np.empty((n, self.vocab), F32), 0
        for blk in self.head_lins:
            out[:, c0:c0 + blk.n] = flat[c0 * n:(c0 + blk.n) * n].reshape(n, blk.n)
            c0 += blk.n
        return out

    def _run(self, run, ddr, record):
        a = len(self.p.descs)
        record()
        q, cnt = self.stage(ddr, a, len(self.p.descs))
        out = run(ddr, q, cnt)
        return (out if isinstance(out, bytearray) else bytearray(out)), cnt

    def generate(self, run, prompt, n_new: int, chunk: int = 0):
        """Greedy decoding with the host in the loop: run(ddr, q, n) -> ddr runs one chunk's queue.
        chunk > 0 feeds the prompt in chunks of that many tokens (the board runtime's prefill), 0
        as one chunk. Returns (ids, logits per run from the prompt's last chunk on, descriptors per
        run)."""
        if not self.head:
            raise ValueError("generate needs the head")
        P = len(prompt)
        spans = [(s, min(chunk, P - s)) for s in range(0, P, chunk)] if chunk else [(0, P)]
        ddr, ids, logits, counts = self.p.ddr, list(prompt), [], []
        for i in range(len(spans) + n_new):
            t0, n = spans[i] if i < len(spans) else (len(ids) - 1, 1)
            toks = ids[t0:t0 + n]
            self.put_input(ddr, t0, self.embed(toks), self.embed_ple(toks) if self.ple_dim else None)
            ddr, cnt = self._run(run, ddr, lambda: self.chunk(t0, n))
            if i >= len(spans) - 1:
                lg = self.logits_of(ddr)
                logits.append(lg)
                counts.append(cnt)
                ids.append(int(np.argmax(lg)))
        return ids, logits, counts

    def generate_mtp(self, run, prompt, n_new: int, oracle=None):
        """Greedy speculative decoding with the MTP head; the tokens equal generate()'s. A round
        verifies [current token, draft] as two rows: a hit emits both rows' picks and flips the
        state copy, a miss emits the correction; the MTP layer then takes the rows the verify
        made known and drafts again. oracle(t, draft) may replace a draft (tests). Returns (ids,
        {position: its logits}, rounds)."""
        if not (self.head and self.mtp and self.verify_rows >= 2):
            raise ValueError("generate_mtp needs the head, the MTP weights and verify_rows >= 2")
        box = [self.p.ddr]

        def go(record) -> None:
            box[0], _ = self._run(run, box[0], record)

        def feed(t: int, toks) -> None:
            self.put_input(box[0], t, self.embed(toks))
        ids, P, parity, rounds = list(prompt), len(prompt), 0, 0
        feed(0, ids)
        go(lambda: self.chunk(0, P))
        seen = {P - 1: self.logits_of(box[0])}
        ids.append(int(np.argmax(seen[P - 1])))
        feed(P, ids[P:])
        go(lambda: self.mtp_chunk(0, P))
        t = P                                          # ids[t] is known, not yet in the caches
        while len(ids) < P + n_new + 1:
            draft = int(np.argmax(self.logits_of(box[0])))
            if oracle is not None:
                draft = oracle(t, draft)
            feed(t + 1, [draft])
            go(lambda: self.chunk(t, 2, all_rows=True, parity=parity, spec=True))
            both = self.logits_rows(box[0], 2)
            rounds += 1
            seen[t] = both[0]
            pick = int(np.argmax(both[0]))
            ids.append(pick)
            if pick == draft:
                seen[t + 1] = both[1]
                ids.append(int(np.argmax(both[1])))
                parity ^= 1
                feed(t + 2, ids[t + 2:t + 3])
                go(lambda: self.mtp_chunk(t, 2))
                t += 2
            else:
                feed(t + 1, [pick])
                go(lambda: self.mtp_chunk(t, 1))
                t += 1
        return ids, seen, rounds
