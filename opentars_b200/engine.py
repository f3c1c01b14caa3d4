"""Batched greedy decoding on one B200 (include/tarscuda_engine.h), fed from a ModelImage.

    low = ModelImage(cfg, weights, max_tokens=256, head=True)
    eng = DecodeEngine(low, batch=64)
    ids, logits = eng.generate(prompts, n_new, chunk=4)     # prompts: [batch][len] token ids

The engine reads the weights from the model's DDR image (uploaded once to HBM) and runs every
sequence's step on the GPU, B sequences at a time; per sequence the tokens and logits equal the
descriptor path's (the reference golden model's) bit for bit. The host only moves token ids, and
the logits when asked for.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import contract as C
from ._lib import lib as _machine_lib

F32 = np.float32


class Lin_t(ctypes.Structure):
    _fields_ = [("w_off", ctypes.c_uint64), ("s_off", ctypes.c_uint64), ("n", ctypes.c_int32), ("k", ctypes.c_int32)]


class Layer_t(ctypes.Structure):
    _fields_ = [("ln_in", ctypes.c_uint64), ("ln_post", ctypes.c_uint64), ("attn_norm", ctypes.c_uint64),
                ("mlp_norm", ctypes.c_uint64), ("qn", ctypes.c_uint64), ("kn", ctypes.c_uint64),
                ("rope_tab", ctypes.c_uint64), ("q", Lin_t), ("k", Lin_t), ("v", Lin_t), ("o", Lin_t),
                ("gate", Lin_t), ("up", Lin_t), ("down", Lin_t * 4), ("n_down", ctypes.c_int32)]


class Model_t(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("rot", ctypes.c_int32), ("vocab", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
                ("act", ctypes.c_int32), ("gemma", ctypes.c_int32), ("eps", ctypes.c_float),
                ("embed_scale", ctypes.c_float), ("final_norm", ctypes.c_uint64), ("n_head_blocks", ctypes.c_int32),
                ("head", Lin_t * 8)]


P = ctypes.c_void_p
ENGINE_SIGNATURES = {
    "tc_engine_create": (ctypes.c_int, [P, ctypes.POINTER(Model_t), ctypes.POINTER(Layer_t), P, ctypes.c_int32,
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "tc_engine_destroy": (ctypes.c_int, [P]),
    "tc_engine_error": (ctypes.c_char_p, [P]),
    "tc_engine_stream": (ctypes.c_void_p, [P]),
    "tc_engine_reset": (ctypes.c_int, [P]),
    "tc_engine_step": (ctypes.c_int, [P, P, ctypes.c_int32]),
    "tc_engine_tokens": (ctypes.c_int, [P, P]),
    "tc_engine_set_tokens": (ctypes.c_int, [P, P]),
    "tc_engine_logits": (ctypes.c_int, [P, P]),
    "tc_engine_sync": (ctypes.c_int, [P]),
    "tc_engine_profile": (ctypes.c_int, [P, P, P, P, ctypes.c_uint32]),
    "tc_argmax": (ctypes.c_int, [P, ctypes.c_int32, ctypes.c_int32, P, P]),
    "tc_engine_reset_seq": (ctypes.c_int, [P, ctypes.c_int32]),
    "tc_engine_positions": (ctypes.c_int, [P, P]),
    "tc_engine_fused": (ctypes.c_int, [P, ctypes.c_int32]),
    "tc_engine_fused_why": (ctypes.c_char_p, [P]),
    "tc_engine_fused_diag": (ctypes.c_int, [P, P]),
    "tc_engine_phase_times": (ctypes.c_int, [P, P, ctypes.c_uint32]),
}
# the fused step's phases, in the order of tc_engine_phase_times' stamps (per layer, then the tail)
LAYER_PHASES = ("norm_quant", "gemm_qkv", "attention", "gemm_o", "norm_quant", "gemm_gate_up", "gated_quant",
                "gemm_down")
TAIL_PHASES = ("norm_quant", "gemm_head", "empty", "empty", "empty", "empty")
KERNEL_KINDS = ("embed", "norm_quant", "gemv", "qk_rope", "attention", "quant", "argmax", "advance")


def lib():
    L = _machine_lib()
    if not getattr(L, "_engine_bound", False):
        for name, (res, args) in ENGINE_SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        L._engine_bound = True
    return L


def _lin(q) -> Lin_t:
    return Lin_t(q.w_off, q.s_off, q.n, q.k)


def model_desc(low) -> tuple[Model_t, ctypes.Array]:
    """The engine's description of a lowered model: shapes and the image offsets of every tensor."""
    if low.wbits != 8 or low.p.base != 0:
        raise ValueError("the decode engine runs W8A8 images laid out at base 0")
    cfg = low.cfg
    L = len(low.types)
    layers = (Layer_t * L)()
    for i, w in enumerate(low.lw):
        ld = layers[i]
        ld.ln_in, ld.ln_post = w["ln_in"].off, w["ln_post"].off
        ld.attn_norm = w["attn_norm"].off if w.get("attn_norm") is not None else 0
        ld.mlp_norm = w["mlp_norm"].off if w.get("mlp_norm") is not None else 0
        ld.qn, ld.kn = w["qn"].off, w["kn"].off
        ld.rope_tab = (low.rope_tabs[w["rope"]] if "rope" in w else low.rope_tab).off
        for name in ("q", "k", "v", "o", "gate", "up"):
            lin = w[name][0] if isinstance(w[name], list) else w[name]
            setattr(ld, name, _lin(lin))
        downs = w["down"] if isinstance(w["down"], list) else [w["down"]]
        if len(downs) > 2 or (isinstance(w["o"], list) and len(w["o"]) > 1):
            raise ValueError("the engine takes down in at most two K blocks and o unsplit")
        for j, lin in enumerate(downs):
            ld.down[j] = _lin(lin)
        ld.n_down = len(downs)
    md = Model_t()
    md.n_layers, md.hidden, md.inter = L, low.H, cfg.intermediate_size
    md.n_heads, md.n_kv, md.head_dim, md.rot = low.nh, low.nkv, low.hd, low.rot
    md.vocab, md.max_tokens = low.vocab, low.T
    md.act = C.ACT_GELU if low.gemma else C.ACT_SILU
    md.gemma = int(low.gemma)
    md.eps = F32(low.eps)
    md.embed_scale = F32(cfg.hidden_size ** 0.5) if low.gemma else F32(1.0)
    md.final_norm = low.final_norm.off
    if len(low.head_lins) > 8:
        raise ValueError("at most 8 head blocks")
    md.n_head_blocks = len(low.head_lins)
    for j, lin in enumerate(low.head_lins):
        md.head[j] = _lin(lin)
    return md, layers


class DecodeEngine:
    def __init__(self, low, batch: int, device: int | None = None):
        from ._lib import check
        from .machine import default_device
        if not low.head:
            raise ValueError("the model image needs its head (head=True)")
        self.low, self.B = low, int(batch)
        self.device = default_device() if device is None else device
        L = lib()
        img = ctypes.c_void_p()                                   # the weights: the model's image in HBM
        n = len(low.p.ddr)
        if L.tc_open(self.device, n, ctypes.byref(img)) != 0:
            raise RuntimeError(f"cannot open a {n}-byte image on CUDA device {self.device}")
        self.img = img
        check(L.tc_upload(img, 0, (ctypes.c_char * n).from_buffer(low.p.ddr), n), img, "upload")
        md, layers = model_desc(low)
        self._md, self._layers = md, layers
        emb = np.ascontiguousarray(low.w["embed_tokens.weight"], dtype=F32)
        h = ctypes.c_void_p()
        rc = L.tc_engine_create(img, ctypes.byref(md), layers, emb.ctypes.data_as(ctypes.c_void_p), self.B,
                                ctypes.byref(h))
        if rc != 0:
            raise RuntimeError(f"tc_engine_create failed ({rc})")
        self.h = h
        self.vocab = low.vocab
        self._tok = np.zeros(self.B, np.int32)

    def _check(self, rc: int, what: str):
        if rc != 0:
            raise RuntimeError(f"{what}: {lib().tc_engine_error(self.h).decode()}")

    def reset(self):
        self._check(lib().tc_engine_reset(self.h), "reset")

    def step(self, tokens: np.ndarray | None, n: int = 1):
        """One chunk: tokens [B, n] ids from the host, or None to feed the previous greedy picks."""
        L = lib()
        if tokens is None:
            self._check(L.tc_engine_step(self.h, None, 1), "step")
            return
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.B, n))
        self._check(L.tc_engine_step(self.h, t.ctypes.data_as(ctypes.c_void_p), n), "step")
        self._keep = t                                            # alive until the copy has run

    def tokens(self) -> np.ndarray:
        self._check(lib().tc_engine_tokens(self.h, self._tok.ctypes.data_as(ctypes.c_void_p)), "tokens")
        return self._tok.copy()

    def set_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.B))
        self._keep = t
        self._check(lib().tc_engine_set_tokens(self.h, t.ctypes.data_as(ctypes.c_void_p)), "set_tokens")

    def logits(self) -> np.ndarray:
        out = np.empty((self.B, self.vocab), F32)
        self._check(lib().tc_engine_logits(self.h, out.ctypes.data_as(ctypes.c_void_p)), "logits")
        return out

    def sync(self):
        self._check(lib().tc_engine_sync(self.h), "sync")

    def reset_seq(self, b: int) -> None:
        """Start sequence b afresh (zeroed KV cache rows, position 0); the others keep theirs."""
        self._check(lib().tc_engine_reset_seq(self.h, int(b)), "reset_seq")

    def positions(self) -> np.ndarray:
        out = np.zeros(self.B, np.int32)
        self._check(lib().tc_engine_positions(self.h, out.ctypes.data_as(ctypes.c_void_p)), "positions")
        return out

    def fused(self, enable: bool | None = None) -> bool:
        """Whether one-token steps run as the fused step kernel (and switch it when enable is given)."""
        rc = lib().tc_engine_fused(self.h, -1 if enable is None else int(bool(enable)))
        if rc < 0:
            raise RuntimeError(f"the fused step is not available: {self.fused_why()}")
        return bool(rc)

    def fused_why(self) -> str:
        return lib().tc_engine_fused_why(self.h).decode()

    def fused_diag(self) -> list[int]:
        out = np.zeros(4, np.int32)
        self._check(lib().tc_engine_fused_diag(self.h, out.ctypes.data_as(ctypes.c_void_p)), "fused_diag")
        return [int(v) for v in out]

    def phase_times(self) -> list[tuple[str, int, float, float, float]]:
        """One fused decode step phase by phase: [(phase, layer (-1: the tail), microseconds from
        the previous barrier to the next, of which until the last CTA arrived at it, and of which
        the barrier itself)]. The tail ends with four empty phases: the barrier alone."""
        L = len(self.low.types)
        nph = 8 * L + 6
        cap = 1024 + (9 * L + 8) * 1024
        st = np.zeros(cap, np.uint64)
        n = lib().tc_engine_phase_times(self.h, st.ctypes.data_as(ctypes.c_void_p), cap)
        if n < 0:
            self._check(n, "phase_times")
        grid = (n - 1024) // (9 * L + 8)
        ex = st[:1024].astype(np.int64)
        arr = st[1024:1024 + grid * (nph + 1)].astype(np.int64).reshape(nph + 1, grid)
        names = [(p, li) for li in range(L) for p in LAYER_PHASES] + [(p, -1) for p in TAIL_PHASES]
        out = []
        for i in range(1, nph + 1):
            last = int(arr[i].max())
            out.append((names[i - 1][0], names[i - 1][1], (ex[i] - ex[i - 1]) / 1e3, (last - ex[i - 1]) / 1e3,
                        (ex[i] - last) / 1e3))
        return out

    def profile(self) -> list[tuple[str, float, int]]:
        """One decode step kernel by kernel: [(kind, ms, algorithmic bytes)]."""
        cap = 4096
        ms = np.zeros(cap, np.float32)
        kind = np.zeros(cap, np.int32)
        nb = np.zeros(cap, np.uint64)
        n = lib().tc_engine_profile(self.h, ms.ctypes.data_as(ctypes.c_void_p), kind.ctypes.data_as(ctypes.c_void_p),
                                    nb.ctypes.data_as(ctypes.c_void_p), cap)
        if n < 0:
            self._check(n, "profile")
        return [(KERNEL_KINDS[kind[i]], float(ms[i]), int(nb[i])) for i in range(n)]

    def generate(self, prompts, n_new: int, chunk: int = 4, keep_logits: bool = True):
        """Greedy decoding of B prompts of equal length: prefill in chunks of `chunk` tokens, then
        n_new single-token steps. Returns (ids [B][len + n_new + 1], logits per step [B][vocab])."""
        prompts = np.asarray(prompts, np.int32).reshape(self.B, -1)
        P = prompts.shape[1]
        self.reset()
        ids = [list(map(int, p)) for p in prompts]
        logits = []
        s = 0
        while s < P:
            n = min(chunk, P - s)
            self.step(prompts[:, s:s + n], n)
            s += n
        for i in range(n_new + 1):
            if i:
                self.step(None)
            if keep_logits:
                logits.append(self.logits())
            nxt = self.tokens()
            for b in range(self.B):
                ids[b].append(int(nxt[b]))
        return ids, logits

    def close(self):
        if getattr(self, "h", None):
            lib().tc_engine_destroy(self.h)
            self.h = None
        if getattr(self, "img", None):
            lib().tc_close(self.img)
            self.img = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
