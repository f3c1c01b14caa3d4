"""The step driver: Qwen3 / Gemma 3 / Gemma 4 / Qwen3.5 text models lowered to tars_mini v0.4
descriptors.

Restates, for the families on the hot path, the reference's program builder and LLM lowering so
that the same DDR image and the same descriptor queues come out byte for byte (pinned by the
committed fixtures):
  * Program (alloc / _put / _emit / build)       tars_mini/compiler.py:134-155, 186-188, 384-391
  * V, Dev emitters (rowop, norm, quant, gemm_rc, gemm_w4, fdot, elt, act, rope)  tars_mini/llm.py:34-178
  * QwenLowering: weights, state, chunk, _la (Qwen3.5's gated DeltaNet layers), _fa_block (with
    Qwen3.5's attention output gate), _mlp, _head, stage, put_input, logits_of, logits_rows,
    generate                                                                  llm.py:213-836
Every linear is W8A8 (ROW_QUANT then GEMM QM_ROWCOL) or W4A16; Gemma 3's down projection runs as
equal K blocks (llm.py:303-321) whose fp32 partials are added by ELT ADD in block order. The
DeltaNet state may be fp16 (state_dtype, the STATE_FP16 ELT / FDOT forms). Qwen3.5's MTP head
(mtp=True: mtp_chunk, two DeltaNet state copies, swap_state, generate_mtp; llm.py:573-612,
838-886) drafts one token per round for greedy speculative decoding. Gemma 4 (per-type head dims,
proportional RoPE, KV sharing, V norm, per-layer embeddings, layer_scalar, the softcapped head)
follows llm.py's gemma4 paths.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from . import contract as C
from .models import head_rows, input_embedding, ple_embedding, quantize_weight, quantize_weight4

F32 = np.float32
ALIGN = 128
GEMV_K = 4096


def pad16(n: int) -> int:
    return -(-n // 16) * 16


@dataclass
class V:
    """A matrix in the image: offset from the program base, shape, row stride in bytes, format."""
    off: int
    rows: int
    cols: int
    ld: int
    fmt: int = C.OUT_FP32

    def rowv(self, r0: int, n: int) -> "V":
        return replace(self, off=self.off + r0 * self.ld, rows=n)

    def colv(self, c0: int, n: int) -> "V":
        return replace(self, off=self.off + c0 * C.ESIZE[self.fmt], cols=n)

    def heads(self, hd: int) -> "V":
        assert self.ld == self.cols * C.ESIZE[self.fmt] and self.cols % hd == 0
        return V(self.off, self.rows * self.cols // hd, hd, hd * C.ESIZE[self.fmt], self.fmt)


@dataclass
class QLin:
    w_off: int
    s_off: int
    b_off: int | None
    n: int
    k: int
    wbits: int = 8


def _ld16(ld: int, rowbytes: int) -> int:
    if ld == rowbytes:
        return 0
    assert ld % 16 == 0 and ld > rowbytes
    return ld // 16


class Program:
    """A DDR image being laid out (bump allocator, 128-byte aligned; offset 0 kept unused) and the
    descriptors emitted against it."""

    def __init__(self, ddr_bytes: int = 1 << 24, base_addr: int = 0):
        self.base = base_addr
        self.ddr = bytearray(base_addr + ddr_bytes)
        self.top = ALIGN
        self.descs: list[bytes] = []
        self.queue_off: int | None = None

    def alloc(self, nbytes: int) -> int:
        off = self.top
        self.top = -(-(off + nbytes) // ALIGN) * ALIGN
        if self.base + self.top > len(self.ddr):
            raise MemoryError(f"program needs {self.top} bytes of DDR, has {len(self.ddr)}")
        return off

    def _put(self, arr: np.ndarray, dtype: str) -> int:
        data = np.ascontiguousarray(arr).astype(dtype).tobytes()
        off = self.alloc(len(data))
        self.ddr[self.base + off:self.base + off + len(data)] = data
        return off

    def _emit(self, **f) -> None:
        self.descs.append(C.encode({"MAGIC": C.MAGIC, "VERSION": C.VERSION, "VALID": 1, "BASE_ADDR": self.base, **f}))

    def build(self) -> tuple[bytearray, int, int]:
        if self.queue_off is None:
            self.queue_off = self.alloc(C.DESC_BYTES * len(self.descs))
            for i, r in enumerate(self.descs):
                a = self.base + self.queue_off + 64 * i
                self.ddr[a:a + 64] = r
        return self.ddr, self.base + self.queue_off, len(self.descs)


class Dev(Program):
    """Descriptor emitters on V views (offsets relative to the program base)."""

    def mat(self, rows: int, cols: int, fmt: int = C.OUT_FP32) -> V:
        es = C.ESIZE[fmt]
        return V(self.alloc(rows * cols * es), rows, cols, cols * es, fmt)

    def put(self, a: np.ndarray, dt: str = "<f4") -> int:
        return self._put(np.asarray(a), dt)

    def const(self, a: np.ndarray) -> V:
        a = np.asarray(a, F32).reshape(1, -1) if np.ndim(a) < 2 else np.asarray(a, F32)
        return V(self.put(a), a.shape[0], a.shape[1], 4 * a.shape[1])

    def rowop(self, x: V, fn: int, y: V, gamma: V | None = None, eps: float = 0.0, start: int = 0,
              scale_out: int = 0, beta: V | None = None) -> None:
        assert x.cols == y.cols and x.rows == y.rows and x.fmt == C.OUT_FP32 and y.fmt != C.OUT_FP16
        self._emit(OPCODE=C.OP_ROW, CTRL=fn, EPI=C.epi(C.ACT_NONE, y.fmt, int(beta is not None)),
                   A_OFF=x.off, Y_OFF=y.off, M=x.rows, N=x.cols, K=start,
                   SCALE_OFF=gamma.off if gamma is not None else scale_out,
                   BIAS_OFF=beta.off if beta is not None else 0,
                   W_OFF=C.f32_bits(eps) if gamma is not None else 0,
                   LDA16=_ld16(x.ld, 4 * x.cols), LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))

    def norm(self, x: V, gamma: V, eps: float, y: V, l2: bool = False) -> None:
        self.rowop(x, C.ROW_L2NORM if l2 else C.ROW_RMSNORM, y, gamma, eps)

    def quant(self, x: V, q: V | None = None, s: int | None = None) -> tuple[V, int]:
        q = self.mat(x.rows, x.cols, C.OUT_INT8) if q is None else q
        s = self.alloc(4 * x.rows) if s is None else s
        self.rowop(x, C.ROW_QUANT, q, scale_out=s)
        return q, s

    def softmax_causal(self, x: V, y: V, first_valid: int) -> None:
        self.rowop(x, C.ROW_SOFTMAX, y, start=first_valid)

    def gemm_rc(self, xq: V, srow: int, w: QLin, y: V, act: int = C.ACT_NONE) -> None:
        assert xq.fmt == C.OUT_INT8 and xq.cols == w.k and y.cols == w.n and srow % 16 == 0 and y.fmt != C.OUT_FP16
        self._emit(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_ROWCOL, fusion=int(act != C.ACT_NONE)),
                   EPI=C.epi(act, y.fmt, int(w.b_off is not None)), A_OFF=xq.off, W_OFF=w.w_off,
                   SCALE_OFF=w.s_off, BIAS_OFF=w.b_off or 0, Y_OFF=y.off, M=xq.rows, N=w.n, K=w.k,
                   HDR_RSV=srow // 16, LDA16=_ld16(xq.ld, xq.cols), LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))

    def gemm_w4(self, x: V, w: QLin, y: V, act: int = C.ACT_NONE) -> None:
        assert x.fmt in (C.OUT_FP32, C.OUT_BF16) and x.cols == w.k and y.cols == w.n
        assert w.wbits == 4 and w.k >= 256 and w.k % 256 == 0 and w.w_off % 128 == 0 and y.fmt != C.OUT_FP16
        adt = C.DT_FP32 if x.fmt == C.OUT_FP32 else C.DT_BF16
        self._emit(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_GROUP, a_dtype=adt, w_dtype=C.DT_INT4,
                                                 fusion=int(act != C.ACT_NONE)),
                   EPI=C.epi(act, y.fmt, int(w.b_off is not None)), A_OFF=x.off, W_OFF=w.w_off,
                   SCALE_OFF=w.s_off, BIAS_OFF=w.b_off or 0, Y_OFF=y.off, M=x.rows, N=w.n, K=w.k,
                   GROUP_SIZE=C.W4_GROUP, LDA16=_ld16(x.ld, C.ESIZE[x.fmt] * x.cols),
                   LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))

    def fdot(self, a: V, b: V, y: V, nn: bool) -> None:
        K = a.cols
        N = b.cols if nn else b.rows
        assert (b.rows if nn else b.cols) == K and y.cols == N and y.rows == a.rows
        brow = C.ESIZE[b.fmt] * b.cols
        self._emit(OPCODE=C.OP_FDOT, CTRL=int(nn), EPI=C.epi(C.ACT_NONE, y.fmt), A_OFF=a.off, W_OFF=b.off,
                   Y_OFF=y.off, M=a.rows, N=N, K=K, GROUP_SIZE=_ld16(b.ld, brow),
                   HDR_RSV=C.STATE_FP16 if b.fmt == C.OUT_FP16 else 0,
                   LDA16=_ld16(a.ld, 4 * a.cols), LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))

    def elt(self, op: int, a: V, b: V, y: V, bmode: int = C.BM_DENSE, arow: bool = False,
            act: int = C.ACT_NONE, c: V | None = None) -> None:
        M, N = y.rows, y.cols
        g = _ld16(b.ld, 4 * N) if bmode == C.BM_DENSE else 0
        self._emit(OPCODE=C.OP_ELT, CTRL=op, EPI=C.epi(act, y.fmt, int(c is not None)),
                   A_OFF=a.off, W_OFF=b.off, Y_OFF=y.off, BIAS_OFF=c.off if c is not None else 0,
                   M=M, N=N, HDR_RSV=bmode | int(arow) << 2 | (C.STATE_FP16 if a.fmt == C.OUT_FP16 else 0),
                   GROUP_SIZE=g, LDA16=0 if arow else _ld16(a.ld, C.ESIZE[a.fmt] * N),
                   LDY16=_ld16(y.ld, N * C.ESIZE[y.fmt]))

    def act(self, x: V, act: int, y: V) -> None:
        """The activation op (OPCODE RELU with EPI.act): y = act(x)."""
        self._emit(OPCODE=C.OP_RELU, CTRL=0, EPI=C.epi(act, y.fmt), A_OFF=x.off, Y_OFF=y.off,
                   M=x.rows, N=x.cols, LDA16=_ld16(x.ld, 4 * x.cols),
                   LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))

    def rope(self, x: V, tab: V, rows_per_pos: int, rot: int, y: V) -> None:
        self._emit(OPCODE=C.OP_ROPE, CTRL=0, EPI=C.epi(C.ACT_NONE, y.fmt), A_OFF=x.off, W_OFF=tab.off,
                   Y_OFF=y.off, M=x.rows, N=x.cols, K=rot, GROUP_SIZE=rows_per_pos,
                   LDA16=_ld16(x.ld, 4 * x.cols), LDY16=_ld16(y.ld, y.cols * C.ESIZE[y.fmt]))


class QwenLowering:
    """A Qwen3 or Gemma 3 text model as data in one DDR image plus per-chunk descriptor queues.

        low = QwenLowering(cfg, weights, max_tokens=256, head=True, queue_cap=4096)
        ids, logits, counts = low.generate(run, prompt, n_new)     # run(ddr, q, n) -> ddr
    """

    def __init__(self, cfg, weights: dict[str, np.ndarray], max_tokens: int, ddr_bytes: int = 1 << 27,
                 head: bool = False, queue_cap: int = 0, scratch_bytes: int = 1 << 22, verify_rows: int = 1,
                 keep_layers: bool = True, wbits: int = 8, state_dtype: str = "fp32", mtp: bool = False):
        if wbits not in (4, 8):
            raise ValueError("wbits must be 4 (W4A16) or 8 (W8A8)")
        if state_dtype not in ("fp32", "fp16"):
            raise ValueError("state_dtype must be fp32 or fp16")
        mt = getattr(cfg, "model_type", "")
        if mt not in ("qwen3", "gemma3_text", "gemma4_text", "qwen3_5_text"):
            raise ValueError(f"model type {mt!r}: this lowering covers Qwen3, Gemma 3 / 4 and Qwen3.5 text")
        self.state_fmt = C.OUT_FP16 if state_dtype == "fp16" else C.OUT_FP32
        self.parity, self.spec = 0, False          # the DeltaNet state copy in use; a verify's last token
        self.mtp = mtp                             # Qwen3.5's MTP head (weights["mtp.*"])
        self.wbits, self.keep_layers = wbits, keep_layers
        self.cfg, self.w, self.T = cfg, weights, max_tokens
        self.verify_rows = verify_rows
        self.p = self.prog = Dev(ddr_bytes=ddr_bytes)
        self.H, self.eps = cfg.hidden_size, cfg.rms_norm_eps
        self.q3 = mt == "qwen3"
        self.gemma = mt == "gemma3_text"
        self.gemma4 = mt == "gemma4_text"
        self.types = list(cfg.layer_types)
        if self.gemma:
            assert set(self.types) <= {"sliding_attention", "full_attention"}
            assert cfg.attn_logit_softcapping is None and cfg.final_logit_softcapping is None
            assert cfg.hidden_activation == "gelu_pytorch_tanh"
            assert max_tokens <= cfg.sliding_window, "the context must fit the sliding window"
        elif self.gemma4:
            assert set(self.types) <= {"sliding_attention", "full_attention"}
            assert getattr(cfg, "attn_logit_softcapping", None) is None
            assert cfg.hidden_activation == "gelu_pytorch_tanh"
            assert not getattr(cfg, "enable_moe_block", False) and not getattr(cfg, "attention_k_eq_v", False)
            assert getattr(cfg, "num_global_key_value_heads", None) in (None, cfg.num_key_value_heads)
            assert max_tokens <= cfg.sliding_window, "the context must fit the sliding window"
        elif self.q3:
            assert set(self.types) == {"full_attention"}
        else:
            assert set(self.types) <= {"linear_attention", "full_attention"}
        # Qwen3.5's linear-attention (gated DeltaNet) dimensions
        self.nk, self.nv = getattr(cfg, "linear_num_key_heads", 0), getattr(cfg, "linear_num_value_heads", 0)
        self.dk, self.dv = getattr(cfg, "linear_key_head_dim", 0), getattr(cfg, "linear_value_head_dim", 0)
        assert self.nk == self.nv, "the GQA repeat of linear attention is not lowered"
        self.nh, self.nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        if self.gemma4:
            # head dims per layer type: a config's per-layer table where it has one, else head_dim for
            # sliding and global_head_dim for full layers (the model's own parameter shapes)
            plc = getattr(cfg, "per_layer_config", None)
            dims = [plc[i].head_dim if plc else (getattr(cfg, "global_head_dim", None) or cfg.head_dim)
                    if t == "full_attention" else cfg.head_dim for i, t in enumerate(self.types)]
            by_type = dict(zip(self.types, dims))
            assert all(by_type[t] == d for t, d in zip(self.types, dims))
            assert not plc or all(p.num_key_value_heads == self.nkv for p in plc)
            self.hd = by_type.get("sliding_attention", by_type["full_attention"])
            self.ghd = by_type.get("full_attention", self.hd)
        else:
            self.hd = self.ghd = cfg.head_dim
        self.ple_dim = (getattr(cfg, "hidden_size_per_layer_input", 0) or 0) if self.gemma4 else 0
        self.first_kv_shared = len(self.types) - (getattr(cfg, "num_kv_shared_layers", 0) if self.gemma4 else 0)
        self.softcap = getattr(cfg, "final_logit_softcapping", None) if self.gemma4 else None
        self.rot = self.hd if (self.gemma or self.gemma4) \
            else int(self.hd * cfg.rope_parameters.get("partial_rotary_factor", 1.0))
        # the attention scaling, folded into q_norm's gamma (Gemma 4: scaling 1.0)
        self.qmul = 1.0 if self.gemma4 else (cfg.query_pre_attn_scalar ** -0.5 if self.gemma else self.hd ** -0.5)
        self.Tp = pad16(max_tokens)
        self.head = head
        self.taps = getattr(cfg, "linear_conv_kernel_dim", 4)
        self.vocab = weights["embed_tokens.weight"].shape[0] if head else 0
        self._state()
        self.queue_cap = queue_cap
        self.qbase = self.p.alloc(64 * queue_cap) if queue_cap else None
        self.scratch0 = self.p.top
        self.scratch_end = self.p.alloc(scratch_bytes) + scratch_bytes
        self._weights()
        self.end = self.p.top

    # ------------------------------------------------------------------ weights (host side)
    def lin(self, w: np.ndarray, bias: np.ndarray | None = None) -> QLin:
        b = self.p.put(np.asarray(bias, F32)) if bias is not None else None
        if self.wbits == 4:
            qw = quantize_weight4(w)
            return QLin(self.p.put(qw.q, "u1"), self.p.put(qw.scale, "<u2"), b, qw.n, qw.k, 4)
        qw = quantize_weight(np.asarray(w, np.float64), per_channel=True)
        assert qw.n % 16 == 0 and qw.k % 16 == 0
        return QLin(self.p.put(qw.q, "i1"), self.p.put(qw.scale), b, qw.n, qw.k)

    def lin_k(self, w: np.ndarray, parts: int = 0) -> list[QLin]:
        """Equal K blocks sharing one per-channel scale (W8) or with their own group scales (W4)."""
        if self.wbits == 4:
            qw = quantize_weight4(w)
            parts = parts or -(-qw.k // GEMV_K)
            kb = qw.k // parts
            assert kb * parts == qw.k and kb % C.W4_GROUP == 0
            return [QLin(self.p.put(np.ascontiguousarray(qw.q[:, c // 2:(c + kb) // 2]), "u1"),
                         self.p.put(np.ascontiguousarray(qw.scale[:, c // C.W4_GROUP:(c + kb) // C.W4_GROUP]), "<u2"),
                         None, qw.n, kb, 4) for c in range(0, qw.k, kb)]
        qw = quantize_weight(np.asarray(w, np.float64), per_channel=True)
        parts = parts or -(-qw.k // GEMV_K)
        kb = qw.k // parts
        assert kb * parts == qw.k and kb % 16 == 0 and qw.n % 16 == 0
        s = self.p.put(qw.scale)
        return [QLin(self.p.put(np.ascontiguousarray(qw.q[:, c:c + kb]), "i1"), s, None, qw.n, kb)
                for c in range(0, qw.k, kb)]

    def _layer_hd(self, t: str) -> int:
        return self.ghd if (self.gemma4 and t == "full_attention") else self.hd

    def gamma1(self, w: np.ndarray, mul: float = 1.0) -> V:
        """Qwen3 / Gemma 4: the RMSNorm weight itself; Gemma 3 and Qwen3.5 (zero-centred weights):
        fp32(1 + w). Times `mul` (the attention scaling folded into q_norm)."""
        g = np.asarray(w, F32) if (self.q3 or self.gemma4) else (F32(1.0) + np.asarray(w, F32)).astype(F32)
        return self.p.const((g * F32(mul)).astype(F32))

    def linear(self, x: V, w: QLin, y: V, act: int = C.ACT_NONE, qs: tuple[V, int] | None = None) -> None:
        if self.wbits == 4:
            self.p.gemm_w4(x, w, y, act)
        else:
            xq, xs = self.p.quant(x) if qs is None else qs
            self.p.gemm_rc(xq, xs, w, y, act)

    def _la_weights(self, L: str) -> dict:
        """A gated DeltaNet layer: q / k / v as three linears (rows of in_proj_qkv), z, b, a (with
        dt_bias as the GEMM bias), -exp(A_log), the conv taps per channel block, the gated norm."""
        W, p = self.w, self.p
        la = L + "linear_attn."
        kd, vd = self.nk * self.dk, self.nv * self.dv
        qkv = W[la + "in_proj_qkv.weight"]
        d = dict(
            ln_in=self.gamma1(W[L + "input_layernorm.weight"]),
            ln_post=self.gamma1(W[L + "post_attention_layernorm.weight"]),
            q=self.lin(qkv[:kd]), k=self.lin(qkv[kd:2 * kd]), v=self.lin(qkv[2 * kd:]),
            z=self.lin(W[la + "in_proj_z.weight"]),
            b=self.lin(W[la + "in_proj_b.weight"]),
            a=self.lin(W[la + "in_proj_a.weight"], W[la + "dt_bias"]),
            negA=p.const(-np.exp(W[la + "A_log"].astype(F32))),
            out=self.lin(W[la + "out_proj.weight"]),
            gnorm=p.const(W[la + "norm.weight"]),
            qscale=p.const(np.full(self.dk, F32(self.dk ** -0.5))),
            kscale=p.const(np.ones(self.dk, F32)),
            gate=self.lin(W[L + "mlp.gate_proj.weight"]), up=self.lin(W[L + "mlp.up_proj.weight"]),
            down=self.lin(W[L + "mlp.down_proj.weight"]))
        cw = W[la + "conv1d.weight"][:, 0, :]                  # [channels, taps]
        self.taps = cw.shape[1]
        d["conv"] = {n: [p.const(cw[o:o + dd, j]) for j in range(self.taps)]
                     for n, o, dd in (("q", 0, kd), ("k", kd, kd), ("v", 2 * kd, vd))}
        return d

    def _fa_weights(self, A: str, li: int | None = None) -> dict:
        W = self.w
        sa = A + "self_attn."
        if self.gemma4:
            t = self.types[li]
            hd = self._layer_hd(t)
            shared = li >= self.first_kv_shared
            g1 = lambda n, mul=1.0: self.gamma1(W[A + n + ".weight"], mul)  # noqa: E731
            d = dict(
                hd=hd, rot=hd, rope=t, kv_shared=shared,
                ln_in=g1("input_layernorm"), attn_norm=g1("post_attention_layernorm"),
                ln_post=g1("pre_feedforward_layernorm"), mlp_norm=g1("post_feedforward_layernorm"),
                q=self.lin(W[sa + "q_proj.weight"]), g=None,
                k=None if shared else self.lin(W[sa + "k_proj.weight"]),
                v=None if shared else self.lin(W[sa + "v_proj.weight"]),
                qn=g1("self_attn.q_norm", self.qmul),
                kn=None if shared else g1("self_attn.k_norm"),
                vn=None if shared else self.p.const(np.ones(hd, F32)),       # V RMSNorm without scale
                o=self.lin_k(W[sa + "o_proj.weight"]),
                gate=self.lin(W[A + "mlp.gate_proj.weight"]), up=self.lin(W[A + "mlp.up_proj.weight"]),
                down=self.lin_k(W[A + "mlp.down_proj.weight"]),
                layer_scalar=self.p.const(W[A + "layer_scalar"]))
            if self.ple_dim:
                d.update(ple_gate=self.lin(W[A + "per_layer_input_gate.weight"]),
                         ple_proj=self.lin(W[A + "per_layer_projection.weight"]),
                         ple_norm=g1("post_per_layer_input_norm"))
            return d
        if self.gemma:
            g1 = lambda n, mul=1.0: self.gamma1(W[A + n + ".weight"], mul)  # noqa: E731
            return dict(
                ln_in=g1("input_layernorm"), attn_norm=g1("post_attention_layernorm"),
                ln_post=g1("pre_feedforward_layernorm"), mlp_norm=g1("post_feedforward_layernorm"),
                q=self.lin(W[sa + "q_proj.weight"]), g=None,
                k=self.lin(W[sa + "k_proj.weight"]), v=self.lin(W[sa + "v_proj.weight"]),
                qn=g1("self_attn.q_norm", self.qmul), kn=g1("self_attn.k_norm"),
                o=self.lin(W[sa + "o_proj.weight"]),
                gate=self.lin(W[A + "mlp.gate_proj.weight"]), up=self.lin(W[A + "mlp.up_proj.weight"]),
                down=self.lin_k(W[A + "mlp.down_proj.weight"]))
        if self.q3:                                            # no output gate
            q, g = self.lin(W[sa + "q_proj.weight"]), None
        else:                                                  # Qwen3.5, per head: the query's rows, then the gate's
            qp = W[sa + "q_proj.weight"].reshape(self.nh, 2, self.hd, self.H)
            q, g = self.lin(qp[:, 0].reshape(-1, self.H)), self.lin(qp[:, 1].reshape(-1, self.H))
        return dict(
            ln_in=self.gamma1(W[A + "input_layernorm.weight"]),
            ln_post=self.gamma1(W[A + "post_attention_layernorm.weight"]),
            q=q, g=g,
            k=self.lin(W[sa + "k_proj.weight"]), v=self.lin(W[sa + "v_proj.weight"]),
            qn=self.gamma1(W[sa + "q_norm.weight"], self.qmul), kn=self.gamma1(W[sa + "k_norm.weight"]),
            o=self.lin(W[sa + "o_proj.weight"]),
            gate=self.lin(W[A + "mlp.gate_proj.weight"]), up=self.lin(W[A + "mlp.up_proj.weight"]),
            down=self.lin(W[A + "mlp.down_proj.weight"]))

    def _weights(self) -> None:
        p = self.p
        self.taps = 4
        self.lw = [self._la_weights(f"layers.{i}.") if t == "linear_attention" else self._fa_weights(f"layers.{i}.", i)
                   for i, t in enumerate(self.types)]
        if self.gemma:
            for w, t in zip(self.lw, self.types):
                w["rope"] = t
        if self.ple_dim:
            self.ple_w = dict(
                model_proj=self.lin(self.w["per_layer_model_projection.weight"]),
                proj_scale=p.const(np.array([F32(self.H ** -0.5)], F32)),
                proj_norm=self.gamma1(self.w["per_layer_projection_norm.weight"]),
                in_scale=p.const(np.array([F32(2.0 ** -0.5)], F32)))
        self.final_norm = self.gamma1(self.w["norm.weight"])
        if self.mtp:
            W = self.w
            self.mw = dict(self._fa_weights("mtp.layers.0."), fc=self.lin(W["mtp.fc.weight"]),
                           ge=self.gamma1(W["mtp.pre_fc_norm_embedding.weight"]),
                           gh=self.gamma1(W["mtp.pre_fc_norm_hidden.weight"]),
                           norm=self.gamma1(W["mtp.norm.weight"]))

        def table(theta: float) -> V:
            """RoPE rows t = cos(t * inv_freq), sin(t * inv_freq) in fp32, as torch computes them."""
            th = F32(theta)
            inv = (1.0 / (th ** (np.arange(0, self.rot, 2, dtype=F32) / F32(self.rot)))).astype(F32)
            fr = (np.arange(self.T, dtype=F32)[:, None] * inv[None, :]).astype(F32)
            return p.const(np.concatenate([np.cos(fr), np.sin(fr)], axis=1).astype(F32))
        if self.gemma4:
            # per layer type, over that type's head dim: default RoPE, or proportional (only the
            # first partial_rotary_factor of the angles rotate; the rest have frequency 0)
            self.rope_tabs = {}
            for t in sorted(set(self.types)):
                hd = self._layer_hd(t)
                rp = self.cfg.rope_parameters[t]
                th = F32(rp["rope_theta"])
                rt = rp.get("rope_type", "default")
                assert rt in ("default", "proportional")
                prop = rp.get("partial_rotary_factor", 1.0) if rt == "proportional" else 1.0
                ang = int(prop * hd // 2)
                inv = np.zeros(hd // 2, F32)
                inv[:ang] = (1.0 / (th ** (np.arange(0, 2 * ang, 2, dtype=F32) / F32(hd)))).astype(F32)
                fr = (np.arange(self.T, dtype=F32)[:, None] * inv[None, :]).astype(F32)
                self.rope_tabs[t] = p.const(np.concatenate([np.cos(fr), np.sin(fr)], axis=1).astype(F32))
        elif self.gemma:
            self.rope_tabs = {t: table(self.cfg.rope_parameters[t]["rope_theta"]) for t in sorted(set(self.types))}
        else:
            self.rope_tab = table(self.cfg.rope_parameters["rope_theta"])
        if self.softcap is not None:
            sc = float(self.softcap)
            self.sc_inv2 = p.const(np.array([F32(2.0 / sc)], F32))
            self.sc_two = p.const(np.array([F32(2.0 * sc)], F32))
            self.sc_val = p.const(np.array([F32(sc)], F32))
        self.head_lins = []
        if self.head:
            e = self.w["embed_tokens.weight"]
            hr = head_rows(e.shape[0])
            self.head_lins = [self.lin(e[r:r + hr]) for r in range(0, e.shape[0], hr)]

    def embed(self, ids) -> np.ndarray:
        return input_embedding(self.cfg, self.w["embed_tokens.weight"][np.asarray(ids)])

    # ------------------------------------------------------------------ state in DDR
    def _state(self) -> None:
        p, T, H = self.p, self.T, self.H
        if self.keep_layers:
            self.xs = [p.mat(T, H) for _ in range(len(self.types) + 1)]
            self.x0 = self.xs[0]
        else:
            self.x0 = p.mat(T, H)
            xb0, xb1 = p.mat(T, H), p.mat(T, H)
            self.xs = [self.x0] + [xb0 if i % 2 == 0 else xb1 for i in range(len(self.types))]
        if self.ple_dim:
            cols = len(self.types) * self.ple_dim
            self.ple0 = p.mat(T, cols)             # the host's per-layer token rows [T, L * ple_dim]
            self.ple = p.mat(T, cols)              # projected
        else:
            self.ple0 = self.ple = None
        self.y = p.mat(T, H)
        kd, vd, hist = self.nk * self.dk, self.nv * self.dv, self.taps - 1
        self.st = []
        last_kv: dict[str, dict] = {}
        for i, t in enumerate(self.types):
            if t == "linear_attention":
                # the conv inputs (rows t + hist; the first hist rows are the zero history) and the
                # DeltaNet state, one [dk, dv] matrix per value head
                # (two copies with the MTP head: a verify's last token updates the other one)
                self.st.append(dict(cin={n: p.mat(T + hist, d) for n, d in (("q", kd), ("k", kd), ("v", vd))},
                                    S=[[p.mat(self.dk, self.dv, self.state_fmt) for _ in range(self.nv)]
                                       for _ in range(2 if self.mtp else 1)]))
            elif i < self.first_kv_shared:         # a KV cache (zero padded)
                hd = self._layer_hd(t)
                kv = dict(kc=p.mat(self.Tp, self.nkv * hd), vc=p.mat(self.Tp, self.nkv * hd))
                self.st.append(kv)
                last_kv[t] = kv
            else:                                  # KV-shared: the last cache of the same layer type
                self.st.append(last_kv[t])
        if self.mtp:                               # the MTP layer's KV cache (row r: token r + 1, hidden r)
            self.mst = dict(kc=p.mat(self.Tp, self.nkv * self.hd), vc=p.mat(self.Tp, self.nkv * self.hd))
        self.logits = p.mat(self.verify_rows, self.vocab) if self.head else None

    def embed_ple(self, ids) -> np.ndarray:
        """Gemma 4's per-layer token rows [len(ids), L * ple_dim] (the host's lookup)."""
        return ple_embedding(self.cfg, self.w["embed_tokens_per_layer.weight"][np.asarray(ids)])

    def input(self, x: np.ndarray, t0: int = 0, ple: np.ndarray | None = None) -> None:
        a = self.p.base + self.x0.off + t0 * self.x0.ld
        self.p.ddr[a:a + x.size * 4] = np.asarray(x, F32).tobytes()
        if ple is not None:
            pa = self.p.base + self.ple0.off + t0 * self.ple0.ld
            self.p.ddr[pa:pa + ple.size * 4] = np.asarray(ple, F32).tobytes()

    # ------------------------------------------------------------------ blocks
    def chunk(self, t0: int, n: int, all_rows: bool = False, parity: int = 0, spec: bool = False) -> None:
        """Tokens t0 .. t0 + n - 1 through every layer, the final norm and (with the head) the last
        token's logits (all_rows: every token's, for a speculative verify). parity: the DeltaNet
        state copy in use; spec: the last token writes the other copy, so a rejected draft leaves
        this one as it was after token n - 2 (accepted: the parity flips)."""
        assert not all_rows or n <= self.verify_rows
        self.parity, self.spec = parity, spec
        p = self.p
        if self.ple_dim:
            p.top = self.scratch0
            self._project_ple(t0, n)
            assert p.top <= self.scratch_end, "scratch_bytes too small for the per-layer projection"
        for i, t in enumerate(self.types):
            p.top = self.scratch0                  # this layer's temporaries over the last layer's
            if t == "linear_attention":
                self._la(i, t0, n)
            else:
                self._fa_block(self.lw[i], self.st[i], self.xs[i].rowv(t0, n), self.xs[i + 1].rowv(t0, n), t0, n, i)
            assert p.top <= self.scratch_end, "scratch_bytes too small for this chunk"
        p.top = self.scratch0
        p.norm(self.xs[-1].rowv(t0, n), self.final_norm, self.eps, self.y.rowv(t0, n))
        if self.head:
            r = n if all_rows else 1
            self._head(self.y.rowv(t0 + n - r, r))
        assert p.top <= self.scratch_end, "scratch_bytes too small for this chunk"
        p.top = self.end

    def _project_ple(self, t0: int, n: int) -> None:
        """Gemma 4's per-layer inputs: the rows' projection [n, L * ple_dim] times H^-0.5, the RMSNorm
        per layer block, plus the host's per-layer token rows, times 2^-0.5."""
        p, P, L_n = self.p, self.ple_dim, len(self.types)
        pw = self.ple_w
        proj = p.mat(n, L_n * P)
        self.linear(self.x0.rowv(t0, n), pw["model_proj"], proj)
        p.elt(C.ELT_MUL, proj, pw["proj_scale"], proj, bmode=C.BM_SCALAR)
        proj_n = p.mat(n, L_n * P)
        p.norm(proj.heads(P), pw["proj_norm"], self.eps, proj_n.heads(P))
        dst = self.ple.rowv(t0, n)
        p.elt(C.ELT_ADD, proj_n, self.ple0.rowv(t0, n), dst)
        p.elt(C.ELT_MUL, dst, pw["in_scale"], dst, bmode=C.BM_SCALAR)

    def swap_state(self) -> None:
        """The second DeltaNet state copy into the first (ELT MUL by an exact 1.0), so that plain
        queues (parity 0) can follow a speculative run."""
        p = self.p
        for st, w in zip(self.st, self.lw):
            if "S" in st:
                one = replace(w["kscale"], rows=1, cols=1, ld=4)
                for a, b in zip(st["S"][1], st["S"][0]):
                    p.elt(C.ELT_MUL, a, one, b, bmode=C.BM_SCALAR)

    def mtp_chunk(self, r0: int, n: int, head: bool = True) -> None:
        """MTP rows r0 .. r0 + n - 1 (row r: the embedding of token r + 1 and the hidden state of
        position r, predicting token r + 2): fc over the two norms, one gated full-attention layer
        with its own KV cache, the norm and (head) the last row's logits on the tied head."""
        p, w, H = self.p, self.mw, self.H
        p.top = self.scratch0
        cat = p.mat(n, 2 * H)
        p.norm(self.x0.rowv(r0 + 1, n), w["ge"], self.eps, cat.colv(0, H))
        p.norm(self.y.rowv(r0, n), w["gh"], self.eps, cat.colv(H, H))
        x, out = p.mat(n, H), p.mat(n, H)
        self.linear(cat, w["fc"], x)
        self._fa_block(w, self.mst, x, out, r0, n)
        if head:
            y = p.mat(1, H)
            p.norm(out.rowv(n - 1, 1), w["norm"], self.eps, y)
            self._head(y)
        assert p.top <= self.scratch_end, "scratch_bytes too small for this chunk"
        p.top = self.end

    def _head(self, y: V) -> None:
        p, r, c0 = self.p, y.rows, 0
        qs = p.quant(y) if self.wbits == 8 else None
        for lin in self.head_lins:
            out = V(self.logits.off + 4 * c0 * r, r, lin.n, 4 * lin.n)
            self.linear(y, lin, out, qs=qs)
            if self.softcap is not None:
                # sc * tanh(x / sc) as 2 sc * sigmoid(2 x / sc) - sc
                p.elt(C.ELT_MUL, out, self.sc_inv2, out, bmode=C.BM_SCALAR)
                p.elt(C.ELT_MUL, out, self.sc_two, out, bmode=C.BM_SCALAR, act=C.ACT_SIGMOID)
                p.elt(C.ELT_SUB, out, self.sc_val, out, bmode=C.BM_SCALAR)
            c0 += lin.n

    def _linear_k(self, x: V, lins, qs, out: V) -> None:
        """A linear whose weights may be split into K blocks: partials added in block order."""
        p, n = self.p, x.rows
        lins = lins if isinstance(lins, list) else [lins]
        c0 = 0
        for i, lin in enumerate(lins):
            part = out if i == 0 else p.mat(n, self.H)
            self.linear(x.colv(c0, lin.k), lin, part, qs=None if qs is None else (qs[0].colv(c0, lin.k), qs[1]))
            if i:
                p.elt(C.ELT_ADD, out, part, out)
            c0 += lin.k

    def _mlp(self, w: dict, x: V, out: V) -> None:
        p, n = self.p, x.rows
        h = p.mat(n, self.H)
        p.norm(x, w["ln_post"], self.eps, h)
        qs = p.quant(h) if self.wbits == 8 else None
        g, u = p.mat(n, w["gate"].n), p.mat(n, w["up"].n)
        self.linear(h, w["gate"], g, act=C.ACT_GELU if (self.gemma or self.gemma4) else C.ACT_SILU, qs=qs)
        self.linear(h, w["up"], u, qs=qs)
        p.elt(C.ELT_MUL, g, u, g)
        gqs = p.quant(g) if self.wbits == 8 else None
        d = p.mat(n, self.H)
        self._linear_k(g, w["down"], gqs, d)
        if w.get("mlp_norm") is not None:
            dn = p.mat(n, self.H)
            p.norm(d, w["mlp_norm"], self.eps, dn)
            d = dn
        p.elt(C.ELT_ADD, x, d, out)

    def _la(self, li: int, t0: int, n: int) -> None:
        """A gated DeltaNet layer (llm.py:642-700): ln_in + quant; the q, k, v projections into the
        conv input rows, z, beta = sigmoid(b), softplus(a + dt_bias); g = -exp(A_log) * softplus,
        decay = exp(g); the causal depthwise conv over the last taps rows (ELT MUL, then MULADD in
        tap order) and SiLU; q and k L2-normed per head (q times dk^-0.5 through gamma); then token
        by token and head by head S = S * decay, kv_mem = S^T k, delta = (v - kv_mem) * beta,
        S += k (x) delta, out = S^T q; the gated RMSNorm per head, times silu(z), out_proj, the
        residual and the MLP."""
        p, w, st = self.p, self.lw[li], self.st[li]
        kd, vd, hist = self.nk * self.dk, self.nv * self.dv, self.taps - 1
        x = self.xs[li].rowv(t0, n)
        h = p.mat(n, self.H)
        p.norm(x, w["ln_in"], self.eps, h)
        qs = p.quant(h) if self.wbits == 8 else None
        for nm in ("q", "k", "v"):
            self.linear(h, w[nm], st["cin"][nm].rowv(hist + t0, n), qs=qs)
        z = p.mat(n, vd)
        self.linear(h, w["z"], z, qs=qs)
        beta, sp = p.mat(n, self.nv), p.mat(n, self.nv)
        self.linear(h, w["b"], beta, act=C.ACT_SIGMOID, qs=qs)
        self.linear(h, w["a"], sp, act=C.ACT_SOFTPLUS, qs=qs)
        g = p.mat(n, self.nv)
        p.elt(C.ELT_MUL, sp, w["negA"], g, bmode=C.BM_ROW)
        decay = p.mat(n, self.nv)
        p.act(g, C.ACT_EXP, decay)
        conv = {}
        for nm, d in (("q", kd), ("k", kd), ("v", vd)):
            src, acc = st["cin"][nm], p.mat(n, d)
            p.elt(C.ELT_MUL, src.rowv(t0, n), w["conv"][nm][0], acc, bmode=C.BM_ROW)
            for j in range(1, self.taps):
                p.elt(C.ELT_MULADD, src.rowv(t0 + j, n), w["conv"][nm][j], acc, bmode=C.BM_ROW, c=acc)
            o = p.mat(n, d)
            p.act(acc, C.ACT_SILU, o)
            conv[nm] = o
        qn, kn = p.mat(n, kd), p.mat(n, kd)
        p.norm(conv["q"].heads(self.dk), w["qscale"], 1e-6, qn.heads(self.dk), l2=True)
        p.norm(conv["k"].heads(self.dk), w["kscale"], 1e-6, kn.heads(self.dk), l2=True)
        qh, kh, vh = qn.heads(self.dk), kn.heads(self.dk), conv["v"].heads(self.dv)
        o = p.mat(n, vd)
        oh = o.heads(self.dv)
        kvm, dl = p.mat(1, self.dv), p.mat(1, self.dv)
        for t in range(n):
            for hh in range(self.nv):
                r = t * self.nv + hh
                # the decay pass reads the state in use; a verify's last token writes the other copy
                S0 = st["S"][self.parity][hh]
                S = st["S"][1 - self.parity][hh] if self.spec and t == n - 1 else S0
                p.elt(C.ELT_MUL, S0, decay.rowv(t, 1).colv(hh, 1), S, bmode=C.BM_SCALAR)
                p.fdot(kh.rowv(r, 1), S, kvm, nn=True)
                p.elt(C.ELT_SUB, vh.rowv(r, 1), kvm, dl)
                p.elt(C.ELT_MUL, dl, beta.rowv(t, 1).colv(hh, 1), dl, bmode=C.BM_SCALAR)
                p.elt(C.ELT_MULADD, dl, kh.rowv(r, 1), S, bmode=C.BM_COL, arow=True, c=S)
                p.fdot(qh.rowv(r, 1), S, oh.rowv(r, 1), nn=True)
        on, og = p.mat(n, vd), p.mat(n, vd)
        p.norm(oh, w["gnorm"], self.eps, on.heads(self.dv))
        p.elt(C.ELT_MUL, z, on, og, act=C.ACT_SILU)
        a = p.mat(n, self.H)
        self.linear(og, w["out"], a)
        x1 = p.mat(n, self.H)
        p.elt(C.ELT_ADD, x, a, x1)
        self._mlp(w, x1, self.xs[li + 1].rowv(t0, n))

    def _fa_block(self, w: dict, st: dict, x: V, out: V, t0: int, n: int, li: int | None = None) -> None:
        p = self.p
        kc, vc = st["kc"], st["vc"]
        nh, nkv = self.nh, self.nkv
        hd, rot = w.get("hd", self.hd), w.get("rot", self.rot)
        h = p.mat(n, self.H)
        p.norm(x, w["ln_in"], self.eps, h)
        qs = p.quant(h) if self.wbits == 8 else None
        q = p.mat(n, nh * hd)
        self.linear(h, w["q"], q, qs=qs)
        if w["g"] is not None:
            g = p.mat(n, nh * hd)
            self.linear(h, w["g"], g, qs=qs)
        qn = p.mat(n, nh * hd)
        p.norm(q.heads(hd), w["qn"], self.eps, qn.heads(hd))
        qr = p.mat(n, nh * hd)
        tab = (self.rope_tabs[w["rope"]] if "rope" in w else self.rope_tab).rowv(t0, (n * nh - 1) // nh + 1)
        p.rope(qn.heads(hd), tab, nh, rot, qr.heads(hd))
        if not w.get("kv_shared", False):          # a KV-shared layer reads an earlier layer's cache
            k = p.mat(n, nkv * hd)
            self.linear(h, w["k"], k, qs=qs)
            if w.get("vn") is not None:            # Gemma 4: V through an RMSNorm without scale
                vr = p.mat(n, nkv * hd)
                self.linear(h, w["v"], vr, qs=qs)
                p.norm(vr.heads(hd), w["vn"], self.eps, vc.rowv(t0, n).heads(hd))
            else:
                self.linear(h, w["v"], vc.rowv(t0, n), qs=qs)  # V straight into the cache
            kn = p.mat(n, nkv * hd)
            p.norm(k.heads(hd), w["kn"], self.eps, kn.heads(hd))
            p.rope(kn.heads(hd), tab, nkv, rot, kc.rowv(t0, n).heads(hd))
        nk = pad16(t0 + n)
        att = p.mat(n, nh * hd)
        sc, pr = p.mat(n, nk), p.mat(n, nk)
        for hh in range(nh):
            kv = hh // (nh // nkv)
            qv = V(qr.off + hh * hd * 4, n, hd, qr.ld)
            kmat = V(kc.off + kv * hd * 4, nk, hd, kc.ld)
            vmat = V(vc.off + kv * hd * 4, nk, hd, vc.ld)
            p.fdot(qv, kmat, sc, nn=False)
            p.softmax_causal(sc, pr, t0 + 1)
            p.fdot(pr, vmat, V(att.off + hh * hd * 4, n, hd, att.ld), nn=True)
        if w["g"] is not None:
            ga = p.mat(n, nh * hd)
            p.elt(C.ELT_MUL, g, att, ga, act=C.ACT_SIGMOID)          # sigmoid(gate) * attention
            att = ga
        aqs = p.quant(att) if self.wbits == 8 else None
        o = p.mat(n, self.H)
        self._linear_k(att, w["o"], aqs, o)
        if w.get("attn_norm") is not None:
            on = p.mat(n, self.H)
            p.norm(o, w["attn_norm"], self.eps, on)
            o = on
        x1 = p.mat(n, self.H)
        p.elt(C.ELT_ADD, x, o, x1)
        x2 = p.mat(n, self.H) if "ple_gate" in w else out
        self._mlp(w, x1, x2)
        if "ple_gate" in w:                        # Gemma 4: the layer's per-layer input, gated
            P = self.ple_dim
            pg = p.mat(n, P)
            self.linear(x2, w["ple_gate"], pg, act=C.ACT_GELU)
            p.elt(C.ELT_MUL, pg, self.ple.rowv(t0, n).colv(li * P, P), pg)
            pp = p.mat(n, self.H)
            self.linear(pg, w["ple_proj"], pp)
            ppn = p.mat(n, self.H)
            p.norm(pp, w["ple_norm"], self.eps, ppn)
            p.elt(C.ELT_ADD, x2, ppn, out)
        if w.get("layer_scalar") is not None:
            p.elt(C.ELT_MUL, out, w["layer_scalar"], out, bmode=C.BM_SCALAR)

    # ------------------------------------------------------------------ running chunk by chunk
    def stage(self, ddr: bytearray, a: int, b: int) -> tuple[int, int]:
        assert self.qbase is not None and b - a <= self.queue_cap, "queue_cap too small"
        q = self.p.base + self.qbase
        for i in range(a, b):
            ddr[q + 64 * (i - a):q + 64 * (i - a + 1)] = self.p.descs[i]
        return q, b - a

    def put_input(self, ddr: bytearray, t0: int, x: np.ndarray, ple: np.ndarray | None = None) -> None:
        a = self.p.base + self.x0.off + t0 * self.x0.ld
        ddr[a:a + x.size * 4] = np.asarray(x, F32).tobytes()
        if ple is not None:
            pa = self.p.base + self.ple0.off + t0 * self.ple0.ld
            ddr[pa:pa + ple.size * 4] = np.asarray(ple, F32).tobytes()

    def logits_of(self, ddr) -> np.ndarray:
        a = self.p.base + self.logits.off
        return np.frombuffer(bytes(ddr[a:a + 4 * self.vocab]), "<f4").copy()

    def logits_rows(self, ddr, n: int) -> np.ndarray:
        a = self.p.base + self.logits.off
        flat = np.frombuffer(bytes(ddr[a:a + 4 * self.vocab * n]), "<f4")
        out, c0 = np.empty((n, self.vocab), F32), 0
        for lin in self.head_lins:
            out[:, c0:c0 + lin.n] = flat[c0 * n:(c0 + lin.n) * n].reshape(n, lin.n)
            c0 += lin.n
        return out

    def generate(self, run, prompt, n_new: int, chunk: int = 0):
        """Greedy decoding with the host in the loop: run(ddr, q, n) -> ddr executes one chunk's
        queue. chunk > 0 feeds the prompt in chunks of that many tokens (the board runtime's
        prefill); 0 feeds it whole (llm.py:815-836). Returns (ids, logits per run, descriptors per run)."""
        assert self.head
        ddr = self.p.ddr
        ids, logits, counts = list(prompt), [], []
        spans = [(s, min(chunk, len(prompt) - s)) for s in range(0, len(prompt), chunk)] if chunk else \
            [(0, len(prompt))]
        for i in range(len(spans) + n_new):
            t0, n = spans[i] if i < len(spans) else (len(ids) - 1, 1)
            toks = ids[t0:t0 + n]
            self.put_input(ddr, t0, self.embed(toks), self.embed_ple(toks) if self.ple_dim else None)
            a = len(self.p.descs)
            self.chunk(t0, n)
            q, cnt = self.stage(ddr, a, len(self.p.descs))
            out = run(ddr, q, cnt)
            ddr = out if isinstance(out, bytearray) else bytearray(out)
            if i >= len(spans) - 1:
                lg = self.logits_of(ddr)
                logits.append(lg)
                counts.append(cnt)
                ids.append(int(np.argmax(lg)))
        return ids, logits, counts

    def generate_mtp(self, run, prompt, n_new: int, oracle=None):
        """Greedy speculative decoding with the MTP head: the tokens of generate(). Each round
        verifies [current, draft] as two rows; a hit emits two tokens and flips the state copy, a
        miss emits the correction and keeps it; the MTP then takes the rows the verify made known
        and drafts the next token. oracle(t, draft) may replace a draft (tests). Returns (token ids,
        {position: its logits}, rounds)."""
        assert self.head and self.mtp and self.verify_rows >= 2
        state = dict(ddr=self.p.ddr)

        def go(emit) -> None:
            a = len(self.p.descs)
            emit()
            q, c = self.stage(state["ddr"], a, len(self.p.descs))
            out = run(state["ddr"], q, c)
            state["ddr"] = out if isinstance(out, bytearray) else bytearray(out)

        def put(t: int, toks) -> None:
            self.put_input(state["ddr"], t, self.embed(toks))
        ids, P, par, rounds = list(prompt), len(prompt), 0, 0
        put(0, ids)
        go(lambda: self.chunk(0, P))
        lg = {P - 1: self.logits_of(state["ddr"])}
        ids.append(int(np.argmax(lg[P - 1])))
        put(P, ids[P:])
        go(lambda: self.mtp_chunk(0, P))                    # rows 0 .. P - 1; the last one drafts
        t = P                                               # ids[t]: known, not yet in the cache
        while len(ids) < P + n_new + 1:
            d = int(np.argmax(self.logits_of(state["ddr"])))
            if oracle is not None:
                d = oracle(t, d)
            put(t + 1, [d])
            go(lambda: self.chunk(t, 2, all_rows=True, parity=par, spec=True))
            rows = self.logits_rows(state["ddr"], 2)
            rounds += 1
            lg[t] = rows[0]
            x = int(np.argmax(rows[0]))
            ids.append(x)
            if x == d:
                lg[t + 1] = rows[1]
                ids.append(int(np.argmax(rows[1])))
                par = 1 - par
                put(t + 2, ids[t + 2:t + 3])
                go(lambda: self.mtp_chunk(t, 2))
                t += 2
            else:
                put(t + 1, [x])
                go(lambda: self.mtp_chunk(t, 1))
                t += 1
        return ids, lg, rounds
