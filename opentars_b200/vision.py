"""Qwen3.5's vision tower lowered to tars_mini v0.4 descriptors (tars_mini/qwen_vit.py).

The tower: a patch embedding (the Conv3d with kernel = stride as one linear over the patch
vector), `depth` blocks of LayerNorm -> qkv -> axial 2-D RoPE on q and k -> attention over the
whole image (FDOT NT, softmax over keys padded to 16 with the padding masked, FDOT NN) -> proj ->
residual, LayerNorm -> fc1 (tanh GELU) -> fc2 -> residual, then the merger: LayerNorm per patch,
the 2x2 spatial-merge block's 4 rows read as one row, fc1 -> GELU -> fc2. Every GEMM has M = the
patch count (or a quarter of it for the merger), so an image runs its linears on the tensor-core
GEMM. The host prepares what the reference's host prepares: the patches in spatial-merge order,
the bilinearly resampled position table and one rotary row per patch.

Restates, so that the same DDR image and the same descriptor queue come out byte for byte:
  * vision_config, head_dim, random_vision             qwen_vit.py:46-86
  * patchify                                           qwen_vit.py:115-129
  * position_embeddings, rope_table: the tower's fp32 host computations (its position-table
    interpolation and axial rotary angles), restated and pinned to transformers' tower
  * VisionLowering (weights, buffers, the image's descriptors, run)   qwen_vit.py:226-418

    cfg = vision_config(**small); w = random_vision(cfg)
    px, grid = patchify(image, cfg)
    low = VisionLowering(cfg, w, patches_max=len(px))
    tokens = low.run(px, position_embeddings(cfg, w, grid), rope_table(cfg, grid))
"""
from __future__ import annotations

import numpy as np

from . import contract as C
from .lowering import QLin, V, Dev, pad16
from .models import quantize_weight

F32 = np.float32

# the 0.8B vision_config (Qwen3.5-0.8B config.json)
VIT_08B = dict(depth=12, hidden_size=768, intermediate_size=3072, num_heads=12, in_channels=3,
               patch_size=16, spatial_merge_size=2, temporal_patch_size=2, out_hidden_size=1024,
               num_position_embeddings=2304, hidden_act="gelu_pytorch_tanh")
VIT_EPS = 1e-6
MASK_NEG = F32(-3.0e38)          # a padded score: exp(that - max) underflows to +0


def vision_config(path: str | None = None, **over):
    """A Qwen3_5VisionConfig: `path`'s config.json vision_config (else the 0.8B numbers), any
    keyword overriding a field."""
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5VisionConfig
    base = dict(VIT_08B)
    if path is not None:
        import json
        from pathlib import Path
        vc = json.loads((Path(path) / "config.json").read_text())["vision_config"]
        base = dict(base, **{k: v for k, v in vc.items() if k != "model_type"})
    base.update(over)
    cfg = Qwen3_5VisionConfig(**base)
    cfg._attn_implementation = "eager"
    return cfg


def head_dim(cfg) -> int:
    return cfg.hidden_size // cfg.num_heads


def random_vision(cfg, seed: int = 0) -> dict[str, np.ndarray]:
    """Random tower weights in the model's state_dict order: norm weights 1 + N(0, 0.1), every
    other parameter (linears, biases, the position table) N(0, 0.02)."""
    import torch
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5VisionModel
    with torch.device("meta"):
        m = Qwen3_5VisionModel(cfg)
    rng = np.random.default_rng(seed)
    w = {}
    for name, p in m.state_dict().items():
        shape = tuple(p.shape)
        if name.endswith(("norm.weight", "norm1.weight", "norm2.weight")):
            a = 1 + rng.normal(0, 0.1, shape)
        else:
            a = rng.normal(0, 0.02, shape)
        w[name] = a.astype(F32)
    return w


# ---------------------------------------------------------------------- host preprocessing
def patchify(img, cfg) -> tuple[np.ndarray, np.ndarray]:
    """A normalised image [C, H, W] (sides multiples of patch * merge) as patches
    [P, C * temporal * patch * patch] in spatial-merge-block order (block row, block column, then
    the row and column inside the block), each flattened (channel, temporal, row, column) with
    both temporal slots holding the still image; and grid_thw [[1, H / patch, W / patch]]."""
    img = np.asarray(img, F32)
    c, hh, ww = img.shape
    ps, ms, tp = cfg.patch_size, cfg.spatial_merge_size, cfg.temporal_patch_size
    if c != cfg.in_channels or hh % (ps * ms) or ww % (ps * ms):
        raise ValueError(f"image {img.shape}: {cfg.in_channels} channels, sides multiples of {ps * ms}")
    gh, gw = hh // ps, ww // ps
    # axes: channel, block row, row in block, pixel row, block column, column in block, pixel column
    x = img.reshape(c, gh // ms, ms, ps, gw // ms, ms, ps).transpose(1, 4, 2, 5, 0, 3, 6)
    x = np.broadcast_to(x[..., None, :, :], x.shape[:5] + (tp, ps, ps))
    return np.ascontiguousarray(x, F32).reshape(gh * gw, c * tp * ps * ps), np.array([[1, gh, gw]])


def _merge_order(h: int, w: int, ms: int) -> np.ndarray:
    """Row-major patch indices of an h x w grid in spatial-merge order: merge blocks row-major,
    then the rows and columns inside a block."""
    r = np.arange(h).reshape(h // ms, ms)[:, None, :, None]
    c = np.arange(w).reshape(w // ms, ms)[None, :, None, :]
    return np.broadcast_to(r * w + c, (h // ms, w // ms, ms, ms)).reshape(-1)


def position_embeddings(cfg, w, grid_thw) -> np.ndarray:
    """The learned position table resampled to the patch grid [P, hidden], as the tower computes it
    in fp32: per grid row and column a linspace over the table's side with aligned corners, the
    four corners' rows weighted by (1 - dh)(1 - dw), (1 - dh) dw, dh (1 - dw), dh dw and added in
    that order, then the patches put in spatial-merge order."""
    import torch
    side = int(cfg.num_position_embeddings ** 0.5)
    tab = torch.from_numpy(np.asarray(w["pos_embed.weight"], F32))
    out = []
    for t, h, wd in np.asarray(grid_thw).tolist():
        hi, wi = torch.linspace(0, side - 1, h), torch.linspace(0, side - 1, wd)
        hf, wf = hi.int(), wi.int()
        hc, wc = (hf + 1).clip(max=side - 1), (wf + 1).clip(max=side - 1)
        dh, dw = hi - hf, wi - wf
        idx = [(hf[:, None] * side + wf[None]).flatten(), (hf[:, None] * side + wc[None]).flatten(),
               (hc[:, None] * side + wf[None]).flatten(), (hc[:, None] * side + wc[None]).flatten()]
        wt = [((1 - dh)[:, None] * (1 - dw)[None]).flatten(), ((1 - dh)[:, None] * dw[None]).flatten(),
              (dh[:, None] * (1 - dw)[None]).flatten(), (dh[:, None] * dw[None]).flatten()]
        pe = tab[idx[0]] * wt[0][:, None]
        for i in range(1, 4):
            pe = pe + tab[idx[i]] * wt[i][:, None]
        pe = pe.numpy()[_merge_order(h, wd, cfg.spatial_merge_size)]
        out.append(np.tile(pe, (t, 1)))
    return np.ascontiguousarray(np.concatenate(out), F32)


def rope_table(cfg, grid_thw) -> np.ndarray:
    """One ROPE table row per patch [P, head_dim]: cos then sin of the axial angles - the patch's
    grid row times the head_dim/4 inverse frequencies, then its grid column times them - in fp32
    (the tower pairs element i with i + head_dim/2, so that half is the whole rotation)."""
    import torch
    dim = head_dim(cfg) // 2
    rp = getattr(cfg, "rope_parameters", None) or {}
    theta = rp.get("rope_theta", 10000.0)                   # the tower's rotary base
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
    rows = []
    for t, h, wd in np.asarray(grid_thw).tolist():
        order = _merge_order(h, wd, cfg.spatial_merge_size)
        pos = torch.from_numpy(np.stack([order // wd, order % wd], axis=-1)).repeat(t, 1)
        rows.append(torch.cat([torch.outer(pos[:, 0].float(), inv), torch.outer(pos[:, 1].float(), inv)], dim=-1))
    ang = torch.cat(rows)
    return torch.cat([ang.cos(), ang.sin()], dim=-1).numpy().astype(F32)


# ---------------------------------------------------------------------- the lowering
class VisionLowering:
    """The tower as v0.4 descriptors. The key axis is padded to a multiple of 16: the padded key
    and value rows are zero and the padded scores are set to MASK_NEG (a MUL by a 0/1 row, then an
    ADD of a 0 / MASK_NEG row), so the padding changes no sum. Weights and buffers are sized for
    `patches_max`; the patches, the position and rotary rows and the two mask rows are written per
    image, so one program serves any image up to that capacity. W8A8 only."""

    def __init__(self, cfg, w, patches_max: int, ddr_bytes: int = 1 << 28, scratch_bytes: int | None = None,
                 wbits: int = 8):
        if wbits != 8:
            raise ValueError("the vision tower is lowered W8A8")
        self.cfg, self.w = cfg, w
        self.H, self.I = cfg.hidden_size, cfg.intermediate_size
        self.nh, self.hd = cfg.num_heads, head_dim(cfg)
        self.K = cfg.in_channels * cfg.temporal_patch_size * cfg.patch_size ** 2
        self.ms2 = cfg.spatial_merge_size ** 2
        self.P, self.npad = patches_max, pad16(patches_max)
        assert self.nh * self.hd == self.H and self.H % 16 == 0 and self.K % 16 == 0
        assert self.hd % 32 == 0, "the rotary width must be a multiple of 32"
        self.eps = VIT_EPS
        self.p = self.prog = Dev(ddr_bytes=ddr_bytes)
        self._weights()
        self._bufs()
        self.scratch0 = self.p.top
        if scratch_bytes is None:                    # the patches, position and rotary rows, widest quant
            scratch_bytes = 4 * patches_max * (self.K + self.ms2 * self.H + 2 * self.H) + (1 << 20)
        self.scratch_end = self.p.alloc(scratch_bytes) + scratch_bytes
        self.end = self.p.top

    def lin(self, w: np.ndarray, b: np.ndarray | None = None) -> QLin:
        qw = quantize_weight(np.asarray(w, np.float64), per_channel=True)
        assert qw.n % 16 == 0 and qw.k % 16 == 0, (qw.n, qw.k)
        b_off = self.p.put(np.asarray(b, F32)) if b is not None else None
        return QLin(self.p.put(qw.q, "i1"), self.p.put(qw.scale), b_off, qw.n, qw.k)

    def _weights(self) -> None:
        w, H, p = self.w, self.H, self.p
        self.pe = self.lin(w["patch_embed.proj.weight"].reshape(H, -1), w["patch_embed.proj.bias"])
        self.blocks = []
        for i in range(self.cfg.depth):
            b = f"blocks.{i}."
            self.blocks.append(dict(
                n1=(p.const(w[b + "norm1.weight"]), p.const(w[b + "norm1.bias"])),
                n2=(p.const(w[b + "norm2.weight"]), p.const(w[b + "norm2.bias"])),
                qkv=self.lin(w[b + "attn.qkv.weight"], w[b + "attn.qkv.bias"]),
                proj=self.lin(w[b + "attn.proj.weight"], w[b + "attn.proj.bias"]),
                fc1=self.lin(w[b + "mlp.linear_fc1.weight"], w[b + "mlp.linear_fc1.bias"]),
                fc2=self.lin(w[b + "mlp.linear_fc2.weight"], w[b + "mlp.linear_fc2.bias"])))
        self.m_norm = (p.const(w["merger.norm.weight"]), p.const(w["merger.norm.bias"]))
        self.m_fc1 = self.lin(w["merger.linear_fc1.weight"], w["merger.linear_fc1.bias"])
        self.m_fc2 = self.lin(w["merger.linear_fc2.weight"], w["merger.linear_fc2.bias"])
        assert self.m_fc1.k == self.ms2 * H, "the merger takes the merge block's rows as one row"
        self.sc_q = p.const(np.array([F32(self.hd ** -0.5)], F32))         # the attention scaling

    def _bufs(self) -> None:
        p, n, npad, H = self.p, self.P, self.npad, self.H
        nm = n // self.ms2
        self.kbuf = p.const(np.zeros((npad, H), F32))        # K and V rows; the padding stays zero
        self.vbuf = p.const(np.zeros((npad, H), F32))
        self.sc = p.const(np.zeros((n, npad), F32))          # one head's scores
        self.prow = p.const(np.zeros((n, npad), F32))        # its softmax
        self.mask = p.const(np.concatenate([np.ones((1, n), F32), np.zeros((1, npad - n), F32)], axis=1))
        self.mbias = p.const(np.concatenate([np.zeros((1, n), F32), np.full((1, npad - n), MASK_NEG, F32)], axis=1))
        self.zrow = p.const(np.zeros((1, H), F32))           # the zero row a copy adds
        # one INT8 activation buffer and one row-scale row, shared by every GEMM
        self.q8 = p.mat(n, max(self.I, self.ms2 * H), C.OUT_INT8)
        self.qs = p.alloc(4 * n)
        self.x = p.mat(n, H)                                 # the residual stream
        self.h = p.mat(n, H)
        self.qkv = p.mat(n, 3 * H)
        self.qd = p.mat(n, H)                                # q and k, dense (the rope's inputs)
        self.kd = p.mat(n, H)
        self.qr = p.mat(n, H)                                # q rotated and scaled
        self.att = p.mat(n, H)
        self.b = p.mat(n, H)                                 # a projection's output
        self.ml = p.mat(n, self.I)
        self.mm = p.mat(nm, self.m_fc1.n)
        self.mt = p.mat(nm, self.ms2 * H)
        self.out = p.mat(nm, self.cfg.out_hidden_size)

    def _ln(self, x: V, nb: tuple[V, V], y: V) -> None:
        self.p.rowop(x, C.ROW_LAYERNORM, y, nb[0], self.eps, beta=nb[1])

    def _quant(self, x: V) -> tuple[V, int]:
        return self.p.quant(x, V(self.q8.off, x.rows, x.cols, self.q8.ld, C.OUT_INT8), self.qs)

    def _linear(self, x: V, w: QLin, y: V, act: int = C.ACT_NONE) -> None:
        xq, xs = self._quant(x)
        self.p.gemm_rc(xq, xs, w, y, act)

    def _emit_image(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray) -> V:
        p, n, H, hd, nh, npad = self.p, patches.shape[0], self.H, self.hd, self.nh, self.npad
        assert patches.shape[1] == self.K and n <= self.P and n % self.ms2 == 0
        assert pos.shape == (n, H) and rope.shape == (n, hd)
        p.top = self.scratch0
        # the mask rows follow this image's patch count
        on, ng = np.zeros(npad, F32), np.zeros(npad, F32)
        on[:n], ng[n:] = 1.0, MASK_NEG
        for buf, row in ((self.mask, on), (self.mbias, ng)):
            a = p.base + buf.off
            p.ddr[a:a + 4 * npad] = row.tobytes()
        x = self.x.rowv(0, n)
        self._linear(p.const(np.asarray(patches, F32)), self.pe, x)      # patch embedding
        p.elt(C.ELT_ADD, x, p.const(np.asarray(pos, F32)), x)            # + position embedding
        ropet = p.const(np.asarray(rope, F32))
        sc = V(self.sc.off, n, npad, self.sc.ld)
        for b in self.blocks:
            h = self.h.rowv(0, n)
            self._ln(x, b["n1"], h)
            qkv = self.qkv.rowv(0, n)
            p.gemm_rc(*self._quant(h), b["qkv"], qkv)
            # q, k, v into dense buffers (uniform row strides for the rope and the head views)
            p.elt(C.ELT_ADD, qkv.colv(0, H), self.zrow, self.qd.rowv(0, n), bmode=C.BM_ROW)
            p.elt(C.ELT_ADD, qkv.colv(H, H), self.zrow, self.kd.rowv(0, n), bmode=C.BM_ROW)
            p.elt(C.ELT_ADD, qkv.colv(2 * H, H), self.zrow, self.vbuf.rowv(0, n), bmode=C.BM_ROW)
            qr = self.qr.rowv(0, n)
            p.rope(self.qd.rowv(0, n).heads(hd), ropet, nh, hd, qr.heads(hd))
            p.elt(C.ELT_MUL, qr, self.sc_q, qr, bmode=C.BM_SCALAR)
            p.rope(self.kd.rowv(0, n).heads(hd), ropet, nh, hd, self.kbuf.rowv(0, n).heads(hd))
            att = self.att.rowv(0, n)
            for hh in range(nh):
                p.fdot(V(qr.off + hh * hd * 4, n, hd, 4 * H), V(self.kbuf.off + hh * hd * 4, npad, hd, 4 * H),
                       sc, nn=False)
                p.elt(C.ELT_MUL, sc, self.mask, sc, bmode=C.BM_ROW)     # padded columns -> +0
                p.elt(C.ELT_ADD, sc, self.mbias, sc, bmode=C.BM_ROW)    # -> MASK_NEG
                p.rowop(sc, C.ROW_SOFTMAX, V(self.prow.off, n, npad, self.prow.ld))
                p.fdot(V(self.prow.off, n, npad, self.prow.ld), V(self.vbuf.off + hh * hd * 4, npad, hd, 4 * H),
                       V(att.off + hh * hd * 4, n, hd, att.ld), nn=True)
            self._linear(att, b["proj"], self.b.rowv(0, n))
            p.elt(C.ELT_ADD, x, self.b.rowv(0, n), x)
            self._ln(x, b["n2"], h)
            ml = self.ml.rowv(0, n)
            p.gemm_rc(*self._quant(h), b["fc1"], ml, C.ACT_GELU)
            self._linear(ml, b["fc2"], self.b.rowv(0, n))
            p.elt(C.ELT_ADD, x, self.b.rowv(0, n), x)
        nm = n // self.ms2
        # the merger's norm per patch row, written so that the merge block's rows are one row
        self._ln(x, self.m_norm, V(self.mt.off, n, H, 4 * H))
        mt = self.mt.rowv(0, nm)
        p.gemm_rc(*self._quant(mt), self.m_fc1, self.mm.rowv(0, nm), C.ACT_GELU)
        out = self.out.rowv(0, nm)
        self._linear(self.mm.rowv(0, nm), self.m_fc2, out)
        assert p.top <= self.scratch_end, "scratch_bytes too small for one image"
        p.top = self.end
        return out

    def emit(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray, blocks: int | None = None) -> V:
        """The image's descriptors (a previous image's queue is dropped); returns the output view
        (the merged tokens, or with `blocks` the patches' hidden state after that many blocks)."""
        n = patches.shape[0]
        keep = self.blocks
        if blocks is not None:
            self.blocks = keep[:blocks]
        try:
            self.p.descs.clear()
            self.p.queue_off = None
            out = self._emit_image(patches, pos, rope)
            return out if blocks is None else self.x.rowv(0, n)
        finally:
            self.blocks = keep

    def run(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray, blocks: int | None = None,
            machine=None) -> np.ndarray:
        """Lower the image, build the program and run it on `machine` (a Machine class; default
        the B200 drop-in Machine): the visual tokens [P / merge^2, out_hidden]."""
        if machine is None:
            from .machine import Machine as machine
        out = self.emit(patches, pos, rope, blocks)
        ddr, q, cnt = self.p.build()
        m = machine(bytearray(ddr))
        st = m.run_queue(q, cnt)
        assert st.done, (st.err_code, st.op_idx)
        return self.read(m, out)

    def read(self, m, v: V) -> np.ndarray:
        a = self.p.base + v.off
        return np.stack([np.frombuffer(m.read(a + r * v.ld, 4 * v.cols), "<f4") for r in range(v.rows)])
