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
  * VisionImage (weights, buffers, the image's descriptors, run): the program the reference's
    tower lowering builds (qwen_vit.py:226-418), byte for byte, from a builder of this package

    cfg = vision_config(**small); w = random_vision(cfg)
    px, grid = patchify(image, cfg)
    tower = VisionImage(cfg, w, patches_max=len(px))
    tokens = tower.run(px, position_embeddings(cfg, w, grid), rope_table(cfg, grid))
"""
from __future__ import annotations

import numpy as np

from . import contract as C
from .model_image import pad16
from .models import quantize_weight
from .program import Buf, Image, Linear

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
    fields = dict(VIT_08B)
    if path is not None:
        import json
        import pathlib
        with open(pathlib.Path(path, "config.json")) as f:
            fields.update((k, v) for k, v in json.load(f)["vision_config"].items() if k != "model_type")
    cfg = Qwen3_5VisionConfig(**{**fields, **over})
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
    gains = ("norm.weight", "norm1.weight", "norm2.weight")
    rng = np.random.default_rng(seed)
    out = {}
    for name, t in m.state_dict().items():
        mean, std = (1.0, 0.1) if name.endswith(gains) else (0.0, 0.02)
        out[name] = rng.normal(mean, std, tuple(t.shape)).astype(F32)
    return out


# ---------------------------------------------------------------------- host preprocessing
def _merge_order(h: int, w: int, ms: int) -> np.ndarray:
    """Row-major patch indices of an h x w grid in spatial-merge order: merge blocks row-major,
    then the rows and columns inside a block."""
    r = np.arange(h).reshape(h // ms, ms)[:, None, :, None]
    c = np.arange(w).reshape(w // ms, ms)[None, :, None, :]
    return np.broadcast_to(r * w + c, (h // ms, w // ms, ms, ms)).reshape(-1)


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
    # the patches row-major as [patch, channel, 1, row, column], then taken in merge order
    tiles = img.reshape(c, gh, ps, gw, ps).transpose(1, 3, 0, 2, 4).reshape(gh * gw, c, 1, ps, ps)
    tiles = tiles[_merge_order(gh, gw, ms)]
    return np.repeat(tiles, tp, axis=2).reshape(gh * gw, -1).astype(F32), np.array([[1, gh, gw]])


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


# ---------------------------------------------------------------------- the tower's program
class VisionImage:
    """The tower as one image and one descriptor queue (W8A8). Keys are padded to a multiple of 16:
    the padded K and V rows stay zero and each head's padded scores are set to MASK_NEG (a MUL by a
    0/1 row, then an ADD of a 0 / MASK_NEG row), so the padding changes no sum. Weights and buffers
    are sized for `patches_max`; the patches, position and rotary rows and the two mask rows are
    written per image, so one program serves any image up to that capacity. Image and queue are
    byte-identical to those of the reference's tower lowering (qwen_vit.py:226-418) for the same
    image (pinned by tests/golden/vision.json)."""

    def __init__(self, cfg, w, patches_max: int, ddr_bytes: int = 1 << 28, scratch_bytes: int | None = None,
                 wbits: int = 8):
        if wbits != 8:
            raise ValueError("the vision tower is W8A8")
        self.cfg, self.w = cfg, w
        self.H, self.I, self.nh, self.hd = cfg.hidden_size, cfg.intermediate_size, cfg.num_heads, head_dim(cfg)
        self.K = cfg.in_channels * cfg.temporal_patch_size * cfg.patch_size ** 2     # one patch vector
        self.ms2 = cfg.spatial_merge_size ** 2                                       # patches per merged token
        self.P, self.npad = patches_max, pad16(patches_max)
        if self.nh * self.hd != self.H or self.H % 16 or self.K % 16 or self.hd % 32:
            raise ValueError("heads x head dim = hidden; hidden, patch vector multiples of 16; rotary of 32")
        self.eps = VIT_EPS
        self.p = Image(ddr_bytes)
        self._place_weights()
        self._place_buffers()
        if scratch_bytes is None:            # the image's patches, position and rotary rows, and slack
            scratch_bytes = 4 * patches_max * (self.K + self.ms2 * self.H + 2 * self.H) + (1 << 20)
        self.scratch0 = self.p.top
        self.scratch_end = self.p.reserve(scratch_bytes) + scratch_bytes
        self.end = self.p.top

    def _linear(self, weight, bias) -> Linear:
        qw = quantize_weight(np.asarray(weight, np.float64), per_channel=True)
        if qw.n % 16 or qw.k % 16:
            raise ValueError(f"linear {qw.n} x {qw.k}: multiples of 16")
        b_off = self.p.store(np.asarray(bias, F32))
        return Linear(self.p.store(qw.q, "i1"), self.p.store(qw.scale), b_off, qw.n, qw.k)

    def _layernorm(self, name: str) -> tuple[Buf, Buf]:
        return self.p.constant(self.w[name + ".weight"]), self.p.constant(self.w[name + ".bias"])

    def _place_weights(self) -> None:
        w, H = self.w, self.H
        self.pe = self._linear(w["patch_embed.proj.weight"].reshape(H, -1), w["patch_embed.proj.bias"])
        self.blocks = []
        for i in range(self.cfg.depth):
            pre = f"blocks.{i}."
            blk = {"n1": self._layernorm(pre + "norm1"), "n2": self._layernorm(pre + "norm2")}
            for key, name in (("qkv", "attn.qkv"), ("proj", "attn.proj"), ("fc1", "mlp.linear_fc1"),
                              ("fc2", "mlp.linear_fc2")):
                blk[key] = self._linear(w[pre + name + ".weight"], w[pre + name + ".bias"])
            self.blocks.append(blk)
        self.m_norm = self._layernorm("merger.norm")
        self.m_fc1 = self._linear(w["merger.linear_fc1.weight"], w["merger.linear_fc1.bias"])
        self.m_fc2 = self._linear(w["merger.linear_fc2.weight"], w["merger.linear_fc2.bias"])
        if self.m_fc1.k != self.ms2 * H:
            raise ValueError("the merger takes a merge block's rows as one row")
        self.sc_q = self.p.constant(np.array([F32(self.hd ** -0.5)], F32))         # the attention scaling

    def _place_buffers(self) -> None:
        p, n, npad, H, I = self.p, self.P, self.npad, self.H, self.I
        zeros = lambda r, c: p.constant(np.zeros((r, c), F32))  # noqa: E731
        self.kbuf, self.vbuf = zeros(npad, H), zeros(npad, H)                # K, V rows; padding stays 0
        self.sc, self.prow = zeros(n, npad), zeros(n, npad)                  # one head's scores, softmax
        keep = np.concatenate([np.ones((1, n), F32), np.zeros((1, npad - n), F32)], axis=1)
        self.mask = p.constant(keep)
        self.mbias = p.constant(np.where(keep > 0, F32(0), MASK_NEG).astype(F32))
        self.zrow = zeros(1, H)                                              # a copy adds this row
        self.q8 = p.matrix(n, max(I, self.ms2 * H), C.OUT_INT8)              # every GEMM's int8 rows
        self.qs = p.reserve(4 * n)                                           # and their row scales
        self.x, self.h = p.matrix(n, H), p.matrix(n, H)                      # residual, normed
        self.qkv = p.matrix(n, 3 * H)
        self.qd, self.kd, self.qr = p.matrix(n, H), p.matrix(n, H), p.matrix(n, H)
        self.att, self.b = p.matrix(n, H), p.matrix(n, H)
        self.ml = p.matrix(n, I)
        nm = n // self.ms2
        self.mm = p.matrix(nm, self.m_fc1.n)
        self.mt = p.matrix(nm, self.ms2 * H)
        self.out = p.matrix(nm, self.cfg.out_hidden_size)

    def _int8(self, x: Buf) -> tuple[Buf, int]:
        """ROW_QUANT of x into the shared int8 buffer."""
        return self.p.quantize(x, Buf(self.q8.off, x.rows, x.cols, self.q8.ld, C.OUT_INT8), self.qs)

    def _dense(self, x: Buf, w: Linear, y: Buf, act: int = C.ACT_NONE) -> None:
        xq, srow = self._int8(x)
        self.p.mm8(xq, srow, w, y, act)

    def _record(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray) -> Buf:
        p, H, hd, nh, npad = self.p, self.H, self.hd, self.nh, self.npad
        n = patches.shape[0]
        if patches.shape[1] != self.K or n > self.P or n % self.ms2 or pos.shape != (n, H) or rope.shape != (n, hd):
            raise ValueError("patches / position rows / rotary rows do not fit the program")
        p.top = self.scratch0
        keep = np.arange(npad) < n                                           # this image's mask rows
        for buf, row in ((self.mask, keep.astype(F32)), (self.mbias, np.where(keep, F32(0), MASK_NEG).astype(F32))):
            at = p.base + buf.off
            p.ddr[at:at + 4 * npad] = row.tobytes()
        x = self.x.rows_at(0, n)
        self._dense(p.constant(np.asarray(patches, F32)), self.pe, x)        # the patch embedding
        p.elt(C.ELT_ADD, x, p.constant(np.asarray(pos, F32)), x)             # + the position rows
        rot = p.constant(np.asarray(rope, F32))
        scores, probs = self.sc._replace(rows=n), self.prow._replace(rows=n)
        h, qkv, qd, kd, qr = (b.rows_at(0, n) for b in (self.h, self.qkv, self.qd, self.kd, self.qr))
        att, proj, ml = self.att.rows_at(0, n), self.b.rows_at(0, n), self.ml.rows_at(0, n)
        keys, vals = self.kbuf.rows_at(0, n), self.vbuf.rows_at(0, n)
        for blk in self.blocks:
            p.row_op(C.ROW_LAYERNORM, x, h, blk["n1"][0], self.eps, beta=blk["n1"][1])
            p.mm8(*self._int8(h), blk["qkv"], qkv)
            # q, k, v copied into dense matrices (one row stride for the rope and the head views)
            for c0, dst in ((0, qd), (H, kd), (2 * H, vals)):
                p.elt(C.ELT_ADD, qkv.cols_at(c0, H), self.zrow, dst, bmode=C.BM_ROW)
            p.rotary(qd.as_heads(hd), rot, nh, hd, qr.as_heads(hd))
            p.elt(C.ELT_MUL, qr, self.sc_q, qr, bmode=C.BM_SCALAR)
            p.rotary(kd.as_heads(hd), rot, nh, hd, keys.as_heads(hd))
            for head in range(nh):
                p.fdot(qr.column_of(head, hd), self.kbuf.column_of(head, hd), scores, nn=False)
                p.elt(C.ELT_MUL, scores, self.mask, scores, bmode=C.BM_ROW)      # padded columns: +0
                p.elt(C.ELT_ADD, scores, self.mbias, scores, bmode=C.BM_ROW)     # then MASK_NEG
                p.row_op(C.ROW_SOFTMAX, scores, probs)
                p.fdot(probs, self.vbuf.column_of(head, hd), att.column_of(head, hd), nn=True)
            self._dense(att, blk["proj"], proj)
            p.elt(C.ELT_ADD, x, proj, x)
            p.row_op(C.ROW_LAYERNORM, x, h, blk["n2"][0], self.eps, beta=blk["n2"][1])
            p.mm8(*self._int8(h), blk["fc1"], ml, C.ACT_GELU)
            self._dense(ml, blk["fc2"], proj)
            p.elt(C.ELT_ADD, x, proj, x)
        nm = n // self.ms2
        # the merger's norm per patch row, laid out so that a merge block's rows are one row
        p.row_op(C.ROW_LAYERNORM, x, Buf(self.mt.off, n, H, 4 * H), self.m_norm[0], self.eps, beta=self.m_norm[1])
        p.mm8(*self._int8(self.mt.rows_at(0, nm)), self.m_fc1, self.mm.rows_at(0, nm), C.ACT_GELU)
        out = self.out.rows_at(0, nm)
        self._dense(self.mm.rows_at(0, nm), self.m_fc2, out)
        if p.top > self.scratch_end:
            raise MemoryError("scratch_bytes too small for one image")
        p.top = self.end
        return out

    def emit(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray, blocks: int | None = None) -> Buf:
        """The image's descriptors (replacing any earlier image's); returns the output matrix: the
        merged tokens, or with `blocks` the patches' hidden state after that many blocks."""
        every = self.blocks
        if blocks is not None:
            self.blocks = every[:blocks]
        try:
            self.p.descs.clear()
            self.p.queue_off = None
            out = self._record(patches, pos, rope)
            return out if blocks is None else self.x.rows_at(0, patches.shape[0])
        finally:
            self.blocks = every

    def run(self, patches: np.ndarray, pos: np.ndarray, rope: np.ndarray, blocks: int | None = None,
            machine=None) -> np.ndarray:
        """Record the image, build the program and run it on `machine` (a Machine class; default the
        drop-in Machine): the visual tokens [P / merge^2, out_hidden]."""
        if machine is None:
            from .machine import Machine as machine
        out = self.emit(patches, pos, rope, blocks)
        ddr, q, cnt = self.p.finish()
        m = machine(bytearray(ddr))
        st = m.run_queue(q, cnt)
        if not st.done:
            raise RuntimeError(f"the tower's queue stopped: {st.err_code} at {st.op_idx}")
        return self.read(m, out)

    def read(self, m, v: Buf) -> np.ndarray:
        at = self.p.base + v.off
        return np.stack([np.frombuffer(m.read(at + r * v.ld, 4 * v.cols), "<f4") for r in range(v.rows)])
