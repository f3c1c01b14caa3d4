"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run in a container that holds the reference checkout (it is never needed at test time):

    PYTHONDONTWRITEBYTECODE=1 python -m tests.golden.make_fixtures --ref <path to openTARS> [--models]

What it stores (all small):
  queues.json.gz   per seeded program (tests/golden/cases.py): the reference golden Machine's
                   end status, ContractError flag, per-descriptor stats and the SHA-256 of the
                   whole DDR image after the run
  numerics.npz     seeded inputs' output bits from the reference's numerics.py functions
  vision.json      (--models) the small Qwen3.5 vision tower on the reference's VisionLowering and
                   golden Machine: built image, queue and output per test image
  mtp.json         (--models) Qwen3.5 with the MTP head: speculative decoding's queues, tokens,
                   verified logits and rounds on the reference's lowering and golden Machine
  models.json      (--models) per-step logits SHA-256 / argmax of the reference's QwenLowering
                   + golden Machine greedy decode for small Qwen3 / Gemma-3 configs, and the
                   SHA-256 of the lowered DDR image and queue bytes
  context.json     (--context) the whole 256-token context at the real head dims (Qwen3: 16 q /
                   8 kv heads of 128; Gemma 3: 4 q / 1 kv head of 256, 5 sliding layers to 1 full):
                   per prompt, every run's logits SHA-256 from the last prompt token to position 255
  gemm_sweep.json  (--gemm) config 1: the SHA-256 of every (M, shape) output of bench.py's GEMM
                   sweep image (bench.build_gemm, seed 1234) run on the reference golden Machine
"""
from __future__ import annotations

import argparse
import gzip
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden import cases  # noqa: E402

QUEUE_SETS = {
    # name: (first seed, count, kinds, descriptors per queue or None, corruption probability)
    "mixed": (0, 400, tuple(cases.GENS), None, 0.06),
    "gemm": (10000, 120, ("gemm",), 4, 0.0),
    "w4": (20000, 80, ("w4",), 3, 0.0),
    "row": (30000, 120, ("row",), 4, 0.0),
    "elt": (40000, 160, ("elt",), 4, 0.0),
    "rope": (50000, 60, ("rope",), 3, 0.0),
    "fdot": (60000, 80, ("fdot",), 3, 0.0),
    "relu": (70000, 60, ("relu",), 4, 0.0),
    "conv": (80000, 40, ("conv",), 2, 0.0),
    "errors": (90000, 120, tuple(cases.GENS), 3, 0.5),
}
CHAINS = (100000, 30)


def ref_modules(ref: str):
    sys.path.insert(0, ref)
    import tars_mini.golden as G
    import tars_mini.numerics as F
    return G, F


def run_ref_queue(G, ddr, qaddr, qlen, gemv_only=False):
    m = G.Machine(bytearray(ddr), gemv_only=gemv_only)
    try:
        st = m.run_queue(qaddr, qlen)
        status = [bool(st.done), int(st.err_code), int(st.op_idx)]
        cerr = False
    except G.ContractError:
        status, cerr = [bool(m.status.done), int(m.status.err_code), int(m.status.op_idx)], True
    stats = [[s.opcode, s.macs, s.bytes_read, s.bytes_written] for s in m.stats]
    return dict(status=status, contract_error=cerr, stats=stats,
                sha256=hashlib.sha256(bytes(m.ddr)).hexdigest())


def make_queues(G):
    out = {}
    for name, (s0, cnt, kinds, nd, pc) in QUEUE_SETS.items():
        rows = []
        for s in range(s0, s0 + cnt):
            ddr, qa, ql = cases.build_case(s, kinds, nd, pc)
            r = run_ref_queue(G, ddr, qa, ql)
            r.update(seed=s, qlen=ql)
            rows.append(r)
        out[name] = dict(kinds=list(kinds), n_desc=nd, p_corrupt=pc, cases=rows)
    s0, cnt = CHAINS
    rows = []
    for s in range(s0, s0 + cnt):
        ddr, qa, ql = cases.build_chain(s)
        r = run_ref_queue(G, ddr, qa, ql)
        r.update(seed=s, qlen=ql)
        rows.append(r)
    out["chains"] = dict(cases=rows)
    return out


def numerics_inputs(seed: int = 7, n: int = 1 << 11):
    """Float32 inputs covering the interesting ranges and every special value."""
    rng = np.random.default_rng(seed)
    parts = [
        rng.uniform(-110, 95, n).astype(np.float32),
        rng.normal(0, 3, n).astype(np.float32),
        (np.exp(rng.uniform(-87, 88, n)) * rng.choice([-1, 1], n)).astype(np.float32),
        rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32).view(np.float32),
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 89.0, -104.0, 88.99, -103.99,
                  20.0, 20.000002, 2.0 ** 126, 1.5 * 2.0 ** 126, 2.0 ** -126, 3.4e38, -3.4e38,
                  0.5, 1.5, 2.5, -0.5, 127.5, -127.5], np.float32),
    ]
    return np.concatenate(parts)


def make_numerics(F):
    x = numerics_inputs()
    res = {"x": x}
    for name in ("exp_f", "recip_f", "rsqrt_f", "gelu_f", "silu_f", "sigmoid_f", "softplus_f", "ftz", "fabs"):
        res[name] = getattr(F, name)(x).view(np.uint32)
    for act in range(8):
        res[f"act{act}"] = F.act_fn(x, act).view(np.uint32)
    res["bf16"] = F.to_bf16_bits(x)
    res["fp16"] = F.to_fp16_bits(x)
    res["from_fp16"] = F.from_fp16_bits(np.arange(1 << 16, dtype=np.uint16)).view(np.uint32)
    rng = np.random.default_rng(8)
    y = x[rng.permutation(x.size)]
    res["fmul"] = F.fmul(x, y).view(np.uint32)
    res["fadd"] = F.fadd(x, y).view(np.uint32)
    res["fmax"] = F.fmax(x, y).view(np.uint32)
    res["q8_inv"] = np.float32(rng.uniform(0.5, 50))
    res["q8"] = F.q8(x, res["q8_inv"]).astype(np.int8)
    # row functions on [64, 256] tiles (with a few special values and zero rows)
    xr = rng.normal(0, 2, (64, 256)).astype(np.float32)
    xr[3] = 0
    xr[5, 7] = np.nan
    xr[6, 9] = np.inf
    xr[7, :] *= np.float32(1e-39)
    res["rows_x"] = xr
    q, s = F.quant_rows(xr)
    res["quant_q"], res["quant_s"] = q, s.view(np.uint32)
    res["sum16"] = F.sum16(xr).view(np.uint32)
    res["max16"] = F.max16(xr).view(np.uint32)
    gam = rng.normal(1, 0.2, 256).astype(np.float32)
    bet = rng.normal(0, 0.2, 256).astype(np.float32)
    res["gamma"], res["beta"] = gam, bet
    res["rmsnorm"] = F.rmsnorm_rows(xr, gam, None, np.float32(1e-6)).view(np.uint32)
    res["layernorm"] = F.layernorm_rows(xr, gam, bet, np.float32(1e-5)).view(np.uint32)
    res["l2norm"] = F.l2norm_rows(xr, gam, None, np.float32(1e-6)).view(np.uint32)
    valid = rng.integers(1, 257, 64)
    res["valid"] = valid
    res["softmax_causal"] = F.softmax_rows_causal(xr, valid).view(np.uint32)
    res["softmax"] = F.softmax_rows(xr).view(np.uint32)
    b = rng.normal(0, 2, (32, 256)).astype(np.float32)
    res["fdot_b"] = b
    res["fdot_nt"] = F.fdot_nt(xr[:16], b).view(np.uint32)
    bn = rng.normal(0, 2, (256, 48)).astype(np.float32)
    res["fdot_bn"] = bn
    res["fdot_nn"] = F.fdot_nn(xr[:16], bn).view(np.uint32)
    tab = rng.uniform(-1, 1, (32, 128)).astype(np.float32)
    res["rope_tab"] = tab
    res["rope"] = F.rope_rows(xr, tab, 2, 128).view(np.uint32)
    xa = (rng.normal(0, 1, (8, 1024)) * (2.0 ** rng.integers(-40, 40, (8, 1024)))).astype(np.float32)
    xa[0, 5] = np.nan
    xa[1, 130] = np.inf
    xa[2, :128] = 0
    res["w4_x"] = xa
    aq, asc = F.align_w4_groups(xa)
    res["w4_q"], res["w4_s"] = aq, asc.view(np.uint32)
    return res


# ------------------------------------------------------------------------- model fixtures
MODEL_CASES = [
    # name, base config (opentars_b200.models name, or a tests.model_runs.DERIVED name), layer types,
    # vocab, max_tokens, prompt, new tokens, DeltaNet state dtype, weight bits (8: W8A8, 4: W4A16)
    ("qwen3_small", "CFG_Q3_SMALL", ["full_attention"] * 3, 4096, 32, [5, 77, 901, 12, 3000, 2, 9], 4, "fp32", 8),
    ("gemma3_small", "G3_SMALL_K2", ["sliding_attention", "full_attention", "sliding_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2], 4, "fp32", 8),
    ("qwen35_small", "CFG_Q35_SMALL", ["linear_attention", "full_attention", "linear_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2, 9], 4, "fp32", 8),
    ("qwen35_small_fp16", "CFG_Q35_SMALL", ["linear_attention", "full_attention", "linear_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2, 9], 4, "fp16", 8),
    ("gemma4_small", "CFG_G4_SMALL", ["sliding_attention", "full_attention", "sliding_attention", "full_attention"],
     4096, 32, [5, 77, 901, 12, 3000, 2], 4, "fp32", 8),
    ("qwen3_small_w4", "CFG_Q3_SMALL", ["full_attention"] * 3, 4096, 32, [5, 77, 901, 12, 3000, 2, 9], 4, "fp32", 4),
    ("gemma4_small_w4", "G4_SMALL_P256",
     ["sliding_attention", "full_attention", "sliding_attention", "full_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2], 4, "fp32", 4),
    ("gemma3_small_w4", "G3_SMALL_K2", ["sliding_attention", "full_attention", "sliding_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2], 4, "fp32", 4),
    ("qwen35_small_w4", "CFG_Q35_SMALL", ["linear_attention", "full_attention", "linear_attention"], 4096, 32,
     [5, 77, 901, 12, 3000, 2, 9], 4, "fp32", 4),
]
REF_BASE = {"CFG_Q35_SMALL": "CFG_SMALL"}     # the reference's name of a base config, where it differs


def gemma4_head_dims(cfg) -> None:
    """The reference's Gemma 4 lowering reads cfg.per_layer_config (per layer: head_dim and
    num_key_value_heads), a field of a newer transformers than the one installed here, whose
    Gemma4TextConfig carries head_dim (sliding layers) and global_head_dim (full layers) instead.
    Give the reference those same dims in that field."""
    from types import SimpleNamespace
    if getattr(cfg, "model_type", "") != "gemma4_text" or hasattr(cfg, "per_layer_config"):
        return
    cfg.per_layer_config = [SimpleNamespace(
        head_dim=cfg.global_head_dim if t == "full_attention" else cfg.head_dim,
        num_key_value_heads=cfg.num_key_value_heads) for t in cfg.layer_types]


def make_models(ref: str):
    import tars_mini.qwen_ref as Q
    from tars_mini import golden as G
    from tars_mini.llm import QwenLowering
    from tests.model_runs import base_config
    out = {}
    for name, base, types, vocab, T, prompt, new, state_dtype, wbits in MODEL_CASES:
        cfg = Q.make_config(base_config(Q, base, REF_BASE), types, vocab=vocab)
        gemma4_head_dims(cfg)
        w = Q.random_weights(cfg, seed=0, embed=True)
        low = QwenLowering(cfg, w, max_tokens=T, ddr_bytes=1 << 26, head=True, queue_cap=4096,
                           state_dtype=state_dtype, wbits=wbits)
        image_sha = hashlib.sha256(bytes(low.p.ddr)).hexdigest()
        queues = []

        def run(ddr, q, n):
            queues.append(hashlib.sha256(bytes(ddr[q:q + 64 * n])).hexdigest())
            m = G.Machine(ddr, gemv_only=True)
            assert m.run_queue(q, n).done
            return m.ddr
        ids, logits, counts = low.generate(run, prompt, new)
        out[name] = dict(base=base, types=types, vocab=vocab, T=T, prompt=prompt, new=new, state_dtype=state_dtype,
                         wbits=wbits, image_sha256=image_sha,
                         queue_sha256=queues, counts=counts, ids=ids,
                         logits_sha256=[hashlib.sha256(lg.astype("<f4").tobytes()).hexdigest() for lg in logits],
                         logits_head=[lg[:8].astype(np.float32).view(np.uint32).tolist() for lg in logits],
                         final_ddr_sha256=hashlib.sha256(bytes(low.p.ddr)).hexdigest())
    return out


# name, layer types, vocab, max_tokens, prompt, new tokens, DeltaNet state dtype
MTP_CASES = [
    ("qwen35_mtp", ["linear_attention"] * 3 + ["full_attention"], 4096, 48, [5, 77, 901, 12, 3000], 8, "fp32"),
    ("qwen35_mtp_fp16", ["linear_attention"] * 3 + ["full_attention"], 4096, 48, [5, 77, 901, 12, 3000], 8, "fp16"),
]
def make_mtp(ref: str):
    """Qwen3.5 with the MTP head on the reference's lowering and golden Machine: plain greedy decode,
    then greedy speculative decode with drafts forced to hit or miss (mtp_oracle); the queues, the
    tokens, every verified position's logits, the round count, and swap_state's queue."""
    import tars_mini.qwen_ref as Q
    from tars_mini import golden as G
    from tars_mini.llm import QwenLowering

    from tests.model_runs import mtp_oracle
    out = {}
    for name, types, vocab, T, prompt, new, state_dtype in MTP_CASES:
        cfg = Q.make_config(Q.CFG_SMALL, types, vocab=vocab)
        w = {**Q.random_weights(cfg, embed=True), **Q.random_mtp(cfg)}

        def mk(**k):
            return QwenLowering(cfg, w, max_tokens=T, ddr_bytes=1 << 25, head=True, queue_cap=8192,
                                state_dtype=state_dtype, **k)
        queues = []

        def run(ddr, q, n):
            queues.append(hashlib.sha256(bytes(ddr[q:q + 64 * n])).hexdigest())
            m = G.Machine(ddr)
            assert m.run_queue(q, n).done
            return m.ddr
        plain_ids, _, _ = mk().generate(run, prompt, new)
        queues.clear()
        low = mk(verify_rows=2, mtp=True)
        image_sha = hashlib.sha256(bytes(low.p.ddr)).hexdigest()
        ids, lg, rounds = low.generate_mtp(run, prompt, new, mtp_oracle(plain_ids, vocab))
        a = len(low.p.descs)
        low.swap_state()
        swap = b"".join(bytes(d) for d in low.p.descs[a:])
        out[name] = dict(types=types, vocab=vocab, T=T, prompt=prompt, new=new, state_dtype=state_dtype,
                         plain_ids=plain_ids, image_sha256=image_sha, queue_sha256=queues, ids=ids, rounds=rounds,
                         logits_sha256={str(k): hashlib.sha256(v.astype("<f4").tobytes()).hexdigest()
                                        for k, v in sorted(lg.items())},
                         swap_sha256=hashlib.sha256(swap).hexdigest())
    return out


VIT_SMALL = dict(depth=2, hidden_size=64, intermediate_size=256, num_heads=2, patch_size=4,
                 spatial_merge_size=2, temporal_patch_size=2, out_hidden_size=48, num_position_embeddings=36)
VIT_IMAGES = (8, 32, 64)             # sides: 4, 64 and 256 patches


def vit_image(size: int, seed: int = 3) -> np.ndarray:
    """A normalised test image [3, size, size]: smooth gradients plus noise."""
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.arange(size), np.arange(size), indexing="ij")
    base = (np.sin(xx / 3.0) + np.cos(yy / 5.0))[:, :, None] / 2.0 + rng.normal(0, 0.3, (size, size, 3))
    return np.ascontiguousarray(base.transpose(2, 0, 1), np.float32)


def make_vision(ref: str):
    """The small Qwen3.5 vision tower on the reference's VisionLowering and golden Machine, per test
    image: the built image and queue, the merged tokens and the hidden state after one block. The
    patches, position rows and rotary rows come from opentars_b200.vision (the reference's host
    helpers need a newer transformers than this one; tests/test_vision.py pins ours to the
    installed tower's own computations)."""
    from tars_mini import qwen_vit as RV

    from opentars_b200 import vision as OV
    cfg = RV.vision_config(**VIT_SMALL)
    w = RV.random_vision(cfg, seed=0)
    out = {}
    for size in VIT_IMAGES:
        px, grid = OV.patchify(vit_image(size), cfg)
        pos, rope = OV.position_embeddings(cfg, w, grid), OV.rope_table(cfg, grid)
        low = RV.VisionLowering(cfg, w, patches_max=len(px), ddr_bytes=1 << 23)
        one = low.run(px, pos, rope, blocks=1)
        tokens = low.run(px, pos, rope)
        ddr, q, n = low.p.build()
        out[str(size)] = dict(patches=len(px), host_sha256=hashlib.sha256(px.tobytes() + pos.tobytes()
                                                                          + rope.tobytes()).hexdigest(),
                              image_sha256=hashlib.sha256(bytes(ddr)).hexdigest(), queue=[q, n],
                              tokens_sha256=hashlib.sha256(tokens.astype("<f4").tobytes()).hexdigest(),
                              block1_sha256=hashlib.sha256(one.astype("<f4").tobytes()).hexdigest())
    return dict(config=VIT_SMALL, seed=0, images=out)


# name, base config, layer types (None: the model's own), prompt seed, new tokens, prefill chunk
FULL_CASES = [
    ("qwen3_0.6b", "CFG_Q3_06B", None, "VOCAB_Q3_06B", 0, 3, 4),
    ("gemma3_1b", "CFG_G3_1B", "LAYERS_G3_1B", "VOCAB_G3_1B", 0, 2, 4),
]


def prompt_ids(seed: int, vocab: int, n: int = 20) -> list[int]:
    """The seeded prompt of configs 3 / 4: n token ids uniform over the vocabulary."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def make_full_models(ref: str, only: str = ""):
    """Full-size models, one sequence: the prompt in prefill chunks of 4, then greedy decode. Each
    chunk is staged and run through the reference's golden Machine exactly as its generate()
    does, with the prompt split as the board runtime prefills it."""
    import tars_mini.qwen_ref as Q
    from tars_mini import golden as G
    from tars_mini.llm import QwenLowering
    out = {}
    for name, base, types, vocab_name, seed, new, chunk in FULL_CASES:
        if only and only != name:
            continue
        t = time.time()
        vocab = getattr(Q, vocab_name)
        cfg = Q.make_config(getattr(Q, base), list(getattr(Q, types)) if types else None, vocab=vocab)
        w = Q.random_weights(cfg, seed=0, embed=True)
        low = QwenLowering(cfg, w, max_tokens=256, ddr_bytes=3 << 29, head=True, queue_cap=8192)
        image_sha = hashlib.sha256(bytes(low.p.ddr)).hexdigest()
        build_s = time.time() - t
        prompt = prompt_ids(seed, vocab)
        ddr, ids, rec = low.p.ddr, list(prompt), []
        spans = [(s, min(chunk, len(prompt) - s)) for s in range(0, len(prompt), chunk)]
        for i in range(len(spans) + new):
            t0, n = spans[i] if i < len(spans) else (len(ids) - 1, 1)
            low.put_input(ddr, t0, low.embed(ids[t0:t0 + n]))
            a = len(low.p.descs)
            low.chunk(t0, n)
            q, cnt = low.stage(ddr, a, len(low.p.descs))
            qsha = hashlib.sha256(bytes(ddr[q:q + 64 * cnt])).hexdigest()
            ts = time.time()
            m = G.Machine(ddr)
            assert m.run_queue(q, cnt).done
            ddr = m.ddr
            r = dict(t0=t0, n=n, count=cnt, queue_sha256=qsha, golden_s=round(time.time() - ts, 2))
            if i >= len(spans) - 1:
                lg = low.logits_of(ddr)
                ids.append(int(np.argmax(lg)))
                r.update(logits_sha256=hashlib.sha256(lg.astype("<f4").tobytes()).hexdigest(),
                         logits_head=lg[:8].view(np.uint32).tolist(), argmax=ids[-1])
            rec.append(r)
            print(name, r, flush=True)
        out[name] = dict(base=base, types=types, vocab=vocab, T=256, prompt=prompt, chunk=chunk, new=new,
                         image_sha256=image_sha, ids=ids, runs=rec, build_s=round(build_s, 1))
    return out


# The whole context (max_tokens 256, positions 0 .. 255) at the real head dims: name, base config,
# layer types, vocab, prompt seeds (one run per prompt). Each prompt is fed one token per run (the
# prefill of a sequence that joins a running batch), then greedy decode up to position 255.
CONTEXT_CASES = [
    ("qwen3_hd128", "Q3_HD128", ["full_attention"] * 2, 4096, (1, 2)),
    ("gemma3_hd256", "G3_HD256", ["sliding_attention"] * 5 + ["full_attention"], 4096, (1, 2)),
]
CONTEXT_T, CONTEXT_PROMPT = 256, 20


def make_context(ref: str, only: str = ""):
    """Per case and prompt: the SHA-256 of the image, and for every run from the last prompt token
    on, its logits' SHA-256, first 8 logits and argmax (the next token)."""
    import tars_mini.qwen_ref as Q
    from tars_mini import golden as G
    from tars_mini.llm import QwenLowering
    from tests.model_runs import base_config
    out = {}
    for name, base, types, vocab, seeds in CONTEXT_CASES:
        if only and only != name:
            continue
        cfg = Q.make_config(base_config(Q, base, REF_BASE), types, vocab=vocab)
        w = Q.random_weights(cfg, seed=0, embed=True)
        runs = []
        for seed in seeds:
            t = time.time()
            low = QwenLowering(cfg, w, max_tokens=CONTEXT_T, ddr_bytes=1 << 26, head=True, queue_cap=4096)
            image_sha = hashlib.sha256(bytes(low.p.ddr)).hexdigest()
            prompt = prompt_ids(seed, vocab, CONTEXT_PROMPT)

            ddr, ids, logits = low.p.ddr, list(prompt), []
            for t0 in range(CONTEXT_T):              # one token per run, as generate() stages a chunk
                low.put_input(ddr, t0, low.embed(ids[t0:t0 + 1]))
                a = len(low.p.descs)
                low.chunk(t0, 1)
                q, cnt = low.stage(ddr, a, len(low.p.descs))
                m = G.Machine(ddr, gemv_only=True)
                assert m.run_queue(q, cnt).done
                ddr = m.ddr
                if t0 >= len(prompt) - 1:
                    lg = low.logits_of(ddr)
                    logits.append(lg)
                    if t0 + 1 < CONTEXT_T:
                        ids.append(int(np.argmax(lg)))
            runs.append(dict(seed=seed, prompt=prompt, ids=ids,
                             logits_sha256=[hashlib.sha256(lg.astype("<f4").tobytes()).hexdigest() for lg in logits],
                             logits_head=[lg[:8].view(np.uint32).tolist() for lg in logits]))
            print(name, seed, f"{time.time() - t:.1f}s", flush=True)
        out[name] = dict(base=base, types=types, vocab=vocab, T=CONTEXT_T, image_sha256=image_sha, runs=runs)
    return out


def make_gemm_sweep(G):
    import bench
    p = bench.build_gemm(1, 0)
    m = G.Machine(bytearray(p["ddr"].tobytes()))
    assert m.run_queue(p["q_setup"], p["n_setup"]).done
    assert m.run_queue(p["q_main"], p["n_main"]).done
    y0, yn = p["y_region"]
    region = np.frombuffer(bytes(m.ddr[y0:y0 + yn]), np.uint8)
    return dict(seed=1234, M=list(bench.GEMM_M), shapes=[list(s) for s in bench.GEMM_SHAPES],
                sha256=bench.gemm_hashes(bench.gemm_outputs(p, [region])))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OPENTARS_REF", ""), required=False)
    ap.add_argument("--models", action="store_true")
    ap.add_argument("--skip-queues", action="store_true")
    ap.add_argument("--full", default="", help="full-size models: 'all' or one name")
    ap.add_argument("--gemm", action="store_true", help="config 1's GEMM sweep")
    ap.add_argument("--context", default="", help="whole-context cases: 'all' or one name")
    a = ap.parse_args()
    if not a.ref:
        raise SystemExit("--ref <path to the openTARS checkout> is required")
    G, F = ref_modules(a.ref)
    t = time.time()
    if not a.skip_queues:
        q = make_queues(G)
        with gzip.open(HERE / "queues.json.gz", "wt") as f:
            json.dump(q, f)
        np.savez_compressed(HERE / "numerics.npz", **make_numerics(F))
        print(f"queues + numerics in {time.time() - t:.1f}s")
    if a.models:
        m = make_models(a.ref)
        (HERE / "models.json").write_text(json.dumps(m, indent=1))
        (HERE / "mtp.json").write_text(json.dumps(make_mtp(a.ref), indent=1))
        (HERE / "vision.json").write_text(json.dumps(make_vision(a.ref), indent=1))
        print(f"models in {time.time() - t:.1f}s")
    if a.full:
        path = HERE / "full_models.json"
        old = json.loads(path.read_text()) if path.exists() else {}
        old.update(make_full_models(a.ref, "" if a.full == "all" else a.full))
        path.write_text(json.dumps(old, indent=1))
        print(f"full models in {time.time() - t:.1f}s")
    if a.context:
        path = HERE / "context.json"
        old = json.loads(path.read_text()) if path.exists() else {}
        old.update(make_context(a.ref, "" if a.context == "all" else a.context))
        path.write_text(json.dumps(old))
        print(f"context cases in {time.time() - t:.1f}s")
    if a.gemm:
        (HERE / "gemm_sweep.json").write_text(json.dumps(make_gemm_sweep(G), indent=1))
        print(f"gemm sweep in {time.time() - t:.1f}s")


if __name__ == "__main__":
    main()
