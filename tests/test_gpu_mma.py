"""The tensor-core W8A8 GEMM (tcgen05, int8 MMA) against the CPU oracle, bit for bit.

Descriptor path: config 1's shapes (prefill GEMM sweep) and edge shapes - M not a multiple of 16
and above one 256-row token tile, N not a multiple of the 128-row weight tile, K below and not a
multiple of the 128-byte K slice, padded row strides - with every quant mode, bias, activation and
output format (fp16 output is ELT-only in the contract). Engine path: the small models decoded with the tensor-core kernel taking every
GEMM of two or more rows (split-K clusters, gated and K-split epilogues).
"""
import numpy as np
import pytest

from oracle import contract as C
from oracle.machine import OracleMachine
from tests.test_gpu_machine import first_difference

pytestmark = pytest.mark.gpu


@pytest.fixture
def mma_min_rows():
    """Sets the tensor-core row threshold for one test and restores it afterwards."""
    from opentars_b200._lib import lib
    prev = []

    def set_rows(n):
        prev.append(lib().tc_set_mma_min_rows(n))

    yield set_rows
    if prev:
        lib().tc_set_mma_min_rows(prev[0])


def _align(x, a=128):
    return -(-x // a) * a


def gemm_image(seed, M, N, K, qm, act, out, bias, pad):
    """One GEMM descriptor over a fresh image: int8 A [M, K] (row stride K + 16 pad), W [N, K],
    fp32 scales uniform in [1e-3, 1e-2] (config 0's distribution), optional bias and row scales."""
    rng = np.random.default_rng(seed)
    lda = K + 16 * pad
    es = C.ESIZE[out]
    ldy = N * es + 16 * pad
    a_off = 0x100
    w_off = _align(a_off + lda * M)
    s_off = _align(w_off + N * K)
    b_off = _align(s_off + 4 * N)
    r_off = _align(b_off + 4 * N)
    y_off = _align(r_off + 4 * M)
    q_off = _align(y_off + ldy * M)
    ddr = bytearray(_align(q_off + 64, 4096))
    for m in range(M):
        ddr[a_off + m * lda:a_off + m * lda + K] = rng.integers(-127, 128, K, dtype=np.int8).tobytes()
    ddr[w_off:w_off + N * K] = rng.integers(-127, 128, N * K, dtype=np.int8).tobytes()
    ns = 1 if qm == C.QM_TENSOR else N
    ddr[s_off:s_off + 4 * ns] = rng.uniform(1e-3, 1e-2, ns).astype("<f4").tobytes()
    f = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1, OPCODE=C.OP_GEMM,
             CTRL=C.ctrl(qm, fusion=int(act != 0)), EPI=C.epi(act, out, int(bias)),
             A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, Y_OFF=y_off, M=M, N=N, K=K,
             LDA16=0 if lda == K else lda // 16, LDY16=0 if ldy == N * es else ldy // 16)
    if bias:
        ddr[b_off:b_off + 4 * N] = rng.normal(0, 4, N).astype("<f4").tobytes()
        f["BIAS_OFF"] = b_off
    if qm == C.QM_ROWCOL:
        ddr[r_off:r_off + 4 * M] = rng.uniform(1e-3, 5e-2, M).astype("<f4").tobytes()
        f["HDR_RSV"] = r_off // 16
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    ddr[q_off:q_off + 64] = C.encode(f)
    return ddr, q_off


SHAPES = [  # (M, N, K, pad)
    (16, 3072, 1024, 0), (64, 1024, 3072, 0), (256, 3072, 1024, 0), (4, 1152, 2816, 0),   # config 1
    (300, 1152, 4096, 1),      # two token tiles, the last one ragged
    (17, 208, 48, 1),          # K below one slice, N not a multiple of the weight tile
    (33, 144, 1040, 0),        # ragged N and K
    (2, 16, 16, 0), (5, 272, 144, 1),
]
MODES = [  # (qm, act, out, bias)
    (C.QM_ROWCOL, C.ACT_NONE, C.OUT_FP32, False), (C.QM_CHANNEL, C.ACT_SILU, C.OUT_BF16, True),
    (C.QM_TENSOR, C.ACT_GELU, C.OUT_INT8, True), (C.QM_ROWCOL, C.ACT_RELU, C.OUT_FP32, False),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_mma_gemm_matches_oracle(shape, mma_min_rows):
    from opentars_b200.machine import Machine
    mma_min_rows(2)
    M, N, K, pad = shape
    for i, mode in enumerate(MODES):
        ddr, qa = gemm_image(1000 * M + N + K + i, M, N, K, *mode, pad)
        m = Machine(bytearray(ddr))
        st = m.run_queue(qa, 1)
        o = OracleMachine(bytearray(ddr))
        so = o.run_queue(qa, 1)
        assert (st.done, st.err_code) == (so.done, so.err_code)
        assert bytes(m.ddr) == bytes(o.ddr), (mode, first_difference(bytes(m.ddr), bytes(o.ddr)))


def test_mma_and_cuda_core_kernels_agree(mma_min_rows):
    """The same GEMM on both kernels (threshold above and below M) gives the same bytes."""
    from opentars_b200.machine import Machine
    ddr, qa = gemm_image(7, 48, 640, 768, C.QM_ROWCOL, C.ACT_SILU, C.OUT_FP32, True, 0)
    outs = []
    for rows in (2, 1 << 20):
        mma_min_rows(rows)
        m = Machine(bytearray(ddr))
        m.run_queue(qa, 1)
        outs.append(bytes(m.ddr))
    assert outs[0] == outs[1]


@pytest.mark.parametrize("batch", [3, 20])
def test_engine_on_tensor_cores_matches_oracle(batch, mma_min_rows):
    """Every engine GEMM of two or more rows on the tensor cores; each sequence equals its own
    single-sequence oracle run."""
    from opentars_b200.engine import DecodeEngine
    from tests import fixtures as FX
    from tests.model_runs import build_image, machine_runner
    mma_min_rows(2)
    for name, fx in sorted(FX.engine_models().items()):
        rng = np.random.default_rng(3)
        P = len(fx["prompt"])
        prompts = [fx["prompt"]] + [list(map(int, rng.integers(0, fx["vocab"], P))) for _ in range(batch - 1)]
        eng = DecodeEngine(build_image(fx), batch=batch)
        ids, logits = eng.generate(prompts, 2, chunk=4)
        eng.close()
        for b in (0, batch - 1):
            low = build_image(fx)
            oids, ologits, _ = low.generate(machine_runner(OracleMachine, []), prompts[b], 2, chunk=4)
            assert ids[b] == oids, (name, b)
            assert all(np.array_equal(lg[b].view(np.uint32), ol.view(np.uint32))
                       for lg, ol in zip(logits, ologits)), (name, b)


def test_gemm_sweep_matches_reference():
    """Config 1 (bench.py --workload gemm): every (M, shape) output of the whole sweep, run through
    the board runtime on the GPU, against the reference golden Machine's hashes."""
    import json

    import bench
    from opentars_b200.board import Cuda
    from tests import fixtures as FX
    want = json.loads((FX.GOLDEN / "gemm_sweep.json").read_text())["sha256"]
    p = bench.build_gemm(1, 0)
    dev = Cuda(len(p["ddr"]))
    dev.mem[:] = p["ddr"]
    dev.to_dev(0, len(p["ddr"]))
    assert dev.run(p["q_setup"], p["n_setup"])[0]
    assert dev.run(p["q_main"], p["n_main"])[0]
    y0, yn = p["y_region"]
    dev.from_dev(y0, yn)
    got = bench.gemm_hashes(bench.gemm_outputs(p, [dev.mem[y0:y0 + yn]]))
    dev.close()
    assert got == want, [k for k in got if got[k] != want[k]]
