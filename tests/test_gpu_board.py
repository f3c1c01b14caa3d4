"""The board-runtime backend (opentars_b200.board.Cuda: mem / to_dev / from_dev / run) and the
captured-queue replay against the reference fixtures: same status, same bytes, run after run."""
import hashlib

import numpy as np
import pytest

from tests import fixtures as FX

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["mixed", "chains", "elt", "w4"])
def test_board_backend_reproduces_fixtures(name):
    from opentars_b200.board import Cuda
    from opentars_b200.machine import ContractError
    for case in FX.queues()[name]["cases"][:60]:
        ddr, qa, ql = FX.build(name, case)
        for replay in (False, True):
            dev = Cuda(len(ddr), graphs=replay)
            dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
            dev.to_dev(0, len(ddr))
            try:
                done, err, op, _ = dev.run(qa, ql)
                cerr = False
            except ContractError:
                done, err, op, cerr = False, 0, 0, True
            dev.from_dev(0, len(ddr))
            assert cerr == case["contract_error"], case["seed"]
            if not cerr:
                assert [done, err, op] == case["status"], case["seed"]
                assert hashlib.sha256(dev.mem.tobytes()).hexdigest() == case["sha256"], (case["seed"], replay)
            dev.close()


def test_graph_replay_is_idempotent_and_sees_new_inputs():
    """A captured queue replayed with new host inputs gives the oracle's result for those inputs."""
    from __graft_entry__ import _gemv_program
    from opentars_b200.board import Cuda
    from oracle.machine import OracleMachine
    ddr, qa, n = _gemv_program(seed=3, M=2)
    dev = Cuda(len(ddr), pinned=True)
    dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
    dev.to_dev(0, len(ddr))
    rng = np.random.default_rng(0)
    for step in range(4):
        x = rng.normal(0, 1, 2 * 1024).astype("<f4")
        dev.mem[0x1000:0x1000 + x.nbytes] = x.view(np.uint8)
        ddr[0x1000:0x1000 + x.nbytes] = x.tobytes()
        dev.to_dev(0x1000, x.nbytes)
        assert dev.run(qa, n)[0]
        dev.from_dev(0x40000, 2 * 4 * 3072)
        o = OracleMachine(bytearray(ddr))
        assert o.run_queue(qa, n).done
        assert dev.mem[0x40000:0x40000 + 2 * 4 * 3072].tobytes() == bytes(o.ddr[0x40000:0x40000 + 2 * 4 * 3072])
    assert len(dev._cache) == 1
    dev.close()


def test_captured_queue_reports_per_descriptor_times():
    import ctypes

    from __graft_entry__ import _gemv_program
    from opentars_b200._lib import Status_t, lib
    from opentars_b200.board import Cuda
    ddr, qa, n = _gemv_program(seed=4)
    dev = Cuda(len(ddr))
    dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
    dev.to_dev(0, len(ddr))
    L = lib()
    st, cop, g = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
    assert L.tc_queue_capture(dev.h, qa, n, 0, 0, 1, ctypes.byref(st), ctypes.byref(cop), ctypes.byref(g)) == 0
    assert st.done and st.op_idx == n
    assert L.tc_graph_launch(g, None) == 0 and L.tc_synchronize(dev.h) == 0
    ms = (ctypes.c_float * n)()
    assert L.tc_graph_times(g, ms, n) == n
    assert all(0 < ms[i] < 100 for i in range(n))
    L.tc_graph_destroy(g)
    dev.close()


def _level_program(seed):
    """Quant -> GEMV units of several GEMV kernel classes (M 1..8, K 1024..3072, N 96..3072; every
    quant mode, bias, activations, fp32 / bf16 / int8 outputs), then a softmax over each fp32 GEMV
    output: three dependency levels, the GEMVs of one class and the row ops of one level batched
    into one launch each."""
    from oracle import contract as C
    rng = np.random.default_rng(seed)
    units = [  # (M, K, N, quant mode, activation, output, bias)
        (1, 1024, 3072, C.QM_ROWCOL, C.ACT_NONE, C.OUT_FP32, False),
        (1, 1024, 640, C.QM_CHANNEL, C.ACT_SILU, C.OUT_FP32, True),
        (1, 512, 208, C.QM_TENSOR, C.ACT_GELU, C.OUT_BF16, True),
        (3, 3072, 1024, C.QM_ROWCOL, C.ACT_RELU, C.OUT_FP32, True),
        (3, 3072, 512, C.QM_ROWCOL, C.ACT_NONE, C.OUT_INT8, False),
        (8, 2048, 256, C.QM_ROWCOL, C.ACT_NONE, C.OUT_FP32, False),
        (2, 1024, 96, C.QM_CHANNEL, C.ACT_NONE, C.OUT_FP32, False),
    ]

    def align(x, a=128):
        return -(-x // a) * a
    off = 0x1000
    lay = []
    for M, K, N, *_ in units:
        x = off; q = align(x + 4 * M * K); sr = align(q + M * K); w = align(sr + 4 * M)
        s = align(w + N * K); b = align(s + 4 * N); y = align(b + 4 * N); z = align(y + 4 * M * N)
        off = align(z + 4 * M * N)
        lay.append((x, q, sr, w, s, b, y, z))
    qa = off
    ddr = bytearray(align(qa + 64 * 3 * len(units) + 4096, 4096))
    descs = []
    base = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1)
    for (M, K, N, qm, act, out, bias), (x, q, sr, w, s, b, y, z) in zip(units, lay):
        ddr[x:x + 4 * M * K] = rng.normal(0, 1, M * K).astype("<f4").tobytes()
        ddr[w:w + N * K] = rng.integers(-127, 128, N * K, dtype=np.int8).tobytes()
        ns = 1 if qm == C.QM_TENSOR else N
        ddr[s:s + 4 * ns] = rng.uniform(1e-3, 1e-2, ns).astype("<f4").tobytes()
        ddr[b:b + 4 * N] = rng.normal(0, 4, N).astype("<f4").tobytes()
        descs.append(C.encode(dict(base, OPCODE=C.OP_ROW, CTRL=C.ROW_QUANT, EPI=C.epi(C.ACT_NONE, C.OUT_INT8),
                                   A_OFF=x, Y_OFF=q, SCALE_OFF=sr, M=M, N=K)))
        f = dict(base, OPCODE=C.OP_GEMM, CTRL=C.ctrl(qm, fusion=int(act != 0)), EPI=C.epi(act, out, int(bias)),
                 A_OFF=q, W_OFF=w, SCALE_OFF=s, Y_OFF=y, M=M, N=N, K=K)
        if qm == C.QM_ROWCOL:
            f["HDR_RSV"] = sr // 16
        if bias:
            f["BIAS_OFF"] = b
        if out == C.OUT_INT8:
            f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
        descs.append(C.encode(f))
        if out == C.OUT_FP32:
            descs.append(C.encode(dict(base, OPCODE=C.OP_ROW, CTRL=C.ROW_SOFTMAX, EPI=C.epi(), A_OFF=y, Y_OFF=z,
                                       M=M, N=N)))
    # queue order interleaves the levels (unit by unit), as a lowering would emit them
    for i, d in enumerate(descs):
        ddr[qa + 64 * i:qa + 64 * (i + 1)] = d
    return ddr, qa, len(descs)


def test_level_capture_batches_and_matches_oracle():
    """The captured graph (levels, batched GEMV and row-op launches) writes the in-order oracle's
    bytes; it launches 6 kernels for 19 descriptors (one row-op launch per level; the GEMVs as a
    3-entry and a 2-entry group and two single launches); the per-level capture gives 3 times."""
    import ctypes

    from opentars_b200._lib import Status_t, lib
    from opentars_b200.board import Cuda
    from oracle.machine import OracleMachine
    L = lib()
    for seed in (1, 2):
        ddr, qa, n = _level_program(seed)
        o = OracleMachine(bytearray(ddr))
        assert o.run_queue(qa, n).done
        dev = Cuda(len(ddr))
        dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
        dev.to_dev(0, len(ddr))
        for _ in range(2):                               # a replay writes the same bytes again
            assert dev.run(qa, n)[0]
            dev.from_dev(0, len(ddr))
            assert dev.mem.tobytes() == bytes(o.ddr)
        g, st = dev.graph(qa, n)
        assert st.done and L.tc_graph_kernels(g) == 6
        st2, cop, gt = Status_t(), ctypes.c_int32(-1), ctypes.c_void_p()
        assert L.tc_queue_capture(dev.h, qa, n, 0, 0, 2, ctypes.byref(st2), ctypes.byref(cop), ctypes.byref(gt)) == 0
        assert L.tc_graph_launch(gt, None) == 0 and L.tc_synchronize(dev.h) == 0
        ms = (ctypes.c_float * n)()
        assert L.tc_graph_times(gt, ms, n) == 3 and all(0 < ms[i] < 100 for i in range(3))
        L.tc_graph_destroy(gt)
        dev.close()


def _w4_level_program(seed):
    """Ten independent W4A16 GEMVs (M 1 - 4, K 256 - 2048; more than one level's scratch slices, so
    two spill into the next level) and two that read earlier outputs as their activations."""
    from oracle import contract as C
    rng = np.random.default_rng(seed)
    shapes = [(1, 1024, 640), (2, 512, 384), (3, 2048, 256), (4, 256, 512), (1, 2048, 1024), (2, 1024, 512),
              (1, 256, 208), (4, 1024, 96), (3, 512, 320), (1, 1024, 64)]

    def align(x, a=128):
        return -(-x // a) * a
    off, lay = 0x1000, []
    for M, K, N in shapes:
        x = off; w = align(x + 4 * M * K); s = align(w + N * K // 2); y = align(s + 2 * N * (K // 128))
        off = align(y + 4 * M * N)
        lay.append((x, w, s, y))
    # two chained GEMVs: unit 4's output (M 1, N 1024) and unit 5's (M 2, N 512) as activations
    chain = []
    for src, N in ((4, 256), (5, 192)):
        M, K = shapes[src][0], shapes[src][2]
        w = off; s = align(w + N * K // 2); y = align(s + 2 * N * (K // 128)); off = align(y + 4 * M * N)
        chain.append((lay[src][3], M, K, N, w, s, y))
    qa = off
    ddr = bytearray(align(qa + 64 * 16 + 4096, 4096))
    base = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, VALID=1)
    ctrl = C.ctrl(C.QM_GROUP, a_dtype=C.DT_FP32, w_dtype=C.DT_INT4)
    descs = []
    for (M, K, N), (x, w, s, y) in zip(shapes, lay):
        ddr[x:x + 4 * M * K] = rng.normal(0, 1, M * K).astype("<f4").tobytes()
        ddr[w:w + N * K // 2] = rng.integers(0, 256, N * K // 2, dtype=np.uint8).tobytes()
        ddr[s:s + 2 * N * (K // 128)] = rng.uniform(1e-3, 2e-2, N * (K // 128)).astype("<f2").tobytes()
        descs.append(C.encode(dict(base, OPCODE=C.OP_GEMM, CTRL=ctrl, EPI=C.epi(), A_OFF=x, W_OFF=w, SCALE_OFF=s,
                                   Y_OFF=y, M=M, N=N, K=K, GROUP_SIZE=128)))
    for x, M, K, N, w, s, y in chain:
        ddr[w:w + N * K // 2] = rng.integers(0, 256, N * K // 2, dtype=np.uint8).tobytes()
        ddr[s:s + 2 * N * (K // 128)] = rng.uniform(1e-3, 2e-2, N * (K // 128)).astype("<f2").tobytes()
        descs.append(C.encode(dict(base, OPCODE=C.OP_GEMM, CTRL=ctrl, EPI=C.epi(), A_OFF=x, W_OFF=w, SCALE_OFF=s,
                                   Y_OFF=y, M=M, N=N, K=K, GROUP_SIZE=128)))
    for i, d in enumerate(descs):
        ddr[qa + 64 * i:qa + 64 * (i + 1)] = d
    return ddr, qa, len(descs)


def test_w4_gemvs_of_a_level_run_side_by_side():
    """Independent W4A16 GEMVs share a capture level (each aligns its rows into its own scratch
    slice, eight per level, the rest in the next level) and the graph writes the in-order oracle's
    bytes, replay after replay; the two GEMVs that read earlier outputs still see them."""
    from opentars_b200.board import Cuda
    from oracle.machine import OracleMachine
    for seed in (3, 4):
        ddr, qa, n = _w4_level_program(seed)
        o = OracleMachine(bytearray(ddr))
        assert o.run_queue(qa, n).done
        dev = Cuda(len(ddr))
        dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
        dev.to_dev(0, len(ddr))
        for _ in range(3):
            assert dev.run(qa, n)[0]
            dev.from_dev(0, len(ddr))
            assert dev.mem.tobytes() == bytes(o.ddr), seed
        dev.close()
