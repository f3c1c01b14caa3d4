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
