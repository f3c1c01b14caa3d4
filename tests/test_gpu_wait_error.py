"""Every spin-wait of the streaming kernels is bounded; one that gives up records a code in a device
word that tc_wait_error reads. On ordinary runs nothing is recorded: after the tensor-core GEMM,
the streamed W4A16 GEMV (drop-in Machine) and the grouped GEMV (the board backend's level-captured
graph) have run, the word still reads 0."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_no_bounded_wait_gives_up_on_ordinary_runs():
    import __graft_entry__ as GE
    from opentars_b200._lib import lib
    from opentars_b200.board import Cuda
    from opentars_b200.machine import Machine
    from tests.test_gpu_board import _level_program
    L = lib()
    assert L.tc_wait_error(1) >= 0                    # readable; start from a clear word
    for ddr, qa, n in (GE._gemv_program(seed=2, M=32), GE._w4_program()):
        assert Machine(bytearray(ddr)).run_queue(qa, n).done
    ddr, qa, n = _level_program(1)
    dev = Cuda(len(ddr))
    dev.mem[:] = np.frombuffer(bytes(ddr), np.uint8)
    dev.to_dev(0, len(ddr))
    assert dev.run(qa, n)[0]
    dev.close()
    assert L.tc_wait_error(0) == 0
