"""Every spin-wait of the streaming kernels is bounded; one that gives up records a code in a device
word that tc_wait_error reads, and the kernel skips the rest of its work and returns.

On ordinary runs nothing is recorded. With the poll limit lowered to 0 (tc_set_spin_limit), every
wait for work gives up at once: the streamed W4A16 GEMV and the persistent tensor-core GEMM must
still return, report their code, leave the context usable, and the next ordinary run must be
clean and bit-exact with the CPU oracle. No fault and no hang is involved: the waits that let a
block's in-flight copies and MMAs finish before it exits keep their full limit."""
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


def _give_up_then_recover(program, codes):
    from opentars_b200._lib import lib
    from opentars_b200.machine import Machine
    from oracle.machine import OracleMachine
    L = lib()
    ddr, qa, n = program
    L.tc_wait_error(1)
    prev = L.tc_set_spin_limit(0)
    try:
        Machine(bytearray(ddr)).run_queue(qa, n)       # returns: the kernel gave up and ended
    finally:
        assert L.tc_set_spin_limit(prev) == 0
    code = L.tc_wait_error(0)
    assert code in codes, code
    assert L.tc_wait_error(1) == code                  # read and clear
    assert L.tc_wait_error(0) == 0
    # the context is still good: an ordinary run is clean and equals the oracle byte for byte
    m = Machine(bytearray(ddr))
    assert m.run_queue(qa, n).done
    o = OracleMachine(bytearray(ddr))
    assert o.run_queue(qa, n).done
    assert bytes(m.ddr) == bytes(o.ddr)
    assert L.tc_wait_error(0) == 0


def test_w4a16_stream_wait_gives_up_and_recovers():
    """The tiled W4A16 GEMV (producer code 13, consumer code 14, partial-sum hand-over 15)."""
    import __graft_entry__ as GE
    _give_up_then_recover(GE._w4_program(), (13, 14, 15))


def test_tensor_core_gemm_wait_gives_up_and_recovers():
    """The tcgen05 GEMM in its persistent mode (M = 32, N = 16384: 128 weight tiles, no cluster):
    producer 1, MMA issuer 2-3, epilogue 4."""
    import __graft_entry__ as GE
    _give_up_then_recover(GE._gemv_program(seed=3, M=32, K=1024, N=16384), (1, 2, 3, 4))


def test_spin_limit_setter_clamps_and_restores():
    from opentars_b200._lib import lib
    L = lib()
    prev = L.tc_set_spin_limit(1 << 30)                # above the maximum: clamped to 2^22
    try:
        assert L.tc_set_spin_limit(5) == 1 << 22
    finally:
        L.tc_set_spin_limit(prev)
