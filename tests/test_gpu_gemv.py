"""The decode GEMV kernels at config 0 / config 2 sizes against the CPU oracle, bit for bit.

W4A16 (config 2: M = 1, K in {4096, 8192}) runs the register-resident kernel; M = 2 the
shared-memory streaming kernel; M = 4 at K = 8192 the register-prefetch kernel. W8A8 (config 0:
M = 1, K = 1024, N = 3072) with its row quantisation."""
import numpy as np
import pytest

import bench
from oracle.machine import OracleMachine

pytestmark = pytest.mark.gpu


def _check(p, nunits=1):
    from opentars_b200.machine import Machine
    m = Machine(bytearray(p["ddr"].tobytes()))
    st = m.run_queue(p["qa"], p["qlen"])
    o = OracleMachine(bytearray(p["ddr"].tobytes()))
    so = o.run_queue(p["qa"], p["qlen"])
    assert (st.done, st.err_code) == (so.done, so.err_code)
    y0, yn = p["outputs"]
    assert bytes(m.ddr[y0:y0 + yn]) == bytes(o.ddr[y0:y0 + yn])


@pytest.mark.parametrize("M,K,N", [(1, 4096, 2048), (1, 8192, 2048), (1, 4096, 8192), (1, 8192, 16384),
                                   (2, 8192, 2048), (4, 8192, 1024), (3, 4096, 1040)])
def test_w4a16_gemv_matches_oracle(M, K, N):
    _check(bench.build_w4(1, 17 + K + N + M, M=M, K=K, N=N))


@pytest.mark.parametrize("units", [1, 3])
def test_w8a8_gemv_config0_matches_oracle(units):
    _check(bench.build_gemv(units, 29 + units))
