"""The decode GEMV kernels at config 0 / config 2 sizes against the CPU oracle, bit for bit.

W4A16 (config 2: M = 1, K in {4096, 8192}) and fresh descriptors with K a multiple of 1024 run the
shared-memory streaming kernel (M <= 4 when its ring fits), the rest the register-prefetch kernel;
the random descriptor programs of test_gpu_machine.py add bf16 activations and K = 256..768.
W8A8 (config 0: M = 1, K = 1024, N = 3072) with its row quantisation."""
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


def _w4_case(seed):
    """One W4A16 descriptor with fp32 activations, K a multiple of 1024 (1024-3072), N a multiple of
    16, M <= 4: special values and wide exponent ranges inside a group, an all-zero group, bias,
    every activation and output format, padded row strides."""
    from oracle import contract as C
    from tests.golden import cases as G
    rng = np.random.default_rng(seed)
    ddr, qa = bytearray(1 << 21), 0x1F0000

    class Bump:                                                   # 16-byte aligned rows, 2 MiB image
        top = 0x100

        def alloc(self, n, align=16):
            off = -(-self.top // align) * align
            self.top = off + n
            assert self.top <= qa
            return off

        def put(self, data, align=16):
            off = self.alloc(len(data), align)
            ddr[off:off + len(data)] = data
            return off

        def rows(self, m, rowbytes, extra16=0):
            return self.alloc((rowbytes + 16 * extra16) * m), rowbytes + 16 * extra16
    h = Bump()
    M, N, K = int(rng.integers(1, 5)), 16 * int(rng.integers(1, 6)), 1024 * int(rng.integers(1, 4))
    act, out, bias = int(rng.integers(0, 8)), int(rng.choice([C.OUT_FP32, C.OUT_BF16, C.OUT_INT8])), seed % 2
    a_off, lda = h.rows(M, 4 * K, int(rng.integers(0, 2)))
    x = G._special_f32(rng, (M, K), 2.0, 0.002 if seed % 3 else 0.0)
    if seed % 4 == 1:
        with np.errstate(over="ignore"):
            x *= (2.0 ** rng.integers(-30, 30, (M, K))).astype(np.float32)
    if seed % 5 == 2:
        x[:, 128:256] = 0.0                                       # an all-zero group
    for m in range(M):
        ddr[a_off + m * lda:a_off + m * lda + 4 * K] = x[m].astype("<f4").tobytes()
    w_off = h.put(rng.integers(0, 256, N * K // 2, dtype=np.uint8).tobytes(), align=128)
    ws = rng.uniform(1e-3, 2e-2, (N, K // 128)).astype(np.float16).view(np.uint16)
    s_off = h.put(ws.astype("<u2").tobytes())
    f = G._base(OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_GROUP, a_dtype=C.DT_FP32, w_dtype=C.DT_INT4, fusion=int(act != 0)),
                EPI=C.epi(act, out, bias), A_OFF=a_off, W_OFF=w_off, SCALE_OFF=s_off, M=M, N=N, K=K,
                GROUP_SIZE=128, LDA16=G._ld16(lda, 4 * K))
    if bias:
        f["BIAS_OFF"] = h.put(rng.normal(0, 1, N).astype("<f4").tobytes())
    if out == C.OUT_INT8:
        f["OUT_SCALE"] = C.f32_bits(float(rng.uniform(0.5, 40)))
    y_off, ldy = h.rows(M, N * C.ESIZE[out], int(rng.integers(0, 2)))
    f.update(Y_OFF=y_off, LDY16=G._ld16(ldy, N * C.ESIZE[out]))
    ddr[qa:qa + 64] = C.encode(f)
    return ddr, qa


def test_w4a16_matches_oracle_on_fresh_descriptors():
    from opentars_b200.machine import Machine
    for seed in range(700, 724):
        ddr, qa = _w4_case(seed)
        m = Machine(bytearray(ddr))
        st = m.run_queue(qa, 1)
        o = OracleMachine(bytearray(ddr))
        so = o.run_queue(qa, 1)
        assert (st.done, st.err_code) == (so.done, so.err_code) == (1, 0), seed
        assert bytes(m.ddr) == bytes(o.ddr), seed
