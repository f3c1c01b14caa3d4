"""The CPU oracle against the reference's own results (the committed golden fixtures) and the
reference tests' known answers. These pin the oracle before any GPU result is judged by it."""
import hashlib
import struct

import numpy as np
import pytest

from oracle import contract as C
from oracle import numerics as F
from oracle.machine import ContractError, OracleMachine
from tests import fixtures as FX

F32 = np.float32


def run_oracle(ddr, qa, ql):
    m = OracleMachine(bytearray(ddr))
    try:
        st = m.run_queue(qa, ql)
        status, cerr = [st.done, st.err_code, st.op_idx], False
    except ContractError:
        status, cerr = [m.status.done, m.status.err_code, m.status.op_idx], True
    return m, status, cerr


@pytest.mark.parametrize("name", sorted(FX.queues()))
def test_oracle_reproduces_reference_queues(name):
    for case in FX.queues()[name]["cases"]:
        ddr, qa, ql = FX.build(name, case)
        assert ql == case["qlen"]
        m, status, cerr = run_oracle(ddr, qa, ql)
        assert (status, cerr) == (case["status"], case["contract_error"]), case["seed"]
        assert [[s.opcode, s.macs, s.bytes_read, s.bytes_written] for s in m.stats] == case["stats"]
        assert hashlib.sha256(bytes(m.ddr)).hexdigest() == case["sha256"], case["seed"]


def test_oracle_numerics_bits():
    z = FX.numerics()
    x = z["x"]
    for name in ("exp_f", "recip_f", "rsqrt_f", "gelu_f", "silu_f", "sigmoid_f", "softplus_f", "ftz", "fabs"):
        assert np.array_equal(getattr(F, name)(x).view(np.uint32), z[name]), name
    for act in range(8):
        assert np.array_equal(F.act_fn(x, act).view(np.uint32), z[f"act{act}"]), act
    assert np.array_equal(F.to_bf16_bits(x), z["bf16"])
    assert np.array_equal(F.to_fp16_bits(x), z["fp16"])
    assert np.array_equal(F.from_fp16_bits(np.arange(1 << 16, dtype=np.uint16)).view(np.uint32), z["from_fp16"])
    rng = np.random.default_rng(8)
    y = x[rng.permutation(x.size)]
    for name in ("fmul", "fadd", "fmax"):
        assert np.array_equal(getattr(F, name)(x, y).view(np.uint32), z[name]), name
    assert np.array_equal(F.q8(x, z["q8_inv"]), z["q8"])
    xr = z["rows_x"]
    q, s = F.quant_rows(xr)
    assert np.array_equal(q, z["quant_q"]) and np.array_equal(s.view(np.uint32), z["quant_s"])
    assert np.array_equal(F.sum16(xr).view(np.uint32), z["sum16"])
    assert np.array_equal(F.max16(xr).view(np.uint32), z["max16"])
    g, b = z["gamma"], z["beta"]
    assert np.array_equal(F.rmsnorm_rows(xr, g, None, F32(1e-6)).view(np.uint32), z["rmsnorm"])
    assert np.array_equal(F.layernorm_rows(xr, g, b, F32(1e-5)).view(np.uint32), z["layernorm"])
    assert np.array_equal(F.l2norm_rows(xr, g, None, F32(1e-6)).view(np.uint32), z["l2norm"])
    assert np.array_equal(F.softmax_rows_causal(xr, z["valid"]).view(np.uint32), z["softmax_causal"])
    assert np.array_equal(F.softmax_rows(xr).view(np.uint32), z["softmax"])
    assert np.array_equal(F.fdot_nt(xr[:16], z["fdot_b"]).view(np.uint32), z["fdot_nt"])
    assert np.array_equal(F.fdot_nn(xr[:16], z["fdot_bn"]).view(np.uint32), z["fdot_nn"])
    assert np.array_equal(F.rope_rows(xr, z["rope_tab"], 2, 128).view(np.uint32), z["rope"])
    aq, asc = F.align_w4_groups(z["w4_x"])
    assert np.array_equal(aq, z["w4_q"]) and np.array_equal(asc.view(np.uint32), z["w4_s"])


# ------------------------------------------------------------------ the reference tests' known answers
DOC_FUSED_DESC = bytes.fromhex(
    "000000807FC4843700000000000020001000020000070000000600000010000000020000000100"
    "000000000000000000150000001A11020000000000020055AA")


def test_worked_example_known_answers():
    """test_contract.py:53-90: the contract document's fused GEMM example."""
    rng = np.random.default_rng(2026)
    M, N, K = 2, 16, 32
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    W = rng.integers(-128, 128, (N, K), dtype=np.int8)
    S = (rng.uniform(0.5, 2.0, N) / 4096).astype(F32)
    B = rng.uniform(-8, 8, N).astype(F32)
    ddr = bytearray(1 << 16)
    ddr[0x100:0x100 + M * K] = A.tobytes()
    ddr[0x200:0x200 + N * K] = W.tobytes()
    ddr[0x600:0x600 + 4 * N] = S.astype("<f4").tobytes()
    ddr[0x700:0x700 + 4 * N] = B.astype("<f4").tobytes()
    raw = C.encode(dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_GEMM, A_OFF=0x100, W_OFF=0x200,
                        SCALE_OFF=0x600, BIAS_OFF=0x700, Y_OFF=0x1000, M=M, N=N, K=K, VALID=1,
                        CTRL=C.ctrl(C.QM_CHANNEL, fusion=1), EPI=C.epi(C.ACT_RELU, C.OUT_BF16, bias=1)))
    assert raw == DOC_FUSED_DESC
    d = C.decode(raw)
    assert (d["CRC32"], d["CTRL"], d["EPI"]) == (0x3784C47F, 0x111A, 0x0015)
    ddr[0x8000:0x8040] = raw
    m = OracleMachine(ddr)
    assert m.run_queue(0x8000, 1).done
    assert struct.unpack("<H", m.read(0x1002, 2))[0] == 0x3F16
    acc = int(A[0].astype(np.int64) @ W[1].astype(np.int64))
    assert acc == -11968
    v = F.fadd(F.fmul(F.i2f(acc), S[1:2]), B[1:2])
    assert C.f32_bits(float(v[0])) == 0x3F15EC68


def test_numerics_known_answers():
    """test_golden.py:16-66 and 308-331, test_w4a16.py:47-67, test_v04.py:48-54."""
    r = F.act_fn(np.array([-0.0, 0.0, -1.0, np.nan, 2.5], F32), C.ACT_RELU)
    assert r.view(np.uint32).tolist() == [0, 0, 0, 0, C.f32_bits(2.5)]
    cases = {0x3F808000: 0x3F80, 0x3F818000: 0x3F82, 0x3F808001: 0x3F81, 0x7F7FFFFF: 0x7F80, 0x7FC12345: 0x7FC0}
    assert F.to_bf16_bits(np.array(list(cases), np.uint32).view(F32)).tolist() == list(cases.values())
    assert F.q8(np.array([0.5, 1.5, 2.5, -0.5, 200.0, -200.0, np.nan], F32), F32(1)).tolist() == [0, 2, 2, 0, 127, -127, 0]
    assert F.i2f(16777217)[()] == F32(16777216) and F.i2f(16777219)[()] == F32(16777220)
    assert F.fmul(np.array([1e-20], F32), np.array([1e-20], F32))[0] == 0
    p2 = np.ldexp(1.0, np.arange(-125, 126)).astype(F32)
    assert (F.recip_f(p2) == (1 / p2.astype(np.float64)).astype(F32)).all()
    assert F.exp_f(np.array([0.0], F32))[0] == 1 and F.rsqrt_f(np.array([4.0], F32))[0] == 0.5
    e = F.exp_f(np.array([np.inf, -np.inf, np.nan, 89.0, -104.0], F32))
    assert e[0] == np.inf and e[1] == 0 and np.isnan(e[2]) and e[3] == np.inf and e[4] == 0
    x = np.zeros((4, 128), F32)
    x[0, :4] = [1.0, -1.0, 0.5, -0.5]
    x[1, :8] = [2 ** 100, -(2 ** 100), 2 ** 90, -(2 ** 90), 1.0, -1.0, 2 ** 80, -(2 ** 80)]
    x[2, :2] = [2 ** -120, -(2 ** -125)]
    x[3, :2] = [3.0, -3.0]
    q, s = F.align_w4_groups(x)
    assert s[0, 0] == F32(2 ** -13) and q[0, 0] == 8192 and q[0, 3] == -4096
    assert s[1, 0] == F32(2 ** 87) and q[1, 0] == 8192 and q[1, 2] == 8 and q[1, 4] == 0
    assert s[2, 0] == F32(2 ** -126) and q[2, 0] == 64 and q[2, 1] == -2
    assert s[3, 0] == F32(2 ** -12) and q[3, 0] == 12288
    xq = np.array([[1, -2, 0.5] + [0] * 13, [0] * 16, [127, -127.5] + [3] * 14], F32)
    qq, ss = F.quant_rows(xq)
    assert (qq[1] == 0).all() and ss[1] == 0 and qq[0, 1] == -127 and ss[0] == F.fmul(F32(2), F.INV127)


def test_oracle_error_priority_and_overlap():
    """test_golden.py:92-143 - error codes in priority order, nothing written, ContractError."""
    ddr = bytearray(1 << 14)
    ddr[0x100:0x110] = bytes(range(16))
    ddr[0x200:0x300] = bytes([1]) * 256
    ddr[0x400:0x404] = struct.pack("<f", 1.0)
    good = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_TENSOR), EPI=C.epi(),
                A_OFF=0x100, W_OFF=0x200, Y_OFF=0x800, SCALE_OFF=0x400, M=1, N=16, K=16, VALID=1)
    for code, change in [(C.E_MAGIC, {"MAGIC": 0x55AA}), (C.E_FIELD, {"CORE_ID": 1, "N": 8}),
                         (C.E_ALIGN, {"N": 8}), (C.E_RANGE, {"BASE_ADDR": 1 << 40})]:
        mem = bytearray(ddr)
        mem[0x2000:0x2040] = C.encode({**good, **change})
        st = OracleMachine(mem).run_queue(0x2000, 1)
        assert (st.done, st.err_code, st.op_idx) == (False, code, 0) and mem[:0x2000] == ddr[:0x2000]
    mem = bytearray(ddr)
    mem[0x2000:0x2040] = C.encode({**good, "Y_OFF": 0x200})
    with pytest.raises(ContractError):
        OracleMachine(mem).run_queue(0x2000, 1)


def test_oracle_reproduces_reference_gemm_sweep_small_m():
    """Config 1's sweep image (bench.build_gemm) at M = 4 and 16 through the oracle: the same
    output hashes as the reference golden Machine's run of the full sweep."""
    import json

    import bench
    from oracle.machine import OracleMachine
    want = json.loads((FX.GOLDEN / "gemm_sweep.json").read_text())["sha256"]
    p = bench.build_gemm(1, 0, ms=(4, 16))
    o = OracleMachine(bytearray(p["ddr"].tobytes()))
    assert o.run_queue(p["q_setup"], p["n_setup"]).done
    assert o.run_queue(p["q_main"], p["n_main"]).done
    y0, yn = p["y_region"]
    got = bench.gemm_hashes(bench.gemm_outputs(p, [np.frombuffer(bytes(o.ddr[y0:y0 + yn]), np.uint8)]))
    assert got == {k: want[k] for k in got}
