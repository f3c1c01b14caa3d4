"""The CUDA Machine against the reference golden model's results (committed fixtures) and the CPU
oracle, bit for bit: whole DDR image, end status, ContractError, per-descriptor stats."""
import hashlib
import struct

import numpy as np
import pytest

from oracle import contract as C
from oracle import numerics as F
from oracle.machine import ContractError as OracleContractError
from oracle.machine import OracleMachine
from tests import fixtures as FX

pytestmark = pytest.mark.gpu


def _machine():
    from opentars_b200.machine import Machine
    return Machine


def run_cuda(ddr, qa, ql, **kw):
    from opentars_b200.machine import ContractError
    m = _machine()(ddr, **kw)
    try:
        st = m.run_queue(qa, ql)
        return m, [st.done, st.err_code, st.op_idx], False
    except ContractError:
        return m, [m.status.done, m.status.err_code, m.status.op_idx], True


def run_oracle(ddr, qa, ql, **kw):
    m = OracleMachine(ddr, **kw)
    try:
        st = m.run_queue(qa, ql)
        return m, [st.done, st.err_code, st.op_idx], False
    except OracleContractError:
        return m, [m.status.done, m.status.err_code, m.status.op_idx], True


def first_difference(a: bytes, b: bytes) -> str:
    x, y = np.frombuffer(a, np.uint8), np.frombuffer(b, np.uint8)
    idx = np.nonzero(x != y)[0]
    return "identical" if idx.size == 0 else f"{idx.size} bytes differ, first at {idx[0]:#x}"


@pytest.mark.parametrize("name", sorted(FX.queues()))
def test_reproduces_reference_fixtures(name):
    bad = []
    for case in FX.queues()[name]["cases"]:
        ddr, qa, ql = FX.build(name, case)
        m, status, cerr = run_cuda(bytearray(ddr), qa, ql)
        got = ([bool(status[0]), status[1], status[2]], cerr,
               [[s.opcode, s.macs, s.bytes_read, s.bytes_written] for s in m.stats],
               hashlib.sha256(bytes(m.ddr)).hexdigest())
        want = (case["status"], case["contract_error"], case["stats"], case["sha256"])
        if got != want:
            om, _, _ = run_oracle(bytearray(ddr), qa, ql)
            bad.append((case["seed"], got[:2], want[:2], first_difference(bytes(m.ddr), bytes(om.ddr))))
    assert not bad, bad[:5]


@pytest.mark.parametrize("kind", ["gemm", "w4", "row", "elt", "rope", "fdot", "relu", "conv"])
def test_matches_oracle_on_fresh_programs(kind):
    from tests.golden import cases
    for seed in range(500000 + 1000 * len(kind), 500000 + 1000 * len(kind) + 25):
        ddr, qa, ql = cases.build_case(seed, (kind,), 4, 0.0)
        m, s1, c1 = run_cuda(bytearray(ddr), qa, ql)
        o, s2, c2 = run_oracle(bytearray(ddr), qa, ql)
        assert (s1, c1) == (s2, c2), seed
        assert bytes(m.ddr) == bytes(o.ddr), (seed, first_difference(bytes(m.ddr), bytes(o.ddr)))


# ------------------------------------------------------------------ behaviour (test_golden.py:69-168)
def _base():
    ddr = bytearray(1 << 14)
    ddr[0x100:0x110] = bytes(range(16))
    ddr[0x200:0x300] = bytes([1]) * 256
    ddr[0x400:0x404] = struct.pack("<f", 1.0)
    good = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_GEMM, CTRL=C.ctrl(C.QM_TENSOR), EPI=C.epi(),
                A_OFF=0x100, W_OFF=0x200, Y_OFF=0x800, SCALE_OFF=0x400, M=1, N=16, K=16, VALID=1)
    return ddr, good


def _run(ddr, *descs):
    mem = bytearray(ddr)
    for i, r in enumerate(descs):
        mem[0x2000 + 64 * i:0x2000 + 64 * (i + 1)] = r
    m = _machine()(mem)
    return m.run_queue(0x2000, len(descs)), m


@pytest.mark.parametrize("code,change", [
    (C.E_MAGIC, {"MAGIC": 0x55AA}), (C.E_VERSION, {"VERSION": 1}), (C.E_VALID, {"VALID": 0}),
    (C.E_OPCODE, {"OPCODE": 0x0F}), (C.E_FIELD, {"CORE_ID": 1}), (C.E_FIELD, {"HDR_RSV": 1}),
    (C.E_FIELD, {"DEP_SIG": 1}), (C.E_FIELD, {"GROUP_SIZE": 128}), (C.E_FIELD, {"CTRL": C.ctrl(C.QM_NONE)}),
    (C.E_FIELD, {"CTRL": C.ctrl(C.QM_TENSOR, a_dtype=C.DT_BF16)}), (C.E_FIELD, {"CTRL": C.ctrl(C.QM_TENSOR, fusion=1)}),
    (C.E_FIELD, {"EPI": C.epi(C.ACT_RELU)}), (C.E_FIELD, {"OUT_SCALE": 1}), (C.E_ALIGN, {"N": 8}),
    (C.E_ALIGN, {"K": 24}), (C.E_ALIGN, {"M": 0}), (C.E_ALIGN, {"A_OFF": 0x108}), (C.E_RANGE, {"Y_OFF": 0x3FF0}),
    (C.E_RANGE, {"BASE_ADDR": 1 << 40}), (C.E_RANGE, {"BASE_ADDR": (1 << 64) - 0x100})])
def test_error_codes_write_nothing(code, change):
    ddr, good = _base()
    st, m = _run(ddr, C.encode({**good, **change}))
    assert (st.done, st.err_code, st.op_idx) == (False, code, 0)
    assert m.ddr[:0x2000] == ddr[:0x2000]


def test_crc_error_and_priority():
    ddr, good = _base()
    assert _run(ddr, C.encode(good, fix_crc=False))[0].err_code == C.E_CRC
    assert _run(ddr, C.encode({**good, "CORE_ID": 1, "N": 8}))[0].err_code == C.E_FIELD


def test_queue_stops_and_keeps_earlier_writes():
    ddr, good = _base()
    st, m = _run(ddr, C.encode(good), C.encode({**good, "MAGIC": 0}), C.encode({**good, "Y_OFF": 0xC00}))
    assert (st.err_code, st.op_idx) == (C.E_MAGIC, 1)
    assert m.read(0x800, 64) != bytes(64) and m.read(0xC00, 64) == bytes(64)


def test_overlap_refused_after_earlier_writes():
    from opentars_b200.machine import ContractError
    ddr, good = _base()
    mem = bytearray(ddr)
    mem[0x2000:0x2040] = C.encode({**good, "Y_OFF": 0xC00})
    mem[0x2040:0x2080] = C.encode({**good, "Y_OFF": 0x200})
    m = _machine()(mem)
    with pytest.raises(ContractError):
        m.run_queue(0x2000, 2)
    assert m.read(0xC00, 64) != bytes(64) and len(m.stats) == 1


def test_sequential_raw_war_waw():
    ddr, good = _base()
    relu = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_RELU, M=1, N=16, VALID=1)
    descs = [C.encode(good),
             C.encode({**relu, "EPI": C.epi(C.ACT_RELU), "A_OFF": 0x800, "Y_OFF": 0xA00}),
             C.encode({**relu, "EPI": C.epi(C.ACT_RELU, C.OUT_BF16), "A_OFF": 0xA00, "Y_OFF": 0x100}),
             C.encode(good)]
    st, m = _run(ddr, *descs)
    assert st.done and st.op_idx == 4
    y0 = np.full(16, np.arange(16).sum(), np.float32)
    assert np.array_equal(np.frombuffer(m.read(0xA00, 64), "<f4"), y0)
    bf = F.to_bf16_bits(y0).astype("<u2").tobytes()
    assert m.read(0x100, 32) == bf
    a3 = np.frombuffer(bf[:16], np.int8).astype(np.int64)
    assert np.array_equal(np.frombuffer(m.read(0x800, 64), "<f4"), np.full(16, a3.sum(), np.float32))


@pytest.mark.parametrize("act", [C.ACT_RELU, C.ACT_RELU6, C.ACT_GELU, C.ACT_SILU, C.ACT_SIGMOID, C.ACT_SOFTPLUS])
@pytest.mark.parametrize("out", [C.OUT_FP32, C.OUT_BF16, C.OUT_INT8])
def test_fusion_equivalence(act, out):
    """GEMM(fused act, out) == GEMM(fp32) then RELU-op(act, out), byte for byte."""
    for seed in range(3):
        rng = np.random.default_rng(seed)
        Mm, Nn, Kk = int(rng.integers(1, 9)), 16 * int(rng.integers(1, 4)), 16 * int(rng.integers(1, 5))
        ddr = bytearray(1 << 16)
        ddr[0x100:0x100 + Mm * Kk] = rng.integers(-128, 128, Mm * Kk, dtype=np.int8).tobytes()
        ddr[0x1000:0x1000 + Nn * Kk] = rng.integers(-128, 128, Nn * Kk, dtype=np.int8).tobytes()
        ddr[0x3000:0x3000 + 4 * Nn] = rng.uniform(1e-4, 1e-2, Nn).astype("<f4").tobytes()
        ddr[0x3400:0x3400 + 4 * Nn] = rng.uniform(-6, 6, Nn).astype("<f4").tobytes()
        inv = C.f32_bits(float(rng.uniform(1, 40))) if out == C.OUT_INT8 else 0
        common = dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_GEMM, A_OFF=0x100, W_OFF=0x1000,
                      SCALE_OFF=0x3000, BIAS_OFF=0x3400, M=Mm, N=Nn, K=Kk, VALID=1)
        descs = [C.encode({**common, "CTRL": C.ctrl(C.QM_CHANNEL, fusion=1), "EPI": C.epi(act, out, 1),
                           "Y_OFF": 0x4000, "OUT_SCALE": inv}),
                 C.encode({**common, "CTRL": C.ctrl(C.QM_CHANNEL), "EPI": C.epi(C.ACT_NONE, C.OUT_FP32, 1),
                           "Y_OFF": 0x6000}),
                 C.encode(dict(MAGIC=C.MAGIC, VERSION=C.VERSION, OPCODE=C.OP_RELU, EPI=C.epi(act, out),
                               A_OFF=0x6000, Y_OFF=0x8000, M=Mm, N=Nn, VALID=1, OUT_SCALE=inv))]
        for i, r in enumerate(descs):
            ddr[0xA000 + 64 * i:0xA000 + 64 * (i + 1)] = r
        m = _machine()(ddr)
        assert m.run_queue(0xA000, 3).done
        nb = Mm * Nn * C.ESIZE[out]
        assert m.read(0x4000, nb) == m.read(0x8000, nb)


@pytest.mark.parametrize("base", [0, 4, 1, 1 << 20, 3 + (1 << 16)])
def test_result_independent_of_base_address(base):
    """The same program at another BASE_ADDR (unaligned ones included) gives the same bytes."""
    from tests.golden import cases
    for seed in range(600000, 600012):
        ddr, qa, ql = cases.build_case(seed, tuple(cases.GENS), 3, 0.0)
        o, so, co = run_oracle(bytearray(ddr), qa, ql)
        big = bytearray(base + len(ddr) + 64 * 8)
        big[base:base + len(ddr)] = ddr
        q2 = base + len(ddr)
        for j in range(ql):
            d = C.decode(bytes(ddr[qa + 64 * j:qa + 64 * (j + 1)]))
            d["BASE_ADDR"] = base
            d.pop("CRC32")
            big[q2 + 64 * j:q2 + 64 * (j + 1)] = C.encode(d)
            # ROWCOL's row scales sit at BASE + 16 HDR_RSV: they move with the base
        m, s, c = run_cuda(big, q2, ql)
        assert (s, c) == (so, co), seed
        assert bytes(m.ddr[base:base + qa]) == bytes(o.ddr[:qa]), seed


def test_host_writes_between_runs_are_seen():
    ddr, good = _base()
    mem = bytearray(ddr)
    mem[0x2000:0x2040] = C.encode(good)
    m1 = _machine()(mem)
    assert m1.run_queue(0x2000, 1).done
    y1 = m1.read(0x800, 64)
    mem[0x100:0x110] = bytes([3]) * 16                   # the host rewrites the input in place
    m2 = _machine()(mem)
    assert m2.run_queue(0x2000, 1).done
    assert m2.read(0x800, 64) != y1
    assert np.array_equal(np.frombuffer(m2.read(0x800, 64), "<f4"), np.full(16, 48.0, np.float32))


def test_descriptor_rewriting_a_later_descriptor():
    """A queue whose first descriptor (RELU, int8 out) writes over the second descriptor's bytes:
    the second is read after the first ran, as the golden model reads each descriptor in turn."""
    from tests.golden import cases
    for seed in range(700000, 700010):
        ddr, qa, ql = cases.build_case(seed, ("relu",), 2, 0.0)
        d = C.decode(bytes(ddr[qa:qa + 64]))
        d.pop("CRC32")
        d.update(Y_OFF=qa + 64, LDY16=0)
        ddr[qa:qa + 64] = C.encode(d)
        m, s1, c1 = run_cuda(bytearray(ddr), qa, ql)
        o, s2, c2 = run_oracle(bytearray(ddr), qa, ql)
        assert (s1, c1) == (s2, c2)
        assert bytes(m.ddr) == bytes(o.ddr)


def test_gemv_only_profile():
    ddr, good = _base()
    mem = bytearray(ddr)
    mem[0x2000:0x2040] = C.encode({**good, "K": 4112})
    assert _machine()(bytearray(mem), gemv_only=True).run_queue(0x2000, 1).err_code == C.E_OPCODE
