"""libtarscuda's host-side logic on the CPU (no device calls): the library loads and exports every
entry point include/tarscuda.h declares; its descriptor validator and footprints agree with the
oracle's restatement of golden.py on the fixture programs and on fuzzed descriptors."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import contract as OC
from oracle import machine as OM
from tests import fixtures as FX

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def L():
    from opentars_b200 import build
    build.build()
    from opentars_b200._lib import lib
    return lib()


def test_library_exports_every_declared_symbol(L):
    header = (ROOT / "include" / "tarscuda.h").read_text()
    declared = set(re.findall(r"\b(tc_[a-z_0-9]+)\s*\(", header))
    assert len(declared) >= 14
    from opentars_b200._lib import SIGNATURES
    assert declared == set(SIGNATURES), declared ^ set(SIGNATURES)
    for name in declared:
        assert hasattr(L, name), name
    assert L.tc_version() == 1


def test_library_exports_every_engine_symbol(L):
    """include/tarscuda_engine.h: the decode engine's entry points and the greedy pick."""
    header = (ROOT / "include" / "tarscuda_engine.h").read_text()
    declared = set(re.findall(r"\b(tc_[a-z_0-9]+)\s*\(", header))
    from opentars_b200.engine import ENGINE_SIGNATURES
    assert declared == set(ENGINE_SIGNATURES), declared ^ set(ENGINE_SIGNATURES)
    for name in declared:
        assert hasattr(L, name), name


def test_pick_rejects_bad_arguments_before_any_device_call(L):
    from opentars_b200.engine import lib as engine_lib
    E = engine_lib()
    buf = ctypes.c_void_p(16)                      # never dereferenced: the checks come first
    assert E.tc_argmax(None, 16, 1, buf, None) == -2
    assert E.tc_argmax(buf, 16, 1, None, None) == -2
    assert E.tc_argmax(buf, 0, 1, buf, None) == -2
    assert E.tc_argmax(buf, 16, 0, buf, None) == -2
    assert E.tc_argmax(buf, 16, (1 << 24) + 1, buf, None) == -2


def test_engine_create_rejects_missing_arguments_before_any_device_call(L):
    from opentars_b200.engine import lib as engine_lib
    E = engine_lib()
    out = ctypes.c_void_p(7)
    assert E.tc_engine_create(None, None, None, None, 1, None) == -2
    assert E.tc_engine_create(None, None, None, None, 1, ctypes.byref(out)) == -2
    assert out.value is None                      # the handle is cleared on every error


def _validate(L, raw, core_id=0, gemv_only=0):
    f = (ctypes.c_uint64 * 23)()
    err = L.tc_validate(bytes(raw), core_id, gemv_only, f)
    return err, dict(zip(OC.FIELDS, (int(v) for v in f)))


def _fuzzed(seed, n):
    """Descriptors from the case generators with random field rewrites."""
    from tests.golden import cases
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        ddr, qa, ql = cases.build_case(int(rng.integers(0, 1 << 30)), n_desc=2, p_corrupt=0.0)
        for j in range(ql):
            raw = bytes(ddr[qa + 64 * j:qa + 64 * (j + 1)])
            d = OC.decode(raw)
            for _ in range(int(rng.integers(0, 3))):
                name = list(OC.FIELDS)[int(rng.integers(0, len(OC.FIELDS)))]
                if name == "CRC32":
                    continue
                hi, lo = OC.FIELDS[name]
                w = hi - lo + 1
                d[name] = int(rng.choice([0, 1, 16, 128, int(rng.integers(0, 1 << min(w, 62)))])) & ((1 << w) - 1)
            out.append(OC.encode({k: v for k, v in d.items() if k != "CRC32"}, fix_crc=rng.random() < 0.97))
    return out


def test_validate_matches_oracle_on_fuzzed_descriptors(L):
    for raw in _fuzzed(1, 300):
        for core, gemv in ((0, 0), (0, 1), (1, 0)):
            err, fields = _validate(L, raw, core, gemv)
            d = OC.decode(raw)
            assert fields == d
            assert err == OM.check(d, raw, core, gemv), (d, err)


def test_validate_matches_oracle_on_fixture_programs(L):
    for name, case in FX.queue_params()[::7]:
        ddr, qa, ql = FX.build(name, case)
        for j in range(ql):
            raw = bytes(ddr[qa + 64 * j:qa + 64 * (j + 1)])
            assert _validate(L, raw)[0] == OM.check(OC.decode(raw), raw, 0, False)


def test_footprints_match_oracle_segments(L):
    from opentars_b200.machine import Machine
    n = 0
    for raw in _fuzzed(2, 200):
        d = OC.decode(raw)
        if OM.check(d, raw, 0, False) != OC.E_OK:
            continue
        reads, y = OM.segments(d)
        r2, y2 = Machine.segments(d)
        assert (r2, y2) == (reads, y)
        assert Machine.extra_out(d) == OM.extra_out(d)
        n += 1
    assert n > 50


def test_huge_base_address_footprint_does_not_wrap(L):
    from opentars_b200.machine import Machine
    d = OC.decode(OC.encode(dict(MAGIC=OC.MAGIC, VERSION=OC.VERSION, VALID=1, OPCODE=OC.OP_GEMM,
                                 CTRL=OC.ctrl(OC.QM_TENSOR), BASE_ADDR=(1 << 64) - 16, A_OFF=0x100,
                                 W_OFF=0x200, Y_OFF=0x800, SCALE_OFF=0x400, M=1, N=16, K=16)))
    assert Machine.segments(d) == OM.segments(d)
    assert Machine.segments(d)[1][0][0] > (1 << 64)
