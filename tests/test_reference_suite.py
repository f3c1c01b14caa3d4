"""The reference's own test suite with the CUDA Machine swapped in for its golden executor.

Runs tests/test_golden.py, test_w4a16.py, test_compiler.py and test_v04.py of a reference checkout
in a separate pytest process with the opentars_b200.drop_in plugin (every queue the reference's
tests build - contract checks, special values, the compiler's GEMM chains, W4A16, the v0.4 ops and
the model blocks against transformers - then executes on the B200). The checkout is taken from
TARS_REFERENCE_ROOT, else baseline/_ref (the reference's package, tests and examples placed there
by hand: it has no installer); without one the test is skipped. Every collected reference test
must pass; the counts are printed.
"""
import os
import subprocess
import sys
import xml.etree.ElementTree as ET
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
FILES = ("test_golden.py", "test_w4a16.py", "test_compiler.py", "test_v04.py")


def _reference_root() -> Path | None:
    env = os.environ.get("TARS_REFERENCE_ROOT")
    for cand in ([Path(env)] if env else []) + [ROOT / "baseline" / "_ref"]:
        if (cand / "tars_mini" / "golden.py").is_file() and all((cand / "tests" / f).is_file() for f in FILES):
            return cand
    return None


def _run(ref: Path, executor: str, report: Path) -> tuple[dict, set, str]:
    env = dict(os.environ, TARS_REFERENCE_ROOT=str(ref), TARS_EXECUTOR=executor,
               PYTHONPATH=os.pathsep.join([str(ROOT), str(ref), os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "opentars_b200.drop_in", "-p", "no:cacheprovider",
                        f"--junitxml={report}", *[str(ref / "tests" / f) for f in FILES]],
                       cwd=ref, env=env, capture_output=True, text=True, timeout=3600)
    assert r.returncode in (0, 1), r.stdout[-3000:] + r.stderr[-3000:]
    suite = ET.parse(report).getroot()
    suite = suite if suite.tag == "testsuite" else suite.find("testsuite")
    counts = {k: int(suite.get(k, 0)) for k in ("tests", "failures", "errors", "skipped")}
    failed = {f"{c.get('classname')}::{c.get('name')}" for c in suite.iter("testcase")
              if c.find("failure") is not None or c.find("error") is not None}
    return counts, failed, r.stdout[-4000:]


def test_reference_suite_outcomes_on_the_cuda_machine_equal_the_golden_executors(tmp_path):
    """Outcome parity: the reference's tests that pass with its own golden executor pass with the
    CUDA Machine, and no other test fails. (A few fail in this image with the golden executor as
    well - the reference's lowering asserts on some configs and its Gemma 4 blocks differ from this
    transformers version; those must fail the same way, not pass by accident.)"""
    ref = _reference_root()
    if ref is None:
        pytest.skip("no reference checkout (TARS_REFERENCE_ROOT or baseline/_ref)")
    gold, gold_failed, _ = _run(ref, "golden", tmp_path / "golden.xml")
    cuda, cuda_failed, out = _run(ref, "cuda", tmp_path / "cuda.xml")
    print("reference suite, golden executor:", gold, "CUDA Machine:", cuda)
    assert cuda["tests"] == gold["tests"] > 0
    assert cuda_failed == gold_failed, (sorted(cuda_failed - gold_failed)[:20], sorted(gold_failed - cuda_failed)[:20],
                                        out)
