"""The drop-in plugin on CPU: install() puts the CUDA Machine, its Status and ContractError into the
reference's golden and compiler modules (checked by identity, in a fresh interpreter; no kernel
runs). Needs a reference checkout (TARS_REFERENCE_ROOT or baseline/_ref); skipped without one."""
import os
import subprocess
import sys

import pytest

from tests.test_reference_suite import ROOT, _reference_root


def test_install_swaps_the_executor_names():
    ref = _reference_root()
    if ref is None:
        pytest.skip("no reference checkout (TARS_REFERENCE_ROOT or baseline/_ref)")
    code = (
        "import tars_mini.golden as G, tars_mini.compiler as Cc\n"
        "gold = G.Machine\n"
        "from opentars_b200 import drop_in, machine as M\n"
        "drop_in.install()\n"
        "assert G.Machine is M.Machine and G.ContractError is M.ContractError and G.Status is M.Status\n"
        "assert Cc.Machine is M.Machine and Cc.Status is M.Status and gold is not M.Machine\n"
        "from tars_mini.golden import Machine\n"
        "assert Machine is M.Machine\n"
        "print('swapped')\n")
    env = dict(os.environ, TARS_REFERENCE_ROOT=str(ref),
               PYTHONPATH=os.pathsep.join([str(ROOT), str(ref), os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "swapped" in r.stdout, r.stderr[-2000:]
