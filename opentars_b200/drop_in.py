"""The B200 Machine swapped in for the reference's golden executor, in the reference's own process.

tars_mini runs every descriptor queue through `tars_mini.golden.Machine` (golden.py:41-492);
`tars_mini.compiler` imported that name at import time (compiler.py:24), and so does every test
module that says `from tars_mini.golden import Machine`. install() replaces the executor, its
status type and its ContractError in both modules with opentars_b200.machine's, so the
reference's lowering, compiler and tests run unchanged on the GPU. As a pytest plugin (it must be
loaded before the test modules import the name):

    TARS_REFERENCE_ROOT=<reference checkout> \
        python -m pytest -p opentars_b200.drop_in <reference>/tests/test_golden.py ...

TARS_EXECUTOR=golden leaves the reference's own executor in place (the same command then runs the
suite as the reference does).
"""
from __future__ import annotations

import os
import sys


def install() -> None:
    root = os.environ.get("TARS_REFERENCE_ROOT")
    if root and root not in sys.path:
        sys.path.insert(0, root)
    import tars_mini.compiler as compiler
    import tars_mini.golden as golden

    from . import machine
    golden.Machine, golden.ContractError, golden.Status = machine.Machine, machine.ContractError, machine.Status
    compiler.Machine, compiler.Status = machine.Machine, machine.Status


def pytest_configure(config) -> None:
    if os.environ.get("TARS_EXECUTOR", "cuda") == "cuda":
        install()
