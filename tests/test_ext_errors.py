"""Errors raised by the kernel extension's argument checks reach Python as exceptions.

A check whose message formats numbers must raise RuntimeError, not crash the process
(the failure mode of an extension that carries its own static copy of the C++ stream
library).  Runs in a child process so a crash cannot take the test session down.
"""

import subprocess
import sys

import pytest

_CHILD = r"""
import torch
import zstep_b200._C as C
t = torch.zeros(1, dtype=torch.int32)
try:
    C.ep_call(0, 0, 9, 0, 1, 512, 1, 8, 128, 128, t, t.float(), None, [0] * 9, [0] * 6, t, t, t, t, t, t, t, t,
              None, 0, None, None, None, 0)
except RuntimeError as e:
    print("RAISED", "bad world 9" in str(e))
"""


def test_numeric_check_message_raises_instead_of_crashing():
    pytest.importorskip("zstep_b200._C", reason="kernel extension not built")
    r = subprocess.run([sys.executable, "-c", _CHILD], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "RAISED True" in r.stdout
