"""The compiled extensions import on a machine without a GPU (every exported symbol
resolves) and expose the kernel entry points the runners call."""

import importlib.util

import pytest
import torch  # noqa: F401  (loads libc10 / libtorch for the extension)


def test_kernel_extension_exports():
    if importlib.util.find_spec("zstep_b200._C") is None:
        pytest.skip("extension not built")
    from zstep_b200 import _C

    for name in ("gemm_mxf8", "quant_mxf8", "add_rmsnorm_quant", "gdn_decode", "gdn_prefill", "attn_decode",
                 "moe_route", "fused_allreduce_norm", "mhc_partial", "mhc_finalize", "rms_quant", "mla_prologue",
                 "mla_absorb_q", "mla_attn", "mla_up", "dsa_index", "gather_sum"):
        assert hasattr(_C, name), name
    assert _C.mhc_slices(4096) == 8


def test_bench_reference_arm_prints_one_json_line():
    """The benchmark's reference arm (`bench.py --impl reference`) exits 0 with one JSON line
    naming the arm, here the reason the reference cannot run on B200."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference"], capture_output=True,
                       text=True, timeout=300, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and ("unavailable" in rec or "value" in rec)
