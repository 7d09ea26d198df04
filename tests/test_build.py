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
