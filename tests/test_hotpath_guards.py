"""Static guard on the step hot path: the methods that run inside a decode / verify CUDA
graph (or on every eager step) must not synchronise with the host.  A `.item()`, `.cpu()`,
`.tolist()`, `.numpy()`, `torch.cuda.synchronize()` or a `dist.barrier/broadcast` there
either breaks graph capture or stalls every step, and such a call slips in easily when
debugging.  The guard parses the sources (no GPU, no import of the extension)."""

import ast
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

HOT = {
    "zstep_b200/models/qwen35.py": {
        "Qwen35Runner": ["_gemm", "_proj_out", "_row_parallel_reduce", "_layers", "_moe", "_lm_head_argmax",
                         "decode_forward", "prefill_forward", "decode_step"],
    },
    "zstep_b200/models/qwen35_spec.py": {"SpecDecoder": ["verify_step", "mtp", "forward"]},
    "zstep_b200/models/deepseek.py": {
        "DeepSeekRunner": ["_reduce", "_site", "_advance", "_attention", "_ffn", "_layers", "decode_forward",
                           "prefill_forward"],
    },
    "zstep_b200/parallel/fused.py": {
        "FusedCollectives": ["protocol_for", "push_target", "allreduce_add_rmsnorm", "allreduce_sum",
                             "argmax_allreduce"],
    },
}
BANNED_METHODS = {"item", "cpu", "tolist", "numpy", "synchronize"}
BANNED_DIST = {"barrier", "broadcast", "all_gather_object", "broadcast_object_list"}


def _offences(fn: ast.FunctionDef) -> list[str]:
    out = []
    for n in ast.walk(fn):
        if not isinstance(n, ast.Call):
            continue
        f = n.func
        if isinstance(f, ast.Attribute) and f.attr in BANNED_METHODS:
            out.append(f".{f.attr}() at line {n.lineno}")
        if isinstance(f, ast.Attribute) and f.attr in BANNED_DIST and isinstance(f.value, ast.Name) \
                and f.value.id == "dist":
            out.append(f"dist.{f.attr}() at line {n.lineno}")
        if isinstance(f, ast.Name) and f.id == "print":
            out.append(f"print() at line {n.lineno}")
    return out


def test_step_methods_do_not_sync_with_the_host():
    problems = []
    for rel, classes in HOT.items():
        tree = ast.parse(open(os.path.join(ROOT, rel)).read())
        found = set()
        for node in ast.walk(tree):
            if isinstance(node, ast.ClassDef) and node.name in classes:
                for fn in node.body:
                    if isinstance(fn, ast.FunctionDef) and fn.name in classes[node.name]:
                        found.add((node.name, fn.name))
                        problems += [f"{rel} {node.name}.{fn.name}: {o}" for o in _offences(fn)]
        for cls, names in classes.items():
            for name in names:  # the guard must not silently skip a renamed method
                assert (cls, name) in found, f"{rel}: {cls}.{name} not found"
    assert not problems, "\n".join(problems)
