"""The reference's own example kernels, traced by this package and bound (CPU only).

Each example script of the reference defines its kernels and @jit launchers with the
public `enigma` API and then compiles them; the rest of the script talks to a Metal
device.  This test parses each script with `ast`, keeps the module-level statements up
to its last `enigma.compile(...)` call (imports, constants, layouts, kernel and launcher
definitions, the compile calls) minus statements that print, write files, run xcrun or
open a Metal runtime, executes them unchanged with this package as `enigma`, and checks
which sm_100a operator each compiled kernel is bound to.  Nothing of the reference is
copied into this repository: the scripts are read from the reference checkout, found
through ENIGMA_REFERENCE or as a `reference` directory beside this repository's
checkout; the test is skipped where neither exists (e.g. on a GPU box).
"""
import ast
import os
from pathlib import Path

import pytest

import enigma

_ROOT = Path(__file__).resolve().parent.parent


def _reference_root():
    cand = os.environ.get("ENIGMA_REFERENCE") or str(_ROOT.parent / "reference")
    p = Path(cand)
    return p if (p / "examples").is_dir() and (p / "enigma").is_dir() else None


REF = _reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not available")

# Calls whose statements are side effects on a Metal host (xcrun, temp dirs, metallib
# files, the Metal runtime), not part of defining or compiling a kernel.
_SIDE_EFFECTS = {"MetalRuntime", "run", "mkdtemp", "CompiledKernel", "open", "Path",
                 "read_bytes", "export_metal"}


def _calls(node):
    for n in ast.walk(node):
        if isinstance(n, ast.Call):
            f = n.func
            yield f.attr if isinstance(f, ast.Attribute) else getattr(f, "id", None)


def _kept(node) -> bool:
    if isinstance(node, (ast.FunctionDef, ast.ClassDef, ast.Import, ast.ImportFrom)):
        return True
    if isinstance(node, (ast.Assign, ast.AnnAssign)):
        return not any(c in _SIDE_EFFECTS for c in _calls(node))
    return False


def _compile_example(name):
    path = REF / "examples" / name
    tree = ast.parse(path.read_text())
    last = max(i for i, n in enumerate(tree.body) if "compile" in set(_calls(n)))
    body = [n for n in tree.body[:last + 1] if _kept(n)]
    ns = {"__file__": str(path), "__name__": "reference_example"}
    exec(compile(ast.Module(body=body, type_ignores=[]), str(path), "exec"), ns)
    return {k: v for k, v in ns.items() if isinstance(v, enigma.CompiledKernel)}


def test_benchmark_rmsnorm_kernel():
    """examples/benchmark_rmsnorm.py:31-84 (TV layout (256,)x(16,), eps 1e-5, 4096^2 fp32)."""
    b = _compile_example("benchmark_rmsnorm.py")["enigma_compiled"].cuda_kernel
    assert (b.op, b.dtype) == ("rmsnorm", "float")
    assert b.params["eps"] == pytest.approx(1e-5)
    assert (b.params["rows"], b.params["hidden"], b.params["vector_run"]) == (4096, 4096, 16)


def test_benchmark_sdpa_kernel():
    """examples/benchmark_sdpa.py:48-158: GQA decode attention, interleaved KV, no scale."""
    ck = _compile_example("benchmark_sdpa.py")["enigma_compiled"]
    b = ck.cuda_kernel
    assert (b.op, b.layout, b.params["causal"]) == ("sdpa", "gqa_interleaved", False)
    assert ck.grid == (128 * 128, 8, 1) and ck.block == (128, 1, 1)


def test_showcase_attention_kernels():
    """examples/showcase_attention.py:94-131: fa_naive and the TV-layout fa_tv launcher."""
    cks = _compile_example("showcase_attention.py")
    for key in ("fa_naive_compiled", "fa_tv_compiled"):
        b = cks[key].cuda_kernel
        assert (b.op, b.layout, b.params["head_dim"], b.params["causal"]) == \
            ("sdpa", "rows", 4, False)
        assert b.params["scale"] == pytest.approx(0.5)
    assert cks["fa_tv_compiled"].grid == (1024, 1, 1)
    assert cks["fa_tv_compiled"].block == (32, 1, 1)


def test_qwen_megakernel():
    """examples/qwen_megakernel.py:228-269: the fused single-layer decode kernel."""
    ck = _compile_example("qwen_megakernel.py")["fused_c"]
    assert (ck.cuda_kernel.op, ck.cuda_kernel.layout) == ("decode", "qwen_fused_f32")
    assert ck.num_params == 26


def test_async_copy_gemm():
    """examples/async_copy_gemm.py:32-79 (tiles staged with 2-D async copies)."""
    b = _compile_example("async_copy_gemm.py")["compiled"].cuda_kernel
    assert (b.op, b.layout, b.params["K"], b.params["N"]) == ("gemm", "async_tiles", 64, 64)


@pytest.mark.parametrize("name,keys", [
    ("vector_add_tv.py", ["compiled"]), ("vector_add.py", ["compiled"]),
    ("benchmark_naive_vs_tv.py", ["naive_compiled", "vec4_compiled", "tv_compiled"])])
def test_elementwise_examples(name, keys):
    cks = _compile_example(name)
    for k in keys:
        b = cks[k].cuda_kernel
        assert (b.op, b.params["op"]) == ("elementwise", 0)
