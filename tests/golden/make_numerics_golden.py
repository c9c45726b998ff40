"""Generate tests/golden/numerics.npz by running the REFERENCE's own numpy checks.

    python tests/golden/make_numerics_golden.py [--reference PATH]

The reference keeps its numerics references inline in its example scripts,
which also compile Metal kernels and talk to a Metal device at import time, so
they cannot be imported whole.  A child process parses each script with `ast`,
takes out only the reference functions and the inline check statements named
below, and executes those nodes unchanged in a namespace holding numpy, the
script's own shape constants (reduced sizes where the script's would be slow)
and seeded inputs.  The outputs are written next to this script; the CPU test
tests/test_numerics_golden.py checks that oracle/numerics.py reproduces them.

Reference pieces executed (file:line in the reference checkout):
  rmsnorm check      examples/benchmark_rmsnorm.py:115-116  (`rms`, `expected`)
  attention_ref      examples/benchmark_sdpa.py:198-208
  FA check           examples/showcase_attention.py:150-153 (`S_ref` .. `O_ref`)
  rmsnorm_np, rope_np, full_decode_np
                     examples/qwen_megakernel.py:308-342
  cache pre-fill     examples/qwen_megakernel.py:358-364
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

CHILD = r'''
import ast, sys
import numpy as np

ROOT = sys.argv[1]
OUT = sys.argv[2]


def parse(rel):
    src = open(f"{ROOT}/{rel}").read()
    return src, ast.parse(src)


def funcs(tree, names):
    """The module-level FunctionDef nodes with these names, as a module."""
    found = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    assert {n.name for n in found} == set(names), (names, [n.name for n in found])
    return ast.Module(body=found, type_ignores=[])


def _targets(n):
    out = []
    if isinstance(n, ast.Assign):
        for t in n.targets:
            while isinstance(t, ast.Subscript):
                t = t.value
            if isinstance(t, ast.Name):
                out.append(t.id)
    return out


def span(tree, first, last):
    """Module-level statements from the assignment to `first` through the last
    assignment to `last` (inclusive), unchanged."""
    body = tree.body
    i = next(k for k, n in enumerate(body) if first in _targets(n))
    j = max(k for k, n in enumerate(body) if last in _targets(n))
    assert i <= j
    return ast.Module(body=body[i:j + 1], type_ignores=[])


def run(mod, ns, rel):
    exec(compile(mod, f"{ROOT}/{rel}", "exec"), ns)
    return ns


out = {}

# ---------------------------------------------------------------- RMSNorm check
rel = "examples/benchmark_rmsnorm.py"
_, tree = parse(rel)
np.random.seed(42)
ROWS, N, EPS = 64, 512, 1e-5
X = np.random.randn(ROWS, N).astype(np.float32)
W = np.random.randn(N).astype(np.float32)
ns = run(span(tree, "rms", "expected"), {"np": np, "X": X, "W": W, "EPS": EPS}, rel)
out.update(rms_X=X, rms_W=W, rms_eps=np.float64(EPS), rms_expected=ns["expected"])

# ---------------------------------------------------------------- GQA attention_ref
rel = "examples/benchmark_sdpa.py"
_, tree = parse(rel)
np.random.seed(42)
T, HQ, G, D, S = 8, 8, 2, 16, 48
Q = np.random.randn(T, HQ, D).astype(np.float32) * 0.1
K = np.random.randn(G, S, D).astype(np.float32) * 0.1
V = np.random.randn(G, S, D).astype(np.float32) * 0.1
ns = run(funcs(tree, ["attention_ref"]), {"np": np, "QMUL": HQ // G}, rel)
out.update(gqa_Q=Q, gqa_K=K, gqa_V=V, gqa_O=ns["attention_ref"](Q, K, V))
# A peaked case (scores of magnitude ~tens): the softmax is dominated by a few keys.
Qp = Q * 40.0
out.update(gqa_Qpeak=Qp, gqa_Opeak=ns["attention_ref"](Qp, K, V))

# ---------------------------------------------------------------- FlashAttention check
rel = "examples/showcase_attention.py"
_, tree = parse(rel)
np.random.seed(1234)
M, NK, DD = 64, 96, 4
Qh = np.random.randn(M, DD).astype(np.float32)
Kh = np.random.randn(NK, DD).astype(np.float32)
Vh = np.random.randn(NK, DD).astype(np.float32)
ns = run(span(tree, "S_ref", "O_ref"), {"np": np, "Qh": Qh, "Kh": Kh, "Vh": Vh, "D": DD}, rel)
out.update(fa_Q=Qh, fa_K=Kh, fa_V=Vh, fa_O=ns["O_ref"])

# ---------------------------------------------------------------- Qwen decode layer
rel = "examples/qwen_megakernel.py"
_, tree = parse(rel)
H, INTER, QH, KVH = 64, 96, 4, 2
HD = H // QH
CACHE_LEN = 9
cst = dict(H=H, INTER=INTER, QH=QH, KVH=KVH, HD=HD, GQA=QH // KVH, QSZ=QH * HD,
           KVSZ=KVH * HD, CACHE_LEN=CACHE_LEN, CACHE_TOTAL=CACHE_LEN + 1, RMS_EPS=1e-6,
           ATTN_SCALE=1.0 / float(HD) ** 0.5)
rng = np.random.default_rng(0)
f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
wts = dict(
    Wq=f(QH * HD, H) / np.sqrt(H), Wk=f(KVH * HD, H) / np.sqrt(H), Wv=f(KVH * HD, H) / np.sqrt(H),
    Wo=f(H, QH * HD) / np.sqrt(QH * HD), Wg=f(INTER, H) / np.sqrt(H), Wu=f(INTER, H) / np.sqrt(H),
    Wd=f(H, INTER) / np.sqrt(INTER),
    w_in_norm=f(H) * 0.1 + 1.0, w_post_norm=f(H) * 0.1 + 1.0,
    w_q_norm=f(HD) * 0.1 + 1.0, w_k_norm=f(HD) * 0.1 + 1.0,
    k_cache=f(KVH, CACHE_LEN + 1, HD) * 0.1, v_cache=f(KVH, CACHE_LEN + 1, HD) * 0.1)
wts = {k: v.astype(np.float32) for k, v in wts.items()}
ang = (np.arange(HD).astype(np.float32) / HD) * (np.pi / 2)
wts["cos_pos"] = np.cos(ang).astype(np.float32)
wts["sin_pos"] = np.sin(ang).astype(np.float32)
x_in = (f(H) * 0.1).astype(np.float32)
ns = {"np": np, **cst, **wts, "x_in": x_in}
run(funcs(tree, ["rmsnorm_np", "rope_np", "full_decode_np"]), ns, rel)
ref_out = ns["full_decode_np"](x_in)
run(span(tree, "norm1_ref", "vc_fused"), ns, rel)
for k, v in wts.items():
    out["qwen_" + k] = v
out.update(qwen_x=x_in, qwen_out=np.asarray(ref_out, np.float32),
           qwen_kc_filled=ns["kc_fused"], qwen_vc_filled=ns["vc_fused"],
           qwen_shape=np.array([H, INTER, QH, KVH, HD, CACHE_LEN]))
xr = f(3, QH, HD)
out.update(rope_x=xr, rope_out=ns["rope_np"](xr, wts["cos_pos"], wts["sin_pos"]))

np.savez_compressed(OUT, **out)
print("wrote", OUT, len(out), "arrays")
'''


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", default=os.environ.get("ENIGMA_REFERENCE"),
                    help="path of the reference checkout (or set ENIGMA_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        sys.exit("give --reference PATH or set ENIGMA_REFERENCE")
    env = dict(os.environ, PYTHONPATH=a.reference)
    r = subprocess.run([sys.executable, "-c", CHILD, a.reference, str(HERE / "numerics.npz")],
                       env=env, capture_output=True, text=True)
    sys.stdout.write(r.stdout)
    if r.returncode != 0:
        sys.exit(r.stderr)


if __name__ == "__main__":
    main()
