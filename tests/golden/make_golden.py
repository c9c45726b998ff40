"""Generate tests/golden/layout_tables.json from the REFERENCE implementation.

    python tests/golden/make_golden.py [--reference PATH]

The reference's pure-Python layout algebra (enigma/tuple.py, enigma/core.py,
enigma/tensor.py) is imported in a child process with PYTHONPATH pointing at
the reference checkout, so its `enigma` never meets this repository's.  The
child evaluates a seeded sweep of cases and prints JSON; this script writes
it next to itself.  The committed JSON is what the tests read (the reference
is not available where the tests run on a GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent

CHILD = r'''
import json, random
from enigma.core import (Layout, coalesce, complement, composition, logical_divide, zipped_divide,
                         blocked_product, recast_layout, make_layout_tv, make_ordered_layout,
                         right_inverse, left_inverse, Swizzle)
from enigma.tensor import Tensor, tensor_zipped_divide, tensor_composition, \
    _compute_value_offsets, _group_contiguous
from enigma.tuple import flatten, idx2crd, crd2idx, compact_order, product

def enc(x):
    if isinstance(x, tuple):
        return [enc(e) for e in x]
    return x

def lay(L):
    return {"shape": enc(L.shape), "stride": enc(L.stride)}

def table(L, limit=512):
    n = L.size()
    return [L(i) for i in range(min(n, limit))]

def safe(fn):
    try:
        return {"ok": fn()}
    except Exception as e:
        return {"err": type(e).__name__}

rng = random.Random(20261201)
out = {"flat": [], "nested": [], "tv": [], "recast": [], "tensor": [], "swizzle": []}

def rand_flat():
    r = rng.randint(1, 4)
    shape = tuple(rng.choice([1, 2, 3, 4, 8, 16]) for _ in range(r))
    stride = tuple(rng.choice([0, 1, 2, 4, 8, 16, 32, 64, 3, 5]) for _ in range(r))
    return Layout(shape, stride) if r > 1 else Layout(shape[0], stride[0])

def rand_compact():
    r = rng.randint(1, 3)
    shape = tuple(rng.choice([2, 4, 8, 16]) for _ in range(r))
    order = tuple(rng.sample(range(r), r))
    return make_ordered_layout(shape, order)

for _ in range(400):
    L = rand_flat()
    M = rand_compact()
    tiler = rng.choice([2, 4, 8, (2, 2), (4, 2), (2, 4)])
    rec = {"L": lay(L), "M": lay(M), "tiler": enc(tiler), "table": table(L), "cosize": L.cosize()}
    rec["coalesce"] = safe(lambda: lay(coalesce(L)))
    rec["complement"] = safe(lambda: lay(complement(L)))
    rec["complement64"] = safe(lambda: lay(complement(L, 64)))
    rec["compose_ML"] = safe(lambda: lay(composition(M, L)))
    rec["compose_LM"] = safe(lambda: lay(composition(L, M)))
    rec["compose_ML_table"] = safe(lambda: table(composition(M, L)))
    rec["right_inverse"] = safe(lambda: lay(right_inverse(L)))
    rec["left_inverse"] = safe(lambda: lay(left_inverse(L)))
    rec["logical_divide"] = safe(lambda: lay(logical_divide(M, tiler if isinstance(tiler, int) else tiler[0])))
    rec["zipped_divide"] = safe(lambda: lay(zipped_divide(M, tiler)))
    rec["blocked_product"] = safe(lambda: lay(blocked_product(L, M)))
    out["flat"].append(rec)

nested = [Layout(((2, 4), 8), ((1, 2), 8)), Layout(((4, 64), (4, 4)), ((64, 4), (16, 1))),
          Layout((4, (2, 2)), (2, (1, 8))), Layout(((2, 2), (2, 2)), ((1, 4), (2, 8)))]
for L in nested:
    out["nested"].append({"L": lay(L), "table": table(L), "coalesce": lay(coalesce(L)),
                          "complement": lay(complement(L)),
                          "zipped_divide": lay(zipped_divide(L, (2, 2))),
                          "compose": safe(lambda: lay(composition(Layout(64, 1), L)))})

tv_cases = [((256,), (0,), (4,), (0,)), ((256,), (0,), (8,), (0,)), ((256,), (0,), (16,), (0,)),
            ((32,), (0,), (2,), (0,)), ((32, 1), (0, 1), (1, 4), (0, 1)),
            ((4, 64), (1, 0), (4, 4), (1, 0)), ((128,), (0,), (4,), (0,)),
            ((8, 32), (1, 0), (2, 4), (0, 1)), ((16, 16), (0, 1), (4, 2), (1, 0))]
for ts, to, vs, vo in tv_cases:
    tiler, tv = make_layout_tv(make_ordered_layout(ts, to), make_ordered_layout(vs, vo))
    tab = [[tv((t, v)) for v in range(tv.size(1))] for t in range(tv.size(0))]
    out["tv"].append({"thr": [list(ts), list(to)], "val": [list(vs), list(vo)],
                      "tiler": enc(tiler), "tv": lay(tv), "table": tab})

for bits_new, bits_old, L in [(128, 32, Layout((4, 8), (1, 4))), (64, 16, Layout((8, 4), (1, 8))),
                              (32, 32, Layout(8, 1)), (128, 16, Layout((2, (8, 4)), (64, (1, 8))))]:
    out["recast"].append({"args": [bits_new, bits_old, lay(L)],
                          "out": lay(recast_layout(bits_new, bits_old, L))})

for rows, n, thr, val, dt in [(4096, 4096, 256, 4, "float"), (4096, 4096, 256, 16, "float"),
                              (64, 8192, 256, 8, "bfloat"), (8, 1024, 128, 8, "bfloat"),
                              (16, 512, 64, 2, "float"), (4, 96, 32, 3, "float")]:
    tiler, tv = make_layout_tv(make_ordered_layout((thr,), (0,)), make_ordered_layout((val,), (0,)))
    X = Tensor("X", 0, dt, Layout((rows, n), (n, 1)))
    g = tensor_zipped_divide(X, (1, tiler[0]))
    blk = g[((None, None), 1)][(0, None)]
    tvx = tensor_composition(blk, tv, tiler)
    per_thread = []
    for t in (0, 1, thr - 1):
        sub = tvx[(t, None)]
        fs, fd = flatten(sub.layout.shape), flatten(sub.layout.stride)
        offs = _compute_value_offsets(fs, fd, product(sub.layout.shape))
        per_thread.append({"t": t, "base": sub.base_offset, "offsets": offs,
                           "groups": [list(gp) for gp in _group_contiguous(offs)]})
    rec = {"rows": rows, "n": n, "thr": thr, "val": val, "dtype": dt, "tiler": enc(tiler),
           "divided": lay(g.layout), "blk": lay(blk.layout), "blk_base": blk.base_offset,
           "tv": lay(tvx.layout), "per_thread": per_thread}
    try:
        tensor_zipped_divide(Tensor("Y", 0, dt, Layout((2, 8), (8, 1))), (1, 16))
        rec["oversize_error"] = None
    except Exception as e:
        rec["oversize_error"] = type(e).__name__
    out["tensor"].append(rec)

for b, m, s in [(3, 3, 6), (3, 4, 7), (2, 2, 5), (1, 4, 3), (0, 3, 3)]:
    sw = Swizzle(b, m, s)
    out["swizzle"].append({"args": [b, m, s], "table": [sw(i) for i in range(1024)]})

out["compact_order"] = [[list(sh), list(o), enc(compact_order(sh, o))]
                        for sh, o in [((4, 8), (1, 0)), ((2, 3, 4), (2, 0, 1)), ((5,), (0,))]]
out["idx2crd"] = [[i, enc(idx2crd(i, ((2, 3), 4)))] for i in range(24)]
print(json.dumps(out))
'''


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ENIGMA_REFERENCE"),
                    help="root of the reference checkout (or set ENIGMA_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference (or ENIGMA_REFERENCE): the reference checkout to import")
    env = dict(os.environ, PYTHONPATH=a.reference, PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True,
                       cwd="/tmp")
    if r.returncode != 0:
        sys.exit(r.stderr)
    data = json.loads(r.stdout)
    (HERE / "layout_tables.json").write_text(json.dumps(data, separators=(",", ":")))
    print(f"wrote {HERE / 'layout_tables.json'} "
          f"({sum(len(v) for v in data.values() if isinstance(v, list))} cases)")


if __name__ == "__main__":
    main()
