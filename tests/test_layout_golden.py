"""Layout algebra vs tables produced by the reference implementation itself
(tests/golden/make_golden.py imports the reference's enigma in a subprocess).
Bit-exact equality is required: these offsets decide every per-thread access."""
import json
from pathlib import Path

import pytest

from enigma.core import (Layout, Swizzle, blocked_product, coalesce, complement, composition,
                         left_inverse, logical_divide, make_layout_tv, make_ordered_layout,
                         recast_layout, right_inverse, zipped_divide)
from enigma.tensor import (Tensor, _compute_value_offsets, _group_contiguous, tensor_composition,
                           tensor_zipped_divide)
from enigma.tuple import compact_order, flatten, idx2crd, product

G = json.loads((Path(__file__).parent / "golden" / "layout_tables.json").read_text())


def dec(x):
    return tuple(dec(e) for e in x) if isinstance(x, list) else x


def L(d):
    return Layout(dec(d["shape"]), dec(d["stride"]))


def lay(x):
    return {"shape": enc(x.shape), "stride": enc(x.stride)}


def enc(x):
    return [enc(e) for e in x] if isinstance(x, tuple) else x


def table(x, limit=512):
    return [x(i) for i in range(min(x.size(), limit))]


def same(expect, fn):
    if "err" in expect:
        with pytest.raises(Exception) as ei:
            fn()
        assert type(ei.value).__name__ == expect["err"]
    else:
        assert fn() == expect["ok"]


@pytest.mark.parametrize("i", range(len(G["flat"])))
def test_flat_ops(i):
    r = G["flat"][i]
    a, m, tiler = L(r["L"]), L(r["M"]), dec(r["tiler"])
    assert table(a) == r["table"]
    assert a.cosize() == r["cosize"]
    same(r["coalesce"], lambda: lay(coalesce(a)))
    same(r["complement"], lambda: lay(complement(a)))
    same(r["complement64"], lambda: lay(complement(a, 64)))
    same(r["compose_ML"], lambda: lay(composition(m, a)))
    same(r["compose_LM"], lambda: lay(composition(a, m)))
    same(r["compose_ML_table"], lambda: table(composition(m, a)))
    same(r["right_inverse"], lambda: lay(right_inverse(a)))
    same(r["left_inverse"], lambda: lay(left_inverse(a)))
    same(r["logical_divide"],
         lambda: lay(logical_divide(m, tiler if isinstance(tiler, int) else tiler[0])))
    same(r["zipped_divide"], lambda: lay(zipped_divide(m, tiler)))
    same(r["blocked_product"], lambda: lay(blocked_product(a, m)))


@pytest.mark.parametrize("r", G["nested"], ids=lambda r: str(r["L"]))
def test_nested(r):
    a = L(r["L"])
    assert table(a) == r["table"]
    assert lay(coalesce(a)) == r["coalesce"]
    assert lay(complement(a)) == r["complement"]
    assert lay(zipped_divide(a, (2, 2))) == r["zipped_divide"]
    same(r["compose"], lambda: lay(composition(Layout(64, 1), a)))


@pytest.mark.parametrize("r", G["tv"], ids=lambda r: f"{r['thr']}x{r['val']}")
def test_make_layout_tv(r):
    (ts, to), (vs, vo) = r["thr"], r["val"]
    tiler, tv = make_layout_tv(make_ordered_layout(tuple(ts), tuple(to)),
                               make_ordered_layout(tuple(vs), tuple(vo)))
    assert enc(tiler) == r["tiler"]
    assert lay(tv) == r["tv"]
    assert [[tv((t, v)) for v in range(tv.size(1))] for t in range(tv.size(0))] == r["table"]


def test_config1_tv_table():
    """make_layout_tv(threads=256, values=4) -> tiler (1024,),
    ((256),(4)):((4),(1)); thread t owns offsets 4t..4t+3 of each 1024 chunk."""
    tiler, tv = make_layout_tv(make_ordered_layout((256,), (0,)), make_ordered_layout((4,), (0,)))
    assert tiler == (1024,) and repr(tv) == "((256),(4)):((4),(1))"
    assert all(tv((t, v)) == 4 * t + v for t in range(256) for v in range(4))


@pytest.mark.parametrize("r", G["recast"], ids=lambda r: str(r["args"][:2]))
def test_recast(r):
    nb, ob, d = r["args"]
    assert lay(recast_layout(nb, ob, L(d))) == r["out"]


@pytest.mark.parametrize("r", G["tensor"], ids=lambda r: f"{r['rows']}x{r['n']}/{r['thr']}x{r['val']}")
def test_tensor_tv_path(r):
    tiler, tv = make_layout_tv(make_ordered_layout((r["thr"],), (0,)),
                               make_ordered_layout((r["val"],), (0,)))
    x = Tensor("X", 0, r["dtype"], Layout((r["rows"], r["n"]), (r["n"], 1)))
    g = tensor_zipped_divide(x, (1, tiler[0]))
    assert lay(g.layout) == r["divided"]
    blk = g[((None, None), 1)][(0, None)]
    assert lay(blk.layout) == r["blk"] and blk.base_offset == r["blk_base"]
    tvx = tensor_composition(blk, tv, tiler)
    assert lay(tvx.layout) == r["tv"]
    for pt in r["per_thread"]:
        sub = tvx[(pt["t"], None)]
        assert sub.base_offset == pt["base"]
        offs = _compute_value_offsets(flatten(sub.layout.shape), flatten(sub.layout.stride),
                                      product(sub.layout.shape))
        assert offs == pt["offsets"]
        assert [list(g) for g in _group_contiguous(offs)] == pt["groups"]
    if r["oversize_error"]:
        with pytest.raises(Exception) as ei:
            tensor_zipped_divide(Tensor("Y", 0, r["dtype"], Layout((2, 8), (8, 1))), (1, 16))
        assert type(ei.value).__name__ == r["oversize_error"]


@pytest.mark.parametrize("r", G["swizzle"], ids=lambda r: str(r["args"]))
def test_swizzle(r):
    sw = Swizzle(*r["args"])
    assert [sw(i) for i in range(1024)] == r["table"]


def test_compact_order_and_idx2crd():
    for sh, o, st in G["compact_order"]:
        assert enc(compact_order(tuple(sh), tuple(o))) == st
    for i, c in G["idx2crd"]:
        assert enc(idx2crd(i, ((2, 3), 4))) == c
