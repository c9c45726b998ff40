"""Loop-carried values of `for i in enigma.range(...)` loops (CPU only): the kernel body is
rewritten before tracing (compiler/loops.py, the counterpart of the reference's AST
preprocessor, enigma/compiler/preprocessor.py:21-215), so values the body rebinds flow
from one iteration to the next and out of the loop, in the trace and in its dump."""
import pytest

import enigma
import dsl_kernels as K
from enigma.compiler.loops import carried_names


@enigma.kernel
def running_sum(A: enigma.f32, Out: enigma.f32):
    i = enigma.thread_position_in_grid
    acc = enigma.metal_cast(0.0, "float")
    big = enigma.metal_cast(-1e30, "float")
    for t in enigma.range(16):
        v = A[i * 16 + enigma.metal_cast(t, "uint")]
        acc = acc + v
        big = enigma.fmax(big, v)
    Out[i] = acc + big


def _ops(builder):
    return list(builder.walk())


def test_carried_names():
    assert carried_names(running_sum.fn) == [["acc", "big"]]


def test_trace_carries_values_through_the_loop():
    from enigma.compiler.kernel import trace_kernel
    b = trace_kernel(running_sum)
    loops = [op for op in _ops(b) if op.op == "scf_for"]
    assert len(loops) == 1
    loop = loops[0]
    assert len(loop.attrs["iter_args"]) == 2 and len(loop.attrs["results"]) == 2
    # the store after the loop reads the loop's results, not the values before it
    store = [op for op in b.ops if op.op == "store"][-1]
    val = store.operands[1]
    add = next(op for op in _ops(b) if op.result is val)
    assert {id(o) for o in add.operands} == {id(r) for r in loop.attrs["results"]}
    # inside the body, the yielded values are computed from the iter_args
    body_ids = {id(op.result) for op in loop.regions[0] if op.result is not None}
    assert all(id(y) in body_ids for y in loop.attrs["yield_vals"])


def test_dump_shows_iter_args_and_yield():
    from enigma.compiler.compiler import format_ir
    from enigma.compiler.kernel import trace_kernel
    src = format_ir(trace_kernel(running_sum))
    assert "yield(" in src and "= scf_for(" in src


def test_lists_of_values_are_carried():
    """The GQA kernel (benchmark_sdpa.py pattern) rebinds list entries m[g], l[g], ox[g],
    oy[g] inside enigma.range: every entry becomes a loop-carried slot."""
    jit, args, thr = K.make_sdpa_gqa(16, 16, 2, 64, 64)    # qmul = 8
    ck = enigma.compile(jit, *args)
    assert ck.cuda_kernel.layout == "gqa_interleaved"
    head = [ln for ln in ck.metal_source.splitlines() if "scf_for(" in ln][0]
    assert head.count("_v") >= 4 * 8


def test_range_constexpr_unrolls():
    @enigma.kernel
    def unrolled(A: enigma.f32, Out: enigma.f32):
        i = enigma.thread_position_in_grid
        s = A[i]
        for _ in enigma.range_constexpr(3):
            s = s * 2.0
        Out[i] = s

    from enigma.compiler.kernel import trace_kernel
    b = trace_kernel(unrolled)
    assert not [op for op in b.walk() if op.op == "scf_for"]
    assert sum(op.op == "mul" for op in b.walk()) == 3


def test_break_inside_traced_loop_is_rejected():
    @enigma.kernel
    def bad(A: enigma.f32, Out: enigma.f32):
        for t in enigma.range(4):
            break
        Out[0] = A[0]

    with pytest.raises(SyntaxError, match="break"):
        enigma.compile(bad)


def test_nested_loops_carry_through_both_levels():
    """An outer enigma.range loop whose carried sum is updated by an inner loop: the inner
    loop carries it too, and the outer loop yields the inner loop's result."""
    @enigma.kernel
    def nested(A: enigma.f32, Out: enigma.f32):
        i = enigma.thread_position_in_grid
        acc = enigma.metal_cast(0.0, "float")
        for r in enigma.range(4):
            for c in enigma.range(8):
                acc = acc + A[i * 32 + enigma.metal_cast(r, "uint") * 8 + enigma.metal_cast(c, "uint")]
        Out[i] = acc

    from enigma.compiler.kernel import trace_kernel
    b = trace_kernel(nested)
    outer = next(op for op in b.ops if op.op == "scf_for")
    inner = next(op for op in outer.regions[0] if op.op == "scf_for")
    assert len(outer.attrs["iter_args"]) == 1 and len(inner.attrs["iter_args"]) == 1
    assert inner.operands[3] is outer.attrs["iter_args"][0]          # inner starts from outer's carry
    assert outer.attrs["yield_vals"][0] is inner.attrs["results"][0]  # outer yields inner's result
    store = [op for op in b.ops if op.op == "store"][-1]
    assert store.operands[1] is outer.attrs["results"][0]


def test_closure_values_are_seen_by_the_rewritten_body():
    scale = 3.0

    @enigma.kernel
    def scaled(A: enigma.f32, Out: enigma.f32):
        i = enigma.thread_position_in_grid
        acc = enigma.metal_cast(0.0, "float")
        for t in enigma.range(2):
            acc = acc + A[i] * scale
        Out[i] = acc

    from enigma.compiler.kernel import trace_kernel
    b = trace_kernel(scaled)
    consts = [op.attrs.get("value") for op in b.walk() if op.op == "const"]
    assert 3.0 in consts
