"""Loop-carried values for `for i in enigma.range(...)` loops in kernel bodies.

A kernel body is traced by running it once in Python, so a plain Python `for` over
`enigma.range(...)` would see its body once and lose every value the body rebinds for the
next iteration.  As in the reference (enigma/compiler/preprocessor.py:21-215), the kernel's
source is rewritten before tracing: each such loop becomes a nested function of
(induction variable, carried values) returning the carried values, and a call of
`_enigma_carry_loop(lo, hi, step, body, *values)` that traces it as one loop with those
values as loop-carried slots (`for_range(..., init=...)`).  Carried names are the names the
body assigns (directly, in tuples, through `x[i] = ...` or `x.attr = ...`) that are already
bound before the loop (parameters or earlier assignments).  `enigma.range_constexpr(...)`
loops become plain Python `range` loops (unrolled at trace time).

When the source cannot be read (functions built with exec from a string) the kernel runs
unchanged and `enigma.range` keeps tracing one iteration without carries.
"""
from __future__ import annotations

import ast
import inspect
import textwrap
import types
from typing import Callable, List, Set


def _is_call_of(node, attr: str) -> bool:
    return (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
            and node.func.attr == attr and isinstance(node.func.value, ast.Name)
            and node.func.value.id == "enigma")


def _target_names(t) -> Set[str]:
    if isinstance(t, ast.Name):
        return {t.id}
    if isinstance(t, (ast.Tuple, ast.List)):
        out: Set[str] = set()
        for e in t.elts:
            out |= _target_names(e)
        return out
    if isinstance(t, (ast.Subscript, ast.Attribute)):
        base = t.value
        while isinstance(base, (ast.Subscript, ast.Attribute)):
            base = base.value
        return {base.id} if isinstance(base, ast.Name) else set()
    if isinstance(t, ast.Starred):
        return _target_names(t.value)
    return set()


def _assigned(stmts) -> Set[str]:
    """Names bound by the statements, not descending into nested function bodies."""
    out: Set[str] = set()
    stack = list(stmts)
    while stack:
        n = stack.pop()
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda, ast.ClassDef)):
            if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
                out.add(n.name)
            continue
        if isinstance(n, ast.Assign):
            for t in n.targets:
                out |= _target_names(t)
        elif isinstance(n, (ast.AugAssign, ast.AnnAssign)):
            out |= _target_names(n.target)
        elif isinstance(n, (ast.For, ast.comprehension)):
            out |= _target_names(n.target)
        elif isinstance(n, ast.withitem) and n.optional_vars is not None:
            out |= _target_names(n.optional_vars)
        elif isinstance(n, ast.NamedExpr):
            out |= _target_names(n.target)
        stack.extend(ast.iter_child_nodes(n))
    return out


def _escapes(stmts, in_loop: bool = False) -> bool:
    """A return, or a break / continue of this loop (not of a loop nested in it), in the
    statements; nested function bodies (rewritten inner loops among them) are skipped."""
    for n in stmts:
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef, ast.Lambda)):
            continue
        if isinstance(n, ast.Return):
            return True
        if isinstance(n, (ast.Break, ast.Continue)) and not in_loop:
            return True
        nested_loop = isinstance(n, (ast.For, ast.While, ast.AsyncFor))
        for field in ("body", "orelse", "handlers", "finalbody"):
            sub = getattr(n, field, None)
            if isinstance(sub, list) and _escapes(sub, in_loop or (nested_loop and field == "body")):
                return True
    return False


class _Rewriter(ast.NodeTransformer):
    def __init__(self, func: ast.FunctionDef):
        self.func = func
        self.params = {a.arg for a in func.args.args + func.args.kwonlyargs}
        self.count = 0
        self.changed = False

    def _bound_before(self, loop: ast.For) -> Set[str]:
        """Parameters and names bound by constructs that start on an earlier line."""
        bound = set(self.params)
        for n in ast.walk(self.func):
            ln = getattr(n, "lineno", None)
            if ln is None or ln >= loop.lineno or n is self.func:
                continue
            if isinstance(n, ast.Assign):
                for t in n.targets:
                    bound |= _target_names(t)
            elif isinstance(n, (ast.AugAssign, ast.AnnAssign, ast.NamedExpr, ast.For)):
                bound |= _target_names(n.target)
            elif isinstance(n, ast.With):
                for it in n.items:
                    if it.optional_vars is not None:
                        bound |= _target_names(it.optional_vars)
            elif isinstance(n, (ast.FunctionDef, ast.ClassDef)):
                bound.add(n.name)
        return bound

    def visit_For(self, node: ast.For):
        self.generic_visit(node)
        if _is_call_of(node.iter, "range_constexpr"):
            self.changed = True
            node.iter = ast.Call(func=ast.Name(id="range", ctx=ast.Load()),
                                 args=node.iter.args, keywords=[])
            return node
        if not _is_call_of(node.iter, "range"):
            return node
        if not isinstance(node.target, ast.Name):
            raise SyntaxError("enigma.range(): the loop variable must be a single name")
        if node.orelse:
            raise SyntaxError("enigma.range(): a for ... else loop cannot be traced")
        if _escapes(node.body):
            raise SyntaxError("enigma.range(): break / continue / return inside the loop "
                              "cannot be traced")
        args = node.iter.args
        if not 1 <= len(args) <= 3:
            raise SyntaxError("enigma.range() takes 1 to 3 arguments")
        lo, hi, step = ((ast.Constant(0), args[0], ast.Constant(1)) if len(args) == 1 else
                        (args[0], args[1], ast.Constant(1)) if len(args) == 2 else tuple(args))
        iv = node.target.id
        carried = sorted((_assigned(node.body) & self._bound_before(node)) - {iv})
        self.changed = True
        name = f"_enigma_loop_body_{self.count}"
        self.count += 1
        body = list(node.body)
        body.append(ast.Return(value=ast.Tuple(
            elts=[ast.Name(id=c, ctx=ast.Load()) for c in carried], ctx=ast.Load())))
        fdef = ast.FunctionDef(
            name=name,
            args=ast.arguments(posonlyargs=[], args=[ast.arg(arg=iv)] +
                               [ast.arg(arg=c) for c in carried], vararg=None, kwonlyargs=[],
                               kw_defaults=[], kwarg=None, defaults=[]),
            body=body, decorator_list=[], returns=None, type_params=[])
        call = ast.Call(func=ast.Name(id="_enigma_carry_loop", ctx=ast.Load()),
                        args=[lo, hi, step, ast.Name(id=name, ctx=ast.Load())] +
                        [ast.Name(id=c, ctx=ast.Load()) for c in carried], keywords=[])
        if carried:
            stmt = ast.Assign(targets=[ast.Tuple(elts=[ast.Name(id=c, ctx=ast.Store())
                                                       for c in carried], ctx=ast.Store())],
                              value=call)
        else:
            stmt = ast.Expr(value=call)
        out = [fdef, stmt]
        for o in out:
            ast.copy_location(o, node)
        return out


def rewrite_range_loops(fn: Callable) -> Callable:
    """The kernel function with its enigma.range loops carrying values (or `fn` itself when
    it has none, or its source is unavailable)."""
    try:
        src = textwrap.dedent(inspect.getsource(fn))
    except (OSError, TypeError):
        return fn
    try:
        tree = ast.parse(src)
    except SyntaxError:
        return fn
    func = next((n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)
                 and n.name == fn.__name__), None)
    if func is None:
        return fn
    rw = _Rewriter(func)
    rw.visit(func)
    if not rw.changed:
        return fn
    func.decorator_list = []
    mod = ast.Module(body=[func], type_ignores=[])
    ast.fix_missing_locations(mod)
    first = fn.__code__.co_firstlineno
    ast.increment_lineno(mod, first - func.lineno)
    code = compile(mod, fn.__code__.co_filename, "exec")
    from .._tracing import _enigma_carry_loop
    ns = dict(fn.__globals__)
    if fn.__closure__:
        for var, cell in zip(fn.__code__.co_freevars, fn.__closure__):
            try:
                ns[var] = cell.cell_contents
            except ValueError:   # cell not yet filled
                pass
    ns["_enigma_carry_loop"] = _enigma_carry_loop
    local: dict = {}
    exec(code, ns, local)
    new = local[fn.__name__]
    if fn.__defaults__:
        new = types.FunctionType(new.__code__, new.__globals__, new.__name__, fn.__defaults__,
                                 new.__closure__)
    new.__module__ = fn.__module__
    new.__wrapped__ = fn
    return new


def carried_names(fn: Callable) -> List[List[str]]:
    """For tests and tooling: the carried names of each enigma.range loop of `fn`, in order."""
    tree = ast.parse(textwrap.dedent(inspect.getsource(fn)))
    func = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef)
                and n.name == fn.__name__)
    rw = _Rewriter(func)
    rw.visit(func)
    out = []
    for n in ast.walk(func):
        if (isinstance(n, ast.Call) and isinstance(n.func, ast.Name)
                and n.func.id == "_enigma_carry_loop"):
            out.append([a.id for a in n.args[4:]])
    return out
