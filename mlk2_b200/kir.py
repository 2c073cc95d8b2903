"""Kernel IR modules in the reference's ``mlk-kernel`` JSON wire format.

Builders for the modules this path runs, written so that their JSON is the
same document the reference's ``KernelModule::toJson`` produces for the same
module (reference compiler/src/support/kernel_ir.cpp:97-254; the shapes follow
compiler/src/passes/lower/lower.to_kernel_ir.cpp:369-425 for fused maps and
tools/mlk-poly/poly_bench.cpp:123-160 for Call modules).
"""
from __future__ import annotations

import json

import numpy as np

# mlkb_expr (include/mlkb200.h)
EXPR_DTYPE = np.dtype(
    [("op", "<i4"), ("a_kind", "<i4"), ("a_index", "<i8"), ("a_value", "<f8"),
     ("b_kind", "<i4"), ("reserved", "<i4"), ("b_index", "<i8"), ("b_value", "<f8")]
)

# MathOp numbering (reference compiler/include/mlk/ir/math_op.h:18-36)
OPS = ["add", "sub", "mul", "div", "neg", "pow", "exp", "log", "sin", "cos", "tan",
       "tanh", "sqrt", "rsqrt", "erf", "gelu"]
OP = {name: i for i, name in enumerate(OPS)}
UNARY = {"neg", "exp", "log", "sin", "cos", "tan", "tanh", "sqrt", "rsqrt", "erf", "gelu"}
# KernelOperand::Kind (reference kernel_ir.h:59-67)
KINDS = ["const", "elem_a", "elem_b", "scalar_param", "temp"]
CONST, ELEM_A, ELEM_B, SCALAR, TEMP = range(5)

A = (ELEM_A, 0, 0.0)
B = (ELEM_B, 0, 0.0)
ZERO = (CONST, 0, 0.0)


def C(v: float):
    return (CONST, 0, float(v))


def T(i: int):
    return (TEMP, int(i), 0.0)


def S(i: int):
    return (SCALAR, int(i), 0.0)


def E(op: str, a, b=ZERO):
    return (OP[op], a[0], a[1], a[2], b[0], 0, b[1], b[2])


def chain(*exprs) -> np.ndarray:
    return np.array(list(exprs), dtype=EXPR_DTYPE)


# y = sin(x*x + 3x): the lowering of examples/scalar/sin_graph.mlk.
SIN_CHAIN = chain(E("mul", A, A), E("mul", C(3), A), E("add", T(0), T(1)), E("sin", T(2)))
# dy/dx = cos(x*x + 3x) * (2x + 3): the calculus-pass derivative of the same chain.
DSIN_CHAIN = chain(E("mul", A, A), E("mul", C(3), A), E("add", T(0), T(1)), E("cos", T(2)),
                   E("mul", C(2), A), E("add", T(4), C(3)), E("mul", T(3), T(5)))


def _operand_json(kind: int, index: int, value: float) -> dict:
    o = {"kind": KINDS[kind]}
    if kind == CONST:
        o["value"] = value
    if kind in (TEMP, SCALAR):
        o["index"] = int(index)
    return o


def _expr_json(e) -> dict:
    return {"op": OPS[int(e["op"])],
            "a": _operand_json(int(e["a_kind"]), int(e["a_index"]), float(e["a_value"])),
            "b": _operand_json(int(e["b_kind"]), int(e["b_index"]), float(e["b_value"]))}


def _buf(name, dtype, inp, dims=None):
    b = {"name": name, "dtype": dtype, "input": inp, "output": not inp, "elements": -1}
    if dims is not None:
        b["dims"] = [int(d) for d in dims]
    return b


def map_module(chains, n_inputs: int = 1, poly7: bool = False, dtype: str = "f32") -> dict:
    """Multi-root fused map: one Loop{Compute; Store} per chain, each storing
    to its own output buffer (inputs first, then outputs, in table order)."""
    bufs = [_buf("x", dtype, True)]
    if n_inputs > 1:
        bufs.append(_buf("w", dtype, True))
    bufs += [_buf(f"y{r}", dtype, False) for r in range(len(chains))]
    nodes = []
    for r, ch in enumerate(chains):
        base = len(nodes)
        nodes.append({"op": "loop", "var": f"i{r}", "begin": 0, "end": -1, "step": 1,
                      "parallel": True, "children": [base + 1, base + 2]})
        comp = {"op": "compute", "math": OPS[int(ch[-1]["op"])]}
        if poly7:
            comp["family"] = "poly7"
        comp.update({"begin": 0, "end": -1, "step": 1, "a": 0})
        if n_inputs > 1:
            comp["b"] = 1
        comp["exprs"] = [_expr_json(e) for e in ch]
        comp["children"] = []
        nodes.append(comp)
        nodes.append({"op": "store", "begin": 0, "end": -1, "step": 1,
                      "out": n_inputs + r, "children": []})
    return {"format": "mlk-kernel", "version": 1, "name": "fused_map", "buffers": bufs,
            "nodes": nodes, "schedule": {}}


def call_module(kind: str, m: int, k: int, n: int = 0, dtypes=("f32", "f32", "f32")) -> dict:
    """Single Call(MatMul | Softmax | ReduceSum) over rank-2 buffers."""
    bufs = [_buf("A", dtypes[0], True, [m, k])]
    call = {"op": "call", "begin": 0, "end": -1, "step": 1, "a": 0}
    if kind == "matmul":
        bufs.append(_buf("B", dtypes[1], True, [k, n]))
        bufs.append(_buf("C", dtypes[2], False, [m, n]))
        call.update({"b": 1, "out": 2})
    elif kind == "softmax":
        bufs.append(_buf("Y", dtypes[-1], False, [m, k]))
        call["out"] = 1
    elif kind == "reducesum":
        bufs.append(_buf("Y", dtypes[-1], False, [m]))
        call["out"] = 1
    else:
        raise ValueError(kind)
    call["children"] = []
    return {"format": "mlk-kernel", "version": 1, "name": "call", "buffers": bufs,
            "nodes": [call], "schedule": {}}


def qk_softmax_module(s: int, d: int, scale: float, temps: bool = False, m: int = 0,
                      dtype: str = "f16") -> dict:
    """The scaled-scores softmax composite: Call(MatMul)(Q[m,d], Kt[d,s]) -> S,
    Loop{Sc = S * scale}, Call(Softmax)(Sc) -> Y (reference composition of
    kernel_buffers.cpp:1001-1085, :342-402 and :290-340). m defaults to s.

    temps=False: S and Sc are outputs (table Q, Kt, S, Sc, Y), the form the
    reference executor runs; MatMul accumulates into S (S += Q*Kt).
    temps=True: S and Sc are temps after the outputs (table Q, Kt, Y, S, Sc),
    only Y is observable -- the fused kernel's form. (The reference's 1-D
    executor does not bind temps to a Call, kernel_buffers.cpp:219-230, so
    only this path runs that form.)"""
    m = m or s
    io = "f64" if dtype == "f64" else "f32"
    q, kt = _buf("Q", dtype, True, [m, d]), _buf("Kt", dtype, True, [d, s])
    sb, scb, yb = (_buf("S", io, False, [m, s]), _buf("Sc", io, False, [m, s]),
                   _buf("Y", io, False, [m, s]))
    if temps:
        for b in (sb, scb):
            b["output"] = False
            b["temp"] = True
        bufs, S_, SC_, Y_ = [q, kt, yb, sb, scb], 3, 4, 2
    else:
        bufs, S_, SC_, Y_ = [q, kt, sb, scb, yb], 2, 3, 4
    nodes = [
        {"op": "call", "begin": 0, "end": -1, "step": 1, "a": 0, "b": 1, "out": S_, "children": []},
        {"op": "loop", "var": "i", "begin": 0, "end": -1, "step": 1, "parallel": True,
         "children": [2, 3]},
        {"op": "compute", "math": "mul", "begin": 0, "end": -1, "step": 1, "a": S_,
         "exprs": [_expr_json(chain(E("mul", A, C(scale)))[0])], "children": []},
        {"op": "store", "begin": 0, "end": -1, "step": 1, "out": SC_, "children": []},
        {"op": "call", "begin": 0, "end": -1, "step": 1, "a": SC_, "out": Y_, "children": []},
    ]
    return {"format": "mlk-kernel", "version": 1, "name": "qk_softmax", "buffers": bufs,
            "nodes": nodes, "schedule": {}}


def merge_roots(modules, names=None) -> dict:
    """One multi-root module from single-output modules over the same input:
    buffer 0 of each (its input) becomes the shared input, each module's
    output its own output buffer, and every node keeps its structure with
    buffer ids and children renumbered. This is the two-output form the
    reference's lowering cannot emit itself (lower.to_kernel_ir.cpp:404-408
    stores every output into outputBuffers[0])."""
    first = modules[0]
    bufs = [dict(first["buffers"][0])]
    nodes = []
    for r, mod in enumerate(modules):
        assert mod["buffers"][0]["input"] and sum(b["output"] for b in mod["buffers"]) == 1
        out = dict(next(b for b in mod["buffers"] if b["output"]))
        if names is not None:
            out["name"] = names[r]
        bufs.append(out)
        remap = {0: 0, next(i for i, b in enumerate(mod["buffers"]) if b["output"]): len(bufs) - 1}
        base = len(nodes)
        for n in mod["nodes"]:
            n = json.loads(json.dumps(n))
            for k in ("a", "b", "out"):
                if k in n:
                    n[k] = remap[n[k]]
            n["children"] = [c + base for c in n.get("children", [])]
            nodes.append(n)
    return {"format": "mlk-kernel", "version": first.get("version", 1), "name": "fused_map",
            "buffers": bufs, "nodes": nodes, "schedule": dict(first.get("schedule", {}))}


def with_static_length(module: dict, n: int) -> dict:
    """A copy of a module compiled for a tensor of static length n0 (loop
    bounds and buffer sizes fixed at n0, as the reference's pipeline emits
    them) with every such n0 replaced by n: the document the same pipeline
    writes for a tensor of length n (its output differs only in those
    numbers)."""
    m = json.loads(json.dumps(module))
    n0 = m["buffers"][0]["elements"]
    for b in m["buffers"]:
        if b.get("elements") == n0:
            b["elements"] = int(n)
        if b.get("dims") == [n0]:
            b["dims"] = [int(n)]
    for node in m["nodes"]:
        if node["op"] == "loop" and node.get("end") == n0:
            node["end"] = int(n)
    return m


def chains_of(module: dict):
    """The expression chain of each Compute node, as mlkb_expr arrays (for
    running a module's chains through the oracle)."""
    out = []
    for n in module["nodes"]:
        if n["op"] != "compute":
            continue
        rows = []
        for e in n["exprs"]:
            ops = []
            for side in ("a", "b"):
                o = e.get(side, {"kind": "const", "value": 0.0})
                ops.append((KINDS.index(o["kind"]), int(o.get("index", 0)), float(o.get("value", 0.0))))
            rows.append((OP[e["op"]], ops[0][0], ops[0][1], ops[0][2], ops[1][0], 0, ops[1][1], ops[1][2]))
        out.append(np.array(rows, dtype=EXPR_DTYPE))
    return out


def dumps(module: dict) -> str:
    return json.dumps(module, separators=(",", ":"))
