"""Graph IR of a lowered tysor function, and its text form.

This mirrors the reference's `GraphFunction` (src/ir/graph.rs:6-45): a list of
values (parameters first, then one value per expression node, in the
post-order in which `GraphBuilder::lower_expr` appends them,
src/ir/builder.rs:12-28, 97-174) and a list of nodes of six kinds
{Constant, Binary, PrimitiveCall, LibraryCall, LibraryCtor, Apply}
(src/ir/graph.rs:15-24).

The DSL front end (lexer, parser, semantic analysis, lowering) is not part of
this package; programs are built with `GraphBuilder`, whose calls follow the
same id-assignment order the reference builder uses, so value ids and the
derived parameter names (`linear_{id}_weight`, training/executor.rs:140-150)
match what the reference produces for the same source.

The text form (`Graph.to_text`) is what the native executor parses
(`tysor_cuda_graph_new` in include/tysor_cuda.h).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Union

# Primitive tensor ops (src/ops/library.rs:49-93: matmul, relu, scale).
PRIMITIVE_OPS = ("matmul", "relu", "scale")
# Library calls the reference runtime executes (graph_executor.rs:114-161),
# plus `transpose`, an extension with no reference counterpart.
LIBRARY_CALLS = ("rms_norm", "cross_entropy", "reshape", "repeat_kv", "flatten_heads",
                 "causal_mask", "rope", "transpose")
# Layer constructors (graph_executor.rs:163-223), plus `RMSNorm`, an
# extension: rms_norm with a learned gain and a configurable eps.
LIBRARY_CTORS = ("linear", "SiLU", "Softmax", "Embedding", "Dropout", "RMSNorm")

NODE_KINDS = ("const", "binary", "primitive", "call", "ctor", "apply")
VALUE_KINDS = ("tensor", "int", "float", "bool", "callable")
BINARY_OPS = ("+", "-", "*", "/")


@dataclass
class Value:
    id: int
    kind: str
    is_parameter: bool = False
    name: str = ""
    # A tensor parameter's annotated dtype (`x: tensor[float16]`); "" when
    # unannotated.  The string is carried and printed, never computed in:
    # every tensor is f32 (runtime/tensor.rs:3-8).
    dtype: str = ""


@dataclass
class Node:
    kind: str
    output: int
    op: str = ""
    binop: str = "+"
    const: Any = None
    inputs: List[int] = field(default_factory=list)


@dataclass
class Graph:
    name: str = "model"
    values: List[Value] = field(default_factory=list)
    nodes: List[Node] = field(default_factory=list)
    outputs: List[int] = field(default_factory=list)
    named: Dict[str, int] = field(default_factory=dict)
    # `train model:` fields (frontend_ir.rs:1037-1069; executor.rs:775-791).
    objective: Optional[str] = None
    lr: float = 0.01
    iterations: int = 1
    optimizer: str = "sgd"
    # Whether a train run was declared for this graph (set by
    # GraphBuilder.train): the reference's --train needs one.
    train_run: bool = False

    # -- queries ---------------------------------------------------------
    def parameters(self) -> List[Value]:
        return [v for v in self.values if v.is_parameter]

    def objective_id(self) -> int:
        """training/executor.rs:528-543: the named objective, else the first output."""
        if self.objective is not None:
            if self.objective not in self.named:
                raise ValueError(f"Could not resolve objective '{self.objective}' in graph")
            return self.named[self.objective]
        if not self.outputs:
            raise ValueError("Graph does not have a return value")
        return self.outputs[0]

    def value_dtypes(self) -> Dict[int, str]:
        """The dtype string each tensor value carries in the reference's local
        executor: a parameter its annotation or "float32"
        (graph_executor.rs:90-93); an embedding lookup the constructor's
        declared return dtype, which builtin constructors leave unset, so
        "float32" (graph_executor.rs:208-213, compiler/builtins/registry.rs);
        `scalar op tensor` the tensor's (tensor.rs:149); every other op its
        first tensor operand's (tensor.rs:121-258, layers.rs:127-322)."""
        dt: Dict[int, str] = {}
        for v in self.values:
            if v.is_parameter and v.kind == "tensor":
                dt[v.id] = v.dtype or "float32"
        ctors: Dict[int, str] = {}
        for n in self.nodes:
            if n.kind == "ctor":
                ctors[n.output] = n.op
                continue
            if n.kind == "apply":
                out = "float32" if ctors.get(n.inputs[0]) == "Embedding" else dt.get(n.inputs[1])
            elif n.kind in ("binary", "primitive", "call"):
                out = next((dt[i] for i in n.inputs if i in dt), None)
            else:
                out = None
            if out is not None:
                dt[n.output] = out
        return dt

    def producer(self, value_id: int) -> Optional[Node]:
        for node in self.nodes:
            if node.output == value_id:
                return node
        return None

    # -- text form -------------------------------------------------------
    def to_text(self) -> str:
        lines = [f"graph {self.name}"]
        for v in self.values:
            lines.append(f"value {v.id} {v.kind} {int(v.is_parameter)} {v.name or '-'}")
        for n in self.nodes:
            if n.kind == "const":
                c = n.const
                if isinstance(c, bool):
                    lines.append(f"node const {n.output} bool {int(c)}")
                elif isinstance(c, int):
                    lines.append(f"node const {n.output} int {c}")
                else:
                    lines.append(f"node const {n.output} float {float(c)!r}")
            elif n.kind == "binary":
                lines.append(f"node binary {n.output} {n.binop} " + " ".join(map(str, n.inputs)))
            elif n.kind == "apply":
                lines.append(f"node apply {n.output} " + " ".join(map(str, n.inputs)))
            else:
                lines.append(f"node {n.kind} {n.output} {n.op} " + " ".join(map(str, n.inputs)))
        for o in self.outputs:
            lines.append(f"output {o}")
        if self.objective is not None or self.outputs:
            lines.append(f"objective {self.objective_id()}")
        lines.append("end")
        return "\n".join(lines) + "\n"


class Ref(int):
    """A reference to an existing graph value (as opposed to a literal)."""


Arg = Union[Ref, int, float, bool]


class GraphBuilder:
    """Builds a `Graph` with the reference builder's value-id order.

    Literal Python ints/floats/bools passed as arguments become Constant
    nodes at the point they are encountered, exactly as `lower_expr` lowers
    constant arguments before the call that consumes them.
    """

    def __init__(self, name: str = "model", param_dtype: str = ""):
        self.g = Graph(name=name)
        self.param_dtype = param_dtype

    # values
    def _value(self, kind: str, name: str = "", is_parameter: bool = False) -> Ref:
        vid = len(self.g.values)
        self.g.values.append(Value(vid, kind, is_parameter, name))
        if name:
            self.g.named[name] = vid
        return Ref(vid)

    def param(self, name: str, dtype: Optional[str] = None) -> Ref:
        """A function parameter (always a tensor on the hot path); `dtype` is
        its annotation (default: the builder's param_dtype)."""
        ref = self._value("tensor", name, True)
        self.g.values[ref].dtype = self.param_dtype if dtype is None else dtype
        return ref

    def _arg(self, a: Arg) -> Ref:
        if isinstance(a, Ref):
            return a
        return self.const(a)

    def const(self, c: Union[int, float, bool]) -> Ref:
        kind = "bool" if isinstance(c, bool) else "int" if isinstance(c, int) else "float"
        out = self._value(kind)
        self.g.nodes.append(Node("const", out, const=c))
        return out

    def binary(self, op: str, lhs: Arg, rhs: Arg) -> Ref:
        if op not in BINARY_OPS:
            raise ValueError(f"unsupported binary op {op}")
        a = self._arg(lhs)
        b = self._arg(rhs)
        kind = "tensor" if "tensor" in (self.g.values[a].kind, self.g.values[b].kind) else "float"
        out = self._value(kind)
        self.g.nodes.append(Node("binary", out, binop=op, inputs=[a, b]))
        return out

    def call(self, op: str, *args: Arg) -> Ref:
        ins = [self._arg(a) for a in args]
        out = self._value("tensor")
        kind = "primitive" if op in PRIMITIVE_OPS else "call"
        self.g.nodes.append(Node(kind, out, op=op, inputs=ins))
        return out

    def ctor(self, op: str, *args: Arg) -> Ref:
        if op not in LIBRARY_CTORS:
            raise ValueError(f"unknown layer constructor {op}")
        ins = [self._arg(a) for a in args]
        out = self._value("callable")
        self.g.nodes.append(Node("ctor", out, op=op, inputs=ins))
        return out

    def apply(self, callee: Ref, *args: Arg) -> Ref:
        ins = [callee] + [self._arg(a) for a in args]
        out = self._value("tensor")
        self.g.nodes.append(Node("apply", out, inputs=ins))
        return out

    # statements
    def let(self, name: str, value: Ref) -> Ref:
        """`name = expr` (VarDecl / Assign, ir/builder.rs:46-64): renames the value."""
        self.g.named[name] = int(value)
        self.g.values[value].name = name
        return value

    def ret(self, value: Ref) -> None:
        self.g.outputs.append(int(value))

    def train(self, objective: Optional[str] = None, lr: float = 0.01, iterations: int = 1,
              optimizer: str = "sgd") -> None:
        self.g.objective = objective
        self.g.lr = lr
        self.g.iterations = iterations
        self.g.optimizer = optimizer
        self.g.train_run = True

    def build(self) -> Graph:
        return self.g


def parse_shape_spec(spec: str):
    """`--shape name=AxBxC` (src/main.rs:98-120): split on 'x', each part a
    positive integer; errors carry the reference's messages."""
    eq = spec.find("=")
    if eq <= 0 or eq + 1 >= len(spec):
        raise ValueError(f"expected --shape name=dimxdim, got '{spec}'")
    name = spec[:eq]
    dims = []
    for part in spec[eq + 1:].split("x"):
        try:
            value = int(part.strip())
        except ValueError:
            raise ValueError(f"invalid dimension '{part}' in shape '{spec}'") from None
        if value <= 0:
            raise ValueError(f"invalid dimension '{part}' in shape '{spec}'")
        dims.append(value)
    return name, dims


def parse_shape_args(items: Sequence[str]) -> Dict[str, List[int]]:
    out: Dict[str, List[int]] = {}
    for item in items:
        name, dims = parse_shape_spec(item)
        out[name] = dims
    return out
