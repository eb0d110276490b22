"""Front end for tysor source (`.ty`): the subset the reference's hot-path
fixtures use, lowered to the graph IR (`graph.py`) in the reference
builder's value-id order, so parameter names such as `linear_{id}_weight`
(training/executor.rs:140-150) come out as the reference's do.

Accepted (src/compiler/parser.rs, frontend_ir.rs, ir/builder.rs):
  * `layer NAME(params): type:` and `fn NAME(params): type:` blocks; a
    parameter is `name[: type]`, a tensor annotation `tensor[dtype]`
    carries its dtype string;
  * statements `name = expr` and `return expr`;
  * expressions: literals (ints, floats, true / false, strings), names,
    `+ - * /` (usual precedence, left-associative), parentheses, calls
    `f(args)`, and pipelines `expr -> f(args) -> g()`;
  * `train NAME:` blocks of `key = value` lines (optimizer, lr,
    iteration, objective; other keys are kept and ignored);
  * `#` comments, blank lines, `config NAME:` blocks (`field : type =
    value`), whose fields are read as `NAME.field`.

Lowering follows the reference builder (ir/builder.rs:97-174): parameters
first, then each statement's expression in post-order; a literal argument
becomes a Constant node where it is met; a call of a builtin constructor
(`linear`, `SiLU`, `Softmax`, `Embedding`, `Dropout`, `RMSNorm`) is a
LibraryCtor, of a primitive (`matmul`, `relu`, `scale`) a PrimitiveCall, of a
library function (`rms_norm`, `cross_entropy`, `reshape`, `repeat_kv`,
`flatten_heads`, `causal_mask`, `rope`, `transpose`, `tied_logits`) a
LibraryCall, of a local variable an Apply.  A pipeline `a -> f(x) -> g()`
is the nested call `g()(f(x)(a))` for constructor stages (the constructor
is created, then its input lowered, then applied) and `f(a, x)` for
function stages.  Calls of user-defined layers are not inlined: the
reference lowers them to LibraryCall nodes its executors reject, and so
does this backend's executor.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple, Union

from .graph import LIBRARY_CALLS, LIBRARY_CTORS, PRIMITIVE_OPS, Graph, GraphBuilder, Ref


class TysorSyntaxError(ValueError):
    """A `.ty` program this front end cannot read (with its line number)."""


# ---- lexer -------------------------------------------------------------------

_TOKEN = re.compile(r"""
    (?P<num>\d+\.\d*(?:[eE][-+]?\d+)?|\d+[eE][-+]?\d+|\.\d+(?:[eE][-+]?\d+)?|\d+)
  | (?P<name>[A-Za-z_][A-Za-z0-9_]*)
  | (?P<str>"[^"\\n]*")
  | (?P<op>->|==|!=|<=|>=|[-+*/()\[\],:=.<>])
""", re.X)


@dataclass
class Tok:
    kind: str  # num name str op nl indent dedent eof
    text: str
    line: int


def tokenize(src: str) -> List[Tok]:
    toks: List[Tok] = []
    indents = [0]
    depth = 0  # open brackets: newlines inside them are not statement ends
    for ln, raw in enumerate(src.splitlines(), 1):
        line = raw.split("#", 1)[0].rstrip()
        if not line.strip():
            continue
        if depth == 0:
            width = len(line) - len(line.lstrip(" \t"))
            if width > indents[-1]:
                indents.append(width)
                toks.append(Tok("indent", "", ln))
            while width < indents[-1]:
                indents.pop()
                toks.append(Tok("dedent", "", ln))
            if width != indents[-1]:
                raise TysorSyntaxError(f"line {ln}: inconsistent indentation")
        pos = len(line) - len(line.lstrip(" \t"))
        while pos < len(line):
            if line[pos] in " \t":
                pos += 1
                continue
            m = _TOKEN.match(line, pos)
            if not m:
                raise TysorSyntaxError(f"line {ln}: unexpected character {line[pos]!r}")
            kind = m.lastgroup
            text = m.group(kind)
            if kind == "op" and text in "([":
                depth += 1
            elif kind == "op" and text in ")]":
                depth -= 1
            toks.append(Tok(kind, text, ln))
            pos = m.end()
        if depth == 0:
            toks.append(Tok("nl", "", ln))
    for _ in indents[1:]:
        toks.append(Tok("dedent", "", len(src.splitlines()) + 1))
    toks.append(Tok("eof", "", len(src.splitlines()) + 1))
    return toks


# ---- syntax tree ---------------------------------------------------------------

@dataclass
class Lit:
    value: Any  # int, float, bool, str, None


@dataclass
class Name:
    id: str
    line: int = 0


@dataclass
class Attr:
    base: str
    attr: str
    line: int = 0


@dataclass
class BinOp:
    op: str
    lhs: Any
    rhs: Any


@dataclass
class Call:
    func: str
    args: List[Any]
    kwargs: List[Tuple[str, Any]] = field(default_factory=list)
    line: int = 0


@dataclass
class Pipe:
    src: Any
    stages: List[Call]


@dataclass
class Param:
    name: str
    type_name: str = ""   # tensor / int / float / bool / "" (unannotated)
    dtype: str = ""       # tensor[dtype]


@dataclass
class Function:
    name: str
    params: List[Param]
    body: List[Tuple[str, Optional[str], Any, int]]  # ("assign", name, expr) / ("return", None, expr)
    is_layer: bool = True


@dataclass
class TrainRun:
    model: str
    settings: Dict[str, Any]


@dataclass
class Module:
    functions: Dict[str, Function]
    trains: Dict[str, TrainRun]
    configs: Dict[str, Dict[str, Any]]


# ---- parser --------------------------------------------------------------------

class _Parser:
    def __init__(self, toks: List[Tok]):
        self.t = toks
        self.i = 0

    def peek(self, k: int = 0) -> Tok:
        return self.t[min(self.i + k, len(self.t) - 1)]

    def next(self) -> Tok:
        tok = self.t[self.i]
        self.i += 1
        return tok

    def expect(self, kind: str, text: Optional[str] = None) -> Tok:
        tok = self.next()
        if tok.kind != kind or (text is not None and tok.text != text):
            want = text if text is not None else kind
            raise TysorSyntaxError(f"line {tok.line}: expected {want!r}, got {tok.text or tok.kind!r}")
        return tok

    def accept(self, kind: str, text: Optional[str] = None) -> bool:
        tok = self.peek()
        if tok.kind == kind and (text is None or tok.text == text):
            self.i += 1
            return True
        return False

    def module(self) -> Module:
        mod = Module({}, {}, {})
        while not self.accept("eof"):
            if self.accept("nl"):
                continue
            head = self.expect("name")
            if head.text in ("layer", "fn"):
                f = self.function(head.text == "layer")
                mod.functions[f.name] = f
            elif head.text == "train":
                tr = self.train()
                mod.trains[tr.model] = tr
            elif head.text == "config":
                name, fields = self.config()
                mod.configs[name] = fields
            else:
                raise TysorSyntaxError(f"line {head.line}: expected layer, fn, train or config, got {head.text!r}")
        return mod

    def type_ref(self) -> Tuple[str, str]:
        if self.accept("op", "("):
            while not self.accept("op", ")"):
                self.type_ref()
                self.accept("op", ",")
            return "tuple", ""
        name = self.expect("name").text
        dtype = ""
        if self.accept("op", "["):
            parts = []
            while not self.accept("op", "]"):
                parts.append(self.next().text)
            dtype = parts[0] if parts and parts[0] not in (",",) else ""
        return name, dtype

    def function(self, is_layer: bool) -> Function:
        name = self.expect("name").text
        self.expect("op", "(")
        params: List[Param] = []
        while not self.accept("op", ")"):
            pname = self.expect("name").text
            tname, dtype = "", ""
            if self.accept("op", ":"):
                tname, dtype = self.type_ref()
            if self.accept("op", "="):
                self.expr()
            params.append(Param(pname, tname, dtype))
            self.accept("op", ",")
        if self.accept("op", ":"):
            if not (self.peek().kind == "nl"):
                self.type_ref()
                self.expect("op", ":")
        self.expect("nl")
        self.expect("indent")
        body = []
        while not self.accept("dedent"):
            if self.accept("nl"):
                continue
            tok = self.peek()
            if tok.kind == "name" and tok.text == "return":
                self.next()
                body.append(("return", None, self.expr(), tok.line))
            elif tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == "=":
                self.next()
                self.next()
                body.append(("assign", tok.text, self.expr(), tok.line))
            else:
                raise TysorSyntaxError(f"line {tok.line}: expected an assignment or return")
            self.expect("nl")
        return Function(name, params, body, is_layer)

    def train(self) -> TrainRun:
        model = self.expect("name").text
        self.expect("op", ":")
        self.expect("nl")
        self.expect("indent")
        settings: Dict[str, Any] = {}
        while not self.accept("dedent"):
            if self.accept("nl"):
                continue
            key = self.expect("name").text
            self.expect("op", "=")
            settings[key] = self.expr()
            self.expect("nl")
        return TrainRun(model, settings)

    def config(self) -> Tuple[str, Dict[str, Any]]:
        name = self.expect("name").text
        self.expect("op", ":")
        self.expect("nl")
        self.expect("indent")
        fields: Dict[str, Any] = {}
        while not self.accept("dedent"):
            if self.accept("nl"):
                continue
            key = self.expect("name").text
            if self.accept("op", ":"):
                self.type_ref()
            self.expect("op", "=")
            value = self.expr()
            if not isinstance(value, Lit):
                raise TysorSyntaxError(f"config field {name}.{key}: expected a literal")
            fields[key] = value.value
            self.expect("nl")
        return name, fields

    # expressions: pipeline < additive < multiplicative < unary < call < atom
    def expr(self) -> Any:
        src = self.additive()
        stages = []
        while self.accept("op", "->"):
            stage = self.postfix()
            if not isinstance(stage, Call):
                raise TysorSyntaxError(f"line {self.peek().line}: a pipeline stage must be a call")
            stages.append(stage)
        return Pipe(src, stages) if stages else src

    def additive(self) -> Any:
        node = self.multiplicative()
        while self.peek().kind == "op" and self.peek().text in "+-" and self.peek().text != "->":
            op = self.next().text
            node = BinOp(op, node, self.multiplicative())
        return node

    def multiplicative(self) -> Any:
        node = self.unary()
        while self.peek().kind == "op" and self.peek().text in ("*", "/"):
            op = self.next().text
            node = BinOp(op, node, self.unary())
        return node

    def unary(self) -> Any:
        if self.peek().kind == "op" and self.peek().text == "-" and self.peek(1).kind == "num":
            self.next()
            v = self.atom()
            return Lit(-v.value)
        return self.postfix()

    def postfix(self) -> Any:
        tok = self.peek()
        if tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == "(":
            self.next()
            self.next()
            args, kwargs = [], []
            while not self.accept("op", ")"):
                if self.peek().kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == ":":
                    key = self.next().text
                    self.next()
                    kwargs.append((key, self.expr()))
                else:
                    args.append(self.expr())
                self.accept("op", ",")
            return Call(tok.text, args, kwargs, tok.line)
        if tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == ".":
            self.next()
            self.next()
            return Attr(tok.text, self.expect("name").text, tok.line)
        return self.atom()

    def atom(self) -> Any:
        tok = self.next()
        if tok.kind == "num":
            return Lit(float(tok.text) if any(c in tok.text for c in ".eE") else int(tok.text))
        if tok.kind == "str":
            return Lit(tok.text[1:-1])
        if tok.kind == "name":
            if tok.text in ("true", "True"):
                return Lit(True)
            if tok.text in ("false", "False"):
                return Lit(False)
            if tok.text == "None":
                return Lit(None)
            return Name(tok.text, tok.line)
        if tok.kind == "op" and tok.text == "(":
            node = self.expr()
            self.expect("op", ")")
            return node
        raise TysorSyntaxError(f"line {tok.line}: unexpected {tok.text or tok.kind!r}")


def parse(src: str) -> Module:
    return _Parser(tokenize(src)).module()


# ---- lowering ------------------------------------------------------------------

class _Lowerer:
    def __init__(self, mod: Module, fn: Function):
        self.mod = mod
        self.fn = fn
        self.b = GraphBuilder(fn.name)
        self.env: Dict[str, Ref] = {}

    def literal(self, node: Any) -> Any:
        """The Python value of a literal or config field, else None."""
        if isinstance(node, Lit):
            return node.value
        if isinstance(node, Attr) and node.base in self.mod.configs:
            cfg = self.mod.configs[node.base]
            if node.attr not in cfg:
                raise TysorSyntaxError(f"line {node.line}: unknown config field {node.base}.{node.attr}")
            return cfg[node.attr]
        return None

    def arg(self, node: Any) -> Union[Ref, int, float, bool]:
        """A call argument: literals stay Python values (the builder makes
        their Constant nodes where the call is lowered)."""
        v = self.literal(node)
        if v is not None and not isinstance(v, str):
            return v
        return self.value(node)

    def value(self, node: Any) -> Ref:
        if isinstance(node, Name):
            if node.id not in self.env:
                raise TysorSyntaxError(f"line {node.line}: unknown name {node.id!r}")
            return self.env[node.id]
        v = self.literal(node)
        if v is not None:
            if isinstance(v, str):
                raise TysorSyntaxError("a string is not a graph value")
            return self.b.const(v)
        if isinstance(node, BinOp):
            return self.b.binary(node.op, self.arg(node.lhs), self.arg(node.rhs))
        if isinstance(node, Call):
            return self.call(node, None)
        if isinstance(node, Pipe):
            return self.pipe(node.src, node.stages)
        raise TysorSyntaxError(f"cannot lower {node!r}")

    def pipe(self, src: Any, stages: List[Call]) -> Ref:
        # a -> s1 -> ... -> sn is sn(...s1(a)...), lowered outermost callee first.
        if not stages:
            return self.value(src)
        *inner, last = stages
        return self.call(last, (src, inner))

    def call(self, node: Call, piped) -> Ref:
        if node.kwargs:
            raise TysorSyntaxError(f"line {node.line}: keyword arguments are not supported ({node.func})")
        f = node.func

        def piped_input() -> Ref:
            src, inner = piped
            return self.pipe(src, inner)

        if f in self.env:
            # calling a constructed layer: Apply(callee, input)
            if piped is not None:
                if node.args:
                    raise TysorSyntaxError(f"line {node.line}: a layer stage takes no arguments")
                return self.b.apply(self.env[f], piped_input())
            if len(node.args) != 1:
                raise TysorSyntaxError(f"line {node.line}: a layer takes one input")
            return self.b.apply(self.env[f], self.value(node.args[0]))
        if f in LIBRARY_CTORS:
            ctor = self.b.ctor(f, *[self.arg(a) for a in node.args])
            if piped is not None:
                return self.b.apply(ctor, piped_input())
            return ctor
        if f in PRIMITIVE_OPS or f in LIBRARY_CALLS or f == "tied_logits":
            args = ([piped_input()] if piped is not None else []) + [self.arg(a) for a in node.args]
            return self.b.call(f, *args)
        if f in self.mod.functions:
            raise TysorSyntaxError(f"line {node.line}: calls of user-defined layers ({f}) are not inlined; "
                                   "the executor runs only library operations")
        raise TysorSyntaxError(f"line {node.line}: unknown function {f!r}")

    def lower(self, train: Optional[TrainRun]) -> Graph:
        for p in self.fn.params:
            if p.type_name not in ("", "tensor"):
                raise TysorSyntaxError(f"parameter {p.name}: only tensor parameters are supported")
            self.env[p.name] = self.b.param(p.name, p.dtype)
        returned = False
        for kind, name, expr, line in self.fn.body:
            if kind == "assign":
                self.env[name] = self.b.let(name, self.value(expr))
            else:
                self.b.ret(self.value(expr))
                returned = True
        if not returned:
            raise TysorSyntaxError(f"{self.fn.name}: no return")
        if train is not None:
            s = train.settings
            obj = s.get("objective")
            lr = self.literal(s["lr"]) if "lr" in s else 0.01
            it = self.literal(s["iteration"]) if "iteration" in s else 1
            opt = self.literal(s["optimizer"]) if "optimizer" in s else "sgd"
            self.b.train(objective=obj.id if isinstance(obj, Name) else None, lr=float(lr),
                         iterations=int(it), optimizer=str(opt))
        return self.b.build()


def lower(src: str, entry: str = "model") -> Graph:
    """The lowered graph of function `entry` of a `.ty` program, with the
    program's `train entry:` settings (objective, lr, iterations, optimizer)
    when it has them."""
    mod = parse(src)
    if entry not in mod.functions:
        raise TysorSyntaxError(f"Entry function '{entry}' not found in lowered module")
    return _Lowerer(mod, mod.functions[entry]).lower(mod.trains.get(entry))
