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
    `f(args)`, and pipelines `expr -> f(args) -> g()`, whose stages may be
    repeated (`f()[n]`: n applications, n known while lowering) or be
    expressions over calls (`x -> relu()[2] * 2`: the calls take the piped
    value, frontend_ir.rs:730-786);
  * `train NAME:` blocks of `key = value` lines (optimizer, lr or
    learning_rate, iteration, objective; other keys are kept and ignored);
    a tuple value makes one run per element, of which the executor trains
    the first (frontend_ir.rs:1108-1125, training/executor.rs:132-138);
  * `#` comments, blank lines, lines starting with `->` (they continue the
    pipeline above), `config NAME:` blocks (`field : type = value`), whose
    fields are read as `NAME.field`.

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
function stages.

Extensions for `examples/llama.ty`-style programs (the reference lowers
none of them to something its executors run: frontend_ir.rs:708-727 makes
a user layer's call a LibraryCall, ir/builder.rs:174 has no conditional,
semantic_analyzer.rs:427-442 knows only declared config fields):
  * user-layer inlining -- a call `F(args)` or stage `x -> F(args)` of a
    user `layer` / `fn` lowers F's body in place, its parameters bound to
    the piped input and the arguments (graph values, or compile-time values
    for literal and config arguments) or to their literal defaults; each
    call makes its own constructors (parameters); recursion is an error;
  * `scale(x, d, h)` -- x times 1 / sqrt(d / h) (attention's 1/sqrt(head
    dim) for width d over h heads; d and h known while lowering); the
    two-argument `scale(x, c)` is the reference's primitive;
  * `config.field` -- a field of the program's only config block, and a
    derived `head_dim` = hidden_dim / n_heads where a config declares those
    two and not head_dim;
  * `a if test else b` -- decided while lowering: a literal, config field or
    comparison of those, or the name of an input (true when the caller
    supplies it; an entry parameter `p=None` the caller does not supply has
    no value); `None` leaves a name without value, and `return a, b` drops a
    None entry;
  * integer arithmetic on compile-time integers in call arguments folds to
    an integer (sizes, counts);
  * a user layer named like a library constructor or function (llama.ty's
    own `RMSNorm`) is the one called.
With these, the reference's examples/llama.ty lowers.
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
  | (?P<op>->|==|!=|<=|>=|&&|\|\||[-+*/()\[\],:=.<>!])
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
        # A line that starts with `->` continues the previous line's pipeline.
        cont = depth == 0 and line.lstrip(" \t").startswith("->") and bool(toks) and toks[-1].kind == "nl"
        if cont:
            toks.pop()
        if depth == 0 and not cont:
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
class Repeat:
    """`f(args)[n]` in a pipeline: the stage applied n times."""
    call: Call
    count: Any
    line: int = 0


@dataclass
class Compare:
    op: str
    lhs: Any
    rhs: Any


@dataclass
class Logic:
    op: str  # "&&" or "||"
    lhs: Any
    rhs: Any


@dataclass
class Not:
    operand: Any


@dataclass
class Cond:
    then: Any
    test: Any
    other: Any
    line: int = 0


@dataclass
class TupleExpr:
    items: List[Any]


NO_DEFAULT = object()


@dataclass
class Param:
    name: str
    type_name: str = ""   # tensor / int / float / bool / "" (unannotated)
    dtype: str = ""       # tensor[dtype]
    default: Any = NO_DEFAULT  # the expression after `=`


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


# Train fields that may hold a tuple of per-run values (one run per
# element, scalars broadcast: frontend_ir.rs:1037-1068, 1108-1125).
TRAIN_VARIANT_FIELDS = ("backend", "target", "device", "optimizer", "lr", "learning_rate", "objective", "iteration")


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
            # tensor[dtype, dims...]: the dtype is the first item; the dims
            # (which may hold brackets, `TransformerDims[:2]`) are skipped.
            parts, depth = [], 1
            while True:
                tok = self.next()
                if tok.kind in ("eof", "nl"):
                    raise TysorSyntaxError(f"line {tok.line}: unclosed '[' in a type")
                if tok.kind == "op" and tok.text == "[":
                    depth += 1
                elif tok.kind == "op" and tok.text == "]":
                    depth -= 1
                    if depth == 0:
                        break
                parts.append(tok.text)
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
            default = NO_DEFAULT
            if self.accept("op", "="):
                default = self.expr()
            params.append(Param(pname, tname, dtype, default))
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
                value = self.expr()
                if self.peek().kind == "op" and self.peek().text == ",":
                    items = [value]
                    while self.accept("op", ","):
                        items.append(self.expr())
                    value = TupleExpr(items)
                body.append(("return", None, value, tok.line))
            elif tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == "=":
                self.next()
                self.next()
                body.append(("assign", tok.text, self.expr(), tok.line))
            elif tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == ":":
                # `name : type = value`: the annotation is not checked here.
                self.next()
                self.next()
                self.type_ref()
                self.expect("op", "=")
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
        arity: Optional[int] = None
        while not self.accept("dedent"):
            if self.accept("nl"):
                continue
            tok = self.expect("name")
            key = tok.text
            self.expect("op", "=")
            value = self.expr()
            if self.peek().kind == "op" and self.peek().text == ",":
                items = [value]
                while self.accept("op", ","):
                    items.append(self.expr())
                value = TupleExpr(items)
            self.expect("nl")
            # The reference's checks of a train declaration
            # (semantic_analyzer.rs:808-850, frontend_ir.rs:1069-1081).
            if key in settings:
                raise TysorSyntaxError(f"line {tok.line}: Duplicate field '{key}' in train '{model}'")
            if key == "subtrain":
                raise TysorSyntaxError(f"line {tok.line}: Field 'subtrain' is no longer supported; use "
                                       "tuple-valued fields on 'train model' instead")
            if isinstance(value, TupleExpr):
                if key not in TRAIN_VARIANT_FIELDS:
                    raise TysorSyntaxError(f"line {tok.line}: Train field '{key}' does not support tuple "
                                           "variants; use a scalar value")
                if not value.items:
                    raise TysorSyntaxError(f"line {tok.line}: Train field '{key}' cannot use an empty tuple")
                if arity is not None and arity != len(value.items):
                    raise TysorSyntaxError(f"line {tok.line}: Tuple-valued train fields must have the same "
                                           "length; use scalar values to broadcast")
                arity = len(value.items)
            settings[key] = value
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

    # expressions: conditional < pipeline < additive < multiplicative < unary < call < atom
    def expr(self) -> Any:
        line = self.peek().line
        node = self.pipeline()
        if self.peek().kind == "name" and self.peek().text == "if":
            self.next()
            test = self.logic_or()
            self.expect("name", "else")
            return Cond(node, test, self.expr(), line)
        return node

    def pipeline(self) -> Any:
        # The operands of `->` are conditions or arithmetic (parser.rs:333-352);
        # a condition lowers only where one is decided (`a if test else b`).
        src = self.logic_or()
        stages = []
        while self.accept("op", "->"):
            line = self.peek().line
            stage = self.logic_or()
            if not _has_stage(stage):
                raise TysorSyntaxError(f"line {line}: a pipeline stage must be a call")
            stages.append(stage)
        return Pipe(src, stages) if stages else src

    # A condition: `||` over `&&` over one comparison, left-associative (the
    # reference's precedence, compiler/parser.rs:351-361).
    def logic_or(self) -> Any:
        node = self.logic_and()
        while self.accept("op", "||"):
            node = Logic("||", node, self.logic_and())
        return node

    def logic_and(self) -> Any:
        node = self.comparison()
        while self.accept("op", "&&"):
            node = Logic("&&", node, self.comparison())
        return node

    def comparison(self) -> Any:
        node = self.additive()
        if self.peek().kind == "op" and self.peek().text in ("==", "!=", "<", ">", "<=", ">="):
            op = self.next().text
            node = Compare(op, node, self.additive())
        return node

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
        if self.peek().kind == "op" and self.peek().text == "-":
            # -e is the binary 0 - e, as the reference lowers a unary minus
            # (compiler/frontend_ir.rs:606-615, parser.rs:402-409).
            self.next()
            return BinOp("-", Lit(0), self.unary())
        if self.accept("op", "!"):
            return Not(self.unary())
        return self.postfix()

    def postfix(self) -> Any:
        tok = self.peek()
        if tok.kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == "(":
            self.next()
            self.next()
            args, kwargs = [], []
            while not self.accept("op", ")"):
                if self.peek().kind == "name" and self.peek(1).kind == "op" and self.peek(1).text == ":":
                    # `name: value`: the reference's builder keeps the value in
                    # its written position and drops the name (ir/builder.rs:119-123).
                    key = self.next().text
                    self.next()
                    value = self.expr()
                    kwargs.append((key, value))
                    args.append(value)
                else:
                    args.append(self.expr())
                self.accept("op", ",")
            call = Call(tok.text, args, kwargs, tok.line)
            if self.peek().kind == "op" and self.peek().text == "[":
                self.next()
                count = self.expr()
                self.expect("op", "]")
                return Repeat(call, count, tok.line)
            return call
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
            if self.accept("op", ")"):
                return TupleExpr([])
            node = self.expr()
            if self.peek().kind == "op" and self.peek().text == ",":
                # (a, b, ...): a tuple, as the reference parses a bracketed
                # expression list (parser.rs:299-311).
                items = [node]
                while self.accept("op", ","):
                    if self.peek().kind == "op" and self.peek().text == ")":
                        break
                    items.append(self.expr())
                node = TupleExpr(items)
            self.expect("op", ")")
            return node
        raise TysorSyntaxError(f"line {tok.line}: unexpected {tok.text or tok.kind!r}")


def _has_stage(node: Any) -> bool:
    """Whether a pipeline stage expression applies something to the piped
    value: a call, a repeated call, or +, -, *, / of expressions with one."""
    if isinstance(node, (Call, Repeat)):
        return True
    if isinstance(node, BinOp):
        return _has_stage(node.lhs) or _has_stage(node.rhs)
    return False


def _identifiers(node: Any, out: set) -> None:
    """The names an expression mentions, callees excluded (the reference's
    collect_expr_identifiers, semantic_analyzer.rs:1090-1129)."""
    if isinstance(node, Name):
        out.add(node.id)
    elif isinstance(node, Attr):
        out.update((node.base, node.attr))
    elif isinstance(node, Call):
        for a in node.args:
            _identifiers(a, out)
    elif isinstance(node, (BinOp, Compare, Logic)):
        _identifiers(node.lhs, out)
        _identifiers(node.rhs, out)
    elif isinstance(node, Not):
        _identifiers(node.operand, out)
    elif isinstance(node, Cond):
        for part in (node.then, node.test, node.other):
            _identifiers(part, out)
    elif isinstance(node, TupleExpr):
        for item in node.items:
            _identifiers(item, out)
    elif isinstance(node, Pipe):
        for part in [node.src] + list(node.stages):
            _identifiers(part, out)
    elif isinstance(node, Repeat):
        _identifiers(node.call, out)
        _identifiers(node.count, out)


def _check_objectives(mod: Module) -> None:
    """A train block's objective is a bare name and, when the program has a
    `layer model`, one of the symbols of that layer: its parameters, the
    names it assigns and the names its expressions mention
    (semantic_analyzer.rs:850-875, 880-893)."""
    model = mod.functions.get("model")
    symbols: set = set()
    if model is not None and model.is_layer:
        symbols.update(p.name for p in model.params)
        for kind, name, value, _ in model.body:
            if kind == "assign":
                symbols.add(name)
            _identifiers(value, symbols)
    for tr in mod.trains.values():
        obj = tr.settings.get("objective")
        if obj is None:
            continue
        for item in (obj.items if isinstance(obj, TupleExpr) else [obj]):
            if not isinstance(item, Name):
                raise TysorSyntaxError("Field 'objective' must reference a named tensor root, not a string "
                                       "literal or arbitrary expression")
            if symbols and item.id not in symbols:
                raise TysorSyntaxError(f"Field 'objective' references unknown model root '{item.id}'")


def parse(src: str) -> Module:
    mod = _Parser(tokenize(src)).module()
    _check_objectives(mod)
    return mod


# ---- lowering ------------------------------------------------------------------

@dataclass
class Const:
    """A compile-time value bound to a name (a literal or config argument of
    an inlined layer, or a parameter's literal default)."""
    value: Any


_ABSENT = object()  # a name bound to `None`: no graph value


@dataclass
class _TrainName:
    """A bare name as a train field's value (`optimizer = sgd`,
    `objective = loss`)."""
    name: str


class _Lowerer:
    def __init__(self, mod: Module, fn: Function, provided: Optional[set] = None):
        self.mod = mod
        self.fn = fn
        self.b = GraphBuilder(fn.name)
        self.env: Dict[str, Any] = {}
        self.provided = provided
        self.stack: List[str] = [fn.name]  # functions being lowered (inlining)
        self.prefix = ""                   # named-value prefix of the inlined body
        self.inlined = 0

    # -- compile-time values ----------------------------------------------------
    def config_field(self, node: Attr) -> Any:
        if node.base == "config":
            if len(self.mod.configs) != 1:
                raise TysorSyntaxError(f"line {node.line}: `config.{node.attr}` needs exactly one config block "
                                       f"({len(self.mod.configs)} declared)")
            cfg = next(iter(self.mod.configs.values()))
        else:
            cfg = self.mod.configs[node.base]
        if node.attr in cfg:
            return cfg[node.attr]
        if node.attr == "head_dim" and "hidden_dim" in cfg and "n_heads" in cfg:
            d, h = cfg["hidden_dim"], cfg["n_heads"]
            if not (isinstance(d, int) and isinstance(h, int) and h > 0 and d % h == 0):
                raise TysorSyntaxError(f"line {node.line}: head_dim: hidden_dim {d} is not a multiple of n_heads {h}")
            return d // h
        raise TysorSyntaxError(f"line {node.line}: unknown config field {node.base}.{node.attr}")

    def const_value(self, node: Any) -> Tuple[bool, Any]:
        """(True, value) when `node` is known while lowering: a literal, a
        config field, a name bound to one, or +, -, *, / and comparisons of
        those (Python arithmetic on the values)."""
        if isinstance(node, Lit):
            return True, node.value
        if isinstance(node, Attr) and (node.base in self.mod.configs or node.base == "config"):
            return True, self.config_field(node)
        if isinstance(node, Name) and isinstance(self.env.get(node.id), Const):
            return True, self.env[node.id].value
        if isinstance(node, (BinOp, Compare)):
            ok1, l = self.const_value(node.lhs)
            ok2, r = self.const_value(node.rhs)
            if not (ok1 and ok2) or isinstance(l, str) or isinstance(r, str) or l is None or r is None:
                return False, None
            ops = {"+": lambda: l + r, "-": lambda: l - r, "*": lambda: l * r, "/": lambda: l / r,
                   "==": lambda: l == r, "!=": lambda: l != r, "<": lambda: l < r, ">": lambda: l > r,
                   "<=": lambda: l <= r, ">=": lambda: l >= r}
            return True, ops[node.op]()
        if isinstance(node, Not):
            ok, v = self.const_value(node.operand)
            return (True, not v) if ok and not isinstance(v, str) and v is not None else (False, None)
        if isinstance(node, Logic):
            ok1, l = self.const_value(node.lhs)
            ok2, r = self.const_value(node.rhs)
            if not (ok1 and ok2) or any(isinstance(x, str) or x is None for x in (l, r)):
                return False, None
            return True, (bool(l) and bool(r)) if node.op == "&&" else (bool(l) or bool(r))
        return False, None

    def literal(self, node: Any) -> Any:
        """The Python value of a literal, a config field or a name bound to a
        compile-time value, else None."""
        if isinstance(node, (Lit, Attr)) or (isinstance(node, Name) and isinstance(self.env.get(node.id), Const)):
            ok, v = self.const_value(node)
            return v if ok else None
        return None

    def test(self, node: Any, line: int) -> bool:
        """The condition of `a if test else b`, decided while lowering: a
        compile-time value, the name of a graph input (true when the caller
        supplies it), or `!`, `&&` and `||` of those."""
        if isinstance(node, Name) and node.id in self.env and not isinstance(self.env[node.id], Const):
            return self.env[node.id] is not _ABSENT
        if isinstance(node, Not):
            return not self.test(node.operand, line)
        if isinstance(node, Logic):
            # Both sides are decided (nothing is evaluated at run time).
            l, r = self.test(node.lhs, line), self.test(node.rhs, line)
            return (l and r) if node.op == "&&" else (l or r)
        ok, v = self.const_value(node)
        if not ok:
            raise TysorSyntaxError(f"line {line}: the condition of `if ... else` must be known while lowering "
                                   "(a literal, a config field, a comparison of those, or an input's name)")
        return bool(v)

    # -- graph values -----------------------------------------------------------
    def arg(self, node: Any) -> Union[Ref, int, float, bool]:
        """A call argument: literals stay Python values (the builder makes
        their Constant nodes where the call is lowered).  Integer arithmetic
        on compile-time integers (`n_kv_heads * config.head_dim`, `n_heads /
        n_kv_heads` when it divides) folds to an integer argument, as sizes
        and counts need; the reference lowers it to a scalar Binary node,
        whose Float its constructors reject."""
        v = self.literal(node)
        if v is not None and not isinstance(v, str):
            return v
        if isinstance(node, BinOp):
            ok, v = self.const_value(node)
            ints = ok and all(isinstance(x, int) and not isinstance(x, bool)
                              for x in (self.const_value(node.lhs)[1], self.const_value(node.rhs)[1]))
            if ints and (node.op != "/" or float(v).is_integer()):
                return int(v)
        return self.value(node)

    def value_or_absent(self, node: Any) -> Any:
        """The value of the right side of an assignment or of a returned
        expression, which may be None (`_ABSENT`): a `None` literal, a name
        bound to None, or a conditional choosing either."""
        if isinstance(node, Cond):
            return self.value_or_absent(node.then if self.test(node.test, node.line) else node.other)
        if isinstance(node, Lit) and node.value is None:
            return _ABSENT
        if isinstance(node, Name) and self.env.get(node.id, None) is _ABSENT:
            return _ABSENT
        return self.value(node)

    def value(self, node: Any) -> Any:
        """A graph value (never None)."""
        if isinstance(node, Cond):
            return self.value(node.then if self.test(node.test, node.line) else node.other)
        if isinstance(node, Name):
            if node.id not in self.env:
                raise TysorSyntaxError(f"line {node.line}: unknown name {node.id!r}")
            v = self.env[node.id]
            if v is _ABSENT:
                raise TysorSyntaxError(f"line {node.line}: {node.id!r} is None here")
            if isinstance(v, Const):
                return self.b.const(v.value)
            return v
        if isinstance(node, Lit) and node.value is None:
            raise TysorSyntaxError("None is not a graph value here")
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
        if isinstance(node, Repeat):
            raise TysorSyntaxError(f"line {node.line}: `f()[n]` repeats a pipeline stage; it needs a piped input")
        if isinstance(node, (Compare, Logic, Not)):
            raise TysorSyntaxError("a comparison or logical expression is a condition of `if ... else`, "
                                   "not a graph value")
        raise TysorSyntaxError(f"cannot lower {node!r}")

    def pipe(self, src: Any, stages: List[Any]) -> Ref:
        # a -> s1 -> ... -> sn is sn(...s1(a)...), lowered outermost callee first
        # (as the reference's builder meets them); `f()[n]` is n stages f().
        if not stages:
            return self.value(src)
        flat: List[Any] = []
        for st in stages:
            if isinstance(st, Repeat):
                flat += [st.call] * self.repeat_count(st)
            else:
                flat.append(st)
        if not flat:
            return self.value(src)
        *inner, last = flat
        return self.stage(last, (src, inner))

    def repeat_count(self, st: Repeat) -> int:
        ok, n = self.const_value(st.count)
        if not ok or not isinstance(n, int) or isinstance(n, bool) or n < 0:
            raise TysorSyntaxError(f"line {st.line}: a stage repetition count must be a non-negative integer "
                                   "known while lowering")
        return n

    def piped_value(self, piped) -> Ref:
        if isinstance(piped, tuple):
            src, inner = piped
            return self.pipe(src, inner)
        return piped

    def stage(self, st: Any, piped) -> Ref:
        """One pipeline stage applied to the piped value (a (source, inner
        stages) pair lowered when the stage needs it, or a lowered value):
        a call; a repeated call; or a binary expression whose operands with
        calls in them are stages on the same piped value (lowered once) and
        whose others are plain values (frontend_ir.rs:730-786)."""
        if isinstance(st, Call):
            return self.call(st, piped)
        if isinstance(st, Repeat):
            n = self.repeat_count(st)
            cur = piped
            for _ in range(n):
                cur = self.call(st.call, cur)
            return self.piped_value(cur)
        if isinstance(st, BinOp):
            cur = self.piped_value(piped)
            lhs = self.stage(st.lhs, cur) if _has_stage(st.lhs) else self.arg(st.lhs)
            rhs = self.stage(st.rhs, cur) if _has_stage(st.rhs) else self.arg(st.rhs)
            return self.b.binary(st.op, lhs, rhs)
        raise TysorSyntaxError(f"cannot use {st!r} as a pipeline stage")

    def call(self, node: Call, piped) -> Ref:
        f = node.func

        def piped_input() -> Ref:
            return self.piped_value(piped)

        if f in self.env and not isinstance(self.env[f], Const):
            # calling a constructed layer: Apply(callee, input)
            if piped is not None:
                if node.args:
                    raise TysorSyntaxError(f"line {node.line}: a layer stage takes no arguments")
                return self.b.apply(self.env[f], piped_input())
            if len(node.args) != 1:
                raise TysorSyntaxError(f"line {node.line}: a layer takes one input")
            return self.b.apply(self.env[f], self.value(node.args[0]))
        if f in self.mod.functions:
            # A user layer shadows a library name (examples/llama.ty defines its own RMSNorm).
            return self.inline(self.mod.functions[f], node, piped_input() if piped is not None else None)
        if f in LIBRARY_CTORS:
            ctor = self.b.ctor(f, *[self.arg(a) for a in node.args])
            if piped is not None:
                return self.b.apply(ctor, piped_input())
            return ctor
        if f == "scale" and len(node.args) + (piped is not None) == 3:
            # scale(x, d, h): x * 1 / sqrt(d / h), attention's 1 / sqrt(head_dim)
            # for a width d split over h heads (d and h known while lowering).
            x = piped_input() if piped is not None else self.value(node.args[0])
            dims = node.args[-2:]
            vals = [self.const_value(d) for d in dims]
            if not all(ok and isinstance(v, (int, float)) and not isinstance(v, bool) for ok, v in vals):
                raise TysorSyntaxError(f"line {node.line}: scale(x, d, h) needs d and h known while lowering")
            d, h = float(vals[0][1]), float(vals[1][1])
            if d <= 0 or h <= 0:
                raise TysorSyntaxError(f"line {node.line}: scale(x, d, h) needs d > 0 and h > 0")
            return self.b.call("scale", x, 1.0 / ((d / h) ** 0.5))
        if f in PRIMITIVE_OPS or f in LIBRARY_CALLS or f == "tied_logits":
            args = ([piped_input()] if piped is not None else []) + [self.arg(a) for a in node.args]
            return self.b.call(f, *args)
        raise TysorSyntaxError(f"line {node.line}: unknown function {f!r}")

    def inline(self, fn: Function, node: Call, piped: Optional[Ref]) -> Ref:
        """A call of a user-defined layer or fn, lowered in place: its
        parameters are bound in order to the piped input (if any) and the
        call's arguments -- graph values, or compile-time values for literal
        and config arguments -- or to their literal defaults; its body's
        constructors make new parameters at every call; its named values are
        prefixed `Name.k.` (k counts inlined calls); its return is the call's
        value."""
        if fn.name in self.stack:
            raise TysorSyntaxError(f"line {node.line}: recursive call of {fn.name!r}")
        actual: List[Any] = ([piped] if piped is not None else [])
        for a in node.args:
            ok, v = self.const_value(a)
            actual.append(Const(v) if ok and not isinstance(v, str) else self.value(a))
        if len(actual) > len(fn.params):
            raise TysorSyntaxError(f"line {node.line}: {fn.name} takes {len(fn.params)} arguments, "
                                   f"{len(actual)} given")
        local: Dict[str, Any] = {}
        for i, p in enumerate(fn.params):
            if i < len(actual):
                local[p.name] = actual[i]
            elif p.default is not NO_DEFAULT:
                ok, v = self.const_value(p.default)
                if not ok:
                    raise TysorSyntaxError(f"{fn.name}: the default of {p.name} must be a literal")
                local[p.name] = _ABSENT if v is None else Const(v)
            else:
                raise TysorSyntaxError(f"line {node.line}: {fn.name}: missing argument {p.name!r}")
        saved = (self.env, self.prefix)
        self.env = local
        self.prefix = f"{saved[1]}{fn.name}.{self.inlined}."
        self.inlined += 1
        self.stack.append(fn.name)
        try:
            result = self.body(fn)
        finally:
            self.stack.pop()
            self.env, self.prefix = saved
        if result is None or isinstance(result, list):
            raise TysorSyntaxError(f"line {node.line}: {fn.name} must return one value to be called")
        return result

    def body(self, fn: Function) -> Any:
        """Lowers fn's statements into the graph; returns its return value
        (a list for a tuple return; None without a return)."""
        for kind, name, expr, line in fn.body:
            if kind == "assign":
                v = self.value_or_absent(expr)
                self.env[name] = v if v is _ABSENT else self.b.let(self.prefix + name, v)
            else:
                if isinstance(expr, TupleExpr):
                    # an entry without value (None) is dropped from the outputs
                    return [self.value_or_absent(e) for e in expr.items]
                v = self.value_or_absent(expr)
                if v is _ABSENT:
                    raise TysorSyntaxError(f"line {line}: {fn.name} returns None")
                return v
        return None

    def lower(self, train: Optional[TrainRun]) -> Graph:
        for p in self.fn.params:
            if p.type_name not in ("", "tensor"):
                raise TysorSyntaxError(f"parameter {p.name}: only tensor parameters are supported")
            supplied = self.provided is None or p.name in self.provided
            if not supplied and p.default is not NO_DEFAULT and isinstance(p.default, Lit) and p.default.value is None:
                self.env[p.name] = _ABSENT  # an optional input the caller did not supply
            else:
                self.env[p.name] = self.b.param(p.name, p.dtype)
        result = self.body(self.fn)
        if result is None:
            raise TysorSyntaxError(f"{self.fn.name}: no return")
        for r in (result if isinstance(result, list) else [result]):
            if r is not _ABSENT:
                self.b.ret(r)
        if train is not None:
            # The executor trains the first run of the block
            # (training/executor.rs:132-138, 774-790): each field's first
            # tuple element; lr an int or float (else 0.01), iteration an
            # int (else 1), optimizer a name or string (else "sgd").
            fields: Dict[str, Any] = {}
            for key, node in train.settings.items():
                key = "lr" if key == "learning_rate" else key
                if key in ("objective", "lr", "iteration", "optimizer"):  # the others are not read
                    fields[key] = self.train_value(node.items[0] if isinstance(node, TupleExpr) else node)
            obj, lr, it, opt = (fields.get(k) for k in ("objective", "lr", "iteration", "optimizer"))
            if isinstance(opt, _TrainName):
                opt = opt.name
            is_int = lambda v: isinstance(v, int) and not isinstance(v, bool)
            self.b.train(objective=obj.name if isinstance(obj, _TrainName) else None,
                         lr=float(lr) if is_int(lr) or isinstance(lr, float) else 0.01,
                         iterations=it if is_int(it) else 1,
                         optimizer=opt if isinstance(opt, str) else "sgd")
        return self.b.build()

    def train_value(self, node: Any) -> Any:
        """A train field's value: a bare name stands for itself (the
        reference evaluates an identifier to its name,
        frontend_ir.rs:1170-1176), anything else must be known while
        lowering."""
        if isinstance(node, Name):
            return _TrainName(node.id)
        ok, v = self.const_value(node)
        if not ok:
            raise TysorSyntaxError("a train field's value must be a name or known while lowering")
        return v


def lower(src: str, entry: str = "model", inputs: Optional[List[str]] = None) -> Graph:
    """The lowered graph of function `entry` of a `.ty` program, with the
    settings of the program's `train model:` block (objective, lr,
    iterations, optimizer) when the entry is `layer model` and the block
    exists (else Graph.train_run is false).  `inputs`: the graph inputs the caller supplies (the
    CLI's `--shape` names); an entry parameter whose default is `None` and
    that is not among them has no graph value (`x if targets else y` then
    takes y).  None: every parameter is an input."""
    mod = parse(src)
    if entry not in mod.functions:
        raise TysorSyntaxError(f"Entry function '{entry}' not found in lowered module")
    provided = None if inputs is None else set(inputs)
    fn = mod.functions[entry]
    # The reference plans train runs only for `layer model` with `train
    # model`, and its executor trains the run of the entry
    # (frontend_ir.rs:458-465, training/executor.rs:132-138).
    train = mod.trains.get("model") if entry == "model" and fn.is_layer else None
    return _Lowerer(mod, fn, provided).lower(train)
