"""`python -m tysor_b200 <input.ty> [--run] [--backward] [--train] [--backend cuda]
[--shape name=AxB ...] [--entry name]`: the reference CLI's execution paths
(src/main.rs:44-96, 268-312) on the CUDA backend.

The flags, the `--shape` syntax and errors, the exit codes (2 for a bad
command line, 1 for a failed program) and the printed sections
(`--- Execution Output ---`, `--- Gradient Output ---`, `--- Training
Output ---`) are the reference's; the program is read by `frontend.py` (the
hot-path subset of the DSL) and runs on the device through the C ABI.
`--backend` accepts `cuda` only: the reference's other backends are not part
of this build, and there is no CPU fallback.  TYSOR_CUDA_DEVICE picks the
device (default 0); TYSOR_DUMP_DIR also writes every printed result as raw
f32 (runtime.py).
"""
from __future__ import annotations

import os
import sys
from typing import List, Optional

from .frontend import TysorSyntaxError, lower
from .graph import parse_shape_spec

USAGE = ("tysor <input.ty> [--run] [--backward] [--train] [--entry <name>] [--backend <cuda>] "
         "[--shape <name>=<dim>x<dim>...]")
REFERENCE_BACKENDS = ("local", "metal", "pytorch")
# The reference CLI's compiler-introspection and code-emission flags
# (src/main.rs:57-66): they print the reference compiler's stages, which
# this build does not include.
REFERENCE_COMPILER_FLAGS = ("--emit-metal", "--emit-pytorch", "--tokens", "--ast", "--semantics", "--ir",
                            "--print-pipeline")


class CliError(ValueError):
    pass


def parse_cli(argv: List[str]):
    opts = {"input": None, "run": False, "backward": False, "train": False, "entry": "model",
            "backend": "cuda", "shapes": {}}
    args = list(argv)
    while args:
        a = args.pop(0)
        if a in ("--run", "--backward", "--train"):
            opts[a[2:]] = True
        elif a == "--entry":
            if not args:
                raise CliError("missing value for --entry")
            opts["entry"] = args.pop(0)
        elif a == "--backend":
            if not args:
                raise CliError("missing value for --backend")
            b = args.pop(0)
            if b in REFERENCE_BACKENDS:
                raise CliError(f"backend '{b}' is not part of this build: it runs the cuda backend")
            if b != "cuda":
                raise CliError(f"unsupported backend '{b}'")
            opts["backend"] = b
        elif a == "--shape":
            if not args:
                raise CliError("missing value for --shape")
            try:
                name, dims = parse_shape_spec(args.pop(0))
            except ValueError as e:
                raise CliError(str(e)) from None
            opts["shapes"][name] = dims
        elif a in REFERENCE_COMPILER_FLAGS:
            raise CliError(f"option {a} belongs to the reference compiler, which this build does not include")
        elif a.startswith("--"):
            raise CliError(f"unknown option: {a}")
        else:
            if opts["input"] is not None:
                raise CliError("multiple input paths provided")
            opts["input"] = a
    if opts["input"] is None:
        raise CliError("missing input path")
    return opts


def main(argv: Optional[List[str]] = None) -> int:
    try:
        opts = parse_cli(sys.argv[1:] if argv is None else argv)
    except CliError as e:
        print(f"error: {e}", file=sys.stderr)
        print(f"usage: {USAGE}", file=sys.stderr)
        return 2
    try:
        with open(opts["input"]) as f:
            src = f.read()
    except OSError as e:
        print(f"error: could not read {opts['input']}: {e}", file=sys.stderr)
        return 1
    try:
        # An entry parameter declared `name=None` is an input only when it is
        # given a --shape.
        graph = lower(src, opts["entry"], inputs=list(opts["shapes"]))
    except TysorSyntaxError as e:
        print(str(e), file=sys.stderr)
        return 1
    if not (opts["run"] or opts["backward"] or opts["train"]):
        return 0
    from .native import NativeError
    from .runtime import CudaContext, backward_cuda_module, run_cuda_module, train_cuda_module
    try:
        with CudaContext(int(os.environ.get("TYSOR_CUDA_DEVICE", "0"))) as ctx:
            if opts["run"]:
                run_cuda_module(ctx, graph, opts["shapes"])
            if opts["backward"]:
                backward_cuda_module(ctx, graph, opts["shapes"])
            if opts["train"]:
                if not graph.train_run:
                    # training/executor.rs:132-138: --train needs the `train model` run.
                    raise ValueError("Train executor requires a resolved 'train model' execution run")
                train_cuda_module(ctx, graph, opts["shapes"])
    except (NativeError, ValueError) as e:
        print(str(e), file=sys.stderr)
        return 1
    return 0
