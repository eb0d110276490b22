"""The reference-side Rust glue under rust/ (uncompiled here: no cargo on
these machines) is pinned on the CPU:

* every function of include/tysor_cuda.h has exactly one declaration in the
  `extern "C"` block of rust/src/backend/cuda/native.rs, with the same
  parameter names, count and C-to-Rust types, and nothing else is declared;
* rust/tysor_cuda.patch applies cleanly to the reference crate (when a
  checkout is available: TYSOR_REFERENCE_DIR or ../reference), and after it
  every `BackendKind` dispatch that names PyTorch also names Cuda, and the
  harness forwards --backend for --backward;
* the Rust entry points the patch calls exist in rust/src/backend/cuda/.
"""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tysor_cuda.h")
RUST = os.path.join(ROOT, "rust")

C_TO_RUST = {"void*": "*mut c_void", "const float*": "*const f32", "float*": "*mut f32", "size_t": "usize",
             "uint32_t": "u32", "uint64_t": "u64", "int64_t": "i64", "const int64_t*": "*const i64",
             "int64_t*": "*mut i64", "int": "c_int", "int*": "*mut c_int", "bool": "bool", "double": "f64",
             "float": "f32", "const char*": "*const c_char", "const uint8_t*": "*const u8", "uint8_t*": "*mut u8",
             "void": None}


def _norm(t):
    return " ".join(t.replace("*", " * ").split()).replace(" *", "*")


def header_decls():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    text = re.sub(r"enum\s*\{.*?\};", "", text, flags=re.S)
    text = "\n".join(l for l in text.splitlines() if not l.strip().startswith(("#", "extern", "}")))
    out = {}
    for ret, name, args in re.findall(r"([A-Za-z_][\w\s\*]*?)\b(tysor_cuda_\w+)\s*\(([^)]*)\)\s*;", text):
        params = []
        if args.strip() not in ("", "void"):
            for p in args.split(","):
                p = p.strip()
                arr = re.search(r"(\w+)\s*\[\d+\]$", p)
                if arr:
                    p = p[:arr.start()] + "* " + arr.group(1)
                m = re.match(r"(.*?)(\w+)$", p)
                params.append((m.group(2), C_TO_RUST[_norm(m.group(1))]))
        out[name] = (params, C_TO_RUST[_norm(ret)])
    return out


def rust_decls():
    src = open(os.path.join(RUST, "src", "backend", "cuda", "native.rs")).read()
    block = src[src.index('unsafe extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    out = {}
    for name, args, ret in re.findall(r"pub fn (tysor_cuda_\w+)\(([^)]*)\)(?:\s*->\s*([^;]+))?;", block):
        params = []
        for p in [a.strip() for a in args.split(",") if a.strip()]:
            n, t = p.split(":", 1)
            params.append((n.strip(), t.strip()))
        assert name not in out, f"{name} declared twice"
        out[name] = (params, ret.strip() if ret else None)
    return out


def test_rust_extern_block_matches_the_header():
    h, r = header_decls(), rust_decls()
    assert len(h) > 70
    assert sorted(h) == sorted(r), (set(h) ^ set(r))
    for name in h:
        assert r[name] == h[name], (name, r[name], h[name])


def reference_dir():
    for cand in (os.environ.get("TYSOR_REFERENCE_DIR"), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isfile(os.path.join(cand, "src", "backend", "core", "kind.rs")):
            return cand
    return None


def test_patch_applies_and_every_dispatch_names_cuda(tmp_path):
    ref = reference_dir()
    if ref is None or shutil.which("patch") is None:
        pytest.skip("no reference checkout (TYSOR_REFERENCE_DIR) or no `patch` here")
    crate = tmp_path / "tysor"
    shutil.copytree(ref, crate, ignore=shutil.ignore_patterns("target", ".git"))
    res = subprocess.run(["patch", "-p1", "-i", os.path.join(RUST, "tysor_cuda.patch")], cwd=crate,
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    shutil.copytree(os.path.join(RUST, "src"), crate / "src", dirs_exist_ok=True)
    shutil.copy(os.path.join(RUST, "build_cuda.rs"), crate / "build_cuda.rs")
    for path in crate.rglob("*.rs"):
        text = path.read_text()
        if "BackendKind::PyTorch =>" in text:
            assert "BackendKind::Cuda" in text, path
    assert "pub mod cuda;" in (crate / "src" / "backend" / "mod.rs").read_text()
    assert 'include!("build_cuda.rs");' in (crate / "build.rs").read_text()
    rt = (crate / "src" / "bin" / "run_tests.rs").read_text()
    back = rt[rt.index('cmd.push("--backward".to_string());'):]
    assert back.index('cmd.push("--backend".to_string());') < back.index("} else if args.train")
    assert "matches!(backend, Backend::Metal | Backend::Cuda)" in rt


def test_patch_calls_entry_points_that_exist():
    patch = open(os.path.join(RUST, "tysor_cuda.patch")).read()
    runtime = open(os.path.join(RUST, "src", "backend", "cuda", "runtime.rs")).read()
    called = set(re.findall(r"\b(run_cuda_\w+)\b", patch))
    assert called == {"run_cuda_module", "run_cuda_backward_module", "run_cuda_train_module"}
    for name in called:
        # one definition with the device, one stub without it
        assert len(re.findall(rf"pub fn {name}\(", runtime)) == 2, name
