"""The product path never reaches the oracle: no source of the package, the
C header or the Rust glue names the oracle's module or libraries, and the
built CUDA library links neither of them.  The oracle is the checker of the
tests, smoke() and bench.py's CPU legs only."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRODUCT_DIRS = ["tysor_b200", "include", "rust"]
SOURCE_EXT = (".py", ".cu", ".cuh", ".h", ".cc", ".cpp", ".rs", ".patch")
# The oracle's Python module, its C restatement and its shared libraries.
ORACLE_NAMES = re.compile(r"\boracle\b|tysor_local|libtysor_oracle")


def product_sources():
    for d in PRODUCT_DIRS:
        for dirpath, dirnames, filenames in os.walk(os.path.join(ROOT, d)):
            dirnames[:] = [n for n in dirnames if n not in ("_build", "__pycache__")]
            for f in filenames:
                if f.endswith(SOURCE_EXT):
                    yield os.path.join(dirpath, f)


def test_product_sources_do_not_name_the_oracle():
    for planted in ("from oracle import local", "ctypes.CDLL('oracle/libtysor_oracle.so')", "tysor_local.c"):
        assert ORACLE_NAMES.search(planted)
    files = list(product_sources())
    assert any(f.endswith("executor.cu") for f in files) and any(f.endswith("runtime.py") for f in files)
    hits = []
    for path in files:
        with open(path, encoding="utf-8", errors="replace") as fh:
            for n, line in enumerate(fh, 1):
                if ORACLE_NAMES.search(line):
                    hits.append(f"{os.path.relpath(path, ROOT)}:{n}: {line.strip()}")
    assert not hits, "product sources name the oracle:\n" + "\n".join(hits)


def test_cuda_library_links_no_oracle_library():
    from tysor_b200 import build, native

    if not os.path.exists(native.LIB_PATH):
        build.build()
    if shutil.which("readelf") is None:
        pytest.skip("readelf not available")
    out = subprocess.run(["readelf", "-d", native.LIB_PATH], capture_output=True, text=True, check=True).stdout
    needed = re.findall(r"\(NEEDED\)\s+Shared library: \[([^\]]+)\]", out)
    assert needed, "no dynamic dependencies read from the library"
    assert not [n for n in needed if "oracle" in n], needed
