"""The reference's hot-path fixtures (run_tests.rs:34-66 allowlists, shapes
from run_tests.rs:229-267) through the device executor, against the oracle
restatement of the local backend: forward values, --backward gradients and
--train losses / final parameters.  The harness tolerance of the reference
(|a-b| <= max(5e-3, 5e-3|b|) on printed text, run_tests.rs:454-456) is far
looser than the bars used here: rel 1e-5 for values and gradients, rel 1e-4
for training losses."""
import numpy as np
import pytest

import local as L
from tysor_b200.programs import FIXTURES

pytestmark = pytest.mark.gpu


def close(got, want, rtol):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    assert got.shape == want.shape
    err = np.abs(got - want)
    assert np.all(err <= rtol * np.maximum(np.abs(want), 1.0)), (got, want)


def cases(mode):
    return [f for f in FIXTURES.values() if mode in f.modes]


@pytest.mark.parametrize("fx", cases("run"), ids=lambda f: f.name)
def test_run_fixture(cuda_ctx, fx):
    from tysor_b200.runtime import CudaGraphExecutor
    g = fx.build()
    want, _ = L.run_forward(g, fx.shapes)
    ex = CudaGraphExecutor(cuda_ctx, g, fx.shapes)
    got = ex.run()
    assert got.shape == want.shape
    assert got.dtype == want.dtype  # the printed dtype string (tensor.rs:48-58)
    close(got.data, want.data, 1e-5)
    ex.close()


@pytest.mark.parametrize("fx", cases("backward"), ids=lambda f: f.name)
def test_backward_fixture(cuda_ctx, fx):
    from tysor_b200.runtime import CudaGraphExecutor
    g = fx.build()
    want = L.backward_report(g, fx.shapes)
    ex = CudaGraphExecutor(cuda_ctx, g, fx.shapes)
    got = ex.backward()
    assert [n for n, _ in got] == [n for n, _ in want]
    for (_, gt), (_, wt) in zip(got, want):
        assert gt.shape == wt.shape
        assert gt.dtype == wt.dtype
        close(gt.data, wt.data, 1e-5)
    ex.close()


@pytest.mark.parametrize("fx", cases("train"), ids=lambda f: f.name)
def test_train_fixture(cuda_ctx, fx):
    from tysor_b200.runtime import CudaGraphExecutor
    g = fx.build()
    want_losses, want_params = L.train(g, fx.shapes)
    ex = CudaGraphExecutor(cuda_ctx, g, fx.shapes)
    got_losses = ex.train()
    close(got_losses, want_losses, 1e-4)
    got_params = ex.parameters()
    assert sorted(got_params) == sorted(want_params)
    for name, t in want_params.items():
        close(got_params[name], t.data, 1e-5)
    ex.close()


def test_cli_paths_dump_full_precision_results(cuda_ctx, tmp_path, monkeypatch, capsys):
    """run/backward/train_cuda_module print the reference's text and, with
    TYSOR_DUMP_DIR set, write the same results as raw f32 files that match
    the oracle at full precision (the text keeps 4 decimals)."""
    from tysor_b200.runtime import (DUMP_ENV, backward_cuda_module, read_dump, run_cuda_module,
                                    train_cuda_module)
    monkeypatch.setenv(DUMP_ENV, str(tmp_path))
    run_fx = cases("run")[0]
    g = run_fx.build()
    run_cuda_module(cuda_ctx, g, run_fx.shapes)
    want, _ = L.run_forward(g, run_fx.shapes)
    got = read_dump("output", str(tmp_path))
    assert got.shape == want.shape
    close(got.data, want.data, 1e-5)
    assert "--- Execution Output ---" in capsys.readouterr().out

    bw = cases("backward")[0]
    g = bw.build()
    backward_cuda_module(cuda_ctx, g, bw.shapes)
    for name, wt in L.backward_report(g, bw.shapes):
        close(read_dump(f"{name}_grad", str(tmp_path)).data, wt.data, 1e-5)

    tr = cases("train")[0]
    g = tr.build()
    train_cuda_module(cuda_ctx, g, tr.shapes)
    want_losses, want_params = L.train(g, tr.shapes)
    close(read_dump("losses", str(tmp_path)).data, want_losses, 1e-4)
    for name, t in want_params.items():
        close(read_dump(f"param_{name}", str(tmp_path)).data, t.data, 1e-5)
    assert "backend=cuda" in capsys.readouterr().out
