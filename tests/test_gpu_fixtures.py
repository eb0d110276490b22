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
