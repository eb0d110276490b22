"""The text the CUDA backend prints for a tensor (runtime.format_tensor)
against the reference's print_tensor_body (tensor.rs:48-69) as the oracle
restates it: shape list, dtype, and every value with Rust's `{:.4}`."""
import numpy as np

import local as L
from tysor_b200.runtime import HostTensor, format_tensor


def _both(shape, values, dtype="float32"):
    data = np.asarray(values, np.float32)
    got = format_tensor(HostTensor(list(shape), data, dtype))
    want = L.format_tensor(L.Tensor(list(shape), data.copy(), dtype))
    return got, want


def test_known_answer():
    got, _ = _both([2, 3], [0.125, 0.25, 0.375, 0.5, 0.625, 0.75])
    assert got == "shape=[2, 3] dtype=float32\nvalues=[0.1250, 0.2500, 0.3750, 0.5000, 0.6250, 0.7500]"


def test_special_values_print_like_rust():
    got, want = _both([6], [np.nan, np.inf, -np.inf, -0.0, 1e20, -123.45675])
    assert got == want
    assert got.split("\n")[1] == "values=[NaN, inf, -inf, -0.0000, 100000002004087734272.0000, -123.4567]"


def test_rounding_matches_the_oracle_on_random_values():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(500), rng.uniform(-1e4, 1e4, 500),
                           np.round(rng.uniform(-10, 10, 200), 5)]).astype(np.float32)
    got, want = _both([len(vals)], vals, "float16")
    assert got == want
    assert got.startswith(f"shape=[{len(vals)}] dtype=float16\n")


def test_binary_dump_round_trips_bit_exactly(tmp_path):
    """The TYSOR_DUMP_DIR side channel keeps every bit of the values."""
    from tysor_b200.runtime import dump_tensor, read_dump
    vals = np.random.default_rng(3).standard_normal(37).astype(np.float32)
    vals[[0, 5]] = [np.nan, -0.0]
    path = dump_tensor("w/eird name", HostTensor([37], vals, "float16"), str(tmp_path))
    assert path.endswith("w_eird_name.f32")
    back = read_dump("w/eird name", str(tmp_path))
    assert back.shape == [37] and back.dtype == "float16"
    np.testing.assert_array_equal(back.data.view(np.uint32), vals.view(np.uint32))


def test_no_dump_without_a_directory(monkeypatch):
    from tysor_b200.runtime import DUMP_ENV, dump_tensor
    monkeypatch.delenv(DUMP_ENV, raising=False)
    assert dump_tensor("x", HostTensor([1], np.zeros(1, np.float32))) is None


def test_fixture_dtype_strings_follow_the_reference_rules():
    """Every allowlisted fixture declares `tensor[float16]` parameters; the
    oracle's forward carries that string to the output except where an
    Embedding (whose builtin constructor declares no dtype) produces the
    values, and the graph's own dtype pass agrees for every fixture."""
    import local as L
    from tysor_b200.programs import FIXTURES
    seen = set()
    for fx in FIXTURES.values():
        g = fx.build()
        assert all(v.dtype == "float16" for v in g.parameters())
        if "run" not in fx.modes:
            continue
        want, _ = L.run_forward(g, fx.shapes)
        assert g.value_dtypes()[g.outputs[0]] == want.dtype, fx.name
        seen.add(want.dtype)
    assert seen == {"float16", "float32"}  # the transformer fixture starts at an Embedding


def test_matmul_engine_names_are_checked_before_any_device_work(monkeypatch):
    """CudaContext takes its matmul engine from the argument or from
    TYSOR_CUDA_MATMUL; an unknown name is refused before the library is
    asked for a device."""
    import pytest

    from tysor_b200.runtime import CudaContext
    with pytest.raises(ValueError, match="strict16"):
        CudaContext(0, matmul="bogus")
    monkeypatch.setenv("TYSOR_CUDA_MATMUL", "tf32x9")
    with pytest.raises(ValueError, match="tf32x9"):
        CudaContext(0)
