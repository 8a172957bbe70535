"""The device-side tolerance check (used by the full-size GPU parity tests)
applies the same rules as the host one: run both on CPU tensors, on outputs
inside the tolerance and on outputs with one planted error."""

import numpy as np
import pytest
import torch

from tolerances import check_close, check_close_device

rng = np.random.default_rng(7)


def _case(category):
    if category == "matmul":
        A = rng.uniform(-1, 1, (40, 24)).astype(np.float32)
        B = rng.uniform(-1, 1, (24, 36)).astype(np.float32)
        want = (A.astype(np.float64) @ B).astype(np.float32)
        return {"A": A, "B": B}, {"C": want}
    if category == "attention":
        v = rng.standard_normal((2, 3, 50, 16)).astype(np.float32)
        want = rng.standard_normal((2, 3, 50, 16)).astype(np.float32)
        return {"v": v}, {"out": want}
    if category == "colreduce_f64":
        x = rng.uniform(-1, 1, (300, 64))
        return {"x": x}, {"colsum": x.sum(0), "colmax": x.max(0)}
    if category == "rowsum_i32":
        x = rng.integers(-100, 101, (30, 70)).astype(np.int32)
        return {"x": x}, {"out": x.sum(1).astype(np.int32)}
    want = rng.standard_normal((33, 100)).astype(np.float32)
    if category == "softmax":
        want = np.abs(want) / 100
    return {}, {"out": want}


@pytest.mark.parametrize("category", ["pointwise_f32", "rmsnorm", "softmax", "colreduce_f64",
                                      "rowsum_i32", "matmul", "attention"])
def test_device_check_agrees_with_host_check(category):
    inputs, wants = _case(category)
    tin = {k: torch.from_numpy(v) for k, v in inputs.items()}
    for name, want in wants.items():
        tw = torch.from_numpy(want)
        # inside the tolerance: a tiny relative perturbation
        if want.dtype.kind == "f":
            rel = 1e-14 if want.dtype == np.float64 else 1e-7
            close = want * (1 + rel) if name != "colmax" else want.copy()
        else:
            close = want.copy()
        ok_h, _ = check_close(category, name, close, want, inputs)
        ok_d, _ = check_close_device(category, name, torch.from_numpy(close), tw, tin,
                                     rows_per_chunk=7)
        assert ok_h and ok_d, (category, name)
        # one planted error far outside every rule
        bad = close.copy()
        bad.flat[5] = bad.flat[5] + (1 if want.dtype.kind in "iu" else 0.5 + abs(bad.flat[5]))
        ok_h, _ = check_close(category, name, bad, want, inputs)
        ok_d, msg = check_close_device(category, name, torch.from_numpy(bad), tw, tin,
                                       rows_per_chunk=7)
        assert not ok_h and not ok_d, (category, name)
        assert "1 of" in msg


def test_device_check_reports_shape_mismatch():
    ok, msg = check_close_device("softmax", "out", torch.zeros(2, 3), torch.zeros(3, 2))
    assert not ok and "shape" in msg
