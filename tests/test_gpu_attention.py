"""Attention at sizes the CPU oracle is too slow for: several query tiles,
sequence lengths that do not fill the last 128-query or 64-key tile,
head_dim 32, 64 and 128, causal and not, checked on the GPU against a float64
softmax(Q K^T * scale) V of the same inputs with the attention tolerance."""

import tempfile

import numpy as np
import pytest

from gpu_util import run_on_gpu
from tolerances import check_close

CASES = [
    dict(batch=1, heads=3, seq=1000, head_dim=128, causal=True),
    dict(batch=2, heads=2, seq=777, head_dim=64, causal=True),
    dict(batch=1, heads=2, seq=640, head_dim=128, causal=False),
    dict(batch=1, heads=4, seq=300, head_dim=32, causal=True),
    dict(batch=1, heads=1, seq=129, head_dim=64, causal=False),
]


def _reference(inputs, scale, causal):
    q, k, v = (inputs[n].astype(np.float64) for n in "qkv")
    s = q @ k.transpose(0, 1, 3, 2) * scale
    if causal:
        n = s.shape[-1]
        s = np.where(np.tril(np.ones((n, n), bool)), s, -np.inf)
    w = np.exp(s - s.max(-1, keepdims=True))
    return w / w.sum(-1, keepdims=True) @ v


@pytest.mark.gpu
@pytest.mark.parametrize("kw", CASES, ids=lambda kw: "{batch}x{heads}x{seq}x{head_dim}{c}".format(
    c="c" if kw["causal"] else "n", **kw))
def test_attention_matches_float64_reference(cuda, kw):
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel
    p = workloads.attention(**kw)
    inputs = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td))
        assert kern.sidecar["category"] == "attention"
        got = run_on_gpu(kern, p, inputs, cuda)
    want = _reference(inputs, p.params["scale"], kw["causal"])
    ok, msg = check_close("attention", "out", got["out"], want, inputs, causal=kw["causal"])
    assert ok, msg


@pytest.mark.gpu
def test_non_finite_values_propagate_like_the_reference(cuda):
    """NaN (as CUDA arithmetic writes it, 0x7FFFFFFF, and as numpy does) and
    infinity in V survive the kernel's in-shared-memory rounding of V: the
    output has NaN and infinity exactly where the float64 reference has
    them, and the other values agree within the attention tolerance."""
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel
    kw = dict(batch=1, heads=2, seq=200, head_dim=64, causal=True)
    p = workloads.attention(**kw)
    inputs = p.make_inputs()
    v = inputs["v"].copy()
    v.view(np.uint32)[0, 0, 5, 3] = 0x7FFFFFFF
    v[0, 1, 70, 10] = np.nan
    v[0, 0, 9, 7] = np.inf
    v[0, 1, 100, 20] = -np.inf
    inputs["v"] = v
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td))
        got = run_on_gpu(kern, p, inputs, cuda)["out"]
    want = _reference(inputs, p.params["scale"], True)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isposinf(got), np.isposinf(want))
    assert np.array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    vmax = np.abs(v[np.isfinite(v)]).max()
    keys = np.minimum(np.arange(kw["seq"]) + 1, kw["seq"])[None, None, :, None]
    tol = 1e-3 * (np.abs(want) + vmax / np.sqrt(keys))
    assert (np.abs(got - want)[fin] <= np.broadcast_to(tol, want.shape)[fin]).all()


@pytest.mark.gpu
@pytest.mark.parametrize("kw", [dict(batch=1, heads=3, seq=640, head_dim=128, causal=True),
                                dict(batch=2, heads=1, seq=300, head_dim=64, causal=True),
                                dict(batch=1, heads=2, seq=384, head_dim=128, causal=False)],
                         ids=["640c", "300x64c", "384n"])
def test_cta_pair_kernel_matches_float64_reference(cuda, kw):
    """The CTA-pair variant (tcgen05 cta_group::2, 256 query rows per pair,
    half of every K and V chunk per CTA), forced on: a partial last pair,
    head_dim 64 and 128, causal (the lower tile's last key tile fully
    masked) and not."""
    from emmy_ptx import workloads
    from emmy_ptx.compiler import Compiler
    from emmy_ptx.runtime import Kernel
    from emmy_ptx.sm100 import attention
    p = workloads.attention(**kw)
    inputs = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        comp = Compiler(p.write(td), target="sm_100a", ptx_version="8.7")
        ptx, side = attention.emit(comp, attention.match(comp), pair=True)
        assert side["cluster"] == [2, 1, 1] and side["cta_group"] == 2
        kern = Kernel(ptx, comp.entry, Kernel._arg_specs(comp),
                      {"grid": comp.kmeta["grid"], "block": comp.kmeta["block"]}, side)
        got = run_on_gpu(kern, p, inputs, cuda)
    want = _reference(inputs, p.params["scale"], kw["causal"])
    ok, msg = check_close("attention", "out", got["out"], want, inputs, causal=kw["causal"])
    assert ok, msg


@pytest.mark.gpu
def test_ptx_isa_8_7_epilogue_matches_float64_reference(cuda):
    """Below PTX ISA 8.8 the epilogue stores 16 bytes per instruction
    instead of 32 (``st.global.v8`` needs 8.8); that kernel is checked too."""
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel
    kw = dict(batch=1, heads=3, seq=640, head_dim=128, causal=True)
    p = workloads.attention(**kw)
    inputs = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td), ptx_version="8.7")
        assert "st.global.v8" not in kern.ptx
        got = run_on_gpu(kern, p, inputs, cuda)
    want = _reference(inputs, p.params["scale"], True)
    ok, msg = check_close("attention", "out", got["out"], want, inputs, causal=True)
    assert ok, msg
