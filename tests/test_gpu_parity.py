"""GPU parity: the sm_100a kernels, called through the C ABI, against the
CPU oracle on the same seeded inputs; and the reference compiler's own PTX
(committed fixture, JIT-compiled by the driver) against the same oracle."""

import tempfile
from pathlib import Path

import pytest

import cases
from gpu_util import output_init, run_on_gpu
from tolerances import check_close

GOLDEN = Path(__file__).resolve().parent / "golden" / "problems"

LOWERED = {"pointwise_zoo", "pointwise_mixed", "pointwise_f32", "pointwise_i32", "rmsnorm", "softmax", "rowsum_i32", "matmul", "attention",
           "colreduce_f64", "bit_ops", "rowsum_f64", "offset_copy"}

PARITY = [t for t, (name, _) in cases.PARITY.items() if name in LOWERED]


def _oracle(problem, ir_path, inputs):
    from oracle import simt
    return simt.run_package(ir_path, inputs, out_init=output_init(problem))


@pytest.mark.gpu
@pytest.mark.parametrize("geometry", ["tuned", "meta"])
@pytest.mark.parametrize("tag", PARITY)
def test_sm100_kernel_matches_oracle(cuda, tag, geometry):
    from emmy_ptx.runtime import Kernel
    p = cases.problem(tag)
    inputs = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        ir_path = p.write(td)
        kern = Kernel.from_ir(ir_path)
        got = run_on_gpu(kern, p, inputs, cuda, geometry=geometry)
        want = _oracle(p, ir_path, inputs)
    for o in p.outputs:
        ok, msg = check_close(p.category, o, got[o], want[o], inputs)
        assert ok, msg


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["pointwise_i32_64x256", "pointwise_i32_33x100"])
def test_torch_int_semantics_kernel_matches_oracle(cuda, tag):
    """``int_semantics="torch"`` (floor division, divisor-signed remainder)
    on the sm_100a pointwise kernel, bit for bit against the oracle's mode of
    the same name (itself checked against torch on the CPU)."""
    from emmy_ptx.runtime import Kernel
    from oracle import simt
    p = cases.problem(tag)
    inputs = p.make_inputs()
    assert (inputs["a"] < 0).any() and (inputs["b"] < 0).any()
    with tempfile.TemporaryDirectory() as td:
        ir_path = p.write(td)
        kern = Kernel.from_ir(ir_path, int_semantics="torch")
        got = run_on_gpu(kern, p, inputs, cuda)
        want = simt.run_package(ir_path, inputs, out_init=output_init(p), int_semantics="torch")
        trunc = simt.run_package(ir_path, inputs, out_init=output_init(p))
    for o in p.outputs:
        ok, msg = check_close(p.category, o, got[o], want[o], inputs)
        assert ok, msg
    assert (got["q"] != trunc["q"]).any(), "the torch mode changed nothing"


@pytest.mark.gpu
@pytest.mark.parametrize("tag", list(cases.PARITY))
def test_reference_ptx_matches_oracle(cuda, tag):
    """Oracle 1: the reference compiler's sm_89 PTX on the B200."""
    from emmy_ptx.runtime import Kernel
    d = GOLDEN / tag
    ir_path = next(d.glob("*.ir.json"))
    p = cases.problem(tag)
    inputs = p.make_inputs()
    kern = Kernel.from_ptx((d / "ref.ptx").read_text(), ir_path)
    got = run_on_gpu(kern, p, inputs, cuda, geometry="meta")
    want = _oracle(p, ir_path, inputs)
    for o in p.outputs:
        ok, msg = check_close(p.category, o, got[o], want[o], inputs)
        assert ok, msg


@pytest.mark.gpu
@pytest.mark.parametrize("name,kw", [("rmsnorm", dict(rows=64, cols=1024)),
                                     ("softmax", dict(rows=32, cols=16384)),
                                     ("pointwise_i32", dict(rows=64, cols=256))])
def test_chunked_host_pipeline_matches_oracle(cuda, name, kw, tmp_path):
    """The end-to-end host-buffer path (row blocks on two streams) gives the
    oracle's result for the full problem."""
    from emmy_ptx.pipeline import ChunkedHostRunner
    from emmy_ptx.runtime import PinnedArray
    from oracle import simt
    r = ChunkedHostRunner(name, chunks=4, slots=2, workdir=str(tmp_path), **kw)
    p = r.full
    inputs = p.make_inputs()
    host = {}
    for n, a in inputs.items():
        host[n] = PinnedArray(a.shape, a.dtype)
        host[n].array[...] = a
    outs = {o: PinnedArray(p.tensor(o)["shape"], {"f32": "float32", "s32": "int32",
                                                  "f64": "float64"}[p.tensor(o)["dtype"]])
            for o in p.outputs}
    want = simt.run_problem(p, inputs, str(tmp_path / "oracle"))
    for call in range(2):           # the second call reuses the slots and events
        for o in outs.values():
            o.array[...] = 0
        r.run(host, outs)
        for o in p.outputs:
            ok, msg = check_close(p.category, o, outs[o].array, want[o], inputs)
            assert ok, f"call {call + 1}: {msg}"
    r.free()


@pytest.mark.gpu
def test_two_binds_of_a_tensor_map_kernel_keep_their_own_buffers(cuda):
    """A tensor-map kernel keeps its TMA descriptors in module globals that
    every bind shares.  Two binds on different buffers, launched in the
    order first, second, first, each compute on their own buffers (the
    runtime writes a launch's maps again when another bind replaced them)."""
    import numpy as np
    import torch
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel
    p = workloads.build("matmul", m=256, n=256, k=128)
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td))
    assert kern.sidecar.get("tensormaps")
    sets, launches = [], []
    for seed in (1, 2):
        host = p.make_inputs(seed=seed)
        dev = {n: torch.from_numpy(v).to(cuda) for n, v in host.items()}
        dev["C"] = torch.full((256, 256), float("nan"), device=cuda)
        sets.append((host, dev))
        launches.append(kern.bind(dev))
    for i in (0, 1, 0):
        sets[i][1]["C"].fill_(float("nan"))
        launches[i]()
        torch.cuda.synchronize()
        host, dev = sets[i]
        want = host["A"].astype(np.float64) @ host["B"].astype(np.float64)
        ok, msg = check_close("matmul", f"C of bind {i}", dev["C"].cpu().numpy(), want, host)
        assert ok, msg
    assert kern.status() == 0


@pytest.mark.gpu
def test_misaligned_argument_is_refused_before_launch(cuda):
    """A pointer 4 bytes off the 32-byte vectors of the pointwise kernel is
    refused at bind time; nothing is launched."""
    import torch
    from emmy_ptx import workloads
    from emmy_ptx.runtime import EmmyRuntimeError, Kernel
    p = workloads.build("pointwise_f32", rows=64, cols=256)
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td))
    assert kern.alignment >= 16
    n = 64 * 256
    x = torch.zeros(n + 8, device=cuda)
    y = torch.zeros(n, device=cuda)
    out = torch.zeros(n, device=cuda)
    with pytest.raises(EmmyRuntimeError, match="aligned"):
        kern.bind({"x": x[1:n + 1], "y": y, "out": out})
    assert kern.launches == 0


@pytest.mark.gpu
@pytest.mark.parametrize("split", [2, 4])
def test_split_k_matmul_matches_oracle(cuda, split):
    """A split-K matmul (forced on a small shape): K slices accumulate into
    their own partial tiles, the reduce entry sums them in slice order."""
    from emmy_ptx import workloads
    from emmy_ptx.compiler import Compiler
    from emmy_ptx.runtime import Kernel
    from emmy_ptx.sm100 import matmul
    p = workloads.build("matmul", m=256, n=256, k=1024)
    inputs = p.make_inputs()
    with tempfile.TemporaryDirectory() as td:
        ir_path = p.write(td)
        comp = Compiler(ir_path, target="sm_100a", ptx_version="8.8")
        ptx, side = matmul.emit(comp, matmul.match(comp), split_k=split)
        assert side["split_k"] == split
        geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
        kern = Kernel(ptx, comp.entry, Kernel._arg_specs(comp), geom, side)
        got = run_on_gpu(kern, p, inputs, cuda)
        want = _oracle(p, ir_path, inputs)
    ok, msg = check_close(p.category, "C", got["C"], want["C"], inputs)
    assert ok, msg
