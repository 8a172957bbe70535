"""Parity at the BASELINE configurations' full shapes -- the kernels bench.py
times, specialised exactly as it times them (Kernel.from_ir defaults, tuned
geometry).

Each sm_100a kernel is compared on the same device inputs (seeded on the
host, as every other parity test) with two references:

1. the reference compiler's own PTX for the same IR package
   (``tests/golden/problems/<tag>_full/ref.ptx``, written by the unmodified
   reference ``compiler.py``), JIT-loaded on the same B200 and launched with
   the meta.json geometry -- the north star's first oracle;
2. the same computation in float64 (int64 for integers) with torch on the
   device: a closed form that does not share the kernels' approximations.

The CPU oracle (``oracle.simt``) is far too slow at these sizes; it is pinned
against the reference on the small parity cases instead.  Integer outputs
must match bit for bit; floats use ``tests/tolerances.py``.  The full-size
problems take 0.27-2.6 GB of inputs each and run one at a time.
"""

import math
import tempfile
from pathlib import Path

import numpy as np
import pytest

import cases
from gpu_util import SENTINEL
from tolerances import check_close_device

GOLDEN = Path(__file__).resolve().parent / "golden" / "problems"
TORCH_DT = {"f32": "float32", "f64": "float64", "s32": "int32"}


def _outputs(torch, p, device):
    out = {}
    for o in p.outputs:
        t = p.tensor(o)
        dt = getattr(torch, TORCH_DT[t["dtype"]])
        fill = SENTINEL[t["dtype"]]
        out[o] = torch.full(t["shape"], float(fill) if dt.is_floating_point else int(fill),
                            dtype=dt, device=device)
    return out


def _float64_reference(torch, p, x):
    """The config's computation in float64 / int64 on the device."""
    c = p.category
    if c == "pointwise_f32":
        a = x["x"].double()
        return {"out": a * torch.sigmoid(a) + x["y"].double()}
    if c == "pointwise_i32":
        # the reference's integer semantics: truncating div.s32 / rem.s32
        # (compiler.py:1383-1385), arithmetic shifts
        a, b = x["a"].long(), x["b"].long()
        q = torch.div(a, b, rounding_mode="trunc")
        return {"q": q.int(), "r": (a - b * q).int(), "s": ((a << 3) >> 1).int()}
    if c == "rmsnorm":
        a = x["x"].double()
        eps = p.params["eps"]
        return {"out": a * torch.rsqrt(a.square().mean(1, keepdim=True) + eps)
                * x["w"].double()}
    if c == "softmax":
        out = torch.empty(x["x"].shape, dtype=torch.float64, device=x["x"].device)
        for r0 in range(0, out.shape[0], 1024):
            out[r0:r0 + 1024] = torch.softmax(x["x"][r0:r0 + 1024].double(), dim=1)
        return {"out": out}
    if c == "colreduce_f64":
        return {"colsum": x["x"].sum(0), "colmax": x["x"].amax(0)}
    if c == "rowsum_i32":
        return {"out": x["x"].long().sum(1).int()}
    if c == "matmul":
        return {"C": x["A"].double() @ x["B"].double()}
    if c == "attention":
        q, k, v = x["q"], x["k"], x["v"]
        B, H, S, D = q.shape
        scale = 1.0 / math.sqrt(D)
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
        out = torch.empty(q.shape, dtype=torch.float64, device=q.device)
        for b in range(B):
            for h0 in range(0, H, 8):
                s = (q[b, h0:h0 + 8].double() @ k[b, h0:h0 + 8].double().transpose(-1, -2)) * scale
                s.masked_fill_(~mask, float("-inf"))
                out[b, h0:h0 + 8] = torch.softmax(s, dim=-1) @ v[b, h0:h0 + 8].double()
                del s
        return {"out": out}
    raise AssertionError(c)


@pytest.mark.gpu
@pytest.mark.parametrize("tag", list(cases.FULL))
def test_full_size_kernel_matches_reference_ptx_and_float64(cuda, tag):
    import torch
    from emmy_ptx.runtime import Kernel

    p = cases.problem(tag)
    host = p.make_inputs()
    x = {n: torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for n, a in host.items()}
    del host
    with tempfile.TemporaryDirectory() as td:
        ir = p.write(td)
        mine = Kernel.from_ir(ir)                       # what bench.py times
        ref = Kernel.from_ptx((GOLDEN / tag / "ref.ptx").read_text(), ir)
    got = _outputs(torch, p, cuda)
    mine.launch({**x, **got})
    torch.cuda.synchronize()
    assert mine.status() == 0, f"kernel status word {mine.status():#x}"
    mine.free_scratch()
    theirs = _outputs(torch, p, cuda)
    ref.launch({**x, **theirs}, geometry="meta")
    torch.cuda.synchronize()
    causal = bool(p.params.get("causal", True))
    report = []
    for o in p.outputs:
        g = got[o]
        if g.dtype.is_floating_point:
            assert not torch.isnan(g).any(), f"{o}: unwritten (NaN sentinel) elements"
        else:
            assert not (g == int(SENTINEL[p.tensor(o)["dtype"]])).any(), f"{o}: unwritten"
        ok, msg = check_close_device(p.category, f"{o} vs reference PTX", g, theirs[o], x,
                                     causal=causal)
        assert ok, msg
        report.append(msg)
    del theirs
    torch.cuda.empty_cache()
    want = _float64_reference(torch, p, x)
    for o in p.outputs:
        ok, msg = check_close_device(p.category, f"{o} vs float64", got[o], want[o], x,
                                     causal=causal)
        assert ok, msg
        report.append(msg)
    print(tag, "; ".join(report))
    del want, got, x
    torch.cuda.empty_cache()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,split", [(2048, 2)])
def test_matmul_shard_with_split_k_matches_float64(cuda, rows, split):
    """The row shard of the 8192^3 matmul at 4 ranks (2048 rows of C) is cut
    along K (its pair tiles alone fill 3.46 waves of the 74 CTA pairs); the
    partial tiles, summed by the reduce entry, give C within the matmul
    tolerance of float64, and twice in a row the same bits."""
    import torch
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel
    p = workloads.build("matmul", m=rows, n=8192, k=8192)
    host = p.make_inputs()
    x = {n: torch.from_numpy(a).to(cuda) for n, a in host.items()}
    del host
    with tempfile.TemporaryDirectory() as td:
        kern = Kernel.from_ir(p.write(td))
    assert kern.sidecar["split_k"] == split and kern.sidecar["postlaunch"]
    got = _outputs(torch, p, cuda)
    launch = kern.bind({**x, **got})
    launch()
    torch.cuda.synchronize()
    first = got["C"].clone()
    launch()
    torch.cuda.synchronize()
    assert kern.status() == 0
    assert torch.equal(first, got["C"]), "split-K sums are not deterministic"
    want = x["A"].double() @ x["B"].double()
    ok, msg = check_close_device("matmul", "C vs float64", got["C"], want, x)
    assert ok, msg
    kern.free_scratch()
