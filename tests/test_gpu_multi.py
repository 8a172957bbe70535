"""Two GPUs: the fused all-gathers (emmy_ptx.dist.FusedGather) -- each rank's
matmul or attention epilogue storing its output rows into both ranks' full
output over NVLink -- against the full result computed on the host.
Skipped with fewer than two GPUs.
The ranks are child processes with a short process-group timeout, and the
parent stops them by PID if they do not finish."""

import os
import socket

import numpy as np
import pytest

KW = {"matmul": dict(m=512, n=384, k=256),
      # 16 (batch x head) pairs per rank: two head groups, so the shard's
      # kernel splits group 1 itself; 192 keys leave a partial query tile
      "attention": dict(batch=4, heads=8, seq=192, head_dim=64),
      "softmax": dict(rows=300, cols=32768),
      "rmsnorm": dict(rows=64, cols=4096)}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, name, mode="fused"):
    import sys
    from datetime import timedelta
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "emmy-ptx_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import ctypes
    import torch
    import torch.distributed as dist
    from emmy_ptx import dist as edist
    from emmy_ptx import workloads
    from emmy_ptx.runtime import check, init, lib
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    init(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=device)
    try:
        kw = KW[name]
        full = workloads.build(name, **kw)
        inputs = full.make_inputs()
        shard = edist.shard_inputs(name, inputs, rank, world)
        stream = torch.cuda.Stream(device)
        if mode == "copy":
            fused = edist.CopyGather(name, rank, world, out_dir, chunks=2, **kw)
        else:
            fused = edist.FusedGather(name, rank, world, out_dir, **kw)
        dev = {n: torch.from_numpy(v).to(device) for n, v in shard.items()}
        out = fused.part.outputs[0]
        dev[out] = torch.empty(fused.part.tensor(out)["shape"], dtype=torch.float32,
                               device=device)
        shape = full.tensor(out)["shape"]
        fused.bind(dev, stream=stream)
        results = []
        for _ in range(2):                       # two calls in a row
            check(lib().ert_memset_d8(fused.out.local.ptr, 0xFF, fused.out.nbytes, 0),
                  "ert_memset_d8")
            torch.cuda.synchronize()
            dist.barrier()
            with torch.cuda.stream(stream):
                fused.launch()
                fused.wait()
            torch.cuda.synchronize()
            host = np.empty(shape, np.float32)
            check(lib().ert_memcpy_dtoh(host.ctypes.data_as(ctypes.c_void_p),
                                        fused.out.local.ptr, host.nbytes, 0), "ert_memcpy_dtoh")
            check(lib().ert_stream_sync(0), "ert_stream_sync")
            results.append(host)
        assert fused.kernel.status() == 0
        dist.barrier()
        fused.close()
        np.savez(os.path.join(out_dir, f"rank{rank}{mode}.npz"), first=results[0],
                 second=results[1])
    finally:
        dist.destroy_process_group()


def _host_result(name, inputs, p):
    if name == "softmax":
        x = inputs["x"].astype(np.float64)
        e = np.exp(x - x.max(1, keepdims=True))
        return (e / e.sum(1, keepdims=True)).astype(np.float32)
    if name == "rmsnorm":
        x = inputs["x"].astype(np.float64)
        return (x / np.sqrt((x * x).mean(1, keepdims=True) + p.params["eps"])
                * inputs["w"]).astype(np.float32)
    if name == "matmul":
        return (inputs["A"].astype(np.float64) @ inputs["B"].astype(np.float64)).astype(np.float32)
    q, k, v = (inputs[n].astype(np.float64) for n in "qkv")
    s = q @ k.transpose(0, 1, 3, 2) * p.params["scale"]
    n = s.shape[-1]
    s = np.where(np.tril(np.ones((n, n), bool)), s, -np.inf)
    w = np.exp(s - s.max(-1, keepdims=True))
    return ((w / w.sum(-1, keepdims=True)) @ v).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("name,mode", [("matmul", "fused"), ("attention", "fused"),
                                       ("softmax", "fused"), ("rmsnorm", "fused"),
                                       ("softmax", "copy"), ("rmsnorm", "copy"),
                                       ("matmul", "copy"), ("attention", "copy")])
def test_fused_gather_on_two_gpus(tmp_path, name, mode):
    """``fused``: the kernels' epilogues store into both ranks' outputs;
    ``copy``: the kernels write this rank's rows of its own full output (two
    row blocks) and the copy engines move them into the peer's."""
    import torch
    import torch.multiprocessing as mp
    from emmy_ptx import workloads
    from tolerances import check_close
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), name, mode))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    stuck = [p for p in procs if p.is_alive()]
    for p in stuck:
        p.kill()
        p.join(timeout=10)
    assert not stuck, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    full = workloads.build(name, **KW[name])
    inputs = full.make_inputs()
    want = _host_result(name, inputs, full)
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}{mode}.npz")
        for k in ("first", "second"):
            ok, msg = check_close(name, f"{name} rank {r} {k}", got[k], want, inputs)
            assert ok, msg


@pytest.mark.gpu
@pytest.mark.parametrize("name,kw", [("softmax", dict(rows=296, cols=32768)),
                                     ("softmax", dict(rows=6, cols=2052)),
                                     ("rmsnorm", dict(rows=64, cols=4096))])
def test_row_gather_epilogue_on_one_gpu(cuda, tmp_path, name, kw):
    """The row kernels' gather variant, with two buffers of one GPU standing
    in for two ranks' full outputs: rank 1's shard stores each row into both
    at row ``row0 + row``, bit-identical to the regular kernel's row, and
    leaves the other rank's rows and its own ``out`` argument untouched."""
    import struct
    import torch
    from emmy_ptx import dist as edist
    from emmy_ptx import workloads
    from emmy_ptx.compiler import Compiler
    from emmy_ptx.runtime import Kernel
    from emmy_ptx.sm100 import rows
    world, rank = 2, 1
    full = workloads.build(name, **kw)
    R, C = full.tensor("out")["shape"]
    part, _ = edist.shard_problem(name, rank, world, **kw)
    shard = edist.shard_inputs(name, full.make_inputs(), rank, world)
    ir = part.write(tmp_path / "shard")
    plain = Kernel.from_ir(ir)
    comp = Compiler(ir, target="sm_100a", ptx_version="8.8")
    ptx, side = rows.emit(comp, rows.match(comp), gather=world)
    geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
    fused = Kernel(ptx, comp.entry, Kernel._arg_specs(comp), geom, side)
    dev = {n: torch.from_numpy(v).to(cuda) for n, v in shard.items()}
    ref = torch.full((R // world, C), float("nan"), device=cuda)
    plain.launch({**dev, "out": ref})
    dests = [torch.full((R, C), float("nan"), device=cuda) for _ in range(world)]
    fused.set_global("emmy_gather_dst", struct.pack("<2Q", *(d.data_ptr() for d in dests)))
    fused.set_global("emmy_gather_n", struct.pack("<I", world))
    fused.set_global("emmy_gather_row0", struct.pack("<I", rank * (R // world)))
    own = torch.full((R // world, C), float("nan"), device=cuda)
    for _ in range(2):                                      # two calls in a row
        for d in dests:
            d.fill_(float("nan"))
        fused.launch({**dev, "out": own})
        torch.cuda.synchronize()
        assert fused.status() == 0
        for d in dests:
            assert torch.equal(d[R // world:], ref), "gathered rows differ from the kernel's"
            assert torch.isnan(d[:R // world]).all(), "wrote outside its rows"
        assert torch.isnan(own).all(), "the gather variant wrote its own out argument"
