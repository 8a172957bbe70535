"""Multi-GPU execution: shard a problem, run each shard, all-gather outputs.

One process per GPU (torchrun); ``torch.distributed`` with NCCL over
NVLink/NVSwitch is the plumbing.  Every Emmy category partitions into
independent shards with a single exchange step, an all-gather of the
outputs (no collective is needed to *compute* a shard):

=================  ==========================  ===============================
category           partition                   gathered output layout
=================  ==========================  ===============================
pointwise          rows of [R, C]              rows, contiguous
rmsnorm / softmax  rows                        rows, contiguous
rowsum_i32         rows                        rows, contiguous
colreduce_f64      columns (x[:, c0:c1] slab)  per-rank column vectors, then
                                               concatenated in rank order
matmul             row blocks of C (A sliced,  rows, contiguous
                   B replicated)
attention          (batch x heads) pairs       pairs, contiguous
=================  ==========================  ===============================

Shards are equal-sized (the partitioned extent must divide by the world
size); each rank's shard is an ordinary IR package of the shard's shape, so
the same compiler and kernels run it.

Two ways to do the exchange step for matmul:

* ``all_gather_outputs``: the kernel writes its C shard, then NCCL
  ``all_gather_into_tensor`` (what the north star names);
* ``FusedGatherMatmul``: the kernel's epilogue stores each finished C tile
  straight into every rank's full C over NVLink (buffers mapped with CUDA
  IPC, ``PeerBuffer``), so the exchange overlaps the remaining tiles' MMAs
  and no separate collective moves data.  A one-element NCCL all-reduce on
  the same stream then tells every rank that all kernels have finished.
"""

from __future__ import annotations

import os
import struct

import numpy as np

from . import workloads

PARTITION = {
    "pointwise_f32": "rows", "pointwise_i32": "rows", "rmsnorm": "rows",
    "softmax": "rows", "rowsum_i32": "rows", "colreduce_f64": "cols",
    "matmul": "m", "attention": "pairs",
}

FULL_DEFAULTS = {
    "pointwise_f32": dict(rows=4096, cols=4096), "pointwise_i32": dict(rows=4096, cols=4096),
    "rmsnorm": dict(rows=8192, cols=4096), "softmax": dict(rows=8192, cols=32768),
    "rowsum_i32": dict(rows=65536, cols=1024), "colreduce_f64": dict(rows=16384, cols=4096),
    "matmul": dict(m=8192, n=8192, k=8192),
    "attention": dict(batch=8, heads=32, seq=4096, head_dim=128),
}


def shard_range(total: int, rank: int, world: int):
    """Equal contiguous block ``[start, start + count)`` of ``total``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if total % world:
        raise ValueError(f"{total} does not divide into {world} equal shards")
    count = total // world
    return rank * count, count


def shard_problem(name: str, rank: int, world: int, **kw):
    """The IR package of ``rank``'s shard of problem ``name``."""
    full = dict(FULL_DEFAULTS[name])
    full.update(kw)
    part = PARTITION[name]
    shard = dict(full)
    if part == "rows":
        _, shard["rows"] = shard_range(full["rows"], rank, world)
    elif part == "cols":
        _, shard["cols"] = shard_range(full["cols"], rank, world)
    elif part == "m":
        _, shard["m"] = shard_range(full["m"], rank, world)
    elif part == "pairs":
        pairs = full["batch"] * full["heads"]
        _, n = shard_range(pairs, rank, world)
        shard["batch"], shard["heads"] = 1, n
    return workloads.build(name, **shard), full


def shard_inputs(name: str, full_inputs: dict, rank: int, world: int) -> dict:
    """Slice the full host inputs down to ``rank``'s shard (contiguous)."""
    part = PARTITION[name]
    out = {}
    for k, v in full_inputs.items():
        if part == "rows":
            if v.ndim >= 2:
                s, n = shard_range(v.shape[0], rank, world)
                v = v[s:s + n]
        elif part == "cols":
            s, n = shard_range(v.shape[1], rank, world)
            v = v[:, s:s + n]
        elif part == "m":
            if k == "A":
                s, n = shard_range(v.shape[0], rank, world)
                v = v[s:s + n]
        elif part == "pairs":
            b, h = v.shape[:2]
            flat = v.reshape(b * h, *v.shape[2:])
            s, n = shard_range(b * h, rank, world)
            v = flat[s:s + n][None]
        out[k] = np.ascontiguousarray(v)
    return out


def assemble(gathered: dict, full_shape: dict) -> dict:
    """Reshape all-gathered flat outputs into the full outputs.  Every
    partition is contiguous and rank-ordered (row blocks, column blocks of
    the per-column results, (batch, head) pairs), so the rank-major
    concatenation is already the full output in row-major order."""
    return {o: np.asarray(flat).reshape(full_shape[o]) for o, flat in gathered.items()}


def all_gather_outputs(shards: dict, group=None) -> dict:
    """``torch.distributed.all_gather_into_tensor`` of every output shard
    (rank-major, flat).  Works with NCCL (CUDA tensors) and gloo (CPU)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = {}
    for name, t in shards.items():
        flat = t.reshape(-1).contiguous()
        full = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(full, flat, group=group)
        out[name] = full
    return out


def bench_sharded(names, workdir, device, stream, rank, world, steps=5, warmup=2):
    """Strong scaling of the row-sharded path: each rank runs 1/world of the
    rows of every problem in ``names``; reports the kernel-only step time
    and the step time including the NCCL all-gather of the outputs (both max
    over ranks) and the corresponding whole-job GB/s."""
    import torch
    import torch.distributed as dist
    from .runtime import Kernel
    launches, outs, total_bytes = [], [], 0
    for name in names:
        p, full = shard_problem(name, rank, world)
        ir = p.write(os.path.join(workdir, f"shard_{name}_{rank}"))
        k = Kernel.from_ir(ir)
        host = p.make_inputs(seed=p.seed + 1000 + rank)
        dev = {n: torch.from_numpy(v).to(device) for n, v in host.items()}
        for o in p.outputs:
            t = p.tensor(o)
            dev[o] = torch.empty(t["shape"], dtype={"f32": torch.float32, "s32": torch.int32,
                                                    "f64": torch.float64}[t["dtype"]],
                                 device=device)
            outs.append(dev[o])
        launches.append((k.bind(dev, stream=stream), dev))
        total_bytes += p.algorithmic_bytes() * world
    gathered = [torch.empty(world * t.numel(), dtype=t.dtype, device=device) for t in outs]

    def step(gather):
        with torch.cuda.stream(stream):
            for launch, _ in launches:
                launch()
            if gather:
                for g, t in zip(gathered, outs):
                    dist.all_gather_into_tensor(g, t.reshape(-1))

    res = {}
    for gather in (False, True):
        for _ in range(warmup):
            step(gather)
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            step(gather)
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / steps], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        key = "gather_incl" if gather else "kernel_only"
        res[key + "_ms"] = round(float(t.item()), 4)
        res[key + "_gbs"] = round(total_bytes / float(t.item()) / 1e6, 1)
    res["partition"] = "rows (1/N of 8192 rows per rank), NCCL all_gather_into_tensor of outputs"
    return res


# ----------------------------------------------------------------------------
# fused exchange: kernels store into peers' buffers over NVLink
# ----------------------------------------------------------------------------
class _IpcOps:
    """The device-memory calls PeerBuffer makes (runtime's, by default)."""

    def alloc(self, nbytes):
        from .runtime import DeviceBuffer
        return DeviceBuffer(nbytes)

    def handle(self, ptr):
        from .runtime import ipc_handle
        return ipc_handle(ptr)

    def open(self, handle):
        from .runtime import ipc_open
        return ipc_open(handle)

    def close(self, ptr):
        from .runtime import ipc_close
        ipc_close(ptr)


class PeerBuffer:
    """One device buffer per rank, mapped into every other rank with CUDA
    IPC.  ``ptrs[r]`` is rank r's buffer as this process addresses it (its
    own buffer for r == rank), so a kernel given the table can store into
    every rank's copy.  Collective: every rank constructs and closes it."""

    def __init__(self, nbytes: int, group=None, ops=None):
        import torch.distributed as dist
        self.ops = ops or _IpcOps()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = int(nbytes)
        self.local, self.ptrs, self._opened = None, [], []
        # every rank takes the same collective steps whatever fails, so a
        # failure on one rank raises on all of them instead of leaving the
        # others waiting in a collective
        handle, err = None, None
        try:
            self.local = self.ops.alloc(self.nbytes)
            handle = self.ops.handle(self.local.ptr)
        except Exception as exc:  # noqa: BLE001
            err = f"{type(exc).__name__}: {exc}"
        handles = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle, err), group=group)
        failed = [(r, e) for r, _, e in handles if e]
        if failed:
            if self.local is not None:
                self.local.free()
            raise RuntimeError(f"PeerBuffer: rank {failed[0][0]} could not export its "
                               f"buffer: {failed[0][1]}")
        err = None
        try:
            for r, h, _ in sorted(handles, key=lambda x: x[0]):
                if r == self.rank:
                    self.ptrs.append(self.local.ptr)
                else:
                    p = self.ops.open(h)
                    self._opened.append(p)
                    self.ptrs.append(p)
        except Exception as exc:  # noqa: BLE001
            err = f"{type(exc).__name__}: {exc}"
        status = [None] * self.world
        dist.all_gather_object(status, err, group=group)
        if any(status):
            bad = next(i for i, e in enumerate(status) if e)
            self.close()
            raise RuntimeError(f"PeerBuffer: rank {bad} could not map a peer: {status[bad]}")

    def close(self):
        """Unmap peers, wait for every rank to do the same, then free."""
        import torch.distributed as dist
        for p in self._opened:
            self.ops.close(p)
        self._opened = []
        dist.barrier(group=self.group)
        if self.local is not None:
            self.local.free()
            self.local = None


class FusedGather:
    """Rank ``rank``'s shard of ``name`` ("matmul": row blocks of C;
    "attention": (batch x head) pairs of O; "rmsnorm" / "softmax": row
    blocks) whose epilogue all-gathers the output: after ``launch()`` and
    ``wait()`` on every rank, ``out`` holds the full output on every rank.
    ``bind`` takes the shard's buffers (its own output buffer is not
    written)."""

    def __init__(self, name: str, rank: int, world: int, workdir, group=None, **kw):
        from .compiler import Compiler
        from .runtime import Kernel
        from .sm100 import attention, matmul, rows
        if name not in ("matmul", "attention", "rmsnorm", "softmax"):
            raise ValueError(f"no fused all-gather for {name}")
        self.name, self.rank, self.world, self.group = name, rank, world, group
        self.part, self.full = shard_problem(name, rank, world, **kw)
        ir = self.part.write(os.path.join(workdir, f"fused_{name}_{rank}"))
        comp = Compiler(ir, target="sm_100a", ptx_version="8.7")
        mod = {"matmul": matmul, "attention": attention}.get(name, rows)
        ptx, side = mod.emit(comp, mod.match(comp), gather=world)
        geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
        self.kernel = Kernel(ptx, comp.entry, Kernel._arg_specs(comp), geom, side)
        f = self.full
        if name == "matmul":
            total = f["m"] * f["n"] * 4
            row0 = rank * self.part.tensor("A")["shape"][0]
        elif name in ("rmsnorm", "softmax"):
            total = f["rows"] * f["cols"] * 4
            row0 = rank * self.part.tensor("x")["shape"][0]
        else:
            total = f["batch"] * f["heads"] * f["seq"] * f["head_dim"] * 4
            row0 = rank * self.part.tensor("q")["shape"][1] * f["seq"]
        self.out = PeerBuffer(total, group)
        # each rank starts with the next rank's buffer and goes round, so at
        # any moment the ranks' stores go to different destinations
        order = [self.out.ptrs[(rank + 1 + i) % world] for i in range(world)]
        self.kernel.set_global("emmy_gather_dst", struct.pack(f"<{world}Q", *order))
        self.kernel.set_global("emmy_gather_n", struct.pack("<I", world))
        self.kernel.set_global("emmy_gather_row0", struct.pack("<I", row0))
        self._launch = None
        self._flag = None

    def bind(self, buffers: dict, stream=None):
        import torch
        self._launch = self.kernel.bind(buffers, stream=stream)
        self._flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda",
                                                                          torch.cuda.current_device()))
        return self

    def launch(self):
        self._launch()

    def wait(self):
        """Stream-ordered completion barrier: a one-element all-reduce that
        finishes only after every rank's kernel (and so its stores into
        this rank's output) has finished."""
        import torch.distributed as dist
        dist.all_reduce(self._flag, group=self.group)

    def close(self):
        self.kernel.free_scratch()
        self.out.close()


class CopyGather:
    """Rank ``rank``'s shard of ``name`` whose output all-gather runs on the
    copy engines.  Every partition with a contiguous, rank-major output
    (rows, row blocks of C, (batch x head) pairs) works: the shard's kernel
    writes straight into this rank's part of its full output (``out.local``),
    then one device-to-device copy per peer (``ert_memcpy_dtod`` into the
    peer's full output, mapped with CUDA IPC) moves it over NVLink, one
    stream per peer so the copies run on several engines at once.  With
    ``chunks`` > 1 the shard runs as that many sub-shards (separate
    launches), and a sub-shard's copies overlap the next one's kernel.
    After ``launch()`` and ``wait()`` on every rank, ``out.local`` holds the
    full output everywhere."""

    def __init__(self, name: str, rank: int, world: int, workdir, chunks: int = 1,
                 group=None, **kw):
        from .runtime import Event, Kernel, Stream
        if PARTITION[name] == "cols":
            raise ValueError(f"{name}'s output is not rank-major contiguous")
        self.name, self.rank, self.world, self.group = name, rank, world, group
        self.part, self.full = shard_problem(name, rank, world, **kw)
        self.sub, _ = shard_problem(name, rank * chunks, world * chunks, **kw)
        self.chunks = chunks
        self.kernel = Kernel.from_ir(self.sub.write(os.path.join(workdir,
                                                                 f"copyg_{name}_{rank}")))
        # one module per sub-shard: a tensor-map kernel keeps its maps in
        # module globals, so each sub-shard's launch has its own
        self.kernels = [self.kernel] + [
            Kernel(self.kernel.ptx, self.kernel.entry, self.kernel.args,
                   self.kernel.meta_geom, self.kernel.sidecar) for _ in range(chunks - 1)]
        out = self.part.outputs[0]
        self.out_name = out
        numel = lambda p, t: int(np.prod(p.tensor(t)["shape"]))  # noqa: E731
        self.sub_bytes = numel(self.sub, out) * 4
        self.part_bytes = numel(self.part, out) * 4
        self.out = PeerBuffer(self.part_bytes * world, group)
        self.copy_streams = [Stream() for _ in range(world)]
        self.k_done = [Event() for _ in range(chunks)]
        self.c_done = [Event() for _ in range(world)]
        self._launches = None

    def bind(self, buffers: dict, stream=None):
        """``buffers``: the shard's inputs; an input that the sub-shards
        split (its sub-shard shape differs from the shard's) is cut into
        consecutive blocks, the others are shared.  The output argument is
        this rank's part of ``out.local``."""
        from .runtime import _stream_handle
        self.stream = _stream_handle(stream)
        self._launches = []
        for c in range(self.chunks):
            bufs = {}
            for t in self.part.inputs:
                ten = buffers[t]
                ptr = ten.data_ptr() if hasattr(ten, "data_ptr") else int(ten)
                if self.sub.tensor(t)["shape"] != self.part.tensor(t)["shape"]:
                    esz = ten.element_size() if hasattr(ten, "element_size") else 4
                    ptr += c * int(np.prod(self.sub.tensor(t)["shape"])) * esz
                bufs[t] = ptr
            bufs[self.out_name] = (self.out.local.ptr + self.rank * self.part_bytes
                                   + c * self.sub_bytes)
            self._launches.append(self.kernels[c].bind(bufs, stream=self.stream))
        return self

    def launch(self):
        from .runtime import check, lib
        L = lib()
        nbytes = self.sub_bytes
        for c, launch in enumerate(self._launches):
            launch()
            self.k_done[c].record(self.stream)
            off = self.rank * self.part_bytes + c * self.sub_bytes
            for i in range(1, self.world):
                d = (self.rank + i) % self.world
                cs = self.copy_streams[d]
                cs.wait(self.k_done[c])
                check(L.ert_memcpy_dtod(self.out.ptrs[d] + off, self.out.local.ptr + off,
                                        nbytes, cs.handle), "ert_memcpy_dtod")
        # the launching stream waits for every copy
        for i in range(1, self.world):
            d = (self.rank + i) % self.world
            self.c_done[d].record(self.copy_streams[d])
            check(L.ert_stream_wait_event(self.stream, self.c_done[d].handle),
                  "ert_stream_wait_event")

    def wait(self):
        """Stream-ordered completion barrier: a one-element all-reduce that
        finishes only after every rank's copies into this rank have."""
        import torch
        import torch.distributed as dist
        if not hasattr(self, "_flag"):
            self._flag = torch.zeros(1, dtype=torch.int32,
                                     device=torch.device("cuda", torch.cuda.current_device()))
        dist.all_reduce(self._flag, group=self.group)

    def close(self):
        for s in self.copy_streams:
            s.synchronize()
        for k in self.kernels:
            k.free_scratch()
        self.out.close()
        for s in self.copy_streams:
            s.destroy()
        for e in self.k_done + self.c_done:
            e.destroy()


class FusedGatherMatmul(FusedGather):
    """``FusedGather("matmul", ...)``."""

    def __init__(self, rank: int, world: int, workdir, group=None, **kw):
        super().__init__("matmul", rank, world, workdir, group, **kw)


def bench_fused_gather(name, workdir, device, stream, rank, world, steps=5, warmup=2, **kw):
    """Strong scaling of ``name`` ("matmul" or "attention"): kernel only,
    kernel + NCCL all-gather of the output, and the fused kernel whose
    epilogue stores into every rank's output (each max over ranks, ms and
    whole-job TFLOP/s)."""
    import torch
    import torch.distributed as dist
    from .runtime import Kernel
    p, full = shard_problem(name, rank, world, **kw)
    fullp = workloads.build(name, **full)
    flops = fullp.algorithmic_flops()
    host = p.make_inputs(seed=p.seed + 1000 + rank)
    dev = {n: torch.from_numpy(v).to(device) for n, v in host.items()}
    out = p.outputs[0]
    dev[out] = torch.empty(p.tensor(out)["shape"], dtype=torch.float32, device=device)
    plain = Kernel.from_ir(p.write(os.path.join(workdir, f"{name}_shard_{rank}")))
    plain_launch = plain.bind(dev, stream=stream)
    gathered = torch.empty(world * dev[out].numel(), dtype=torch.float32, device=device)
    fused = FusedGather(name, rank, world, workdir, **kw).bind(dev, stream=stream)

    def run(step):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / steps], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def kernel_only():
        with torch.cuda.stream(stream):
            plain_launch()

    def nccl():
        with torch.cuda.stream(stream):
            plain_launch()
            dist.all_gather_into_tensor(gathered, dev[out].reshape(-1))

    def fused_step():
        with torch.cuda.stream(stream):
            fused.launch()
            fused.wait()

    res = {}
    for key, fn in (("kernel_only", kernel_only), ("nccl_gather_incl", nccl),
                    ("fused_gather_incl", fused_step)):
        ms = run(fn)
        res[key + "_ms"] = round(ms, 4)
        res[key + "_tflops"] = round(flops / ms / 1e9, 1)
    torch.cuda.synchronize()
    fused.close()
    plain.free_scratch()
    # the copy engines instead: two sub-shard launches, each followed by one
    # copy per peer
    copy = CopyGather(name, rank, world, workdir, chunks=2, **kw).bind(dev, stream=stream)

    def copy_step():
        with torch.cuda.stream(stream):
            copy.launch()
            copy.wait()

    ms = run(copy_step)
    res["copy_gather_incl_ms"] = round(ms, 4)
    res["copy_gather_incl_tflops"] = round(flops / ms / 1e9, 1)
    torch.cuda.synchronize()
    copy.close()
    if name == "matmul":
        res["partition"] = (f"row blocks of C ({full['m'] // world} of {full['m']} rows per rank, "
                            "B replicated)")
    else:
        res["partition"] = f"(batch x head) pairs ({full['batch'] * full['heads'] // world} per rank)"
    return res


def bench_matmul_gather(workdir, device, stream, rank, world, steps=5, warmup=2, **kw):
    return bench_fused_gather("matmul", workdir, device, stream, rank, world, steps, warmup, **kw)
