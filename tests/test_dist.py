"""Sharded execution across ranks: world_size-2 gloo processes on the CPU.

Each rank slices its shard of the full seeded inputs (emmy_ptx.dist), runs
the shard's own IR package (through the oracle, since there is no GPU here),
all-gathers the outputs with the same collective the GPU path uses, and
must reproduce the unsharded result exactly.
"""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

SMALL = {
    "pointwise_f32": dict(rows=8, cols=64),
    "pointwise_i32": dict(rows=8, cols=64),
    "rmsnorm": dict(rows=4, cols=256),
    "softmax": dict(rows=4, cols=512),
    "rowsum_i32": dict(rows=8, cols=64),
    "colreduce_f64": dict(rows=32, cols=128),
    "matmul": dict(m=256, n=128, k=32),
    "attention": dict(batch=2, heads=2, seq=32, head_dim=32),
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, kw, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "emmy-ptx_b200")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    from emmy_ptx import dist as edist
    from emmy_ptx import workloads
    from oracle import simt
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full_p = workloads.build(name, **kw)
        full_inputs = full_p.make_inputs()
        shard_p, _ = edist.shard_problem(name, rank, world, **kw)
        shard_in = edist.shard_inputs(name, full_inputs, rank, world)
        with tempfile.TemporaryDirectory() as td:
            outs = simt.run_problem(shard_p, shard_in, td)
        tensors = {o: torch.from_numpy(np.ascontiguousarray(v)) for o, v in outs.items()}
        gathered = edist.all_gather_outputs(tensors)
        shapes = {o: full_p.tensor(o)["shape"] for o in full_p.outputs}
        full = edist.assemble({o: t.numpy() for o, t in gathered.items()}, shapes)
        if rank == 0:
            np.savez(os.path.join(out_dir, "gathered.npz"), **full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", list(SMALL))
def test_two_rank_shards_gather_to_the_full_result(name, tmp_path):
    from emmy_ptx import workloads
    from oracle import simt
    kw = SMALL[name]
    mp.start_processes(_worker, args=(2, _free_port(), name, kw, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    got = np.load(tmp_path / "gathered.npz")
    p = workloads.build(name, **kw)
    with tempfile.TemporaryDirectory() as td:
        want = simt.run_problem(p, p.make_inputs(), td)
    for o in p.outputs:
        np.testing.assert_array_equal(got[o], want[o])


def test_shard_ranges_cover_exactly_once():
    from emmy_ptx import dist as edist
    for world in (1, 2, 4, 8):
        spans = [edist.shard_range(64, r, world) for r in range(world)]
        covered = sorted(i for s, n in spans for i in range(s, s + n))
        assert covered == list(range(64))
    with pytest.raises(ValueError):
        edist.shard_range(10, 0, 4)


def _dropout_worker(rank, world, port, out_dir):
    """Rank 1 leaves before the collective; rank 0 must get an error from
    the process group's timeout instead of waiting forever."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return                              # leaves between steps, nothing in flight
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "emmy-ptx_b200"))
    from emmy_ptx import dist as edist
    try:
        edist.all_gather_outputs({"out": torch.ones(4)})
        result = "no error"
    except Exception as exc:  # noqa: BLE001
        result = "error: " + type(exc).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(result)


def test_a_rank_that_leaves_is_detected_by_the_collective_timeout(tmp_path):
    mp.start_processes(_dropout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    assert (tmp_path / "rank0.txt").read_text().startswith("error")


class _FakeBuf:
    def __init__(self, ptr):
        self.ptr = ptr
        self.freed = False

    def free(self):
        self.freed = True


class _FakeIpc:
    """Device calls of PeerBuffer, on the host: rank r's buffer is at
    0x1000 * (r + 1); a handle names its owner; opening gives a distinct
    mapped address."""

    def __init__(self, rank):
        self.rank = rank
        self.closed = []
        self.buf = None

    def alloc(self, nbytes):
        self.buf = _FakeBuf(0x1000 * (self.rank + 1))
        return self.buf

    def handle(self, ptr):
        return b"owner=%d" % (ptr // 0x1000 - 1)

    def open(self, handle):
        owner = int(handle.split(b"=")[1])
        return 0x100000 * (owner + 1) + 0x10 * (self.rank + 1)

    def close(self, ptr):
        self.closed.append(ptr)


def _peer_worker(rank, world, port, out_dir):
    import json
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "emmy-ptx_b200"))
    import torch.distributed as dist
    from emmy_ptx import dist as edist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops = _FakeIpc(rank)
        pb = edist.PeerBuffer(4096, ops=ops)
        ptrs = list(pb.ptrs)
        pb.close()
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump({"ptrs": ptrs, "closed": ops.closed, "freed": ops.buf.freed}, f)
    finally:
        dist.destroy_process_group()


def test_peer_buffer_tables_are_rank_ordered(tmp_path):
    """Every rank's table lists rank 0..N-1: its own buffer in its own slot,
    each peer's buffer as opened from that peer's handle; close() unmaps
    every opened peer and frees the local buffer."""
    import json
    world = 3
    mp.start_processes(_peer_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        d = json.loads((tmp_path / f"r{r}.json").read_text())
        want = [0x1000 * (r + 1) if o == r else 0x100000 * (o + 1) + 0x10 * (r + 1)
                for o in range(world)]
        assert d["ptrs"] == want
        assert sorted(d["closed"]) == sorted(p for o, p in enumerate(want) if o != r)
        assert d["freed"]


def test_copy_gather_offsets_cover_the_output_once():
    """The copy-engine gather's sub-shards: for every partition with a
    rank-major contiguous output, rank r's chunk c lands at
    r * part + c * sub bytes, and the chunks of all ranks tile the full
    output exactly once (checked on the shapes alone, no device)."""
    from emmy_ptx import dist as edist
    for name, kw in [("softmax", dict(rows=64, cols=256)), ("rmsnorm", dict(rows=32, cols=128)),
                     ("matmul", dict(m=512, n=128, k=64)),
                     ("attention", dict(batch=2, heads=4, seq=64, head_dim=32))]:
        world, chunks = 2, 2
        full = edist.workloads.build(name, **kw)
        out = full.outputs[0]
        total = int(np.prod(full.tensor(out)["shape"])) * 4
        spans = []
        for r in range(world):
            part, _ = edist.shard_problem(name, r, world, **kw)
            sub, _ = edist.shard_problem(name, r * chunks, world * chunks, **kw)
            pb = int(np.prod(part.tensor(out)["shape"])) * 4
            sb = int(np.prod(sub.tensor(out)["shape"])) * 4
            assert pb == chunks * sb and world * pb == total, name
            spans += [(r * pb + c * sb, sb) for c in range(chunks)]
        pos = 0
        for off, n in sorted(spans):
            assert off == pos, name
            pos += n
        assert pos == total, name
