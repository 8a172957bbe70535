"""Host-buffer pipeline: overlap host->device copies, kernels and
device->host copies for row-partitioned problems, through the C ABI only.

A problem whose rows are independent (pointwise, RMSNorm, softmax, row
sums; see ``dist.PARTITION``) is cut into ``chunks`` equal row blocks.  The
kernel is compiled once for the chunk shape.  Three streams of the C ABI
(``ert_stream_create``) carry the work, one per engine:

* ``h2d``: chunk c's inputs into device slot ``c % slots``;
* ``compute``: the kernel on that slot;
* ``d2h``: the slot's outputs back to the host.

Events order them per slot: the kernel waits for its inputs' copy and for
the previous copy-out of the slot's outputs; the copy-out waits for the
kernel; the next copy-in of a slot waits for the kernel that read it.  So
copy-in of chunk c+1 runs while chunk c computes and chunk c-1 copies out,
and neither copy direction ever queues behind the other.  Several runners
may share one ``PipelineStreams`` so that consecutive problems chain
without draining the link in between.  Host arrays must be page-locked
(``runtime.PinnedArray``) for the copies to be asynchronous.

Every call here is an ``ert_*`` call of ``include/emmy_rt.h``, so a C caller
can run the same loop.
"""

from __future__ import annotations

import os
import tempfile

import numpy as np

from . import dist, workloads
from .runtime import DeviceBuffer, Event, Kernel, NP_DTYPE, PinnedArray, Stream, check, lib


class PipelineStreams:
    """The three streams of a pipeline (copy-in, compute, copy-out)."""

    def __init__(self):
        self.h2d, self.compute, self.d2h = Stream(), Stream(), Stream()

    def all(self):
        return (self.h2d, self.compute, self.d2h)

    def after(self, event: Event):
        """All three streams wait for ``event`` (e.g. a step's start mark)."""
        for s in self.all():
            s.wait(event)

    def join(self, stream: Stream, marks: list) -> None:
        """``stream`` waits for all work queued so far on the three streams
        (``marks``: three Events of the caller's, re-recorded here)."""
        for s, ev in zip(self.all(), marks):
            ev.record(s)
            stream.wait(ev)

    def synchronize(self):
        for s in self.all():
            s.synchronize()

    def destroy(self):
        for s in self.all():
            s.destroy()


class _Slot:
    def __init__(self, kernel: Kernel, stream: Stream):
        self.bufs = {}
        for a in kernel.args:
            n = int(np.prod(a["shape"])) * np.dtype(NP_DTYPE[a["dtype"]]).itemsize
            self.bufs[a["name"]] = DeviceBuffer(n)
        self.launch = kernel.bind({k: b.ptr for k, b in self.bufs.items()},
                                  stream=stream.handle)
        self.in_ready, self.k_done, self.out_done = Event(), Event(), Event()

    def free(self):
        for b in self.bufs.values():
            b.free()
        for e in (self.in_ready, self.k_done, self.out_done):
            e.destroy()


class ChunkedHostRunner:
    def __init__(self, name: str, chunks: int = 16, slots: int = 3, workdir=None,
                 streams: PipelineStreams | None = None, **kw):
        if dist.PARTITION[name] != "rows":
            raise ValueError(f"{name} is not partitioned by rows")
        if slots < 2:
            raise ValueError("the pipeline needs at least two device slots")
        self.name = name
        self.chunks = chunks
        self.full = workloads.build(name, **kw)
        self.part, _ = dist.shard_problem(name, 0, chunks, **kw)
        wd = workdir or tempfile.mkdtemp(prefix="emmy_pipe_")
        self.kernel = Kernel.from_ir(self.part.write(os.path.join(wd, f"{name}_chunk{chunks}")))
        self.own_streams = streams is None
        self.ps = streams or PipelineStreams()
        self.slots = [_Slot(self.kernel, self.ps.compute) for _ in range(min(slots, chunks))]
        self.row_split = {t: self.full.tensor(t)["shape"][0] != self.part.tensor(t)["shape"][0]
                          for t in self.full.inputs + self.full.outputs}
        self.last_bytes = (0, 0)

    @property
    def streams(self):
        return list(self.ps.all())

    def run(self, host_in: dict, host_out: dict, sync=True):
        """``host_in``/``host_out``: full-size PinnedArray (or contiguous
        numpy) per tensor name.  Queues every chunk; with ``sync`` waits for
        the last copy-out."""
        L = lib()
        h2d_s, cmp_s, d2h_s = (s.handle for s in self.ps.all())
        h2d = d2h = 0
        for c in range(self.chunks):
            slot = self.slots[c % len(self.slots)]
            if slot.k_done.recorded:            # the slot's inputs were read
                self.ps.h2d.wait(slot.k_done)
            for t in self.full.inputs:
                arr = host_in[t].array if isinstance(host_in[t], PinnedArray) else host_in[t]
                src = arr.reshape(self.chunks, -1)[c] if self.row_split[t] else arr.reshape(-1)
                check(L.ert_memcpy_htod(slot.bufs[t].ptr, src.ctypes.data, src.nbytes, h2d_s),
                      "ert_memcpy_htod")
                h2d += src.nbytes
            slot.in_ready.record(h2d_s)
            self.ps.compute.wait(slot.in_ready)
            if slot.out_done.recorded:          # the slot's outputs were copied out
                self.ps.compute.wait(slot.out_done)
            slot.launch()
            slot.k_done.record(cmp_s)
            self.ps.d2h.wait(slot.k_done)
            for t in self.full.outputs:
                arr = host_out[t].array if isinstance(host_out[t], PinnedArray) else host_out[t]
                dst = arr.reshape(self.chunks, -1)[c]
                check(L.ert_memcpy_dtoh(dst.ctypes.data, slot.bufs[t].ptr, dst.nbytes, d2h_s),
                      "ert_memcpy_dtoh")
                d2h += dst.nbytes
            slot.out_done.record(d2h_s)
        if sync:
            self.ps.d2h.synchronize()
        self.last_bytes = (h2d, d2h)
        return host_out

    def free(self):
        self.ps.synchronize()
        for s in self.slots:
            s.free()
        self.slots = []
        if self.own_streams:
            self.ps.destroy()
