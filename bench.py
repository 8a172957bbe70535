#!/usr/bin/env python
"""Benchmark: Emmy kernels lowered to sm_100a, launched through libemmy_rt.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload (the fused row kernels): one step is
the RMSNorm kernel over x[8192, 4096] followed by the row-softmax kernel
over logits[8192, 32768], both compiled from their Emmy IR packages by
``emmy_ptx.Compiler(target="sm_100a")`` and launched through the C ABI.
``value`` = algorithmic HBM bytes of the whole config (every input read
once, every output written once) / device time of the step, in GB/s.
Inputs (2.4 GB per step) are larger than the 126 MB L2, so no flush is
needed between steps.

N > 1 (torchrun): strong scaling, the north star's sharded path -- every
rank runs its 1/N of the rows of both kernels, and both full outputs are on
every rank at the end of the timed step (max over ranks).  The exchange is
``GATHER_MODE``: by default the row kernels' gather variant stores every
output row into every rank's output over NVLink.  The same step with NCCL
``all_gather_into_tensor``, with the copy-engine gather, and with the
kernels alone, and the matmul / attention shards (NCCL, copy-engine and
fused epilogue gathers), are reported under ``"sharded"``.

``e2e`` is the same config through the host-buffer pipeline of the C ABI
(pinned host rows -> device -> kernels -> pinned host, every step; each
rank moves its own rows).

The CPU baseline (``cpu_baseline`` at N=1, and ``--impl reference``) is the
same computation with torch's CPU operators on every host core over the
whole config (oracle/torch_cpu.py): the reference compiler itself runs no
kernels, it writes PTX for an outside runner.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "emmy-ptx_b200"))

NVLINK_GBS = 770.0    # peer copy per direction per GPU, measured on this pool
# how the headline step's outputs reach every rank at N > 1: "fused" (the row
# kernels' epilogues store into every rank's output) or "copy" (the kernels
# write this rank's rows locally, the copy engines move them to the peers)
GATHER_MODE = "fused"
COPY_CHUNKS = 2
METRIC = "HBM GB/s (pointwise/norm) & TFLOP/s (matmul/attn) vs ref PTX, at 1/2/4/8 B200"
HEADLINE = ("rmsnorm", "softmax")
WORKLOAD = "config 2: RMSNorm [8192,4096] + row softmax [8192,32768], f32"
GOLDEN = ROOT / "tests" / "golden" / "problems"
DTYPES = {"f32": "float32", "f64": "float64", "s32": "int32", "bf16": "bfloat16",
          "f16": "float16", "u8": "uint8"}


def peaks():
    try:
        m = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return {"hbm_gbs": float(m["hbm_gbs"]), "bf16_tflops": float(m["bf16_tflops"]),
                "source": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------
class Clocks:
    """Samples SM clock and clock-event (throttle) reasons through NVML in a
    background thread while the timed region runs (reading only)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index, period_s=0.002):
        self.index = device_index
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self.error = None

    def _handle(self, pynvml):
        try:
            import torch
            props = torch.cuda.get_device_properties(self.index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = self._handle(pynvml)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # noqa: BLE001
            self.error = f"nvml unavailable: {exc}"
            return
        self._stop = threading.Event()

        def loop():
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self._stop.is_set():
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    self.reasons |= int(get_reasons(h))
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(self.period)
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def stop(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error or "no samples"]}
        self._stop.set()
        self._thread.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for bit, n in self.REASONS.items() if self.reasons & bit),
                "samples": len(self.samples), "source": "NVML, 2 ms period"}


# ----------------------------------------------------------------------------
# problems on the device
# ----------------------------------------------------------------------------
class Bound:
    """One compiled problem with device buffers and a pre-bound launch."""

    def __init__(self, name, workdir, device, stream, seed_offset=0, rows=None,
                 ptx=None, general=False, **kw):
        import torch
        from emmy_ptx import workloads
        from emmy_ptx.runtime import Kernel
        if rows is not None:
            kw["rows"] = rows
        self.problem = p = workloads.build(name, **kw)
        tag = "_ref" if ptx else ("_general" if general else "")
        ir = p.write(os.path.join(workdir, name + tag + str(rows or "")))
        if ptx:
            self.kernel = Kernel.from_ptx(ptx, ir)
        elif general:
            # the general statement-level lowering, bypassing the category kernel
            from emmy_ptx.compiler import Compiler
            from emmy_ptx.sm100 import general as general_path
            comp = Compiler(ir, target="sm_100a", ptx_version="8.7")
            gptx, side = general_path.emit(comp)
            geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
            self.kernel = Kernel(gptx, comp.entry, Kernel._arg_specs(comp), geom, side)
        else:
            self.kernel = Kernel.from_ir(ir)
        self.host = p.make_inputs(seed=p.seed + seed_offset)
        self.dev = {k: torch.from_numpy(v).to(device) for k, v in self.host.items()}
        for o in p.outputs:
            t = p.tensor(o)
            self.dev[o] = torch.empty(t["shape"], dtype=getattr(torch, DTYPES[t["dtype"]]),
                                      device=device)
        self.launch = self.kernel.bind(self.dev, stream=stream,
                                       geometry="meta" if ptx else "tuned")
        self.bytes = p.algorithmic_bytes()
        self.flops = p.algorithmic_flops()


def _events(n):
    import torch
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def time_kernel(bound, reps, warmup, stream):
    """Average device time of back-to-back launches (inputs > L2 or
    compute-bound, as stated per category)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            bound.launch()
    torch.cuda.synchronize()
    s, e = _events(2)
    with torch.cuda.stream(stream):
        s.record(stream)
        for _ in range(reps):
            bound.launch()
        e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


# ----------------------------------------------------------------------------
# end to end through the host-buffer C-ABI path
# ----------------------------------------------------------------------------
def link_probe(device, h2d_bytes, d2h_bytes, barrier, max_over_ranks, reps=3, chunks=16):
    """The ceiling of the end-to-end step: the same volume moved the same way
    with no kernels -- every rank copies its step's inputs in and outputs out
    (pinned host buffers, one stream per direction, both in flight at once,
    each direction in ``chunks`` copies as the pipeline makes them), all
    ranks starting together after a barrier, timed with CUDA events, max
    over ranks; best of ``reps`` after a warm-up.  Returns (ms, this rank's
    own ms)."""
    import torch
    h_in = torch.empty(h2d_bytes // 4, dtype=torch.float32).pin_memory()
    h_out = torch.empty(d2h_bytes // 4, dtype=torch.float32).pin_memory()
    d_in = torch.empty(h2d_bytes // 4, device=device)
    d_out = torch.zeros(d2h_bytes // 4, device=device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    cur = torch.cuda.current_stream(device)
    best = mine = None
    for i in range(reps + 1):
        torch.cuda.synchronize(device)
        barrier()
        a, e = _events(2)
        a.record(cur)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            for dst, src in zip(d_in.chunk(chunks), h_in.chunk(chunks)):
                dst.copy_(src, non_blocking=True)
        with torch.cuda.stream(s_out):
            for dst, src in zip(h_out.chunk(chunks), d_out.chunk(chunks)):
                dst.copy_(src, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        e.record(cur)
        torch.cuda.synchronize(device)
        t = a.elapsed_time(e)
        tmax = max_over_ranks(t)
        if i:
            if best is None or tmax < best:
                best, mine = tmax, t
    del h_in, h_out, d_in, d_out
    return best, mine


def e2e_measure(names, workdir, steps, warmup, seed_offset, chunks=16, slots=3, rows_div=1,
                barrier=None):
    """The same step through the public host-buffer API: pinned host inputs
    -> device, the kernels, device -> pinned host outputs, every step.  Rows
    are cut into ``chunks`` blocks; copy-in, kernels and copy-out run on three
    streams of the C ABI, ordered per device slot by events
    (emmy_ptx.pipeline), and the problems share the streams so one step's
    copies never drain the link between problems.  ``barrier`` (several
    ranks): called after the warm-up, so that every rank's timed steps run
    at the same time and share the host links as they would in a job."""
    from emmy_ptx.pipeline import ChunkedHostRunner, PipelineStreams
    from emmy_ptx.runtime import Event, PinnedArray
    ps = PipelineStreams()
    runners = []
    total_bytes = 0
    for name in names:
        kw = {}
        if rows_div > 1:          # this rank's 1/rows_div of the rows
            from emmy_ptx import dist as edist
            kw["rows"] = edist.FULL_DEFAULTS[name]["rows"] // rows_div
        r = ChunkedHostRunner(name, chunks=chunks, slots=slots, workdir=workdir, streams=ps,
                              **kw)
        p = r.full
        host = {}
        for n, arr in p.make_inputs(seed=p.seed + seed_offset).items():
            pa = PinnedArray(arr.shape, arr.dtype)
            pa.array[...] = arr
            host[n] = pa
        outs = {o: PinnedArray(p.tensor(o)["shape"], DTYPES[p.tensor(o)["dtype"]])
                for o in p.outputs}
        runners.append((r, host, outs))
        total_bytes += p.algorithmic_bytes()
    for _ in range(warmup):
        for r, host, outs in runners:
            r.run(host, outs, sync=False)
    ps.synchronize()
    if barrier is not None:
        barrier()
    start, end = Event(), Event()
    marks = [Event() for _ in range(3)]
    start.record(ps.h2d)
    ps.after(start)
    h2d = d2h = 0
    for _ in range(steps):
        for r, host, outs in runners:
            r.run(host, outs, sync=False)
            h2d += r.last_bytes[0]
            d2h += r.last_bytes[1]
    ps.join(ps.d2h, marks)
    end.record(ps.d2h)
    end.synchronize()
    ms = start.elapsed_ms(end) / steps
    launches = sum(r.kernel.launches for r, _, _ in runners)
    for r, host, outs in runners:
        r.free()
        for pa in list(host.values()) + list(outs.values()):
            pa.free()
    for ev in [start, end] + marks:
        ev.destroy()
    ps.destroy()
    return {"ms_per_step": ms, "bytes": total_bytes, "h2d": h2d // steps, "d2h": d2h // steps,
            "launches": launches, "chunks": chunks, "slots": slots}


# ----------------------------------------------------------------------------
# CPU baseline: torch CPU operators over the whole configuration
# ----------------------------------------------------------------------------
def cpu_baseline(problems, steps, warmup, host_inputs=None):
    """The headline step's computation with torch's CPU operators on every
    host core (oracle/torch_cpu.py), over the whole configuration: RMSNorm
    by formula on x[8192, 4096], then torch.softmax on [8192, 32768].
    Median of ``steps`` timed steps after ``warmup``."""
    import torch
    sys.path.insert(0, str(ROOT))
    from oracle import torch_cpu
    inputs = None
    if host_inputs is not None:
        inputs = [{k: torch.from_numpy(v) for k, v in h.items()} for h in host_inputs]
    med, times, n = torch_cpu.time_problems(problems, steps, warmup, inputs=inputs)
    nbytes = sum(p.algorithmic_bytes() for p in problems)
    return {"value": round(nbytes / med / 1e9, 3), "unit": "GB/s", "cores": n,
            "kind": "port", "engine": "torch-cpu",
            "cpu": torch_cpu.cpu_model(),
            "sample": f"the whole config-2 step (RMSNorm 8192x4096 + softmax 8192x32768, "
                      f"{nbytes} algorithmic bytes) with torch {torch.__version__} CPU ops on "
                      f"{n} threads; median of {steps} after {warmup} warm-up, "
                      f"{statistics.median(times) * 1e3:.1f} ms per step"}


# ----------------------------------------------------------------------------
def run_reference(args):
    """The reference arm.  The reference compiler runs no kernels of its own
    (it writes PTX for an outside runner), so its CPU counterpart is the
    computation its IR states, evaluated by torch's CPU operators on every
    host core over the same configuration (oracle/torch_cpu.py).  Rank 0
    only; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from emmy_ptx import workloads
    problems = [workloads.build(n) for n in HEADLINE]
    cb = cpu_baseline(problems, args.steps, args.warmup)
    value = cb["value"]
    step_bytes = sum(p.algorithmic_bytes() for p in problems)
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_bytes / value / 1e6, 3),
        "higher_is_better": True, "scaling": "strong" if args.gpus > 1 else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded torch.Generator inputs of the config's shapes)",
        "config": config_block(args.gpus),
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def categories_sweep(workdir, device, stream, pk):
    """Every BASELINE config: this backend's kernel vs the reference
    compiler's PTX on the same B200 (back-to-back launches)."""
    from emmy_ptx import workloads
    out = {}
    tf32 = tf32_peak(device)
    out["tf32_peak_tflops"] = {"value": round(tf32, 1),
                               "how": "cuBLAS tf32 (torch.matmul, allow_tf32) 8192^3 f32 on this "
                                      "GPU, best of 10 after 3 warm-up"}
    sweep = list(workloads.FULL_SIZE.items()) + [("16-/8-bit (beyond the BASELINE configs)",
                                                 ("matmul_bf16", "matmul_e4m3"))]
    for cfg, names in sweep:
        for name in names:
            entry = {"config": cfg}
            try:
                mine = Bound(name, workdir, device, stream)
            except SystemExit as exc:
                out[name] = {"config": cfg, "error": str(exc).splitlines()[0]}
                continue
            compute = mine.flops > 0
            reps = 3 if compute else 10
            ms = time_kernel(mine, reps, 2, stream)
            entry["ms"] = round(ms, 4)
            if compute and mine.kernel.sidecar.get("operand_dtype") in ("bf16", "f16"):
                entry["tflops"] = round(mine.flops / ms / 1e9, 2)
                entry["frac_bf16_peak"] = round(mine.flops / ms / 1e9 / pk["bf16_tflops"], 3)
                entry["bf16_peak"] = f"{pk['bf16_tflops']:.1f} TFLOP/s (measured cuBLAS bf16)"
            elif compute and mine.kernel.sidecar.get("operand_dtype") in ("e4m3", "e5m2"):
                fp8 = 2 * pk["bf16_tflops"]
                entry["tflops"] = round(mine.flops / ms / 1e9, 2)
                entry["frac_fp8_peak"] = round(mine.flops / ms / 1e9 / fp8, 3)
                entry["fp8_peak"] = f"{fp8:.1f} TFLOP/s = 2 x measured bf16"
            elif compute:
                issued = mine.kernel.sidecar.get("tensor_flops_issued", mine.flops)
                entry["tflops"] = round(mine.flops / ms / 1e9, 2)
                entry["tflops_issued"] = round(issued / ms / 1e9, 2)
                entry["frac_tf32_alg"] = round(mine.flops / ms / 1e9 / tf32, 3)
                entry["frac_tf32_issued"] = round(issued / ms / 1e9 / tf32, 3)
                entry["tf32_peak"] = f"{tf32:.1f} TFLOP/s (measured cuBLAS tf32, this GPU)"
            else:
                entry["gbs"] = round(mine.bytes / ms / 1e6, 1)
                entry["frac_hbm"] = round(mine.bytes / ms / 1e6 / pk["hbm_gbs"], 3)
            ref = GOLDEN / f"{name}_full" / "ref.ptx"
            if ref.exists():
                rb = Bound(name, workdir, device, stream, ptx=ref.read_text())
                rms = time_kernel(rb, 1 if compute else 5, 1, stream)
                entry["ref_ptx_ms"] = round(rms, 4)
                entry["speedup_vs_ref_ptx"] = round(rms / ms, 2)
                del rb
                # the general statement-level lowering of the same IR
                gb = Bound(name, workdir, device, stream, general=True)
                gms = time_kernel(gb, 1 if compute else 5, 1, stream)
                entry["general_path_ms"] = round(gms, 4)
                entry["general_path_vs_ref_ptx"] = round(rms / gms, 2)
                del gb
            del mine
            out[name] = entry
    return out


def config_block(world):
    c = {"workload": WORKLOAD, "rows_total": 8192, "rows_per_rank": 8192 // world,
         "l2": "inputs larger than L2 (2.4 GB per step at N=1; at N>1 each rank's shard "
               "plus the 1.2 GB of gathered outputs)"}
    if world > 1:
        c["exchange"] = ("each rank runs its 1/N of the rows of both kernels; their "
                         "epilogues store every output row into every rank's full output "
                         "over NVLink (peer stores), then a one-element NCCL all-reduce "
                         "marks completion, inside the timed step")
        c["parallelism"] = f"rows/{world}"
    return c


class HeadlineStep:
    """The headline step on this rank.  N=1: the whole config.  N>1 (strong
    scaling): this rank's 1/N of the rows of every problem (each rank's rows
    seeded on their own), and both full outputs on every rank at the end of
    the step.  ``gather="fused"``: the row kernels' gather variant stores
    every output row into every rank's full output over NVLink
    (dist.FusedGather), then a one-element NCCL all-reduce on the stream
    marks completion; ``gather="copy"``: the kernels into this rank's part
    of its full output, copy engines to the peers (dist.CopyGather);
    ``gather="nccl"``: the plain kernels, then NCCL all_gather_into_tensor of
    every output."""

    def __init__(self, workdir, device, stream, rank, world, gather="fused"):
        import torch
        from emmy_ptx import dist as edist
        from emmy_ptx import workloads
        self.world, self.stream, self.gather = world, stream, gather
        rows = {n: edist.FULL_DEFAULTS[n]["rows"] for n in HEADLINE}
        self.bounds = [Bound(n, workdir, device, stream, seed_offset=rank,
                             rows=rows[n] // world if world > 1 else None) for n in HEADLINE]
        self.full_bytes = sum(workloads.build(n).algorithmic_bytes() for n in HEADLINE)
        self.outs, self.gathered, self.fused = [], [], []
        if world > 1 and gather == "nccl":
            for b in self.bounds:
                for o in b.problem.outputs:
                    t = b.dev[o]
                    self.outs.append(t.reshape(-1))
                    self.gathered.append(torch.empty(world * t.numel(), dtype=t.dtype,
                                                     device=device))
        elif world > 1 and gather == "copy":
            for b in self.bounds:
                cg = edist.CopyGather(b.problem.name, rank, world, workdir, chunks=COPY_CHUNKS)
                self.fused.append(cg.bind(b.dev, stream=stream))
        elif world > 1:
            for b in self.bounds:
                fg = edist.FusedGather(b.problem.name, rank, world, workdir)
                self.fused.append(fg.bind(b.dev, stream=stream))
        # bytes each rank sends to its peers per step (fused: the row stores
        # to the other ranks' outputs)
        self.peer_bytes = [sum(int(b.dev[o].numel()) * b.dev[o].element_size()
                               for o in b.problem.outputs) * (world - 1) for b in self.bounds]

    @property
    def kernels(self):
        return [f.kernel for f in self.fused] if self.fused else [b.kernel for b in self.bounds]

    def launch_marked(self, marks=None):
        """Queue one step; record ``marks[i]`` after kernel i and the last
        mark after the exchange."""
        import torch.distributed as dist
        launches = [f.launch for f in self.fused] if self.fused else \
            [b.launch for b in self.bounds]
        for i, launch in enumerate(launches):
            launch()
            if marks is not None:
                marks[i].record(self.stream)
        if self.fused:
            self.fused[-1].wait()        # every rank's kernels have finished
        for g, t in zip(self.gathered, self.outs):
            dist.all_gather_into_tensor(g, t)
        if marks is not None:
            marks[len(launches)].record(self.stream)

    def close(self):
        for f in self.fused:
            f.close()
        self.fused = []


def time_headline(hs, steps, warmup, barrier):
    """W warm-up steps, then K timed steps bracketed by barrier + sync; CUDA
    events on the launching stream.  Returns (step ms, per-kernel ms,
    gather ms)."""
    import torch
    stream = hs.stream
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            hs.launch_marked()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    nb = len(hs.bounds)
    start = _events(1)[0]
    marks = [_events(nb + 1) for _ in range(steps)]
    with torch.cuda.stream(stream):
        start.record(stream)
        for k in range(steps):
            hs.launch_marked(marks[k])
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    total = start.elapsed_time(marks[-1][-1])
    per = [0.0] * nb
    gather = 0.0
    prev = start
    for k in range(steps):
        for j in range(nb):
            per[j] += prev.elapsed_time(marks[k][j])
            prev = marks[k][j]
        gather += prev.elapsed_time(marks[k][nb])
        prev = marks[k][nb]
    return total / steps, [x / steps for x in per], gather / steps


def tf32_peak(device, n=8192, reps=10):
    """cuBLAS tf32 throughput (torch.matmul, allow_tf32) at n^3 on this GPU,
    best of ``reps`` after warm-up: the denominator for the tf32 tensor-core
    kernels.  2 n^3 flop per product."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        g = torch.Generator(device=device).manual_seed(0)
        a = torch.rand(n, n, device=device, generator=g)
        b = torch.rand(n, n, device=device, generator=g)
        for _ in range(3):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(reps):
            s, e = _events(2)
            s.record()
            torch.matmul(a, b)
            e.record()
            torch.cuda.synchronize()
            t = s.elapsed_time(e)
            best = t if best is None else min(best, t)
        del a, b
        return 2 * n ** 3 / best / 1e9
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def run_b200(args):
    import torch
    import torch.distributed as dist
    from emmy_ptx.runtime import init
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    init(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([float(x)], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    pk = peaks()
    stream = torch.cuda.Stream(device)
    workdir = tempfile.mkdtemp(prefix="emmy_bench_")
    hs = HeadlineStep(workdir, device, stream, rank, world, gather=GATHER_MODE)
    clocks = Clocks(local)
    clocks.start()
    step_ms, per_kernel, gather_ms = time_headline(hs, args.steps, args.warmup, barrier)
    clk = clocks.stop()
    bounds = hs.bounds
    launches = args.steps * len(bounds)
    step_ms = max_over_ranks(step_ms)
    value = hs.full_bytes / step_ms / 1e6

    # dominant kernel (largest share of the kernels' time): roofline.  One
    # GPU: HBM.  N>1: the gather kernels are bound by the bytes each rank
    # must send to its peers over NVLink.
    j = max(range(len(bounds)), key=lambda i: per_kernel[i])
    dom, dk = bounds[j], hs.kernels[j]
    if world == 1:
        achieved = dom.bytes / per_kernel[j] / 1e6
        roofline = {"kernel": dk.entry, "bound": "hbm", "achieved": round(achieved, 1),
                    "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "frac": round(achieved / pk["hbm_gbs"], 4),
                    "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs)"
                    if pk["source"] == "measured" else "fallback 6650 GB/s",
                    "algorithmic_bytes_per_launch": dom.bytes,
                    "ms_per_launch": round(per_kernel[j], 4)}
        roofline.update(_traffic(dk.entry, dom.bytes))
    else:
        nv = hs.peer_bytes[j]
        achieved = nv / max_over_ranks(per_kernel[j]) / 1e6
        roofline = {"kernel": dk.entry + (" (gather variant)" if GATHER_MODE == "fused" else
                                          " + copy-engine gather"), "bound": "nvlink",
                    "achieved": round(achieved, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                    "frac": round(achieved / NVLINK_GBS, 4),
                    "peak_source": "peer copy measured on this pool, per direction per GPU",
                    "peer_bytes_per_launch": nv,
                    "ms_per_launch": round(max_over_ranks(per_kernel[j]), 4), "traffic": None}
    kernels = {k.entry: {"ms": round(per_kernel[i], 4),
                         "gbs": round(b.bytes / per_kernel[i] / 1e6, 1),
                         "frac": round(b.bytes / per_kernel[i] / 1e6 / pk["hbm_gbs"], 4)}
               for i, (b, k) in enumerate(zip(bounds, hs.kernels))}
    hosts = [b.host for b in bounds] if world == 1 else None
    problems = [b.problem for b in bounds]
    sharded = None
    if world > 1:
        # the same step with the plain kernels and NCCL all_gather_into_tensor
        hs.close()
        del bounds, hs
        torch.cuda.empty_cache()
        hn = HeadlineStep(workdir, device, stream, rank, world, gather="nccl")
        n_ms, n_per, n_gather = time_headline(hn, max(3, args.steps // 2), 3, barrier)
        kernel_only = max_over_ranks(sum(n_per))
        full_bytes = hn.full_bytes
        del hn
        torch.cuda.empty_cache()
        other = "copy" if GATHER_MODE == "fused" else "fused"
        # the other exchange, timed beside the headline: every rank runs the
        # same code, so an error here is raised on every rank at the same
        # step and is reported, not fatal
        try:
            ho = HeadlineStep(workdir, device, stream, rank, world, gather=other)
            o_ms, _, _ = time_headline(ho, max(3, args.steps // 2), 3, barrier)
            ho.close()
            del ho
            other_ms = round(max_over_ranks(o_ms), 4)
        except Exception as exc:  # noqa: BLE001
            other_ms = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.empty_cache()
        sharded = {"config2": {
            f"{GATHER_MODE}_gather_incl_ms": round(step_ms, 4),
            f"{other}_gather_incl_ms": other_ms,
            "nccl_gather_incl_ms": round(max_over_ranks(n_ms), 4),
            "kernel_only_ms": round(kernel_only, 4),
            "kernel_only_gbs": round(full_bytes / kernel_only / 1e6, 1),
            "headline_exchange": GATHER_MODE,
            "partition": f"rows ({8192 // world} of 8192 per rank)"}}
    else:
        del bounds, hs
    torch.cuda.empty_cache()

    # end to end through the host-buffer API: each rank moves its own rows
    # 16 row blocks per rank: the copy-in of a block overlaps the copy-out of
    # the one before, and each block boundary costs a kernel and two event
    # hand-offs (measured per step on one B200, ms: 8 blocks 26.7, 16 26.8,
    # 32 28.0, 64 30.7, against 24.75 for the same copies with no kernels)
    chunks = 16
    barrier()
    # four warm-up steps: the first steps through fresh pinned buffers and an
    # idle host link ran up to 7% slower (28.5 against 26.7 ms per step)
    e2e = e2e_measure(HEADLINE, workdir, max(5, args.steps // 4), 4, rank,
                      chunks=chunks, rows_div=world, barrier=barrier)
    et = max_over_ranks(e2e["ms_per_step"])
    e2e_value = world * e2e["bytes"] / et / 1e6
    # the same copies with no kernels, all ranks at once: the step's ceiling
    link_ms, link_mine = link_probe(device, e2e["h2d"] // 4 * 4, e2e["d2h"] // 4 * 4,
                                    barrier, max_over_ranks, chunks=2 * chunks)
    link_total = world * (e2e["h2d"] + e2e["d2h"]) / link_ms / 1e6
    links = [round((e2e["h2d"] + e2e["d2h"]) / link_mine / 1e6, 1)]
    if world > 1:
        allv = [None] * world
        dist.all_gather_object(allv, links[0])
        links = allv
    pcie_total = world * (e2e["h2d"] + e2e["d2h"]) / et / 1e6

    if world > 1:
        from emmy_ptx import dist as edist
        # matmul 8192^3 in row blocks and causal attention 8x32x4096x128 in
        # (batch x head) pairs: NCCL all-gather vs the fused epilogue gather
        for name in ("matmul", "attention"):
            # every rank runs the same code, so an error raised here is raised
            # on every rank at the same step and is reported, not fatal
            try:
                sharded[name] = edist.bench_fused_gather(name, workdir, device, stream, rank,
                                                         world, steps=5, warmup=3)
            except Exception as exc:  # noqa: BLE001
                sharded[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            torch.cuda.empty_cache()

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded torch.Generator inputs of the config's shapes)",
        "config": config_block(world),
        "launch": "sm_100a PTX via libemmy_rt C ABI (cuLaunchKernelEx)",
        "kernels": kernels,
        "roofline": roofline,
        "clocks": clk,
        "gpu_launches": launches,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": e2e["h2d"] * world, "d2h_bytes_per_step": e2e["d2h"] * world,
                "ms_per_step": round(et, 3),
                "link_both_ways_gbs": round(link_total, 1),
                "link_ms_per_step": round(link_ms, 3),
                "link_per_rank_gbs": links,
                "link": f"the step's copies alone (no kernels), both directions at once, "
                        f"{2 * chunks} copies per direction as the pipeline makes them, "
                        f"all ranks together, max over ranks",
                "frac_of_link": round(pcie_total / link_total, 3),
                "path": f"emmy_ptx.pipeline.ChunkedHostRunner: pinned host -> ert_memcpy_htod "
                        f"-> launch -> ert_memcpy_dtoh, {e2e['chunks']} row blocks per rank "
                        f"over {e2e['slots']} device slots on three C-ABI streams"},
    }
    if world > 1:
        line["exchange_ms_per_step"] = round(max_over_ranks(gather_ms), 4)
    if sharded is not None:
        line["sharded"] = sharded
    if rank == 0 and world == 1:
        if not args.no_categories:
            line["categories"] = categories_sweep(workdir, device, stream, pk)
        line["cpu_baseline"] = cpu_baseline(problems, 5, 1, host_inputs=hosts)
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _traffic(entry, algorithmic_bytes):
    """DRAM bytes per launch of ``entry`` from the committed full-size ncu
    capture (profiles/traffic.json: ``dram__bytes_read.sum +
    dram__bytes_write.sum`` of a steady-state launch, with the previous
    launch's dirty L2 lines written back inside it), scaled to this launch's
    algorithmic bytes when the launch is a row shard (traffic of a row kernel
    grows in proportion to its rows)."""
    f = ROOT / "profiles" / "traffic.json"
    try:
        rec = json.loads(f.read_text())[entry]
        rec["dram_bytes_per_launch"], rec["algorithmic_bytes"], rec["summary"]
    except Exception:  # noqa: BLE001
        return {"traffic": None}
    t = rec["dram_bytes_per_launch"] * algorithmic_bytes / rec["algorithmic_bytes"]
    return {"traffic": int(t), "traffic_over_algorithmic": round(t / algorithmic_bytes, 4),
            "traffic_source": rec["summary"]}


def run_kernel_only(args):
    """Profiling mode: ``--launches`` launches of one category kernel of this
    backend at the size given by ``--size k=v ...`` (builder keywords)."""
    import torch
    from emmy_ptx import workloads
    from emmy_ptx.runtime import Kernel, init
    kw = {}
    for item in args.size:
        k, v = item.split("=")
        kw[k] = int(v)
    init(0)
    dev = torch.device("cuda", 0)
    p = workloads.build(args.kernel, **kw)
    ir = p.write(tempfile.mkdtemp(prefix="emmy_prof_"))
    kern = Kernel.from_ir(ir)
    bufs = {}
    g = torch.Generator(device=dev).manual_seed(p.seed)
    for name in p.inputs:
        t = p.tensor(name)
        if t["dtype"] == "s32":
            bufs[name] = torch.randint(1, 1000, t["shape"], device=dev, generator=g,
                                       dtype=torch.int32)
        else:
            bufs[name] = torch.randn(t["shape"], device=dev, generator=g,
                                     dtype=getattr(torch, DTYPES[t["dtype"]]))
    for name in p.outputs:
        t = p.tensor(name)
        bufs[name] = torch.empty(t["shape"], device=dev, dtype=getattr(torch, DTYPES[t["dtype"]]))
    launch = kern.bind(bufs)
    for _ in range(args.launches):
        launch()
    torch.cuda.synchronize()
    status = kern.status()
    print(json.dumps({"kernel": kern.entry, "size": kw, "launches": args.launches,
                      "status": status}))
    return 1 if status else 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default=None,
                    help="profiling mode: launch one category kernel (workload builder name)")
    ap.add_argument("--size", nargs="*", default=[], help="builder keywords, k=v")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-categories", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel:
        return run_kernel_only(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    raise SystemExit(main())
