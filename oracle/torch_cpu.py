"""torch-CPU evaluation of the BASELINE configurations' computations.

TEST INFRASTRUCTURE AND CPU BASELINE ONLY.  Only tests/, __graft_entry__ and
bench.py's CPU-baseline leg (and its ``--impl reference`` arm) may import
this module; the product never does.

The reference compiler runs no kernels itself: it writes PTX and leaves
launching to an outside runner (reference README.md:49-50).  So the CPU
anchor for its hot path is the computation its IR states, evaluated with
torch's own multi-threaded CPU operators over the whole configuration --
what a user without a GPU would run.  Semantics follow the reference's
lowering where it differs from torch:

* ``pointwise_i32``: the reference lowers int32 ``floor_divide`` and
  ``remainder`` to truncating ``div.s32`` / ``rem.s32``
  (compiler.py:1383-1385), so this uses ``rounding_mode="trunc"`` and
  ``torch.fmod``; the shifts are ``shl.b32`` / ``shr.s32`` (1374-1404).
* ``rmsnorm``: ``x * rsqrt(mean(x^2) + eps) * w`` (rsqrt at 1297-1301).
* ``softmax``: max-subtracted ``exp`` / sum (1121-1127), ``torch.softmax``.
* ``colreduce_f64``: column sum and max (the segmented tree, 1933-2012).
* ``rowsum_i32``: exact integer row sums.
* ``matmul``: ``A @ B`` in f32.
* ``attention``: causal scaled-dot-product attention, one chunk of heads
  at a time.
"""

from __future__ import annotations

import os
import statistics
import time


def threads() -> int:
    """All host cores this process may run on."""
    return len(os.sched_getaffinity(0))


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def pointwise_f32(x, y):
    import torch
    return {"out": x * torch.sigmoid(x) + y}


def pointwise_i32(a, b):
    import torch
    return {"q": torch.div(a, b, rounding_mode="trunc"), "r": torch.fmod(a, b),
            "s": torch.bitwise_right_shift(torch.bitwise_left_shift(a, 3), 1)}


def rmsnorm(x, w, eps=1e-6):
    import torch
    return {"out": x * torch.rsqrt(x.square().mean(1, keepdim=True) + eps) * w}


def softmax(x):
    import torch
    return {"out": torch.softmax(x, dim=1)}


def colreduce_f64(x):
    return {"colsum": x.sum(0), "colmax": x.amax(0)}


def rowsum_i32(x):
    import torch
    return {"out": x.sum(1, dtype=torch.int32)}


def matmul(A, B):
    return {"C": A @ B}


def attention(q, k, v, heads_per_chunk=8):
    import torch
    import torch.nn.functional as F
    out = torch.empty_like(q)
    qf, kf, vf, of = (t.reshape(-1, *t.shape[-2:]) for t in (q, k, v, out))
    for h0 in range(0, qf.shape[0], heads_per_chunk):
        sl = slice(h0, h0 + heads_per_chunk)
        of[sl] = F.scaled_dot_product_attention(qf[sl], kf[sl], vf[sl], is_causal=True)
    return {"out": out}


FUNCS = {"pointwise_f32": pointwise_f32, "pointwise_i32": pointwise_i32, "rmsnorm": rmsnorm,
         "softmax": softmax, "colreduce_f64": colreduce_f64, "rowsum_i32": rowsum_i32,
         "matmul": matmul, "attention": attention}


def run(category, inputs: dict, params: dict | None = None) -> dict:
    """Evaluate one configuration on torch CPU tensors ``inputs`` (named as
    the IR package's inputs)."""
    f = FUNCS[category]
    if category == "rmsnorm":
        return f(inputs["x"], inputs["w"], (params or {}).get("eps", 1e-6))
    return f(**inputs)


def time_problems(problems, steps, warmup, nthreads=None, inputs=None):
    """Median seconds per step of evaluating every problem of ``problems``
    (workload Problems) once, on ``nthreads`` torch threads (all cores by
    default), after ``warmup`` untimed steps.  Returns (seconds per step,
    per-step times, threads used)."""
    import torch
    n = nthreads or threads()
    torch.set_num_threads(n)
    if inputs is None:
        inputs = [{k: torch.from_numpy(v) for k, v in p.make_inputs().items()} for p in problems]
    for _ in range(warmup):
        for p, x in zip(problems, inputs):
            run(p.category, x, p.params)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for p, x in zip(problems, inputs):
            run(p.category, x, p.params)
        times.append(time.perf_counter() - t0)
    return statistics.median(times), times, n
