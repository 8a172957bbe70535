"""Parity tolerances, one rule per category (stated here, used everywhere).

Integer, predicate and index outputs: bit-exact.
f32 pointwise:   |a - b| <= 1e-5 * max(|b|, 1)
f32 RMSNorm:     |a - b| <= 1e-5 * max(|b|, 1e-3)
f32 softmax:     |a - b| <= 1e-5 * max(|b|, 1/cols)
f64 col sum:     |a - b| <= 1e-12 * sum_i |x_i| (per column); col max exact
f64 row sum:     |a - b| <= 1e-12 * sum_j |x_j| (per row)
bit ops:         bitcast, pad: bit-exact; pow: |a - b| <= 1e-5 * max(|b|, 1)
f32 matmul (3xTF32 on tcgen05), and bf16/f16 matmul into f32:
                 |a - b| <= 1e-3 * (|b| + ||A_i|| * ||B_j|| / sqrt(K))
f32 attention:   |a - b| <= 1e-3 * (|b| + max_j |v_j| / sqrt(keys attended))
"""

import math

import numpy as np


def as_float(x):
    """Float64 values of an input (bf16 inputs travel as uint16 bits)."""
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return x.astype(np.float64)


def _bad(a, b, tol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = np.abs(a - b)
    ok = (err <= tol) | (np.isnan(a) & np.isnan(b)) | (a == b)
    return ok, err


def check_close(category, name, got, want, inputs=None, causal=True):
    """Returns (ok, message)."""
    got = np.asarray(got)
    want = np.asarray(want)
    if got.shape != want.shape:
        return False, f"{name}: shape {got.shape} != {want.shape}"
    if want.dtype.kind in "iub":
        bad = got != want
        if bad.any():
            idx = np.argwhere(bad)[0]
            return False, (f"{name}: {int(bad.sum())} of {bad.size} integers differ; first at "
                           f"{tuple(idx)}: got {got[tuple(idx)]}, want {want[tuple(idx)]}")
        return True, ""
    b = np.abs(want.astype(np.float64))
    if category in ("pointwise_f32", "pointwise"):
        tol = 1e-5 * np.maximum(b, 1.0)
    elif category == "rmsnorm":
        tol = 1e-5 * np.maximum(b, 1e-3)
    elif category == "softmax":
        tol = 1e-5 * np.maximum(b, 1.0 / want.shape[-1])
    elif category == "colreduce_f64":
        if name == "colmax":
            tol = np.zeros_like(b)
        else:
            tol = 1e-12 * np.abs(inputs["x"]).sum(0)
    elif category == "rowsum_f64":
        tol = 1e-12 * np.abs(inputs["x"]).sum(1)
    elif category == "bit_ops":
        tol = 1e-5 * np.maximum(b, 1.0) if name == "o_pow" else np.zeros_like(b)
    elif category in ("matmul", "matmul_lowp"):
        A, B = (as_float(inputs[n]) for n in ("A", "B"))
        na = np.linalg.norm(A, axis=1)[:, None]
        nb = np.linalg.norm(B, axis=0)[None, :]
        tol = 1e-3 * (b + na * nb / np.sqrt(A.shape[1]))
    elif category == "attention":
        v = np.abs(inputs["v"]).max(axis=-1).max(axis=-1)[..., None, None]
        seq = want.shape[-2]
        keys = np.arange(1, seq + 1, dtype=np.float64)[:, None] if causal \
            else np.full((seq, 1), float(seq))
        tol = 1e-3 * (b + v / np.sqrt(keys))
    else:
        tol = 1e-5 * np.maximum(b, 1.0)
    ok, err = _bad(got, want, tol)
    if not ok.all():
        idx = tuple(np.argwhere(~ok)[0])
        return False, (f"{name}: {int((~ok).sum())} of {ok.size} values out of tolerance; "
                       f"first at {idx}: got {got[idx]!r}, want {want[idx]!r}, "
                       f"max err {float(err.max()):.3g}")
    return True, ""


def assert_close(category, name, got, want, inputs=None):
    ok, msg = check_close(category, name, got, want, inputs)
    assert ok, msg


def check_close_device(category, name, got, want, inputs=None, causal=True, rows_per_chunk=None):
    """The rules above on device tensors (torch, float64 arithmetic), in row
    chunks so full-size outputs need no host copy and bounded scratch.
    ``inputs`` holds device tensors.  Returns (ok, message)."""
    import torch
    if tuple(got.shape) != tuple(want.shape):
        return False, f"{name}: shape {tuple(got.shape)} != {tuple(want.shape)}"
    if not want.dtype.is_floating_point:
        bad = got != want
        nbad = int(bad.sum())
        if nbad:
            idx = tuple(int(i) for i in torch.nonzero(bad)[0])
            return False, (f"{name}: {nbad} of {bad.numel()} integers differ; first at {idx}: "
                           f"got {int(got[idx])}, want {int(want[idx])}")
        return True, ""
    # per-category tolerance parts that do not depend on the chunk
    lead = want.shape[:-1]
    if category == "matmul":
        A, B = inputs["A"].double(), inputs["B"].double()
        na = torch.linalg.vector_norm(A, dim=1)[:, None]
        nb = torch.linalg.vector_norm(B, dim=0)[None, :]
        cross = na * nb / math.sqrt(A.shape[1])
    elif category == "attention":
        seq = want.shape[-2]
        vmax = inputs["v"].abs().amax(dim=(-1, -2)).double()          # [B, H]
        keys = (torch.arange(1, seq + 1, device=want.device, dtype=torch.float64) if causal
                else torch.full((seq,), float(seq), device=want.device, dtype=torch.float64))
        cross = (vmax[..., None] / keys.sqrt())[..., None]            # [B, H, S, 1]
    elif category == "colreduce_f64" and name != "colmax":
        cross = 1e-12 * inputs["x"].abs().sum(0)
    g2 = got.reshape(-1, want.shape[-1])
    w2 = want.reshape(-1, want.shape[-1])
    rows = g2.shape[0]
    step = rows_per_chunk or max(1, (1 << 25) // want.shape[-1])
    worst, nbad, first = 0.0, 0, None
    for r0 in range(0, rows, step):
        a = g2[r0:r0 + step].double()
        b = w2[r0:r0 + step].double()
        ab = b.abs()
        if category in ("pointwise_f32", "pointwise"):
            tol = 1e-5 * ab.clamp(min=1.0)
        elif category == "rmsnorm":
            tol = 1e-5 * ab.clamp(min=1e-3)
        elif category == "softmax":
            tol = 1e-5 * ab.clamp(min=1.0 / want.shape[-1])
        elif category == "colreduce_f64":
            tol = torch.zeros_like(ab) if name == "colmax" else cross.reshape(1, -1)
        elif category == "matmul":
            tol = 1e-3 * (ab + cross[r0:r0 + step])
        elif category == "attention":
            tol = 1e-3 * (ab + cross.reshape(-1, 1)[r0:r0 + step])
        else:
            tol = 1e-5 * ab.clamp(min=1.0)
        err = (a - b).abs()
        ok = (err <= tol) | (torch.isnan(a) & torch.isnan(b)) | (a == b)
        n = int((~ok).sum())
        if n and first is None:
            i = torch.nonzero(~ok)[0]
            first = (r0 + int(i[0]), int(i[1]), float(a[i[0], i[1]]), float(b[i[0], i[1]]))
        nbad += n
        e = err[~torch.isnan(err)]
        if e.numel():
            worst = max(worst, float(e.max()))
    if nbad:
        r, c, ga, wb = first
        return False, (f"{name}: {nbad} of {want.numel()} values out of tolerance; first at "
                       f"row {r} col {c}: got {ga!r}, want {wb!r}, max err {worst:.3g}")
    return True, f"{name}: max err {worst:.3g}"
