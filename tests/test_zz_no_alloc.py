"""ert_attention_noalloc (libemmy_noalloc.so): the attention launch whose
K-split scratch is a fixed device array, checked against the regular
(allocating) path.

The file name sorts last so that pytest collects it after every other test;
the GPU case must also pass alone in a fresh process.
"""

import ctypes
import re
import tempfile
from pathlib import Path

import numpy as np
import pytest

from emmy_ptx import workloads
from emmy_ptx import runtime as rt

HEADER = Path(__file__).resolve().parent.parent / "include" / "emmy_noalloc.h"
LIB_PATH = rt.LIB_PATH.parent / "libemmy_noalloc.so"
ERT_E_TOO_LARGE = -5


def _lib():
    rt.lib()                      # libemmy_rt first: the no-alloc library links to it
    lib = ctypes.CDLL(str(LIB_PATH))
    f = lib.ert_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                  ctypes.POINTER(rt.ErtGeom), ctypes.POINTER(ctypes.c_void_p),
                  ctypes.c_uint64, ctypes.c_uint64,
                  ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                  ctypes.c_uint64, ctypes.c_char_p, ctypes.c_size_t]
    return lib


def _scratch_limit():
    m = re.search(r"#define ERT_NOALLOC_SCRATCH_BYTES \((\d+)ull << (\d+)\)", HEADER.read_text())
    return int(m.group(1)) << int(m.group(2))


def test_library_exports_the_declared_entry():
    declared = re.findall(r"^int\s+(ert_\w+)\s*\(", HEADER.read_text(), re.M)
    assert declared == ["ert_attention_noalloc"]
    lib = _lib()
    assert all(hasattr(lib, n) for n in declared)


def test_oversized_request_is_rejected_before_any_device_work():
    """The full-size problem (8 x 32 heads x 4096 x 128) needs 1 GiB of
    pre-pass scratch (K's tf32 lo part and the rounded V); the call refuses
    it with ERT_E_TOO_LARGE and a message, before it touches a device (so
    this runs without a GPU)."""
    lib = _lib()
    g = rt.ErtGeom()
    argv = (ctypes.c_void_p * 1)(None)
    err = ctypes.create_string_buffer(512)
    rc = lib.ert_attention_noalloc(1, 1, 1, ctypes.byref(g), argv, 1, 1,
                                   8 * 32, 4096, 128, 0, err, len(err))
    assert rc == ERT_E_TOO_LARGE
    msg = err.value.decode()
    assert "scratch" in msg and str(_scratch_limit()) in msg


def test_bad_head_dim_is_an_argument_error():
    lib = _lib()
    g = rt.ErtGeom()
    argv = (ctypes.c_void_p * 1)(None)
    err = ctypes.create_string_buffer(256)
    rc = lib.ert_attention_noalloc(1, 1, 1, ctypes.byref(g), argv, 1, 1, 4, 64, 48, 0,
                                   err, len(err))
    assert rc == -2 and "head_dim" in err.value.decode()


@pytest.mark.gpu
def test_noalloc_matches_the_allocating_path(cuda):
    import torch
    from tolerances import check_close

    p = workloads.attention(batch=2, heads=4, seq=320, head_dim=128)
    ir = p.write(tempfile.mkdtemp(prefix="emmy_noalloc_"))
    inputs = p.make_inputs()
    dev = {n: torch.from_numpy(v).to(cuda) for n, v in inputs.items()}
    shape = p.tensor("out")["shape"]

    # the regular entry point: scratch allocated by the runtime on first bind
    regular = rt.Kernel.from_ir(ir)
    out_ref = torch.full(shape, float("nan"), device=cuda)
    regular.launch({**dev, "out": out_ref})
    torch.cuda.synchronize()
    assert regular.status() == 0
    want = out_ref.cpu().numpy()

    # the no-alloc entry point, on its own module (it rewrites the module's
    # tensor-map globals)
    k = rt.Kernel.from_ir(ir)
    lib = _lib()
    out = torch.full(shape, float("nan"), device=cuda)
    bufs = {**dev, "out": out}
    vals = [ctypes.c_uint64(bufs[a["name"]].data_ptr()) for a in k.args]
    argv = (ctypes.c_void_p * len(vals))(*[ctypes.addressof(v) for v in vals])
    geom = k.geometry("tuned")
    ksplit = k.module.function(k.entry + "_ksplit")
    bh, seq, dim = 2 * 4, 320, 128
    stream = torch.cuda.current_stream().cuda_stream
    err = ctypes.create_string_buffer(512)
    free_after = []
    for call in range(2):
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = lib.ert_attention_noalloc(k.module.handle.value, k.function, ksplit,
                                       ctypes.byref(geom), argv,
                                       dev["k"].data_ptr(), dev["v"].data_ptr(),
                                       bh, seq, dim, stream, err, len(err))
        assert rc == 0, err.value.decode()
        torch.cuda.synchronize()
        free_after.append((free_before, torch.cuda.mem_get_info()[0]))
        assert k.status() == 0
        got = out.cpu().numpy()
        assert not np.isnan(got).any()
        ok, msg = check_close("attention", f"out (call {call + 1})", got, want, inputs)
        assert ok, msg
    assert not k.scratch, "the no-alloc path allocated runtime scratch"
    # the device's free memory does not move across the second call (the
    # first may load the library's device image, array included)
    assert free_after[1][0] == free_after[1][1], free_after


@pytest.mark.gpu
def test_shape_other_than_the_compiled_one_is_refused(cuda):
    """The pre-pass writes the element count compiled into the module, so a
    smaller stated shape would pass the size check and then write past the
    array.  The call refuses any shape but the compiled one, before it writes
    a tensor map or launches (the output stays untouched)."""
    import torch

    p = workloads.attention(batch=1, heads=2, seq=256, head_dim=64)
    ir = p.write(tempfile.mkdtemp(prefix="emmy_noalloc_shape_"))
    k = rt.Kernel.from_ir(ir)
    lib = _lib()
    shape = p.tensor("out")["shape"]
    inputs = {n: torch.from_numpy(v).to(cuda) for n, v in p.make_inputs().items()}
    out = torch.full(shape, 3.0, device=cuda)
    bufs = {**inputs, "out": out}
    vals = [ctypes.c_uint64(bufs[a["name"]].data_ptr()) for a in k.args]
    argv = (ctypes.c_void_p * len(vals))(*[ctypes.addressof(v) for v in vals])
    geom = k.geometry("tuned")
    ksplit = k.module.function(k.entry + "_ksplit")
    err = ctypes.create_string_buffer(512)
    for bh, seq, dim in [(2, 128, 64), (1, 256, 64), (2, 256, 32), (4, 256, 64)]:
        rc = lib.ert_attention_noalloc(k.module.handle.value, k.function, ksplit,
                                       ctypes.byref(geom), argv,
                                       inputs["k"].data_ptr(), inputs["v"].data_ptr(),
                                       bh, seq, dim, 0, err, len(err))
        assert rc == -2, (bh, seq, dim, rc)
        assert "not compiled for" in err.value.decode()
    torch.cuda.synchronize()
    assert bool((out == 3.0).all()), "a refused call launched the kernel"
