"""libemmy_rt.so: loads without a GPU and exports every include/emmy_rt.h symbol."""

import ctypes
import re
from pathlib import Path

import pytest

from emmy_ptx import runtime as rt

HEADER = Path(__file__).resolve().parent.parent / "include" / "emmy_rt.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(ert_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = declared()
    assert "ert_launch" in names and "ert_module_load" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(rt.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert set(declared()) <= set(rt.EXPORTED)


def test_abi_version():
    assert rt.lib().ert_abi_version() == 2


def test_streams_and_events_are_on_the_abi():
    """A C caller can run the host-buffer pipeline (copies and launches on
    streams of its own, ordered by events) without another CUDA runtime."""
    names = declared()
    for n in ("ert_stream_create", "ert_stream_destroy", "ert_stream_wait_event",
              "ert_event_create", "ert_event_record", "ert_event_sync", "ert_event_destroy"):
        assert n in names, n


def test_no_driver_is_an_error_not_a_crash():
    if rt.device_count() > 0:
        pytest.skip("a GPU is present")
    rc = rt.lib().ert_init(0)
    assert rc != 0
    assert rt.last_error()


def test_runtime_refuses_to_run_without_a_device():
    if rt.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(rt.EmmyRuntimeError):
        rt.init(0)


def test_required_alignment_follows_the_widest_vector_access():
    """Kernel.bind refuses a pointer off the alignment the module's widest
    global vector access (or a bulk copy) needs, instead of launching a
    kernel that would fault on it."""
    assert rt.required_alignment("ld.global.f32 %f1, [%rd1];") == 0
    assert rt.required_alignment("ld.global.nc.v4.f32 {%f1,%f2,%f3,%f4}, [%rd1];") == 16
    assert rt.required_alignment("ld.global.nc.v2.f64 {%fd1,%fd2}, [%rd1];") == 16
    assert rt.required_alignment(
        "ld.global.nc.L1::no_allocate.v8.f32 {%f1}, [%rd1];\nst.global.v4.f32 [%rd2], {%f1};") == 32
    assert rt.required_alignment("st.global.v8.b32 [%rd1], {%r1};") == 32
    assert rt.required_alignment(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%r1], [%rd1], 16, [%r2];"
    ) == 16


def test_register_split_is_checked_against_the_loaded_function():
    """A kernel whose warpgroups re-divide registers (setmaxnreg) is refused
    when the loaded function has fewer registers per thread than the split
    assumes -- setmaxnreg.inc would wait forever -- and accepted otherwise."""
    class FakeModule:
        def __init__(self, regs):
            self.regs = regs

        def attrs(self, entry):
            return {"num_regs": self.regs}

    side = {"register_split": {"launch": 168, "registers_by_block": {
        "384": 128 * (224 + 96) + 128 * 168, "256": 128 * (224 + 96)}}}
    k = rt.Kernel.__new__(rt.Kernel)
    k.entry, k.sidecar = "k_attention_causal", side
    k.module = FakeModule(168)
    k._check_register_split()                   # fits
    k.module = FakeModule(160)
    with pytest.raises(rt.EmmyRuntimeError, match="registers"):
        k._check_register_split()
    k.sidecar = {}
    k._check_register_split()                   # nothing to check
