"""Load and launch compiled Emmy kernels through libemmy_rt.so (C ABI).

This is the runner the reference leaves to an outside harness
(README.md:49-50, 91-92): it takes the PTX and the meta.json contract,
JIT-loads the module on the current device and launches the entry with its
pointer/scalar parameters in ``arg_order``.  Everything crosses the C ABI
declared in ``include/emmy_rt.h`` as plain integers and pointers; PyTorch
tensors are accepted only as a convenience (their ``data_ptr()``), so the
runtime also works with raw device pointers from any allocator.

There is no CPU fallback: if ``libemmy_rt.so`` is missing, or no GPU is
present, every call raises :class:`EmmyRuntimeError`.
"""

from __future__ import annotations

import ctypes
import json
import re
import threading
from pathlib import Path

import numpy as np

_LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = _LIB_DIR / "libemmy_rt.so"

_lock = threading.Lock()
_lib = None

# CUtensorMapDataType values (cuda.h)
TMAP_DTYPE = {"u8": 0, "u16": 1, "u32": 2, "s32": 3, "u64": 4, "s64": 5,
              "f16": 6, "f32": 7, "f64": 8, "bf16": 9, "f32_ftz": 10, "tf32": 11,
              "tf32_ftz": 12}
TMAP_SWIZZLE = {"none": 0, "32B": 1, "64B": 2, "128B": 3, "128B_atom32B": 4,
                "128B_atom32B_flip8B": 5, "128B_atom64B": 6}

_CTYPE = {"f32": ctypes.c_float, "f64": ctypes.c_double, "s32": ctypes.c_int32,
          "u32": ctypes.c_uint32, "s64": ctypes.c_int64}
NP_DTYPE = {"f32": np.float32, "f64": np.float64, "s32": np.int32, "u32": np.uint32,
            "s64": np.int64}


class EmmyRuntimeError(RuntimeError):
    pass


class ErtGeom(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_uint * 3), ("block", ctypes.c_uint * 3),
                ("cluster", ctypes.c_uint * 3), ("shared_bytes", ctypes.c_uint)]


_SIGS = {
    "ert_abi_version": ([], ctypes.c_int),
    "ert_device_count": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "ert_init": ([ctypes.c_int], ctypes.c_int),
    "ert_module_load": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64), ctypes.c_char_p,
                         ctypes.c_size_t], ctypes.c_int),
    "ert_module_unload": ([ctypes.c_uint64], ctypes.c_int),
    "ert_function": ([ctypes.c_uint64, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)],
                     ctypes.c_int),
    "ert_function_attrs": ([ctypes.c_uint64] + [ctypes.POINTER(ctypes.c_int)] * 4, ctypes.c_int),
    "ert_launch": ([ctypes.c_uint64, ctypes.POINTER(ErtGeom), ctypes.POINTER(ctypes.c_void_p),
                    ctypes.c_uint64], ctypes.c_int),
    "ert_module_global": ([ctypes.c_uint64, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64),
                           ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "ert_tensormap_encode": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                              ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                              ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                              ctypes.c_int, ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "ert_memcpy_htod": ([ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint64],
                        ctypes.c_int),
    "ert_memcpy_dtoh": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_uint64],
                        ctypes.c_int),
    "ert_memcpy_dtod": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_uint64],
                        ctypes.c_int),
    "ert_memset_d8": ([ctypes.c_uint64, ctypes.c_ubyte, ctypes.c_size_t, ctypes.c_uint64],
                      ctypes.c_int),
    "ert_stream_sync": ([ctypes.c_uint64], ctypes.c_int),
    "ert_stream_create": ([ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "ert_stream_destroy": ([ctypes.c_uint64], ctypes.c_int),
    "ert_stream_wait_event": ([ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "ert_mem_alloc": ([ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t], ctypes.c_int),
    "ert_mem_free": ([ctypes.c_uint64], ctypes.c_int),
    "ert_ipc_get_handle": ([ctypes.c_uint64, ctypes.c_void_p], ctypes.c_int),
    "ert_ipc_open": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "ert_ipc_close": ([ctypes.c_uint64], ctypes.c_int),
    "ert_host_alloc": ([ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t], ctypes.c_int),
    "ert_host_free": ([ctypes.c_void_p], ctypes.c_int),
    "ert_event_create": ([ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "ert_event_record": ([ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "ert_event_elapsed": ([ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_float)],
                          ctypes.c_int),
    "ert_event_sync": ([ctypes.c_uint64], ctypes.c_int),
    "ert_event_destroy": ([ctypes.c_uint64], ctypes.c_int),
    "ert_status": ([ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint64],
                   ctypes.c_int),
    "ert_last_error": ([], ctypes.c_char_p),
}

EXPORTED = tuple(_SIGS)


def lib():
    """The loaded libemmy_rt.so (raises if it was not built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise EmmyRuntimeError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python __graft_entry__.py` (build()) or `make -C emmy-ptx_b200/csrc`")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (argtypes, restype) in _SIGS.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = handle
        return _lib


def last_error() -> str:
    msg = lib().ert_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str):
    if rc != 0:
        raise EmmyRuntimeError(f"{what} failed ({rc}): {last_error()}")


def device_count() -> int:
    n = ctypes.c_int(0)
    check(lib().ert_device_count(ctypes.byref(n)), "ert_device_count")
    return n.value


IPC_HANDLE_BYTES = 64


def ipc_handle(dptr: int) -> bytes:
    """CUDA IPC handle of a buffer from ``ert_mem_alloc`` (``DeviceBuffer``)."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().ert_ipc_get_handle(int(dptr), buf), "ert_ipc_get_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    """Map another process's buffer into this one; returns its device pointer."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise EmmyRuntimeError(f"IPC handle of {len(handle)} bytes")
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    p = ctypes.c_uint64(0)
    check(lib().ert_ipc_open(buf, ctypes.byref(p)), "ert_ipc_open")
    return p.value


def ipc_close(dptr: int):
    check(lib().ert_ipc_close(int(dptr)), "ert_ipc_close")


_initialised = set()


def init(device: int = 0):
    """Make ``device``'s primary context current (shared with torch)."""
    check(lib().ert_init(int(device)), f"ert_init({device})")
    _initialised.add(int(device))


def _stream_handle(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    h = getattr(stream, "cuda_stream", None)
    if h is None:
        raise TypeError(f"not a stream: {stream!r}")
    return int(h)


_VEC_ACCESS = re.compile(r"\b(?:ld|st)\.global[.\w:]*?\.v(\d)\.[bfsu](\d+)\b")


def required_alignment(ptx: str) -> int:
    """The address alignment a module's global accesses need: the largest
    vector access (``ld/st.global...vN.<type>``), 16 bytes if it moves data
    with bulk copies (TMA, ``cp.async.bulk``), else 0.  A pointer argument
    off that alignment would fault the kernel, so ``Kernel.bind`` refuses
    it."""
    need = 0
    for n, bits in _VEC_ACCESS.findall(ptx):
        need = max(need, int(n) * int(bits) // 8)
    if "cp.async.bulk" in ptx:
        need = max(need, 16)
    return need


def _ptr(x) -> int:
    if isinstance(x, int):
        return x
    dp = getattr(x, "data_ptr", None)
    if dp is None:
        raise TypeError(f"not a device buffer: {type(x).__name__}")
    return int(dp())


class Stream:
    """A non-blocking CUDA stream owned through the C ABI
    (``ert_stream_create``), usable wherever a stream is accepted."""

    def __init__(self):
        h = ctypes.c_uint64(0)
        check(lib().ert_stream_create(ctypes.byref(h)), "ert_stream_create")
        self.handle = h.value

    @property
    def cuda_stream(self) -> int:
        return self.handle

    def wait(self, event: "Event"):
        """Later work on this stream waits for ``event``'s last record."""
        check(lib().ert_stream_wait_event(self.handle, event.handle), "ert_stream_wait_event")

    def synchronize(self):
        check(lib().ert_stream_sync(self.handle), "ert_stream_sync")

    def destroy(self):
        if self.handle:
            check(lib().ert_stream_destroy(self.handle), "ert_stream_destroy")
            self.handle = 0


class Event:
    """A CUDA event through the C ABI (timing and stream ordering)."""

    def __init__(self):
        h = ctypes.c_uint64(0)
        check(lib().ert_event_create(ctypes.byref(h)), "ert_event_create")
        self.handle = h.value
        self.recorded = False

    def record(self, stream=None):
        check(lib().ert_event_record(self.handle, _stream_handle(stream)), "ert_event_record")
        self.recorded = True

    def synchronize(self):
        check(lib().ert_event_sync(self.handle), "ert_event_sync")

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0)
        check(lib().ert_event_elapsed(self.handle, end.handle, ctypes.byref(ms)),
              "ert_event_elapsed")
        return ms.value

    def destroy(self):
        if self.handle:
            check(lib().ert_event_destroy(self.handle), "ert_event_destroy")
            self.handle = 0


class Module:
    """A JIT-loaded PTX module on the current device."""

    def __init__(self, ptx: str):
        self.handle = ctypes.c_uint64(0)
        log = ctypes.create_string_buffer(16384)
        rc = lib().ert_module_load(ptx.encode(), ctypes.byref(self.handle), log, len(log))
        if rc != 0:
            raise EmmyRuntimeError(f"module load failed ({rc}): {last_error()}")
        self._fns: dict = {}

    def function(self, entry: str) -> int:
        if entry not in self._fns:
            fn = ctypes.c_uint64(0)
            check(lib().ert_function(self.handle.value, entry.encode(), ctypes.byref(fn)),
                  f"ert_function({entry})")
            self._fns[entry] = fn.value
        return self._fns[entry]

    def attrs(self, entry: str) -> dict:
        vals = [ctypes.c_int(0) for _ in range(4)]
        check(lib().ert_function_attrs(self.function(entry), *[ctypes.byref(v) for v in vals]),
              "ert_function_attrs")
        return dict(zip(("num_regs", "max_threads", "static_shared", "local_bytes"),
                        (v.value for v in vals)))

    def global_ptr(self, name: str):
        p, n = ctypes.c_uint64(0), ctypes.c_size_t(0)
        check(lib().ert_module_global(self.handle.value, name.encode(), ctypes.byref(p),
                                      ctypes.byref(n)), f"ert_module_global({name})")
        return p.value, n.value

    def status(self, stream=None) -> int:
        code = ctypes.c_uint32(0)
        check(lib().ert_status(self.handle.value, ctypes.byref(code), _stream_handle(stream)),
              "ert_status")
        return code.value

    def unload(self):
        if self.handle.value:
            lib().ert_module_unload(self.handle.value)
            self.handle = ctypes.c_uint64(0)


def encode_tensormap(spec: dict, base_ptr: int) -> bytes:
    """cuTensorMapEncodeTiled for a sidecar tensor-map spec."""
    rank = len(spec["dims"])
    buf = (ctypes.c_uint8 * (128 + 64))()
    addr = ctypes.addressof(buf)
    aligned = (addr + 63) & ~63
    dims = (ctypes.c_uint64 * rank)(*spec["dims"])
    strides = (ctypes.c_uint64 * max(1, rank - 1))(*(spec["strides"] or [0]))
    box = (ctypes.c_uint32 * rank)(*spec["box"])
    estr = (ctypes.c_uint32 * rank)(*(spec.get("elem_strides") or [1] * rank))
    check(lib().ert_tensormap_encode(ctypes.c_void_p(aligned), TMAP_DTYPE[spec["dtype"]], rank,
                                     base_ptr + int(spec.get("offset_bytes", 0)), dims, strides,
                                     box, estr, TMAP_SWIZZLE[spec.get("swizzle", "none")],
                                     int(spec.get("l2_promotion", 2)),
                                     int(spec.get("oob_fill", 0))),
          "ert_tensormap_encode")
    return ctypes.string_at(aligned, 128)


class Kernel:
    """A compiled kernel ready to launch on the current device.

    ``args`` describes the parameters in arg_order:
    ``[{"name", "dtype", "shape", "scalar"}]``.  ``sidecar`` carries the
    launch needs of sm_100a kernels; kernels from other compilers (the
    reference's sm_89 PTX) launch with the meta.json geometry.
    """

    def __init__(self, ptx: str, entry: str, args: list, meta_geom: dict,
                 sidecar: dict | None = None, device: int | None = None):
        if device is not None or not _initialised:
            init(0 if device is None else device)
        self.ptx = ptx
        self.entry = entry
        self.args = args
        self.meta_geom = meta_geom
        self.sidecar = sidecar or {}
        self.module = Module(ptx)
        self.function = self.module.function(entry)
        self._check_register_split()
        self.alignment = required_alignment(ptx)
        self._tmap_cache: dict = {}
        self.launches = 0
        # scratch buffers the kernel needs beyond its arguments (sidecar
        # "scratch": [{"name", "bytes"}]); allocated on first bind, freed
        # with the kernel
        self.scratch: dict = {}

    def _check_register_split(self):
        """A kernel whose warpgroups re-divide their registers
        (``setmaxnreg``, sidecar ``register_split``) must have been given the
        launch register count the split assumes: ``setmaxnreg.inc`` beyond
        the block's registers waits forever.  Refuse it before any launch."""
        rs = self.sidecar.get("register_split")
        if not rs:
            return
        have = self.module.attrs(self.entry)["num_regs"]
        for threads, need in rs["registers_by_block"].items():
            if have < rs["launch"] or need > int(threads) * have:
                raise EmmyRuntimeError(
                    f"{self.entry}: {have} registers per thread at launch; its register "
                    f"split needs {rs['launch']} ({need} registers over {threads} threads)")

    # -- construction ----------------------------------------------------
    @staticmethod
    def _arg_specs(comp):
        specs = []
        for name in comp.arg_order:
            a = comp.args.get(name) or {"name": name, "dtype": comp.dtype_of(name),
                                        "shape": comp.shape_of(name)}
            specs.append({"name": name, "dtype": a.get("dtype", "f32"),
                          "shape": [int(s) for s in a.get("shape", [])],
                          "scalar": bool(a.get("scalar")) or len(a.get("shape", [])) == 0})
        return specs

    @classmethod
    def from_ir(cls, ir_path, *, target="sm_100a", ptx_version="8.8",
                int_semantics="reference", device=None):
        from .compiler import Compiler
        comp = Compiler(ir_path, target=target, ptx_version=ptx_version,
                        int_semantics=int_semantics)
        ptx = comp.compile()
        geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
        return cls(ptx, comp.entry, cls._arg_specs(comp), geom, comp.sidecar(), device)

    @classmethod
    def from_ptx(cls, ptx: str, ir_path, *, device=None):
        """A kernel from PTX another compiler made for the same package
        (launched with the meta.json geometry)."""
        from .compiler import Compiler
        comp = Compiler(ir_path, target="sm_100a", ptx_version="8.7")
        geom = {"grid": comp.kmeta.get("grid") or [1], "block": comp.kmeta.get("block") or [1]}
        return cls(ptx, comp.entry, cls._arg_specs(comp), geom, None, device)

    # -- launching ----------------------------------------------------------
    def geometry(self, which="tuned") -> ErtGeom:
        """``"tuned"``: the sidecar's grid; ``"meta"``: meta.json's grid.
        Block shape, dynamic shared memory and cluster shape are properties
        of the kernel and come from the sidecar either way."""
        use_side = which == "tuned" and bool(self.sidecar.get("grid"))
        src = self.sidecar if use_side else self.meta_geom

        def three(v):
            v = [v] if isinstance(v, int) else list(v or [1])
            return (v + [1, 1, 1])[:3]
        g = ErtGeom()
        g.grid[:] = three(src.get("grid"))
        g.block[:] = three(self.sidecar.get("block") or self.meta_geom.get("block"))
        g.cluster[:] = three(self.sidecar.get("cluster"))
        g.shared_bytes = int(self.sidecar.get("shared_bytes", 0))
        return g

    def _prepare_tensormaps(self, ptrs: dict, stream: int):
        maps = self.sidecar.get("tensormaps") or []
        if not maps:
            return
        key = tuple(ptrs.get(m["arg"]) for m in maps)
        if self._tmap_cache.get("key") == key:
            return
        for m in maps:
            desc = encode_tensormap(m, ptrs[m["arg"]])
            dptr, size = self.module.global_ptr(m["global"])
            if size < 128:
                raise EmmyRuntimeError(f"tensor map global {m['global']} is {size} bytes")
            staged = ctypes.create_string_buffer(desc, 128)
            check(lib().ert_memcpy_htod(dptr, staged, 128, stream), "ert_memcpy_htod(tensormap)")
            check(lib().ert_stream_sync(stream), "ert_stream_sync")
        self._tmap_cache["key"] = key

    def _scratch_ptrs(self) -> dict:
        """``{"@name": device pointer}`` for the sidecar's scratch buffers."""
        for sc in self.sidecar.get("scratch") or []:
            if sc["name"] not in self.scratch:
                self.scratch[sc["name"]] = DeviceBuffer(int(sc["bytes"]))
        return {"@" + k: b.ptr for k, b in self.scratch.items()}

    def bind(self, buffers: dict, *, stream=None, geometry="tuned"):
        """Resolve ``buffers`` (every argument name -> device pointer, or a
        scalar value) once; the returned launch object re-launches with no
        per-call argument marshalling.  Auxiliary launches the sidecar lists
        under ``prelaunch`` (e.g. a pre-pass over an input into scratch
        memory) run first, and those under ``postlaunch`` (e.g. the sum of a
        split-K kernel's partial tiles) after it, on the same stream."""
        s = _stream_handle(stream)
        values = []
        ptrs = {}
        for a in self.args:
            if a["name"] not in buffers:
                raise EmmyRuntimeError(f"missing argument {a['name']!r}")
            v = buffers[a["name"]]
            if a["scalar"]:
                values.append(_CTYPE.get(a["dtype"], ctypes.c_int32)(v))
            else:
                self._validate(a, v)
                p = _ptr(v)
                if self.alignment and p % self.alignment:
                    raise EmmyRuntimeError(
                        f"argument {a['name']!r}: address {p:#x} is not {self.alignment}-byte "
                        f"aligned, as {self.entry}'s vector accesses need")
                ptrs[a["name"]] = p
                values.append(ctypes.c_uint64(p))
        ptrs.update(self._scratch_ptrs())
        self._prepare_tensormaps(ptrs, s)
        main = BoundLaunch(self, values, self.geometry(geometry), s, tmap_ptrs=ptrs)
        def aux_launches(key):
            out = []
            for aux in self.sidecar.get(key) or []:
                fn = self.module.function(aux["entry"])
                vals = [ctypes.c_uint64(ptrs[a]) for a in aux["args"]]
                g = ErtGeom()
                g.grid[:] = (list(aux["grid"]) + [1, 1, 1])[:3]
                g.block[:] = (list(aux["block"]) + [1, 1, 1])[:3]
                g.cluster[:] = (1, 1, 1)
                g.shared_bytes = int(aux.get("shared_bytes", 0))
                out.append(BoundLaunch(self, vals, g, s, function=fn))
            return out
        # prelaunch entries (pre-passes) before the kernel, postlaunch
        # entries (the split-K reduction) after it, all on the same stream
        pre, post = aux_launches("prelaunch"), aux_launches("postlaunch")
        return main if not (pre or post) else LaunchSequence(pre + [main] + post)

    def launch(self, buffers: dict, *, stream=None, geometry="tuned"):
        """Launch with ``buffers`` mapping every argument name to a device
        pointer (int or object with ``data_ptr()``) or a scalar value."""
        self.bind(buffers, stream=stream, geometry=geometry)()

    def status(self, stream=None) -> int:
        return self.module.status(stream)

    def set_global(self, name: str, data: bytes, stream=None):
        """Copy ``data`` into the module-scope variable ``name`` (stream-ordered;
        the host buffer is staged before this returns)."""
        dptr, size = self.module.global_ptr(name)
        if len(data) > size:
            raise EmmyRuntimeError(f"{len(data)} bytes for module global {name} of {size}")
        staged = ctypes.create_string_buffer(bytes(data), len(data))
        check(lib().ert_memcpy_htod(dptr, staged, len(data), _stream_handle(stream)),
              "ert_memcpy_htod(global)")
        check(lib().ert_stream_sync(_stream_handle(stream)), "ert_stream_sync")

    def free_scratch(self):
        for buf in self.scratch.values():
            buf.free()
        self.scratch = {}

    @staticmethod
    def _validate(a, v):
        shape = getattr(v, "shape", None)
        if shape is not None and hasattr(v, "is_contiguous"):
            n = 1
            for s in a["shape"]:
                n *= s
            if v.numel() != n:
                raise EmmyRuntimeError(f"argument {a['name']!r}: {v.numel()} elements, "
                                       f"meta.json says {n}")
            if not v.is_contiguous():
                raise EmmyRuntimeError(f"argument {a['name']!r} must be contiguous")
            if getattr(v, "is_cuda", True) is False:
                raise EmmyRuntimeError(f"argument {a['name']!r} is not on the GPU")


class BoundLaunch:
    """A kernel launch with its arguments marshalled (see Kernel.bind)."""

    def __init__(self, kernel: Kernel, values: list, geom: ErtGeom, stream: int,
                 function: int | None = None, tmap_ptrs: dict | None = None):
        self.kernel = kernel
        self.values = values          # keeps the ctypes values alive
        self.argv = (ctypes.c_void_p * len(values))(
            *[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in values])
        self.geom = geom
        self.stream = stream
        self._launch = lib().ert_launch
        self._fn = kernel.function if function is None else function
        # the tensor maps live in the module's globals, shared by every bind
        # of the kernel: a launch whose buffers differ from the last bind's
        # writes its own maps again first (stream-ordered, so earlier
        # launches still read theirs)
        maps = kernel.sidecar.get("tensormaps") or []
        self._tmap_ptrs = tmap_ptrs if maps and tmap_ptrs is not None else None
        self._tmap_key = (tuple(tmap_ptrs.get(m["arg"]) for m in maps)
                          if self._tmap_ptrs is not None else None)

    def __call__(self):
        if self._tmap_ptrs is not None and \
                self.kernel._tmap_cache.get("key") != self._tmap_key:
            self.kernel._prepare_tensormaps(self._tmap_ptrs, self.stream)
        rc = self._launch(self._fn, ctypes.byref(self.geom), self.argv, self.stream)
        if rc != 0:
            check(rc, f"launch of {self.kernel.entry}")
        self.kernel.launches += 1


class LaunchSequence:
    """Several bound launches issued in order on one stream."""

    def __init__(self, launches: list):
        self.launches = launches

    def __call__(self):
        for launch in self.launches:
            launch()


# ----------------------------------------------------------------------------
# host-buffer path (the C-ABI call a non-torch caller makes)
# ----------------------------------------------------------------------------
class PinnedArray:
    """A numpy array in page-locked host memory (ert_host_alloc)."""

    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape)) * self.dtype.itemsize
        self.ptr = ctypes.c_void_p(0)
        check(lib().ert_host_alloc(ctypes.byref(self.ptr), max(1, self.nbytes)), "ert_host_alloc")
        raw = (ctypes.c_uint8 * max(1, self.nbytes)).from_address(self.ptr.value)
        self.array = np.frombuffer(raw, dtype=self.dtype, count=int(np.prod(self.shape))) \
            .reshape(self.shape)

    def free(self):
        if self.ptr.value:
            lib().ert_host_free(self.ptr)
            self.ptr = ctypes.c_void_p(0)


class DeviceBuffer:
    """Device memory from ert_mem_alloc (no torch involved)."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        p = ctypes.c_uint64(0)
        check(lib().ert_mem_alloc(ctypes.byref(p), max(1, self.nbytes)), "ert_mem_alloc")
        self.ptr = p.value

    def data_ptr(self):
        return self.ptr

    def free(self):
        if self.ptr:
            lib().ert_mem_free(self.ptr)
            self.ptr = 0


class HostRunner:
    """Runs a Kernel on host arrays: host->device copies of the inputs, the
    launch, device->host copies of the outputs, all on one stream."""

    def __init__(self, kernel: Kernel, outputs: list, stream=None):
        self.kernel = kernel
        self.outputs = list(outputs)
        self.stream = _stream_handle(stream)
        self.dev = {}
        for a in kernel.args:
            if not a["scalar"]:
                n = int(np.prod(a["shape"])) * np.dtype(NP_DTYPE[a["dtype"]]).itemsize
                self.dev[a["name"]] = DeviceBuffer(n)

    def run(self, host: dict, out: dict | None = None, sync=True) -> dict:
        out = out or {}
        h2d = d2h = 0
        for a in self.kernel.args:
            name = a["name"]
            if a["scalar"] or name in self.outputs:
                continue
            arr = host[name]
            src = arr.array if isinstance(arr, PinnedArray) else np.ascontiguousarray(arr)
            check(lib().ert_memcpy_htod(self.dev[name].ptr, src.ctypes.data, src.nbytes,
                                        self.stream), "ert_memcpy_htod")
            h2d += src.nbytes
        bufs = {a["name"]: (host[a["name"]] if a["scalar"] else self.dev[a["name"]].ptr)
                for a in self.kernel.args}
        self.kernel.launch(bufs, stream=self.stream)
        results = {}
        for name in self.outputs:
            a = next(x for x in self.kernel.args if x["name"] == name)
            dst = out.get(name)
            if dst is None:
                dst = np.empty(a["shape"], NP_DTYPE[a["dtype"]])
            arr = dst.array if isinstance(dst, PinnedArray) else dst
            check(lib().ert_memcpy_dtoh(arr.ctypes.data, self.dev[name].ptr, arr.nbytes,
                                        self.stream), "ert_memcpy_dtoh")
            d2h += arr.nbytes
            results[name] = arr
        if sync:
            check(lib().ert_stream_sync(self.stream), "ert_stream_sync")
        self.last_bytes = (h2d, d2h)
        return results

    def free(self):
        for b in self.dev.values():
            b.free()
        self.dev = {}


def load_sidecar(path) -> dict:
    return json.loads(Path(path).read_text())


__all__ = ["Kernel", "Module", "Stream", "Event", "HostRunner", "PinnedArray", "DeviceBuffer", "LaunchSequence", "init",
           "ipc_handle", "ipc_open", "ipc_close",
           "device_count", "EmmyRuntimeError", "LIB_PATH", "EXPORTED"]
