"""Emmy Kernel IR -> PTX, B200-native backend (drop-in for emmy-ptx).

Public surface kept from the reference (emmy_ptx/compiler.py:56-67, 211-250,
2159-2245; __init__.py:3-19): ``Compiler(ir_path, *, target, ptx_version)``
with ``.compile() -> str`` and ``.check() -> list[str]``,
``compile_file(path, *, target, ptx_version, cache_dir)``, ``ptx_header``,
``SUPPORTED_TARGETS``/``SUPPORTED_VERSIONS``.  The IR + meta.json contract is
the reference's: the entry point is the kernel's name (else meta ``entry``),
``.param`` names are ``p_<arg>`` in meta ``arg_order`` (else inputs then
outputs, with a stderr warning when no meta.json exists), and launch
geometry comes from meta.json.  Errors raise ``SystemExit`` with the
statement context, bad targets/versions raise ``ValueError``.

What changes: ``target="sm_100a"`` (PTX ISA 8.6-8.8) selects B200 lowering.
Instead of lowering statement by statement, the kernel is recognised as one
of Emmy's categories and emitted as a hand-written sm_100a kernel for that
category (``emmy_ptx.sm100``).  A kernel that no category takes, and every
kernel for another target, goes through the general statement-level
lowering (``emmy_ptx.sm100.general``).  Extra launch needs (a tuned grid,
dynamic shared memory, tensor maps, the status word, pre-launch entries) are
described by ``Compiler.sidecar()`` and consumed by ``emmy_ptx.runtime``; the
PTX itself keeps the meta.json parameter list and is correct under the
meta.json geometry.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
import sys
from pathlib import Path

from . import ir as I
from .sm100.ops import dtype_name

SUPPORTED_TARGETS = {
    "sm_70", "sm_75", "sm_80", "sm_86", "sm_89", "sm_90", "sm_100", "sm_100a",
}
SUPPORTED_VERSIONS = {"7.0", "7.5", "8.0", "8.5", "8.6", "8.7", "8.8", "9.0"}

B200_TARGET = "sm_100a"
B200_MIN_VERSION = (8, 6)
B200_DEFAULT_VERSION = "8.7"


def float_bits(value: float) -> int:
    """IEEE-754 binary32 bits of ``value``."""
    return struct.unpack("<I", struct.pack("<f", float(value)))[0]


def float16_bits(value: float) -> int:
    """IEEE-754 binary16 bits of ``value``."""
    return struct.unpack("<H", struct.pack("<e", float(value)))[0]


def float64_bits(value: float) -> int:
    """IEEE-754 binary64 bits of ``value``."""
    return struct.unpack("<Q", struct.pack("<d", float(value)))[0]


def sanitize(name: str) -> str:
    return "".join(c if c.isalnum() or c == "_" else "_" for c in name)


def _vtuple(v: str):
    major, minor = v.split(".")
    return int(major), int(minor)


def ptx_header(version: str = "8.0", target: str = "sm_89") -> str:
    if target not in SUPPORTED_TARGETS:
        raise ValueError(f"unsupported target {target!r}; choose from {sorted(SUPPORTED_TARGETS)}")
    if version not in SUPPORTED_VERSIONS:
        raise ValueError(f"unsupported PTX version {version!r}; choose from {sorted(SUPPORTED_VERSIONS)}")
    if target == B200_TARGET and _vtuple(version) < B200_MIN_VERSION:
        raise ValueError(f"PTX ISA {version} cannot target {target}; use 8.6 or later "
                         f"(e.g. --version {B200_DEFAULT_VERSION})")
    return f".version {version}\n.target {target}\n.address_size 64\n"


class Compiler:
    """Reads one IR package and lowers its kernel.

    ``int_semantics`` (keyword, default ``"reference"``) chooses integer
    ``floor_divide``/``remainder``: ``"reference"`` truncates like the
    reference's ``div.s32``/``rem.s32`` (compiler.py:1383-1385);
    ``"torch"`` floors like ``torch.floor_divide``/``torch.remainder``.
    """

    def __init__(self, ir_path, *, target: str = "sm_89", ptx_version: str = "8.0",
                 int_semantics: str = "reference"):
        self.ir_path = Path(ir_path)
        self.target = target
        self.ptx_version = ptx_version
        if int_semantics not in ("reference", "torch"):
            raise ValueError("int_semantics must be 'reference' or 'torch'")
        self.int_semantics = int_semantics
        self.raw = json.loads(self.ir_path.read_text())
        self.graph = self._parse_graph(self.raw)
        self.kernel = self._find_kernel()
        if getattr(self.kernel, "serial", None):
            raise SystemExit(
                "KernelOp.serial is not empty: serial axes are launched one "
                "coordinate at a time with runtime integer parameters, which "
                "this compiler does not implement")
        self.meta = self._find_meta()
        self.kmeta = self._kernel_meta()
        self.entry = self.kernel.name or self.kmeta.get("entry", self.kernel.name)
        self.tensors: dict = {}
        for node in self.raw.get("nodes", {}).values():
            for out in node.get("outputs", []):
                self.tensors[out["name"]] = out
        for arg in self.kmeta.get("args", []):
            self.tensors.setdefault(arg["name"], {
                "name": arg["name"], "shape": arg.get("shape", []),
                "dtype": arg.get("dtype", "f32")})
        self.arg_order = list(self.kmeta.get("arg_order")
                              or (list(self.kernel.inputs) + list(self.kernel.outputs)))
        self.args = {a["name"]: a for a in self.kmeta.get("args", [])}
        self.smem_names = {s.name for s in I.walk(self.kernel.body) if isinstance(s, I.Smem)}
        self._result = None

    # ------------------------------------------------------------------
    # reader (same resolution rules as the reference, compiler.py:255-324)
    # ------------------------------------------------------------------
    @staticmethod
    def _parse_graph(raw):
        try:
            return I.Graph.from_dict(raw)
        except I.IRParseError as exc:
            raise SystemExit(f"IR parse error: {exc}") from exc

    def _find_kernel(self):
        for node in self.graph.nodes.values():
            if isinstance(node.op, I.KernelOp):
                return node.op
        raise SystemExit("no KernelOp found in IR")

    def _meta_mentions_kernel(self, meta: dict) -> bool:
        kernels = meta.get("kernels")
        if not isinstance(kernels, list) or not kernels:
            return False
        if len(kernels) == 1:
            return True
        return any(k.get("entry") == self.kernel.name for k in kernels)

    def _find_meta(self) -> dict:
        sibling = self.ir_path.with_name("meta.json")
        if sibling.exists():
            return json.loads(sibling.read_text())
        for folder in [self.ir_path.parent, *self.ir_path.parent.parents]:
            candidate = folder / "meta.json"
            if candidate.exists():
                meta = json.loads(candidate.read_text())
                if self._meta_mentions_kernel(meta):
                    return meta
        print(f"warning: no meta.json found for {self.ir_path}; using the IR's own "
              "argument order (inputs followed by outputs)", file=sys.stderr)
        return {}

    def _kernel_meta(self) -> dict:
        if not self.meta:
            return {}
        kernels = self.meta.get("kernels")
        if not isinstance(kernels, list) or not kernels:
            raise SystemExit("meta.json has no kernels")
        for k in kernels:
            if k.get("entry") == self.kernel.name:
                return k
        if len(kernels) == 1:
            return kernels[0]
        raise SystemExit(
            f"kernel {self.kernel.name!r} is not listed in meta.json "
            f"({', '.join(str(k.get('entry')) for k in kernels)}); its argument "
            "order would be wrong")

    def shape_of(self, name: str):
        if name not in self.tensors:
            raise SystemExit(f"unknown buffer {name!r}")
        return [int(x) for x in self.tensors[name].get("shape", [])]

    def dtype_of(self, name: str):
        if name not in self.tensors:
            raise SystemExit(f"unknown buffer {name!r}")
        return dtype_name(self.tensors[name].get("dtype", "f32"))

    # ------------------------------------------------------------------
    def plan(self):
        """The category plan for the sm_100a backend: ``(category, plan)``;
        ``("general", reasons)`` when no category recogniser takes the
        kernel."""
        from .sm100 import select
        return select.choose(self)

    def check(self) -> list:
        """Validate without producing PTX (reference compiler.py:2159-2200),
        plus what only lowering finds: an unsupported construct, shared
        memory beyond 227 KB, and a launch geometry the kernel cannot run
        under (block not a multiple of 32 or above 1024 threads, a tile the
        meta.json grid does not cover)."""
        issues = []
        if not self.ir_path.exists():
            return [f"IR file not found: {self.ir_path}"]
        if getattr(self.kernel, "serial", None):
            issues.append("KernelOp.serial is not empty (not implemented)")
            return issues
        if not self.kmeta:
            issues.append("no meta.json found — argument order and launch geometry are unknown")
        try:
            ptx_header(self.ptx_version, self.target)
        except ValueError as exc:
            issues.append(str(exc))
            return issues
        if any(isinstance(s, I.SetMaxNReg) for s in I.walk(self.kernel.body)):
            issues.append("SetMaxNReg will be dropped (its register split cannot be "
                          "checked against the launch)")
        block = self._geom_product("block")
        grid = self._geom_product("grid")
        if block is not None and (block % 32 or block > 1024):
            issues.append(f"meta.json block of {block} threads: must be a multiple of 32, "
                          "at most 1024")
        if block and grid:
            for tile in (s for s in I.walk(self.kernel.body) if isinstance(s, I.Tile)):
                if not all(a.extent.is_static for a in tile.axes):
                    continue
                n = 1
                for a in tile.axes:
                    n *= int(a.extent.as_static())
                width = int(tile.block_threads) if tile.block_threads else block
                if grid * width < n:
                    issues.append(f"meta.json grid of {grid} blocks x {width} threads covers "
                                  f"{grid * width} of the tile's {n} elements (the reference "
                                  "leaves the rest unwritten; this backend loops over them)")
        try:
            self._lower()
        except SystemExit as exc:
            issues.append(str(exc))
        return issues

    def _geom_product(self, key):
        v = self.kmeta.get(key)
        if not v:
            return None
        v = [v] if isinstance(v, int) else list(v)
        n = 1
        for x in v:
            n *= int(x)
        return n

    def _lower(self):
        if self._result is None:
            ptx_header(self.ptx_version, self.target)
            from .sm100 import select
            if self.target == B200_TARGET:
                category, plan = select.choose(self)
            else:
                category, plan = "general", [f"target {self.target}: tensor-core and "
                                             "category kernels are sm_100a only"]
            ptx, sidecar = select.emit(self, category, plan)
            sidecar = dict(sidecar)
            sidecar.setdefault("entry", self.entry)
            sidecar.setdefault("arg_order", list(self.arg_order))
            sidecar.setdefault("meta_grid", list(self.kmeta.get("grid") or []))
            sidecar.setdefault("meta_block", list(self.kmeta.get("block") or []))
            self._result = (ptx, sidecar)
        return self._result

    def compile(self) -> str:
        return self._lower()[0]

    def sidecar(self) -> dict:
        """Launch needs beyond meta.json: tuned grid, dynamic shared memory,
        cluster shape, tensor maps to encode, the status word."""
        return self._lower()[1]


def _cache_key(path, target, ptx_version) -> str:
    """sha256 of the IR bytes, the sibling meta.json and target:version
    (the reference's key, compiler.py:2238-2245)."""
    h = hashlib.sha256()
    h.update(Path(path).read_bytes())
    meta = Path(path).with_name("meta.json")
    if meta.exists():
        h.update(meta.read_bytes())
    h.update(f"{target}:{ptx_version}".encode())
    return h.hexdigest()[:16]


def compile_file(path, *, target: str = "sm_89", ptx_version: str = "8.0",
                 cache_dir=None) -> str:
    """Compile ``path``; with ``cache_dir`` the PTX (and its launch sidecar,
    ``<key>.json``) is cached by IR hash."""
    return compile_cached(path, target=target, ptx_version=ptx_version, cache_dir=cache_dir)[0]


def compile_cached(path, *, target: str = "sm_89", ptx_version: str = "8.0",
                   cache_dir=None):
    """``compile_file`` that also returns the launch sidecar: ``(ptx,
    sidecar)``.  On a cache hit both come from the cache (``<key>.ptx`` and
    ``<key>.json``); the sidecar is None if the cache holds none."""
    if cache_dir is not None:
        os.makedirs(cache_dir, exist_ok=True)
        key = _cache_key(path, target, ptx_version)
        cache_path = os.path.join(cache_dir, key + ".ptx")
        side_path = os.path.join(cache_dir, key + ".json")
        if os.path.exists(cache_path):
            with open(cache_path) as f:
                ptx = f.read()
            sidecar = None
            if os.path.exists(side_path):
                with open(side_path) as f:
                    sidecar = json.load(f)
            return ptx, sidecar
    comp = Compiler(path, target=target, ptx_version=ptx_version)
    result = comp.compile()
    sidecar = comp.sidecar()
    if cache_dir is not None:
        with open(cache_path, "w") as f:
            f.write(result)
        with open(side_path, "w") as f:
            json.dump(sidecar, f, indent=1)
    return result, sidecar
