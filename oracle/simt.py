"""CPU oracle: a lane-parallel interpreter of Emmy Kernel IR.

TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this module; the product never calls it.

It restates, statement by statement, what the PTX emitted by the reference
compiler computes (emmy_ptx/compiler.py in the reference; line numbers
below).  Every thread of the launch is one numpy lane.  Lanes run in
lockstep: a statement finishes for all lanes before the next starts, which
is what the IR's barriers (``Sync``, the ``bar.sync`` between tree levels,
``cp.async.wait_group``) guarantee on the GPU for race-free IR.  Divergence
(the tile guard, ``Cond``, loops whose trip count differs per lane) is a
boolean lane mask; a statement updates only active lanes, as a predicated
PTX instruction would.  Reductions therefore combine values in exactly the
order the reference's threads do (strided per-thread partials, then the
butterfly shuffle, then the shared-memory tree), so float results agree with
the reference's GPU results up to the ulp-level error of its ``*.approx``
instructions.

Out-of-bounds global or shared accesses by an active lane raise
``OracleError`` instead of reading garbage.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_PKG = _HERE.parent / "emmy-ptx_b200"
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

from emmy_ptx import ir as I  # noqa: E402  (IR node classes only)

from .ops import (NP, OracleError, binary_expr, coerce, cvt_rzi_s32,  # noqa: E402
                  dtype_name, is_float, op_on_values)

_BYTES = {"f32": 4, "s32": 4, "u32": 4, "f64": 8, "s64": 8, "f16": 2, "bf16": 2, "u8": 1}


def _prod(xs):
    n = 1
    for x in xs:
        n *= int(x)
    return n


class Interpreter:
    """Runs one KernelOp over a 1-D launch of ``grid x block`` threads."""

    def __init__(self, kernel: I.KernelOp, tensors: dict, args: dict,
                 grid: int, block: int, int_semantics: str = "reference"):
        self.kernel = kernel
        self.int_semantics = int_semantics
        self.tensors = tensors          # name -> {"shape", "dtype"}
        self.args = args                # meta args by name
        self.grid = int(grid)
        self.block = int(block)
        if self.block % 32:
            raise OracleError("block size must be a multiple of 32")
        n = self.grid * self.block
        g = np.arange(n, dtype=np.int64)
        self.tid = (g % self.block).astype(np.int32)
        self.cta = (g // self.block).astype(np.int32)
        self.n = n
        self.vals: dict = {}
        self.buf: dict = {}
        self.smem: dict = {}

    # ------------------------------------------------------------------
    def shape_of(self, name):
        if name in self.smem:
            return self.smem[name]["extents"]
        if name not in self.tensors:
            raise OracleError(f"unknown buffer {name!r}")
        return list(self.tensors[name].get("shape", []))

    def dtype_of(self, name):
        if name in self.smem:
            return self.smem[name]["dtype"]
        if name not in self.tensors:
            raise OracleError(f"unknown buffer {name!r}")
        return dtype_name(self.tensors[name].get("dtype", "f32"))

    def _full(self, v, dt):
        a = np.asarray(v)
        if a.shape != (self.n,):
            a = np.broadcast_to(a, (self.n,))
        return a.astype(NP[dt], copy=True)

    def set(self, name, value, dt, mask):
        dt = dtype_name(dt)
        new = self._full(value, dt)
        old = self.vals.get(name)
        if old is not None and old[1] == dt:
            new = np.where(mask, new, old[0])
        self.vals[name] = (new, dt)

    def get(self, name):
        if name not in self.vals:
            raise OracleError(f"unknown variable {name!r}")
        return self.vals[name]

    # ------------------------------------------------------------------
    # expressions (compiler.py:626-861)
    # ------------------------------------------------------------------
    def expr(self, e):
        if isinstance(e, str):
            e = I.Var(e)
        if isinstance(e, I.Literal):
            name = dtype_name(e.dtype)
            if name.startswith("s") or name.startswith("i") or name == "int" \
                    or isinstance(e.value, int):
                return np.int32(int(e.value)), "s32"
            if name == "f64":
                return np.float64(e.value), "f64"
            if name == "f16":
                raise OracleError("f16 literals are unsupported")
            return np.float32(e.value), "f32"
        if isinstance(e, I.Var):
            return self.get(e.name)
        if isinstance(e, I.BinaryExpr):
            a, adt = self.expr(e.left)
            b, bdt = self.expr(e.right)
            return binary_expr(e.op, a, adt, b, bdt)
        if isinstance(e, I.TernaryExpr):
            p = self.to_pred(e.cond)
            a, adt = self.expr(e.if_true)
            b, bdt = self.expr(e.if_false)
            target = "f64" if "f64" in (adt, bdt) else (
                "f32" if (is_float(adt) or is_float(bdt)) else "s32")
            return np.where(p, coerce(a, adt, target), coerce(b, bdt, target)), target
        if isinstance(e, I.CastExpr):
            v, src = self.expr(e.expr)
            dst = dtype_name(e.dtype)
            if dst == src:
                return v, src
            if dst == "f32" and not is_float(src):
                return np.asarray(v).astype(np.float32), "f32"
            if dst == "s32" and is_float(src):
                return cvt_rzi_s32(v), "s32"
            raise OracleError(f"unsupported cast {src} -> {dst}")
        if isinstance(e, I.Builtin):
            table = {"threadIdx.x": self.tid, "blockIdx.x": self.cta,
                     "blockDim.x": np.int32(self.block),
                     "gridDim.x": np.int32(self.grid),
                     "threadIdx.y": np.int32(0), "threadIdx.z": np.int32(0),
                     "blockIdx.y": np.int32(0), "blockIdx.z": np.int32(0),
                     "blockDim.y": np.int32(1), "blockDim.z": np.int32(1)}
            if e.name not in table:
                raise OracleError(f"unsupported builtin {e.name!r}")
            return table[e.name], "s32"
        if isinstance(e, I.FuncCallExpr):
            vs = [self.expr(a) for a in e.args]
            return op_on_values(e.name, [v for v, _ in vs], [d for _, d in vs], "f32")
        if isinstance(e, I.FlatIndex):
            return self.flatten(e.buffer, e.index), "s32"
        raise OracleError(f"unsupported expression {type(e).__name__}")

    def to_pred(self, e):
        v, dt = self.expr(e)
        if dt == "pred":
            return np.asarray(v, bool)
        return np.asarray(v) != 0

    def flatten(self, name, indices):
        """Row-major flat index (compiler.py:536-564)."""
        shape = self.shape_of(name)
        indices = tuple(indices or ())
        if not indices:
            return np.int64(0)
        if len(indices) != len(shape):
            raise OracleError(f"index rank {len(indices)} != shape rank {len(shape)} for {name}")
        flat = np.int64(0)
        stride = 1
        for idx, ext in zip(reversed(indices), reversed(shape)):
            v, _ = self.expr(idx)
            flat = flat + np.asarray(v, np.int64) * stride
            stride *= int(ext)
        return flat

    def _add_last(self, index, k):
        idx = list(index)
        if k and idx:
            idx[-1] = I.BinaryExpr("+", idx[-1], I.Literal(k, "int"))
        return idx

    # ------------------------------------------------------------------
    # memory
    # ------------------------------------------------------------------
    def _check(self, name, flat, mask, size):
        f = np.broadcast_to(np.asarray(flat, np.int64), (self.n,))
        bad = mask & ((f < 0) | (f >= size))
        if bad.any():
            lane = int(np.argmax(bad))
            raise OracleError(
                f"out-of-bounds access to {name!r}: index {int(f[lane])} of {size} "
                f"(thread {int(self.tid[lane])} of block {int(self.cta[lane])})")
        return np.where(mask, f, 0)

    def load_elem(self, name, flat, mask):
        if name in self.smem:
            arr = self.smem[name]["data"]
            f = self._check(name, flat, mask, arr.shape[1])
            return arr[self.cta, f]
        arr = self.buf[name]
        f = self._check(name, flat, mask, arr.size)
        return arr[f]

    def store_elem(self, name, flat, value, mask, atomic=None):
        if not mask.any():
            return
        if name in self.smem:
            arr = self.smem[name]["data"]
            f = self._check(name, flat, mask, arr.shape[1])
            arr[self.cta[mask], f[mask]] = np.broadcast_to(value, (self.n,))[mask]
            return
        arr = self.buf[name]
        f = self._check(name, flat, mask, arr.size)
        v = np.broadcast_to(np.asarray(value, arr.dtype), (self.n,))[mask]
        if atomic:
            op = "add" if atomic is True else str(atomic)
            if op != "add":
                raise OracleError(f"unsupported atomic op {op!r}")
            np.add.at(arr, f[mask], v)
        else:
            arr[f[mask]] = v

    # ------------------------------------------------------------------
    # statements (compiler.py:1409-2104)
    # ------------------------------------------------------------------
    def stmts(self, body, mask):
        for s in body or ():
            self.stmt(s, mask)

    def stmt(self, s, mask):
        if isinstance(s, (list, tuple)):
            return self.stmts(s, mask)
        method = getattr(self, "s_" + type(s).__name__, None)
        if method is None:
            raise OracleError(f"unsupported statement {type(s).__name__}")
        method(s, mask)

    def s_Smem(self, s, mask):
        return

    def s_Sync(self, s, mask):
        return

    def s_SetMaxNReg(self, s, mask):
        return

    def s_CpAsyncCommit(self, s, mask):
        return

    def s_CpAsyncWait(self, s, mask):
        return

    def s_Tile(self, s, mask):
        """compiler.py:1463-1585: one thread per tile element."""
        extents = []
        for axis in s.axes:
            if not axis.extent.is_static:
                raise OracleError(f"dynamic tile axis {axis.name!r} is unsupported")
            extents.append(int(axis.extent.as_static()))
        n = _prod(extents)
        tid = self.tid.astype(np.int64)
        cta = self.cta.astype(np.int64)
        if s.block_threads:
            width = int(s.block_threads)
            t = tid % width if s.aux_threads else tid
            gid = cta * width + t
        else:
            gid = cta * self.block + tid
        mask = mask & (gid < n)
        strides = [1] * len(extents)
        for i in range(len(extents) - 2, -1, -1):
            strides[i] = strides[i + 1] * extents[i + 1]
        raster = None
        if s.raster_group and s.raster_axes:
            names = [a.name for a in s.axes]
            if s.raster_axes[0] in names and s.raster_axes[1] in names:
                mi, ni = names.index(s.raster_axes[0]), names.index(s.raster_axes[1])
                if ni == mi + 1:
                    gi, oi = (mi, ni) if s.raster_orient == "m" else (ni, mi)
                    g = min(int(s.raster_group), extents[gi])
                    if extents[gi] > 1 and g > 1:
                        raster = (gi, oi, g)
        if raster is not None:                      # compiler.py:1513-1561
            gi, oi, g = raster
            ea, eb = extents[gi], extents[oi]
            mi2, ni2 = min(gi, oi), max(gi, oi)
            sub = gid // strides[ni2]
            if mi2 != 0:
                sub = sub % (ea * eb)
            if ea % g == 0:
                ra = (sub // (g * eb)) * g + sub % g
                rb = (sub % (g * eb)) // g
            else:
                grp = sub // (g * eb)
                rsz = np.minimum(ea - grp * g, g)
                tmp = sub % (g * eb)
                ra = grp * g + tmp % rsz
                rb = tmp // rsz
        for i, (axis, ext, stride) in enumerate(zip(s.axes, extents, strides)):
            if ext == 1:
                v = np.zeros(self.n, np.int64)
            elif raster is not None and i == gi:
                v = ra
            elif raster is not None and i == oi:
                v = rb
            elif i == len(extents) - 1:
                v = gid % ext
            elif i == 0:
                v = gid // stride
            else:
                v = (gid // stride) % ext
            self.vals[axis.name] = (v.astype(np.int32), "s32")
        self.stmts(s.body, mask)

    def s_Load(self, s, mask):
        """compiler.py:1587-1629."""
        names = s.names
        src = s.input
        dt = dtype_name(s.dtype) if s.dtype is not None else self.dtype_of(src)
        if dt != self.dtype_of(src):
            raise OracleError(f"Load of {src!r} as {dt} from a {self.dtype_of(src)} buffer")
        for k, name in enumerate(names):
            if name is None:
                continue
            flat = self.flatten(src, self._add_last(tuple(s.index or ()), k))
            self.set(name, self.load_elem(src, flat, mask), dt, mask)

    def s_Assign(self, s, mask):
        dt = dtype_name(s.dtype) if s.dtype is not None else self.get(s.args[0])[1]
        vs = [self.get(a) for a in s.args]
        v, rdt = op_on_values(s.op, [x for x, _ in vs], [d for _, d in vs], dt,
                              self.int_semantics)
        self.set(s.name, v, rdt, mask)

    def s_Let(self, s, mask):
        v, dt = self.expr(s.value)
        self.set(s.name, v, dtype_name(s.dtype) if s.dtype is not None else dt, mask)

    def s_Accum(self, s, mask):
        """compiler.py:1649-1659: in-place update of the accumulator."""
        if s.name not in self.vals:
            raise OracleError(f"Accum {s.name}: accumulator was not seeded")
        acc, acc_dt = self.vals[s.name]
        dt = dtype_name(s.dtype) if s.dtype is not None else acc_dt
        a, adt = self.get(s.base) if s.base else (acc, acc_dt)
        b, bdt = self.get(s.value)
        v, rdt = op_on_values(s.op, (a, b), (adt, bdt), dt)
        self.set(s.name, v, rdt, mask)

    def s_Write(self, s, mask):
        """compiler.py:1661-1719; values are converted to the buffer dtype."""
        out = s.output
        dt = dtype_name(s.value_dtype) if s.value_dtype is not None else self.dtype_of(out)
        if out not in self.smem:
            dt = self.dtype_of(out)
        for k, name in enumerate(s.values):
            if name is None:
                continue
            v, vdt = self.get(name)
            if vdt != dt:
                v = coerce(v, vdt, dt)
            flat = self.flatten(out, self._add_last(tuple(s.index or ()), k))
            self.store_elem(out, flat, v, mask, atomic=s.atomic if out not in self.smem else None)

    def s_Init(self, s, mask):
        dt = dtype_name(s.dtype) if s.dtype is not None else "f32"
        val = float(s.identity) if is_float(dt) else int(s.identity)
        self.set(s.name, val, dt, mask)

    def s_Cond(self, s, mask):
        p = self.to_pred(s.cond)
        self.stmts(s.body, mask & p)
        self.stmts(s.else_body, mask & ~p)

    def _seed(self, body, loop_axis, mask):
        """compiler.py:1741-1759."""
        seen = set()
        for st in body:
            if isinstance(st, I.Accum) and st.name not in seen:
                if loop_axis is not None and st.axes and loop_axis not in st.axes:
                    continue
                seen.add(st.name)
                dt = dtype_name(st.dtype) if st.dtype is not None else "f32"
                ident = st.op.identity
                if ident is None:
                    raise OracleError(f"no identity for accumulator op {st.op.name}")
                self.set(st.name, float(ident) if is_float(dt) else int(ident), dt, mask)

    def _scope(self, axis, run):
        old = self.vals.get(axis)
        try:
            run()
        finally:
            if old is not None:
                self.vals[axis] = old
            else:
                self.vals.pop(axis, None)

    def s_Loop(self, s, mask):
        """compiler.py:1761-1793."""
        if not s.axis.extent.is_static:
            raise OracleError(f"dynamic loop axis {s.axis.name!r} is unsupported")
        extent = int(s.axis.extent.as_static())
        if s.seed:
            self._seed(s.body, s.axis.name, mask)

        def run():
            for i in range(extent):
                self.vals[s.axis.name] = (np.full(self.n, i, np.int32), "s32")
                self.stmts(s.body, mask)
        self._scope(s.axis.name, run)

    def s_StridedLoop(self, s, mask):
        """compiler.py:1831-1867: counter from ``start`` by ``step`` while
        ``counter < end`` (signed), per lane."""
        axis = s.axis.name
        if s.seed:
            self._seed(s.body, axis, mask)
        start, _ = self.expr(s.start)
        step, _ = self.expr(s.step)
        if s.end is None:
            if not s.axis.extent.is_static:
                raise OracleError(f"dynamic strided loop axis {axis!r} is unsupported")
            end = np.int64(int(s.axis.extent.as_static()))
        else:
            end = np.asarray(self.expr(s.end)[0], np.int64)
        counter = np.broadcast_to(np.asarray(start, np.int64), (self.n,)).copy()
        step = np.broadcast_to(np.asarray(step, np.int64), (self.n,))

        def run():
            nonlocal counter
            active = mask & (counter < end)
            while active.any():
                self.vals[axis] = (counter.astype(np.int32), "s32")
                self.stmts(s.body, active)
                counter = np.where(active, counter + step, counter)
                active = active & (counter < end)
        self._scope(axis, run)

    def _shfl_xor(self, v, step):
        idx = np.arange(self.n, dtype=np.int64) ^ int(step)
        return np.asarray(v)[idx]

    def s_WarpShuffle(self, s, mask):
        """compiler.py:1877-1902: butterfly over ``length`` lanes."""
        dt = dtype_name(s.dtype)
        step = int(s.length) // 2
        while step > 0:
            for st, stb in zip(s.state, s.state_b):
                v, vdt = self.get(st)
                if vdt != dt:
                    raise OracleError(f"WarpShuffle of a {vdt} value as {dt}")
                self.set(stb, self._shfl_xor(v, step), dt, mask)
            self.stmts(s.combine_states, mask)
            step //= 2

    def s_TreeHalve(self, s, mask):
        """compiler.py:1933-2006: shared-memory tree, flat (slot t) or
        segmented (slot t*scale + iv, root iv)."""
        dt = dtype_name(s.dtype)
        tid = np.asarray(self.get(s.tid_var)[0], np.int64)
        bufs, states, sbs = list(s.bufs), list(s.state), list(s.state_b)
        if len(bufs) == 1 and len(states) > 1:
            bufs = bufs * len(states)
        iv = scale = None
        if s.inner is not None:
            iv_name, scale = s.inner
            scale = int(scale)
            iv = np.asarray(self.get(iv_name)[0], np.int64)

        def slot(plus):
            if iv is None:
                return tid + plus
            return tid * scale + iv + plus * scale

        step = int(s.length) // 2
        while step > 0:
            on = mask & (tid < step)
            for buf, st, stb in zip(bufs, states, sbs):
                self.set(st, self.load_elem(buf, slot(0), on), dt, on)
                self.set(stb, self.load_elem(buf, slot(step), on), dt, on)
            self.stmts(s.combine_states, on)
            for buf, st in zip(bufs, states):
                self.store_elem(buf, slot(0), self.get(st)[0], on)
            step //= 2
        for buf, st in zip(bufs, states):
            root = iv if iv is not None else np.int64(0)
            self.set(st, self.load_elem(buf, root, mask), dt, mask)

    def s_CpAsyncCopy(self, s, mask):
        """compiler.py:2014-2034: ``nbytes`` from global to shared."""
        if s.swizzle not in (None, "NONE"):
            raise OracleError(f"unsupported cp.async swizzle {s.swizzle!r}")
        flat = self.flatten(s.smem, s.smem_index) if s.smem_index else np.int64(0)
        if s.lane_index is not None:
            cols = self.shape_of(s.smem)[-1]
            row = np.asarray(self.expr(s.lane_index[0])[0], np.int64)
            col = np.asarray(self.expr(s.lane_index[1])[0], np.int64)
            flat = flat + row * cols + col
        src_flat = self.flatten(s.src, s.src_index)
        sdt, gdt = self.dtype_of(s.smem), self.dtype_of(s.src)
        if sdt != gdt:
            raise OracleError("cp.async between buffers of different dtypes")
        n = int(s.nbytes) // _BYTES[sdt]
        for e in range(n):
            v = self.load_elem(s.src, src_flat + e, mask)
            self.store_elem(s.smem, flat + e, v, mask)

    def s_Select(self, s, mask):
        """compiler.py:2057-2071."""
        branches = list(s.branches)
        if not branches:
            raise OracleError(f"Select {s.name} has no branches")
        out, dt = self.expr(branches[-1].value)
        out = self._full(out, dt)
        for br in reversed(branches[:-1]):
            p = self.to_pred(br.select)
            v, vdt = self.expr(br.value)
            out = np.where(p, coerce(v, vdt, dt), out)
        self.set(s.name, out, dt, mask)

    def s_ZeroPrologue(self, s, mask):
        """compiler.py:2073-2104 (intent: block 0 zeroes ``words`` words)."""
        words = int(s.words)
        if words <= 0 or not (mask & (self.cta == 0)).any():
            return
        arr = self.buf[s.dst]
        arr.view(np.uint8)[: 4 * words] = 0

    # ------------------------------------------------------------------
    def run(self, buffers: dict, scalars: dict | None = None):
        """Execute the kernel; ``buffers`` maps tensor names to arrays
        (outputs included, with their initial contents).  Returns the
        output buffers reshaped."""
        for name, arr in buffers.items():
            dt = self.dtype_of(name)
            self.buf[name] = np.array(arr, dtype=NP[dt], copy=True).reshape(-1)
        for s in I.walk(self.kernel.body):
            if isinstance(s, I.Smem):
                self.smem[s.name] = {
                    "extents": [int(e) for e in s.extents],
                    "dtype": dtype_name(s.dtype),
                    "data": np.zeros((self.grid, _prod(s.extents)), NP[dtype_name(s.dtype)]),
                }
        everyone = np.ones(self.n, bool)
        for name, v in (scalars or {}).items():     # compiler.py:2116-2136
            dt = dtype_name(self.args.get(name, {}).get("dtype", "f32"))
            self.set(name, v, dt, everyone)
        self.vals["lane"] = ((self.tid & 31).astype(np.int32), "s32")
        self.vals["warp"] = ((self.tid >> 5).astype(np.int32), "s32")
        self.vals["threadIdx.x"] = (self.tid, "s32")
        self.stmts(self.kernel.body, everyone)
        return {name: self.buf[name].reshape(self.shape_of(name))
                for name in self.kernel.outputs}


# ----------------------------------------------------------------------------
# package-level entry points (mirroring the reference's reader,
# compiler.py:211-250, 275-310)
# ----------------------------------------------------------------------------
def load_package(ir_path):
    ir_path = Path(ir_path)
    raw = json.loads(ir_path.read_text())
    graph = I.Graph.from_dict(raw)
    kernel = next((n.op for n in graph.nodes.values() if isinstance(n.op, I.KernelOp)), None)
    if kernel is None:
        raise OracleError("no KernelOp found in IR")
    meta_path = ir_path.with_name("meta.json")
    if not meta_path.exists():
        raise OracleError("the oracle needs meta.json for the launch geometry")
    meta = json.loads(meta_path.read_text())
    kmeta = next((k for k in meta["kernels"] if k.get("entry") == kernel.name),
                 meta["kernels"][0])
    tensors = {}
    for node in raw.get("nodes", {}).values():
        for out in node.get("outputs", []):
            tensors[out["name"]] = out
    for arg in kmeta.get("args", []):
        tensors.setdefault(arg["name"], arg)
    return kernel, tensors, kmeta


def run_package(ir_path, inputs: dict, out_init=None, scalars=None,
                int_semantics="reference"):
    """Run an IR package on host arrays; returns ``{output: array}``.

    ``out_init`` gives the initial contents of output buffers (default
    zeros) so that unwritten elements can be detected by the caller.
    ``int_semantics`` as for the backend's Compiler option.
    """
    kernel, tensors, kmeta = load_package(ir_path)
    grid = _prod(kmeta.get("grid", [1]))
    block = _prod(kmeta.get("block", [1]))
    interp = Interpreter(kernel, tensors, {a["name"]: a for a in kmeta.get("args", [])},
                         grid, block, int_semantics)
    bufs = dict(inputs)
    for name in kernel.outputs:
        t = tensors[name]
        dt = dtype_name(t.get("dtype", "f32"))
        if out_init is not None and name in out_init:
            bufs[name] = np.asarray(out_init[name], NP[dt])
        else:
            bufs[name] = np.zeros(_prod(t.get("shape", [])), NP[dt])
    return interp.run(bufs, scalars)


def run_problem(problem, inputs: dict, workdir, out_init=None):
    """Write a workloads.Problem package to ``workdir`` and run it."""
    ir_path = problem.write(workdir)
    return run_package(ir_path, inputs, out_init)


__all__ = ["Interpreter", "run_package", "run_problem", "load_package", "OracleError"]
