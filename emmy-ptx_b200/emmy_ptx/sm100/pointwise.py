"""Pointwise category: any elementwise IR -> a v4 grid-stride sm_100a kernel.

Recognised IR (what the reference lowers one thread per tile element,
compiler.py:1463-1585, 1587-1719): a single ``Tile`` whose body is only
``Load``/``Let``/``Assign``/``Write``, where every load and write addresses
``flat = w * tile_element + k`` for component ``k < w`` (the identity map,
with the reference's grouped 2/4-wide names), every tensor is covered
exactly once, and every component computes the same expression.  The
element program is the expression DAG of each output.

Generated kernel: each thread walks groups of 4 consecutive elements with a
grid-stride loop, unrolled U groups deep so U x (inputs) 16-byte loads are
in flight before any arithmetic; 8-byte dtypes move as two 16-byte halves.
A scalar tail handles a size that is not a multiple of 4.  There is no
integer division in the loop (the reference decodes every tile coordinate
with div/rem, compiler.py:1563-1582).  Correct for any grid and block size.
"""

from __future__ import annotations

from dataclasses import dataclass

from .. import ir as I
from .common import (NoMatch, Program, Sym, declare_params, emit_program,
                     flat_affine, launch_block, literal_sym, nbytes, prod,
                     row_major_strides, shift_components, const_value)
from .ops import F32_ONLY, Ops, dtype_name, is_float
from .ptx import KernelBuilder, MEM_TYPE, wide_vectors

GROUP = 4


def result_dtype(name, arg_dts, dtype):
    """Static result dtype of an op, following the emitter's rules."""
    name = getattr(name, "name", str(name))
    dt = dtype_name(dtype) or "f32"
    if name in ("greater", "greater_equal", "less", "less_equal", "equal", "not_equal",
                "logical_not"):
        return "pred"
    if name in ("logical_and", "logical_or"):
        return "pred" if list(arg_dts) == ["pred", "pred"] else "s32"
    if name in ("negative", "neg"):
        return arg_dts[0]
    if name in F32_ONLY:
        return "f32"
    if name in ("absolute", "abs"):
        return dt if dt in ("f32", "f64") else "s32"
    if name in ("where", "copy", "pad", "bitcast"):
        return dt
    if is_float(dt):
        return dt
    return "s32"


@dataclass
class PointwisePlan:
    n_elems: int
    width: int
    program: Program
    dtypes: dict          # tensor -> dtype
    inputs: list
    outputs: list


def match(comp) -> PointwisePlan:
    body = comp.kernel.body
    if len(body) != 1 or not isinstance(body[0], I.Tile):
        raise NoMatch("not a single Tile")
    tile = body[0]
    if tile.aux_threads:
        raise NoMatch("aux threads")
    extents = []
    for ax in tile.axes:
        if not ax.extent.is_static:
            raise NoMatch("dynamic tile axis")
        extents.append(int(ax.extent.as_static()))
    tstrides = row_major_strides(extents)
    axis_names = [a.name for a in tile.axes]
    n_tile = prod(extents)

    env, dts, consts = {}, {}, {}
    width = None
    writes = {}
    tensor_dt = {}

    def check_index(name, index, k, w):
        shape = comp.shape_of(name)
        idx = list(index or ())
        if k and idx:
            idx[-1] = I.BinaryExpr("+", idx[-1], I.Literal(k, "int"))
        fa = flat_affine(shape, tuple(idx), consts)
        if fa is None:
            raise NoMatch(f"non-affine index into {name}")
        want = {a: w * s for a, s in zip(axis_names, tstrides) if e_of(a) > 1}
        got = {key: v for key, v in fa.items() if key is not None and e_of(key) > 1}
        if got != want or fa.get(None, 0) != k:
            raise NoMatch(f"{name} is not indexed by the identity map")
        if n_tile * w != prod(shape):
            raise NoMatch(f"tile does not cover {name} exactly once")

    ext_of = dict(zip(axis_names, extents))

    def e_of(a):
        return ext_of.get(a, 2)

    for s in tile.body:
        if isinstance(s, I.Load):
            dt = dtype_name(s.dtype) if s.dtype is not None else comp.dtype_of(s.input)
            if s.input in getattr(comp, "smem_names", ()) or dt != dtype_name(comp.dtype_of(s.input)):
                raise NoMatch("load type differs from buffer type")
            w = len(s.names)
            width = w if width is None else width
            if w != width:
                raise NoMatch("mixed vector widths")
            for k, nm in enumerate(s.names):
                if nm is None:
                    continue
                check_index(s.input, s.index, k, w)
                env[nm] = Sym("in", s.input, k)
                dts[nm] = dt
            tensor_dt[s.input] = dt
        elif isinstance(s, I.Let):
            v = s.value
            if isinstance(v, I.Literal):
                sym = literal_sym(v)
            elif isinstance(v, I.Var) and v.name in env:
                sym = env[v.name]
            else:
                c = const_value(v, consts)
                if c is None:
                    raise NoMatch("Let of a non-constant expression")
                sym = Sym("const", int(c), "s32")
            if s.dtype is not None and dtype_name(s.dtype) != (dts.get(v.name) if isinstance(v, I.Var) else sym.b):
                # the reference keeps the register and relabels its dtype
                # (compiler.py:1644-1647); only same-kind relabels are safe
                want = dtype_name(s.dtype)
                have = sym.b if sym.kind == "const" else dts.get(getattr(v, "name", None))
                if not ({want, have} <= {"s32", "u32"}):
                    raise NoMatch("Let that relabels a value's dtype")
            env[s.name] = sym
            dts[s.name] = sym.b if sym.kind == "const" else dts[v.name]
            if sym.kind == "const" and sym.b == "s32":
                consts[s.name] = sym.a
        elif isinstance(s, I.Assign):
            for a in s.args:
                if a not in env:
                    raise NoMatch(f"unknown value {a}")
            dt = dtype_name(s.dtype) if s.dtype is not None else dts[s.args[0]]
            opname = getattr(s.op, "name", str(s.op))
            env[s.name] = Sym("op", opname, dt, tuple(env[a] for a in s.args))
            dts[s.name] = result_dtype(opname, [dts[a] for a in s.args], dt)
        elif isinstance(s, I.Write):
            if s.atomic:
                raise NoMatch("atomic write")
            w = len(s.values)
            width = w if width is None else width
            if w != width:
                raise NoMatch("mixed vector widths")
            for k, v in enumerate(s.values):
                if v is None:
                    continue
                if v not in env:
                    raise NoMatch(f"unknown value {v}")
                check_index(s.output, s.index, k, w)
                writes[(s.output, k)] = (env[v], dts[v])
            tensor_dt[s.output] = dtype_name(comp.dtype_of(s.output))
        else:
            raise NoMatch(f"{type(s).__name__} in a pointwise tile")

    if not writes or width is None:
        raise NoMatch("no writes")
    outs = {}
    out_dts = {}
    for (t, k), (sym, vdt) in writes.items():
        canon = shift_components(sym, k)
        if t in outs and outs[t] != canon:
            raise NoMatch("components compute different expressions")
        outs[t] = canon
        out_dts[t] = vdt
    for t in outs:
        if any((t, k) not in writes for k in range(width)):
            raise NoMatch(f"output {t} not written for every component")
    # a value stored to a buffer of another dtype is converted on the way
    # out (compiler.py:1666-1677, 1707-1709)
    final = {}
    for t, sym in outs.items():
        bdt = tensor_dt[t]
        if out_dts[t] != bdt:
            sym = Sym("op", "copy", bdt, (sym,))
        final[t] = sym
    prog = Program.from_outputs(final)
    for s in prog.nodes:
        if s.kind == "in" and s.b != 0:
            raise NoMatch("an element reads a neighbouring element")
    inputs = [t for t in comp.kernel.inputs if t in tensor_dt and t not in final]
    for t in prog.inputs():
        if t not in inputs:
            inputs.append(t)
    return PointwisePlan(n_tile * width, width, prog, tensor_dt, inputs, list(final))


# ----------------------------------------------------------------------------
def _vec_io(b, op, base, off_bytes, dt, regs, load):
    """One group of ``dt`` at ``base + off``: 4 or 8 elements of a 4-byte
    type in one v4 / v8 access, 4 elements of an 8-byte type as two v2."""
    mt = MEM_TYPE[dt]
    sz = nbytes(dt)
    if sz == 4:
        parts = [(0, regs)]
    else:
        parts = [(0, regs[:2]), (16, regs[2:])]
    for delta, rs in parts:
        vec = f"v{len(rs)}"
        addr = f"[{base}+{delta}]" if delta else f"[{base}]"
        if load:
            b.ins(f"ld.global.nc.{vec}.{mt} {{{', '.join(rs)}}}, {addr};")
        else:
            b.ins(f"st.global.{vec}.{mt} {addr}, {{{', '.join(rs)}}};")


def emit(comp, plan: PointwisePlan):
    b = KernelBuilder(comp.entry, comp.target, comp.ptx_version)
    block = launch_block(comp) or 256
    ptrs = declare_params(b, comp)
    ops = Ops(b, getattr(comp, "int_semantics", "reference"))
    prog = plan.program
    n = plan.n_elems
    # 32-byte groups (ld/st .v8, PTX ISA 8.8) when every tensor has 4-byte
    # elements and the element program is small, with half the unroll: the
    # same bytes in flight per thread in half the instructions
    gw = GROUP
    if wide_vectors(comp.ptx_version) and prog.op_count() <= 24 and \
            all(nbytes(plan.dtypes[t]) == 4 for t in plan.inputs + plan.outputs):
        gw = 2 * GROUP
    ngroups = n // gw
    tail = n - ngroups * gw
    U = 4 if prog.op_count() <= 24 else 2
    U = max(1, U * GROUP // gw)

    # hoisted constants (defined before every loop that uses them)
    for s in prog.nodes:
        if s.kind == "const":
            ops.const(s.a, s.b)
    leaves_param = {Sym("param", p): (ptrs[p], dtype_name(comp.args.get(p, {}).get("dtype", "f32")))
                    for p in prog.params()}

    tid, cta, ntid, ncta, gid, stride, g = b.regs("r", 7)
    b.ins(f"mov.u32 {tid}, %tid.x;")
    b.ins(f"mov.u32 {cta}, %ctaid.x;")
    b.ins(f"mov.u32 {ntid}, %ntid.x;")
    b.ins(f"mov.u32 {ncta}, %nctaid.x;")
    b.ins(f"mad.lo.u32 {gid}, {cta}, {ntid}, {tid};")
    b.ins(f"mul.lo.u32 {stride}, {ncta}, {ntid};")
    b.ins(f"mov.u32 {g}, {gid};")

    def body(units):
        """Load, compute and store len(units) groups at group indices
        ``units`` (registers)."""
        loaded = []
        addrs = {}
        for ui, gi in enumerate(units):
            for t in plan.inputs + plan.outputs:
                off = b.reg("rd")
                b.ins(f"mul.wide.u32 {off}, {gi}, {gw * nbytes(plan.dtypes[t])};")
                a = b.reg("rd")
                b.ins(f"add.s64 {a}, {ptrs[t]}, {off};")
                addrs[(ui, t)] = a
        for ui in range(len(units)):
            leaves = dict(leaves_param)
            regs_by_t = {}
            for t in plan.inputs:
                dt = plan.dtypes[t]
                rs = [b.reg_for(dt) for _ in range(gw)]
                _vec_io(b, "ld", addrs[(ui, t)], 0, dt, rs, load=True)
                regs_by_t[t] = rs
            loaded.append(regs_by_t)
        for ui in range(len(units)):
            outs = {t: [] for t in plan.outputs}
            for e in range(gw):
                leaves = dict(leaves_param)
                for t in plan.inputs:
                    leaves[Sym("in", t, 0)] = (loaded[ui][t][e], plan.dtypes[t])
                vals = emit_program(ops, prog, leaves)
                for t in plan.outputs:
                    reg, vdt = vals[prog.outputs[t]]
                    if vdt != plan.dtypes[t]:
                        reg = ops.coerce((reg, vdt), plan.dtypes[t])
                    outs[t].append(reg)
            for t in plan.outputs:
                _vec_io(b, "st", addrs[(ui, t)], 0, plan.dtypes[t], outs[t], load=False)

    main, rem, rem_end = b.label("MAIN"), b.label("REM"), b.label("REM_END")
    p = b.reg("p")
    if U > 1 and ngroups:
        last = b.reg("r")
        b.place(main)
        b.ins(f"mad.lo.u32 {last}, {stride}, {U - 1}, {g};")
        b.ins(f"setp.ge.u32 {p}, {last}, {ngroups};")
        b.ins(f"@{p} bra {rem};")
        units = [g]
        for u in range(1, U):
            gu = b.reg("r")
            b.ins(f"mad.lo.u32 {gu}, {stride}, {u}, {g};")
            units.append(gu)
        body(units)
        b.ins(f"mad.lo.u32 {g}, {stride}, {U}, {g};")
        b.ins(f"bra.uni {main};")
    if ngroups:
        b.place(rem)
        b.ins(f"setp.ge.u32 {p}, {g}, {ngroups};")
        b.ins(f"@{p} bra {rem_end};")
        body([g])
        b.ins(f"add.u32 {g}, {g}, {stride};")
        b.ins(f"bra.uni {rem};")
        b.place(rem_end)
    if tail:
        done = b.label("TAIL_END")
        b.ins(f"setp.ge.u32 {p}, {gid}, {tail};")
        b.ins(f"@{p} bra {done};")
        e = b.reg("r")
        b.ins(f"add.u32 {e}, {gid}, {ngroups * gw};")
        leaves = dict(leaves_param)
        addrs = {}
        for t in plan.inputs + plan.outputs:
            off, a = b.reg("rd"), b.reg("rd")
            b.ins(f"mul.wide.u32 {off}, {e}, {nbytes(plan.dtypes[t])};")
            b.ins(f"add.s64 {a}, {ptrs[t]}, {off};")
            addrs[t] = a
        for t in plan.inputs:
            dt = plan.dtypes[t]
            r = b.reg_for(dt)
            b.ins(f"ld.global.nc.{MEM_TYPE[dt]} {r}, [{addrs[t]}];")
            leaves[Sym("in", t, 0)] = (r, dt)
        vals = emit_program(ops, prog, leaves)
        for t in plan.outputs:
            reg, vdt = vals[prog.outputs[t]]
            if vdt != plan.dtypes[t]:
                reg = ops.coerce((reg, vdt), plan.dtypes[t])
            b.ins(f"st.global.{MEM_TYPE[plan.dtypes[t]]} [{addrs[t]}], {reg};")
        b.place(done)

    per_thread = U * gw
    grid = max(1, -(-n // (per_thread * block)))
    sidecar = {
        "category": "pointwise",
        "grid": [grid, 1, 1],
        "block": [block, 1, 1],
        "shared_bytes": 0,
        "cluster": [1, 1, 1],
        "algorithmic_bytes": sum(n * nbytes(plan.dtypes[t]) for t in plan.inputs + plan.outputs),
        "unroll": U,
        "vector_bytes": gw * 4 if gw > GROUP else 16,
    }
    return b.render(), sidecar
