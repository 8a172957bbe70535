"""Row category: fused row reductions + row maps (RMSNorm, softmax, row sums).

Recognised IR (the reference's cooperative row pattern): a Tile over
``(r, t)`` with ``t`` the thread-in-block axis (extent = threads per block);
strided column loops ``for c = t; c < C/w; c += T`` whose bodies load
``x[r, c*w + k]`` (row tensors) and ``v[c*w + k]`` (row-broadcast vectors)
and accumulate (``Accum``) per-element expressions; after each reducing
loop the cross-thread combine the reference lowers with a warp butterfly
and a shared-memory tree (WarpShuffle / lane-0 smem Write / Sync /
TreeHalve, compiler.py:1877-2006), using the accumulator's own operator;
scalar Let/Assign on the reduced values; and finally either a strided
column loop writing ``out[r, c*w + k]`` or a ``t == 0`` write of a per-row
scalar ``out[r]``.

The semantics extracted are: for each reduction j, ``R_j = op_j over c of
e_j(x[r, c], v[c], R_<j)``; then ``out[r, c] = f(x[r, c], v[c], R)`` or
``out[r] = g(R)``.

Generated kernel (sm_100a): a block per row, persistent over rows; every
thread keeps its share of the row in registers (16-byte vector loads,
issued before any arithmetic) so the row is read from HBM exactly once, all
reductions run on-chip (``shfl.sync.bfly`` butterflies, ``redux.sync`` for
32-bit integers, one shared-memory slot per warp), and outputs are written
with 16-byte stores.  The reference reads the row once per loop (3x for
softmax, 2x for RMSNorm).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .. import ir as I
from .common import (NoMatch, Program, Sym, declare_params, emit_program, flat_affine,
                     launch_block, literal_sym, nbytes, prod, shift_components,
                     const_value)
from .ops import Ops, dtype_name, is_float
from .pointwise import result_dtype
from .ptx import KernelBuilder, MEM_TYPE, f32_hex, f64_hex, wide_vectors
from .tc import TC

# Accum operator -> (combine op for the element-program emitter)
_RED_OPS = {"sum": "add", "add": "add", "prod": "multiply", "multiply": "multiply",
            "max": "max", "amax": "max", "maximum": "max",
            "min": "min", "amin": "min", "minimum": "min"}
_IDENT = {"add": 0.0, "multiply": 1.0, "max": float("-inf"), "min": float("inf")}
_INT_IDENT = {"add": 0, "multiply": 1, "max": -2**31, "min": 2**31 - 1}

MAX_REG_GROUPS = 16          # 16-byte groups per thread kept in registers
PREFETCH_MIN_GROUPS = 8      # rows this large stream the next row into smem
PREFETCH_MAX_BYTES = 192 * 1024
PREFETCH_PIECES = 16
PERSISTENT_BLOCKS = 148      # one block per SM (B200)


@dataclass
class Reduction:
    op: str                  # add / multiply / max / min
    dtype: str
    expr: Sym                # element expression (components shifted to 0)


@dataclass
class RowPlan:
    rows: int
    cols: int
    threads: int
    width: int                       # IR vector width w
    row_tensors: list                # [R, C] inputs
    vec_tensors: list                # [C] inputs
    reductions: list                 # [Reduction]
    row_outputs: dict = field(default_factory=dict)     # name -> Sym (element)
    scalar_outputs: dict = field(default_factory=dict)  # name -> Sym (per row)
    dtypes: dict = field(default_factory=dict)


class _Env:
    def __init__(self):
        self.sym = {}
        self.dt = {}
        self.consts = {}


def _red_op(op):
    name = getattr(op, "name", str(op))
    r = _RED_OPS.get(name)
    if r is None:
        raise NoMatch(f"unsupported accumulator op {name}")
    return r


def match(comp) -> RowPlan:
    body = comp.kernel.body
    if len(body) != 1 or not isinstance(body[0], I.Tile):
        raise NoMatch("not a single Tile")
    tile = body[0]
    if len(tile.axes) != 2 or tile.aux_threads:
        raise NoMatch("row tiles have exactly (row, thread) axes")
    r_ax, t_ax = tile.axes
    if not (r_ax.extent.is_static and t_ax.extent.is_static):
        raise NoMatch("dynamic axes")
    R, T = int(r_ax.extent.as_static()), int(t_ax.extent.as_static())
    block = launch_block(comp) or int(tile.block_threads or T)
    if tile.block_threads and int(tile.block_threads) != T:
        raise NoMatch("thread axis does not match block_threads")
    if block != T:
        raise NoMatch(f"meta.json block ({block}) != thread axis extent ({T})")
    if T % 32 or T > 1024:
        raise NoMatch("threads per row must be a multiple of 32 and at most 1024")
    rv, tv = r_ax.name, t_ax.name
    env = _Env()
    env.dt[tv] = "s32"
    plan = RowPlan(R, 0, T, 0, [], [], [])
    red_of = {}          # accumulator name -> reduction index
    pending = []         # accumulators waiting for their cross-thread combine
    stmts = list(tile.body)
    i = 0

    def loop_columns(loop):
        if not isinstance(loop.start, I.Var) or loop.start.name != tv:
            raise NoMatch("column loop does not start at the thread index")
        step = const_value(loop.step, env.consts)
        if step != T:
            raise NoMatch("column loop step is not the block size")
        if loop.end is not None:
            raise NoMatch("column loop with an explicit end")
        if not loop.axis.extent.is_static:
            raise NoMatch("dynamic column loop")
        return int(loop.axis.extent.as_static())

    def load_syms(s, cvar, n_groups):
        dt = dtype_name(s.dtype) if s.dtype is not None else comp.dtype_of(s.input)
        if dt != comp.dtype_of(s.input) or s.input in comp.smem_names:
            raise NoMatch("load type differs from buffer type")
        shape = comp.shape_of(s.input)
        w = len(s.names)
        if plan.width and w != plan.width:
            raise NoMatch("mixed vector widths")
        plan.width = w
        cols = n_groups * w
        if plan.cols and plan.cols != cols:
            raise NoMatch("column loops disagree on the row length")
        plan.cols = cols
        for k, nm in enumerate(s.names):
            idx = list(s.index)
            if k:
                idx[-1] = I.BinaryExpr("+", idx[-1], I.Literal(k, "int"))
            fa = flat_affine(shape, tuple(idx), env.consts)
            if fa is None:
                raise NoMatch(f"non-affine index into {s.input}")
            coef = {key: v for key, v in fa.items() if key is not None}
            if shape == [R, cols] and coef == {rv: cols, cvar: w} and fa[None] == k:
                if s.input not in plan.row_tensors:
                    plan.row_tensors.append(s.input)
                env.sym[nm] = Sym("in", s.input, k)
            elif shape == [cols] and coef == {cvar: w} and fa[None] == k:
                if s.input not in plan.vec_tensors:
                    plan.vec_tensors.append(s.input)
                env.sym[nm] = Sym("vec", s.input, k)
            else:
                raise NoMatch(f"{s.input} is not indexed as a row or a column vector")
            env.dt[nm] = dt
            plan.dtypes[s.input] = dt

    def element_stmt(s, loop_vars):
        if isinstance(s, I.Let):
            _let(s)
        elif isinstance(s, I.Assign):
            _assign(s)
        else:
            raise NoMatch(f"{type(s).__name__} in a column loop")

    def _let(s):
        v = s.value
        if isinstance(v, I.Literal):
            sym = literal_sym(v)
        elif isinstance(v, I.Var) and v.name in env.sym:
            sym = env.sym[v.name]
        else:
            c = const_value(v, env.consts)
            if c is None:
                raise NoMatch("Let of a non-constant expression")
            sym = Sym("const", int(c), "s32")
        env.sym[s.name] = sym
        dt = dtype_name(s.dtype) if s.dtype is not None else (
            sym.b if sym.kind == "const" else env.dt[v.name])
        env.dt[s.name] = dt
        if sym.kind == "const" and sym.b == "s32":
            env.consts[s.name] = sym.a

    def _assign(s):
        for a in s.args:
            if a not in env.sym:
                raise NoMatch(f"unknown value {a}")
        dt = dtype_name(s.dtype) if s.dtype is not None else env.dt[s.args[0]]
        opname = getattr(s.op, "name", str(s.op))
        env.sym[s.name] = Sym("op", opname, dt, tuple(env.sym[a] for a in s.args))
        env.dt[s.name] = result_dtype(opname, [env.dt[a] for a in s.args], dt)

    while i < len(stmts):
        s = stmts[i]
        if isinstance(s, I.Smem):
            i += 1
            continue
        if isinstance(s, I.StridedLoop) and s.seed:
            ngroups = loop_columns(s)
            cvar = s.axis.name
            accs = {}
            for st in s.body:
                if isinstance(st, I.Load):
                    load_syms(st, cvar, ngroups)
                elif isinstance(st, I.Accum):
                    if st.base is not None or st.value not in env.sym:
                        raise NoMatch("accumulator update is not acc op= value")
                    op = _red_op(st.op)
                    dt = dtype_name(st.dtype) if st.dtype is not None else "f32"
                    val = env.sym[st.value]
                    comps = [x.b for x in _leaves(val) if x.kind in ("in", "vec")]
                    k = comps[0] if comps else 0
                    canon = shift_components(val, k)
                    prev = accs.get(st.name)
                    if prev is None:
                        accs[st.name] = (op, dt, canon)
                    elif prev != (op, dt, canon):
                        raise NoMatch("accumulator updates differ between components")
                else:
                    element_stmt(st, {cvar})
            if not accs:
                raise NoMatch("seeded column loop without accumulators")
            for name, (op, dt, canon) in accs.items():
                red_of[name] = len(plan.reductions)
                plan.reductions.append(Reduction(op, dt, canon))
                pending.append(name)
            i += 1
            continue
        if isinstance(s, (I.WarpShuffle, I.TreeHalve)):
            for st_name in s.state:
                if st_name not in pending and st_name not in red_of:
                    raise NoMatch("cross-thread combine of a non-accumulator")
            for c in s.combine_states:
                if not isinstance(c, I.Accum) or c.name not in red_of:
                    raise NoMatch("combine step is not an accumulator update")
                if _red_op(c.op) != plan.reductions[red_of[c.name]].op:
                    raise NoMatch("combine operator differs from the accumulator's")
            if isinstance(s, I.TreeHalve):
                for st_name in s.state:
                    if st_name in pending:
                        pending.remove(st_name)
                        env.sym[st_name] = Sym("red", red_of[st_name])
                        env.dt[st_name] = plan.reductions[red_of[st_name]].dtype
            i += 1
            continue
        if isinstance(s, I.Sync):
            i += 1
            continue
        if isinstance(s, I.Cond):
            # lane-0 staging write of a pending accumulator, or a t==0 write
            # of per-row scalars
            writes = [w for w in s.body if isinstance(w, I.Write)]
            if s.else_body or len(writes) != len(s.body) or not writes:
                raise NoMatch("unsupported Cond in a row kernel")
            if all(w.output in comp.smem_names for w in writes):
                if any(v not in pending for w in writes for v in w.values):
                    raise NoMatch("staging write of a non-accumulator")
                i += 1
                continue
            cond_ok = (isinstance(s.cond, I.BinaryExpr) and s.cond.op == "=="
                       and isinstance(s.cond.left, I.Var) and s.cond.left.name == tv
                       and const_value(s.cond.right) == 0)
            if not cond_ok:
                raise NoMatch("per-row write not guarded by t == 0")
            for w in writes:
                if len(w.values) != 1 or w.atomic:
                    raise NoMatch("per-row write of several values")
                shape = comp.shape_of(w.output)
                fa = flat_affine(shape, tuple(w.index), env.consts)
                if shape != [R] or fa != {None: 0, rv: 1}:
                    raise NoMatch("per-row output is not out[r]")
                v = w.values[0]
                if v not in env.sym or v in pending:
                    raise NoMatch("per-row output of an unreduced value")
                plan.scalar_outputs[w.output] = env.sym[v]
                plan.dtypes[w.output] = comp.dtype_of(w.output)
            i += 1
            continue
        if isinstance(s, (I.Let, I.Assign)):
            element_stmt(s, set())
            i += 1
            continue
        if isinstance(s, I.StridedLoop) and not s.seed:
            ngroups = loop_columns(s)
            cvar = s.axis.name
            outs = {}
            for st in s.body:
                if isinstance(st, I.Load):
                    load_syms(st, cvar, ngroups)
                elif isinstance(st, I.Write):
                    shape = comp.shape_of(st.output)
                    w = len(st.values)
                    if st.atomic or w != plan.width:
                        raise NoMatch("row output write")
                    for k, v in enumerate(st.values):
                        idx = list(st.index)
                        if k:
                            idx[-1] = I.BinaryExpr("+", idx[-1], I.Literal(k, "int"))
                        fa = flat_affine(shape, tuple(idx), env.consts)
                        if fa is None or shape != [R, plan.cols] or \
                                {a: b for a, b in fa.items() if a is not None} != {rv: plan.cols, cvar: w} \
                                or fa[None] != k:
                            raise NoMatch(f"{st.output} is not written as out[r, c]")
                        if v not in env.sym:
                            raise NoMatch(f"unknown value {v}")
                        canon = shift_components(env.sym[v], k)
                        bdt = comp.dtype_of(st.output)
                        if env.dt[v] != bdt:
                            canon = Sym("op", "copy", bdt, (canon,))
                        if st.output in outs and outs[st.output] != canon:
                            raise NoMatch("output components compute different expressions")
                        outs[st.output] = canon
                    plan.dtypes[st.output] = comp.dtype_of(st.output)
                else:
                    element_stmt(st, {cvar})
            plan.row_outputs.update(outs)
            i += 1
            continue
        raise NoMatch(f"{type(s).__name__} in a row kernel")

    if pending:
        raise NoMatch("accumulators used without a cross-thread combine")
    if not plan.reductions or not (plan.row_outputs or plan.scalar_outputs):
        raise NoMatch("no reduction or no output")
    for s in _all_syms(plan):
        if s.kind == "in" and s.b != 0 or s.kind == "vec" and s.b != 0:
            raise NoMatch("an element reads a neighbouring element")
    return plan


def _leaves(s, out=None):
    if out is None:
        out = []
    if s.kind == "op":
        for a in s.args:
            _leaves(a, out)
    else:
        out.append(s)
    return out


def _all_syms(plan):
    roots = [r.expr for r in plan.reductions] + list(plan.row_outputs.values()) + \
        list(plan.scalar_outputs.values())
    seen = []
    for r in roots:
        seen.extend(Program.from_outputs({"_": r}).nodes)
    return seen


# ----------------------------------------------------------------------------
# emission
# ----------------------------------------------------------------------------
def _combine(b, op, dt, acc, other):
    """acc = acc op other (in place)."""
    if op == "add":
        ins = {"f32": "add.f32", "f64": "add.f64", "s32": "add.s32"}[dt]
    elif op == "multiply":
        ins = {"f32": "mul.f32", "f64": "mul.f64", "s32": "mul.lo.s32"}[dt]
    elif op == "max":
        ins = {"f32": "max.f32", "f64": "max.f64", "s32": "max.s32"}[dt]
    else:
        ins = {"f32": "min.f32", "f64": "min.f64", "s32": "min.s32"}[dt]
    b.ins(f"{ins} {acc}, {acc}, {other};")


def _identity(ops, op, dt):
    if is_float(dt):
        return ops.const(_IDENT[op], dt)[0]
    return ops.const(_INT_IDENT[op], "s32")[0]


def _warp_allreduce(b, op, dt, acc):
    """Butterfly all-reduce over the 32 lanes (every lane gets the total)."""
    if dt == "s32" and op in ("add", "max", "min"):
        b.ins(f"redux.sync.{op}.s32 {acc}, {acc}, 0xffffffff;")
        return
    for step in (16, 8, 4, 2, 1):
        if dt == "f64":
            lo, hi, lo2, hi2 = b.regs("r", 4)
            o = b.reg("fd")
            b.ins(f"mov.b64 {{{lo}, {hi}}}, {acc};")
            b.ins(f"shfl.sync.bfly.b32 {lo2}, {lo}, {step}, 0x1f, 0xffffffff;")
            b.ins(f"shfl.sync.bfly.b32 {hi2}, {hi}, {step}, 0x1f, 0xffffffff;")
            b.ins(f"mov.b64 {o}, {{{lo2}, {hi2}}};")
        else:
            o = b.reg_for(dt)
            b.ins(f"shfl.sync.bfly.b32 {o}, {acc}, {step}, 0x1f, 0xffffffff;")
        _combine(b, op, dt, acc, o)


def emit(comp, plan: RowPlan, gather: int = 0):
    """``gather`` > 0: the all-gather variant for a row shard.  Instead of
    writing ``out``, every output row is stored into up to ``gather``
    full-size output buffers (this rank's and its peers', over NVLink) at
    row ``emmy_gather_row0 + row``; the module globals ``emmy_gather_dst``
    (``gather`` u64 pointers), ``emmy_gather_n`` (how many are used) and
    ``emmy_gather_row0`` are set by the host before the first launch.
    Plain stores only: no multicast, no waits on another GPU."""
    if gather and (len(plan.row_outputs) != 1 or plan.scalar_outputs):
        raise ValueError("the gather variant needs exactly one row output")
    b = KernelBuilder(comp.entry, comp.target, comp.ptx_version)
    T = plan.threads
    nw = T // 32
    ptrs = declare_params(b, comp)
    ops = Ops(b, getattr(comp, "int_semantics", "reference"))
    C = plan.cols
    # elements per vector: 8 (32-byte loads and stores, PTX ISA 8.8) when
    # every row tensor has 4-byte elements and the row splits evenly into
    # 8-element vectors across the block; else 4, or 1 for odd widths.
    # 32-byte accesses took the full-size softmax from 371 to 349 us.
    elem4 = all(nbytes(plan.dtypes[t]) == 4
                for t in plan.row_tensors + plan.vec_tensors + list(plan.row_outputs))
    if wide_vectors(comp.ptx_version) and elem4 and C % (8 * T) == 0:
        V = 8
    else:
        V = 4 if C % 4 == 0 else 1
    nvec = C // V                     # vectors per row
    G = -(-nvec // T)                 # vectors per thread
    units = G * V // 4 if V >= 4 else G          # 16-byte units per thread
    if units > MAX_REG_GROUPS:
        raise NoMatch(f"row of {C} elements does not fit in registers "
                      f"({G} vectors per thread)")
    ragged = nvec % T != 0
    # Large rows (one block per SM at this register footprint) are streamed:
    # while a row is reduced in registers, the next row arrives in shared
    # memory through cp.async.bulk, so loads are always in flight.  (Sharing
    # a row between the CTAs of a cluster, to fit more CTAs per SM, measured
    # slower: the per-row cluster barriers cost more than it gains.)
    row_bytes = C * sum(nbytes(plan.dtypes[t]) for t in plan.row_tensors)
    prefetch = (units >= PREFETCH_MIN_GROUPS and len(plan.row_tensors) == 1 and not ragged
                and V in (4, 8) and row_bytes <= PREFETCH_MAX_BYTES)

    b.directive(f".maxntid {T}, 1, 1")
    # all constants up front
    progs = [Program.from_outputs({"_": r.expr}) for r in plan.reductions]
    out_prog = Program.from_outputs(dict(plan.row_outputs)) if plan.row_outputs else None
    sc_prog = Program.from_outputs(dict(plan.scalar_outputs)) if plan.scalar_outputs else None
    for pr in progs + [p for p in (out_prog, sc_prog) if p]:
        for s in pr.nodes:
            if s.kind == "const":
                ops.const(s.a, s.b)
    for r in plan.reductions:
        _identity(ops, r.op, r.dtype)

    # shared memory: one slot per warp, per reduction, per row parity
    slot_bytes = 8
    nred = len(plan.reductions)
    b.module(f".shared .align 16 .b8 red_slots[{2 * nred * nw * slot_bytes}];")
    if gather:
        b.module(f".global .align 8 .b8 emmy_gather_dst[{8 * gather}];")
        b.module(".global .align 4 .u32 emmy_gather_n;")
        b.module(".global .align 4 .u32 emmy_gather_row0;")
    if prefetch:
        b.module(".shared .align 8 .b8 row_bar[8];")
        b.module(".shared .align 4 .u32 row_abort;")
        b.module(".extern .shared .align 128 .b8 row_buf[];")

    tid, cta, ncta, lane, warp = b.regs("r", 5)
    b.ins(f"mov.u32 {tid}, %tid.x;")
    b.ins(f"mov.u32 {cta}, %ctaid.x;")
    b.ins(f"mov.u32 {ncta}, %nctaid.x;")
    b.ins(f"and.b32 {lane}, {tid}, 31;")
    b.ins(f"shr.u32 {warp}, {tid}, 5;")
    sbase = b.reg("r")
    b.ins(f"mov.u32 {sbase}, red_slots;")

    # per-thread vector validity (ragged rows)
    valid = []
    for g in range(G):
        if ragged and (g + 1) * T > nvec:
            p = b.reg("p")
            b.ins(f"setp.lt.u32 {p}, {tid}, {nvec - g * T};")
            valid.append(p)
        else:
            valid.append(None)

    def addr_of(base, g, elem_bytes, row_off=None):
        """Address of this thread's vector g (columns (tid + g*T)*V ...)."""
        off = b.reg("rd")
        b.ins(f"mul.wide.u32 {off}, {tid}, {V * elem_bytes};")
        a = b.reg("rd")
        b.ins(f"add.s64 {a}, {base}, {off};")
        if g:
            b.ins(f"add.s64 {a}, {a}, {g * T * V * elem_bytes};")
        if row_off is not None:
            b.ins(f"add.s64 {a}, {a}, {row_off};")
        return a

    def vec_io(addr, dt, regs, load, pred, nc=True):
        mt = MEM_TYPE[dt]
        guard = f"@{pred} " if pred else ""
        sz = nbytes(dt)
        if V == 1:
            if load:
                b.ins(f"{guard}ld.global{'.nc' if nc else ''}.{mt} {regs[0]}, [{addr}];")
            else:
                b.ins(f"{guard}st.global.{mt} [{addr}], {regs[0]};")
            return
        parts = [(0, regs)] if sz == 4 else [(0, regs[:2]), (16, regs[2:])]
        for delta, rs in parts:
            a = f"[{addr}+{delta}]" if delta else f"[{addr}]"
            if load:
                b.ins(f"{guard}ld.global{'.nc' if nc else ''}.v{len(rs)}.{mt} {{{', '.join(rs)}}}, {a};")
            else:
                b.ins(f"{guard}st.global.v{len(rs)}.{mt} {a}, {{{', '.join(rs)}}};")

    gdst, gpred, grow0 = [], [], None
    if gather:
        gn = b.reg("r")
        grow0 = b.reg("r")
        b.ins(f"ld.global.u32 {gn}, [emmy_gather_n];")
        b.ins(f"ld.global.u32 {grow0}, [emmy_gather_row0];")
        for d in range(gather):
            gd, pd = b.reg("rd"), b.reg("p")
            b.ins(f"ld.global.u64 {gd}, [emmy_gather_dst+{8 * d}];")
            b.ins(f"setp.lt.u32 {pd}, {d}, {gn};")
            gdst.append(gd)
            gpred.append(pd)

    # broadcast vectors: loaded once, before the row loop
    vec_regs = {}
    for t in plan.vec_tensors:
        dt = plan.dtypes[t]
        vec_regs[t] = []
        for g in range(G):
            rs = [b.reg_for(dt) for _ in range(V)]
            if valid[g]:
                for r_ in rs:
                    b.ins(f"mov.{'f32' if dt == 'f32' else 'f64' if dt == 'f64' else 'b32'} {r_}, "
                          f"{f32_hex(0) if dt == 'f32' else f64_hex(0) if dt == 'f64' else 0};")
            vec_io(addr_of(ptrs[t], g, nbytes(dt)), dt, rs, True, valid[g])
            vec_regs[t].append(rs)

    if prefetch:
        rt_ = plan.row_tensors[0]
        rbar, rabort, rbuf = b.regs("r", 3)
        b.ins(f"mov.u32 {rbar}, row_bar;")
        b.ins(f"mov.u32 {rabort}, row_abort;")
        b.ins(f"mov.u32 {rbuf}, row_buf;")
        tc = TC(b, rabort)
        p0 = b.reg("p")
        b.ins(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip0 = b.label("PF_INIT")
        b.ins(f"@!{p0} bra {skip0};")
        tc.init(rbar, 1)
        b.ins(f"st.shared.u32 [{rabort}], 0;")
        b.ins("fence.mbarrier_init.release.cluster;")
        b.place(skip0)
        b.ins(f"bar.sync 2, {T};")

        # the row buffer is refilled piece by piece: piece k (groups
        # [k*G/npc, (k+1)*G/npc), contiguous in the row) of the next row is
        # requested as soon as every thread has piece k of this row in
        # registers, so the next row's reads overlap this row's smem reads
        npc = max(d for d in range(1, min(PREFETCH_PIECES, G) + 1) if G % d == 0)
        piece = row_bytes // npc

        def issue_head(r_reg):
            """Thread 0: arm the row barrier for row ``r_reg``; returns the
            predicate "thread 0 and the row exists" and the row's address."""
            pp, pi = b.regs("p", 2)
            b.ins(f"setp.lt.u32 {pp}, {r_reg}, {plan.rows};")
            b.ins(f"and.pred {pi}, {pp}, {p0};")
            src = b.reg("rd")
            b.ins(f"mul.wide.u32 {src}, {r_reg}, {row_bytes};")
            b.ins(f"add.s64 {src}, {src}, {ptrs[rt_]};")
            sk = b.label("PF_ARM")
            b.ins(f"@!{pi} bra {sk};")
            b.ins("fence.proxy.async.shared::cta;")
            tc.arrive_expect_tx(rbar, row_bytes)
            b.place(sk)
            return pi, src

        def issue_piece(pi, src, k):
            b.ins(f"@{pi} cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
                  f"[{rbuf}+{k * piece}], [{src}+{k * piece}], {piece}, [{rbar}];")

        pi0, src0 = issue_head(cta)
        for k in range(npc):
            issue_piece(pi0, src0, k)
        pf_it = b.reg("r")
        b.ins(f"mov.u32 {pf_it}, 0;")

    row, parity = b.regs("r", 2)
    b.ins(f"mov.u32 {row}, {cta};")
    b.ins(f"mov.u32 {parity}, 0;")
    top, done = b.label("ROW"), b.label("ROW_END")
    pdone = b.reg("p")
    b.place(top)
    b.ins(f"setp.ge.u32 {pdone}, {row}, {plan.rows};")
    b.ins(f"@{pdone} bra {done};")

    row_off = {}
    for t in plan.row_tensors + list(plan.row_outputs):
        o = b.reg("rd")
        b.ins(f"mul.wide.u32 {o}, {row}, {C * nbytes(plan.dtypes[t])};")
        row_off[t] = o
    gather_off = {}
    if gather:
        grow = b.reg("r")
        b.ins(f"add.u32 {grow}, {grow0}, {row};")
        for t in plan.row_outputs:
            o = b.reg("rd")
            b.ins(f"mul.wide.u32 {o}, {grow}, {C * nbytes(plan.dtypes[t])};")
            gather_off[t] = o
    x_regs = {}
    if prefetch:
        dt = plan.dtypes[rt_]
        par = b.reg("r")
        b.ins(f"and.b32 {par}, {pf_it}, 1;")
        tc.wait(rbar, par, done, role=9, uniform=True)
        sa = b.reg("r")
        b.ins(f"mad.lo.u32 {sa}, {tid}, {V * nbytes(dt)}, {rbuf};")
        nxt = b.reg("r")
        b.ins(f"add.u32 {nxt}, {row}, {ncta};")
        pin, srcn = issue_head(nxt)
        x_regs[rt_] = []
        per = G // npc
        for k in range(npc):
            for g in range(k * per, (k + 1) * per):
                rs = [b.reg_for(dt) for _ in range(V)]
                for h in range(V // 4):
                    b.ins(f"ld.shared.v4.{MEM_TYPE[dt]} {{{', '.join(rs[4 * h:4 * h + 4])}}}, "
                          f"[{sa}+{g * T * V * nbytes(dt) + 16 * h}];")
                x_regs[rt_].append(rs)
            # every thread has piece k in registers: refill it with the next row's
            b.ins(f"bar.sync 2, {T};")
            issue_piece(pin, srcn, k)
        b.ins(f"add.u32 {pf_it}, {pf_it}, 1;")
    for t in plan.row_tensors:
        if prefetch:
            continue
        dt = plan.dtypes[t]
        x_regs[t] = []
        for g in range(G):
            rs = [b.reg_for(dt) for _ in range(V)]
            vec_io(addr_of(ptrs[t], g, nbytes(dt), row_off[t]), dt, rs, True, valid[g])
            x_regs[t].append(rs)

    def element_leaves(g, e):
        lv = {}
        for t in plan.row_tensors:
            lv[Sym("in", t, 0)] = (x_regs[t][g][e], plan.dtypes[t])
        for t in plan.vec_tensors:
            lv[Sym("vec", t, 0)] = (vec_regs[t][g][e], plan.dtypes[t])
        return lv

    def is_row_scalar(sym, memo={}):
        if sym not in memo:
            if sym.kind in ("in", "vec"):
                memo[sym] = False
            elif sym.kind == "op":
                memo[sym] = all(is_row_scalar(a) for a in sym.args)
            else:
                memo[sym] = True
        return memo[sym]

    def hoist_scalars(prog_list, known):
        """Emit, once per row, every node that depends only on reductions,
        constants and parameters."""
        for pr in prog_list:
            for s in pr.nodes:
                if s.kind == "op" and s not in known and is_row_scalar(s) and \
                        all(a in known or a.kind == "const" for a in s.args):
                    args = [known[a] if a in known else ops.const(a.a, a.b) for a in s.args]
                    known[s] = ops.emit(s.a, args, s.b)

    # per-element values of every phase, reused by later phases: the row
    # is in registers, so an expression a later loop recomputes from the
    # same inputs (softmax's exp(x - max) in the sum and in the output) is
    # the same value, computed once
    elem_vals = {}
    reduced = {}
    for j, red in enumerate(plan.reductions):
        hoist_scalars([progs[j]], reduced)
        acc = b.reg_for(red.dtype)
        ident = _identity(ops, red.op, red.dtype)
        b.ins(f"mov.{'f32' if red.dtype == 'f32' else 'f64' if red.dtype == 'f64' else 'b32'} "
              f"{acc}, {ident};")
        for g in range(G):
            skip = None
            if valid[g]:
                skip = b.label("RSKIP")
                b.ins(f"@!{valid[g]} bra {skip};")
            for e in range(V):
                lv = element_leaves(g, e)
                lv.update(elem_vals.get((g, e), {}))
                lv.update(reduced)
                vals = emit_program(ops, progs[j], lv)
                elem_vals[(g, e)] = vals
                reg, vdt = vals[red.expr]
                if vdt != red.dtype:
                    reg = ops.coerce((reg, vdt), red.dtype)
                _combine(b, red.op, red.dtype, acc, reg)
            if skip:
                b.place(skip)
        _warp_allreduce(b, red.op, red.dtype, acc)
        # cross-warp: lane 0 stores, everyone combines all slots
        if nw > 1:
            slot = b.reg("r")
            b.ins(f"mad.lo.u32 {slot}, {parity}, {nred * nw * slot_bytes}, {sbase};")
            if j:
                b.ins(f"add.u32 {slot}, {slot}, {j * nw * slot_bytes};")
            st_addr = b.reg("r")
            b.ins(f"mad.lo.u32 {st_addr}, {warp}, {slot_bytes}, {slot};")
            p0 = b.reg("p")
            b.ins(f"setp.eq.u32 {p0}, {lane}, 0;")
            mt = {"f32": "f32", "f64": "f64"}.get(red.dtype, "s32")
            b.ins(f"@{p0} st.shared.{mt} [{st_addr}], {acc};")
            b.ins(f"bar.sync 1, {T};")
            b.ins(f"ld.shared.{mt} {acc}, [{slot}];")
            for w_ in range(1, nw):
                o = b.reg_for(red.dtype)
                b.ins(f"ld.shared.{mt} {o}, [{slot}+{w_ * slot_bytes}];")
                _combine(b, red.op, red.dtype, acc, o)
        reduced[Sym("red", j)] = (acc, red.dtype)

    hoist_scalars([p for p in (out_prog, sc_prog) if p], reduced)
    if plan.scalar_outputs:
        vals = emit_program(ops, sc_prog, dict(reduced))
        p0 = b.reg("p")
        skipw = b.label("SCALAR_SKIP")
        b.ins(f"setp.ne.u32 {p0}, {tid}, 0;")
        b.ins(f"@{p0} bra {skipw};")
        for t, sym in plan.scalar_outputs.items():
            reg, vdt = vals[sym]
            dt = plan.dtypes[t]
            if vdt != dt:
                reg = ops.coerce((reg, vdt), dt)
            off, a = b.reg("rd"), b.reg("rd")
            b.ins(f"mul.wide.u32 {off}, {row}, {nbytes(dt)};")
            b.ins(f"add.s64 {a}, {ptrs[t]}, {off};")
            b.ins(f"st.global.{MEM_TYPE[dt]} [{a}], {reg};")
        b.place(skipw)

    if plan.row_outputs:
        for g in range(G):
            outs = {t: [] for t in plan.row_outputs}
            for e in range(V):
                lv = element_leaves(g, e)
                lv.update(elem_vals.get((g, e), {}))
                lv.update(reduced)
                vals = emit_program(ops, out_prog, lv)
                for t, sym in plan.row_outputs.items():
                    reg, vdt = vals[sym]
                    if vdt != plan.dtypes[t]:
                        reg = ops.coerce((reg, vdt), plan.dtypes[t])
                    outs[t].append(reg)
            for t in plan.row_outputs:
                dt = plan.dtypes[t]
                if not gather:
                    vec_io(addr_of(ptrs[t], g, nbytes(dt), row_off[t]), dt, outs[t], False,
                           valid[g])
                    continue
                # the same vector into every destination's row row0 + row
                for d in range(gather):
                    pr_ = gpred[d]
                    if valid[g]:
                        pr_ = b.reg("p")
                        b.ins(f"and.pred {pr_}, {gpred[d]}, {valid[g]};")
                    vec_io(addr_of(gdst[d], g, nbytes(dt), gather_off[t]), dt, outs[t], False,
                           pr_)

    b.ins(f"add.u32 {row}, {row}, {ncta};")
    b.ins(f"xor.b32 {parity}, {parity}, 1;")
    b.ins(f"bra.uni {top};")
    b.place(done)

    alg = plan.rows * C * sum(nbytes(plan.dtypes[t]) for t in plan.row_tensors) \
        + C * sum(nbytes(plan.dtypes[t]) for t in plan.vec_tensors) \
        + plan.rows * C * sum(nbytes(plan.dtypes[t]) for t in plan.row_outputs) \
        + plan.rows * sum(nbytes(plan.dtypes[t]) for t in plan.scalar_outputs)
    sidecar = {
        "category": "rows",
        "grid": [min(plan.rows, PERSISTENT_BLOCKS) if prefetch else plan.rows, 1, 1],
        "block": [T, 1, 1],
        "shared_bytes": row_bytes if prefetch else 0,
        "row_prefetch": prefetch,
        "cluster": [1, 1, 1],
        "algorithmic_bytes": alg,
        "vectors_per_thread": G,
    }
    if gather:
        sidecar["gather"] = {"max_destinations": gather, "destinations": "emmy_gather_dst",
                             "count": "emmy_gather_n", "row0": "emmy_gather_row0",
                             "writes_out": False}
    return b.render(), sidecar
