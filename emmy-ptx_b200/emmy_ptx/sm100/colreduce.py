"""Column (segmented / transposed) reductions over dim 0 of a row-major [R, C].

Recognised IR (the reference's "coop-t" pattern, compiler.py:1933-2006): a
Tile over ``(cb, w, l)`` where column ``c = cb*L + l`` (``l`` the lane axis
of extent L) and ``w`` a row group; a seeded row loop ``for rr = w;
rr < R; rr += W`` accumulating per-element expressions of ``x[rr, c]``;
staging writes of the accumulators to shared memory at ``w*L + l``; a
segmented TreeHalve over ``w`` with ``inner=(l, L)`` using each
accumulator's operator; and ``w == 0`` writes ``out_j[c] = acc_j``.

Semantics: ``out_j[c] = op_j over r of e_j(x[r, c])``.

Generated kernel (sm_100a): a column strip of 32 lanes x 16 bytes per block
(64 f64 / 128 f32 columns; one 512-byte segment per row per warp, fully
coalesced), rows split across the S blocks of a thread-block cluster and
interleaved across the warps of each block, four rows in flight per warp.
Partials are combined in shared memory within a block, then across the
cluster through distributed shared memory (``mapa`` +
``ld.shared::cluster``) in a fixed rank order, so the result is
deterministic and needs neither atomics nor scratch memory.  Clusters walk
the column strips persistently, so any grid size is correct.
"""

from __future__ import annotations

from dataclasses import dataclass

from .. import ir as I
from .common import (NoMatch, Program, Sym, declare_params, emit_program, flat_affine,
                     launch_block, literal_sym, nbytes, const_value)
from .ops import Ops, dtype_name, is_float
from .pointwise import result_dtype
from .ptx import KernelBuilder, MEM_TYPE
from .rows import _RED_OPS, _IDENT, _INT_IDENT, _combine

ROWS_IN_FLIGHT = 4


@dataclass
class ColPlan:
    rows: int
    cols: int
    tensor: str
    dtype: str
    reductions: list          # [(op, dtype, Sym)]
    outputs: list             # output tensor per reduction


def _red_op(op):
    name = getattr(op, "name", str(op))
    if name not in _RED_OPS:
        raise NoMatch(f"unsupported accumulator op {name}")
    return _RED_OPS[name]


def match(comp) -> ColPlan:
    body = comp.kernel.body
    if len(body) != 1 or not isinstance(body[0], I.Tile):
        raise NoMatch("not a single Tile")
    tile = body[0]
    if len(tile.axes) != 3 or tile.aux_threads:
        raise NoMatch("column tiles have (column block, row group, lane) axes")
    if not all(a.extent.is_static for a in tile.axes):
        raise NoMatch("dynamic axes")
    cb, wg, ln = tile.axes
    NB, W, L = (int(a.extent.as_static()) for a in tile.axes)
    block = launch_block(comp) or int(tile.block_threads or 0)
    if block != W * L or (tile.block_threads and int(tile.block_threads) != W * L):
        raise NoMatch("block is not (row groups x lanes)")
    env, dts, consts = {}, {}, {}
    accs, order = {}, []
    staged, combined = set(), set()
    outs = {}
    plan_tensor = None
    R = C = None
    for s in tile.body:
        if isinstance(s, (I.Smem, I.Sync)):
            continue
        if isinstance(s, I.StridedLoop) and s.seed:
            if not (isinstance(s.start, I.Var) and s.start.name == wg.name):
                raise NoMatch("row loop does not start at the row group")
            if const_value(s.step, consts) != W or s.end is not None \
                    or not s.axis.extent.is_static:
                raise NoMatch("row loop does not stride by the row groups")
            R = int(s.axis.extent.as_static())
            rr = s.axis.name
            for st in s.body:
                if isinstance(st, I.Load):
                    if len(st.names) != 1:
                        raise NoMatch("grouped loads in a column reduction")
                    shape = comp.shape_of(st.input)
                    dt = dtype_name(st.dtype) if st.dtype is not None else comp.dtype_of(st.input)
                    if dt != comp.dtype_of(st.input) or len(shape) != 2:
                        raise NoMatch("load type or rank")
                    fa = flat_affine(shape, tuple(st.index), consts)
                    if fa != {None: 0, rr: shape[1], cb.name: L, ln.name: 1} or shape[0] != R \
                            or shape[1] != NB * L:
                        raise NoMatch("load is not x[rr, cb*L + l]")
                    if plan_tensor not in (None, st.input):
                        raise NoMatch("two reduced tensors")
                    plan_tensor, C = st.input, shape[1]
                    env[st.names[0]] = Sym("in", st.input, 0)
                    dts[st.names[0]] = dt
                elif isinstance(st, I.Assign):
                    if any(a not in env for a in st.args):
                        raise NoMatch("unknown value")
                    dt = dtype_name(st.dtype) if st.dtype is not None else dts[st.args[0]]
                    name = getattr(st.op, "name", str(st.op))
                    env[st.name] = Sym("op", name, dt, tuple(env[a] for a in st.args))
                    dts[st.name] = result_dtype(name, [dts[a] for a in st.args], dt)
                elif isinstance(st, I.Let) and isinstance(st.value, I.Literal):
                    env[st.name] = literal_sym(st.value)
                    dts[st.name] = env[st.name].b
                elif isinstance(st, I.Accum):
                    if st.base is not None or st.value not in env or st.name in accs:
                        raise NoMatch("accumulator update is not acc op= value")
                    dt = dtype_name(st.dtype) if st.dtype is not None else "f32"
                    accs[st.name] = (_red_op(st.op), dt, env[st.value])
                    order.append(st.name)
                else:
                    raise NoMatch(f"{type(st).__name__} in the row loop")
            continue
        if isinstance(s, I.Write) and s.output in comp.smem_names:
            fa = flat_affine([W * L], tuple(s.index), consts)
            if fa != {None: 0, wg.name: L, ln.name: 1} or len(s.values) != 1 \
                    or s.values[0] not in accs:
                raise NoMatch("staging write is not smem[w*L + l] = acc")
            staged.add(s.values[0])
            continue
        if isinstance(s, I.TreeHalve):
            if s.tid_var != wg.name or s.inner is None or tuple(s.inner) != (ln.name, L) \
                    or int(s.length) != W:
                raise NoMatch("tree is not the segmented tree over the row groups")
            for c in s.combine_states:
                if not isinstance(c, I.Accum) or c.name not in accs or \
                        _red_op(c.op) != accs[c.name][0]:
                    raise NoMatch("tree combine differs from the accumulator")
            combined.update(s.state)
            continue
        if isinstance(s, I.Cond):
            cond_ok = (isinstance(s.cond, I.BinaryExpr) and s.cond.op == "=="
                       and isinstance(s.cond.left, I.Var) and s.cond.left.name == wg.name
                       and const_value(s.cond.right) == 0)
            if not cond_ok or s.else_body:
                raise NoMatch("output writes not guarded by w == 0")
            for w in s.body:
                if not isinstance(w, I.Write) or len(w.values) != 1 or w.atomic:
                    raise NoMatch("unsupported output write")
                fa = flat_affine(comp.shape_of(w.output), tuple(w.index), consts)
                if fa != {None: 0, cb.name: L, ln.name: 1} or comp.shape_of(w.output) != [C]:
                    raise NoMatch("output is not out[cb*L + l]")
                if w.values[0] not in accs or w.values[0] not in combined:
                    raise NoMatch("output of an uncombined value")
                outs[w.output] = w.values[0]
            continue
        raise NoMatch(f"{type(s).__name__} in a column-reduction tile")
    if not outs or plan_tensor is None:
        raise NoMatch("no outputs")
    if set(outs.values()) - staged:
        raise NoMatch("accumulator written without staging")
    reds, out_names = [], []
    for o, a in outs.items():
        op, dt, expr = accs[a]
        if dtype_name(comp.dtype_of(o)) != dt:
            raise NoMatch("output dtype differs from the accumulator")
        reds.append((op, dt, expr))
        out_names.append(o)
    return ColPlan(R, C, plan_tensor, dtype_name(comp.dtype_of(plan_tensor)), reds, out_names)


# ----------------------------------------------------------------------------
def _cluster_size(meta_grid, strips, cap=8):
    """Largest power of two <= cap that divides the meta.json grid (so the
    kernel also launches under the meta geometry)."""
    s = cap
    while s > 1 and (meta_grid % s):
        s //= 2
    return s


def emit(comp, plan: ColPlan):
    b = KernelBuilder(comp.entry, comp.target, comp.ptx_version)
    T = launch_block(comp)
    NW = T // 32
    dt = plan.dtype
    esz = nbytes(dt)
    VL = 16 // esz if plan.cols % (32 * (16 // esz)) == 0 else 1
    CW = 32 * VL
    strips = -(-plan.cols // CW)
    meta_grid = 1
    for g in (comp.kmeta.get("grid") or [1]):
        meta_grid *= int(g)
    S = _cluster_size(meta_grid, strips)
    RS = -(-plan.rows // S)                    # rows per cluster rank
    nred = len(plan.reductions)
    b.directive(f".maxntid {T}, 1, 1")
    if S > 1:
        b.directive(f".reqnctapercluster {S}, 1, 1")
    ptrs = declare_params(b, comp)
    ops = Ops(b, getattr(comp, "int_semantics", "reference"))
    mt = MEM_TYPE[dt]
    rt = {"f32": "f32", "f64": "f64"}.get(dt, "b32")
    progs = [Program.from_outputs({"_": e}) for _, _, e in plan.reductions]
    for pr in progs:
        for s in pr.nodes:
            if s.kind == "const":
                ops.const(s.a, s.b)
    idents = []
    for op, rdt, _ in plan.reductions:
        idents.append(ops.const(_IDENT[op], rdt)[0] if is_float(rdt)
                      else ops.const(_INT_IDENT[op], "s32")[0])

    # shared memory: per-warp partials, then the block partial read by rank 0
    rsz = 8
    warp_part = nred * NW * CW * rsz
    b.module(f".shared .align 16 .b8 col_warp[{warp_part}];")
    b.module(f".shared .align 16 .b8 col_block[{nred * CW * rsz}];")

    tid, lane, warp = b.regs("r", 3)
    b.ins(f"mov.u32 {tid}, %tid.x;")
    b.ins(f"and.b32 {lane}, {tid}, 31;")
    b.ins(f"shr.u32 {warp}, {tid}, 5;")
    strip, nstrip, rank = b.regs("r", 3)
    b.ins(f"mov.u32 {strip}, %clusterid.x;")
    b.ins(f"mov.u32 {nstrip}, %nclusterid.x;")
    b.ins(f"mov.u32 {rank}, %cluster_ctarank;")
    wbase, bbase = b.regs("r", 2)
    b.ins(f"mov.u32 {wbase}, col_warp;")
    b.ins(f"mov.u32 {bbase}, col_block;")
    r0, r1 = b.regs("r", 2)
    b.ins(f"mul.lo.u32 {r0}, {rank}, {RS};")
    b.ins(f"min.u32 {r0}, {r0}, {plan.rows};")
    b.ins(f"add.u32 {r1}, {r0}, {RS};")
    b.ins(f"min.u32 {r1}, {r1}, {plan.rows};")

    top, done = b.label("STRIP"), b.label("STRIP_END")
    p = b.reg("p")
    b.place(top)
    b.ins(f"setp.ge.u32 {p}, {strip}, {strips};")
    b.ins(f"@{p} bra {done};")
    col0 = b.reg("r")                     # first column of this lane
    b.ins(f"mad.lo.u32 {col0}, {strip}, {CW}, 0;")
    b.ins(f"mad.lo.u32 {col0}, {lane}, {VL}, {col0};")
    pcol = b.reg("p")
    b.ins(f"setp.lt.u32 {pcol}, {col0}, {plan.cols};")
    colbase = b.reg("rd")
    b.ins(f"mul.wide.u32 {colbase}, {col0}, {esz};")
    b.ins(f"add.s64 {colbase}, {ptrs[plan.tensor]}, {colbase};")

    accs = [[b.reg_for(rdt) for _ in range(VL)] for _, rdt, _ in plan.reductions]
    for j, (op, rdt, _) in enumerate(plan.reductions):
        for a in accs[j]:
            b.ins(f"mov.{ {'f32': 'f32', 'f64': 'f64'}.get(rdt, 'b32') } {a}, {idents[j]};")

    # rows: r = r0 + warp + NW*i, ROWS_IN_FLIGHT at a time
    rr = b.reg("r")
    b.ins(f"add.u32 {rr}, {r0}, {warp};")
    loop, lend = b.label("ROWS"), b.label("ROWS_END")
    b.place(loop)
    b.ins(f"setp.ge.u32 {p}, {rr}, {r1};")
    b.ins(f"@{p} bra {lend};")
    vals = []
    preds = []
    for u in range(ROWS_IN_FLIGHT):
        ru = b.reg("r")
        b.ins(f"add.u32 {ru}, {rr}, {u * NW};")
        pu = b.reg("p")
        b.ins(f"setp.lt.u32 {pu}, {ru}, {r1};")
        b.ins(f"and.pred {pu}, {pu}, {pcol};")
        off = b.reg("rd")
        b.ins(f"mul.wide.u32 {off}, {ru}, {plan.cols * esz};")
        a = b.reg("rd")
        b.ins(f"add.s64 {a}, {colbase}, {off};")
        rs = [b.reg_for(dt) for _ in range(VL)]
        if VL == 1:
            b.ins(f"@{pu} ld.global.nc.L1::no_allocate.{mt} {rs[0]}, [{a}];")
        else:
            b.ins(f"@{pu} ld.global.nc.L1::no_allocate.v{VL}.{mt} {{{', '.join(rs)}}}, [{a}];")
        vals.append(rs)
        preds.append(pu)
    for u in range(ROWS_IN_FLIGHT):
        skip = b.label("RSKIP")
        b.ins(f"@!{preds[u]} bra {skip};")
        for v in range(VL):
            lv = {Sym("in", plan.tensor, 0): (vals[u][v], dt)}
            for j, (op, rdt, e) in enumerate(plan.reductions):
                got = emit_program(ops, progs[j], lv)
                reg, vdt = got[e]
                if vdt != rdt:
                    reg = ops.coerce((reg, vdt), rdt)
                _combine(b, op, rdt, accs[j][v], reg)
        b.place(skip)
    b.ins(f"add.u32 {rr}, {rr}, {ROWS_IN_FLIGHT * NW};")
    b.ins(f"bra.uni {loop};")
    b.place(lend)

    # block combine: every warp stores its lane partials, warp 0 reduces
    # over the warps in order
    for j in range(nred):
        for v in range(VL):
            a = b.reg("r")
            b.ins(f"mad.lo.u32 {a}, {warp}, {CW * rsz}, {wbase};")
            b.ins(f"mad.lo.u32 {a}, {lane}, {VL * rsz}, {a};")
            b.ins(f"st.shared.{rt if rt != 'b32' else 's32'} [{a}+{(j * NW * CW + v) * rsz}], {accs[j][v]};")
    b.ins(f"bar.sync 1, {T};")
    w0 = b.label("W0_END")
    pw = b.reg("p")
    b.ins(f"setp.ne.u32 {pw}, {warp}, 0;")
    b.ins(f"@{pw} bra {w0};")
    for j, (op, rdt, _) in enumerate(plan.reductions):
        st = rt if rt != "b32" else "s32"
        for v in range(VL):
            a = b.reg("r")
            b.ins(f"mad.lo.u32 {a}, {lane}, {VL * rsz}, {wbase};")
            for w_ in range(1, NW):
                o = b.reg_for(rdt)
                b.ins(f"ld.shared.{st} {o}, [{a}+{((j * NW + w_) * CW + v) * rsz}];")
                _combine(b, op, rdt, accs[j][v], o)
            ab = b.reg("r")
            b.ins(f"mad.lo.u32 {ab}, {lane}, {VL * rsz}, {bbase};")
            b.ins(f"st.shared.{st} [{ab}+{(j * CW + v) * rsz}], {accs[j][v]};")
    b.place(w0)

    # cluster combine: rank 0 reads every rank's block partial in order
    if S > 1:
        b.ins("barrier.cluster.arrive.release.aligned;")
        b.ins("barrier.cluster.wait.acquire.aligned;")
    fin = b.label("FINAL_END")
    pf = b.reg("p")
    b.ins(f"setp.ne.u32 {pf}, {tid}, {tid};")           # false
    b.ins(f"setp.ne.or.u32 {pf}, {rank}, 0, {pf};")
    b.ins(f"setp.ne.or.u32 {pf}, {warp}, 0, {pf};")
    b.ins(f"@{pf} bra {fin};")
    for j, (op, rdt, _) in enumerate(plan.reductions):
        st = rt if rt != "b32" else "s32"
        for v in range(VL):
            ab = b.reg("r")
            b.ins(f"mad.lo.u32 {ab}, {lane}, {VL * rsz}, {bbase};")
            b.ins(f"add.u32 {ab}, {ab}, {(j * CW + v) * rsz};")
            if S > 1:
                for k in range(1, S):
                    ra = b.reg("r")
                    b.ins(f"mapa.shared::cluster.u32 {ra}, {ab}, {k};")
                    o = b.reg_for(rdt)
                    b.ins(f"ld.shared::cluster.{st} {o}, [{ra}];")
                    _combine(b, op, rdt, accs[j][v], o)
        # write the lane's VL columns of output j
        o_name = plan.outputs[j]
        oa = b.reg("rd")
        b.ins(f"mul.wide.u32 {oa}, {col0}, {esz};")
        b.ins(f"add.s64 {oa}, {ptrs[o_name]}, {oa};")
        if VL == 1:
            b.ins(f"@{pcol} st.global.{mt} [{oa}], {accs[j][0]};")
        else:
            b.ins(f"@{pcol} st.global.v{VL}.{mt} [{oa}], {{{', '.join(accs[j])}}};")
    b.place(fin)
    if S > 1:
        # keep every rank's shared memory alive until rank 0 has read it
        b.ins("barrier.cluster.arrive.release.aligned;")
        b.ins("barrier.cluster.wait.acquire.aligned;")
    else:
        b.ins(f"bar.sync 1, {T};")
    b.ins(f"add.u32 {strip}, {strip}, {nstrip};")
    b.ins(f"bra.uni {top};")
    b.place(done)

    grid = strips * S
    alg = plan.rows * plan.cols * esz + len(plan.outputs) * plan.cols * esz
    sidecar = {
        "category": "colreduce",
        "grid": [grid, 1, 1],
        "block": [T, 1, 1],
        "shared_bytes": 0,
        "cluster": [S, 1, 1],
        "algorithmic_bytes": alg,
        "column_strip": CW,
    }
    return b.render(), sidecar
