"""Attention category: (causal) softmax(Q K^T * scale) V in f32 on tcgen05.

Recognised IR (the reference lowers it per query row, one warp per row,
compiler.py:1121-1127 exp, 1649-1659 accumulation, 1877-1928 shuffles): a
Tile over ``(b, h, i, lane)`` whose key loop ``for j in [0, i+1)`` (causal)
or ``[0, S)`` loads ``k[b,h,j,:]``, reduces ``q . k`` across the warp,
multiplies by a scale constant, updates a running max with an ``Accum``
``max``, rescales a running sum and output accumulators by
``exp(m_old - m_new)``, adds ``exp(s - m_new)`` and ``p * v[b,h,j,:]``, and
finally writes ``o / l``.

Generated kernel (sm_100a), persistent over (batch*head, 128-query tiles):
heads in groups of up to 8 (so the CTAs running at one time share the K/V of
a few heads in L2), and inside a group the heaviest causal tiles first.  The
items are dealt by a static schedule computed at emit time (each item to
the CTA whose items so far cost least) and stored in the module, so that
causal items of 1 to S/128 key tiles leave no CTA with much more work than
the others:

* a pre-pass entry (``<entry>_ksplit``) writes K's tf32 lo part (K minus
  K with its low 13 bits cleared; the kernel loads K itself as the hi part,
  which the tensor core reads with those bits dropped) and V rounded to the
  nearest tf32 value, into scratch memory (each head's K and V are used by
  every query tile of the
  head, so doing this in the attention kernel would repeat the work S/128
  times; the tensor core drops the low 13 bits of an f32 operand, so an
  unrounded V would bias every product towards zero).  With more than one
  head group the pre-pass covers group 0 only, and warps 8-11 of the
  kernel write the later groups while the other warps compute: it takes chunks
  (up to 128 per group) from a counter in global memory and releases each
  on its group's count, which the producers acquire before their first
  load of a group's K lo / rounded V.  The 384-thread launch has 168
  registers per thread; warps 0-3 raise theirs to 224 and warps 4-7 lower
  theirs to 96 (``setmaxnreg``).  On a 256-thread launch (the meta.json
  block) every warp splits first and then takes its role.
* warps 0-3 (softmax): thread r owns query row r of the tile.  It loads its
  Q row, folds in scale * log2(e), splits it into tf32 hi/lo, stores hi into
  TMEM and lo into shared memory (the A operands of S = Q K^T, which is
  then in log2 units).  Per 128-key tile: ``tcgen05.ld`` of its 128
  scores, the causal mask (diagonal tiles only), tree max, lazy rescaling
  of the O accumulator in TMEM (only when the row max grew by more than
  2^8), P = 2^(s - m) written over the scores in TMEM (the A operand of
  O += P V), tree sum.
* warps 4 and 6 (one thread each): TMA producers of K and V.  K arrives in
  chunks of 32 dims x 128 keys (a hi box and a lo box, K-major, 128-byte
  swizzle) through a 3-slot ring, each slot released after its part of
  QK^T; V in chunks of 64 keys (one box per 32 dims, N-major, 128-byte
  swizzle / 32-byte atoms) through a 2-slot ring, each released after its
  part of PV.
* warp 5 (one thread): owns TMEM (512 columns: Q hi, O, two 128-column S/P
  buffers) and issues ``tcgen05.mma.kind::tf32`` with N = 128:
  S = Qhi Khi + Qhi Klo + Qlo Khi (3xTF32; Q hi from TMEM, Q lo from shared
  memory) into one S buffer while the softmax works on the other.  At N = 64
  an MMA measured 44 cycles against 32 of arithmetic; at N = 128 it runs at
  the arithmetic rate.
* warp 7 (one thread): issues O += P V (P from TMEM).  An MMA instruction
  holds its issuing thread ~44 cycles, so two issuers keep the tensor core
  busier than one; a barrier per S buffer orders QK^T(t+2) after PV(t).

All waits are bounded (tc.py); the status word reports a timeout.
"""

from __future__ import annotations

import heapq
import math
from dataclasses import dataclass

from .. import ir as I
from .common import NoMatch, declare_params, launch_block
from .ops import dtype_name
from .ptx import KernelBuilder, f32_hex, wide_vectors
from .tc import STATUS_NO_PREPASS, STATUS_TIMEOUT, TC, idesc_tf32, smem_desc_hi, split_launch

BQ = 128           # queries per tile (TMEM lanes)
BKV = 128          # keys per S tile (the N of each QK^T MMA)
BOX_KEYS = 64      # keys per TMA box, K and V alike (one shape for both kernels)
VC_KEYS = 64       # keys per V chunk
K_CHUNKS = 3       # one CTA per tile: K ring slots (2 with the gather stage)
VS = 2             #                   V ring slots
PAIR_K_CHUNKS = 6  # CTA pairs: K ring slots of half chunks (4 with the gather stage)
PAIR_VS = 4        #            V ring slots of half chunks
# CTA pairs (tcgen05 cta_group::2): correct and bit-identical to one CTA per
# tile, but not faster at 8x32x4096x128 (3.77-3.98 against 3.78-3.79 ms on
# one box): the doubled K/V lookahead removes the load waits, and an M=256
# MMA then costs ~77 cycles per CTA against 64.  Off unless asked for.
PAIR = False
LOG2E = 1.4426950408889634
ROLE_SOFTMAX, ROLE_PRODUCER, ROLE_MMA = 5, 6, 7
# arrivals of the softmax warps on the barriers the MMA issuers wait on (P
# ready, Q ready): 4 = one per warp, 128 = one per thread
ARRIVALS = 4
# K's lo part and the rounded V of every head group but the first are
# written inside the kernel, by split warps (8-11) that take chunks of the work
# from a shared counter while the other warps compute; the pre-pass then
# covers group 0 only.  (CTA pairs keep the whole pre-pass.)
INLINE_SPLIT = True
SPLIT_CHUNKS = 128         # chunks per head group, at most
PREPASS_GROUPS = 1         # head groups the pre-pass covers (2 measured within noise: +0.4%)
ROLE_SPLIT = 8
# With nine to twelve warps an SM sub-partition holds three, so ptxas gives
# each thread at most 168 registers at launch.  The warpgroups then re-divide
# them (setmaxnreg): the softmax warps take REG_SOFTMAX, the producer / MMA
# warps lower theirs to REG_ISSUE, the split warps keep the launch count.  The shares
# must fit the launch's registers (checked against ptxas's count).
REG_LAUNCH, REG_SOFTMAX, REG_ISSUE = 168, 224, 96
# split warps per CTA (warps 8-11, one warpgroup): against one, two measured 0.03 ms and
# four another 0.05 ms faster (alternating pairs); more would cut the launch below 168
SPLIT_WARPS = 4
# vectors of K and of V per lane in flight (the largest that divides); 8 measured
# 0.12 ms slower than 4 (alternating pairs)
SPLIT_UNROLLS = (1, 2, 4)
assert 128 * (REG_SOFTMAX + REG_ISSUE) + 32 * SPLIT_WARPS * REG_LAUNCH <= \
    (256 + 32 * SPLIT_WARPS) * REG_LAUNCH
assert 128 * (REG_SOFTMAX + REG_ISSUE) <= 256 * REG_LAUNCH     # the 256-thread launch


@dataclass
class AttnPlan:
    batch: int
    heads: int
    seq: int
    dim: int
    scale: float
    causal: bool
    q: str
    k: str
    v: str
    out: str


def _walk(stmts):
    return list(I.walk(stmts))


def match(comp) -> AttnPlan:
    ins, outs = list(comp.kernel.inputs), list(comp.kernel.outputs)
    if len(ins) != 3 or len(outs) != 1:
        raise NoMatch("attention has q, k, v inputs and one output")
    shapes = [comp.shape_of(t) for t in ins + outs]
    if any(len(s) != 4 for s in shapes) or len({tuple(s) for s in shapes}) != 1:
        raise NoMatch("q, k, v and out must share one [B, H, S, D] shape")
    if any(comp.dtype_of(t) != "f32" for t in ins + outs):
        raise NoMatch("f32 attention only")
    B, H, S, D = shapes[0]
    body = comp.kernel.body
    if len(body) != 1 or not isinstance(body[0], I.Tile) or len(body[0].axes) != 4:
        raise NoMatch("attention tile has (b, h, i, lane) axes")
    tile = body[0]
    i_axis = tile.axes[2].name
    loops = [s for s in _walk(tile.body) if isinstance(s, I.StridedLoop)]
    if len(loops) != 1:
        raise NoMatch("one key loop")
    loop = loops[0]
    inner = _walk(loop.body)
    if not any(isinstance(s, I.WarpShuffle) for s in inner):
        raise NoMatch("no cross-lane dot product")
    if not any(isinstance(s, I.Accum) and getattr(s.op, "name", s.op) == "max" for s in inner):
        raise NoMatch("no running max")
    if sum(1 for s in inner if isinstance(s, I.Assign) and getattr(s.op, "name", s.op) == "exp") < 2:
        raise NoMatch("no online-softmax exponentials")
    loaded = {s.input for s in inner if isinstance(s, I.Load)}
    if loaded != {ins[1], ins[2]}:
        raise NoMatch("key loop must load k and v")
    # causal: end = i + 1
    causal = False
    if loop.end is not None:
        e = loop.end
        if not (isinstance(e, I.BinaryExpr) and e.op == "+" and isinstance(e.left, I.Var)
                and e.left.name == i_axis and isinstance(e.right, I.Literal)
                and int(e.right.value) == 1):
            raise NoMatch("key loop end is not i + 1")
        causal = True
    # the scale: a float Let multiplied into the reduced dot product
    lets = {s.name: s.value for s in _walk(tile.body) if isinstance(s, I.Let)}
    scale = None
    shuffled = {st for s in inner if isinstance(s, I.WarpShuffle) for st in s.state}
    for s in inner:
        if isinstance(s, I.Assign) and getattr(s.op, "name", s.op) == "multiply" \
                and len(s.args) == 2 and s.args[0] in shuffled:
            v = lets.get(s.args[1])
            if isinstance(v, I.Literal):
                scale = float(v.value)
    if scale is None:
        raise NoMatch("no scale constant applied to the scores")
    if D % 32 or D > 128:
        raise NoMatch("head_dim must be a multiple of 32 and at most 128")
    return AttnPlan(B, H, S, D, scale, causal, ins[0], ins[1], ins[2], outs[0])


def _split_values(b, x, y):
    """K values ``x`` -> their tf32 lo parts (K minus K with its low 13 bits
    cleared, exact); V values ``y`` -> rounded to the nearest tf32
    (``cvt.rna``).  Returns the two register lists."""
    lo = b.regs("f", len(x))
    vr = b.regs("r", len(y))
    for e in range(len(x)):
        hb = b.reg("r")
        b.ins(f"mov.b32 {hb}, {x[e]};")
        b.ins(f"and.b32 {hb}, {hb}, 0xFFFFE000;")
        hf = b.reg("f")
        b.ins(f"mov.b32 {hf}, {hb};")
        b.ins(f"sub.f32 {lo[e]}, {x[e]}, {hf};")
        b.ins(f"cvt.rna.tf32.f32 {vr[e]}, {y[e]};")
    return lo, vr


def emit_kv_prepass(target: str, version: str, entry: str, n_elems: int, block: int = 256,
                    split_groups: tuple | None = None) -> str:
    """The pre-pass entry ``entry(k, v, k_lo, v_r)``.  The tensor core reads
    an f32 operand as tf32 by dropping its low 13 bits, so the kernel loads
    K itself as the hi operand of 3xTF32 QK^T (the hardware forms
    hi = K with the low 13 bits cleared) and this entry writes only
    ``lo = K - hi`` (exact).  V is rounded to the nearest tf32 value
    (``cvt.rna``: ties away from zero; NaN and infinity kept), so that the
    tensor core reads V unbiased.  Grid-stride over vectors of 8 floats
    (32-byte accesses, PTX ISA 8.8) or 4 below 8.8; ``n_elems`` a multiple
    of the vector; returned without the module header.  With 32-byte
    vectors and 16 blocks per SM the full-size pass (2 GB) measured 0.332
    ms against 0.368 with 16-byte vectors and 8 blocks per SM.

    ``split_groups = (groups, chunks, covered)``: the attention kernel
    splits every head group from ``covered`` on itself (``emit``, the split
    warps), and this entry covers the first ``covered`` groups (``n_elems``
    = their elements).  Its thread 0 also prepares the kernel's split state
    in the module globals: the ``k_lo`` / ``v_r`` addresses, the chunk
    counter at zero, and the per-group chunks-done counts (the covered
    groups complete, the others zero)."""
    vw = 8 if wide_vectors(version) else 4
    assert n_elems % vw == 0
    b = KernelBuilder(entry, target, version)
    b.directive(f".maxntid {block}, 1, 1")
    names = ("k", "v", "k_lo", "v_r")
    ptrs = []
    for nm in names:
        pp = b.param(nm, ".u64")
        r = b.reg("rd")
        b.ins(f"ld.param.u64 {r}, [{pp}];")
        b.ins(f"cvta.to.global.u64 {r}, {r};")
        ptrs.append(r)
    g, stride, t, nt = b.regs("r", 4)
    b.ins(f"mov.u32 {g}, %ctaid.x;")
    b.ins(f"mov.u32 {nt}, %ntid.x;")
    b.ins(f"mov.u32 {stride}, %nctaid.x;")
    b.ins(f"mul.lo.u32 {stride}, {stride}, {nt};")
    b.ins(f"mov.u32 {t}, %tid.x;")
    if split_groups is not None:
        ngroups, nchunks, covered = split_groups
        p0 = b.reg("p")
        b.ins(f"or.b32 {g}, {g}, {t};")
        b.ins(f"setp.ne.u32 {p0}, {g}, 0;")
        skip = b.label("SPLIT_INIT_DONE")
        b.ins(f"@{p0} bra {skip};")
        ga = b.reg("rd")
        for nm, glob in ((names[2], "emmy_split_lo"), (names[3], "emmy_split_vr")):
            b.ins(f"mov.u64 {ga}, {glob};")
            b.ins(f"st.global.u64 [{ga}], {ptrs[names.index(nm)]};")
        zero, full = b.regs("r", 2)
        b.ins(f"mov.u32 {zero}, 0;")
        b.ins(f"mov.u32 {full}, {nchunks};")
        b.ins(f"mov.u64 {ga}, emmy_split_next;")
        b.ins(f"st.global.u32 [{ga}], {zero};")
        b.ins(f"mov.u64 {ga}, emmy_split_done;")
        i, pi, v_ = b.reg("r"), b.reg("p"), b.reg("r")
        loop, ldone = b.label("SPLIT_ZERO"), b.label("SPLIT_ZERO_END")
        b.ins(f"mov.u32 {i}, 0;")
        b.place(loop)
        b.ins(f"setp.ge.u32 {pi}, {i}, {ngroups};")
        b.ins(f"@{pi} bra {ldone};")
        # the groups this pre-pass covers are complete, the others not begun
        b.ins(f"setp.lt.u32 {pi}, {i}, {covered};")
        b.ins(f"selp.b32 {v_}, {full}, {zero}, {pi};")
        b.ins(f"st.global.u32 [{ga}], {v_};")
        b.ins(f"add.s64 {ga}, {ga}, 4;")
        b.ins(f"add.u32 {i}, {i}, 1;")
        b.ins(f"bra {loop};")
        b.place(ldone)
        b.place(skip)
        b.ins(f"mov.u32 {g}, %ctaid.x;")
    b.ins(f"mad.lo.u32 {g}, {g}, {nt}, {t};")
    top, done = b.label("PRE"), b.label("PRE_END")
    p = b.reg("p")
    b.place(top)
    b.ins(f"setp.ge.u32 {p}, {g}, {n_elems // vw};")
    b.ins(f"@{p} bra {done};")
    off = b.reg("rd")
    b.ins(f"mul.wide.u32 {off}, {g}, {vw * 4};")
    a = {nm: b.reg("rd") for nm in names}
    for nm, base_ in zip(names, ptrs):
        b.ins(f"add.s64 {a[nm]}, {base_}, {off};")
    x = b.regs("f", vw)
    y = b.regs("f", vw)
    b.ins(f"ld.global.nc.L1::no_allocate.v{vw}.f32 {{{', '.join(x)}}}, [{a['k']}];")
    b.ins(f"ld.global.nc.L1::no_allocate.v{vw}.f32 {{{', '.join(y)}}}, [{a['v']}];")
    lo, vr = _split_values(b, x, y)
    b.ins(f"st.global.v{vw}.f32 [{a['k_lo']}], {{{', '.join(lo)}}};")
    b.ins(f"st.global.v{vw}.b32 [{a['v_r']}], {{{', '.join(vr)}}};")
    b.ins(f"add.u32 {g}, {g}, {stride};")
    b.ins(f"bra.uni {top};")
    b.place(done)
    return b.render(header=False)


# heads per scheduling group (largest divisor of batch*heads not above this)
HEAD_GROUP = 8


def head_group(bh: int) -> int:
    return max(g for g in range(1, min(HEAD_GROUP, bh) + 1) if bh % g == 0)


# items above this are dealt round-robin (the tables would bloat the module)
SCHED_MAX_ITEMS = 16384
# fixed cost of changing work item (staging Q, the epilogue, the first K
# loads of a head) in eighths of a 128-key tile, measured at ~2.4 tiles
ITEM_COST_8THS = 19


def item_schedule(costs, ncta):
    """Static schedule: items in order, each to the CTA whose items so far
    cost least (ties to the lower index) -- what a shared work queue would
    hand out, computed ahead.  Returns (items of CTA 0, then CTA 1, ...;
    each CTA's offsets into that list, ncta + 1 entries).  Items keep their
    order inside a CTA's list, so CTAs that run at the same time still work
    on the same few heads."""
    heap = [(0, i) for i in range(ncta)]
    lists = [[] for _ in range(ncta)]
    for w, c in enumerate(costs):
        t, i = heapq.heappop(heap)
        lists[i].append(w)
        heapq.heappush(heap, (t + c, i))
    work = [w for lst in lists for w in lst]
    offs = [0]
    for lst in lists:
        offs.append(offs[-1] + len(lst))
    return work, offs


def pair_ok(comp, plan: AttnPlan) -> bool:
    """CTA pairs split each K chunk by keys and each V chunk by head dims
    (32-dim boxes, so head_dim 64 or 128), need two query tiles per head,
    and an even grid under the meta.json geometry (a cluster of two)."""
    g = comp.kmeta.get("grid") or [1]
    g = [g] if isinstance(g, int) else list(g)
    return (PAIR and plan.dim in (64, 128) and plan.seq > BQ and g[0] % 2 == 0)


def shape_global(heads_total: int, seq: int, head_dim: int) -> str:
    """Name of the module global that records an attention module's compiled
    shape ((batch*heads) x keys x head_dim)."""
    return f"emmy_attn_shape_{heads_total}x{seq}x{head_dim}"


# ----------------------------------------------------------------------------
def emit(comp, plan: AttnPlan, gather: int = 0, pair=None):
    """``gather`` > 0: the all-gather variant for a (batch x head) shard.
    Instead of writing ``out``, the epilogue stores every finished query
    tile into each of the up to ``gather`` destinations in the module global
    ``emmy_gather_dst`` (``emmy_gather_n`` used), at row
    ``emmy_gather_row0 + pair * seq + query`` of a [rows, head_dim] view:
    every rank's full output, peers' copies mapped over NVLink.

    ``pair`` (default: ``pair_ok``): a cluster of two CTAs computes 256
    query rows of one head with ``tcgen05.mma.cta_group::2`` (M=256).  Each
    CTA owns 128 rows (its Q, S, P and O) and loads half of every K chunk
    (64 of its 128 keys) and half of every V chunk (half of the head dims);
    the even CTA issues every MMA.  Per CTA the K and V rings then hold
    twice as many chunks in the same shared memory."""
    B, H, S, D = plan.batch, plan.heads, plan.seq, plan.dim
    if pair is None:
        pair = pair_ok(comp, plan)
    CG = 2 if pair else 1
    T = launch_block(comp) or 256
    if T != 256:
        raise NoMatch(f"the tcgen05 attention kernel needs 256 threads per block (meta.json has {T})")
    G = head_group(B * H)
    NG = B * H // G                    # head groups
    # in-kernel split: chunks of a head group, each a whole number of the
    # split warps' 32-lane vector rows
    SVW = 8 if wide_vectors(comp.ptx_version) else 4
    nvg = G * S * D // SVW             # vectors per head group
    CH = max([c for c in range(1, SPLIT_CHUNKS + 1) if nvg % (32 * c) == 0] or [0])
    PG = PREPASS_GROUPS                # head groups the pre-pass covers
    inline = INLINE_SPLIT and not pair and NG > PG and CH > 0
    CHV = nvg // CH if inline else 0   # vectors per chunk
    SUN = max(u for u in SPLIT_UNROLLS if (CHV // 32) % u == 0) if inline else 1
    SW = SPLIT_WARPS if inline else 0
    TL = T + 32 * SW                   # launch block: the split warps are warps 8 ...
    DC = D // 32                       # 32-dim chunks
    nqt = -(-S // BQ)
    nqu = -(-nqt // CG)                # query units: tiles, or pairs of tiles
    items = B * H * nqu
    if pair:
        KCH = 4 if gather else PAIR_K_CHUNKS
        NVS = PAIR_VS
    else:
        KCH = 2 if gather else K_CHUNKS
        NVS = VS
    VPT = BKV // VC_KEYS               # V chunks per S tile
    KC_KEYS = BKV // CG                # keys of a K chunk this CTA loads
    VDC = DC // CG                     # 32-dim boxes of a V chunk this CTA loads
    # shared memory: Q lo (the A operand of Qlo Khi: 128 rows, K-major,
    # 128-byte swizzle, one 16 KB box per 32 dims) | K ring (a slot: 32 dims
    # of this CTA's keys of a 128-key chunk, hi box then lo box) | V ring (a
    # slot: 64 keys, one box per 32 of this CTA's dims) | barriers
    Q_LO = 0
    K_BOX = KC_KEYS * 128              # 16 KB (8 KB per CTA of a pair)
    K_SLOT = 2 * K_BOX
    K_RING = Q_LO + BQ * D * 4
    V_BOX = VC_KEYS * 128              # 8 KB
    V_SLOT = VDC * V_BOX
    V_RING = K_RING + KCH * K_SLOT
    BAR = V_RING + NVS * V_SLOT
    # gather mode: a 32x32 transpose stage per softmax warp (rows padded to
    # 144 B), so stores to peers are row-contiguous
    BAR_BYTES = 320
    EPI = BAR + BAR_BYTES
    EPI_ROW = 144
    EPI_WARP = 32 * EPI_ROW
    SMEM = EPI + (4 * EPI_WARP if gather else 0) + 1024
    assert SMEM <= 232448, SMEM
    # TMEM columns: Q hi | O accumulator | S/P buffer 0 | S/P buffer 1
    C_QHI, C_O, C_S0, C_S1 = 0, 128, 256, 384
    VW = 8 if wide_vectors(comp.ptx_version) else 4    # floats per epilogue store
    TMEM_COLS = 512
    split_entry = comp.entry + "_ksplit"

    b = KernelBuilder(comp.entry, comp.target, comp.ptx_version)
    b.module(".global .align 128 .b8 tmap_Khi[128];")
    b.module(".global .align 128 .b8 tmap_Klo[128];")
    b.module(".global .align 128 .b8 tmap_V[128];")
    # the compiled shape, in a global's name: a launcher that brings its own
    # tensor maps and scratch (libemmy_noalloc) looks this name up to refuse
    # a shape the module was not compiled for, with no device read
    b.module(f".visible .global .align 4 .u32 {shape_global(B * H, S, D)} = 1;")
    b.module(".extern .shared .align 1024 .b8 dsmem[];")
    if gather:
        b.module(f".global .align 8 .b8 emmy_gather_dst[{8 * gather}];")
        b.module(".global .align 4 .u32 emmy_gather_n;")
        b.module(".global .align 4 .u32 emmy_gather_row0;")
    if inline:
        # split state, prepared by the pre-pass entry before every launch
        b.module(".global .align 8 .u64 emmy_split_lo;")
        b.module(".global .align 8 .u64 emmy_split_vr;")
        b.module(".global .align 4 .u32 emmy_split_next;")
        b.module(f".global .align 4 .b8 emmy_split_done[{4 * NG}];")
    b.directive(f".maxntid {TL}, 1, 1")
    if inline:
        b.directive(f".maxnreg {REG_LAUNCH}")
    if pair:
        # launching without the cluster of two fails at launch time
        b.directive(".reqnctapercluster 2, 1, 1")
    ptrs = declare_params(b, comp)
    pQ, pO = ptrs[plan.q], ptrs[plan.out]

    tid, warp, lane = b.regs("r", 3)
    b.ins(f"mov.u32 {tid}, %tid.x;")
    b.ins(f"shr.u32 {warp}, {tid}, 5;")
    b.ins(f"and.b32 {lane}, {tid}, 31;")
    base = b.reg("r")
    b.ins(f"mov.u32 {base}, dsmem;")
    b.ins(f"add.u32 {base}, {base}, 1023;")
    b.ins(f"and.b32 {base}, {base}, 0xFFFFFC00;")
    bars = b.reg("r")
    b.ins(f"add.u32 {bars}, {base}, {BAR};")
    # barriers: K ring ([KCH]) and V ring ([NVS]), Q ready, S full / P full
    # per S buffer, O (PV) done
    KF, KE = 0, 8 * PAIR_K_CHUNKS
    VF = 2 * 8 * PAIR_K_CHUNKS
    VE = VF + 8 * PAIR_VS
    QR = VE + 8 * PAIR_VS
    SF, PF = QR + 8, QR + 24
    # OF completes once per PV (the softmax waits on it only to rescale O,
    # when the barrier is at most one phase past the awaited PV); OFIN once
    # per work item, after its last PV -- the epilogue's wait.  A parity wait
    # on OF there could see the barrier a phase *behind* the last PV and
    # pass early.
    OF, DRAIN, OFIN, FIN = QR + 40, QR + 48, QR + 56, QR + 64
    # PE[b] completes when a PV that read the P in S buffer b is done (the
    # QK^T issuer's wait before it overwrites the buffer); DRAIN2 is the PV
    # issuer's own drain at teardown
    PE, DRAIN2 = QR + 80, QR + 96
    slot, abort = b.regs("r", 2)
    b.ins(f"add.u32 {slot}, {bars}, {QR + 72};")
    b.ins(f"add.u32 {abort}, {bars}, {QR + 76};")
    assert DRAIN2 + 8 <= BAR_BYTES

    tc = TC(b, abort, cta_group=CG)

    p = b.reg("p")
    skip = b.label("INIT_DONE")
    b.ins(f"setp.ne.u32 {p}, {tid}, 0;")
    b.ins(f"@{p} bra {skip};")
    for s in range(KCH):
        for off in (KF, KE):
            tc.init(f"{bars}+{off + 8 * s}", 1)
    for s in range(NVS):
        for off in (VF, VE):
            tc.init(f"{bars}+{off + 8 * s}", 1)
    tc.init(f"{bars}+{QR}", ARRIVALS * CG)    # the softmax warps of the pair
    for k in range(2):
        tc.init(f"{bars}+{SF + 8 * k}", 1)
        tc.init(f"{bars}+{PF + 8 * k}", ARRIVALS * CG)
    tc.init(f"{bars}+{OF}", 1)
    tc.init(f"{bars}+{OFIN}", 1)
    tc.init(f"{bars}+{DRAIN}", 1)
    tc.init(f"{bars}+{FIN}", 1)
    for k in range(2):
        tc.init(f"{bars}+{PE + 8 * k}", 1)
    tc.init(f"{bars}+{DRAIN2}", 1)
    b.ins(f"st.shared.u32 [{abort}], 0;")
    b.ins("fence.mbarrier_init.release.cluster;")
    b.place(skip)
    skip2 = b.label("ALLOC_DONE")
    b.ins(f"setp.ne.u32 {p}, {warp}, 5;")
    b.ins(f"@{p} bra {skip2};")
    tc.tmem_alloc(slot, TMEM_COLS)
    b.place(skip2)
    b.ins("tcgen05.fence::before_thread_sync;")
    if pair:
        # both CTAs' barriers are initialised before either CTA's TMA bytes,
        # MMA commits or arrivals can reach them
        b.ins("barrier.cluster.arrive.release.aligned;")
        b.ins("barrier.cluster.wait.acquire.aligned;")
    else:
        b.ins("bar.sync 0;")
    b.ins("tcgen05.fence::after_thread_sync;")
    tmem = b.reg("r")
    b.ins(f"ld.shared.u32 {tmem}, [{slot}];")
    cta, ncta, rank = b.regs("r", 3)
    lead = b.reg("p")                     # this CTA issues the MMAs
    if pair:
        # cta / ncta count CTA pairs; the leader is rank 0 of the cluster
        b.ins(f"mov.u32 {cta}, %clusterid.x;")
        b.ins(f"mov.u32 {ncta}, %nclusterid.x;")
        b.ins(f"mov.u32 {rank}, %cluster_ctarank;")
        lbars, pbars = b.regs("r", 2)     # the leader's and the peer's barrier blocks
        b.ins(f"mapa.shared::cluster.u32 {lbars}, {bars}, 0;")
        prk = b.reg("r")
        b.ins(f"xor.b32 {prk}, {rank}, 1;")
        b.ins(f"mapa.shared::cluster.u32 {pbars}, {bars}, {prk};")
        tc.peer_abort = b.reg("r")
        b.ins(f"add.u32 {tc.peer_abort}, {pbars}, {QR + 76};")
    else:
        b.ins(f"mov.u32 {cta}, %ctaid.x;")
        b.ins(f"mov.u32 {ncta}, %nctaid.x;")
        b.ins(f"mov.u32 {rank}, 0;")
    b.ins(f"setp.eq.u32 {lead}, {rank}, 0;")
    END = b.label("END")

    def remote(reg_base, off, s=None):
        """shared::cluster address of barrier ``off`` (+ 8*s) in the
        barrier block at ``reg_base`` (the leader's or the peer's)."""
        r = b.reg("r")
        if s is None:
            b.ins(f"add.u32 {r}, {reg_base}, {off};")
        else:
            b.ins(f"mad.lo.u32 {r}, {s}, 8, {reg_base};")
            b.ins(f"add.u32 {r}, {r}, {off};")
        return r

    # the item sequence of this CTA (or pair): a precomputed table when the
    # launch has the grid the table was built for, else every ncta-th item
    ncta_tab = min(items, 148 // CG)
    use_tab = b.reg("p")
    kbeg, kend, kstep = b.regs("r", 3)
    b.ins(f"mov.u32 {kbeg}, {cta};")
    b.ins(f"mov.u32 {kend}, {items};")
    b.ins(f"mov.u32 {kstep}, {ncta};")
    if items <= SCHED_MAX_ITEMS:
        def unit_cost(w):
            qu = nqu - 1 - (w % (G * nqu)) // G
            keys = min((qu + 1) * BQ * CG, S) if plan.causal else S
            return 8 * -(-keys // BKV) + ITEM_COST_8THS
        work, offs = item_schedule([unit_cost(w) for w in range(items)], ncta_tab)
        b.module(f".global .align 4 .u32 emmy_work[{items}] = {{{', '.join(map(str, work))}}};")
        b.module(f".global .align 4 .u32 emmy_work_off[{ncta_tab + 1}] = "
                 f"{{{', '.join(map(str, offs))}}};")
        b.ins(f"setp.eq.u32 {use_tab}, {ncta}, {ncta_tab};")
        ta, to_ = b.reg("rd"), b.reg("rd")
        b.ins(f"mov.u64 {ta}, emmy_work_off;")
        b.ins(f"mul.wide.u32 {to_}, {cta}, 4;")
        b.ins(f"add.s64 {ta}, {ta}, {to_};")
        b.ins(f"@{use_tab} ld.global.nc.u32 {kbeg}, [{ta}];")
        b.ins(f"@{use_tab} ld.global.nc.u32 {kend}, [{ta}+4];")
        b.ins(f"@{use_tab} mov.u32 {kstep}, 1;")
    else:
        b.ins(f"setp.ne.u32 {use_tab}, 0, 0;")

    def item_at(k):
        """Item at position k of this CTA's sequence."""
        w = b.reg("r")
        b.ins(f"mov.u32 {w}, {k};")
        if items <= SCHED_MAX_ITEMS:
            a, o = b.reg("rd"), b.reg("rd")
            b.ins(f"mov.u64 {a}, emmy_work;")
            b.ins(f"mul.wide.u32 {o}, {k}, 4;")
            b.ins(f"add.s64 {a}, {a}, {o};")
            b.ins(f"@{use_tab} ld.global.nc.u32 {w}, [{a}];")
        return w

    def item_coords(w):
        """Work item -> (bh, qu): heads in groups of G, and inside a group
        the heaviest query units (a 128-query tile, or a pair of them)
        first.  CTAs that run at the same time then read the K/V of a few
        heads, which stay in L2."""
        bh, qu, g, r = b.regs("r", 4)
        b.ins(f"div.u32 {g}, {w}, {G * nqu};")
        b.ins(f"rem.u32 {r}, {w}, {G * nqu};")
        b.ins(f"div.u32 {qu}, {r}, {G};")
        b.ins(f"sub.u32 {qu}, {nqu - 1}, {qu};")
        b.ins(f"rem.u32 {r}, {r}, {G};")
        b.ins(f"mad.lo.u32 {bh}, {g}, {G}, {r};")
        return bh, qu

    def own_tile(qu):
        """This CTA's 128-query tile of query unit qu."""
        if not pair:
            return qu
        qt = b.reg("r")
        b.ins(f"mad.lo.u32 {qt}, {qu}, 2, {rank};")
        return qt

    def n_kv(qu):
        """128-key tiles of query unit qu (the pair's count for a pair: its
        lower tile's last key tile is then fully masked)."""
        n = b.reg("r")
        if plan.causal:
            b.ins(f"mad.lo.u32 {n}, {qu}, {BQ * CG}, {BQ * CG};")
            b.ins(f"min.u32 {n}, {n}, {S};")
            b.ins(f"add.u32 {n}, {n}, {BKV - 1};")
            b.ins(f"div.u32 {n}, {n}, {BKV};")
        else:
            b.ins(f"mov.u32 {n}, {-(-S // BKV)};")
        return n

    def item_loop(body_fn, label):
        """body_fn(w, k) for each item w of this CTA's sequence (k: its
        position, for the roles that look one item ahead)."""
        k = b.reg("r")
        top, done = b.label(label), b.label(label + "_END")
        pt = b.reg("p")
        b.ins(f"mov.u32 {k}, {kbeg};")
        b.place(top)
        b.ins(f"setp.ge.u32 {pt}, {k}, {kend};")
        b.ins(f"@{pt} bra.uni {done};")
        body_fn(item_at(k), k)
        b.ins(f"add.u32 {k}, {k}, {kstep};")
        b.ins(f"bra.uni {top};")
        b.place(done)

    def kv_loop(nkv, body_fn, t, label):
        j = b.reg("r")
        top, done = b.label(label), b.label(label + "_END")
        pk = b.reg("p")
        b.ins(f"mov.u32 {j}, 0;")
        b.place(top)
        b.ins(f"setp.ge.u32 {pk}, {j}, {nkv};")
        b.ins(f"@{pk} bra.uni {done};")
        body_fn(j)
        b.ins(f"add.u32 {j}, {j}, 1;")
        if t is not None:
            b.ins(f"add.u32 {t}, {t}, 1;")
        b.ins(f"bra.uni {top};")
        b.place(done)

    def ring(t, n):
        """Slot and phase parity of use number t of an n-slot ring."""
        s, ph = b.regs("r", 2)
        if n & (n - 1) == 0:
            b.ins(f"and.b32 {s}, {t}, {n - 1};")
            b.ins(f"shr.u32 {ph}, {t}, {n.bit_length() - 1};")
        else:
            b.ins(f"rem.u32 {s}, {t}, {n};")
            b.ins(f"div.u32 {ph}, {t}, {n};")
        b.ins(f"and.b32 {ph}, {ph}, 1;")
        return s, ph

    def bar_at(off, s=None):
        r = b.reg("r")
        if s is None:
            b.ins(f"add.u32 {r}, {bars}, {off};")
        else:
            b.ins(f"mad.lo.u32 {r}, {s}, 8, {bars};")
            b.ins(f"add.u32 {r}, {r}, {off};")
        return r

    def parity(t, flip=False):
        r = b.reg("r")
        b.ins(f"and.b32 {r}, {t}, 1;")
        if flip:
            b.ins(f"xor.b32 {r}, {r}, 1;")
        return r

    roles = [b.label("SOFTMAX"), b.label("PRODUCER_K"), b.label("MMA_QK"), b.label("PRODUCER_V"),
             b.label("MMA_PV")]
    pr = b.reg("p")
    if inline:
        # warps 8-11 split; a launch without them (the meta.json block of
        # 256 threads) has every warp split first, then take its role
        pall, nth = b.reg("p"), b.reg("r")
        SPLIT, DISPATCH = b.label("SPLIT"), b.label("DISPATCH")
        b.ins(f"mov.u32 {nth}, %ntid.x;")
        b.ins(f"setp.lt.u32 {pall}, {nth}, {TL};")
        b.ins(f"@{pall} bra.uni {SPLIT};")
        b.ins(f"setp.ge.u32 {pr}, {warp}, 8;")
        b.ins(f"@{pr} bra.uni {SPLIT};")
        b.place(DISPATCH)
    if inline:
        # register split per warpgroup, each right before its own roles so
        # that a role's code is reached from one budget only: warps 0-3 take
        # registers, warps 4-7 hand theirs back
        wg1 = b.label("WG_ISSUE")
        b.ins(f"setp.ge.u32 {pr}, {warp}, 4;")
        b.ins(f"@{pr} bra {wg1};")
        b.ins(f"setmaxnreg.inc.sync.aligned.u32 {REG_SOFTMAX};")
        b.ins(f"bra.uni {roles[0]};")
        b.place(wg1)
        b.ins(f"setmaxnreg.dec.sync.aligned.u32 {REG_ISSUE};")
    else:
        b.ins(f"setp.lt.u32 {pr}, {warp}, 4;")
        b.ins(f"@{pr} bra {roles[0]};")
    b.ins(f"setp.eq.u32 {pr}, {warp}, 4;")
    b.ins(f"@{pr} bra {roles[1]};")
    b.ins(f"setp.eq.u32 {pr}, {warp}, 5;")
    b.ins(f"@{pr} bra {roles[2]};")
    b.ins(f"setp.eq.u32 {pr}, {warp}, 6;")
    b.ins(f"@{pr} bra {roles[3]};")
    b.ins(f"bra.uni {roles[4]};")              # warp 7

    if inline:
        # ---- split warps: K's lo part and the rounded V of groups 1.. --------
        # Chunk c (groups 1.. in order, CH chunks each) is taken from the
        # shared counter, so the resident warps share the work whatever the
        # grid; a chunk's completion is released on its group's counter,
        # which the producers acquire before their TMA loads of that group.
        b.place(SPLIT)
        lo_b, vr_b, ga = b.regs("rd", 3)
        b.ins(f"mov.u64 {ga}, emmy_split_lo;")
        b.ins(f"ld.global.u64 {lo_b}, [{ga}];")
        b.ins(f"mov.u64 {ga}, emmy_split_vr;")
        b.ins(f"ld.global.u64 {vr_b}, [{ga}];")
        # the pre-pass entry records the scratch addresses; without it there
        # is nothing to write to: report and leave (the producers' bounded
        # waits then end the kernel)
        pz, pz2 = b.regs("p", 2)
        have = b.label("SPLIT_HAVE_SCRATCH")
        b.ins(f"setp.eq.u64 {pz}, {lo_b}, 0;")
        b.ins(f"setp.eq.u64 {pz2}, {vr_b}, 0;")
        b.ins(f"or.pred {pz}, {pz}, {pz2};")
        b.ins(f"@!{pz} bra.uni {have};")
        tc.raise_abort(STATUS_NO_PREPASS)
        b.ins(f"bra.uni {END};")
        b.place(have)
        nxt, dn = b.regs("rd", 2)
        b.ins(f"mov.u64 {nxt}, emmy_split_next;")
        b.ins(f"mov.u64 {dn}, emmy_split_done;")
        pl0 = b.reg("p")
        b.ins(f"setp.eq.u32 {pl0}, {lane}, 0;")
        loff = b.reg("rd")                 # this lane's first vector in a chunk
        b.ins(f"mul.wide.u32 {loff}, {lane}, {SVW * 4};")
        c = b.reg("r")
        stop = b.label("SPLIT_NEXT")
        send = b.label("SPLIT_END")
        b.place(stop)
        b.ins(f"@{pl0} atom.global.add.u32 {c}, [{nxt}], 1;")
        b.ins(f"shfl.sync.idx.b32 {c}, {c}, 0, 0x1f, 0xffffffff;")
        pc = b.reg("p")
        b.ins(f"setp.ge.u32 {pc}, {c}, {(NG - PG) * CH};")
        b.ins(f"@{pc} bra.uni {send};")
        cg = b.reg("r")                    # chunk index counting the pre-pass groups
        b.ins(f"add.u32 {cg}, {c}, {PG * CH};")
        grp = b.reg("r")
        b.ins(f"div.u32 {grp}, {cg}, {CH};")
        off = b.reg("rd")
        b.ins(f"mul.wide.u32 {off}, {cg}, {CHV * SVW * 4};")
        b.ins(f"add.s64 {off}, {off}, {loff};")
        pk, pv, plo, pvr = b.regs("rd", 4)
        for dst, base_ in ((pk, ptrs[plan.k]), (pv, ptrs[plan.v]), (plo, lo_b), (pvr, vr_b)):
            b.ins(f"add.s64 {dst}, {base_}, {off};")
        step = 32 * SVW * 4                # bytes between a lane's vectors
        trips = b.reg("r")
        b.ins(f"mov.u32 {trips}, {CHV // 32 // SUN};")
        ltop = b.label("SPLIT_VEC")
        b.place(ltop)
        xs, ys = [], []
        for u in range(SUN):
            x = b.regs("f", SVW)
            y = b.regs("f", SVW)
            b.ins(f"ld.global.nc.L1::no_allocate.v{SVW}.f32 {{{', '.join(x)}}}, "
                  f"[{pk}+{u * step}];")
            b.ins(f"ld.global.nc.L1::no_allocate.v{SVW}.f32 {{{', '.join(y)}}}, "
                  f"[{pv}+{u * step}];")
            xs.append(x)
            ys.append(y)
        for u in range(SUN):
            lo, vr = _split_values(b, xs[u], ys[u])
            b.ins(f"st.global.v{SVW}.f32 [{plo}+{u * step}], {{{', '.join(lo)}}};")
            b.ins(f"st.global.v{SVW}.b32 [{pvr}+{u * step}], {{{', '.join(vr)}}};")
        for r_ in (pk, pv, plo, pvr):
            b.ins(f"add.s64 {r_}, {r_}, {SUN * step};")
        pt_ = b.reg("p")
        b.ins(f"sub.u32 {trips}, {trips}, 1;")
        b.ins(f"setp.ne.u32 {pt_}, {trips}, 0;")
        b.ins(f"@{pt_} bra.uni {ltop};")
        # this warp's writes of the chunk, then its release on the group
        b.ins("fence.proxy.async.global;")
        b.ins("bar.warp.sync 0xffffffff;")
        ga4 = b.reg("rd")
        b.ins(f"mul.wide.u32 {ga4}, {grp}, 4;")
        b.ins(f"add.s64 {ga4}, {ga4}, {dn};")
        b.ins(f"@{pl0} red.release.gpu.global.add.u32 [{ga4}], 1;")
        b.ins(f"bra.uni {stop};")
        b.place(send)
        b.ins(f"@{pall} bra.uni {DISPATCH};")
        b.ins(f"bra.uni {END};")

    def wait_split(w):
        """The producers' wait (before the TMA loads of item w's K lo or
        rounded V): every chunk of w's head group is done.  Bounded like
        every wait; a timeout sets the status word and leaves."""
        if not inline:
            return
        g_, a_, o_ = b.reg("r"), b.reg("rd"), b.reg("rd")
        b.ins(f"div.u32 {g_}, {w}, {G * nqu};")
        b.ins(f"mov.u64 {a_}, emmy_split_done;")
        b.ins(f"mul.wide.u32 {o_}, {g_}, 4;")
        b.ins(f"add.s64 {a_}, {a_}, {o_};")
        v_, fl = b.regs("r", 2)
        pw, pf = b.regs("p", 2)
        t0, t1 = b.regs("rd", 2)
        ok, top = b.label("SPLIT_READY"), b.label("SPLIT_WAIT")
        b.ins(f"ld.acquire.gpu.global.u32 {v_}, [{a_}];")
        b.ins(f"setp.ge.u32 {pw}, {v_}, {CH};")
        b.ins(f"@{pw} bra {ok};")
        b.ins(f"mov.u64 {t0}, %globaltimer;")
        b.place(top)
        b.ins("nanosleep.u32 256;")
        b.ins(f"ld.acquire.gpu.global.u32 {v_}, [{a_}];")
        b.ins(f"setp.ge.u32 {pw}, {v_}, {CH};")
        b.ins(f"@{pw} bra {ok};")
        b.ins(f"ld.volatile.shared.u32 {fl}, [{abort}];")
        b.ins(f"setp.ne.u32 {pf}, {fl}, 0;")
        b.ins(f"@{pf} bra {END};")
        b.ins(f"mov.u64 {t1}, %globaltimer;")
        b.ins(f"sub.u64 {t1}, {t1}, {t0};")
        b.ins(f"setp.lt.u64 {pf}, {t1}, {tc.limit_ns};")
        b.ins(f"@{pf} bra {top};")
        tc.raise_abort(STATUS_TIMEOUT + ROLE_SPLIT)
        b.ins(f"bra {END};")
        b.place(ok)
        # the group's generic-proxy writes, acquired above, before this
        # thread's async-proxy (TMA) reads of them
        b.ins("fence.proxy.async.global;")

    # ---- producers: K (hi and lo) on warp 4, V on warp 6 -----------------------
    # Separate threads, so a K slot is refilled as soon as its QK^T chunk is
    # done, not after a V slot of an earlier tile is released by its PV.
    def producer_start(label, names):
        b.place(label)
        b.ins(f"setp.ne.u32 {pr}, {lane}, 0;")
        b.ins(f"@{pr} bra {END};")
        maps = [tc.tmap_address(n) for n in names]
        for tm in maps:
            b.ins(f"fence.proxy.tensormap::generic.acquire.gpu [{tm}], 128;")
            b.ins(f"prefetch.tensormap [{tm}];")
        return maps

    def full_barrier(off, s, nbytes):
        """Announce ``nbytes`` on full barrier off[s] (the leader does, for
        both CTAs of a pair) and return the barrier this CTA's TMA bytes
        count on (the leader's)."""
        if not pair:
            fb = bar_at(off, s)
            tc.arrive_expect_tx(fb, nbytes)
            return fb
        sk = b.label("EXPECTED")
        b.ins(f"@!{lead} bra {sk};")
        tc.arrive_expect_tx(bar_at(off, s), CG * nbytes)
        b.place(sk)
        return remote(lbars, off, s)

    # K: per S tile, DC chunks (32 dims of 128 keys: this CTA's keys, hi and
    # lo; boxes of 64 keys)
    tmKh, tmKl = producer_start(roles[1], ("tmap_Khi", "tmap_Klo"))
    t_kp = b.reg("r")
    b.ins(f"mov.u32 {t_kp}, 0;")

    def prod_k_item(w, _k):
        bh, qu = item_coords(w)
        nkv = n_kv(qu)
        wait_split(w)

        def tile(j):
            k0 = b.reg("r")
            b.ins(f"mul.lo.u32 {k0}, {j}, {BKV};")
            if pair:
                b.ins(f"mad.lo.u32 {k0}, {rank}, {KC_KEYS}, {k0};")
            for c in range(DC):
                s, ph = ring(t_kp, KCH)
                flip = b.reg("r")
                b.ins(f"xor.b32 {flip}, {ph}, 1;")
                tc.wait(bar_at(KE, s), flip, END, ROLE_PRODUCER)
                fb = full_barrier(KF, s, K_SLOT)
                dst = b.reg("r")
                b.ins(f"mad.lo.u32 {dst}, {s}, {K_SLOT}, {base};")
                b.ins(f"add.u32 {dst}, {dst}, {K_RING};")
                x = b.reg("r")
                b.ins(f"mov.u32 {x}, {32 * c};")
                for half, tm in ((0, tmKh), (K_BOX, tmKl)):
                    for kb in range(KC_KEYS // BOX_KEYS):
                        y, d = b.regs("r", 2)
                        b.ins(f"add.u32 {y}, {k0}, {kb * BOX_KEYS};")
                        b.ins(f"add.u32 {d}, {dst}, {half + kb * BOX_KEYS * 128};")
                        tc.tma_load_3d(d, tm, x, y, bh, fb, pair)
                b.ins(f"add.u32 {t_kp}, {t_kp}, 1;")
        kv_loop(nkv, tile, None, "PKKV")

    item_loop(prod_k_item, "PKIT")
    b.ins(f"bra.uni {END};")

    # V: per S tile, VPT chunks of 64 keys (one box per 32 dims)
    (tmV,) = producer_start(roles[3], ("tmap_V",))
    t_vp = b.reg("r")
    b.ins(f"mov.u32 {t_vp}, 0;")

    def prod_v_item(w, _k):
        bh, qu = item_coords(w)
        nkv = n_kv(qu)
        wait_split(w)
        x0 = b.reg("r")                   # this CTA's first head dim
        b.ins(f"mul.lo.u32 {x0}, {rank}, {32 * VDC};")

        def tile(j):
            for v in range(VPT):
                s, ph = ring(t_vp, NVS)
                flip = b.reg("r")
                b.ins(f"xor.b32 {flip}, {ph}, 1;")
                tc.wait(bar_at(VE, s), flip, END, ROLE_PRODUCER)
                fb = full_barrier(VF, s, V_SLOT)
                dst = b.reg("r")
                b.ins(f"mad.lo.u32 {dst}, {s}, {V_SLOT}, {base};")
                b.ins(f"add.u32 {dst}, {dst}, {V_RING};")
                k0 = b.reg("r")
                b.ins(f"mad.lo.u32 {k0}, {j}, {BKV}, {v * VC_KEYS};")
                for c in range(VDC):
                    x, a_ = b.regs("r", 2)
                    b.ins(f"add.u32 {x}, {x0}, {32 * c};")
                    b.ins(f"add.u32 {a_}, {dst}, {c * V_BOX};")
                    tc.tma_load_3d(a_, tmV, x, k0, bh, fb, pair)
                b.ins(f"add.u32 {t_vp}, {t_vp}, 1;")
        kv_loop(nkv, tile, None, "PVKV")

    item_loop(prod_v_item, "PVIT")
    b.ins(f"bra.uni {END};")

    # ---- MMA -------------------------------------------------------------------
    # Two issuing threads.  Warp 5 issues QK(t) into S buffer t%2 (3xTF32),
    # warp 7 issues PV(t) from the P the softmax wrote over that buffer,
    # accumulating in the O columns.  A tcgen05.mma holds its issuing thread
    # ~44 cycles while an N=128 one runs 64 on the tensor core, so one thread
    # issuing all 64 MMAs of a tile, with their waits and commits, left the
    # tensor core idle part of the time; the cost is per thread, and two
    # issuers overlap it.  MMAs of different threads are not ordered against
    # each other: QK(t+2), which overwrites the buffer PV(t) reads, first
    # waits on PE[t%2], which PV(t)'s commit completes.
    def mma_role(label):
        b.place(label)
        b.ins(f"setp.ne.u32 {pr}, {lane}, 0;")
        b.ins(f"@{pr} bra {END};")
        b.ins(f"@!{lead} bra {END};")         # the pair's MMAs are the leader's

    mma = f"tcgen05.mma.cta_group::{CG}.kind::tf32"

    def release(off, s=None):
        """Commit to barrier off(+8s) of this CTA and, in a pair, of the
        peer (the same completed MMAs free or fill both CTAs' buffers)."""
        tc.commit(bar_at(off, s))
        if pair:
            tc.commit(remote(pbars, off, s))
    kdesc = smem_desc_hi(16, 8 * 128, "128B")                  # K, Q lo: K-major rows of 128 B
    vdesc = smem_desc_hi(V_BOX, 4 * 128, "128B_base32B")       # V: N-major, 32-dim box stride

    def preds():
        pt, pf = b.regs("p", 2)
        b.ins(f"setp.eq.u32 {pt}, 0, 0;")
        b.ins(f"setp.ne.u32 {pf}, 0, 0;")
        return pt, pf

    def desc(addr, const):
        a4 = b.reg("r")
        b.ins(f"shr.u32 {a4}, {addr}, 4;")
        b.ins(f"and.b32 {a4}, {a4}, 0x3FFF;")
        d = b.reg("rd")
        b.ins(f"cvt.u64.u32 {d}, {a4};")
        b.ins(f"or.b64 {d}, {d}, 0x{const:016X};")
        return d

    def advance(slot, ph, n):
        """Ring slot and phase parity of the next use (no division)."""
        pw = b.reg("p")
        b.ins(f"add.u32 {slot}, {slot}, 1;")
        b.ins(f"setp.eq.u32 {pw}, {slot}, {n};")
        b.ins(f"@{pw} mov.u32 {slot}, 0;")
        b.ins(f"@{pw} xor.b32 {ph}, {ph}, 1;")

    def s_col(tg):
        c = b.reg("r")
        b.ins(f"and.b32 {c}, {tg}, 1;")
        b.ins(f"mad.lo.u32 {c}, {c}, {C_S1 - C_S0}, {C_S0};")
        b.ins(f"add.u32 {c}, {c}, {tmem};")
        return c

    def buf_phase(tg):
        bi, ph = b.regs("r", 2)
        b.ins(f"and.b32 {bi}, {tg}, 1;")
        b.ins(f"shr.u32 {ph}, {tg}, 1;")
        b.ins(f"and.b32 {ph}, {ph}, 1;")
        return bi, ph

    # -- QK^T issuer (warp 5).  Everything an MMA needs that does not change
    # from tile to tile is computed once: Q lo descriptors, Q hi TMEM
    # addresses, the K ring's base descriptor.
    mma_role(roles[2])
    id_s = b.reg("r")
    b.ins(f"mov.u32 {id_s}, {idesc_tf32(BQ * CG, BKV, False, False)};")
    ptrue, pfalse = preds()
    a_ = b.reg("r")
    b.ins(f"add.u32 {a_}, {base}, {Q_LO};")
    dqlo = desc(a_, kdesc)
    dq = []                               # Q lo descriptor of k-step kk
    for kk in range(D // 8):
        c, w_ = divmod(kk, 4)
        r_ = b.reg("rd")
        b.ins(f"add.s64 {r_}, {dqlo}, {(c * BQ * 128 + w_ * 32) >> 4};")
        dq.append(r_)
    qh = []                               # Q hi TMEM address of k-step kk
    for kk in range(D // 8):
        r_ = b.reg("r")
        b.ins(f"add.u32 {r_}, {tmem}, {C_QHI + 8 * kk};")
        qh.append(r_)
    a_ = b.reg("r")
    b.ins(f"add.u32 {a_}, {base}, {K_RING};")
    dk0 = desc(a_, kdesc)                 # K slot 0 (hi box; lo at + K_BOX)
    ks, kph, t_m, it_m = b.regs("r", 4)   # K ring slot and parity, S tiles, items
    for r_ in (ks, kph, t_m, it_m):
        b.ins(f"mov.u32 {r_}, 0;")

    def qk_item(w, _k):
        bh, qu = item_coords(w)
        nkv = n_kv(qu)
        tc.wait(bar_at(QR), parity(it_m), END, ROLE_MMA)
        b.ins("tcgen05.fence::after_thread_sync;")

        def tile(j):
            # S buffer t%2 is free once PV(t-2), which read its P, is done
            bi, ph = buf_phase(t_m)
            p2 = b.reg("p")
            free = b.label("S_FREE")
            b.ins(f"setp.lt.u32 {p2}, {t_m}, 2;")
            b.ins(f"@{p2} bra.uni {free};")
            b.ins(f"xor.b32 {ph}, {ph}, 1;")
            tc.wait(bar_at(PE, bi), ph, END, ROLE_MMA)
            b.ins("tcgen05.fence::after_thread_sync;")
            b.place(free)
            ts = s_col(t_m)
            for c in range(DC):
                tc.wait(bar_at(KF, ks), kph, END, ROLE_MMA)
                b.ins("tcgen05.fence::after_thread_sync;")
                dk = b.reg("rd")
                b.ins(f"mad.wide.u32 {dk}, {ks}, {K_SLOT >> 4}, {dk0};")
                for w_ in range(4):
                    kk = 4 * c + w_
                    dh, dl = b.regs("rd", 2)
                    b.ins(f"add.s64 {dh}, {dk}, {(w_ * 32) >> 4};")
                    b.ins(f"add.s64 {dl}, {dk}, {(K_BOX + w_ * 32) >> 4};")
                    # hi*hi and hi*lo with Q hi from TMEM, lo*hi with Q lo
                    # from shared memory
                    b.ins(f"{mma} [{ts}], [{qh[kk]}], {dh}, {id_s}, "
                          f"{pfalse if kk == 0 else ptrue};")
                    b.ins(f"{mma} [{ts}], [{qh[kk]}], {dl}, {id_s}, {ptrue};")
                    b.ins(f"{mma} [{ts}], {dq[kk]}, {dh}, {id_s}, {ptrue};")
                release(KE, ks)
                advance(ks, kph, KCH)
            release(SF, bi)
        kv_loop(nkv, tile, t_m, "MKV")
        b.ins(f"add.u32 {it_m}, {it_m}, 1;")
    item_loop(qk_item, "MIT")
    b.ins(f"bra.uni {END};")

    # -- PV issuer (warp 7): O += P V for every S tile, VPT chunks of 64 keys,
    # each released (VE) as soon as its MMAs are done; then OF (per tile),
    # PE (the S buffer is free again) and, after an item's last tile, OFIN.
    mma_role(roles[4])
    id_o = b.reg("r")
    b.ins(f"mov.u32 {id_o}, {idesc_tf32(BQ * CG, D, False, True)};")
    ptrue, _ = preds()
    a_ = b.reg("r")
    b.ins(f"add.u32 {a_}, {base}, {V_RING};")
    dv0 = desc(a_, vdesc)                 # V slot 0
    to = b.reg("r")
    b.ins(f"add.u32 {to}, {tmem}, {C_O};")
    vs, vph, t_p = b.regs("r", 3)         # V ring slot and parity, S tiles
    for r_ in (vs, vph, t_p):
        b.ins(f"mov.u32 {r_}, 0;")

    def pv_item(w, _k):
        bh, qu = item_coords(w)
        nkv = n_kv(qu)
        t0 = b.reg("r")
        b.ins(f"mov.u32 {t0}, {t_p};")

        def tile(j):
            first_pred = b.reg("p")       # accumulate after the item's first tile
            b.ins(f"setp.ne.u32 {first_pred}, {t_p}, {t0};")
            bi, ph = buf_phase(t_p)
            tc.wait(bar_at(PF, bi), ph, END, ROLE_MMA)
            sc = s_col(t_p)
            for v in range(VPT):
                tc.wait(bar_at(VF, vs), vph, END, ROLE_MMA)
                b.ins("tcgen05.fence::after_thread_sync;")
                dv = b.reg("rd")
                b.ins(f"mad.wide.u32 {dv}, {vs}, {V_SLOT >> 4}, {dv0};")
                for kk in range(VC_KEYS // 8):
                    dvk = b.reg("rd")
                    b.ins(f"add.s64 {dvk}, {dv}, {(kk * 8 * 128) >> 4};")
                    pa = b.reg("r")
                    b.ins(f"add.u32 {pa}, {sc}, {v * VC_KEYS + 8 * kk};")
                    b.ins(f"{mma} [{to}], [{pa}], {dvk}, {id_o}, "
                          f"{first_pred if v == 0 and kk == 0 else ptrue};")
                release(VE, vs)
                advance(vs, vph, NVS)
            release(OF)
            tc.commit(bar_at(PE, bi))     # only this CTA's QK^T issuer waits on it
        kv_loop(nkv, tile, t_p, "PKV")
        release(OFIN)
    item_loop(pv_item, "PIT")
    b.ins(f"bra.uni {END};")

    # ---- softmax / lazy correction / epilogue ------------------------------------
    b.place(roles[0])
    q4 = b.reg("r")
    b.ins(f"shl.b32 {q4}, {warp}, 21;")              # (32*warp) << 16: TMEM lane base
    lbase = b.reg("r")
    b.ins(f"add.u32 {lbase}, {tmem}, {q4};")
    t_x, it_x = b.regs("r", 2)
    b.ins(f"mov.u32 {t_x}, 0;")
    b.ins(f"mov.u32 {it_x}, 0;")
    qscale = plan.scale * LOG2E
    if gather:
        # the destination pointers are read where they are used (the
        # softmax's 128 scores per thread leave no registers to hold them)
        gn, grow0 = b.regs("r", 2)
        b.ins(f"ld.global.u32 {gn}, [emmy_gather_n];")
        b.ins(f"ld.global.u32 {grow0}, [emmy_gather_row0];")
        # this warp's stage: written at row = lane, read at row lane/8 (+4i),
        # 16-byte column chunk lane%8
        st_w, st_r, sub_row, sub_col = b.regs("r", 4)
        b.ins(f"mad.lo.u32 {st_w}, {warp}, {EPI_WARP}, {base};")
        b.ins(f"add.u32 {st_w}, {st_w}, {EPI};")
        b.ins(f"shr.u32 {sub_row}, {lane}, 3;")
        b.ins(f"and.b32 {sub_col}, {lane}, 7;")
        b.ins(f"mad.lo.u32 {st_r}, {sub_row}, {EPI_ROW}, {st_w};")
        b.ins(f"mad.lo.u32 {st_r}, {sub_col}, 16, {st_r};")
        b.ins(f"shl.b32 {sub_col}, {sub_col}, 2;")
        b.ins(f"mad.lo.u32 {st_w}, {lane}, {EPI_ROW}, {st_w};")
    ninf = "0fFF800000"

    def tree(vals, op):
        """Pairwise reduction (log depth) of registers ``vals``."""
        vals = list(vals)
        while len(vals) > 1:
            nxt = []
            for i in range(0, len(vals) - 1, 2):
                r = b.reg("f")
                b.ins(f"{op}.f32 {r}, {vals[i]}, {vals[i + 1]};")
                nxt.append(r)
            if len(vals) % 2:
                nxt.append(vals[-1])
            vals = nxt
        return vals[0]

    def to_leader(off, s=None):
        """Arrive on barrier off(+8s) of the MMA-issuing CTA: this CTA's,
        or the pair leader's.  With one arrival per warp, the warp first
        synchronises (its lanes' TMEM and shared-memory writes, each already
        complete and fenced, are then ordered before lane 0's arrival), and
        lane 0 arrives for all 32."""
        if ARRIVALS == 4:
            b.ins("bar.warp.sync 0xffffffff;")
            pa = b.reg("p")
            b.ins(f"setp.eq.u32 {pa}, {lane}, 0;")
            sk = b.label("ARRIVED")
            b.ins(f"@!{pa} bra {sk};")
        if pair:
            tc.arrive_cluster(remote(lbars, off, s))
        else:
            tc.arrive(bar_at(off, s))
        if ARRIVALS == 4:
            b.place(sk)
            b.ins("bar.warp.sync 0xffffffff;")

    def row_of(w):
        """Item w: (bh, query unit, this CTA's query tile, this thread's
        query, in range?, row byte offset)."""
        bh, qu = item_coords(w)
        qt = own_tile(qu)
        qi = b.reg("r")                          # this thread's query index
        b.ins(f"mad.lo.u32 {qi}, {qt}, {BQ}, {tid};")
        pq = b.reg("p")
        b.ins(f"setp.lt.u32 {pq}, {qi}, {S};")
        rowoff = b.reg("rd")
        b.ins(f"mul.wide.u32 {rowoff}, {bh}, {S * D * 4};")
        qo = b.reg("rd")
        b.ins(f"mul.wide.u32 {qo}, {qi}, {D * 4};")
        b.ins(f"add.s64 {rowoff}, {rowoff}, {qo};")
        return bh, qu, qt, qi, pq, rowoff

    def stage_q(w):
        """Q of item w into TMEM (hi) and shared memory (lo), then Q ready.
        Called for the next item as soon as the current item's last QK^T
        is complete (its S tile has been seen), so the QK^T issuer can start
        the next item while this item's epilogue runs."""
        bh, qu, qt, qi, pq, rowoff = row_of(w)
        # Q * scale * log2(e) -> tf32 hi (TMEM) and lo (shared memory): scores
        # come out in log2 units.  Row r of Q lo goes to row r of each 32-dim
        # box with the 128-byte swizzle (16-byte unit u at u ^ (r % 8)), the
        # layout the K-major smem descriptor describes.
        qrow = b.reg("r")
        b.ins(f"mad.lo.u32 {qrow}, {tid}, 128, {base};")
        b.ins(f"add.u32 {qrow}, {qrow}, {Q_LO};")
        r8 = b.reg("r")
        b.ins(f"and.b32 {r8}, {tid}, 7;")
        # 1. the warp loads its 32 rows coalesced (lane l: dims 4l..4l+3 of
        #    a row, 512 bytes per instruction) into the Q lo region, in the
        #    swizzled layout (32-dim box c = l / 8, 16-byte unit u = l % 8)
        wrow0 = b.reg("r")                      # the warp's first row
        b.ins(f"and.b32 {wrow0}, {tid}, 0xFFFFFFE0;")
        lanes = D // 4
        pl_ = b.reg("p")
        b.ins(f"setp.lt.u32 {pl_}, {lane}, {lanes};")
        lc, lu = b.regs("r", 2)
        b.ins(f"shr.u32 {lc}, {lane}, 3;")
        b.ins(f"and.b32 {lu}, {lane}, 7;")
        # global address of (the warp's first row, dim 4 * lane):
        # rowoff is this thread's row, so subtract tid rows, add wrow0 rows
        wb, t1, w1 = b.regs("rd", 3)
        b.ins(f"mul.wide.u32 {t1}, {tid}, {D * 4};")
        b.ins(f"mul.wide.u32 {w1}, {wrow0}, {D * 4};")
        b.ins(f"sub.s64 {wb}, {rowoff}, {t1};")
        b.ins(f"add.s64 {wb}, {wb}, {w1};")
        loff = b.reg("rd")
        b.ins(f"mul.wide.u32 {loff}, {lane}, 16;")
        b.ins(f"add.s64 {wb}, {wb}, {loff};")
        b.ins(f"add.s64 {wb}, {wb}, {pQ};")
        # the warp's first row within the sequence (qi - tid + wrow0); rows
        # at or past S (a partial last query tile) are not loaded
        qrow0 = b.reg("r")
        b.ins(f"sub.u32 {qrow0}, {qi}, {tid};")
        b.ins(f"add.u32 {qrow0}, {qrow0}, {wrow0};")
        vals = []
        for i in range(32):
            v4 = b.regs("r", 4)
            for e in range(4):
                b.ins(f"mov.b32 {v4[e]}, 0;")
            rr = b.reg("r")
            b.ins(f"add.u32 {rr}, {qrow0}, {i};")
            pr_ = b.reg("p")
            b.ins(f"setp.lt.and.u32 {pr_}, {rr}, {S}, {pl_};")
            b.ins(f"@{pr_} ld.global.nc.v4.b32 {{{', '.join(v4)}}}, [{wb}+{i * D * 4}];")
            vals.append(v4)
        # smem address of (row wrow0 + i, box lc, unit lu): swizzle by row % 8
        sbase = b.reg("r")
        b.ins(f"mad.lo.u32 {sbase}, {lc}, {BQ * 128}, {base};")
        b.ins(f"add.u32 {sbase}, {sbase}, {Q_LO};")
        b.ins(f"mad.lo.u32 {sbase}, {wrow0}, 128, {sbase};")
        pst = b.reg("p")
        b.ins(f"setp.lt.u32 {pst}, {lane}, {lanes};")
        for i in range(32):
            ua = b.reg("r")
            b.ins(f"xor.b32 {ua}, {lu}, {i % 8};")
            b.ins(f"shl.b32 {ua}, {ua}, 4;")
            b.ins(f"add.u32 {ua}, {ua}, {sbase};")
            b.ins(f"@{pst} st.shared.v4.b32 [{ua}+{i * 128}], {{{', '.join(vals[i])}}};")
        b.ins("bar.warp.sync 0xffffffff;")
        # 2. each thread reads its own row back, splits it, writes lo in place
        for c in range(DC):
            raw = []
            addrs = []
            for u in range(8):
                ua = b.reg("r")
                b.ins(f"xor.b32 {ua}, {r8}, {u};")
                b.ins(f"shl.b32 {ua}, {ua}, 4;")
                b.ins(f"add.u32 {ua}, {ua}, {qrow};")
                v4 = b.regs("f", 4)
                b.ins(f"ld.shared.v4.f32 {{{', '.join(v4)}}}, [{ua}+{c * BQ * 128}];")
                raw += v4
                addrs.append(ua)
            x = raw
            hi = b.regs("r", 32)
            lo = b.regs("r", 32)
            for e in range(32):
                # hi = x rounded to nearest tf32 (ties away), as two integer
                # operations (cvt.rna is several times dearer here, on the
                # path between items); lo = x - hi is exact.  A NaN or an
                # infinity in Q still reaches S through lo, as with cvt.rna.
                b.ins(f"mul.f32 {x[e]}, {x[e]}, {f32_hex(qscale)};")
                xb = b.reg("r")
                b.ins(f"mov.b32 {xb}, {x[e]};")
                b.ins(f"add.u32 {hi[e]}, {xb}, 4096;")
                b.ins(f"and.b32 {hi[e]}, {hi[e]}, 0xFFFFE000;")
                hf, lf = b.regs("f", 2)
                b.ins(f"mov.b32 {hf}, {hi[e]};")
                b.ins(f"sub.f32 {lf}, {x[e]}, {hf};")
                b.ins(f"mov.b32 {lo[e]}, {lf};")
            b.ins(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{lbase}+{C_QHI + 32 * c}], "
                  f"{{{', '.join(hi)}}};")
            for u in range(8):
                b.ins(f"st.shared.v4.b32 [{addrs[u]}+{c * BQ * 128}], "
                      f"{{{', '.join(lo[4 * u:4 * u + 4])}}};")
        b.ins("tcgen05.wait::st.sync.aligned;")
        b.ins("fence.proxy.async.shared::cta;")           # Q lo, for the tensor core
        b.ins("tcgen05.fence::before_thread_sync;")
        to_leader(QR)

    def prefetch_q(w):
        """One thread asks L2 for item w's Q block (128 contiguous rows),
        an item ahead of its staging, so the staging loads hit L2."""
        bh, qu = item_coords(w)
        qt = own_tile(qu)
        r0, nrow = b.regs("r", 2)
        b.ins(f"mad.lo.u32 {r0}, {bh}, {S}, 0;")
        b.ins(f"mad.lo.u32 {r0}, {qt}, {BQ}, {r0};")
        b.ins(f"mul.lo.u32 {nrow}, {qt}, {BQ};")
        b.ins(f"sub.u32 {nrow}, {S}, {nrow};")
        b.ins(f"min.u32 {nrow}, {nrow}, {BQ};")
        b.ins(f"mul.lo.u32 {nrow}, {nrow}, {D * 4};")
        qa = b.reg("rd")
        b.ins(f"mul.wide.u32 {qa}, {r0}, {D * 4};")
        b.ins(f"add.s64 {qa}, {qa}, {pQ};")
        b.ins(f"cp.async.bulk.prefetch.L2.global [{qa}], {nrow};")

    def soft_item(w, kpos):
        bh, qu, qt, qi, pq, rowoff = row_of(w)
        nkv = n_kv(qu)
        kn = b.reg("r")                   # the next item's position
        b.ins(f"add.u32 {kn}, {kpos}, {kstep};")
        pp = b.reg("p")
        nopf = b.label("NO_Q_PREFETCH")
        b.ins(f"setp.ge.u32 {pp}, {kn}, {kend};")
        b.ins(f"@{pp} bra.uni {nopf};")
        b.ins(f"setp.ne.u32 {pp}, {tid}, 0;")
        b.ins(f"@{pp} bra {nopf};")
        prefetch_q(item_at(kn))
        b.place(nopf)
        b.ins("bar.warp.sync 0xffffffff;")
        qfirst = b.reg("r")                      # the item's first query
        b.ins(f"mul.lo.u32 {qfirst}, {qt}, {BQ};")
        m, l_ = b.regs("f", 2)            # m: the max P is scaled by (log2 units)
        b.ins(f"mov.f32 {m}, {ninf};")
        b.ins(f"mov.f32 {l_}, 0f00000000;")
        t0 = b.reg("r")
        b.ins(f"mov.u32 {t0}, {t_x};")

        def tile(j):
            bi, ph = buf_phase(t_x)
            tc.wait(bar_at(SF, bi), ph, END, ROLE_SOFTMAX, uniform=True)
            b.ins("tcgen05.fence::after_thread_sync;")
            scol = b.reg("r")
            b.ins(f"mad.lo.u32 {scol}, {bi}, {C_S1 - C_S0}, {lbase};")
            b.ins(f"add.u32 {scol}, {scol}, {C_S0};")
            sv = b.regs("f", BKV)
            for h in range(BKV // 32):
                b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(sv[32 * h:32 * h + 32])}}}, "
                      f"[{scol}+{32 * h}];")
            b.ins("tcgen05.wait::ld.sync.aligned;")
            # mask only tiles that reach past the item's first query (the
            # diagonal) or past the sequence end; the branch is uniform
            k0 = b.reg("r")
            b.ins(f"mul.lo.u32 {k0}, {j}, {BKV};")
            kl_ = b.reg("r")
            b.ins(f"add.u32 {kl_}, {k0}, {BKV - 1};")
            pmask = b.reg("p")
            if plan.causal:
                b.ins(f"setp.gt.u32 {pmask}, {kl_}, {qfirst};")
            else:
                b.ins(f"setp.ge.u32 {pmask}, {kl_}, {S};")
            nomask = b.label("NOMASK")
            b.ins(f"@!{pmask} bra.uni {nomask};")
            lim = b.reg("r")                      # keys c < lim are visible
            if plan.causal:
                b.ins(f"add.u32 {lim}, {qi}, 1;")
                b.ins(f"min.u32 {lim}, {lim}, {S};")
            else:
                b.ins(f"mov.u32 {lim}, {S};")
            b.ins(f"sub.u32 {lim}, {lim}, {k0};")
            for e in range(BKV):
                pc = b.reg("p")
                b.ins(f"setp.lt.s32 {pc}, {e}, {lim};")
                b.ins(f"selp.f32 {sv[e]}, {sv[e]}, {ninf}, {pc};")
            b.place(nomask)
            mx = b.reg("f")
            b.ins(f"max.f32 {mx}, {tree(sv, 'max')}, {m};")
            # lazy rescaling: keep the reference max unless the tile's max
            # exceeds it by more than 2^8 (P stays below 256)
            thr = b.reg("f")
            b.ins(f"add.f32 {thr}, {m}, 0f41000000;")
            need = b.reg("p")
            b.ins(f"setp.gt.f32 {need}, {mx}, {thr};")
            corr = b.reg("f")
            dm = b.reg("f")
            b.ins(f"sub.f32 {dm}, {m}, {mx};")
            b.ins(f"ex2.approx.f32 {corr}, {dm};")
            pinf = b.reg("p")
            b.ins(f"setp.eq.f32 {pinf}, {m}, {ninf};")
            b.ins(f"selp.f32 {corr}, 0f00000000, {corr}, {pinf};")
            b.ins(f"selp.f32 {corr}, {corr}, 0f3F800000, {need};")
            pany = b.reg("p")
            pfirst = b.reg("p")
            b.ins(f"setp.eq.u32 {pfirst}, {t_x}, {t0};")
            b.ins(f"vote.sync.any.pred {pany}, {need}, 0xffffffff;")
            no_rs = b.label("NO_RESCALE")
            b.ins(f"@{pfirst} bra.uni {no_rs};")
            b.ins(f"@!{pany} bra.uni {no_rs};")
            prev = b.reg("r")
            b.ins(f"sub.u32 {prev}, {t_x}, 1;")
            tc.wait(bar_at(OF), parity(prev), END, ROLE_SOFTMAX, uniform=True)
            b.ins("tcgen05.fence::after_thread_sync;")
            for c in range(DC):
                ov = b.regs("f", 32)
                b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, "
                      f"[{lbase}+{C_O + 32 * c}];")
                b.ins("tcgen05.wait::ld.sync.aligned;")
                for e in range(32):
                    b.ins(f"mul.f32 {ov[e]}, {ov[e]}, {corr};")
                b.ins(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{lbase}+{C_O + 32 * c}], "
                      f"{{{', '.join(ov)}}};")
            b.ins("tcgen05.wait::st.sync.aligned;")
            b.place(no_rs)
            b.ins(f"mul.f32 {l_}, {l_}, {corr};")
            b.ins(f"selp.f32 {m}, {mx}, {m}, {need};")
            msub = b.reg("f")
            pm = b.reg("p")
            b.ins(f"setp.eq.f32 {pm}, {m}, {ninf};")
            b.ins(f"selp.f32 {msub}, 0f00000000, {m}, {pm};")
            for e in range(BKV):
                t_ = b.reg("f")
                b.ins(f"sub.f32 {t_}, {sv[e]}, {msub};")
                b.ins(f"ex2.approx.ftz.f32 {sv[e]}, {t_};")
                # P as the tensor core will read it (tf32: low 13 bits
                # dropped); the row sum below uses the same values, so
                # O / l carries no truncation bias
                b.ins(f"and.b32 {sv[e]}, {sv[e]}, 0xFFFFE000;")
            for h in range(BKV // 32):
                b.ins(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{scol}+{32 * h}], "
                      f"{{{', '.join(sv[32 * h:32 * h + 32])}}};")
            b.ins(f"add.f32 {l_}, {l_}, {tree(sv, 'add')};")
            b.ins("tcgen05.wait::st.sync.aligned;")
            b.ins("tcgen05.fence::before_thread_sync;")
            to_leader(PF, bi)
        kv_loop(nkv, tile, t_x, "XKV")
        # the next item's Q: its buffers are free once this item's last
        # QK^T is complete, which the last tile's S wait has seen
        pn = b.reg("p")
        nonext = b.label("NO_NEXT_Q")
        b.ins(f"setp.ge.u32 {pn}, {kn}, {kend};")
        b.ins(f"@{pn} bra.uni {nonext};")
        stage_q(item_at(kn))
        b.place(nonext)
        # epilogue: wait for the item's last PV (one OFIN phase per item),
        # out = O * (1 / l)
        tc.wait(bar_at(OFIN), parity(it_x), END, ROLE_SOFTMAX, uniform=True)
        b.ins("tcgen05.fence::after_thread_sync;")
        il = b.reg("f")
        b.ins(f"rcp.rn.f32 {il}, {l_};")
        oaddr = b.reg("rd")
        b.ins(f"add.s64 {oaddr}, {rowoff}, {pO};")
        if gather:
            # rows of this warp's 32 queries in the [B*H*S, D] view
            rbase = b.reg("r")
            b.ins(f"mad.lo.u32 {rbase}, {qt}, {BQ}, {sub_row};")
            b.ins(f"mad.lo.u32 {rbase}, {warp}, 32, {rbase};")
            pbase = b.reg("r")
            b.ins(f"mad.lo.u32 {pbase}, {bh}, {S}, {grow0};")
            for c in range(DC):
                ov = b.regs("f", 32)
                b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, "
                      f"[{lbase}+{C_O + 32 * c}];")
                b.ins("tcgen05.wait::ld.sync.aligned;")
                for g in range(8):
                    v4 = b.regs("f", 4)
                    for e in range(4):
                        b.ins(f"mul.f32 {v4[e]}, {ov[4 * g + e]}, {il};")
                    b.ins(f"st.shared.v4.f32 [{st_w}+{16 * g}], {{{', '.join(v4)}}};")
                b.ins("bar.warp.sync 0xffffffff;")
                coff = b.reg("rd")
                col = b.reg("r")
                b.ins(f"add.u32 {col}, {sub_col}, {32 * c};")
                b.ins(f"mul.wide.u32 {coff}, {col}, 4;")
                for i in range(8):
                    w = b.regs("f", 4)
                    b.ins(f"ld.shared.v4.f32 {{{', '.join(w)}}}, [{st_r}+{4 * i * EPI_ROW}];")
                    qr = b.reg("r")
                    b.ins(f"add.u32 {qr}, {rbase}, {4 * i};")
                    pr = b.reg("p")
                    b.ins(f"setp.lt.u32 {pr}, {qr}, {S};")
                    b.ins(f"add.u32 {qr}, {qr}, {pbase};")
                    ro = b.reg("rd")
                    b.ins(f"mul.wide.u32 {ro}, {qr}, {D * 4};")
                    b.ins(f"add.s64 {ro}, {ro}, {coff};")
                    for d in range(gather):
                        od, gd, pd = b.reg("rd"), b.reg("rd"), b.reg("p")
                        b.ins(f"ld.global.u64 {gd}, [emmy_gather_dst+{8 * d}];")
                        b.ins(f"add.s64 {od}, {ro}, {gd};")
                        b.ins(f"setp.lt.and.u32 {pd}, {d}, {gn}, {pr};")
                        b.ins(f"@{pd} st.global.v4.f32 [{od}], {{{', '.join(w)}}};")
                b.ins("bar.warp.sync 0xffffffff;")
        for c in range(0 if gather else DC):
            ov = b.regs("f", 32)
            b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, "
                  f"[{lbase}+{C_O + 32 * c}];")
            b.ins("tcgen05.wait::ld.sync.aligned;")
            # one thread writes its row: 32-byte stores (PTX ISA 8.8) fill
            # whole sectors and halve the store instructions; the epilogue
            # shares the memory pipe with the MMA threads' mbarrier polls as
            # the next item starts
            for g in range(32 // VW):
                vv = b.regs("f", VW)
                for e in range(VW):
                    b.ins(f"mul.f32 {vv[e]}, {ov[VW * g + e]}, {il};")
                b.ins(f"@{pq} st.global.v{VW}.f32 [{oaddr}+{(32 * c + VW * g) * 4}], "
                      f"{{{', '.join(vv)}}};")
        b.ins("tcgen05.fence::before_thread_sync;")
        b.ins(f"add.u32 {it_x}, {it_x}, 1;")
    pfq = b.reg("p")
    noq = b.label("NO_FIRST_Q")
    b.ins(f"setp.ge.u32 {pfq}, {kbeg}, {kend};")
    b.ins(f"@{pfq} bra.uni {noq};")
    stage_q(item_at(kbeg))                # the first item's Q
    b.place(noq)
    item_loop(soft_item, "XIT")

    # ---- teardown -----------------------------------------------------------------
    b.place(END)
    # the PV issuer's MMAs (a commit covers only its own thread's) are done
    # before the block's last barrier; warp 5 then drains its own and frees
    # TMEM
    pd, pdl = b.reg("p"), b.label("PV_DRAINED")
    b.ins(f"setp.eq.u32 {pd}, {tid}, 224;")
    b.ins(f"and.pred {pd}, {pd}, {lead};")
    b.ins(f"@!{pd} bra {pdl};")
    tc.commit(f"{bars}+{DRAIN2}")
    tc.wait(f"{bars}+{DRAIN2}", 0, pdl, ROLE_MMA, peer=False)
    b.place(pdl)
    b.ins("bar.warp.sync 0xffffffff;")
    b.ins("bar.sync 0;")
    fin = b.label("FIN")
    b.ins(f"setp.ne.u32 {p}, {warp}, 5;")
    b.ins(f"@{p} bra {fin};")
    b.ins("bar.warp.sync 0xffffffff;")
    pl = b.reg("p")
    dl = b.label("DRAIN_DONE")
    b.ins(f"setp.ne.u32 {pl}, {lane}, 0;")
    b.ins(f"@{pl} bra {dl};")
    if pair:
        # the follower reports that it is done and then waits until the
        # leader's MMAs (which write its TMEM and read its shared memory)
        # have drained; the leader drains, waits for the follower, answers
        fl = b.label("LEADER_FIN")
        b.ins(f"@{lead} bra {fl};")
        tc.arrive_cluster(remote(pbars, FIN))
        tc.wait(f"{bars}+{FIN}", 0, dl, ROLE_MMA, peer=False)
        b.ins(f"bra.uni {dl};")
        b.place(fl)
        tc.commit(f"{bars}+{DRAIN}")
        tc.wait(f"{bars}+{DRAIN}", 0, dl, ROLE_MMA, peer=False)
        tc.wait(f"{bars}+{FIN}", 0, dl, ROLE_MMA, peer=False)
        tc.arrive_cluster(remote(pbars, FIN))
    else:
        tc.commit(f"{bars}+{DRAIN}")
        tc.wait(f"{bars}+{DRAIN}", 0, dl, ROLE_MMA)
    b.place(dl)
    b.ins("bar.warp.sync 0xffffffff;")
    b.ins("tcgen05.fence::after_thread_sync;")
    tc.tmem_dealloc(tmem, TMEM_COLS)
    b.place(fin)

    pre_elems = PG * G * S * D if inline else B * H * S * D
    ptx = b.render() + "\n" + emit_kv_prepass(comp.target, comp.ptx_version, split_entry,
                                              pre_elems,
                                              split_groups=(NG, CH, PG) if inline else None)

    pairs = B * H * (S * (S + 1) // 2 if plan.causal else S * S)
    kv_tiles = 0                      # (128-query tile, 128-key tile) products issued
    for qu in range(nqu):
        keys = min(S, (qu + 1) * BQ * CG) if plan.causal else S
        kv_tiles += CG * -(-keys // BKV)
    kv_tiles *= B * H
    # tensor work actually issued: S (3 products) and PV (1 product) per key tile
    issued = kv_tiles * (3 * 2 * BQ * BKV * D + 2 * BQ * D * BKV)
    kbytes = B * H * S * D * 4
    tmap = lambda g, arg, sw: {"global": g, "arg": arg, "dtype": "f32",  # noqa: E731
                               "dims": [D, S, B * H], "strides": [D * 4, S * D * 4],
                               "box": [32, BOX_KEYS, 1], "swizzle": sw}
    sidecar = {
        "category": "attention",
        "grid": [CG * min(items, 148 // CG), 1, 1],
        "block": [TL, 1, 1],
        "shared_bytes": SMEM,
        "cluster": [CG, 1, 1],
        "scratch": [{"name": "k_lo", "bytes": kbytes},
                    {"name": "v_r", "bytes": kbytes}],
        "prelaunch": [split_launch(split_entry, [plan.k, plan.v, "@k_lo", "@v_r"],
                                   pre_elems, max_blocks=148 * 16,
                                   vec=8 if wide_vectors(comp.ptx_version) else 4)],
        "inline_split": {"groups": NG, "chunks_per_group": CH,
                         "warps": list(range(8, 8 + SW))} if inline else None,
        # setmaxnreg shares: registers per thread at launch, and the total the
        # warpgroups hold after the split, for the tuned block and the
        # meta.json one (the runtime refuses a build with fewer at launch)
        "register_split": {"launch": REG_LAUNCH, "softmax": REG_SOFTMAX, "issue": REG_ISSUE,
                           "registers_by_block": {
                               str(TL): 128 * (REG_SOFTMAX + REG_ISSUE) + 32 * SW * REG_LAUNCH,
                               str(T): 128 * (REG_SOFTMAX + REG_ISSUE)}} if inline else None,
        "tensormaps": [tmap("tmap_Khi", plan.k, "128B"),     # K itself: hi = K, low bits dropped
                       tmap("tmap_Klo", "@k_lo", "128B"),
                       tmap("tmap_V", "@v_r", "128B_atom32B")],
        "algorithmic_flops": 4 * pairs * D,
        "tensor_flops_issued": issued,
        "tile": [BQ * CG, BKV, D],
        "cta_group": CG,
        "status_word": "emmy_status",
    }
    if gather:
        sidecar["gather"] = {"max_destinations": gather, "destinations": "emmy_gather_dst",
                             "count": "emmy_gather_n", "row0": "emmy_gather_row0",
                             "writes_out": False}
    return ptx, sidecar
