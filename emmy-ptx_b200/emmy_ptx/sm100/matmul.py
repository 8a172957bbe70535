"""Matmul category: C[M,N] = A[M,K] @ B[K,N] in f32 on the tcgen05 tensor cores.

Recognised IR: a kernel with inputs A [M, K] and B [K, N] (f32) and output
C [M, N] (f32) whose body multiplies values taken from A and from B
(directly, or through shared-memory tiles staged with cp.async) and
accumulates the products with a ``sum`` Accum -- the reference's SIMT GEMM
lowering (compiler.py:1649-1659 accumulation, 1761-1867 K loops, 2014-2040
cp.async staging) -- and writes C.  Parity with the IR's semantics is what
the tests check against the oracle.

Generated kernel (sm_100a), persistent over 128 x BN output tiles:

* f32 (3xTF32): the tensor core reads an f32 operand as tf32 by dropping
  its low 13 bits, so A and B themselves are the hi operands (hi = x with
  those bits cleared), and two pre-pass entries (``<entry>_split_a``,
  ``_split_b``) write only ``lo = x - hi`` (exact) to scratch memory.  Each
  operand tile is used by many output tiles, so splitting inside the kernel
  would repeat the work (and two warps doing it could not keep up with the
  tensor core).
* warp 0, one thread: TMA producer.  A tiles (K-major, 64-byte swizzle,
  128 rows x 16 f32; hi and lo) and B tiles (N-major, 128-byte swizzle with
  32-byte atoms -- the only N-major layout tcgen05 accepts for 32-bit
  operands -- BN/32 boxes of 32 f32 x 16 rows; hi and lo) land in a 4-stage
  shared-memory ring, signalled on ``full[s]`` mbarriers with transaction
  counts.  bf16/f16: A K-major and B N-major with the 128-byte swizzle, 64
  elements per 128-byte row, no split.
* warp 1, one thread: ``tcgen05.mma.cta_group::1`` M=128 N=BN into a TMEM
  accumulator -- ``kind::tf32`` K=8 with three products per k-slice
  (hi*hi + hi*lo + lo*hi), or ``kind::f16`` K=16 with one;
  ``tcgen05.commit`` frees the stage (``empty[s]``) and, at the end of a
  tile, hands the accumulator to the epilogue.  Two TMEM accumulators
  (2 x BN columns) let the next tile's MMAs overlap the epilogue of the
  previous one.
* warps 4-7: epilogue.  ``tcgen05.ld.32x32b.x32`` moves 32 columns of a
  warp's 32 TMEM lanes (rows) into registers; 16-byte stores to C (or, in
  the all-gather variant, row-contiguous stores into every rank's C).

Every mbarrier wait is bounded (see tc.py); on timeout the kernel records a
status code and tears down, freeing its TMEM.
"""

from __future__ import annotations

from dataclasses import dataclass

from .. import ir as I
from .common import NoMatch, declare_params, launch_block
from .ops import dtype_name
from .ptx import KernelBuilder
from .tc import (STATUS_NO_PREPASS, TC, emit_tf32_split, idesc_f8, idesc_f16, idesc_tf32,
                 smem_desc_hi, split_launch)

BM = 128
BK = 16
STAGES = 4
PAIR_STAGES = 6          # a pair's stages are smaller (half of each B tile per CTA)
GROUP_M = 8
PAIR = True              # CTA pairs (tcgen05 cta_group::2) where the shapes allow
ROLE_PRODUCER, ROLE_MMA, ROLE_EPILOGUE, ROLE_TEARDOWN = 1, 2, 4, 5
SPLIT_K_CHOICES = (1, 2)      # K slices per output tile (f32), see choose_split_k
SPLIT_K_MIN_K = 1024          # at least this much K per slice
SPLIT_K_MIN_GAIN = 0.05       # wave efficiency a split must add to be used


def wave_efficiency(units: int, slots: int) -> float:
    """Busy fraction of ``slots`` concurrent workers over ``units`` equal
    work units (the last wave partly idle)."""
    return units / (-(-units // slots) * slots)


def choose_split_k(ntiles: int, slots: int, k: int, bk: int) -> int:
    """K slices per tile for an f32 matmul whose tiles fill the GPU badly:
    a 2048 x 8192 shard has 256 pair tiles for 74 CTA pairs (3.46 waves,
    0.865 busy); cut in two along K it is 512 units in 6.92 waves (0.988),
    and measured 1.10 against 1.16 ms.  A slice writes its partial tile to
    scratch and a reduce entry sums the slices, so a split must gain
    SPLIT_K_MIN_GAIN of wave efficiency.  Four slices of a 1024-row shard
    (0.865 -> 0.988 busy) measured no faster (0.607 against 0.609 ms): the
    partial tiles and their sum cost what the fuller waves save."""
    best, best_eff = 1, wave_efficiency(ntiles, slots)
    for s in SPLIT_K_CHOICES[1:]:
        if k % (s * bk) or k // s < SPLIT_K_MIN_K:
            continue
        e = wave_efficiency(ntiles * s, slots)
        if e > best_eff + SPLIT_K_MIN_GAIN:
            best, best_eff = s, e
    return best


@dataclass
class MatmulPlan:
    m: int
    n: int
    k: int
    a: str
    b: str
    c: str
    dtype: str = "f32"           # A and B: f32 (3xTF32), f16 / bf16 (kind::f16),
    #                              e4m3 / e5m2 fp8 codes (kind::f8f6f4)


def match(comp) -> MatmulPlan:
    ins, outs = list(comp.kernel.inputs), list(comp.kernel.outputs)
    if len(ins) != 2 or len(outs) != 1:
        raise NoMatch("matmul has two inputs and one output")
    a, b_, c = ins[0], ins[1], outs[0]
    sa, sb, sc = comp.shape_of(a), comp.shape_of(b_), comp.shape_of(c)
    if len(sa) != 2 or len(sb) != 2 or len(sc) != 2:
        raise NoMatch("matmul operands are matrices")
    M, K = sa
    K2, N = sb
    if K != K2 or sc != [M, N]:
        raise NoMatch("shapes are not [M,K] @ [K,N] -> [M,N]")
    da, db = comp.dtype_of(a), comp.dtype_of(b_)
    if comp.dtype_of(c) != "f32" or da != db or da not in ("f32", "f16", "bf16", "u8"):
        raise NoMatch("A and B both f32, f16, bf16 or fp8 codes, C f32")
    # the body must take products of A-derived and B-derived values and sum them
    src = {}            # smem buffer -> global tensor it stages
    origin = {}         # value name -> tensor it was loaded from
    decoded = {}        # tensor -> fp8 format its codes are decoded as
    product = set()
    summed = False
    writes_c = False
    for s in I.walk(comp.kernel.body):
        if isinstance(s, I.CpAsyncCopy):
            src[s.smem] = s.src
        elif isinstance(s, I.Load):
            t = src.get(s.input, s.input)
            for nm in s.names:
                origin[nm] = t
        elif isinstance(s, I.Assign) and getattr(s.op, "name", s.op) in (
                "from_f8e4m3", "from_f8e5m2") and len(s.args) == 1 and s.args[0] in origin:
            t = origin[s.args[0]]
            origin[s.name] = t
            decoded[t] = "e4m3" if s.op.name == "from_f8e4m3" else "e5m2"
        elif isinstance(s, I.Assign) and getattr(s.op, "name", s.op) == "multiply" \
                and len(s.args) == 2:
            if {origin.get(s.args[0]), origin.get(s.args[1])} == {a, b_}:
                product.add(s.name)
        elif isinstance(s, I.Accum) and getattr(s.op, "name", s.op) in ("sum", "add"):
            if s.value in product:
                summed = True
        elif isinstance(s, I.Write) and s.output == c:
            writes_c = True
    if not (summed and writes_c):
        raise NoMatch("no sum of A*B products written to C")
    if da == "u8":
        fmts = {decoded.get(a), decoded.get(b_)}
        if len(fmts) != 1 or None in fmts:
            raise NoMatch("byte operands must both be decoded with one fp8 format")
        da = fmts.pop()
    per16 = 16 // {"f32": 4, "f16": 2, "bf16": 2}.get(da, 1)
    if N % per16 or K % per16:
        raise NoMatch(f"N and K must be multiples of {per16} (16-byte row strides for TMA)")
    return MatmulPlan(M, N, K, a, b_, c, da)


# ----------------------------------------------------------------------------
def pair_ok(comp, plan: MatmulPlan) -> bool:
    """CTA pairs need more than one 128-row block and 256-column tiles, and
    an even grid under the meta.json geometry too (a cluster of two)."""
    g = comp.kmeta.get("grid") or [1]
    g = [g] if isinstance(g, int) else list(g)
    return PAIR and plan.m > BM and plan.n > 128 and g[0] % 2 == 0


def _emit_record_part(target: str, version: str, entry: str) -> str:
    """``entry(part)``: one thread stores the partial tiles' scratch address
    into the module global ``emmy_part`` (a prelaunch of split-K kernels).
    Returned without the module header."""
    b = KernelBuilder(entry, target, version)
    b.directive(".maxntid 32, 1, 1")
    pp = b.param("part", ".u64")
    r, g = b.regs("rd", 2)
    t = b.reg("r")
    p = b.reg("p")
    b.ins(f"ld.param.u64 {r}, [{pp}];")
    b.ins(f"cvta.to.global.u64 {r}, {r};")
    b.ins(f"mov.u32 {t}, %tid.x;")
    b.ins(f"setp.ne.u32 {p}, {t}, 0;")
    done = b.label("PART_DONE")
    b.ins(f"@{p} bra {done};")
    b.ins(f"mov.u64 {g}, emmy_part;")
    b.ins(f"st.global.u64 [{g}], {r};")
    b.place(done)
    return b.render(header=False)


def _emit_reduce(target: str, version: str, entry: str, n: int, slices: int,
                 block: int = 256) -> str:
    """``entry(part, c)``: ``c[i] = part[0][i] + part[1][i] + ...`` over the
    ``slices`` partial results of ``n`` values each, added in slice order
    (deterministic).  Grid-stride over 16-byte vectors; returned without the
    module header."""
    assert n % 4 == 0
    b = KernelBuilder(entry, target, version)
    b.directive(f".maxntid {block}, 1, 1")
    pp, pc = b.param("part", ".u64"), b.param("c", ".u64")
    part, c = b.regs("rd", 2)
    for r, p_ in ((part, pp), (c, pc)):
        b.ins(f"ld.param.u64 {r}, [{p_}];")
        b.ins(f"cvta.to.global.u64 {r}, {r};")
    g, stride, t, nt = b.regs("r", 4)
    b.ins(f"mov.u32 {g}, %ctaid.x;")
    b.ins(f"mov.u32 {nt}, %ntid.x;")
    b.ins(f"mov.u32 {stride}, %nctaid.x;")
    b.ins(f"mul.lo.u32 {stride}, {stride}, {nt};")
    b.ins(f"mov.u32 {t}, %tid.x;")
    b.ins(f"mad.lo.u32 {g}, {g}, {nt}, {t};")
    top, done = b.label("RED"), b.label("RED_END")
    p = b.reg("p")
    b.place(top)
    b.ins(f"setp.ge.u32 {p}, {g}, {n // 4};")
    b.ins(f"@{p} bra {done};")
    off = b.reg("rd")
    b.ins(f"mul.wide.u32 {off}, {g}, 16;")
    src = b.reg("rd")
    b.ins(f"add.s64 {src}, {part}, {off};")
    vals = []
    for sl in range(slices):
        v = b.regs("f", 4)
        b.ins(f"ld.global.nc.L1::no_allocate.v4.f32 {{{', '.join(v)}}}, [{src}+{sl * n * 4}];")
        vals.append(v)
    acc = vals[0]
    for v in vals[1:]:
        for e in range(4):
            b.ins(f"add.rn.f32 {acc[e]}, {acc[e]}, {v[e]};")
    dst = b.reg("rd")
    b.ins(f"add.s64 {dst}, {c}, {off};")
    b.ins(f"st.global.v4.f32 [{dst}], {{{', '.join(acc)}}};")
    b.ins(f"add.u32 {g}, {g}, {stride};")
    b.ins(f"bra.uni {top};")
    b.place(done)
    return b.render(header=False)


def emit(comp, plan: MatmulPlan, gather: int = 0, pair=None, split_k=None):
    """``gather`` > 0: the all-gather variant for a row shard of C.  Instead
    of writing ``C``, the epilogue stores every finished tile into each of
    the up to ``gather`` destinations listed in the module global
    ``emmy_gather_dst`` (``emmy_gather_n`` of them used) at row
    ``emmy_gather_row0 + m``: every rank's full C, peers' copies mapped over
    NVLink, so the exchange overlaps the next tile's MMAs.

    ``pair`` (default: ``pair_ok``): a cluster of two CTAs computes each
    256 x BN tile with ``tcgen05.mma.cta_group::2`` (M=256).  Each CTA
    loads its own 128 rows of A and half of the B columns; the even CTA
    (the leader) issues every MMA, which reads both CTAs' shared memory and
    accumulates into both CTAs' TMEM (128 rows each).  Per CTA, a k-stage
    moves a third less data than with a 128 x BN tile per CTA."""
    M, N, K = plan.m, plan.n, plan.k
    if pair is None:
        pair = pair_ok(comp, plan)
    fp8 = plan.dtype in ("e4m3", "e5m2")
    lowp = plan.dtype in ("f16", "bf16") or fp8
    esz = 1 if fp8 else (2 if lowp else 4)
    BK = (128 // esz) if lowp else 16     # elements per stage (128- / 64-byte rows)
    KMMA = 32 // esz if lowp else 8       # K per MMA: 32 bytes of each operand row
    # 128 x 256 tiles whenever N allows: even for a 1024-row shard (256
    # tiles on 148 SMs) they beat 128 x 128 tiles, 0.76 against 0.95 ms
    BN = 256 if N > 128 else 128
    CG = 2 if pair else 1                 # CTAs per MMA
    TM = BM * CG                          # rows of C per tile
    BNC = BN // CG                        # B columns each CTA loads
    NST = PAIR_STAGES if pair else STAGES
    GM = GROUP_M // CG                    # grouped raster: the same 1024 rows either way
    T = launch_block(comp) or 256
    if T < 256 or T % 32:
        raise NoMatch(f"the tcgen05 matmul needs 256 threads per block (meta.json has {T})")
    KT = -(-K // BK)
    tiles_m, tiles_n = -(-M // TM), -(-N // BN)
    ntiles = tiles_m * tiles_n
    # split-K (f32 only, not in the gather variant): SK K slices per tile,
    # KTS stages each; unit u is tile u % ntiles, slice u // ntiles
    if split_k is None:
        split_k = 1 if (lowp or gather) else choose_split_k(ntiles, 148 // CG, K, BK)
    SK = int(split_k)
    if SK > 1 and (lowp or gather or KT % SK):
        raise ValueError(f"split-K {SK} needs an f32 matmul without gather and K/{BK} "
                         f"divisible by it")
    KTS = KT // SK
    nunits = ntiles * SK
    A_STAGE = BM * BK * esz               # 8 KB (tf32) / 16 KB (16-bit)
    B_STAGE = BNC * BK * esz              # 16 KB / 32 KB (BN=256; half that per CTA of a pair)
    if lowp:                              # no split: raw tiles only
        A_RAW = A_LO = 0
        B_RAW = B_LO = NST * A_STAGE
        BAR = B_RAW + NST * B_STAGE
    else:
        A_RAW, A_LO = 0, NST * A_STAGE
        B_RAW = 2 * NST * A_STAGE
        B_LO = B_RAW + NST * B_STAGE
        BAR = B_LO + NST * B_STAGE        # barriers after the tiles
    BOXN = 128 // esz                     # B box width: 128 bytes
    # gather mode: a 32x32 transpose stage per epilogue warp (rows padded to
    # 144 B, conflict-free both ways), so stores to peers are row-contiguous
    EPI = BAR + 256
    EPI_ROW = 144
    EPI_WARP = 32 * EPI_ROW
    SMEM = (EPI + (4 * EPI_WARP if gather else 0)) + 1024   # + alignment slack
    TMEM_COLS = 2 * BN

    b = KernelBuilder(comp.entry, comp.target, comp.ptx_version)
    b.module(".global .align 128 .b8 tmap_A[128];")
    b.module(".global .align 128 .b8 tmap_B[128];")
    if not lowp:
        b.module(".global .align 128 .b8 tmap_Alo[128];")
        b.module(".global .align 128 .b8 tmap_Blo[128];")
    b.module(".extern .shared .align 1024 .b8 dsmem[];")
    if gather:
        b.module(f".global .align 8 .b8 emmy_gather_dst[{8 * gather}];")
        b.module(".global .align 4 .u32 emmy_gather_n;")
        b.module(".global .align 4 .u32 emmy_gather_row0;")
    if SK > 1:
        # the partial tiles' scratch, recorded by the <entry>_part prelaunch
        b.module(".global .align 8 .u64 emmy_part;")
    b.directive(f".maxntid {T}, 1, 1")
    if pair:
        # launching without the cluster of two fails at launch time
        b.directive(".reqnctapercluster 2, 1, 1")
    b.directive(".maxnreg 168")
    ptrs = declare_params(b, comp)
    pC = ptrs[plan.c]

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
    FULL, EMPTY = 0, 8 * NST
    ACCF = EMPTY + 8 * NST
    ACCE, DRAIN, FIN = ACCF + 16, ACCF + 32, ACCF + 40
    slot, abort = b.regs("r", 2)
    b.ins(f"add.u32 {slot}, {bars}, {FIN + 8};")
    b.ins(f"add.u32 {abort}, {bars}, {FIN + 12};")
    assert FIN + 16 <= 256
    tc = TC(b, abort, cta_group=CG)

    # ---- setup ----------------------------------------------------------------
    p = b.reg("p")
    skip = b.label("INIT_DONE")
    b.ins(f"setp.ne.u32 {p}, {tid}, 0;")
    b.ins(f"@{p} bra {skip};")
    for s in range(NST):
        tc.init(f"{bars}+{FULL + 8 * s}", 1)
        tc.init(f"{bars}+{EMPTY + 8 * s}", 1)
    for a in range(2):
        tc.init(f"{bars}+{ACCF + 8 * a}", 1)
        tc.init(f"{bars}+{ACCE + 8 * a}", 128 * CG)     # every epilogue thread of the pair
    tc.init(f"{bars}+{DRAIN}", 1)
    tc.init(f"{bars}+{FIN}", 1)
    b.ins(f"st.shared.u32 [{abort}], 0;")
    b.ins("fence.mbarrier_init.release.cluster;")
    b.place(skip)
    skip2 = b.label("ALLOC_DONE")
    b.ins(f"setp.ne.u32 {p}, {warp}, 1;")
    b.ins(f"@{p} bra {skip2};")
    tc.tmem_alloc(slot, TMEM_COLS)
    b.place(skip2)
    if pair:
        # both CTAs' barriers are initialised before either CTA's TMA or
        # MMA completions can reach them
        b.ins("barrier.cluster.arrive.release.aligned;")
        b.ins("barrier.cluster.wait.acquire.aligned;")
    else:
        b.ins(f"bar.sync 0, {T};")
    b.ins("tcgen05.fence::after_thread_sync;")
    tmem = b.reg("r")
    b.ins(f"ld.shared.u32 {tmem}, [{slot}];")
    cta, ncta = b.regs("r", 2)
    rank = b.reg("r")
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
        b.ins(f"add.u32 {tc.peer_abort}, {pbars}, {FIN + 12};")
    else:
        b.ins(f"mov.u32 {cta}, %ctaid.x;")
        b.ins(f"mov.u32 {ncta}, %nctaid.x;")
        b.ins(f"mov.u32 {rank}, 0;")
    b.ins(f"setp.eq.u32 {lead}, {rank}, 0;")
    END = b.label("END")

    def tile_coords(tile):
        """Grouped raster: GM row blocks sweep all column blocks."""
        grp, first, gsz, inner, mb, nb = b.regs("r", 6)
        b.ins(f"div.u32 {grp}, {tile}, {GM * tiles_n};")
        b.ins(f"mul.lo.u32 {first}, {grp}, {GM};")
        b.ins(f"sub.u32 {gsz}, {tiles_m}, {first};")
        b.ins(f"min.u32 {gsz}, {gsz}, {GM};")
        b.ins(f"rem.u32 {inner}, {tile}, {GM * tiles_n};")
        b.ins(f"rem.u32 {mb}, {inner}, {gsz};")
        b.ins(f"add.u32 {mb}, {mb}, {first};")
        b.ins(f"div.u32 {nb}, {inner}, {gsz};")
        return mb, nb

    def stage_of(it):
        s, ph = b.regs("r", 2)
        b.ins(f"rem.u32 {s}, {it}, {NST};")
        b.ins(f"div.u32 {ph}, {it}, {NST};")
        b.ins(f"and.b32 {ph}, {ph}, 1;")
        return s, ph

    def remote(reg_base, off, s=None):
        """shared::cluster address of barrier ``off`` (+ 8*s) in the
        barrier block at ``reg_base``."""
        r = b.reg("r")
        if s is None:
            b.ins(f"add.u32 {r}, {reg_base}, {off};")
        else:
            b.ins(f"mad.lo.u32 {r}, {s}, 8, {reg_base};")
            b.ins(f"add.u32 {r}, {r}, {off};")
        return r

    def bar_at(off, s):
        r = b.reg("r")
        b.ins(f"mad.lo.u32 {r}, {s}, 8, {bars};")
        if off:
            b.ins(f"add.u32 {r}, {r}, {off};")
        return r

    kslice = {}                          # the current unit's K slice register

    def tile_loop(body_fn, label):
        """for unit = ctaid; unit < nunits; unit += nctaid: body_fn(tile),
        with unit = slice * ntiles + tile (split-K) or unit = tile."""
        unit = b.reg("r")
        top, done = b.label(label), b.label(label + "_END")
        pt = b.reg("p")
        b.ins(f"mov.u32 {unit}, {cta};")
        b.place(top)
        b.ins(f"setp.ge.u32 {pt}, {unit}, {nunits};")
        b.ins(f"@{pt} bra.uni {done};")
        if SK > 1:
            tile, ksl = b.regs("r", 2)
            b.ins(f"rem.u32 {tile}, {unit}, {ntiles};")
            b.ins(f"div.u32 {ksl}, {unit}, {ntiles};")
            kslice["reg"] = ksl
        else:
            tile = unit
        body_fn(tile)
        b.ins(f"add.u32 {unit}, {unit}, {ncta};")
        b.ins(f"bra.uni {top};")
        b.place(done)

    def k_loop(body_fn, it, label):
        ks = b.reg("r")
        top, done = b.label(label), b.label(label + "_END")
        pk = b.reg("p")
        b.ins(f"mov.u32 {ks}, 0;")
        b.place(top)
        b.ins(f"setp.ge.u32 {pk}, {ks}, {KTS};")
        b.ins(f"@{pk} bra.uni {done};")
        body_fn(ks)
        b.ins(f"add.u32 {ks}, {ks}, 1;")
        b.ins(f"add.u32 {it}, {it}, 1;")
        b.ins(f"bra.uni {top};")
        b.place(done)

    roles = [b.label("PRODUCER"), b.label("MMA"), b.label("SPLIT"), b.label("EPILOGUE")]
    pr = b.reg("p")
    b.ins(f"setp.eq.u32 {pr}, {warp}, 0;")
    b.ins(f"@{pr} bra {roles[0]};")
    b.ins(f"setp.eq.u32 {pr}, {warp}, 1;")
    b.ins(f"@{pr} bra {roles[1]};")
    b.ins(f"setp.lt.u32 {pr}, {warp}, 4;")
    b.ins(f"@{pr} bra {roles[2]};")
    b.ins(f"setp.lt.u32 {pr}, {warp}, 8;")
    b.ins(f"@{pr} bra {roles[3]};")
    b.ins(f"bra.uni {END};")

    # ---- producer --------------------------------------------------------------
    b.place(roles[0])
    b.ins(f"setp.ne.u32 {pr}, {lane}, 0;")
    b.ins(f"@{pr} bra {END};")
    tmA = tc.tmap_address("tmap_A")
    tmB = tc.tmap_address("tmap_B")
    maps = [tmA, tmB]
    if not lowp:
        tmAl = tc.tmap_address("tmap_Alo")
        tmBl = tc.tmap_address("tmap_Blo")
        maps += [tmAl, tmBl]
    for tm_ in maps:
        b.ins(f"fence.proxy.tensormap::generic.acquire.gpu [{tm_}], 128;")
        b.ins(f"prefetch.tensormap [{tm_}];")
    it_p = b.reg("r")
    b.ins(f"mov.u32 {it_p}, 0;")

    def producer_tile(tile):
        mb, nb = tile_coords(tile)
        m0, n0 = b.regs("r", 2)
        b.ins(f"mul.lo.u32 {m0}, {mb}, {TM};")
        b.ins(f"mul.lo.u32 {n0}, {nb}, {BN};")
        if pair:                            # this CTA's rows of A, columns of B
            b.ins(f"mad.lo.u32 {m0}, {rank}, {BM}, {m0};")
            b.ins(f"mad.lo.u32 {n0}, {rank}, {BNC}, {n0};")

        def kstep(ks):
            s, ph = stage_of(it_p)
            pw = b.reg("r")
            b.ins(f"xor.b32 {pw}, {ph}, 1;")
            tc.wait(bar_at(EMPTY, s), pw, END, ROLE_PRODUCER)
            parts = [(tmA, tmB, A_RAW, B_RAW)]
            if not lowp:                    # the pre-split lo halves too
                parts.append((tmAl, tmBl, A_LO, B_LO))
            nbytes = CG * len(parts) * (A_STAGE + B_STAGE)
            if pair:
                # both CTAs' tiles are counted on the leader's full barrier;
                # the leader announces the bytes of both
                full = remote(lbars, FULL, s)
                pe = b.label("EXPECTED")
                b.ins(f"@!{lead} bra {pe};")
                tc.arrive_expect_tx(bar_at(FULL, s), nbytes)
                b.place(pe)
            else:
                full = bar_at(FULL, s)
                tc.arrive_expect_tx(full, nbytes)
            k0 = b.reg("r")
            if SK > 1:                      # this unit's K slice
                b.ins(f"mad.lo.u32 {k0}, {kslice['reg']}, {KTS}, {ks};")
                b.ins(f"mul.lo.u32 {k0}, {k0}, {BK};")
            else:
                b.ins(f"mul.lo.u32 {k0}, {ks}, {BK};")
            for (tma_, tmb_, a_reg, b_reg) in parts:
                dA = b.reg("r")
                b.ins(f"mad.lo.u32 {dA}, {s}, {A_STAGE}, {base};")
                if a_reg:
                    b.ins(f"add.u32 {dA}, {dA}, {a_reg};")
                tc.tma_load_2d(dA, tma_, k0, m0, full, pair)
                dB = b.reg("r")
                b.ins(f"mad.lo.u32 {dB}, {s}, {B_STAGE}, {base};")
                b.ins(f"add.u32 {dB}, {dB}, {b_reg};")
                for c in range(BNC // BOXN):
                    x = b.reg("r")
                    b.ins(f"add.u32 {x}, {n0}, {BOXN * c};")
                    d = b.reg("r")
                    b.ins(f"add.u32 {d}, {dB}, {c * BOXN * BK * esz};")
                    tc.tma_load_2d(d, tmb_, x, k0, full, pair)
        k_loop(kstep, it_p, "PK")
    tile_loop(producer_tile, "PT")
    b.ins(f"bra.uni {END};")

    # ---- MMA -------------------------------------------------------------------
    b.place(roles[1])
    b.ins(f"setp.ne.u32 {pr}, {lane}, 0;")
    b.ins(f"@{pr} bra {END};")
    b.ins(f"@!{lead} bra {END};")             # the pair's MMAs are the leader's
    idesc = b.reg("r")
    if fp8:
        b.ins(f"mov.u32 {idesc}, {idesc_f8(TM, BN, False, True, plan.dtype)};")
    elif lowp:
        b.ins(f"mov.u32 {idesc}, {idesc_f16(TM, BN, False, True, plan.dtype)};")
    if lowp:
        # A K-major, 128-byte rows (64 halves), 8-row atoms; B N-major with
        # the 128-byte swizzle: LBO = stride between 64-column boxes, SBO =
        # stride between 8-row K groups
        ka = smem_desc_hi(16, 8 * 128, "128B")
        kb = smem_desc_hi(BOXN * BK * esz, 8 * 128, "128B")
    else:
        b.ins(f"mov.u32 {idesc}, {idesc_tf32(TM, BN, False, True)};")
        ka = smem_desc_hi(16, 8 * 64, "64B")      # K-major, 64-byte rows, 8-row atoms
        # N-major tf32 operands need the 128-byte swizzle with 32-byte atoms
        # (4-row K groups): LBO = stride between 32-column chunks, SBO = stride
        # between 4-row K groups
        kb = smem_desc_hi(32 * BK * 4, 4 * 128, "128B_base32B")
    ptrue = b.reg("p")
    b.ins(f"setp.eq.u32 {ptrue}, 0, 0;")
    it_m, tl_m = b.regs("r", 2)
    b.ins(f"mov.u32 {it_m}, 0;")
    b.ins(f"mov.u32 {tl_m}, 0;")

    def release(off, s):
        """Commit to barrier ``off``+8s of this CTA and, in a pair, of the
        peer: the same completed MMAs free both CTAs' stage / fill both
        CTAs' accumulators."""
        tc.commit(bar_at(off, s))
        if pair:
            tc.commit(remote(pbars, off, s))

    def desc(addr, const):
        a4 = b.reg("r")
        b.ins(f"shr.u32 {a4}, {addr}, 4;")
        b.ins(f"and.b32 {a4}, {a4}, 0x3FFF;")
        d = b.reg("rd")
        b.ins(f"cvt.u64.u32 {d}, {a4};")
        b.ins(f"or.b64 {d}, {d}, 0x{const:016X};")
        return d

    def mma_tile(tile):
        a, aph = b.regs("r", 2)
        b.ins(f"and.b32 {a}, {tl_m}, 1;")
        b.ins(f"shr.u32 {aph}, {tl_m}, 1;")
        b.ins(f"and.b32 {aph}, {aph}, 1;")
        b.ins(f"xor.b32 {aph}, {aph}, 1;")
        tc.wait(bar_at(ACCE, a), aph, END, ROLE_MMA)
        b.ins("tcgen05.fence::after_thread_sync;")
        dt = b.reg("r")
        b.ins(f"mad.lo.u32 {dt}, {a}, {BN}, {tmem};")

        def kstep_lowp(ks):
            s, ph = stage_of(it_m)
            tc.wait(bar_at(FULL, s), ph, END, ROLE_MMA)
            b.ins("tcgen05.fence::after_thread_sync;")
            ah, bh = b.regs("r", 2)
            b.ins(f"mad.lo.u32 {ah}, {s}, {A_STAGE}, {base};")
            b.ins(f"mad.lo.u32 {bh}, {s}, {B_STAGE}, {base};")
            b.ins(f"add.u32 {bh}, {bh}, {B_RAW};")
            da_, db_ = desc(ah, ka), desc(bh, kb)
            pacc = b.reg("p")
            b.ins(f"setp.ne.u32 {pacc}, {ks}, 0;")
            for kk in range(BK // KMMA):
                if kk:
                    # KMMA elements = 32 bytes along A's rows; KMMA rows of B
                    b.ins(f"add.s64 {da_}, {da_}, 2;")
                    b.ins(f"add.s64 {db_}, {db_}, {(KMMA * 128) >> 4};")
                mma = tc.mma_f8 if fp8 else tc.mma_f16
                mma(dt, da_, db_, idesc, pacc if kk == 0 else ptrue)
            release(EMPTY, s)

        def kstep(ks):
            s, ph = stage_of(it_m)
            tc.wait(bar_at(FULL, s), ph, END, ROLE_MMA)
            b.ins("tcgen05.fence::after_thread_sync;")
            ah, al, bh, bl = b.regs("r", 4)
            b.ins(f"mad.lo.u32 {ah}, {s}, {A_STAGE}, {base};")
            b.ins(f"add.u32 {al}, {ah}, {A_LO - A_RAW};")
            b.ins(f"mad.lo.u32 {bh}, {s}, {B_STAGE}, {base};")
            b.ins(f"add.u32 {bh}, {bh}, {B_RAW};")
            b.ins(f"add.u32 {bl}, {bh}, {B_LO - B_RAW};")
            dah, dal = desc(ah, ka), desc(al, ka)
            dbh, dbl = desc(bh, kb), desc(bl, kb)
            pacc = b.reg("p")
            b.ins(f"setp.ne.u32 {pacc}, {ks}, 0;")
            for kk in range(BK // 8):
                if kk:
                    for r_, inc in ((dah, 2), (dal, 2), (dbh, 64), (dbl, 64)):
                        b.ins(f"add.s64 {r_}, {r_}, {inc};")
                tc.mma_tf32(dt, dah, dbh, idesc, pacc if kk == 0 else ptrue)
                tc.mma_tf32(dt, dah, dbl, idesc, ptrue)
                tc.mma_tf32(dt, dal, dbh, idesc, ptrue)
            release(EMPTY, s)
        k_loop(kstep_lowp if lowp else kstep, it_m, "MK")
        release(ACCF, a)
        b.ins(f"add.u32 {tl_m}, {tl_m}, 1;")
    tile_loop(mma_tile, "MT")
    b.ins(f"bra.uni {END};")

    # ---- warps 2-3: idle (the tf32 split is a pre-pass) -----------------------
    b.place(roles[2])
    b.ins(f"bra.uni {END};")

    # ---- epilogue --------------------------------------------------------------
    b.place(roles[3])
    q = b.reg("r")
    b.ins(f"and.b32 {q}, {warp}, 3;")
    lane_base = b.reg("r")
    b.ins(f"shl.b32 {lane_base}, {q}, 21;")             # (32*q) << 16
    b.ins(f"add.u32 {lane_base}, {lane_base}, {tmem};")
    tl_e = b.reg("r")
    b.ins(f"mov.u32 {tl_e}, 0;")
    if SK > 1:
        # the _part prelaunch records the scratch for the partial tiles;
        # without it there is nowhere to write: report and leave (the other
        # roles' bounded waits then end the kernel)
        part_base = b.reg("rd")
        b.ins(f"ld.global.u64 {part_base}, [emmy_part];")
        pz = b.reg("p")
        have = b.label("HAVE_PART")
        b.ins(f"setp.ne.u64 {pz}, {part_base}, 0;")
        b.ins(f"@{pz} bra.uni {have};")
        tc.raise_abort(STATUS_NO_PREPASS)
        b.ins(f"bra.uni {END};")
        b.place(have)
    if gather:
        gdst = b.regs("rd", gather)
        gn, grow0 = b.regs("r", 2)
        gon = b.regs("p", gather)
        b.ins(f"ld.global.u32 {gn}, [emmy_gather_n];")
        b.ins(f"ld.global.u32 {grow0}, [emmy_gather_row0];")
        for d in range(gather):
            b.ins(f"ld.global.u64 {gdst[d]}, [emmy_gather_dst+{8 * d}];")
            b.ins(f"setp.lt.u32 {gon[d]}, {d}, {gn};")
        # this warp's transpose stage: written at row = lane, read at
        # row = lane/8 (+4i), 16-byte column chunk lane%8
        st_w, st_r, sub_row, sub_col = b.regs("r", 4)
        b.ins(f"mad.lo.u32 {st_w}, {q}, {EPI_WARP}, {base};")
        b.ins(f"add.u32 {st_w}, {st_w}, {EPI};")
        b.ins(f"shr.u32 {sub_row}, {lane}, 3;")
        b.ins(f"and.b32 {sub_col}, {lane}, 7;")
        b.ins(f"mad.lo.u32 {st_r}, {sub_row}, {EPI_ROW}, {st_w};")
        b.ins(f"mad.lo.u32 {st_r}, {sub_col}, 16, {st_r};")
        b.ins(f"shl.b32 {sub_col}, {sub_col}, 2;")
        b.ins(f"mad.lo.u32 {st_w}, {lane}, {EPI_ROW}, {st_w};")

    def epi_tile(tile):
        mb, nb = tile_coords(tile)
        a, aph = b.regs("r", 2)
        b.ins(f"and.b32 {a}, {tl_e}, 1;")
        b.ins(f"shr.u32 {aph}, {tl_e}, 1;")
        b.ins(f"and.b32 {aph}, {aph}, 1;")
        tc.wait(bar_at(ACCF, a), aph, END, ROLE_EPILOGUE, uniform=True)
        b.ins("tcgen05.fence::after_thread_sync;")
        row, n0 = b.regs("r", 2)
        b.ins(f"mad.lo.u32 {row}, {mb}, {TM}, {lane};")
        b.ins(f"mad.lo.u32 {row}, {q}, 32, {row};")
        if pair:
            b.ins(f"mad.lo.u32 {row}, {rank}, {BM}, {row};")
        b.ins(f"mul.lo.u32 {n0}, {nb}, {BN};")
        prow = b.reg("p")
        b.ins(f"setp.lt.u32 {prow}, {row}, {M};")
        rowaddr = b.reg("rd")
        b.ins(f"mul.wide.u32 {rowaddr}, {row}, {N * 4};")
        if SK > 1:
            # slice s of the tile goes to part[s] (M x N f32 each); the reduce
            # entry sums the slices into C in slice order
            po = b.reg("rd")
            b.ins(f"mul.wide.u32 {po}, {kslice['reg']}, {M * N * 4};")
            b.ins(f"add.s64 {rowaddr}, {rowaddr}, {po};")
            b.ins(f"add.s64 {rowaddr}, {rowaddr}, {part_base};")
        else:
            b.ins(f"add.s64 {rowaddr}, {rowaddr}, {pC};")
        taddr = b.reg("r")
        b.ins(f"mad.lo.u32 {taddr}, {a}, {BN}, {lane_base};")
        if gather:
            # lane l moves row l of each 32x32 chunk into the stage, then
            # writes rows (l/8 + 4i), 16 B at column 4*(l%8): each store
            # instruction covers four contiguous 128-byte row segments
            rbase = b.reg("r")
            b.ins(f"mad.lo.u32 {rbase}, {mb}, {TM}, {sub_row};")
            b.ins(f"mad.lo.u32 {rbase}, {q}, 32, {rbase};")
            if pair:
                b.ins(f"mad.lo.u32 {rbase}, {rank}, {BM}, {rbase};")
            for cb in range(BN // 32):
                v = b.regs("f", 32)
                b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(v)}}}, "
                      f"[{taddr}+{cb * 32}];")
                b.ins("tcgen05.wait::ld.sync.aligned;")
                for g in range(8):
                    b.ins(f"st.shared.v4.f32 [{st_w}+{16 * g}], {{{', '.join(v[4 * g:4 * g + 4])}}};")
                b.ins("bar.warp.sync 0xffffffff;")
                col = b.reg("r")
                b.ins(f"add.u32 {col}, {n0}, {cb * 32};")
                b.ins(f"add.u32 {col}, {col}, {sub_col};")
                pcol = b.reg("p")
                b.ins(f"setp.lt.u32 {pcol}, {col}, {N};")
                coff = b.reg("rd")
                b.ins(f"mul.wide.u32 {coff}, {col}, 4;")
                for i in range(8):
                    w = b.regs("f", 4)
                    b.ins(f"ld.shared.v4.f32 {{{', '.join(w)}}}, [{st_r}+{4 * i * EPI_ROW}];")
                    r_i = b.reg("r")
                    b.ins(f"add.u32 {r_i}, {rbase}, {4 * i};")
                    pr = b.reg("p")
                    b.ins(f"setp.lt.and.u32 {pr}, {r_i}, {M}, {pcol};")
                    b.ins(f"add.u32 {r_i}, {r_i}, {grow0};")
                    ro = b.reg("rd")
                    b.ins(f"mul.wide.u32 {ro}, {r_i}, {N * 4};")
                    b.ins(f"add.s64 {ro}, {ro}, {coff};")
                    for d in range(gather):
                        od, pd = b.reg("rd"), b.reg("p")
                        b.ins(f"add.s64 {od}, {ro}, {gdst[d]};")
                        b.ins(f"and.pred {pd}, {pr}, {gon[d]};")
                        b.ins(f"@{pd} st.global.v4.f32 [{od}], {{{', '.join(w)}}};")
                b.ins("bar.warp.sync 0xffffffff;")
        for cb in range(0 if gather else BN // 32):
            v = b.regs("f", 32)
            b.ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(v)}}}, [{taddr}+{cb * 32}];")
            b.ins("tcgen05.wait::ld.sync.aligned;")
            for g in range(8):
                col = b.reg("r")
                b.ins(f"add.u32 {col}, {n0}, {cb * 32 + 4 * g};")
                pc = b.reg("p")
                b.ins(f"setp.lt.and.u32 {pc}, {col}, {N}, {prow};")
                off = b.reg("rd")
                b.ins(f"mul.wide.u32 {off}, {col}, 4;")
                vals = ', '.join(v[4 * g:4 * g + 4])
                b.ins(f"add.s64 {off}, {off}, {rowaddr};")
                b.ins(f"@{pc} st.global.v4.f32 [{off}], {{{vals}}};")
        b.ins("tcgen05.fence::before_thread_sync;")
        if pair:                        # the leader's MMAs wait for both epilogues
            tc.arrive_cluster(remote(lbars, ACCE, a))
        else:
            tc.arrive(bar_at(ACCE, a))
        b.ins(f"add.u32 {tl_e}, {tl_e}, 1;")
    tile_loop(epi_tile, "ET")

    # ---- teardown -----------------------------------------------------------------
    b.place(END)
    b.ins(f"bar.sync 0, {T};")
    fin = b.label("FIN")
    b.ins(f"setp.ne.u32 {p}, {warp}, 1;")
    b.ins(f"@{p} bra {fin};")
    b.ins("bar.warp.sync 0xffffffff;")
    # drain: every MMA this block issued has finished before TMEM is freed
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
        tc.wait(f"{bars}+{FIN}", 0, dl, ROLE_TEARDOWN, peer=False)
        b.ins(f"bra.uni {dl};")
        b.place(fl)
        tc.commit(f"{bars}+{DRAIN}")
        tc.wait(f"{bars}+{DRAIN}", 0, dl, ROLE_MMA, peer=False)
        tc.wait(f"{bars}+{FIN}", 0, dl, ROLE_TEARDOWN, peer=False)
        tc.arrive_cluster(remote(pbars, FIN))
    else:
        tc.commit(f"{bars}+{DRAIN}")
        tc.wait(f"{bars}+{DRAIN}", 0, dl, ROLE_MMA)
    b.place(dl)
    b.ins("bar.warp.sync 0xffffffff;")
    b.ins("tcgen05.fence::after_thread_sync;")
    tc.tmem_dealloc(tmem, TMEM_COLS)
    b.place(fin)

    sidecar = {
        "category": "matmul",
        "grid": [CG * min(nunits, 148 // CG), 1, 1],
        "block": [T, 1, 1],
        "shared_bytes": SMEM,
        "cluster": [CG, 1, 1],
        "tensormaps": [
            {"global": "tmap_A", "arg": plan.a,      # f32: the hi part, low bits dropped
             "dtype": "u8" if fp8 else plan.dtype,
             "dims": [K, M], "strides": [K * esz], "box": [BK, BM],
             "swizzle": "128B" if lowp else "64B"},
            {"global": "tmap_B", "arg": plan.b,
             "dtype": "u8" if fp8 else plan.dtype,
             "dims": [N, K], "strides": [N * esz], "box": [BOXN, BK],
             "swizzle": "128B" if lowp else "128B_atom32B"},
        ] + ([] if lowp else [
            {"global": "tmap_Alo", "arg": "@a_lo", "dtype": "f32", "dims": [K, M],
             "strides": [K * 4], "box": [BK, BM], "swizzle": "64B"},
            {"global": "tmap_Blo", "arg": "@b_lo", "dtype": "f32", "dims": [N, K],
             "strides": [N * 4], "box": [BOXN, BK], "swizzle": "128B_atom32B"},
        ]),
        "algorithmic_flops": 2 * M * N * K,
        "tensor_flops_issued": (1 if lowp else 3) * 2 * tiles_m * TM * tiles_n * BN * KT * BK,
        "operand_dtype": plan.dtype,
        "tile": [TM, BN, BK],
        "cta_group": CG,
        "stages": NST,
        "status_word": "emmy_status",
    }
    ptx = b.render()
    if not lowp:
        # 3xTF32: A and B are their own hi parts; two pre-pass entries write
        # their lo parts once to scratch memory (each operand tile is used by
        # many output tiles, so splitting inside the kernel repeats the work)
        sa, sb = comp.entry + "_split_a", comp.entry + "_split_b"
        ptx += "\n" + emit_tf32_split(comp.target, comp.ptx_version, sa, M * K)
        ptx += "\n" + emit_tf32_split(comp.target, comp.ptx_version, sb, K * N)
        sidecar["scratch"] = [{"name": "a_lo", "bytes": M * K * 4},
                              {"name": "b_lo", "bytes": K * N * 4}]
        sidecar["prelaunch"] = [split_launch(sa, [plan.a, "@a_lo"], M * K),
                                split_launch(sb, [plan.b, "@b_lo"], K * N)]
        if SK > 1:
            sp, sr = comp.entry + "_part", comp.entry + "_reduce"
            ptx += "\n" + _emit_record_part(comp.target, comp.ptx_version, sp)
            ptx += "\n" + _emit_reduce(comp.target, comp.ptx_version, sr, M * N, SK)
            sidecar["scratch"].append({"name": "c_part", "bytes": SK * M * N * 4})
            sidecar["prelaunch"].append({"entry": sp, "args": ["@c_part"],
                                         "grid": [1, 1, 1], "block": [32, 1, 1]})
            sidecar["postlaunch"] = [split_launch(sr, ["@c_part", plan.c], M * N,
                                                  max_blocks=148 * 8)]
        sidecar["split_k"] = SK
    if gather:
        sidecar["gather"] = {"max_destinations": gather, "destinations": "emmy_gather_dst",
                             "count": "emmy_gather_n", "row0": "emmy_gather_row0",
                             "writes_c": False}
    return ptx, sidecar
