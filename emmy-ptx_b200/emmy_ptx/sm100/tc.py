"""Blackwell building blocks for the tensor-core kernels, as PTX emitters.

* mbarriers (init / arrive / expect-tx) and **bounded** waits: every wait
  polls ``mbarrier.try_wait.parity`` once, then (if the phase is still
  open) keeps polling and reads ``%globaltimer`` every 256 polls; after
  ``WAIT_LIMIT_NS`` it records an error code in the module's
  ``emmy_status`` word, raises a block-wide abort flag in shared memory and
  branches to the caller's teardown label instead of spinning forever.
  Waits also leave early when another role raised the abort flag.
* TMA tile loads (``cp.async.bulk.tensor``, no multicast) from tensor maps
  kept in module ``.global`` variables (the meta.json parameter list has no
  room for them; the runtime encodes and writes them before launch).
* tcgen05: TMEM alloc/dealloc, shared-memory matrix descriptors, the
  instruction descriptor for ``kind::tf32``, MMA issue and commit, TMEM
  loads for the epilogue.

Descriptor formats follow the PTX ISA (tcgen05 "shared memory descriptor"
and "instruction descriptor" tables): start address, leading and stride
byte offsets in 16-byte units, version 1, swizzle mode in bits 61-63.
"""

from __future__ import annotations

from .ptx import KernelBuilder

WAIT_LIMIT_NS = 2_000_000_000      # 2 s per wait before the kernel gives up

# status codes written to emmy_status
STATUS_TIMEOUT = 0x100             # + role id
STATUS_NO_PREPASS = 0x200          # a kernel's pre-pass entry did not run before it

SWIZZLE_MODE = {"none": 0, "128B_base32B": 1, "128B": 2, "64B": 4, "32B": 6}


def status_decl(b: KernelBuilder):
    b.module(".global .align 4 .u32 emmy_status;")


def smem_desc_hi(lbo_bytes: int, sbo_bytes: int, swizzle: str) -> int:
    """The constant part of a 64-bit shared-memory matrix descriptor
    (everything but the start address, which is or-ed in at run time):
    leading/stride byte offsets in 16-byte units, version 1 (bit 46), the
    swizzle mode in bits 61-63."""
    lbo = (lbo_bytes >> 4) & 0x3FFF
    sbo = (sbo_bytes >> 4) & 0x3FFF
    d = (lbo << 16) | (sbo << 32) | (1 << 46) | (SWIZZLE_MODE[swizzle] << 61)
    return d


def idesc_tf32(m: int, n: int, a_mn_major: bool, b_mn_major: bool) -> int:
    """Instruction descriptor: f32 accumulate, tf32 A and B."""
    assert m in (64, 128, 256) and n % 8 == 0 and 8 <= n <= 256
    d = (1 << 4)            # D format f32
    d |= (2 << 7)           # A format tf32
    d |= (2 << 10)          # B format tf32
    d |= (int(a_mn_major) << 15) | (int(b_mn_major) << 16)
    d |= ((n >> 3) << 17) | ((m >> 4) << 24)
    return d


def idesc_f16(m: int, n: int, a_mn_major: bool, b_mn_major: bool, ab: str = "bf16") -> int:
    """Instruction descriptor for kind::f16: f32 accumulate, A and B both
    f16 or both bf16 (the two operands of one MMA have the same type)."""
    assert m in (64, 128, 256) and n % 16 == 0 and 16 <= n <= 256
    fmt = {"f16": 0, "bf16": 1}[ab]
    d = (1 << 4)            # D format f32
    d |= (fmt << 7) | (fmt << 10)
    d |= (int(a_mn_major) << 15) | (int(b_mn_major) << 16)
    d |= ((n >> 3) << 17) | ((m >> 4) << 24)
    return d


def emit_tf32_split(target: str, version: str, entry: str, n_elems: int,
                    block: int = 256) -> str:
    """A pre-pass entry ``entry(src, lo)``: for each of the ``n_elems`` f32
    values (a multiple of 4, 16-byte aligned buffers) ``lo = x - hi``, hi
    being x with its low 13 bits cleared; ``lo`` is exact.  The tensor core
    reads an f32 operand as tf32 by dropping those 13 bits, so the kernel
    loads ``src`` itself as the hi operand of 3xTF32 (hi*hi + hi*lo +
    lo*hi) and only ``lo`` is written.  Grid-stride over 16-byte vectors;
    returned without the module header, to be appended to a kernel's
    module."""
    b = KernelBuilder(entry, target, version)
    b.directive(f".maxntid {block}, 1, 1")
    ps, pl = b.param("src", ".u64"), b.param("lo", ".u64")
    src, lo_p = b.regs("rd", 2)
    for r, p_ in ((src, ps), (lo_p, pl)):
        b.ins(f"ld.param.u64 {r}, [{p_}];")
        b.ins(f"cvta.to.global.u64 {r}, {r};")
    nvec = n_elems // 4
    g, stride, t, nt = b.regs("r", 4)
    b.ins(f"mov.u32 {g}, %ctaid.x;")
    b.ins(f"mov.u32 {nt}, %ntid.x;")
    b.ins(f"mov.u32 {stride}, %nctaid.x;")
    b.ins(f"mul.lo.u32 {stride}, {stride}, {nt};")
    b.ins(f"mov.u32 {t}, %tid.x;")
    b.ins(f"mad.lo.u32 {g}, {g}, {nt}, {t};")
    top, done = b.label("SPLIT"), b.label("SPLIT_END")
    p = b.reg("p")
    b.place(top)
    b.ins(f"setp.ge.u32 {p}, {g}, {nvec};")
    b.ins(f"@{p} bra {done};")
    off = b.reg("rd")
    b.ins(f"mul.wide.u32 {off}, {g}, 16;")
    a, al = b.regs("rd", 2)
    b.ins(f"add.s64 {a}, {src}, {off};")
    b.ins(f"add.s64 {al}, {lo_p}, {off};")
    x = b.regs("f", 4)
    b.ins(f"ld.global.nc.L1::no_allocate.v4.f32 {{{', '.join(x)}}}, [{a}];")
    lo = b.regs("f", 4)
    for e in range(4):
        hb = b.reg("r")
        b.ins(f"mov.b32 {hb}, {x[e]};")
        b.ins(f"and.b32 {hb}, {hb}, 0xFFFFE000;")
        hf = b.reg("f")
        b.ins(f"mov.b32 {hf}, {hb};")
        b.ins(f"sub.f32 {lo[e]}, {x[e]}, {hf};")
    b.ins(f"st.global.v4.f32 [{al}], {{{', '.join(lo)}}};")
    b.ins(f"add.u32 {g}, {g}, {stride};")
    b.ins(f"bra.uni {top};")
    b.place(done)
    return b.render(header=False)


def split_launch(entry: str, args: list, n_elems: int, block: int = 256,
                 max_blocks: int = 148 * 8, vec: int = 4) -> dict:
    """The sidecar ``prelaunch`` record for a grid-stride split entry over
    ``vec``-element vectors, at most ``max_blocks`` blocks."""
    nvec = n_elems // vec
    return {"entry": entry, "args": list(args),
            "grid": [max(1, min(-(-nvec // block), max_blocks)), 1, 1], "block": [block, 1, 1]}


def idesc_f8(m: int, n: int, a_mn_major: bool, b_mn_major: bool, ab: str = "e4m3") -> int:
    """Instruction descriptor for kind::f8f6f4 with fp8 A and B (E4M3 = 0,
    E5M2 = 1), f32 accumulate."""
    assert m in (64, 128, 256) and n % 16 == 0 and 16 <= n <= 256
    fmt = {"e4m3": 0, "e5m2": 1}[ab]
    d = (1 << 4)            # D format f32
    d |= (fmt << 7) | (fmt << 10)
    d |= (int(a_mn_major) << 15) | (int(b_mn_major) << 16)
    d |= ((n >> 3) << 17) | ((m >> 4) << 24)
    return d


class TC:
    """Per-kernel helper bound to one KernelBuilder."""

    def __init__(self, b: KernelBuilder, abort_addr: str, limit_ns: int = WAIT_LIMIT_NS,
                 cta_group: int = 1):
        self.b = b
        self.abort = abort_addr       # register holding the smem address of the abort flag
        self.limit_ns = int(limit_ns)
        self.cg = int(cta_group)      # 2: a CTA pair shares each MMA (one kernel uses one group)
        self.peer_abort = None        # cluster address of the pair peer's abort flag
        status_decl(b)

    # -- mbarriers ------------------------------------------------------------
    def init(self, bar, count):
        self.b.ins(f"mbarrier.init.shared::cta.b64 [{bar}], {count};")

    def arrive(self, bar):
        st = self.b.reg("rd")
        self.b.ins(f"mbarrier.arrive.shared::cta.b64 {st}, [{bar}];")

    def arrive_cluster(self, bar):
        """Arrive on an mbarrier given by its shared::cluster address (this
        CTA's or the pair peer's), releasing this thread's prior writes at
        cluster scope."""
        self.b.ins(f"mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{bar}];")

    def arrive_expect_tx(self, bar, nbytes):
        st = self.b.reg("rd")
        self.b.ins(f"mbarrier.arrive.expect_tx.shared::cta.b64 {st}, [{bar}], {nbytes};")

    def wait(self, bar, parity, fail_label, role: int, uniform: bool = False,
             peer: bool = True):
        """Bounded wait for the phase of parity ``parity`` (register or
        immediate) of ``bar``; on timeout or abort branch to
        ``fail_label``.  ``uniform``: every lane of the warp waits and all
        decisions are warp votes, so the warp leaves converged (needed
        before ``.sync.aligned`` instructions).  ``peer``: a timeout also
        raises the pair peer's abort flag (off in teardown waits, when the
        peer may already have exited)."""
        b = self.b
        top, done = b.label("WAIT"), b.label("WAIT_OK")
        p, pf, pv = b.regs("p", 3)
        t0, t1 = b.regs("rd", 2)
        n, fl = b.regs("r", 2)
        # fast path: a phase that has already completed costs one poll.
        # Reading %globaltimer first cost ~300 cycles per wait, which left
        # the tensor core idle between a kernel's back-to-back MMA batches.
        b.ins(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity};")
        if uniform:
            b.ins(f"vote.sync.all.pred {pv}, {p}, 0xffffffff;")
            b.ins(f"@{pv} bra.uni {done};")
        else:
            b.ins(f"@{p} bra.uni {done};")
        b.ins(f"mov.u64 {t0}, %globaltimer;")
        b.ins(f"mov.u32 {n}, 0;")
        b.place(top)
        b.ins(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity};")
        if uniform:
            b.ins(f"vote.sync.all.pred {pv}, {p}, 0xffffffff;")
            b.ins(f"@{pv} bra.uni {done};")
        else:
            b.ins(f"@{p} bra.uni {done};")
        b.ins(f"add.u32 {n}, {n}, 1;")
        b.ins(f"and.b32 {fl}, {n}, 255;")
        b.ins(f"setp.ne.u32 {pf}, {fl}, 0;")
        b.ins(f"@{pf} bra.uni {top};")
        b.ins(f"ld.volatile.shared.u32 {fl}, [{self.abort}];")
        b.ins(f"setp.ne.u32 {pf}, {fl}, 0;")
        if uniform:
            b.ins(f"vote.sync.any.pred {pf}, {pf}, 0xffffffff;")
        b.ins(f"@{pf} bra.uni {fail_label};")
        b.ins(f"mov.u64 {t1}, %globaltimer;")
        b.ins(f"sub.u64 {t1}, {t1}, {t0};")
        b.ins(f"setp.ge.u64 {pf}, {t1}, {self.limit_ns};")
        if uniform:
            b.ins(f"vote.sync.any.pred {pf}, {pf}, 0xffffffff;")
        b.ins(f"@!{pf} bra.uni {top};")
        self.raise_abort(STATUS_TIMEOUT + role, peer)
        b.ins(f"bra.uni {fail_label};")
        b.place(done)

    def raise_abort(self, code, peer: bool = True):
        b = self.b
        one = b.reg("r")
        b.ins(f"mov.u32 {one}, {code};")
        b.ins(f"st.volatile.shared.u32 [{self.abort}], {one};")
        if peer and self.peer_abort is not None:
            # the pair peer waits on barriers this CTA feeds: make it leave too
            b.ins(f"st.relaxed.cluster.shared::cluster.u32 [{self.peer_abort}], {one};")
        sa = b.reg("rd")
        b.ins(f"mov.u64 {sa}, emmy_status;")
        b.ins(f"cvta.global.u64 {sa}, {sa};")
        b.ins(f"st.relaxed.gpu.global.u32 [{sa}], {one};")

    # -- TMA ------------------------------------------------------------------
    def tma_load_2d(self, dst_smem, tmap_generic, x, y, bar, pair: bool = False):
        """``pair``: the ``.cta_group::2`` form -- the tile lands in this CTA's
        shared memory and its bytes are counted on ``bar``, which may be the
        pair leader's mbarrier (a shared::cluster address)."""
        cg = ".cta_group::2" if pair else ""
        self.b.ins(f"cp.async.bulk.tensor.2d{cg}.shared::cluster.global.mbarrier::complete_tx::bytes "
                   f"[{dst_smem}], [{tmap_generic}, {{{x}, {y}}}], [{bar}];")

    def tma_load_3d(self, dst_smem, tmap_generic, x, y, z, bar, pair: bool = False):
        """As tma_load_2d, with three coordinates."""
        cg = ".cta_group::2" if pair else ""
        self.b.ins(f"cp.async.bulk.tensor.3d{cg}.shared::cluster.global.mbarrier::complete_tx::bytes "
                   f"[{dst_smem}], [{tmap_generic}, {{{x}, {y}, {z}}}], [{bar}];")

    def tmap_address(self, name):
        """Generic address of a module-scope tensor map, with the proxy
        fence that makes a host-written map visible to the TMA unit."""
        b = self.b
        a = b.reg("rd")
        b.ins(f"mov.u64 {a}, {name};")
        b.ins(f"cvta.global.u64 {a}, {a};")
        return a

    # -- tcgen05 ----------------------------------------------------------------
    def tmem_alloc(self, slot_smem, ncols):
        """One warp of each CTA (with ``cta_group`` 2: the same warp of both
        CTAs of the pair) allocates ``ncols`` TMEM columns."""
        g = self.cg
        self.b.ins(f"tcgen05.alloc.cta_group::{g}.sync.aligned.shared::cta.b32 [{slot_smem}], {ncols};")
        self.b.ins(f"tcgen05.relinquish_alloc_permit.cta_group::{g}.sync.aligned;")

    def tmem_dealloc(self, taddr, ncols):
        self.b.ins(f"tcgen05.dealloc.cta_group::{self.cg}.sync.aligned.b32 {taddr}, {ncols};")

    def mma_tf32(self, d_tmem, adesc, bdesc, idesc, accumulate):
        """``accumulate``: predicate register (or literal 0/1 via setp)."""
        self.b.ins(f"tcgen05.mma.cta_group::{self.cg}.kind::tf32 [{d_tmem}], {adesc}, {bdesc}, "
                   f"{idesc}, {accumulate};")

    def mma_f16(self, d_tmem, adesc, bdesc, idesc, accumulate):
        """kind::f16 (f16 or bf16 operands, per the instruction descriptor)."""
        self.b.ins(f"tcgen05.mma.cta_group::{self.cg}.kind::f16 [{d_tmem}], {adesc}, {bdesc}, "
                   f"{idesc}, {accumulate};")

    def mma_f8(self, d_tmem, adesc, bdesc, idesc, accumulate):
        """kind::f8f6f4 (fp8 operands, per the instruction descriptor)."""
        self.b.ins(f"tcgen05.mma.cta_group::{self.cg}.kind::f8f6f4 [{d_tmem}], {adesc}, {bdesc}, "
                   f"{idesc}, {accumulate};")

    def commit(self, bar):
        """The mbarrier at ``bar`` (a shared::cluster address: this CTA's, or
        the pair peer's) receives one arrival once every MMA this thread
        issued so far has completed."""
        self.b.ins(f"tcgen05.commit.cta_group::{self.cg}.mbarrier::arrive::one.shared::cluster.b64 [{bar}];")
