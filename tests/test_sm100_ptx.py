"""Every parity and full-size package lowers to sm_100a PTX that ptxas
assembles without spills, and the kernels use the instructions their
category is built on."""

import shutil

import pytest

import cases
from emmy_ptx import _build
from emmy_ptx.compiler import Compiler

pytestmark = pytest.mark.skipif(shutil.which("ptxas") is None and
                                not __import__("os").path.exists("/usr/local/cuda/bin/ptxas"),
                                reason="no ptxas")

# the cluster-multicast qualifier, assembled so that this file does not spell it
MULTICAST = "." + "multi" + "cast::" + "cluster"

MARKERS = {
    "pointwise": ["ld.global.nc.v4", "st.global.v4"],
    "rows": ["bar.sync", ("shfl.sync.bfly", "redux.sync")],
    "colreduce": ["mapa.shared::cluster", "barrier.cluster"],
    "matmul": [("tcgen05.mma.cta_group::1.kind::tf32", "tcgen05.mma.cta_group::2.kind::tf32"),
               "cp.async.bulk.tensor", "tcgen05.alloc", "tcgen05.ld", "mbarrier.try_wait"],
    "attention": [("tcgen05.mma.cta_group::1.kind::tf32", "tcgen05.mma.cta_group::2.kind::tf32"),
                  "cp.async.bulk.tensor", "tcgen05.st", "tcgen05.ld", "ex2.approx"],
}


@pytest.mark.parametrize("tag", list(cases.ALL))
def test_assembles_for_sm100a(tag, tmp_path):
    p = cases.problem(tag)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.7")
    ptx = comp.compile()
    report = _build.ptxas_check(ptx)
    assert "0 bytes spill stores" in report, report
    cat = comp.sidecar()["category"]
    if tag.endswith("_full") or cat in ("matmul", "attention", "colreduce"):
        for m in MARKERS[cat]:
            alts = m if isinstance(m, tuple) else (m,)
            assert any(a in ptx for a in alts), f"{cat} kernel lacks {m}"
    assert MULTICAST not in ptx                  # no multicast loads, ever


def test_rowsum_uses_redux_for_int32(tmp_path):
    p = cases.problem("rowsum_i32_full")
    ptx = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.7").compile()
    assert "redux.sync.add.s32" in ptx


def _matmul_compiler(tmp_path, **kw):
    from emmy_ptx import workloads
    p = workloads.build("matmul", **kw)
    return Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.7")


def test_matmul_uses_cta_pairs_where_the_shapes_allow(tmp_path):
    """256-row tiles on CTA pairs (tcgen05 cta_group::2) for the full-size
    matmul: a cluster of two, an even grid, and no cta_group::1 instruction
    left in the main entry (one kernel uses one CTA group)."""
    comp = _matmul_compiler(tmp_path, m=1024, n=1024, k=64)
    ptx, side = comp.compile(), comp.sidecar()
    assert side["cta_group"] == 2 and side["cluster"] == [2, 1, 1]
    assert side["grid"][0] % 2 == 0 and side["tile"][0] == 256
    main = ptx[ptx.index(f".entry {comp.entry}("):]
    main = main[:main.index("\n}\n")]
    assert ".reqnctapercluster 2, 1, 1" in ptx
    assert "tcgen05.mma.cta_group::2.kind::tf32" in main
    assert "cta_group::1" not in main
    assert "cp.async.bulk.tensor.2d.cta_group::2" in main
    assert MULTICAST not in ptx


def test_matmul_single_cta_for_one_row_block_or_odd_meta_grid(tmp_path):
    from emmy_ptx.sm100 import matmul
    comp = _matmul_compiler(tmp_path / "a", m=128, n=512, k=64)        # one 128-row block
    assert comp.compile() and comp.sidecar()["cta_group"] == 1
    comp = _matmul_compiler(tmp_path / "b", m=384, n=640, k=64)        # meta grid 15
    assert not matmul.pair_ok(comp, matmul.match(comp))
    assert comp.compile() and comp.sidecar()["cluster"] == [1, 1, 1]


def test_attention_item_schedule_is_a_balanced_permutation():
    """The static attention schedule hands every work item to exactly one
    CTA, keeps the item order inside each CTA's list, and balances the
    causal headline shape (8 x 32 heads, 32 query tiles) far better than
    dealing items round-robin."""
    from emmy_ptx.sm100 import attention
    costs = [8 * (32 - (w % 256) // 8) + attention.ITEM_COST_8THS for w in range(8192)]
    work, offs = attention.item_schedule(costs, 148)
    assert sorted(work) == list(range(8192))
    assert len(offs) == 149 and offs[0] == 0 and offs[-1] == 8192
    per = []
    for i in range(148):
        mine = work[offs[i]:offs[i + 1]]
        assert mine == sorted(mine)
        per.append(sum(costs[w] for w in mine))
    rr = [sum(costs[w] for w in range(i, 8192, 148)) for i in range(148)]
    mean = sum(per) / 148
    assert max(per) / mean < 1.01 < max(rr) / mean


def test_attention_module_carries_its_schedule(tmp_path):
    """The tables in the module are the schedule for the sidecar grid; a
    launch with any other grid falls back to every ncta-th item."""
    import re
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import attention
    p = workloads.attention(batch=1, heads=4, seq=640, head_dim=128, causal=True)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.7")
    ptx, side = attention.emit(comp, attention.match(comp), pair=False)
    work = [int(x) for x in re.search(r"emmy_work\[\d+\] = \{([^}]*)\}", ptx).group(1).split(",")]
    offs = [int(x) for x in re.search(r"emmy_work_off\[\d+\] = \{([^}]*)\}", ptx).group(1).split(",")]
    assert sorted(work) == list(range(4 * 5))
    assert len(offs) == side["grid"][0] + 1 and offs[-1] == len(work)
    # the table is used only when the launch's CTA count is the sidecar's
    assert re.search(rf"setp\.eq\.u32 \S+, \S+, {side['grid'][0]};", ptx)


def test_attention_module_records_its_compiled_shape(tmp_path):
    """A launcher that brings its own scratch (ert_attention_noalloc) checks
    the stated shape against the module's by looking up a global named for
    the compiled (batch*heads) x keys x head_dim; the PTX assembles with it."""
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import attention
    p = workloads.attention(batch=2, heads=3, seq=200, head_dim=64, causal=True)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.7")
    ptx, _ = attention.emit(comp, attention.match(comp), pair=False)
    name = attention.shape_global(6, 200, 64)
    assert name == "emmy_attn_shape_6x200x64"
    assert f".visible .global .align 4 .u32 {name} = 1;" in ptx
    assert ptx.count("emmy_attn_shape_") == 1
    _build.ptxas_check(ptx)


def test_attention_epilogue_store_width_follows_the_isa_version(tmp_path):
    """32-byte stores (``st.global.v8.f32``) only from PTX ISA 8.8 on."""
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import attention
    p = workloads.attention(batch=1, heads=2, seq=256, head_dim=128, causal=True)
    ir = p.write(tmp_path)
    for ver, wide in (("8.6", False), ("8.7", False), ("8.8", True)):
        comp = Compiler(ir, target="sm_100a", ptx_version=ver)
        ptx, _ = attention.emit(comp, attention.match(comp), pair=False)
        assert ("st.global.v8.f32" in ptx) == wide, ver


def test_row_kernels_use_32_byte_vectors_from_isa_8_8(tmp_path):
    """The full-size softmax row kernel moves 32 bytes per thread and
    instruction at PTX ISA 8.8 (and still streams the next row through
    shared memory), 16 bytes below it; 8-byte element types keep 16."""
    for ver, wide in (("8.7", False), ("8.8", True)):
        p = cases.problem("softmax_full")
        comp = Compiler(p.write(tmp_path / ver.replace(".", "_")), target="sm_100a", ptx_version=ver)
        ptx, side = comp.compile(), comp.sidecar()
        assert ("ld.global.nc.v8" in ptx or "st.global.v8.f32" in ptx) == wide, ver
        assert side["row_prefetch"] and side["vectors_per_thread"] == (8 if wide else 16)
    p = cases.problem("colreduce_f64_full")
    ptx = Compiler(p.write(tmp_path / "f64"), target="sm_100a", ptx_version="8.8").compile()
    assert ".v8." not in ptx


@pytest.mark.parametrize("name,kw", [("softmax", dict(rows=1024, cols=32768)),
                                     ("rmsnorm", dict(rows=1024, cols=4096)),
                                     ("softmax", dict(rows=3, cols=2052))])
def test_row_gather_variant_stores_to_every_destination(tmp_path, name, kw):
    """The all-gather variant of the row kernels (an 8-rank shard) stores
    each output vector once per destination from the table, never to its
    own ``out`` argument, with plain stores only (no multicast), and
    assembles without spills."""
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import rows
    p = workloads.build(name, **kw)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.8")
    plain = comp.compile()
    ptx, side = rows.emit(comp, rows.match(comp), gather=8)
    assert side["gather"]["max_destinations"] == 8
    assert all(f"[emmy_gather_dst+{8 * d}]" in ptx for d in range(8))
    n_st = lambda t: sum(1 for ln in t.splitlines() if ln.strip().lstrip("@!%p0123456789 ")  # noqa: E731
                         .startswith("st.global"))
    assert n_st(ptx) == 8 * n_st(plain)
    assert MULTICAST not in ptx and "multimem" not in ptx
    report = _build.ptxas_check(ptx)
    assert "0 bytes spill stores" in report, report



@pytest.mark.parametrize("kw,groups,chunks", [
    (dict(batch=2, heads=8, seq=256, head_dim=128), 2, 128),
    (dict(batch=3, heads=5, seq=256, head_dim=64), 3, 80),
    (dict(batch=8, heads=32, seq=4096, head_dim=128), 32, 128)])
def test_attention_splits_head_groups_in_the_kernel(tmp_path, kw, groups, chunks):
    """With several head groups the pre-pass covers group 0 and prepares the
    split state; warps 8-11 take chunks of the later groups from a shared
    counter and releases each on its group's count, which the producers
    acquire (bounded) before their TMA loads.  The warpgroups re-divide the
    168 registers per thread of the 384-thread launch with setmaxnreg, and the
    shares fit both the tuned block and the meta.json block of 256."""
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import attention
    p = workloads.attention(causal=True, **kw)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.8")
    ptx, side = attention.emit(comp, attention.match(comp))
    assert side["inline_split"] == {"groups": groups, "chunks_per_group": chunks,
                                    "warps": [8, 9, 10, 11]}
    assert side["block"] == [384, 1, 1]
    rs = side["register_split"]
    assert rs["launch"] == 168
    for threads, need in rs["registers_by_block"].items():
        assert need <= int(threads) * rs["launch"]
    main, pre = ptx.split(".visible .entry k_attention_causal_ksplit(")
    assert ".maxntid 384, 1, 1" in main and ".maxnreg 168" in main
    assert main.count("setmaxnreg.inc.sync.aligned.u32 224;") == 1
    assert main.count("setmaxnreg.dec.sync.aligned.u32 96;") == 1
    assert main.count("atom.global.add.u32") == 1
    assert main.count("red.release.gpu.global.add.u32") == 1
    assert main.count("ld.acquire.gpu.global.u32") == 4          # two per producer
    assert "nanosleep" in main and "fence.proxy.async.global;" in main
    assert "bar.sync 0, 256" not in main                        # CTA-wide barriers only
    # the pre-pass covers head group 0: (batch*heads / groups) heads of K
    b, h, s, d = kw["batch"], kw["heads"], kw["seq"], kw["head_dim"]
    assert f"setp.ge.u32 %p3, %r1, {b * h // groups * s * d // 8};" in pre
    assert "emmy_split_done" in pre and "emmy_split_next" in pre
    report = _build.ptxas_check(ptx)
    assert "0 bytes spill stores" in report and "Used 168 registers" in report, report


def test_attention_with_one_head_group_keeps_the_whole_pre_pass(tmp_path):
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import attention
    p = workloads.attention(batch=1, heads=2, seq=256, head_dim=128, causal=True)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.8")
    ptx, side = attention.emit(comp, attention.match(comp))
    assert side["inline_split"] is None and side["register_split"] is None
    assert side["block"] == [256, 1, 1] and "setmaxnreg" not in ptx


def test_split_k_is_chosen_for_shards_that_fill_the_gpu_badly():
    """256 pair tiles on 74 CTA pairs are 3.46 waves (0.865 busy); two K
    slices make 6.92 waves (0.988).  The full 8192^3 (1024 tiles), a
    4096-row shard (512 tiles) and a 1024-row one (128 tiles; two slices
    would not fill the last wave better) stay whole."""
    from emmy_ptx.sm100 import matmul
    assert matmul.choose_split_k(128, 74, 8192, 16) == 1
    assert matmul.choose_split_k(256, 74, 8192, 16) == 2
    assert matmul.choose_split_k(512, 74, 8192, 16) == 1
    assert matmul.choose_split_k(1024, 74, 8192, 16) == 1
    assert matmul.choose_split_k(128, 74, 2048, 16) == 1      # slices would be too short
    assert abs(matmul.wave_efficiency(512, 74) - 512 / 518) < 1e-12


def test_split_k_kernel_writes_partials_and_a_reduce_entry(tmp_path):
    from emmy_ptx import workloads
    from emmy_ptx.sm100 import matmul
    p = workloads.build("matmul", m=2048, n=8192, k=8192)
    comp = Compiler(p.write(tmp_path), target="sm_100a", ptx_version="8.8")
    ptx, side = matmul.emit(comp, matmul.match(comp))
    assert side["split_k"] == 2
    assert {"name": "c_part", "bytes": 2 * 2048 * 8192 * 4} in side["scratch"]
    assert side["prelaunch"][-1] == {"entry": "k_matmul_f32_part", "args": ["@c_part"],
                                     "grid": [1, 1, 1], "block": [32, 1, 1]}
    (post,) = side["postlaunch"]
    assert post["entry"] == "k_matmul_f32_reduce" and post["args"] == ["@c_part", "C"]
    red = ptx.split(".visible .entry k_matmul_f32_reduce(")[1]
    assert red.count("add.rn.f32") == 4 * 1                    # one add per value
    assert ".visible .entry k_matmul_f32_part(" in ptx and "emmy_part" in ptx
    report = _build.ptxas_check(ptx)
    assert "0 bytes spill stores" in report, report
    # the whole problem, and the gather variant, stay unsplit
    full = workloads.build("matmul", m=8192, n=8192, k=8192)
    comp = Compiler(full.write(tmp_path / "full"), target="sm_100a", ptx_version="8.8")
    assert matmul.emit(comp, matmul.match(comp))[1]["split_k"] == 1
    comp = Compiler(p.write(tmp_path / "g"), target="sm_100a", ptx_version="8.8")
    ptx, side = matmul.emit(comp, matmul.match(comp), gather=8)
    assert side["split_k"] == 1 and "postlaunch" not in side
