"""The general statement-level lowering (emmy_ptx.sm100.general), on the CPU:
every IR package assembles for sm_100a and for the reference's default
target, constructs map to the PTX they should, and errors keep the
reference's conventions."""

import json

import numpy as np
import pytest

from emmy_ptx import _build, workloads
from emmy_ptx.compiler import Compiler
from emmy_ptx.sm100 import general

SMALL = {"pointwise_f32": dict(rows=33, cols=100), "pointwise_i32": dict(rows=33, cols=100),
         "rmsnorm": dict(rows=5, cols=1000), "softmax": dict(rows=3, cols=2052),
         "colreduce_f64": dict(rows=100, cols=64), "rowsum_i32": dict(rows=7, cols=68),
         "matmul": dict(m=128, n=128, k=64),
         "attention": dict(batch=1, heads=2, seq=64, head_dim=128),
         "pointwise_zoo": dict(rows=16, cols=64), "pointwise_mixed": dict(rows=16, cols=64),
         "histogram_i32": dict(rows=16, cols=100, bins=13), "control_flow": dict(n=300),
         "matmul_bf16": dict(m=128, n=128, k=64), "matmul_e4m3": dict(m=128, n=128, k=128),
         "matmul_e5m2": dict(m=128, n=128, k=128), "bit_ops": dict(rows=7, cols=36),
         "rowsum_f64": dict(rows=9, cols=300), "offset_copy": dict(rows=5, cols=68, offset=0, pad=2)}


def _comp(name, tmp_path, target="sm_100a", version="8.7", **kw):
    p = workloads.build(name, **(kw or SMALL[name]))
    ir = p.write(tmp_path / name)
    return p, Compiler(ir, target=target, ptx_version=version)


@pytest.mark.parametrize("target,version", [("sm_100a", "8.7"), ("sm_89", "8.0")])
@pytest.mark.parametrize("name", sorted(SMALL))
def test_every_package_assembles(name, target, version, tmp_path):
    p, comp = _comp(name, tmp_path, target, version)
    ptx, side = general.emit(comp)
    assert ptx.startswith(f".version {version}\n.target {target}\n")
    assert f".visible .entry {comp.entry}(" in ptx
    params = [f"p_{a}" for a in p.inputs + p.outputs]
    order = [ptx.index(f"\t.param .u64 {n}") for n in params]
    assert order == sorted(order), "parameters follow meta arg_order"
    report = _build.ptxas_check(ptx, arch=target)
    assert "0 bytes spill stores" in report
    assert side["grid"] == list(p.grid) and side["block"] == list(p.block)


def test_unmatched_kernels_take_the_general_path(tmp_path):
    for name in ("histogram_i32", "control_flow"):
        _, comp = _comp(name, tmp_path)
        comp.compile()
        side = comp.sidecar()
        assert side["category"] == "general"
        assert any(r.startswith("pointwise:") for r in side["category_reasons"])


def test_zero_prologue_is_a_prelaunch_entry(tmp_path):
    _, comp = _comp("histogram_i32", tmp_path)
    ptx, side = general.emit(comp)
    (pre,) = side["prelaunch"]
    assert pre["entry"] == "k_histogram_i32_zero0" and pre["args"] == ["counts"]
    assert ".visible .entry k_histogram_i32_zero0(" in ptx
    assert "red.global.add.s32" in ptx


def test_integer_butterfly_becomes_redux_on_sm100a(tmp_path):
    _, comp = _comp("rowsum_i32", tmp_path)
    ptx, _ = general.emit(comp)
    assert "redux.sync.add.s32" in ptx and "shfl.sync.bfly" not in ptx
    _, comp89 = _comp("rowsum_i32", tmp_path / "89", "sm_89", "8.0")
    ptx89, _ = general.emit(comp89)
    assert "redux" not in ptx89 and "shfl.sync.bfly.b32" in ptx89


def test_vector_and_read_only_loads(tmp_path):
    _, comp = _comp("pointwise_f32", tmp_path, rows=64, cols=256)
    ptx, _ = general.emit(comp)
    assert "ld.global.nc.v4.f32" in ptx and "st.global.v4.f32" in ptx


@pytest.mark.parametrize("offset,pad,vector", [(4, 4, True), (1, 4, False), (2, 4, False),
                                               (0, 2, False), (0, 4, True)])
def test_grouped_load_is_a_vector_only_when_aligned(tmp_path, offset, pad, vector):
    """A 4-wide group becomes one 16-byte access only when its first
    element is provably 16-byte aligned: the column offset and the row
    length both multiples of 4 (reference tests/test_compiler.py:101-203).
    Anything else stays four scalar accesses, which the GPU requires."""
    _, comp = _comp("offset_copy", tmp_path, rows=8, cols=64, offset=offset, pad=pad)
    ptx, _ = general.emit(comp)
    assert ("ld.global.nc.v4.f32" in ptx) == vector
    assert ("ld.global.nc.f32" in ptx) == (not vector)
    assert "st.global.v4.f32" in ptx


def test_atomic_grouped_write_stays_scalar(tmp_path):
    """Atomic writes of a group are one reduction per element."""
    from emmy_ptx.ir import F32, Axis, Dim, KernelOp, Load, Tile, Write
    from emmy_ptx.workloads import Problem, V, _names, _t, mul
    idx = (V("a0"), mul(V("a1"), 4))
    x = _names("x", 4)
    tile = Tile((Axis("a0", Dim(4)), Axis("a1", Dim(8))),
                (Load(x, "x", idx, F32), Write("out", idx, x, F32, True, "NONE")),
                block_threads=32)
    p = Problem("atomic_add", "atomic_add", KernelOp("k_atomic_add", ("x",), ("out",), (tile,)),
                [_t("x", (4, 32), "f32"), _t("out", (4, 32), "f32")], (1, 1, 1), (32, 1, 1), 0)
    comp = Compiler(p.write(tmp_path / "atomic"), target="sm_100a", ptx_version="8.7")
    ptx, _ = general.emit(comp)
    assert "red.global.add.f32" in ptx or "atom.global.add.f32" in ptx
    assert ".v4" not in "\n".join(line for line in ptx.splitlines() if "red." in line or "atom." in line)
    assert "st.global.v4" not in ptx


def test_a_value_assigned_in_both_branches_is_one_register(tmp_path):
    """``y`` is assigned on both paths of the Cond and read after it: both
    branches must write the same register."""
    _, comp = _comp("control_flow", tmp_path)
    ptx, _ = general.emit(comp)
    body = ptx.split("ELSE_", 1)[1]
    assert "sqrt.rn.f32" in ptx and "COND_END" in body


def test_unsupported_construct_names_the_statement(tmp_path):
    p, comp = _comp("control_flow", tmp_path)
    doc = json.loads(comp.ir_path.read_text())
    body = doc["nodes"]["kernel"]["op_fields"]["body"]
    doc["nodes"]["kernel"]["op_fields"]["body"] = [body[0].replace("'tanh'", "'bogus_fn'")]
    comp.ir_path.write_text(json.dumps(doc))
    with pytest.raises(SystemExit) as exc:
        Compiler(comp.ir_path).compile()
    msg = str(exc.value)
    assert "bogus_fn" in msg and "while lowering statement" in msg


def test_shared_memory_above_48k_is_dynamic(tmp_path):
    _, comp = _comp("matmul", tmp_path)
    ptx, side = general.emit(comp)
    assert ".extern .shared .align 16 .b8 emmy_smem[];" in ptx
    assert side["shared_bytes"] >= 48 * 1024
    assert "cp.async.cg.shared.global" in ptx and "cp.async.wait_group" in ptx


def test_oracle_closed_forms_for_the_general_cases(tmp_path):
    from oracle import simt
    p = workloads.build("histogram_i32", rows=16, cols=100, bins=13)
    inp = p.make_inputs()
    out = simt.run_problem(p, inp, str(tmp_path / "h"),
                           out_init={"counts": np.full(13, 12345, np.int32)})
    assert np.array_equal(out["counts"], np.bincount(inp["x"].ravel(), minlength=13))
    p = workloads.build("control_flow", n=300)
    inp = p.make_inputs()
    out = simt.run_problem(p, inp, str(tmp_path / "c"))
    x = inp["x"].astype(np.float64)
    k = inp["k"].astype(np.int64)
    y = np.where(x > 0, np.sqrt(np.maximum(x, 0)), -x * x)
    sel = np.where(k < 0, -1.0, np.where(k == 0, y ** 3, 10 * y))
    z = np.where(k % 2 == 0, sel, y)
    np.testing.assert_allclose(out["out"], np.tanh(z) + np.arange(300), rtol=1e-5, atol=1e-5)
    q = np.trunc(y * 8).astype(np.int64)
    kq = np.trunc(k / 4).astype(np.int64)
    kr = k - np.trunc(k / -7).astype(np.int64) * -7
    assert np.array_equal(out["out_i"], q + kq + kr)


def test_fp8_decode_tables_match_torch():
    """The oracle's E4M3 / E5M2 decode, written from the format definitions,
    against torch's float8 types for all 256 codes."""
    import torch
    from oracle.ops import F8E4M3, F8E5M2
    codes = torch.arange(256, dtype=torch.uint8)
    assert np.array_equal(F8E4M3, codes.view(torch.float8_e4m3fn).float().numpy(), equal_nan=True)
    assert np.array_equal(F8E5M2, codes.view(torch.float8_e5m2).float().numpy(), equal_nan=True)


def test_oracle_closed_forms_for_low_precision_matmuls(tmp_path):
    from oracle import simt
    from oracle.ops import F8E4M3, F8E5M2
    for name, kw in (("matmul_bf16", dict(m=128, n=128, k=64)),
                     ("matmul_f16", dict(m=128, n=128, k=64)),
                     ("matmul_e4m3", dict(m=128, n=128, k=128)),
                     ("matmul_e5m2", dict(m=128, n=128, k=128))):
        p = workloads.build(name, **kw)
        inp = p.make_inputs()
        out = simt.run_problem(p, inp, str(tmp_path / name))
        if name.endswith("bf16"):
            a, b = ((inp[n].astype(np.uint32) << 16).view(np.float32) for n in "AB")
        elif name.endswith("f16"):
            a, b = inp["A"], inp["B"]
        else:
            tab = F8E4M3 if "e4m3" in name else F8E5M2
            a, b = tab[inp["A"]], tab[inp["B"]]
        want = a.astype(np.float64) @ b.astype(np.float64)
        # exact products, f32 sums: differences are f32 rounding only
        assert np.abs(out["C"] - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), name


def test_fp8_decode_on_targets_without_the_conversion(tmp_path):
    """sm_89 at PTX 8.0 has no fp8 conversion instruction: the decode is
    built from the code's fields instead."""
    _, comp = _comp("matmul_e4m3", tmp_path, "sm_89", "8.0")
    ptx, _ = general.emit(comp)
    assert "e4m3x2" not in ptx and "bfe.u32" in ptx
    _, comp = _comp("matmul_e4m3", tmp_path / "b", "sm_100a", "8.7")
    ptx, _ = general.emit(comp)
    assert "cvt.rn.f16x2.e4m3x2" in ptx
