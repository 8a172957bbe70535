"""The drop-in API surface: names, defaults, errors, meta.json contract."""

import contextlib
import io
import json
import re
import shutil

import pytest

import emmy_ptx
from emmy_ptx import Compiler, compile_file, ptx_header, workloads
from emmy_ptx import compiler as C


@pytest.fixture
def pkg(tmp_path):
    p = workloads.pointwise_f32(rows=8, cols=64)
    return p, p.write(tmp_path / "pw")


def test_exports():
    for name in ("Compiler", "compile_file", "ptx_header", "SUPPORTED_TARGETS",
                 "SUPPORTED_VERSIONS", "__version__"):
        assert hasattr(emmy_ptx, name)
    assert {"sm_89", "sm_100", "sm_100a"} <= emmy_ptx.SUPPORTED_TARGETS
    assert {"8.0", "8.6", "8.7", "8.8"} <= emmy_ptx.SUPPORTED_VERSIONS


def test_ptx_header_and_errors():
    assert ptx_header() == ".version 8.0\n.target sm_89\n.address_size 64\n"
    assert ptx_header("8.7", "sm_100a").startswith(".version 8.7\n.target sm_100a")
    with pytest.raises(ValueError):
        ptx_header("8.0", "sm_42")
    with pytest.raises(ValueError):
        ptx_header("6.5", "sm_89")
    with pytest.raises(ValueError):
        ptx_header("8.0", "sm_100a")          # sm_100a needs ISA 8.6+


def test_float_bit_helpers_match_reference_pins():
    # the reference tests' only numeric pins (test_compiler.py:57-61, 360-368)
    assert C.float_bits(1.0) == 0x3F800000
    assert C.float_bits(float("-inf")) == 0xFF800000
    assert C.float_bits(0.0) == 0
    assert C.float16_bits(1.0) == 0x3C00
    assert C.float16_bits(0.5) == 0x3800
    assert C.float16_bits(-2.0) == 0xC000
    assert C.float64_bits(1.0) == 0x3FF0000000000000


def test_entry_and_param_order_from_meta(pkg):
    p, ir_path = pkg
    ptx = Compiler(ir_path, target="sm_100a", ptx_version="8.7").compile()
    assert ".visible .entry k_silu_add_pointwise(" in ptx
    params = re.findall(r"\.param \.\w+ (p_\w+)", ptx)
    assert params == [f"p_{n}" for n in p.meta()["kernels"][0]["arg_order"]]
    assert ptx.endswith("}\n")
    ptx.encode("ascii")


def test_param_order_follows_meta_not_ir(pkg, tmp_path):
    p, ir_path = pkg
    meta = json.loads((ir_path.parent / "meta.json").read_text())
    meta["kernels"][0]["arg_order"] = ["out", "y", "x"]
    (ir_path.parent / "meta.json").write_text(json.dumps(meta))
    ptx = Compiler(ir_path, target="sm_100a", ptx_version="8.7").compile()
    assert re.findall(r"\.param \.\w+ (p_\w+)", ptx) == ["p_out", "p_y", "p_x"]


def test_missing_meta_falls_back_to_ir_order(pkg, tmp_path):
    p, ir_path = pkg
    lonely = tmp_path / "lonely"
    shutil.copytree(ir_path.parent, lonely)
    (lonely / "meta.json").unlink()
    err = io.StringIO()
    with contextlib.redirect_stderr(err):
        comp = Compiler(lonely / ir_path.name, target="sm_100a", ptx_version="8.7")
    assert "warning: no meta.json found" in err.getvalue()
    assert comp.arg_order == ["x", "y", "out"]


def test_ancestor_meta_is_used_when_it_names_the_kernel(pkg, tmp_path):
    p, ir_path = pkg
    nested = tmp_path / "a" / "b"
    nested.mkdir(parents=True)
    shutil.copy(ir_path, nested / ir_path.name)
    shutil.copy(ir_path.parent / "meta.json", tmp_path / "a" / "meta.json")
    comp = Compiler(nested / ir_path.name, target="sm_100a", ptx_version="8.7")
    assert comp.kmeta["entry"] == "k_silu_add_pointwise"


def test_serial_kernels_are_rejected(pkg):
    p, ir_path = pkg
    doc = json.loads(ir_path.read_text())
    doc["nodes"]["kernel"]["op_fields"]["serial"] = ["s0"]
    ir_path.write_text(json.dumps(doc))
    with pytest.raises(SystemExit, match="serial"):
        Compiler(ir_path, target="sm_100a", ptx_version="8.7")


def test_unlowerable_kernel_fails_loudly_with_reasons(pkg):
    p, ir_path = pkg
    doc = json.loads(ir_path.read_text())
    body = doc["nodes"]["kernel"]["op_fields"]["body"]
    doc["nodes"]["kernel"]["op_fields"]["body"] = [body[0].replace("'sigmoid'", "'bogus_op'")]
    ir_path.write_text(json.dumps(doc))
    with pytest.raises(SystemExit, match="bogus_op|no sm_100a category|unsupported"):
        Compiler(ir_path, target="sm_100a", ptx_version="8.7").compile()


def test_default_target_compiles_through_the_general_lowering(pkg):
    p, ir_path = pkg
    comp = Compiler(ir_path)
    ptx = comp.compile()
    assert ptx.startswith(".version 8.0\n.target sm_89\n")
    assert ".visible .entry k_silu_add_pointwise(" in ptx and ptx.endswith("}\n")
    assert comp.sidecar()["category"] == "general"
    assert "tcgen05" not in ptx and "redux" not in ptx
    assert Compiler(ir_path).check() == []


def test_check_ok_for_b200(pkg):
    p, ir_path = pkg
    assert Compiler(ir_path, target="sm_100a", ptx_version="8.7").check() == []


def test_cache_dir(pkg, tmp_path):
    p, ir_path = pkg
    cache = tmp_path / "cache"
    a = compile_file(ir_path, target="sm_100a", ptx_version="8.7", cache_dir=cache)
    files = sorted(x.suffix for x in cache.iterdir())
    assert files == [".json", ".ptx"]
    assert compile_file(ir_path, target="sm_100a", ptx_version="8.7", cache_dir=cache) == a


def test_compile_is_repeatable(pkg):
    p, ir_path = pkg
    comp = Compiler(ir_path, target="sm_100a", ptx_version="8.7")
    assert comp.compile() == comp.compile()


@pytest.mark.parametrize("name", list(workloads.BUILDERS))
def test_every_config_has_an_sm100a_lowering(name, tmp_path):
    p = workloads.build(name)
    ir_path = p.write(tmp_path / name)
    comp = Compiler(ir_path, target="sm_100a", ptx_version="8.7")
    ptx = comp.compile()
    side = comp.sidecar()
    assert ".target sm_100a" in ptx
    # the kernel keeps the meta.json block size; attention with several head
    # groups adds its split warp to the tuned launch and still runs (split
    # first, then compute) on the meta.json block
    extra = 32 * len(side["inline_split"]["warps"]) if side.get("inline_split") else 0
    assert side["block"][0] == p.block[0] + extra, "the kernel keeps the meta.json block size"
    assert side["arg_order"] == p.inputs + p.outputs
