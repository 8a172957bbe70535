"""The emmy-ptx CLI (reference cli.py:9-70 behaviour)."""

import json
import subprocess
import sys
from pathlib import Path

from emmy_ptx import workloads
from emmy_ptx.cli import main

ROOT = Path(__file__).resolve().parent.parent


def _pkg(tmp_path):
    return workloads.rowsum_i32(rows=8, cols=64).write(tmp_path / "rs")


def test_stdout(tmp_path, capsys):
    ir = _pkg(tmp_path)
    assert main([str(ir), "--target", "sm_100a", "--version", "8.7"]) == 0
    out = capsys.readouterr().out
    assert out.startswith(".version 8.7") and out.endswith("}\n")


def test_output_file_and_sidecar(tmp_path):
    ir = _pkg(tmp_path)
    out = tmp_path / "k.ptx"
    assert main([str(ir), "--target", "sm_100a", "--version", "8.7", "-o", str(out)]) == 0
    side = json.loads((tmp_path / "k.ptx.launch.json").read_text())
    assert side["entry"] == "k_rowsum_i32" and side["category"] == "rows"


def test_output_file_goes_through_the_cache(tmp_path):
    """``--cache-dir D -o out.ptx`` compiles into ``D/<key>.ptx`` (and the
    sidecar into ``D/<key>.json``), as the reference routes ``-o`` through
    compile_file (cli.py:50-66); a second run is a cache hit with identical
    output and sidecar."""
    from emmy_ptx.compiler import _cache_key
    ir = _pkg(tmp_path)
    cache = tmp_path / "cache"
    args = [str(ir), "--target", "sm_100a", "--version", "8.7", "--cache-dir", str(cache)]
    out1, out2 = tmp_path / "a.ptx", tmp_path / "b.ptx"
    assert main(args + ["-o", str(out1)]) == 0
    key = _cache_key(ir, "sm_100a", "8.7")
    cached = cache / f"{key}.ptx"
    assert cached.read_text() == out1.read_text()
    assert (cache / f"{key}.json").exists()
    # a cache hit: the cached PTX is served (mark it to prove it was read)
    cached.write_text(cached.read_text() + "// cached\n")
    assert main(args + ["-o", str(out2)]) == 0
    assert out2.read_text() == cached.read_text()
    assert (json.loads((tmp_path / "b.ptx.launch.json").read_text())
            == json.loads((tmp_path / "a.ptx.launch.json").read_text()))


def test_check(tmp_path, capsys):
    ir = _pkg(tmp_path)
    assert main([str(ir), "--target", "sm_100a", "--version", "8.7", "--check"]) == 0
    assert "OK — no issues found" in capsys.readouterr().out
    assert main([str(ir), "--check"]) == 0      # the default target: general lowering
    assert "OK — no issues found" in capsys.readouterr().out


def test_check_reports_a_grid_that_does_not_cover_the_tile(tmp_path, capsys):
    ir = _pkg(tmp_path)
    meta = json.loads((ir.parent / "meta.json").read_text())
    meta["kernels"][0]["grid"] = [1, 1, 1]
    (ir.parent / "meta.json").write_text(json.dumps(meta))
    assert main([str(ir), "--target", "sm_100a", "--version", "8.7", "--check"]) == 1
    assert "covers" in capsys.readouterr().out


def test_errors_go_to_stderr_with_exit_1(tmp_path, capsys):
    ir = _pkg(tmp_path)
    assert main([str(ir), "--target", "sm_100a", "--version", "8.0"]) == 1
    assert "8.6" in capsys.readouterr().err


def test_module_entry_point(tmp_path):
    ir = _pkg(tmp_path)
    r = subprocess.run([sys.executable, "-m", "emmy_ptx", str(ir), "--target", "sm_100a",
                        "--version", "8.7"], capture_output=True, text=True,
                       env={"PYTHONPATH": str(ROOT / "emmy-ptx_b200"), "PATH": "/usr/bin:/bin"})
    assert r.returncode == 0, r.stderr
    assert ".entry k_rowsum_i32" in r.stdout
