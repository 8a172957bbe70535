"""Compile every IR package in cases.py with the unmodified reference compiler.

Run in a container that has the reference checkout (it is not needed, and not
read, anywhere else):

    python tests/golden/make_ref_ptx.py --reference /path/to/emmy-ptx

For each tag it writes ``problems/<tag>/`` (the IR package: ``*.ir.json`` +
``meta.json``, written by emmy_ptx.workloads) and ``problems/<tag>/ref.ptx``,
the reference compiler's PTX at its defaults (``.target sm_89``,
``.version 8.0``), which the B200 driver JIT-compiles.  The reference imports
``emmy`` (emmy-ml, not installable); ``emmy_shim/`` stands in for it.
"""

import argparse
import os
import importlib.util
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "emmy-ptx_b200"))
sys.path.insert(0, str(HERE / "emmy_shim"))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402


def load_reference(root: Path):
    path = root / "src" / "emmy_ptx" / "compiler.py"
    spec = importlib.util.spec_from_file_location("_reference_emmy_ptx_compiler", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EMMY_PTX_REFERENCE"),
                    required="EMMY_PTX_REFERENCE" not in os.environ,
                    help="root of the reference emmy-ptx checkout (or set "
                         "EMMY_PTX_REFERENCE)")
    ap.add_argument("--tags", nargs="*", default=None)
    ap.add_argument("--no-ptxas", action="store_true")
    args = ap.parse_args()
    ref = load_reference(Path(args.reference))
    for tag in args.tags or list(cases.ALL):
        p = cases.problem(tag)
        d = HERE / "problems" / tag
        ir_path = p.write(d)
        ptx = ref.Compiler(ir_path).compile()
        (d / "ref.ptx").write_text(ptx)
        status = ""
        if not args.no_ptxas:
            r = subprocess.run(["ptxas", "-arch=sm_89", str(d / "ref.ptx"), "-o", "/dev/null"],
                               capture_output=True, text=True)
            status = "ptxas ok" if r.returncode == 0 else "PTXAS FAILED: " + r.stderr.strip()[:300]
        print(f"{tag:28s} {len(ptx):8d} bytes  {status}")


if __name__ == "__main__":
    main()
