"""Command-line entry point, with the reference's flags and exit codes
(cli.py:9-70): PTX to stdout (or ``-o``), ``--check`` prints issues, errors
go to stderr with exit code 1.  With ``-o`` the launch sidecar is written
next to the PTX as ``<output>.launch.json`` for sm_100a kernels."""

import argparse
import json
import sys

from .compiler import SUPPORTED_TARGETS, SUPPORTED_VERSIONS, Compiler


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(
        prog="emmy-ptx",
        description="Compile Emmy Kernel IR to NVIDIA PTX.",
    )
    parser.add_argument("ir_path", help="path to a Kernel IR JSON file")
    parser.add_argument(
        "--target", default="sm_89", choices=sorted(SUPPORTED_TARGETS),
        help="GPU target architecture (default: sm_89; B200 kernels: sm_100a)",
    )
    parser.add_argument(
        "--version", default="8.0", dest="ptx_version",
        choices=sorted(SUPPORTED_VERSIONS),
        help="PTX ISA version (default: 8.0; sm_100a needs 8.6 or later)",
    )
    parser.add_argument("-o", "--output", help="write PTX to this file instead of stdout")
    parser.add_argument(
        "--check", action="store_true",
        help="validate the IR without compiling; print issues and exit",
    )
    parser.add_argument(
        "--cache-dir", default=None,
        help="cache compiled PTX by IR hash (skip recompilation on cache hit)",
    )
    args = parser.parse_args(argv)

    if args.check:
        try:
            compiler = Compiler(args.ir_path, target=args.target, ptx_version=args.ptx_version)
            issues = compiler.check()
        except (SystemExit, Exception) as exc:  # noqa: BLE001
            print(f"error: {exc}", file=sys.stderr)
            return 1
        if issues:
            print(f"{len(issues)} issue(s) found:")
            for issue in issues:
                print(f"  - {issue}")
            return 1
        print("OK — no issues found")
        return 0

    try:
        # every path goes through the cache, as the reference's does
        # (cli.py:50-66): ``-o`` only changes where the PTX is written
        from .compiler import compile_cached
        ptx, sidecar = compile_cached(args.ir_path, target=args.target,
                                      ptx_version=args.ptx_version, cache_dir=args.cache_dir)
    except (SystemExit, ValueError, Exception) as exc:  # noqa: BLE001
        print(str(exc), file=sys.stderr)
        return 1
    if args.output:
        with open(args.output, "w") as f:
            f.write(ptx)
        if sidecar:
            with open(args.output + ".launch.json", "w") as f:
                json.dump(sidecar, f, indent=1)
    else:
        sys.stdout.write(ptx)
        if not ptx.endswith("\n"):
            sys.stdout.write("\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
