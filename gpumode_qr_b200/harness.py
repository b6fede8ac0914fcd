"""Run the reference's own harness with this library's variants registered.

    python -m gpumode_qr_b200.harness --reference /path/to/gpumode_qr [run_baseline args...]

Imports the reference's ``qrbench.variants``, inserts ``b200_geqrf`` (and the
other entries of :data:`gpumode_qr_b200.variants.VARIANTS`) into its
``VARIANTS`` / ``VARIANT_INFO`` before ``scripts/run_baseline.py`` is executed,
then runs that script unchanged: its registry is built from the same dict at
import time (``scripts/run_baseline.py:30-40``), so ``--impl b200_geqrf``,
``--compare --impls b200_geqrf,torch_geqrf``, ``--stress`` and ``--list`` all
work. Results go to ``--db-dir`` (default ``./db``) because the reference tree
may be read-only.
"""

from __future__ import annotations

import argparse
import os
import runpy
import sys
from pathlib import Path

from .variants import register_into_qrbench


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    ap = argparse.ArgumentParser(add_help=False)
    ap.add_argument("--reference", default=os.environ.get("QRBENCH_REFERENCE"))
    known, rest = ap.parse_known_args(argv)
    if not known.reference:
        print("error: pass --reference <gpumode_qr checkout> or set QRBENCH_REFERENCE", file=sys.stderr)
        return 2
    ref = Path(known.reference).resolve()
    script = ref / "scripts" / "run_baseline.py"
    if not script.exists():
        print(f"error: {script} not found", file=sys.stderr)
        return 2
    sys.path.insert(0, str(ref / "src"))
    import qrbench.variants as ref_variants  # noqa: PLC0415 - the reference's module

    register_into_qrbench(ref_variants)
    if "--db-dir" not in rest and "--no-write" not in rest and "--list" not in rest:
        rest += ["--db-dir", str(Path.cwd() / "db")]
    sys.argv = [str(script), *rest]
    try:
        runpy.run_path(str(script), run_name="__main__")
    except SystemExit as e:  # run_baseline ends with raise SystemExit(main())
        return int(e.code or 0)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
