"""Run one small case of a library path, for a profiler capture.

    python -m gpumode_qr_b200.profile_case geqrf B N [--repeat R] [--set KEY=VALUE ...]
    python -m gpumode_qr_b200.profile_case gram B N K [--repeat R]
    python -m gpumode_qr_b200.profile_case gram_geqrf B N K [--repeat R]

The input is drawn from a seeded CPU generator (standard normal), copied to
``cuda:0`` and passed ``R`` times (default 2) to the named entry point, so that a
capture can skip the first (cold) launch with ``ncu -s``. ``--set`` applies
``qrb_set_config`` keys before the calls (for example ``two_level=1``). Prints
one line with the output shape and the number of library kernel launches.
"""

from __future__ import annotations

import argparse
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("path", choices=["geqrf", "gram", "gram_geqrf"])
    ap.add_argument("dims", type=int, nargs="+", help="B N for geqrf; B N K for the Gram paths")
    ap.add_argument("--repeat", type=int, default=2)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--set", action="append", default=[], metavar="KEY=VALUE")
    args = ap.parse_args(argv)

    import torch

    from . import _lib, api

    if not torch.cuda.is_available():
        print("profile_case: a CUDA device is required", file=sys.stderr)
        return 2
    need = 2 if args.path == "geqrf" else 3
    if len(args.dims) != need:
        ap.error(f"{args.path} takes {need} sizes")
    for kv in args.set:
        key, _, val = kv.partition("=")
        _lib.set_config(key, int(val))
    g = torch.Generator().manual_seed(args.seed)
    if args.path == "geqrf":
        b, n = args.dims
        x = torch.randn(b, n, n, generator=g).cuda()
        fn = api.geqrf
    else:
        b, n, k = args.dims
        x = torch.randn(b, n, k, generator=g).cuda()
        fn = api.gram if args.path == "gram" else api.gram_geqrf
    _lib.set_config("launches", 0)
    out = None
    for _ in range(args.repeat):
        out = fn(x)
    torch.cuda.synchronize()
    first = out[0] if isinstance(out, tuple) else out
    print(f"ok {args.path} {tuple(first.shape)} launches={_lib.get_config('launches')}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
