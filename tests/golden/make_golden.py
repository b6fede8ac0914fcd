#!/usr/bin/env python
"""Generate the golden fixtures in this directory from the reference itself.

Run once, on a machine that has the reference ``gpumode_qr`` source tree
(``--reference PATH``, the checkout's root directory); the fixtures are
committed and the tests never need the reference at run time.

Sources of truth:
* the reference's own Triton kernels, ``hh_fused_qr`` and ``hh_panel_qr``
  (``src/qrbench/triton_kernels.py:641-967``), and its blocked driver
  ``_hh_panel_blocked_qr`` (``src/qrbench/variants.py:761-805``), executed on
  the CPU by Triton's interpreter (``TRITON_INTERPRET=1``);
* the reference's oracle, CPU ``torch.geqrf`` (``src/qrbench/reference.py:18-20``);
* the reference's FP64 checker (``src/qrbench/checker.py:79-158``), whose gate
  values on the fixtures are stored for pinning this package's restatement.

Inputs are seeded CPU ``torch.randn`` draws (stored with the outputs).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root directory of the reference gpumode_qr checkout")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    sys.path.insert(0, str(REPO))

    import numpy as np
    import torch
    from qrbench import checker as ref_checker
    from qrbench import triton_kernels as tk
    from qrbench import variants as ref_variants

    from gpumode_qr_b200 import inputs as my_inputs

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    def randn(seed, *shape):
        return torch.randn(*shape, generator=torch.Generator().manual_seed(seed))

    # 1) reference fused kernel (n <= 128 in the reference)
    fused = {}
    cases = [(3, 1), (3, 2), (3, 3), (3, 5), (2, 8), (2, 16), (2, 31), (2, 32), (2, 33), (2, 48), (2, 64)]
    for idx, (b, n) in enumerate(cases):
        A = randn(100 + idx, b, n, n)
        H, tau = tk.hh_fused_qr(A)
        fused[f"n{n}_A"] = A.numpy()
        fused[f"n{n}_H"] = H.numpy()
        fused[f"n{n}_tau"] = tau.numpy()
    # structured small cases
    structured = {}
    z = torch.zeros(2, 8, 8)
    structured["zeros"] = z
    zc = randn(7, 2, 8, 8)
    zc[:, :, 3] = 0.0
    structured["zero_col"] = zc
    structured["upper_tri"] = torch.triu(randn(8, 2, 16, 16))
    u, v = randn(9, 2, 16, 4), randn(10, 2, 4, 16)
    structured["rank4"] = u @ v
    ident = torch.eye(12).expand(2, 12, 12).clone()
    structured["identity"] = ident
    for name, A in structured.items():
        H, tau = tk.hh_fused_qr(A)
        fused[f"{name}_A"] = A.numpy()
        fused[f"{name}_H"] = H.numpy()
        fused[f"{name}_tau"] = tau.numpy()
    np.savez_compressed(HERE / "ref_fused.npz", **fused)

    # 2) reference panel kernel
    panel = {}
    for idx, (b, r, w) in enumerate([(2, 8, 8), (2, 40, 8), (2, 64, 32), (2, 100, 16), (2, 130, 32), (2, 33, 32)]):
        P = randn(200 + idx, b, r, w)
        H, V, tau, T = tk.hh_panel_qr(P)
        key = f"r{r}_w{w}"
        panel[f"{key}_P"] = P.numpy()
        panel[f"{key}_H"] = H.numpy()
        panel[f"{key}_V"] = V.numpy()
        panel[f"{key}_tau"] = tau.numpy()
        panel[f"{key}_T"] = T.numpy()
    np.savez_compressed(HERE / "ref_panel.npz", **panel)

    # 3) reference blocked driver and champion dispatch
    blocked = {}
    for idx, (b, n, w) in enumerate([(2, 48, 32), (2, 100, 32), (1, 176, 32), (2, 70, 16)]):
        A = randn(300 + idx, b, n, n)
        H, tau = ref_variants._hh_panel_blocked_qr(A, w, False)
        key = f"n{n}_w{w}"
        blocked[f"{key}_A"] = A.numpy()
        blocked[f"{key}_H"] = H.numpy()
        blocked[f"{key}_tau"] = tau.numpy()
    champ = ref_variants.VARIANTS[ref_variants.CHAMPION]
    for idx, (b, n) in enumerate([(2, 64), (1, 160)]):
        A = randn(400 + idx, b, n, n)
        H, tau = champ(A)
        blocked[f"champion_n{n}_A"] = A.numpy()
        blocked[f"champion_n{n}_H"] = H.numpy()
        blocked[f"champion_n{n}_tau"] = tau.numpy()
    np.savez_compressed(HERE / "ref_blocked.npz", **blocked)

    # 4) reference oracle (CPU torch.geqrf) on config 1 and stress cases at n=32
    lap = {}
    A1 = my_inputs.make_config_input(my_inputs.config(1))
    H1, t1 = torch.geqrf(A1)
    lap["cfg1_A"], lap["cfg1_H"], lap["cfg1_tau"] = A1.numpy(), H1.numpy(), t1.numpy()
    for prob in my_inputs.stress_cases(32, batch=2):
        H, tau = torch.geqrf(prob.tensor)
        lap[f"{prob.name}_A"] = prob.tensor.numpy()
        lap[f"{prob.name}_H"] = H.numpy()
        lap[f"{prob.name}_tau"] = tau.numpy()
    np.savez_compressed(HERE / "lapack.npz", **lap)

    # 5) reference checker values on fixtures (pins the gate restatement)
    chk = {}

    def record(name, A, H, tau):
        chk[name] = ref_checker.check(A, H, tau).as_dict()

    record("cfg1_geqrf", A1, H1, t1)
    Hbad = H1.clone()
    Hbad[:, 5, 2] += 1e-2  # perturbed reflector entry: must fail the gates
    record("cfg1_perturbed", A1, Hbad, t1)
    record("fused_n33", torch.from_numpy(fused["n33_A"]), torch.from_numpy(fused["n33_H"]),
           torch.from_numpy(fused["n33_tau"]))
    record("blocked_n100", torch.from_numpy(blocked["n100_w32_A"]), torch.from_numpy(blocked["n100_w32_H"]),
           torch.from_numpy(blocked["n100_w32_tau"]))
    (HERE / "ref_checker.json").write_text(json.dumps(chk, indent=1, sort_keys=True))

    # 6) input-generator checksums
    sums = {}
    for cfg in my_inputs.CONFIGS:
        b = cfg.batch if cfg.kind == "iid" else 2
        A = my_inputs.make_config_input(cfg, batch=b).double()
        sums[cfg.name] = {
            "batch": b,
            "sum": A.sum().item(),
            "sumsq": (A * A).sum().item(),
            "first": A.reshape(-1)[:4].tolist(),
        }
    (HERE / "input_checksums.json").write_text(json.dumps(sums, indent=1, sort_keys=True))
    print("wrote fixtures to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
