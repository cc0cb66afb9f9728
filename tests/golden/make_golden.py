"""Extract the reference's known-answer data for the GDN-2 recurrence into small fixtures.

Source (read-only reference checkout, Akseleu-J/atomic-ops):
  numerical/experiments/2026-10-17/controlled-rounding/inputs-seed{0,1,2}.npz
  numerical/experiments/2026-10-17/controlled-rounding/report.json

The reference's experiment (artifacts/current-evidence/...rounding-hypothesis...zip:
executed-source/rounding_adam_hypothesis.py, functions decimal_run / decimal_objective)
evaluates, with Python Decimal at 80 (and 110) significant digits, the token recurrence
    h <- exp(g_t) h ;  v_new = w_t (v_t + theta d_t) - (b_t k_t)^T h ;  h <- h + k_t v_new^T ;
    o_t = 0.5 h^T q_t
on (B=1, L=256, H=1, D=4) float32 inputs, y = concat(o.ravel(), h_final.ravel()) and
  natural:             value = sum(y^2)/2
  cancellation_stress: value = sum(coeff * y)
and the derivative of value w.r.t. theta at theta = 0 (a directional derivative along
`direction` applied to v).  These Decimal numbers are the golden values; no other stored
operator outputs exist in the reference (KNOWN_LIMITATIONS.md:59).

Run from the repository root:  python tests/golden/make_golden.py <reference_root>
"""
from __future__ import annotations

import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REL = "numerical/experiments/2026-10-17/controlled-rounding"


def main(ref_root: str) -> None:
    src = pathlib.Path(ref_root) / REL
    report = json.loads((src / "report.json").read_text())
    arrays = {}
    for seed in (0, 1, 2):
        with np.load(src / f"inputs-seed{seed}.npz") as z:
            for name in z.files:
                arrays[f"seed{seed}_{name}"] = z[name]
    np.savez_compressed(HERE / "known_answer.npz", **arrays)
    cases = []
    for c in report["cases"]:
        cases.append({
            "seed": c["seed"],
            "mode": c["mode"],
            "input_sha256": c["input_sha256"],
            "value_decimal": c["oracle_value_decimal"],
            "gradient_decimal": c["oracle_gradient_decimal"],
            "fp64_results": {r["algorithm"]: {"objective": r["objective"], "gradient": r["gradient"]}
                             for r in c["results"] if r["dtype"] == "fp64"},
        })
    meta = {
        "source": f"{REL}/report.json (+ inputs-seed*.npz)",
        "shape": report["shape"],
        "decimal_precision": report["decimal_precision"],
        "output_scale": 0.5,
        "objective": "y = concat(o.ravel(), h_final.ravel()); natural: sum(y^2)/2; "
                     "cancellation_stress: sum(coeff*y); gradient = d/dtheta at v + theta*direction",
        "cases": cases,
    }
    (HERE / "known_answer.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {HERE / 'known_answer.npz'} and {HERE / 'known_answer.json'} ({len(cases)} cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <root of the reference checkout>")
    main(sys.argv[1])
