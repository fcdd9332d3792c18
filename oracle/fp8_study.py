"""FP8 accuracy study (an FP8 GEMM variant only with an
accuracy study, since the parity tolerance is defined against bf16 numerics).

TEST INFRASTRUCTURE / STUDY ONLY: nothing in the product imports this file.

It runs the reference's unmodified driver with the CPU restatement of its back
end (oracle/_ref/tessera_encode_ref) on the golden case tiles, with the
restatement's Linears fed e4m3 operands (TC_ORACLE_FP8=ffn: FFN1 and FFN2;
=all: every Linear), weights scaled per output channel and activations per
row by max|v| / 448, as an FP8 tensor-core GEMM with those scales would see
them. Each result is compared with the bf16 golden output (the reference's
arithmetic) under the acceptance metrics of the parity tests.

    python oracle/fp8_study.py            # prints one JSON line per (case, mode)
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
sys.path[:0] = [str(HERE), str(REPO / "tessera-inference_b200"), str(REPO / "tests")]

import oracle  # noqa: E402
import synth  # noqa: E402
from golden.make_golden import CASES, case_tile, case_weights  # noqa: E402


def acceptance(m: dict) -> bool:
    return (m["within1"] >= 0.999 and m["scale_rel_p99"] <= 1e-2 and m["scale_rel_max"] <= 2.0 ** -6
            and m["zero_rows_match"] and m["empty_scale_exact"])


def main() -> int:
    binary = HERE / "_ref" / "tessera_encode_ref"
    if not binary.exists():
        sys.exit("build the reference driver first: make -C oracle")
    with tempfile.TemporaryDirectory() as td:
        for case in CASES:
            g = np.load(REPO / "tests" / "golden" / f"{case}_oracle.npz")
            tdir = synth.write_tile_dir(case_tile(case), Path(td) / f"grid_{case}")
            w = case_weights(case, Path(td))
            for mode in ("ffn", "all"):
                out = Path(td) / f"out_{mode}"
                env = dict(os.environ, TC_ORACLE_FP8=mode)
                subprocess.run([str(binary), str(tdir), str(out), str(w)], check=True, env=env, capture_output=True)
                codes = np.load(out / f"grid_{case}.npy")
                scales = np.load(out / f"grid_{case}_scales.npy")
                m = oracle.compare(g["codes"], g["scales"], codes, scales)
                rec = {"case": case, "fp8": mode, "meets_acceptance": acceptance(m)}
                rec.update({k: m[k] for k in ("exact", "within1", "off2plus", "max", "cos_mean", "cos_min",
                                              "scale_rel_p99", "scale_rel_max")})
                print(json.dumps(rec), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
