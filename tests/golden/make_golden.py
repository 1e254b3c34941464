"""Regenerates the golden fixtures in this folder from the reference itself.

CPU (where the reference source tree exists and oracle/_ref has been built from it):
    python tests/golden/make_golden.py rng
  compiles nothing itself; needs oracle/_ref/ref_harness (`make -C oracle ref`), which is the reference's
  own src/sffft.cu built in place, and records the first draws of its nrand() for three seeds.

GPU box (the harness binary travels with the repository):
    python tests/golden/make_golden.py results [OUT_DIR]
  runs the unmodified reference benchmark (ref_harness run ...) and records its RESULT/SELECT rows on B200.
"""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")
SEEDS = [0, 42, 12345]
COUNT = 64


def rng():
    out = {}
    for seed in SEEDS:
        txt = subprocess.run([HARNESS, "rng", str(seed), str(COUNT)], check=True, capture_output=True, text=True).stdout
        out[str(seed)] = [float(v) for v in txt.split()]
    with open(os.path.join(HERE, "ref_rng.json"), "w") as f:
        json.dump({"source": "reference nrand() (src/sffft.cu:308-310) built from source by oracle/ref_harness.cu",
                   "seed_0_means": "default state 88172645463325252", "draws": out}, f, indent=1)


RUNS = [
    ["1", "1", "--max-error", "1e-3", "--io", "fp32", "--kernel", "auto"],
    ["8", "768", "1024", "--kernel", "cached"],
    ["1", "1", "128", "--max-error", "1e-3", "--io", "fp32", "--input-scale", "15000"],
]


def results(out_dir=HERE):
    rows = []
    for args in RUNS:
        p = subprocess.run([HARNESS, "run"] + args, capture_output=True, text=True, timeout=1200)
        rows.append({"args": args, "exit": p.returncode, "stdout": p.stdout})
    with open(os.path.join(out_dir, "ref_results_b200.json"), "w") as f:
        json.dump({"source": "unmodified reference benchmark (src/sffft.cu main) built for sm_100a, run on B200",
                   "runs": rows}, f, indent=1)


if __name__ == "__main__":
    if sys.argv[1] == "rng":
        rng()
    else:
        results(sys.argv[2] if len(sys.argv) > 2 else HERE)
