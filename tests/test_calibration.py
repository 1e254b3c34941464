"""The built-in default plan per length comes from the committed B200 calibration (sffft_b200/csrc/
calibration_b200.csv, made by `python -m sffft_b200.calibrate`): calibration.h must be what make_calibration.py
writes from it, and sffft_default_config must return its plan for every length."""
import os
import subprocess
import sys

import sffft_b200 as sf

CSRC = os.path.join(os.path.dirname(sf.__file__), "csrc")


def test_header_is_generated_from_the_committed_calibration():
    out = subprocess.run([sys.executable, os.path.join(CSRC, "make_calibration.py"),
                          os.path.join(CSRC, "calibration_b200.csv")], capture_output=True, text=True, check=True).stdout
    assert out == open(os.path.join(CSRC, "calibration.h")).read()


def calibrated():
    rows = {}
    for line in open(os.path.join(CSRC, "calibration.h")):
        line = line.strip()
        if line.startswith("{") and '"' in line:
            f = line.strip("{},").split(", ")
            rows[int(f[0])] = f[5].strip('"')
    return rows


def test_default_config_follows_the_calibration():
    rows = calibrated()
    assert sorted(rows) == [128 << i for i in range(8)]
    for L, name in rows.items():
        assert sf.default_config(L) == name


def test_calibration_covers_every_catalog_plan_and_both_io_types():
    seen = set()
    for line in open(os.path.join(CSRC, "calibration_b200.csv")):
        f = line.strip().split(",")
        if f[0] == "CAL":
            seen.add((int(f[1]), f[2], f[3]))
    for L, name in sf.catalog():
        assert (L, name, "fp32") in seen and (L, name, "bf16") in seen
