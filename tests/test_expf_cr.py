"""The fp32-only correctly rounded exp (torch_mcpu_b200/csrc/expf_cr.h).

The generator gen_expf_hard.cpp compares expf_cr with an extended-precision
exp for every fp32 input (about a minute on 8 cores; that full run produced
the committed hard-case table).  Here the same program checks a strided
sample of every 31st input (~1.4e8 values), plus sigmoid and silu of those
inputs, in a few seconds.  CPU only.
"""

import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "torch_mcpu_b200", "csrc")


def test_expf_cr_matches_correctly_rounded_exp_on_a_strided_sample():
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "gen")
        subprocess.run(["g++", "-O2", "-fopenmp", "-ffp-contract=off", "-std=c++17",
                        os.path.join(CSRC, "gen_expf_hard.cpp"), "-I", CSRC, "-o", exe], check=True)
        r = subprocess.run([exe, os.path.join(d, "unused.h"), "31"], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        assert "differing from the correctly rounded exp: 0" in r.stdout
        assert "mismatches over all fp32 inputs: 0" in r.stdout
