"""Writes the reference kernels' outputs on the pin cases as golden fixtures (run on a GPU box,
with oracle/_ref built from the reference sources):

    python tests/golden/make_ref_golden.py

pi05_ref_kernel.npz / molmoact2_ref_kernel.npz hold the action chunks the reference's own
megakernels (src/pi05/mk6.cu, src/molmoact2/mk_ma2.cu) produce on the seeded inputs of
tests/ref_runner.py (PI05_PIN, MA2_PIN). tests/test_oracle_golden.py checks the CPU oracles
against them without a GPU."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import molmoact2_oracle as M  # noqa: E402
from oracle import pi05_oracle as O  # noqa: E402
from tests import ref_runner as R  # noqa: E402

if __name__ == "__main__":
    c = O.make_case(**R.PI05_PIN)
    out = R.run_pi05_ref(R.load("mk_v6_ref"), c)
    np.savez(os.path.join(HERE, "pi05_ref_kernel.npz"), actions=out.numpy(), noise_sum=c.noise.sum().item(),
             **{k: v for k, v in R.PI05_PIN.items()})
    c = M.make_case(**R.MA2_PIN)
    out = R.run_ma2_ref(R.load("mk_ma2_ref"), c)
    np.savez(os.path.join(HERE, "molmoact2_ref_kernel.npz"), actions=out.numpy(), noise_sum=c.noise.sum().item(),
             **{k: v for k, v in R.MA2_PIN.items()})
    print("written")
