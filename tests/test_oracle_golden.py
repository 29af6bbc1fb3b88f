"""CPU: the oracles reproduce the reference kernels' recorded outputs (tests/golden/*_ref_kernel.npz,
written by tests/golden/make_ref_golden.py from the reference's own CUDA kernels on a B200)."""
import os

import numpy as np
import pytest
import torch

from oracle import molmoact2_oracle as M
from oracle import pi05_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    path = os.path.join(GOLD, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not generated yet")
    return np.load(path)


def test_pi05_oracle_matches_reference_kernel_golden():
    from tests import ref_runner as R
    g = _load("pi05_ref_kernel.npz")
    c = O.make_case(**R.PI05_PIN)
    assert abs(c.noise.sum().item() - float(g["noise_sum"])) < 1e-3  # same seeded inputs
    mods, modf = O.modulations(c.w, c.L, c.num_steps)
    ora = O.denoise(R.pi05_dequantised_case(c), mods=mods, mod_final=modf)[0]
    ref = torch.from_numpy(g["actions"])
    assert (ora - ref).abs().max().item() < 5e-3


def test_molmoact2_oracle_matches_reference_kernel_golden():
    from tests import ref_runner as R
    g = _load("molmoact2_ref_kernel.npz")
    c = M.make_case(**R.MA2_PIN)
    assert abs(c.noise.sum().item() - float(g["noise_sum"])) < 1e-3
    ora = M.flow(R.ma2_bf16_case(c), weight_dtype=torch.bfloat16)[0]
    ref = torch.from_numpy(g["actions"])
    assert (ora[:, :c.adim] - ref[:, :c.adim]).abs().max().item() < 1.5e-2


def test_pi05_oracle_self_consistency():
    """Small structural checks of the restatement: zero-step loop is the identity; RoPE rotation
    preserves norms; the embedding is sin|cos."""
    c = O.make_case(seed=5, L=1, T=4, AD=8, Lp=16, B=1, num_steps=2)
    cos, sin = O.rope_tables(7, 4)
    x = torch.randn(4, 256)
    r = O._rope(x, cos, sin)
    assert torch.allclose(r.norm(dim=-1), x.norm(dim=-1), atol=1e-4)
    e = O.sinusoidal_embedding(torch.tensor([0.0]))
    assert torch.allclose(e[0, :512], torch.zeros(512)) and torch.allclose(e[0, 512:], torch.ones(512))
    out = O.denoise(c)
    assert out.shape == (1, 4, 8) and torch.isfinite(out).all()
