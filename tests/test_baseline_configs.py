"""GPU parity at the full BASELINE batch sizes, checked against the CPU fp32 oracle on a spread of
observations (the oracle runs one observation at a time, so only a few are recomputed).

  C2  pi0.5 bf16, bs=64 (full C1 geometry: 18 layers, T=50, prefix 968, 10 steps): the 64-observation
      plan the bench runs (128-token tiles in token groups, stepped-down K-splits, attention units on
      every CTA). Tolerance 2e-2 max-abs against the fp32 oracle on bf16-rounded prefix KV.
  C3  MolmoAct2 bf16, bs=32 (36 blocks, T=30, adim 6, context 493, 10 steps). Tolerance 2e-2 on the
      valid action dims; padded dims come back unchanged.
  C4  pi0.5 with FP8 / NVFP4 weights, prefix 1736, bs=16: against the unquantised fp32 reference,
      within the stated FP8 0.1 / NVFP4 0.3 max-abs tolerances.
"""
import pytest
import torch

from oracle import molmoact2_oracle as M
from oracle import pi05_oracle as O
from tests.pi05_util import err, oracle_bf16_kv, run_engine

TOL = 2e-2
pytestmark = pytest.mark.gpu


def _pi05_obs(c, sel):
    sub = O.Pi05Case(**{**c.__dict__})
    sub.B, sub.noise, sub.k, sub.v = len(sel), c.noise[sel], c.k[sel], c.v[sel]
    sub.valid_len = [c.valid_len[i] for i in sel]
    return sub


def test_c2_bs64_spread(require_gpu):
    c = O.make_case(seed=0, B=64)
    out, eng = run_engine(c)
    eng.close()
    assert torch.isfinite(out).all()
    sel = [0, 17, 42, 63]
    ref = oracle_bf16_kv(_pi05_obs(c, sel))
    for j, b in enumerate(sel):
        mx, cos = err(out[b], ref[j])
        print(f"C2 bs=64 observation {b}: max_abs={mx:.4g} cos={cos:.7f}")
        assert mx < TOL and cos > 0.999, (b, mx, cos)


def test_c3_ma2_bs32_spread(require_gpu):
    from tests.test_ma2_gpu import run
    c = M.make_case(seed=1, B=32)
    out, eng = run(c)
    assert torch.equal(out[..., c.adim:], c.noise[..., c.adim:])
    sel = [0, 13, 31]
    sub = M.Ma2Case(**{**c.__dict__})
    sub.B, sub.noise, sub.kctx, sub.vctx = len(sel), c.noise[sel], c.kctx[sel], c.vctx[sel]
    ref = M.flow(sub)
    for j, b in enumerate(sel):
        mx, cos = err(out[b, :, :c.adim], ref[j, :, :c.adim])
        print(f"C3 bs=32 observation {b}: max_abs={mx:.4g} cos={cos:.7f}")
        assert mx < TOL and cos > 0.999, (b, mx, cos)


@pytest.mark.parametrize("fmt,tol", [("fp8", 0.1), ("nvfp4", 0.3)])
def test_c4_bs16_quantised(require_gpu, fmt, tol):
    from tests.test_quant import _oracle, _run
    c = O.make_case(seed=7, L=18, T=50, AD=32, Lp=1736, B=16, num_steps=10)
    out, _ = _run(c, fmt)
    assert torch.isfinite(out).all()
    sel = [0, 9, 15]
    sub = _pi05_obs(c, sel)
    ref32 = _oracle(sub)
    ref16 = _oracle(sub, weight_dtype=torch.bfloat16)
    for j, b in enumerate(sel):
        mx32, cos32 = err(out[b], ref32[j])
        mx16, cos16 = err(out[b], ref16[j])
        print(f"C4 {fmt} bs=16 observation {b}: vs fp32 max_abs={mx32:.4g} cos={cos32:.6f}; "
              f"vs bf16 max_abs={mx16:.4g} cos={cos16:.6f}")
        assert mx32 < tol, (b, mx32, cos32)
