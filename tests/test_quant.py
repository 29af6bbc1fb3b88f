"""Quantised pi0.5 weights (FP8 per-row E4M3, NVFP4 E2M1 with E4M3 block scales).

CPU: the quantisers in oracle/quant.py round-trip within the formats' resolution.
GPU: the engine loaded through fa_pi05_load_weights_q (FP8: the FP8-streaming kernel; NVFP4:
dequantised at load) must match the fp32 oracle run on the DEQUANTISED weights at the bf16 bar
(max-abs 2e-2); the quantisation error itself (against the
unquantised fp32 and bf16 references) is measured on BASELINE config C4 (prefix 1736, bs=1) and
bounded by the stated tolerances below (FP8 0.1, NVFP4 0.3 max-abs on the action chunk)."""
import pytest
import torch

from oracle import pi05_oracle as O
from oracle import quant as Q
from tests.pi05_util import err

GEMM = ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"]
TOL_FP8_VS_FP32 = 0.1
TOL_NVFP4_VS_FP32 = 0.3


def test_fp8_roundtrip_cpu():
    w = torch.randn(2, 64, 256, generator=torch.Generator().manual_seed(1)) * 0.02
    c, s = Q.fp8_rowwise(w)
    d = Q.fp8_dequant(c, s)
    # E4M3 has 3 mantissa bits: relative rounding error <= 2^-4 of each value (plus subnormals)
    assert ((d - w).abs() <= w.abs() * 2 ** -4 + s[..., None] * 2 ** -9).all()
    assert (d.abs().amax(-1) - w.abs().amax(-1)).abs().max() < 1e-6  # row max is representable


def test_nvfp4_roundtrip_cpu():
    w = torch.randn(2, 32, 128, generator=torch.Generator().manual_seed(2)) * 0.02
    p, bs, ts = Q.nvfp4(w)
    assert p.shape == (2, 32, 64) and bs.shape == (2, 32, 8) and ts.shape == (2,)
    d = Q.nvfp4_dequant(p, bs, ts)
    scale = (bs.view(torch.float8_e4m3fn).float() * ts[:, None, None]).repeat_interleave(16, -1)
    # E2M1 spacing is at most 2 (between 4 and 6) in units of the block scale; nearest rounding
    assert ((d - w).abs() <= scale * 1.0 + 1e-7).all()
    assert (d / scale.clamp(min=1e-30)).abs().max() <= 6.0 + 1e-5


def _quantise(case, fmt):
    w = dict(case.w)
    qs, deq = {}, {}
    for n in GEMM:
        if fmt == "fp8":
            c, s = Q.fp8_rowwise(case.w[n])
            w[n], qs[n], deq[n] = c, s, Q.fp8_dequant(c, s)
        else:
            p, bs, ts = Q.nvfp4(case.w[n])
            w[n], qs[n], deq[n] = p, (bs, ts), Q.nvfp4_dequant(p, bs, ts)
    return w, qs, deq


def _run(case, fmt):
    from flashact_b200 import Pi05ActionExpert
    w, qs, deq = _quantise(case, fmt)
    eng = Pi05ActionExpert(w, num_layers=case.L, horizon=case.T, action_dim=case.AD, max_prefix=case.Lp,
                           max_batch=case.B, num_steps=case.num_steps, wfmt=fmt, qscales=qs)
    eng.bind_prefix_kv(case.k.to(torch.bfloat16).cuda(), case.v.to(torch.bfloat16).cuda(), case.valid_len)
    out = eng.sample_actions(case.noise.cuda()).cpu()
    eng.close()
    return out, deq


def _oracle(case, weights=None, weight_dtype=torch.float32):
    c2 = O.Pi05Case(**{**case.__dict__})
    c2.w = {**case.w, **(weights or {})}
    c2.k, c2.v = case.k.to(torch.bfloat16).float(), case.v.to(torch.bfloat16).float()
    return O.denoise(c2, weight_dtype=weight_dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
def test_quantised_engine_matches_dequantised_oracle(require_gpu, fmt):
    c = O.make_case(seed=61, L=2, T=50, AD=32, Lp=300, B=1, num_steps=3)
    out, deq = _run(c, fmt)
    mx, cos = err(out, _oracle(c, deq))
    print(f"{fmt} engine vs fp32 oracle on the dequantised weights: max_abs={mx:.4g} cos={cos:.7f}")
    assert mx < 2e-2 and cos > 0.9999, (mx, cos)


@pytest.mark.gpu
def test_c4_quantisation_error(require_gpu):
    """prefix 1736 (6 x 256 image + 200 text), bs=1, 10 steps; the FP8 and
    NVFP4 action chunks against the unquantised fp32 and bf16 references."""
    c = O.make_case(seed=7, L=18, T=50, AD=32, Lp=1736, B=1, num_steps=10)
    ref32 = _oracle(c)
    ref16 = _oracle(c, weight_dtype=torch.bfloat16)
    res = {}
    for fmt in ("fp8", "nvfp4"):
        out, _ = _run(c, fmt)
        res[fmt] = (err(out, ref32), err(out, ref16))
        print(f"C4 {fmt}: vs fp32 max_abs={res[fmt][0][0]:.4g} cos={res[fmt][0][1]:.6f}; "
              f"vs bf16 max_abs={res[fmt][1][0]:.4g} cos={res[fmt][1][1]:.6f}")
    assert res["fp8"][0][0] < TOL_FP8_VS_FP32
    assert res["nvfp4"][0][0] < TOL_NVFP4_VS_FP32


def _edge_weights(dtype):
    """Two layers [2][48][256]: random rows, an all-zero row, a zero block, and (layer 1, whose
    amax is 2688 so its tensor scale is exactly 1) a block of 6 with the E2M1 midpoints, signs and
    negative zero, a block that saturates the E4M3 block scale at 448 and a tiny block whose
    block scale underflows to 0."""
    g = torch.Generator().manual_seed(5)
    w = torch.randn(2, 48, 256, generator=g) * 0.02
    w[0, 3] = 0.0
    w[0, 5, 32:48] = 0.0
    w[1] = torch.randn(48, 256, generator=g) * 0.5
    w[1, 0, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -2.5, -5.0, 0.0, -0.0,
                                 0.5, -6.0])
    w[1, 1, :16] = 2688.0
    w[1, 2, :16] = 1e-4
    return w.to(dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_device_fp8_quantiser_bit_exact(require_gpu, dtype):
    from flashact_b200.quant import quantize_fp8_rows
    w = _edge_weights(dtype)
    codes, scale = quantize_fp8_rows(w.cuda())
    rc, rs = Q.fp8_rowwise(w.float())
    assert torch.equal(scale.cpu(), rs)
    assert torch.equal(codes.cpu(), rc)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_device_nvfp4_quantiser_bit_exact(require_gpu, dtype):
    from flashact_b200.quant import quantize_nvfp4
    w = _edge_weights(dtype)
    packed, bs, ts = quantize_nvfp4(w.cuda())
    rp, rbs, rts = Q.nvfp4(w.float())
    assert rts[1].item() == 1.0 and rbs[1, 1, 0].item() == torch.tensor(448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(ts.cpu(), rts)
    assert torch.equal(bs.cpu(), rbs)
    assert torch.equal(packed.cpu(), rp)


@pytest.mark.gpu
def test_device_quantised_weights_load(require_gpu):
    """Codes from the device quantisers drive fa_pi05_load_weights_q like the host ones."""
    from flashact_b200 import Pi05ActionExpert
    from flashact_b200.quant import quantize_fp8_rows
    c = O.make_case(seed=62, L=2, T=50, AD=32, Lp=300, B=1, num_steps=3)
    w = dict(c.w)
    qs, deq = {}, {}
    for n in GEMM:
        codes, s = quantize_fp8_rows(c.w[n].cuda())
        w[n], qs[n], deq[n] = codes, s, Q.fp8_dequant(codes.cpu(), s.cpu())
    eng = Pi05ActionExpert(w, num_layers=c.L, horizon=c.T, action_dim=c.AD, max_prefix=c.Lp, max_batch=c.B,
                           num_steps=c.num_steps, wfmt="fp8", qscales=qs)
    eng.bind_prefix_kv(c.k.to(torch.bfloat16).cuda(), c.v.to(torch.bfloat16).cuda(), c.valid_len)
    out = eng.sample_actions(c.noise.cuda()).cpu()
    eng.close()
    mx, cos = err(out, _oracle(c, deq))
    assert mx < 2e-2 and cos > 0.9999, (mx, cos)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 3, 12])
def test_fp8_stream_matches_dequantised_path(require_gpu, monkeypatch, B):
    """The FP8-streaming kernel (E4M3 tiles expanded into tensor memory, row scales in the epilogue)
    against the same codes dequantised at load into the bf16 kernel (FA_FP8_STREAM=0) and against
    the fp32 oracle: 64-row units at bs=1, 128-row units over two token tiles at bs=3."""
    c = O.make_case(seed=63, L=2, T=50, AD=32, Lp=300, B=B, num_steps=2)
    out_s, deq = _run(c, "fp8")
    monkeypatch.setenv("FA_FP8_STREAM", "0")
    out_d, _ = _run(c, "fp8")
    ref = _oracle(c, deq)
    for name, out in (("stream", out_s), ("dequant", out_d)):
        mx, cos = err(out, ref)
        print(f"B={B} fp8 {name}: max_abs={mx:.4g} cos={cos:.7f}")
        assert mx < 2e-2 and cos > 0.9999, (name, mx, cos)
    assert not torch.equal(out_s, out_d)  # two kernels (scale before vs after the MMAs)
    assert (out_s - out_d).abs().max() < 2e-2
