"""Weight quantisers for the FP8 / NVFP4 parity tests -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py may import this module.

  * FP8: per-output-row E4M3 with scale amax/448, values clamped to +-448, round to nearest
    (the reference's scheme, src/pi05/hybrid_model.py:105-110).
  * NVFP4: E2M1 codes (0, 0.5, 1, 1.5, 2, 3, 4, 6 and negatives) with one E4M3 scale per 16
    consecutive inputs of a row and one fp32 scale per layer matrix (the published NVFP4 block
    format): tensor scale = amax / (448 * 6), block scale = E4M3(block amax / 6 / tensor scale),
    code = nearest E2M1 value of x / (block scale * tensor scale) (ties to the even code).
The matching dequantisers give the exact values the engine computes with.
"""
from __future__ import annotations

import torch

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def fp8_rowwise(w: torch.Tensor):
    """w [..., rows, K] -> (codes uint8 [..., rows, K], scale fp32 [..., rows])."""
    s = w.float().abs().amax(dim=-1).clamp(min=1e-8) / 448.0
    q = (w.float() / s[..., None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), s.float()


def fp8_dequant(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return codes.view(torch.float8_e4m3fn).float() * scale[..., None]


def nvfp4(w: torch.Tensor):
    """w [L, rows, K] (K % 16 == 0) -> (packed codes uint8 [L, rows, K/2], block scales E4M3 as
    uint8 [L, rows, K/16], tensor scale fp32 [L])."""
    w = w.float()
    L, R, K = w.shape
    ts = (w.abs().amax(dim=(1, 2)) / (448.0 * 6.0)).clamp(min=1e-12)  # [L]
    blk = w.view(L, R, K // 16, 16)
    bs = (blk.abs().amax(-1) / 6.0 / ts[:, None, None]).clamp(max=448.0).to(torch.float8_e4m3fn)  # [L,R,K/16]
    scale = bs.float() * ts[:, None, None]
    x = blk / torch.where(scale > 0, scale, torch.ones_like(scale))[..., None]
    mag = x.abs().clamp(max=6.0)
    # nearest E2M1 magnitude, ties to the even code (the one with mantissa bit 0)
    d = (mag[..., None] - _E2M1).abs()
    idx = d.argmin(-1)
    tie = (d - d.min(-1, keepdim=True).values).abs() < 1e-12
    even = tie & (torch.arange(8) % 2 == 0)
    idx = torch.where(tie.sum(-1) > 1, even.float().argmax(-1), idx)
    code = idx | ((x < 0) & (idx > 0)).to(torch.int64) << 3
    code = code.view(L, R, K).to(torch.uint8)
    packed = code[..., 0::2] | (code[..., 1::2] << 4)
    return packed.contiguous(), bs.view(torch.uint8).contiguous(), ts.float()


def nvfp4_dequant(packed: torch.Tensor, bscale: torch.Tensor, tscale: torch.Tensor) -> torch.Tensor:
    L, R, K2 = packed.shape
    lo, hi = packed & 15, packed >> 4
    code = torch.stack([lo, hi], -1).view(L, R, 2 * K2).long()
    mag = _E2M1[code & 7]
    val = torch.where(code >= 8, -mag, mag)
    bs = bscale.view(torch.float8_e4m3fn).float().repeat_interleave(16, -1)
    return val * bs * tscale[:, None, None]
