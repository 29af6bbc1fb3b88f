"""On-device FP8 / NVFP4 weight quantisation (fa_quantize_fp8_rows / fa_quantize_nvfp4 in
include/flashact.h): the codes and scales Pi05ActionExpert(wfmt="fp8" | "nvfp4") takes, computed
on the GPU from bf16 / fp16 / fp32 weights. The reference quantises on the host inside
HybridPi05._pack_weights (src/pi05/hybrid_model.py:105-110). No CPU fallback."""
from __future__ import annotations

import ctypes

import torch

from . import _capi as C
from .pi05 import _DT, _stream_ptr


def _prep(w: torch.Tensor):
    if not w.is_cuda:
        raise C.FlashActError(C.FA_ERR_INVALID, "the weights must be a CUDA tensor")
    if w.dtype not in _DT:
        w = w.float()
    w = w.contiguous()
    w3 = w.view(-1, w.shape[-2], w.shape[-1]) if w.dim() >= 2 else w.view(1, 1, -1)
    return w, w3.shape


def _check(lib, st):
    if st != C.FA_OK:
        raise C.FlashActError(st, lib.fa_last_error(None).decode(errors="replace"))


def quantize_fp8_rows(w: torch.Tensor):
    """w [..., rows, K] -> (codes uint8 [..., rows, K], scale fp32 [..., rows]); per-row E4M3
    with scale max(amax, 1e-8) / 448."""
    lib = C.load_library()
    w, (L, R, K) = _prep(w)
    with torch.cuda.device(w.device):
        codes = torch.empty(w.shape, dtype=torch.uint8, device=w.device)
        scale = torch.empty(w.shape[:-1], dtype=torch.float32, device=w.device)
        _check(lib, lib.fa_quantize_fp8_rows(ctypes.c_void_p(w.data_ptr()), _DT[w.dtype], L, R, K,
                                             ctypes.c_void_p(codes.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
                                             _stream_ptr()))
    return codes, scale


def quantize_nvfp4(w: torch.Tensor):
    """w [L, rows, K] (K % 16 == 0) -> (packed E2M1 codes uint8 [L, rows, K/2], E4M3 block scales
    as uint8 [L, rows, K/16], fp32 tensor scale [L])."""
    lib = C.load_library()
    if w.dim() != 3:
        raise C.FlashActError(C.FA_ERR_INVALID, "nvfp4 quantisation takes [L, rows, K]")
    w, (L, R, K) = _prep(w)
    with torch.cuda.device(w.device):
        packed = torch.empty(L, R, K // 2, dtype=torch.uint8, device=w.device)
        bscale = torch.empty(L, R, K // 16, dtype=torch.uint8, device=w.device)
        tscale = torch.empty(L, dtype=torch.float32, device=w.device)
        _check(lib, lib.fa_quantize_nvfp4(ctypes.c_void_p(w.data_ptr()), _DT[w.dtype], L, R, K,
                                          ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(bscale.data_ptr()),
                                          ctypes.c_void_p(tscale.data_ptr()), _stream_ptr()))
    return packed, bscale, tscale
