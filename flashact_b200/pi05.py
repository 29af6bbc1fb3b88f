"""pi0.5 action-expert denoise engine: Python host mirror of the reference's deployment path.

The reference's caller (src/pi05/hybrid_model.py: HybridPi05._pack_weights :76-133, the KV
handoff + launch in predict :188-222) maps onto three calls here: construct (weight load +
on-device conditioning), bind_prefix_kv, sample_actions. Everything runs through the C ABI of
libflashact.so; torch is only used to hold device memory and name the current stream. There is
no CPU fallback: without the library or an sm_100 GPU the constructor raises.
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi as C

_DT = {torch.float32: C.FA_DT_F32, torch.bfloat16: C.FA_DT_BF16, torch.float16: C.FA_DT_F16}


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class Pi05ActionExpert:
    """Owns one fa_handle on one device. Weights: dict with the keys of
    flashact_b200._capi.PI05_WEIGHT_FIELDS, [out][in] row-major, stacked over layers."""

    def __init__(self, weights: dict, *, num_layers=18, horizon=50, action_dim=32, max_prefix=968, max_batch=1,
                 num_steps=10, device: int = 0, mods=None, mod_final=None, wfmt: str = "bf16", qscales=None):
        """wfmt "fp8" / "nvfp4": the seven GEMM weights are codes (uint8) and qscales maps each of
        them to its scales -- fp8: per-row fp32 [L][rows]; nvfp4: (E4M3 block scales as uint8
        [L][rows][K/16], fp32 per-layer scale [L]) -- see fa_qscale in include/flashact.h."""
        self.lib = C.load_library()
        self.device = device
        self.cfg = C.FaConfig(num_layers, 1024, 8, 1, 256, 4096, horizon, action_dim, max_prefix, max_batch,
                              num_steps, 0)
        self.horizon, self.action_dim, self.max_batch = horizon, action_dim, max_batch
        h = ctypes.c_void_p()
        st = self.lib.fa_create(C.FA_MODEL_PI05, ctypes.byref(self.cfg), device, ctypes.byref(h))
        C.check(self.lib, None, st)
        self.h = h
        self._kv_keep = None
        self.batch = 0
        keep = []
        w = C.FaPi05Weights()
        for name in C.PI05_WEIGHT_FIELDS:
            t = weights.get(name)
            if t is None:  # conditioning weights left out: modulations are passed in (mods, mod_final)
                setattr(w, name, C.FaTensor(None, C.FA_DT_F32))
                continue
            quantised = wfmt != "bf16" and name in C.PI05_QUANT_FIELDS
            if t.dtype not in _DT and not quantised:
                t = t.float()
            t = t.contiguous()
            keep.append(t)
            setattr(w, name, C.FaTensor(t.data_ptr(), _DT.get(t.dtype, C.FA_DT_F32)))
        if wfmt == "bf16":
            self._check(self.lib.fa_pi05_load_weights(self.h, ctypes.byref(w), C.FA_WFMT_BF16))
        else:
            qs = C.FaPi05QScales()
            for name in C.PI05_QUANT_FIELDS:
                sc = qscales[name]
                blk, ten = (sc if isinstance(sc, (tuple, list)) else (sc, None))
                blk = blk.contiguous()
                keep.append(blk)
                tp = None
                if ten is not None:
                    ten = ten.float().contiguous()
                    keep.append(ten)
                    tp = ten.data_ptr()
                setattr(qs, name, C.FaQScale(blk.data_ptr(), tp))
            fmt = {"fp8": C.FA_WFMT_FP8, "nvfp4": C.FA_WFMT_NVFP4}[wfmt]
            self._check(self.lib.fa_pi05_load_weights_q(self.h, ctypes.byref(w), fmt, ctypes.byref(qs)))
        if mods is not None:
            m = mods.float().contiguous()
            mf = mod_final.float().contiguous()
            self._check(self.lib.fa_set_modulation(self.h, m.data_ptr(), mf.data_ptr()))

    def _check(self, st):
        C.check(self.lib, self.h, st)

    def bind_prefix_kv(self, k: torch.Tensor, v: torch.Tensor, valid_len=None, layout: str = "compact", stream=None,
                       keep_mask: torch.Tensor | None = None):
        """k, v: [B][L][rows][256] bf16 on this device (other dtypes converted). Either valid_len
        (the first valid_len[b] rows are the compacted prefix) or keep_mask [B][rows] (the
        prefix pad mask: its True rows, in order, are gathered on the device)."""
        k = k.to(device=f"cuda:{self.device}", dtype=torch.bfloat16).contiguous()
        v = v.to(device=f"cuda:{self.device}", dtype=torch.bfloat16).contiguous()
        B, rows = k.shape[0], k.shape[2]
        lay = C.FA_KV_FLASHRT_INTERLEAVED if layout == "flashrt" else C.FA_KV_COMPACT_SPLIT_HALF
        if keep_mask is not None:
            m = keep_mask.to(device=f"cuda:{self.device}", dtype=torch.uint8).contiguous()
            self._check(self.lib.fa_bind_prefix_kv_masked(self.h, B, k.data_ptr(), v.data_ptr(), rows, m.data_ptr(), lay,
                                                          _stream_ptr(stream)))
        else:
            vl = (ctypes.c_int * B)(*[int(x) for x in valid_len])
            self._check(self.lib.fa_bind_prefix_kv(self.h, B, k.data_ptr(), v.data_ptr(), rows, vl, lay,
                                                   _stream_ptr(stream)))
        self.batch = B

    def sample_actions(self, noise: torch.Tensor, out: torch.Tensor | None = None, stream=None,
                       sync: bool = True) -> torch.Tensor:
        """noise [B][T][AD] fp32 (host or device). Returns actions, same shape, on noise's device
        unless `out` is given. sync=True waits and reports in-kernel timeouts."""
        noise = noise.float().contiguous()
        if out is None:
            out = torch.empty_like(noise)
        self._check(self.lib.fa_sample_actions(self.h, self.batch, noise.data_ptr(), out.data_ptr(),
                                               _stream_ptr(stream)))
        if sync:
            self.sync(stream)
        return out

    def sync(self, stream=None):
        self._check(self.lib.fa_sync(self.h, _stream_ptr(stream)))

    def set_stage_timing(self, enable=True):
        self._check(self.lib.fa_set_stage_timing(self.h, int(enable)))

    STAGES = ["embed/norm1", "qkv", "attention", "merge", "o_proj", "norm2", "gate_up", "down", "final"]

    def stage_times_ns(self):
        arr = (ctypes.c_uint64 * 9)()
        self._check(self.lib.fa_get_stage_cycles(self.h, arr, 9))
        return dict(zip(self.STAGES, list(arr)))

    def launch_count(self) -> int:
        return int(self.lib.fa_last_launch_count(self.h))

    def inject_fault(self, barrier_index: int, spin_limit: int = 0):
        self._check(self.lib.fa_set_fault_injection(self.h, barrier_index, spin_limit))

    def close(self):
        if getattr(self, "h", None):
            self.lib.fa_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


QUANT_FIELDS = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")


def quantized_weights(weights: dict, device):
    """The seven GEMM weights of `weights` quantised to FP8 on the GPU (flashact_b200.quant):
    returns (weights with codes in place of those seven, qscales) for
    Pi05ActionExpert(..., wfmt="fp8", qscales=...)."""
    from .quant import quantize_fp8_rows
    w, qs = dict(weights), {}
    for n in QUANT_FIELDS:
        w[n], qs[n] = quantize_fp8_rows(weights[n].to(device))
    return w, qs


OPENPI_EXPERT = "paligemma_with_expert.gemma_expert.model."


def weights_from_openpi(source, num_layers: int = 18) -> dict:
    """The engine's weight dict (keys of flashact_b200._capi.PI05_WEIGHT_FIELDS) from an openpi
    pi0.5 checkpoint: a state dict, or the path of a .safetensors file (read lazily, tensor by
    tensor) or of a torch checkpoint. Key names as the reference reads them
    (src/pi05/hybrid_model.py:76-133): `paligemma_with_expert.gemma_expert.model.layers.{i}.`
    `self_attn.{q,k,v,o}_proj.weight`, `mlp.{gate,up,down}_proj.weight`,
    `{input,post_attention}_layernorm.dense.{weight,bias}`, `...model.norm.dense.{weight,bias}`,
    `time_mlp_{in,out}.{weight,bias}`, `action_{in,out}_proj.{weight,bias}`. Per-layer tensors are
    stacked over the layers; dtypes are kept (the engine packs bf16 / fp16 / fp32 on the device)."""
    if isinstance(source, (str, bytes)) or hasattr(source, "__fspath__"):
        import os
        path = os.fspath(source)
        if str(path).endswith(".safetensors"):
            from safetensors import safe_open
            handle = safe_open(str(path), framework="pt", device="cpu")
            get = handle.get_tensor
        else:
            sd = torch.load(path, map_location="cpu", mmap=True, weights_only=True)
            get = sd.__getitem__
    else:
        get = source.__getitem__
    layer = OPENPI_EXPERT + "layers.{}."

    def stack(name):
        return torch.stack([get(layer.format(i) + name) for i in range(num_layers)])

    return {
        "wq": stack("self_attn.q_proj.weight"), "wk": stack("self_attn.k_proj.weight"),
        "wv": stack("self_attn.v_proj.weight"), "wo": stack("self_attn.o_proj.weight"),
        "w_gate": stack("mlp.gate_proj.weight"), "w_up": stack("mlp.up_proj.weight"),
        "w_down": stack("mlp.down_proj.weight"),
        "ln_in_w": stack("input_layernorm.dense.weight"), "ln_in_b": stack("input_layernorm.dense.bias"),
        "ln_post_w": stack("post_attention_layernorm.dense.weight"),
        "ln_post_b": stack("post_attention_layernorm.dense.bias"),
        "norm_w": get(OPENPI_EXPERT + "norm.dense.weight"), "norm_b": get(OPENPI_EXPERT + "norm.dense.bias"),
        "time_in_w": get("time_mlp_in.weight"), "time_in_b": get("time_mlp_in.bias"),
        "time_out_w": get("time_mlp_out.weight"), "time_out_b": get("time_mlp_out.bias"),
        "ain_w": get("action_in_proj.weight"), "ain_b": get("action_in_proj.bias"),
        "aout_w": get("action_out_proj.weight"), "aout_b": get("action_out_proj.bias"),
    }
