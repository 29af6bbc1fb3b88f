"""MolmoAct2 action-expert flow engine: Python host mirror of the reference's MolmoAct2 path.

The reference replaces the model's `_run_action_flow_loop` with its packing + one kernel launch
(benchmarks/molmoact2/eval_e2e.py:105-144): weights packed once, the model's modulation cache
passed as mods / mod_final, the per-block cross-attention context compacted to its valid tokens,
the rope cache, then `launch`. Here: construct (weight load), set_modulation, bind_context,
sample_actions — all through the C ABI of libflashact.so. No CPU fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi as C
from .pi05 import _DT, _stream_ptr


class MolmoAct2ActionExpert:
    """weights: dict with the keys of flashact_b200._capi.MA2_WEIGHT_FIELDS ([out][in], stacked
    over blocks). mods [N][L][3][3][768], mod_final [N][2][768]: the model's modulation cache."""

    def __init__(self, weights: dict, mods, mod_final, *, num_layers=36, horizon=30, action_dim=32,
                 valid_action_dim=6, max_context=493, max_batch=1, num_steps=10, device: int = 0,
                 rope_cos=None, rope_sin=None):
        self.lib = C.load_library()
        self.device = device
        self.cfg = C.FaConfig(num_layers, 768, 8, 8, 96, 3072, horizon, action_dim, max_context, max_batch,
                              num_steps, valid_action_dim)
        h = ctypes.c_void_p()
        C.check(self.lib, None, self.lib.fa_create(C.FA_MODEL_MOLMOACT2, ctypes.byref(self.cfg), device,
                                                   ctypes.byref(h)))
        self.h = h
        self.batch = 0
        keep, w = [], C.FaMa2Weights()
        alias = {"ain_w": "w_ain", "ain_b": "b_ain", "aout_w": "w_aout", "aout_b": "b_aout"}
        for name in C.MA2_WEIGHT_FIELDS:
            t = weights[name] if name in weights else weights[alias[name]]
            if t.dtype not in _DT:
                t = t.float()
            t = t.contiguous()
            keep.append(t)
            setattr(w, name, C.FaTensor(t.data_ptr(), _DT[t.dtype]))
        self._check(self.lib.fa_ma2_load_weights(self.h, ctypes.byref(w)))
        self.set_modulation(mods, mod_final)
        if rope_cos is not None:
            cs, sn = rope_cos.float().contiguous(), rope_sin.float().contiguous()
            self._check(self.lib.fa_ma2_set_rope(self.h, cs.data_ptr(), sn.data_ptr()))

    def _check(self, st):
        C.check(self.lib, self.h, st)

    def set_modulation(self, mods, mod_final):
        m, mf = mods.float().contiguous(), mod_final.float().contiguous()
        self._check(self.lib.fa_set_modulation(self.h, m.data_ptr(), mf.data_ptr()))

    def bind_context(self, k: torch.Tensor, v: torch.Tensor, ctx_len=None, stream=None,
                     keep_mask: torch.Tensor | None = None):
        """k, v: [B][L][rows][768] projected cross-attention context: either the first ctx_len[b]
        rows are valid, or keep_mask [B][rows] marks them (the model's cross mask == its max;
        gathered on the device)."""
        k = k.to(device=f"cuda:{self.device}", dtype=torch.bfloat16).contiguous()
        v = v.to(device=f"cuda:{self.device}", dtype=torch.bfloat16).contiguous()
        B, rows = k.shape[0], k.shape[2]
        if keep_mask is not None:
            m = keep_mask.to(device=f"cuda:{self.device}", dtype=torch.uint8).contiguous()
            self._check(self.lib.fa_bind_prefix_kv_masked(self.h, B, k.data_ptr(), v.data_ptr(), rows, m.data_ptr(), 0,
                                                          _stream_ptr(stream)))
        else:
            lens = (ctypes.c_int * B)(*[int(x) for x in ctx_len])
            self._check(self.lib.fa_bind_prefix_kv(self.h, B, k.data_ptr(), v.data_ptr(), rows, lens, 0,
                                                   _stream_ptr(stream)))
        self.batch = B

    def sample_actions(self, noise: torch.Tensor, out=None, stream=None, sync=True):
        noise = noise.float().contiguous()
        if out is None:
            out = torch.empty_like(noise)
        self._check(self.lib.fa_sample_actions(self.h, self.batch, noise.data_ptr(), out.data_ptr(),
                                               _stream_ptr(stream)))
        if sync:
            self._check(self.lib.fa_sync(self.h, _stream_ptr(stream)))
        return out

    def sync(self, stream=None):
        self._check(self.lib.fa_sync(self.h, _stream_ptr(stream)))

    def launch_count(self) -> int:
        return int(self.lib.fa_last_launch_count(self.h))

    def set_stage_timing(self, enable=True):
        self._check(self.lib.fa_set_stage_timing(self.h, int(enable)))

    STAGES = ["embed/norm1", "qkv", "self_attn", "self_out", "norm2", "cross_q", "cross_attn", "merge", "cross_out",
              "norm3", "gate_up", "down", "final"]

    def stage_times_ns(self):
        arr = (ctypes.c_uint64 * 13)()
        self._check(self.lib.fa_get_stage_cycles(self.h, arr, 13))
        return dict(zip(self.STAGES, list(arr)))

    def close(self):
        if getattr(self, "h", None):
            self.lib.fa_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
