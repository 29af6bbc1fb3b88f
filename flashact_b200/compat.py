"""Drop-in replacements for the reference's two pybind `launch` entry points.

The reference builds one torch extension per model whose only function is `launch(...)`:
  * pi0.5      src/pi05/binding.cpp:28-37       (called at src/pi05/hybrid_model.py:215-221,
                                                 benchmarks/pi05/eval_numerics.py:101-107)
  * MolmoAct2  src/molmoact2/binding.cpp:28-35  (called at src/molmoact2/eval_e2e.py:141-143,
                                                 benchmarks/molmoact2/eval_numerics.py:147-150)
`pi05_launch` / `ma2_launch` take exactly those arguments (same order, same tensors, same
in-place contract: the action chunk is written into `x_t[:Tv]` on the current stream) and map
them onto the C ABI: the first call for a given set of weight tensors creates and loads an
engine (cached on the weights' data pointers), every call binds the prefix KV / context and runs
`fa_sample_actions`. A caller switches by replacing `ext.launch` with these functions, e.g.
`ext = types.SimpleNamespace(launch=flashact_b200.compat.pi05_launch)`.

Argument handling:
  * pi0.5 weights arrive FP8 E4M3 with per-row scales in the reference's packed row order
    (W1 = [Q rope-pair interleaved | K interleaved | V], W2 = gate/up interleaved,
    src/pi05/hybrid_model.py:100-110); the codes and scales are put back in model row order and
    loaded as FP8, so the engine streams E4M3 with the row scales applied to the fp32
    accumulators, the reference's own W8A16 scheme (FA_FP8_STREAM=0 dequantises them at load
    into the bf16 kernel instead).
  * mods / mod_final are used as given (the reference precomputes them on the host).
  * RoPE tables: the engine derives the action tokens' rotation from the prefix length with
    theta = 10000 (src/pi05/pack_weights.py:54-58), which is what the reference's callers pass;
    MolmoAct2's tables are taken from the call.
  * Scratch tensors (x, xp, xn, q, attn, hmlp, bufs, scores, probs) and nblocks / nthreads are
    accepted and unused: the engine owns its scratch and sizes its grid to the GPU.
  * stage_cycles (when non-empty) receives per-stage nanoseconds instead of clock cycles.
Errors raise flashact_b200.FlashActError (the reference raises on launch failure only).
"""
from __future__ import annotations

import ctypes

import torch

from .molmoact2 import MolmoAct2ActionExpert
from .pi05 import Pi05ActionExpert

_engines: dict = {}


def _dev_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _pi05_weights(w1, wo, w2, w3, s1, so_, s2, s3, w_ain, b_ain, w_aout, b_aout):
    """The reference's packed FP8 tensors -> (weights with codes in model row order, qscales)."""
    L = w1.shape[0]
    dev = w1.device
    p = torch.arange(1024, device=dev)
    qsrc = torch.stack([p // 128 * 256 + p % 128, p // 128 * 256 + p % 128 + 128], 1).reshape(-1)
    jk = torch.arange(128, device=dev)
    ksrc = torch.stack([jk, jk + 128], 1).reshape(-1)

    def unpermute(x, src, rows):  # packed row i holds model row src[i]
        out = torch.empty((L, rows) + tuple(x.shape[2:]), dtype=x.dtype, device=dev)
        out[:, src] = x
        return out.contiguous()

    c1, sc1 = w1.view(torch.uint8), s1.float()
    c2, sc2 = w2.view(torch.uint8).view(L, 4096, 2, 1024), s2.float().view(L, 4096, 2)
    codes = {"wq": unpermute(c1[:, :2048], qsrc, 2048), "wk": unpermute(c1[:, 2048:2304], ksrc, 256),
             "wv": c1[:, 2304:].contiguous(), "wo": wo.view(torch.uint8).contiguous(),
             "w_gate": c2[:, :, 0].contiguous(), "w_up": c2[:, :, 1].contiguous(),
             "w_down": w3.view(torch.uint8).contiguous()}
    scales = {"wq": unpermute(sc1[:, :2048], qsrc, 2048), "wk": unpermute(sc1[:, 2048:2304], ksrc, 256),
              "wv": sc1[:, 2304:].contiguous(), "wo": so_.float().contiguous(),
              "w_gate": sc2[:, :, 0].contiguous(), "w_up": sc2[:, :, 1].contiguous(), "w_down": s3.float().contiguous()}
    return {**codes, "ain_w": w_ain, "ain_b": b_ain, "aout_w": w_aout, "aout_b": b_aout}, scales


def _write_stage_times(eng, stage_cycles):
    """Per-stage nanoseconds into stage_cycles, asynchronously on the launch stream when it is a
    contiguous 64-bit device tensor (the reference fills it from inside its kernel)."""
    if stage_cycles is None or stage_cycles.numel() == 0:
        return
    if stage_cycles.is_cuda and stage_cycles.dtype in (torch.int64, torch.uint64) and stage_cycles.is_contiguous():
        eng._check(eng.lib.fa_get_stage_cycles(eng.h, ctypes.cast(stage_cycles.data_ptr(), ctypes.POINTER(ctypes.c_uint64)),
                                               min(stage_cycles.numel(), 16)))
        return
    t = eng.stage_times_ns()
    vals = torch.tensor(list(t.values())[: stage_cycles.numel()], dtype=torch.int64)
    stage_cycles.view(-1)[: vals.numel()].copy_(vals.to(stage_cycles.device).to(stage_cycles.dtype))


def pi05_launch(w1, wo, w2, w3, s1, so_, s2, s3, mods, mod_final, rope_cos, rope_sin,
                w_ain, b_ain, w_aout, b_aout, kvsrc_k, kvsrc_v, srows, kcache, vtcache,
                Lp, Lmax, num_steps, Tv, x_t, x, xp, stage_cycles, xn, q, attn, hmlp,
                scores, probs, nblocks, nthreads):
    """Same arguments and effect as the reference's pi0.5 `launch` (src/pi05/binding.cpp:28-37):
    runs `num_steps` Euler steps on x_t[:Tv] in place. With srows > 0 the prefix comes from
    kvsrc_k / kvsrc_v ([L][srows][256] bf16, FlashRT's interleaved RoPE layout, first Lp rows);
    otherwise from kcache [L][Lmax][256] / vtcache [L][256][Lmax] (fp16, first Lp keys)."""
    dev = _dev_index(x_t)
    L = int(w1.shape[0])
    key = ("pi05", dev, w1.data_ptr(), wo.data_ptr(), w2.data_ptr(), w3.data_ptr(), mods.data_ptr(), int(Tv),
           int(num_steps), int(Lmax))
    eng = _engines.get(key)
    if eng is None:
        weights, qscales = _pi05_weights(w1, wo, w2, w3, s1, so_, s2, s3, w_ain, b_ain, w_aout, b_aout)
        eng = Pi05ActionExpert(weights, num_layers=L, horizon=int(Tv), action_dim=int(x_t.shape[1]),
                               max_prefix=max(int(Lmax), int(srows)), max_batch=1, num_steps=int(num_steps),
                               device=dev, mods=mods, mod_final=mod_final, wfmt="fp8", qscales=qscales)
        _engines[key] = eng
    if stage_cycles is not None and stage_cycles.numel() > 0:
        eng.set_stage_timing(True)
    if int(srows) > 0:
        eng.bind_prefix_kv(kvsrc_k.view(1, L, int(srows), 256), kvsrc_v.view(1, L, int(srows), 256), [int(Lp)],
                           layout="flashrt")
    else:
        k = kcache[:, : int(Lmax)].to(torch.bfloat16).unsqueeze(0)
        v = vtcache.transpose(1, 2).to(torch.bfloat16).unsqueeze(0)
        eng.bind_prefix_kv(k, v, [int(Lp)])
    chunk = x_t[: int(Tv)]
    eng.sample_actions(chunk, out=chunk, sync=False)
    _write_stage_times(eng, stage_cycles)


def ma2_launch(ws, bs, mods, mod_final, rope_cos, rope_sin, w_ain, b_ain, w_aout, b_aout, kctx, vtctx,
               Lk, Lkmax, Tv, adim, num_steps, x_t, x, xp, stage_cycles, bufs, scores, probs, nblocks, nthreads):
    """Same arguments and effect as the reference's MolmoAct2 `launch`
    (src/molmoact2/binding.cpp:28-35): ws / bs = (qkv, self-out, cross-q, cross-out, gate/up
    interleaved, down) bf16 weights / fp32 biases; kctx [L][Lkmax][768] and vtctx [L][768][Lkmax]
    bf16 with the first Lk context tokens valid; x_t[:Tv] is integrated in place on dims < adim."""
    dev = _dev_index(x_t)
    L, F2, Dm = (int(v) for v in ws[4].shape)
    key = ("ma2", dev, ws[0].data_ptr(), ws[4].data_ptr(), ws[5].data_ptr(), mods.data_ptr(), int(Tv), int(adim),
           int(num_steps), int(Lkmax))
    eng = _engines.get(key)
    if eng is None:
        gu = ws[4].view(L, F2 // 2, 2, Dm)
        bgu = bs[4].view(L, F2 // 2, 2)
        weights = {"w_qkv": ws[0], "b_qkv": bs[0], "w_so": ws[1], "b_so": bs[1], "w_cq": ws[2], "b_cq": bs[2],
                   "w_co": ws[3], "b_co": bs[3], "w_gate": gu[:, :, 0], "b_gate": bgu[:, :, 0], "w_up": gu[:, :, 1],
                   "b_up": bgu[:, :, 1], "w_down": ws[5], "b_down": bs[5], "w_ain": w_ain, "b_ain": b_ain,
                   "w_aout": w_aout, "b_aout": b_aout}
        eng = MolmoAct2ActionExpert(weights, mods, mod_final, num_layers=L, horizon=int(Tv),
                                    action_dim=int(x_t.shape[1]), valid_action_dim=int(adim),
                                    max_context=int(Lkmax), max_batch=1, num_steps=int(num_steps), device=dev,
                                    rope_cos=rope_cos[: int(Tv)], rope_sin=rope_sin[: int(Tv)])
        _engines[key] = eng
    if stage_cycles is not None and stage_cycles.numel() > 0:
        eng.set_stage_timing(True)
    eng.bind_context(kctx.unsqueeze(0), vtctx.transpose(1, 2).unsqueeze(0), [int(Lk)])
    chunk = x_t[: int(Tv)]
    eng.sample_actions(chunk, out=chunk, sync=False)
    _write_stage_times(eng, stage_cycles)


def clear_cache():
    """Drops the cached engines (their device memory is freed)."""
    for eng in _engines.values():
        eng.close()
    _engines.clear()
