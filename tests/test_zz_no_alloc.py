"""GPU test of fa_pi05_modulations_noalloc, the allocation-free conditioning entry point.

It exists for callers that cannot allocate device memory when they need the adaRMS modulations
(for example a control process whose memory budget is fixed after start-up); its scratch is a
static array inside the library. The test calls it twice in a row through the C ABI and checks
its modulations against the CPU oracle's conditioning chain (fp32 tolerance), and that actions
sampled with them agree with actions from the existing path, where fa_pi05_load_weights computes
the modulations itself, within the suite's bf16 tolerance. It runs with fp32 and with bf16
weights, and at 20 Euler steps, where the conditioning kernels need more than 48 KB of shared
memory.
This file is collected last so that a run stopping at the first failure has run every other test.
"""
import ctypes

import pytest
import torch

from oracle import pi05_oracle as O
from tests.pi05_util import engine_for, err

TOL = 2e-2
pytestmark = pytest.mark.gpu


MOD_TOL = 1e-4  # fp32 conditioning chain on the GPU vs the same chain on the CPU


def _device_weights(case, dtype=torch.float32):
    from flashact_b200 import _capi as C
    keep, w = [], C.FaPi05Weights()
    code = {torch.float32: C.FA_DT_F32, torch.bfloat16: C.FA_DT_BF16}[dtype]
    for name in C.PI05_WEIGHT_FIELDS:
        t = case.w[name].to(dtype).contiguous().cuda()
        keep.append(t)
        setattr(w, name, C.FaTensor(t.data_ptr(), code))
    return w, keep


@pytest.mark.parametrize("dtype,num_steps", [(torch.float32, 3), (torch.bfloat16, 3), (torch.float32, 20)])
def test_noalloc_modulations_match_load_weights(require_gpu, dtype, num_steps):
    from flashact_b200 import _capi as C
    lib = C.load_library()
    c = O.make_case(seed=21, L=2, T=50, AD=32, Lp=128, B=1, num_steps=num_steps)
    if dtype != torch.float32:  # both paths (and the oracle) then see the same rounded weights
        c.w = {n: t.to(dtype).float() for n, t in c.w.items()}
    want_mods, want_modf = O.modulations(c.w, c.L, c.num_steps)
    k = c.k.to(torch.bfloat16).cuda()
    v = c.v.to(torch.bfloat16).cuda()
    noise = c.noise.cuda()

    ref_eng = engine_for(c)  # existing path: modulations computed inside fa_pi05_load_weights
    ref_eng.bind_prefix_kv(k, v, c.valid_len)
    ref = ref_eng.sample_actions(noise).cpu()

    w, keep = _device_weights(c, dtype)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    results = []
    for _ in range(2):  # two calls in a row share the static scratch
        mods = torch.full((c.num_steps, c.L, 2, 3072), float("nan"), device="cuda")
        modf = torch.full((c.num_steps, 3072), float("nan"), device="cuda")
        st = lib.fa_pi05_modulations_noalloc(ctypes.byref(w), c.L, c.num_steps, mods.data_ptr(), modf.data_ptr(),
                                             stream)
        assert st == C.FA_OK, lib.fa_last_error(None)
        torch.cuda.synchronize()
        assert torch.isfinite(mods).all() and torch.isfinite(modf).all()
        assert (mods.cpu() - want_mods).abs().max().item() < MOD_TOL
        assert (modf.cpu() - want_modf).abs().max().item() < MOD_TOL
        eng = engine_for(c, mods=mods, mod_final=modf)
        eng.bind_prefix_kv(k, v, c.valid_len)
        out = eng.sample_actions(noise).cpu()
        mx, cos = err(out, ref)
        assert mx < TOL, (mx, cos)
        results.append((mods.cpu(), modf.cpu(), out))
        eng.close()
    assert torch.equal(results[0][0], results[1][0]) and torch.equal(results[0][1], results[1][1])
    ref_eng.close()


def test_noalloc_rejects_too_many_steps(require_gpu):
    from flashact_b200 import _capi as C
    lib = C.load_library()
    c = O.make_case(seed=22, L=1, T=10, AD=8, Lp=16, B=1, num_steps=1)
    w, keep = _device_weights(c)
    mods = torch.empty(51, 1, 2, 3072, device="cuda")
    modf = torch.empty(51, 3072, device="cuda")
    st = lib.fa_pi05_modulations_noalloc(ctypes.byref(w), 1, 51, mods.data_ptr(), modf.data_ptr(), None)
    assert st == C.FA_ERR_INVALID
    assert b"50" in lib.fa_last_error(None)
