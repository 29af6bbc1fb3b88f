"""Pins the CPU oracles (and our kernel) to the reference's OWN CUDA kernels, live on a GPU.

The reference megakernels (src/pi05/mk6.cu, src/molmoact2/mk_ma2.cu) are compiled from their
sources for sm_100a by oracle/build_ref.py and launched through their own `launch` bindings
(tests/ref_runner.py), at their compiled shapes: pi0.5 with 18 layers and <= 16 action tokens
(FP8 W8A16, fp16 activations), MolmoAct2 with 36 blocks and 32 (30 valid) tokens (bf16).
Measured on B200: pi0.5 oracle vs reference kernel max-abs 2.6e-4; our kernel vs reference
kernel 2.7e-3; MolmoAct2 oracle vs reference kernel 2.9e-3.
"""
import pytest
import torch

from oracle import molmoact2_oracle as M
from oracle import pi05_oracle as O
from tests import ref_runner as R
from tests.pi05_util import engine_for, err

pytestmark = pytest.mark.gpu


def _ext(name):
    try:
        return R.load(name)
    except FileNotFoundError as e:
        pytest.skip(str(e))


def test_pi05_oracle_and_kernel_match_reference_kernel(require_gpu):
    ext = _ext("mk_v6_ref")
    c = O.make_case(**R.PI05_PIN)
    ref_kernel = R.run_pi05_ref(ext, c)
    c2 = R.pi05_dequantised_case(c)
    mods, modf = O.modulations(c.w, c.L, c.num_steps)
    ora = O.denoise(c2, mods=mods, mod_final=modf)[0]
    mx, cos = err(ref_kernel, ora)
    print(f"pi0.5 reference kernel vs oracle: max_abs={mx:.4g} cos={cos:.7f}")
    assert torch.isfinite(ref_kernel).all()
    assert mx < 5e-3 and cos > 0.99999, (mx, cos)
    eng = engine_for(c2, mods=mods, mod_final=modf)  # our kernel, bf16 copies of the same weights
    eng.bind_prefix_kv(c2.k.to(torch.bfloat16).cuda(), c2.v.to(torch.bfloat16).cuda(), c2.valid_len)
    ours = eng.sample_actions(c.noise.cuda()).cpu()[0]
    mx2, cos2 = err(ours, ref_kernel)
    print(f"pi0.5 our kernel vs reference kernel: max_abs={mx2:.4g} cos={cos2:.7f}")
    assert mx2 < 2e-2 and cos2 > 0.9999, (mx2, cos2)


def test_molmoact2_oracle_matches_reference_kernel(require_gpu):
    ext = _ext("mk_ma2_ref")
    c = M.make_case(**R.MA2_PIN)
    ref_kernel = R.run_ma2_ref(ext, c)
    ora = M.flow(R.ma2_bf16_case(c), weight_dtype=torch.bfloat16)[0]
    mx, cos = err(ref_kernel[:, :c.adim], ora[:, :c.adim])
    print(f"MolmoAct2 reference kernel vs oracle: max_abs={mx:.4g} cos={cos:.7f}")
    assert torch.isfinite(ref_kernel).all()
    assert mx < 1.5e-2 and cos > 0.9999, (mx, cos)


def test_pi05_compat_launch_matches_reference_kernel(require_gpu):
    """flashact_b200.compat.pi05_launch takes the reference launch() arguments unchanged (FP8
    packed weights, fp16 kcache / vtcache, x_t in place) and must reproduce the reference kernel."""
    from flashact_b200 import compat
    ext = _ext("mk_v6_ref")
    c = O.make_case(**R.PI05_PIN)
    ref_kernel = R.run_pi05_ref(ext, c)
    args, xt_d, x0 = R.pi05_ref_args(c)
    xt_d.copy_(x0)
    compat.pi05_launch(*args)
    torch.cuda.synchronize()
    ours = xt_d[:c.T].cpu()
    compat.clear_cache()
    mx, cos = err(ours, ref_kernel)
    print(f"pi0.5 compat launch vs reference kernel: max_abs={mx:.4g} cos={cos:.7f}")
    assert mx < 2e-2 and cos > 0.9999, (mx, cos)


def test_ma2_compat_launch_matches_reference_kernel(require_gpu):
    """flashact_b200.compat.ma2_launch with the reference MolmoAct2 launch() arguments."""
    from flashact_b200 import compat
    ext = _ext("mk_ma2_ref")
    c = M.make_case(**R.MA2_PIN)
    ref_kernel = R.run_ma2_ref(ext, c)
    args, xt_d, x0 = R.ma2_ref_args(c)
    xt_d.copy_(x0)
    compat.ma2_launch(*args)
    torch.cuda.synchronize()
    ours = xt_d[:c.T].cpu()
    compat.clear_cache()
    mx, cos = err(ours[:, :c.adim], ref_kernel[:, :c.adim])
    print(f"MolmoAct2 compat launch vs reference kernel: max_abs={mx:.4g} cos={cos:.7f}")
    assert mx < 2e-2 and cos > 0.9999, (mx, cos)
    assert torch.equal(ours[:, c.adim:], ref_kernel[:, c.adim:])


def test_pi05_compat_back_to_back_async(require_gpu):
    """Five compat launches queued back to back with no host synchronisation in between, each on new
    prefix KV written into the same kcache / vtcache buffers (a robot's successive observations):
    after the first call, a launch with an unchanged batch and prefix length re-copies the cache on
    the stream without re-planning or synchronising, like the reference's in-launch KV handoff
    (src/pi05/mk6.cu:258-277). Each chunk must match the reference kernel on the same KV."""
    import time
    from flashact_b200 import compat
    ext = _ext("mk_v6_ref")
    c = O.make_case(**R.PI05_PIN)
    args, xt_d, x0 = R.pi05_ref_args(c)
    kc, vt = args[19], args[20]
    g = torch.Generator(device="cuda").manual_seed(17)
    kvs = [(torch.randn(kc.shape, generator=g, device="cuda").half(), torch.randn(vt.shape, generator=g, device="cuda").half())
           for _ in range(5)]

    def run(launch):
        outs = []
        for k_, v_ in kvs:
            kc.copy_(k_)
            vt.copy_(v_)
            xt_d.copy_(x0)
            launch(*args)
            outs.append(xt_d[:c.T].clone())
        return outs

    run(compat.pi05_launch)  # engine creation + the first (planning) bind
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ours = run(compat.pi05_launch)
    t_queue = time.perf_counter() - t0  # host time to queue five launches (no synchronisation inside)
    torch.cuda.synchronize()
    ref = run(ext.launch)
    torch.cuda.synchronize()
    compat.clear_cache()
    print(f"five async compat launches queued in {t_queue * 1e3:.2f} ms of host time")
    assert t_queue < 0.025, t_queue  # each launch runs ~9 ms on the GPU: a host sync per call would show
    for i, (a, b) in enumerate(zip(ours, ref)):
        mx, cos = err(a.cpu(), b.cpu())
        print(f"launch {i}: compat vs reference kernel max_abs={mx:.4g} cos={cos:.7f}")
        assert mx < 2e-2 and cos > 0.9999, (i, mx, cos)
