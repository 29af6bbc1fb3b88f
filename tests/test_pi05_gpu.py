"""GPU parity of the pi0.5 megakernel (through the C ABI) against the CPU fp32 oracle.

Tolerance (north_star): bf16 weights/activations vs the fp32 reference, max-abs 2e-2 on the
action chunk."""
import pytest
import torch

from oracle import pi05_oracle as O
from tests.pi05_util import engine_for, err, oracle_bf16_kv, run_engine

TOL = 2e-2
pytestmark = pytest.mark.gpu


def test_small_single(require_gpu):
    c = O.make_case(seed=3, L=2, T=50, Lp=300, B=1, num_steps=2)
    out, _ = run_engine(c)
    ref = oracle_bf16_kv(c)
    mx, cos = err(out, ref)
    assert torch.isfinite(out).all()
    assert mx < TOL and cos > 0.9999, (mx, cos)


def test_small_batch_ragged_prefix(require_gpu):
    """Observations with different valid prefix lengths (incl. a partial chunk and an empty
    prefix): each uses its own RoPE positions and key mask."""
    c = O.make_case(seed=4, L=2, T=50, Lp=300, B=3, num_steps=2, valid_len=[300, 77, 0])
    out, _ = run_engine(c)
    ref = oracle_bf16_kv(c)
    mx, cos = err(out, ref)
    assert mx < TOL and cos > 0.9999, (mx, cos)


def test_short_horizon(require_gpu):
    c = O.make_case(seed=5, L=1, T=10, AD=7, Lp=128, B=1, num_steps=3)
    out, _ = run_engine(c)
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL, (mx, cos)


def test_flashrt_interleaved_kv(require_gpu):
    c = O.make_case(seed=6, L=2, T=50, Lp=200, B=1, num_steps=2)
    out, _ = run_engine(c, layout="flashrt")
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL, (mx, cos)


def test_deterministic_repeat(require_gpu):
    c = O.make_case(seed=7, L=2, T=50, Lp=256, B=1, num_steps=2)
    a, eng = run_engine(c)
    b = eng.sample_actions(c.noise.cuda()).cpu()
    assert torch.equal(a, b)


def test_baseline_config_bs1(require_gpu):
    """18 layers, T=50, Lp=968, N=10, bs=1, vs the fp32 oracle (C0)."""
    c = O.make_case(seed=0)
    out, _ = run_engine(c)
    ref = O.denoise(c)  # fp32 KV and weights: the C0 reference actions
    mx, cos = err(out, ref)
    print(f"baseline bs=1 max_abs={mx:.4g} cos={cos:.7f}")
    assert mx < TOL and cos > 0.999, (mx, cos)


def test_barrier_timeout_reported(require_gpu):
    """Host-side fault injection: block 0 skips a grid barrier; every wait is bounded, the launch
    ends with its error word set, fa_sync reports FA_ERR_TIMEOUT and the context stays usable."""
    from flashact_b200 import FlashActError
    c = O.make_case(seed=8, L=1, T=50, Lp=128, B=1, num_steps=1)
    good, eng = run_engine(c)
    eng.inject_fault(barrier_index=3, spin_limit=20000)
    with pytest.raises(FlashActError) as ei:
        eng.sample_actions(c.noise.cuda())
    assert "FA_ERR_TIMEOUT" in str(ei.value)
    eng.inject_fault(-1, 0)
    again = eng.sample_actions(c.noise.cuda()).cpu()
    assert torch.equal(good, again)


def test_masked_bind_equals_host_compaction(require_gpu):
    """fa_bind_prefix_kv_masked gathers the pad-masked prefix on the device; the result must be
    bit-identical to binding the host-compacted prefix (compact_kv, src/pi05/pack_weights.py:60-70)."""
    c = O.make_case(seed=21, L=2, T=50, AD=32, Lp=300, B=2, num_steps=2)
    g = torch.Generator().manual_seed(3)
    rows = 360
    keep = torch.rand(c.B, rows, generator=g) < 0.8
    kfull = torch.randn(c.B, c.L, rows, 256, generator=g).to(torch.bfloat16)
    vfull = torch.randn(c.B, c.L, rows, 256, generator=g).to(torch.bfloat16)
    counts = keep.sum(1).tolist()
    kc = torch.zeros(c.B, c.L, rows, 256, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    for b in range(c.B):
        kc[b, :, : counts[b]] = kfull[b][:, keep[b]]
        vc[b, :, : counts[b]] = vfull[b][:, keep[b]]
    eng = engine_for(c)
    eng.bind_prefix_kv(kfull.cuda(), vfull.cuda(), keep_mask=keep.cuda())
    out_masked = eng.sample_actions(c.noise.cuda()).cpu()
    eng.bind_prefix_kv(kc.cuda(), vc.cuda(), counts)
    out_compact = eng.sample_actions(c.noise.cuda()).cpu()
    assert torch.equal(out_masked, out_compact)


def test_max_prefix_and_horizon(require_gpu):
    """Capacity edges: the longest prefix the engine binds (31 full 128-key chunks = 3968 keys)
    and the longest horizon (64 action tokens, one whole 64-token tile)."""
    c = O.make_case(seed=9, L=1, T=64, AD=32, Lp=3968, B=1, num_steps=1)
    out, _ = run_engine(c)
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL and cos > 0.9999, (mx, cos)


def test_many_token_groups(require_gpu):
    """12 observations = 600 tokens: 128-token tiles in 3 token groups, several GEMM units per
    CTA and stage, K-splits stepped down (the large-batch plan), ragged prefixes."""
    c = O.make_case(seed=11, L=1, T=50, AD=32, Lp=256, B=12, num_steps=1,
                    valid_len=[256, 200, 129, 128, 127, 64, 1, 0, 256, 255, 100, 33])
    out, _ = run_engine(c)
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL and cos > 0.9999, (mx, cos)


def test_batch_permutation_full_size(require_gpu):
    """Full C1 geometry (18 layers, T=50, prefix 968, 10 steps) at 8 observations: permuting the
    observations permutes the action chunks bit for bit (every token column, chunk and split is
    computed the same way wherever it sits), and each chunk matches its bs=1 run at the bf16 bar."""
    c = O.make_case(seed=10, B=8)
    out, eng = run_engine(c)
    perm = [3, 0, 7, 1, 6, 2, 5, 4]
    eng.bind_prefix_kv(c.k[perm].to(torch.bfloat16).cuda(), c.v[perm].to(torch.bfloat16).cuda(),
                       [c.valid_len[i] for i in perm])
    out_p = eng.sample_actions(c.noise[perm].cuda()).cpu()
    assert torch.equal(out_p, out[perm])
    one = O.Pi05Case(**{**c.__dict__})
    one.B, one.noise, one.k, one.v, one.valid_len = 1, c.noise[5:6], c.k[5:6], c.v[5:6], c.valid_len[5:6]
    out1, _ = run_engine(one)
    mx, cos = err(out1, out[5:6])
    assert mx < TOL and cos > 0.9999, (mx, cos)


@pytest.mark.parametrize("T,AD,B,num_steps", [(1, 1, 3, 2), (17, 5, 2, 1), (63, 32, 1, 1), (50, 32, 1, 50)])
def test_odd_shapes(require_gpu, T, AD, B, num_steps):
    """Horizons 1 / 17 / 63 (partial 16-token chunks, the scalar V-transpose path), action dims
    1 / 5, and the longest schedule (50 Euler steps)."""
    c = O.make_case(seed=12 + T, L=1, T=T, AD=AD, Lp=130, B=B, num_steps=num_steps)
    out, _ = run_engine(c)
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL and cos > 0.9999, (mx, cos)


@pytest.mark.parametrize("B,valid", [(3, [300, 77, 0]), (12, [256, 200, 129, 128, 127, 64, 1, 0, 256, 255, 100, 33])])
def test_whole_unit_attention(require_gpu, monkeypatch, B, valid):
    """Whole-unit attention (one unit per observation and head pair over all its key chunks, two-pass
    softmax, no merge stage; the plan above 36 observations) forced on small ragged batches,
    empty and partial prefixes included, against the fp32 oracle."""
    monkeypatch.setenv("FA_ATTN_WHOLE", "1")
    c = O.make_case(seed=40 + B, L=2, T=50, AD=32, Lp=300, B=B, num_steps=2, valid_len=valid)
    out, _ = run_engine(c)
    mx, cos = err(out, oracle_bf16_kv(c))
    assert mx < TOL and cos > 0.9999, (mx, cos)
