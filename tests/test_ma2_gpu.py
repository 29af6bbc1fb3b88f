"""GPU parity of the MolmoAct2 megakernel (through the C ABI) against the CPU oracle.

Tolerance: bf16 weights / activations vs the fp32 oracle on the valid action dims, max-abs 2e-2
(the bar the north_star sets for bf16); padded action dims must come back unchanged."""
import pytest
import torch

from oracle import molmoact2_oracle as M
from tests.pi05_util import err

TOL = 2e-2
pytestmark = pytest.mark.gpu


def run(c):
    from flashact_b200 import MolmoAct2ActionExpert
    eng = MolmoAct2ActionExpert(c.w, c.mods, c.mod_final, num_layers=c.L, horizon=c.T, action_dim=c.AD,
                                valid_action_dim=c.adim, max_context=c.Lk, max_batch=c.B, num_steps=c.num_steps,
                                rope_cos=c.rope_cos, rope_sin=c.rope_sin)
    eng.bind_context(c.kctx, c.vctx, [c.Lk] * c.B)
    return eng.sample_actions(c.noise.cuda()).cpu(), eng


def oracle_bf16(c):
    c2 = M.Ma2Case(**{**c.__dict__})
    c2.w = {**c.w, "w_aout": c.w["w_aout"].to(torch.bfloat16).float()}
    c2.kctx, c2.vctx = c.kctx.to(torch.bfloat16).float(), c.vctx.to(torch.bfloat16).float()
    return M.flow(c2)


@pytest.mark.parametrize("tm", ["0", "1"])
def test_ma2_small(require_gpu, monkeypatch, tm):
    """One observation against the fp32 oracle, with the weight-major GEMMs ("0", the default) and
    the opt-in token-major GEMMs ("1": activation tile as the M=64 A operand)."""
    monkeypatch.setenv("FA_MA2_TM", tm)
    c = M.make_case(seed=51, L=2, T=30, Lk=300, B=1, num_steps=2)
    out, _ = run(c)
    ref = oracle_bf16(c)
    mx, cos = err(out[..., :c.adim], ref[..., :c.adim])
    assert torch.isfinite(out).all()
    assert mx < TOL and cos > 0.9999, (mx, cos)
    assert torch.equal(out[..., c.adim:], c.noise[..., c.adim:])


def test_ma2_batch_short_context(require_gpu):
    c = M.make_case(seed=52, L=2, T=30, Lk=129, B=3, num_steps=2)
    out, _ = run(c)
    mx, cos = err(out[..., :c.adim], oracle_bf16(c)[..., :c.adim])
    assert mx < TOL, (mx, cos)


def test_ma2_config_c3(require_gpu):
    """BASELINE config C3 (MolmoAct2 as wired in the reference): 36 blocks, T=30, adim 6,
    Lk=493, 10 steps, bs=1, against the fp32 oracle."""
    c = M.make_case(seed=1)
    out, _ = run(c)
    mx, cos = err(out[..., :c.adim], M.flow(c)[..., :c.adim])
    print(f"MolmoAct2 C3 max_abs={mx:.4g} cos={cos:.7f}")
    assert mx < TOL and cos > 0.999, (mx, cos)


def test_ma2_masked_context_equals_host_compaction(require_gpu):
    """The cross-attention context gathered on the device from a keep mask (the model's cross mask
    == its max, benchmarks/molmoact2/eval_e2e.py:108-125) equals binding the host-compacted one."""
    from flashact_b200 import MolmoAct2ActionExpert
    c = M.make_case(seed=53, L=2, T=30, Lk=200, B=2, num_steps=2)
    g = torch.Generator().manual_seed(5)
    rows = 260
    keep = torch.rand(c.B, rows, generator=g) < 0.75
    kfull = torch.randn(c.B, c.L, rows, 768, generator=g).to(torch.bfloat16)
    vfull = torch.randn(c.B, c.L, rows, 768, generator=g).to(torch.bfloat16)
    counts = keep.sum(1).tolist()
    kc = torch.zeros_like(kfull)
    vc = torch.zeros_like(vfull)
    for b in range(c.B):
        kc[b, :, : counts[b]] = kfull[b][:, keep[b]]
        vc[b, :, : counts[b]] = vfull[b][:, keep[b]]
    eng = MolmoAct2ActionExpert(c.w, c.mods, c.mod_final, num_layers=c.L, horizon=c.T, action_dim=c.AD,
                                valid_action_dim=c.adim, max_context=rows, max_batch=c.B, num_steps=c.num_steps,
                                rope_cos=c.rope_cos, rope_sin=c.rope_sin)
    eng.bind_context(kfull, vfull, keep_mask=keep)
    out_masked = eng.sample_actions(c.noise.cuda()).cpu()
    eng.bind_context(kc, vc, counts)
    out_compact = eng.sample_actions(c.noise.cuda()).cpu()
    assert torch.equal(out_masked, out_compact)


def test_ma2_max_context_and_horizon(require_gpu):
    """Capacity edges: 4096 context tokens (128 chunks of 32 keys, the merge's maximum) and 32
    action tokens (the padded horizon), all 32 action dims integrated."""
    c = M.make_case(seed=53, L=1, T=32, Lk=4096, B=1, num_steps=1, adim=32)
    out, _ = run(c)
    mx, cos = err(out, oracle_bf16(c))
    assert mx < TOL and cos > 0.9999, (mx, cos)


def test_ma2_many_token_groups(require_gpu):
    """20 observations = 600 tokens: 128-token tiles over several token groups and several GEMM
    units per CTA (the large-batch plan)."""
    c = M.make_case(seed=54, L=1, T=30, Lk=64, B=20, num_steps=1)
    out, _ = run(c)
    mx, cos = err(out[..., :c.adim], oracle_bf16(c)[..., :c.adim])
    assert mx < TOL and cos > 0.9999, (mx, cos)


@pytest.mark.parametrize("T,adim,Lk,B", [(1, 1, 1, 2), (7, 6, 33, 3), (30, 6, 4064, 1)])
def test_ma2_odd_shapes(require_gpu, T, adim, Lk, B):
    """One action token and one context token, partial 32-key chunks, and 127 context chunks."""
    c = M.make_case(seed=55 + T, L=1, T=T, Lk=Lk, B=B, num_steps=2, adim=adim)
    out, _ = run(c)
    mx, cos = err(out[..., :adim], oracle_bf16(c)[..., :adim])
    assert mx < TOL and cos > 0.9999, (mx, cos)
    assert torch.equal(out[..., adim:], c.noise[..., adim:])


@pytest.mark.parametrize("selfq", ["8", "32"])
def test_ma2_self_attention_unit_sizes(require_gpu, monkeypatch, selfq):
    """Self-attention units of 8 query tokens (the small-batch plan) and of all 30 tokens (the
    large-batch plan) on the same small case, against the fp32 oracle."""
    monkeypatch.setenv("FA_MA2_SELFQ", selfq)
    c = M.make_case(seed=54, L=2, T=30, Lk=300, B=3, num_steps=2)
    out, _ = run(c)
    mx, cos = err(out[..., :c.adim], oracle_bf16(c)[..., :c.adim])
    assert mx < TOL and cos > 0.9999, (mx, cos)
    assert torch.equal(out[..., c.adim:], c.noise[..., c.adim:])


@pytest.mark.parametrize("whole", ["0", "1"])
def test_ma2_ragged_context_lengths(require_gpu, monkeypatch, whole):
    """Contexts of 1, 127, 128, 129 and 493 tokens in one batch: empty-but-one, partial and exact
    128-key tensor-core chunks of the cross-attention, with per-chunk units and a merge ("0") and
    with whole (observation, head) units and an online softmax over the chunks ("1")."""
    from flashact_b200 import MolmoAct2ActionExpert
    monkeypatch.setenv("FA_MA2_XWHOLE", whole)
    c = M.make_case(seed=55, L=2, T=30, Lk=493, B=5, num_steps=2)
    lens = [1, 127, 128, 129, 493]
    for b, n in enumerate(lens):
        c.kctx[b, :, n:] = 0
        c.vctx[b, :, n:] = 0
    eng = MolmoAct2ActionExpert(c.w, c.mods, c.mod_final, num_layers=c.L, horizon=c.T, action_dim=c.AD,
                                valid_action_dim=c.adim, max_context=c.Lk, max_batch=c.B, num_steps=c.num_steps,
                                rope_cos=c.rope_cos, rope_sin=c.rope_sin)
    eng.bind_context(c.kctx, c.vctx, lens)
    out = eng.sample_actions(c.noise.cuda()).cpu()
    outs = []
    for b, n in enumerate(lens):
        sub = M.Ma2Case(**{**c.__dict__})
        sub.B, sub.noise, sub.Lk = 1, c.noise[b:b + 1], n
        sub.kctx, sub.vctx = c.kctx[b:b + 1, :, :n], c.vctx[b:b + 1, :, :n]
        outs.append(oracle_bf16(sub)[0])
    ref = torch.stack(outs)
    mx, cos = err(out[..., :c.adim], ref[..., :c.adim])
    assert mx < TOL and cos > 0.9999, (mx, cos)
