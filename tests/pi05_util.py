"""Shared helpers for the pi0.5 tests: build the engine from an oracle case and compare."""
import torch

from oracle import pi05_oracle as O


def engine_for(case, **kw):
    from flashact_b200 import Pi05ActionExpert
    return Pi05ActionExpert(case.w, num_layers=case.L, horizon=case.T, action_dim=case.AD,
                            max_prefix=max(case.Lp, 1), max_batch=case.B, num_steps=case.num_steps, **kw)


def run_engine(case, eng=None, layout="compact"):
    eng = eng or engine_for(case)
    k = case.k.to(torch.bfloat16).cuda()
    v = case.v.to(torch.bfloat16).cuda()
    if layout == "flashrt":  # store K with rotary pairs interleaved (2d, 2d+1)
        k = torch.stack([k[..., :128], k[..., 128:]], dim=-1).reshape(k.shape).contiguous()
    eng.bind_prefix_kv(k, v, case.valid_len, layout=layout)
    out = eng.sample_actions(case.noise.cuda())
    return out.cpu(), eng


def oracle_bf16_kv(case, **kw):
    """Oracle with the prefix KV rounded to bf16 (the engine binds bf16 KV), fp32 math."""
    c2 = O.Pi05Case(**{**case.__dict__})
    c2.k = case.k.to(torch.bfloat16).float()
    c2.v = case.v.to(torch.bfloat16).float()
    return O.denoise(c2, **kw)


def err(a, b):
    d = (a.float() - b.float()).abs()
    cos = torch.nn.functional.cosine_similarity(a.float().ravel(), b.float().ravel(), dim=0).item()
    return d.max().item(), cos
