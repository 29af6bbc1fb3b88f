"""CPU fp32 oracle of the pi0.5 action-expert denoise loop — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this
module, and only as the checker or the timed CPU baseline. The product path (the C-ABI library)
never calls it.

What it restates (citations relative to the reference project GautamSharda/FlashAct):
  * schedule: t_0 = 1, dt = -1/N, x_t += dt * v (benchmarks/pi05/eval_numerics.py:60-68,
    src/pi05/mk6.cu:128);
  * conditioning: openpi create_sinusoidal_pos_embedding(t, 1024, 4e-3, 4.0) in float64,
    cond = silu(time_mlp_out(silu(time_mlp_in(emb)))), per-layer adaRMS modulations from
    input_layernorm.dense / post_attention_layernorm.dense, final from model.norm.dense, each
    output split scale | shift | gate (src/pi05/hybrid_model.py:111-128, pack_weights.py:26-45);
  * embed x = W_ain x_t + b (mk6.cu:280-289); adaRMSNorm xn = x rsqrt(mean x^2 + 1e-6) (1+scale)
    + shift and the gated residual x += gate * y (mk6.cu:139-164, :302, :429);
  * attention: q = Wq xn, k = Wk xn, v = Wv xn; split-half RoPE (pairs d, d+128, theta 1e4) at
    positions valid_len + t (pack_weights.py:54-58, mk6.cu:221-244); the action tokens attend to
    every valid prefix key and every action token, one shared KV head, scale 1/16, fp32 softmax
    (mk6.cu:313-419);
  * GeGLU MLP h = gelu_tanh(W_g xn) * (W_u xn), y = W_d h (mk6.cu:435-495);
  * final adaRMS with mod_final (scale|shift), v = W_aout xn + b (mk6.cu:503-515).

The reference's own CPU path is openpi's PI0Pytorch.denoise_step, which lives in an empty git
submodule (third_party/openpi) of the reference and is not available here; this restatement is
written from the kernel semantics above. Its agreement with the reference's own CUDA kernel
(src/pi05/mk6.cu, compiled from source into oracle/_ref) is checked by tests/test_ref_pin.py on
a GPU; without that run, parity with openpi itself is unpinned.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

D, H, HD, F = 1024, 8, 256, 4096


@dataclass
class Pi05Case:
    """Seeded synthetic inputs. Generation order (torch.manual_seed(seed), CPU fp32 randn):
    per layer i: wq, wk, wv, wo, w_gate, w_up, w_down, ln_in_w, ln_in_b, ln_post_w, ln_post_b;
    then norm_w, norm_b, time_in_w, time_in_b, time_out_w, time_out_b, ain_w, ain_b, aout_w,
    aout_b; then per observation: prefix K [L][Lp][256], prefix V [L][Lp][256], noise [T][AD].
    Weights ~ N(0, 0.02), biases ~ 0.02 N(0, 1), K/V and noise ~ N(0, 1)."""
    L: int
    T: int
    AD: int
    Lp: int
    B: int
    num_steps: int
    w: dict = field(default_factory=dict)
    k: torch.Tensor = None  # [B][L][Lp][256]
    v: torch.Tensor = None
    noise: torch.Tensor = None  # [B][T][AD]
    valid_len: list = None


def make_case(seed=0, L=18, T=50, AD=32, Lp=968, B=1, num_steps=10, valid_len=None) -> Pi05Case:
    g = torch.Generator().manual_seed(seed)

    def W(*shape):
        return torch.randn(*shape, generator=g) * 0.02

    c = Pi05Case(L=L, T=T, AD=AD, Lp=Lp, B=B, num_steps=num_steps)
    per = {n: [] for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "ln_in_w", "ln_in_b", "ln_post_w",
                           "ln_post_b")}
    for _ in range(L):
        per["wq"].append(W(H * HD, D))
        per["wk"].append(W(HD, D))
        per["wv"].append(W(HD, D))
        per["wo"].append(W(D, H * HD))
        per["w_gate"].append(W(F, D))
        per["w_up"].append(W(F, D))
        per["w_down"].append(W(D, F))
        per["ln_in_w"].append(W(3 * D, D))
        per["ln_in_b"].append(W(3 * D))
        per["ln_post_w"].append(W(3 * D, D))
        per["ln_post_b"].append(W(3 * D))
    c.w = {n: torch.stack(v).contiguous() for n, v in per.items()}
    c.w["norm_w"] = W(3 * D, D)
    c.w["norm_b"] = W(3 * D)
    c.w["time_in_w"] = W(D, D)
    c.w["time_in_b"] = W(D)
    c.w["time_out_w"] = W(D, D)
    c.w["time_out_b"] = W(D)
    c.w["ain_w"] = W(D, AD)
    c.w["ain_b"] = W(D)
    c.w["aout_w"] = W(AD, D)
    c.w["aout_b"] = W(AD)
    ks, vs, ns = [], [], []
    for _ in range(B):
        ks.append(torch.randn(L, Lp, HD, generator=g))
        vs.append(torch.randn(L, Lp, HD, generator=g))
        ns.append(torch.randn(T, AD, generator=g))
    c.k, c.v, c.noise = torch.stack(ks), torch.stack(vs), torch.stack(ns)
    c.valid_len = list(valid_len) if valid_len is not None else [Lp] * B
    return c


def sinusoidal_embedding(t: torch.Tensor, dim=D, min_period=4e-3, max_period=4.0) -> torch.Tensor:
    """openpi create_sinusoidal_pos_embedding: float64 periods log-spaced in [min, max], sin | cos."""
    frac = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** frac
    arg = (1.0 / period * 2 * math.pi)[None, :] * t.to(torch.float64)[:, None]
    return torch.cat([torch.sin(arg), torch.cos(arg)], dim=1).to(torch.float32)


def modulations(w: dict, L: int, num_steps: int):
    """mods [N][L][2][3072] (input / post-attention adaRMS) and mod_final [N][3072]."""
    t = torch.tensor([1.0 - i / num_steps for i in range(num_steps)], dtype=torch.float32)
    emb = sinusoidal_embedding(t)
    silu = torch.nn.functional.silu
    lin = torch.nn.functional.linear
    h = silu(lin(emb, w["time_in_w"].float(), w["time_in_b"].float()))
    cond = silu(lin(h, w["time_out_w"].float(), w["time_out_b"].float()))
    mods = torch.zeros(num_steps, L, 2, 3 * D)
    for l in range(L):
        mods[:, l, 0] = lin(cond, w["ln_in_w"][l].float(), w["ln_in_b"][l].float())
        mods[:, l, 1] = lin(cond, w["ln_post_w"][l].float(), w["ln_post_b"][l].float())
    mod_final = lin(cond, w["norm_w"].float(), w["norm_b"].float())
    return mods, mod_final


def rope_tables(start: int, T: int):
    inv = 1.0 / (10000.0 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))
    pos = torch.arange(start, start + T, dtype=torch.float32)
    ang = torch.outer(pos, inv)
    return ang.cos(), ang.sin()


def _rope(x, cos, sin):
    """split-half rotation of the last dim (256): pairs (d, d+128)."""
    x1, x2 = x[..., :128], x[..., 128:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def _adarms(x, mod):
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    return x * r * (1 + mod[:D]) + mod[D:2 * D]


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def denoise(c: Pi05Case, mods=None, mod_final=None, weight_dtype=torch.float32, max_obs=None) -> torch.Tensor:
    """Runs the N-step Euler loop for every observation; returns actions [B][T][AD] fp32.
    weight_dtype=torch.bfloat16 rounds the GEMM weights to bf16 first (isolates the kernel's
    activation rounding from weight rounding); the math stays fp32."""
    L, T, N = c.L, c.T, c.num_steps
    if mods is None:
        mods, mod_final = modulations(c.w, L, N)
    rw = lambda n: c.w[n].to(weight_dtype).float()
    wq, wk, wv, wo = rw("wq"), rw("wk"), rw("wv"), rw("wo")
    wg, wu, wd = rw("w_gate"), rw("w_up"), rw("w_down")
    ain_w, ain_b, aout_w, aout_b = (c.w[n].float() for n in ("ain_w", "ain_b", "aout_w", "aout_b"))
    dt = -1.0 / N
    outs = []
    for b in range(c.B if max_obs is None else min(c.B, max_obs)):
        vl = c.valid_len[b]
        cos, sin = rope_tables(vl, T)
        kp, vp = c.k[b, :, :vl].float(), c.v[b, :, :vl].float()
        x_t = c.noise[b].float().clone()
        for s in range(N):
            x = x_t @ ain_w.T + ain_b
            for l in range(L):
                m_in, m_post = mods[s, l, 0], mods[s, l, 1]
                xn = _adarms(x, m_in)
                q = (xn @ wq[l].T).view(T, H, HD)
                k = xn @ wk[l].T
                v = xn @ wv[l].T
                q = _rope(q, cos[:, None, :], sin[:, None, :])
                k = _rope(k, cos, sin)
                K = torch.cat([kp[l], k], 0)
                V = torch.cat([vp[l], v], 0)
                sc = torch.einsum("thd,kd->htk", q, K) / 16.0
                p = torch.softmax(sc, dim=-1)
                att = torch.einsum("htk,kd->thd", p, V).reshape(T, H * HD)
                x = x + m_in[2 * D:] * (att @ wo[l].T)
                xn2 = _adarms(x, m_post)
                h = gelu_tanh(xn2 @ wg[l].T) * (xn2 @ wu[l].T)
                x = x + m_post[2 * D:] * (h @ wd[l].T)
            xf = _adarms(x, mod_final[s])
            v_t = xf @ aout_w.T + aout_b
            x_t = x_t + dt * v_t
        outs.append(x_t)
    return torch.stack(outs)
