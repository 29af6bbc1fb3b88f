"""CPU fp32 oracle of the MolmoAct2 action-expert flow loop — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py may import this module, and only as the
checker or the timed CPU baseline.

Restated from the reference's kernel semantics (paths relative to GautamSharda/FlashAct):
  * schedule: x <- noise; for i in 0..N-1: x += (1/N) v(x, t_i), t_i = i/N, with the action-dim
    mask applied to v (benchmarks/molmoact2/eval_numerics.py:59-75; src/molmoact2/mk_ma2.cu:
    115, 565);
  * embed x = W_ain x_t + b (mk_ma2.cu:259-268);
  * per DiT block (mk_ma2.cu:273-556), with modulations mods[s][l][n] = (scale, shift, gate) for
    n = self-attention, cross-attention, MLP:
      xn = rms(x) (1 + scale) + shift (eps 1e-6, mk_ma2.cu:130-158);
      q, k, v = W_qkv xn + b; per head (8 x 96) weightless RMS norm of q and k, half-split RoPE
      over 48 pairs from the given cos/sin tables at positions 0..Tv-1; softmax(q k^T / sqrt(96))
      over the Tv action tokens; x += gate * (W_so attn + b_so) (mk_ma2.cu:293-394);
      qc = W_cq xn + b, weightless RMS per head; softmax(qc kctx^T / sqrt(96)) over the Lk context
      keys (already projected and normed, as the reference receives them); x += gate *
      (W_co attn + b_co) (mk_ma2.cu:397-539);
      h = silu(W_g xn + b_g) * (W_u xn + b_u); x += gate * (W_d h + b_d) (mk_ma2.cu:543-550);
  * final: xn = rms(x) (1 + scale_f) + shift_f, v = W_aout xn + b_aout on a < adim (mk_ma2.cu:
    558-575).

The reference's own CPU path (HF remote code of allenai/MolmoAct2-SO100_101) is absent. Its
modulation MLP cannot be inspected, so modulations are an INPUT here exactly as they are to the
reference kernel; the synthetic generator stands in with low-rank linear maps of a sin-cos time
embedding (flagged as a stand-in). Agreement with the reference's CUDA kernel
(src/molmoact2/mk_ma2.cu compiled into oracle/_ref) is checked by tests/test_ref_pin.py on a GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

D, H, HD, F = 768, 8, 96, 3072


@dataclass
class Ma2Case:
    L: int
    T: int   # valid action tokens (Tv)
    AD: int  # action dim of the buffers (32)
    adim: int  # valid action dims
    Lk: int
    B: int
    num_steps: int
    w: dict = field(default_factory=dict)
    kctx: torch.Tensor = None  # [B][L][Lk][768]
    vctx: torch.Tensor = None
    noise: torch.Tensor = None  # [B][T][AD], dims >= adim zero
    mods: torch.Tensor = None   # [N][L][3][3][768] (scale, shift, gate)
    mod_final: torch.Tensor = None  # [N][2][768] (scale, shift)
    rope_cos: torch.Tensor = None   # [T][48]
    rope_sin: torch.Tensor = None


def time_embedding(t: torch.Tensor, dim=D) -> torch.Tensor:
    """sin | cos of t over log-spaced periods in [4e-3, 4] (float64 -> fp32)."""
    frac = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = 4e-3 * (4.0 / 4e-3) ** frac
    arg = (2 * math.pi / period)[None, :] * t.to(torch.float64)[:, None]
    return torch.cat([torch.sin(arg), torch.cos(arg)], dim=1).to(torch.float32)


def rope_tables(T: int, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))
    ang = torch.outer(torch.arange(T, dtype=torch.float32), inv)
    return ang.cos(), ang.sin()


def make_case(seed=1, L=36, T=30, AD=32, adim=6, Lk=493, B=1, num_steps=10, rank=16) -> Ma2Case:
    """Generation order (torch.manual_seed-style generator, CPU fp32): per layer w_qkv, b_qkv,
    w_so, b_so, w_cq, b_cq, w_co, b_co, w_gate, b_gate, w_up, b_up, w_down, b_down; then w_ain,
    b_ain, w_aout, b_aout; modulation stand-in U [L][9*768][rank], V [rank][768], Uf [2*768][rank];
    then per observation kctx [L][Lk][768], vctx, noise [T][AD]. Weights N(0, 0.02), biases
    0.02 N(0, 1), context and noise N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    W = lambda *s: torch.randn(*s, generator=g) * 0.02
    c = Ma2Case(L=L, T=T, AD=AD, adim=adim, Lk=Lk, B=B, num_steps=num_steps)
    names = [("w_qkv", (3 * D, D)), ("b_qkv", (3 * D,)), ("w_so", (D, D)), ("b_so", (D,)), ("w_cq", (D, D)),
             ("b_cq", (D,)), ("w_co", (D, D)), ("b_co", (D,)), ("w_gate", (F, D)), ("b_gate", (F,)),
             ("w_up", (F, D)), ("b_up", (F,)), ("w_down", (D, F)), ("b_down", (D,))]
    per = {n: [] for n, _ in names}
    for _ in range(L):
        for n, shp in names:
            per[n].append(W(*shp))
    c.w = {n: torch.stack(v).contiguous() for n, v in per.items()}
    c.w["w_ain"], c.w["b_ain"] = W(D, AD), W(D)
    c.w["w_aout"], c.w["b_aout"] = W(AD, D), W(AD)
    U = torch.randn(L, 9 * D, rank, generator=g) * 0.02
    V = torch.randn(rank, D, generator=g) * 0.02 * 10
    Uf = torch.randn(2 * D, rank, generator=g) * 0.02
    t = torch.tensor([i / num_steps for i in range(num_steps)], dtype=torch.float32)
    z = time_embedding(t) @ V.T  # [N][rank]
    c.mods = torch.einsum("lor,nr->nlo", U, z).reshape(num_steps, L, 3, 3, D).contiguous()
    c.mod_final = (z @ Uf.T).reshape(num_steps, 2, D).contiguous()
    ks, vs, ns = [], [], []
    for _ in range(B):
        ks.append(torch.randn(L, Lk, D, generator=g))
        vs.append(torch.randn(L, Lk, D, generator=g))
        n = torch.randn(T, AD, generator=g)
        n[:, adim:] = 0
        ns.append(n)
    c.kctx, c.vctx, c.noise = torch.stack(ks), torch.stack(vs), torch.stack(ns)
    c.rope_cos, c.rope_sin = rope_tables(T)
    return c


def _rms(x, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def _mod(x, scale, shift):
    return _rms(x) * (1 + scale) + shift


def flow(c: Ma2Case, weight_dtype=torch.float32, max_obs=None) -> torch.Tensor:
    """Runs the N-step loop per observation; returns x [B][T][AD] fp32 (dims >= adim keep noise)."""
    rw = lambda n: c.w[n].to(weight_dtype).float()
    wq, wso, wcq, wco, wg, wu, wd = (rw(n) for n in ("w_qkv", "w_so", "w_cq", "w_co", "w_gate", "w_up", "w_down"))
    b = {n: c.w[n].float() for n in c.w if n.startswith("b_")}
    T, L, N = c.T, c.L, c.num_steps
    cos, sin = c.rope_cos[:T], c.rope_sin[:T]
    scl = 1.0 / math.sqrt(HD)
    outs = []
    for ob in range(c.B if max_obs is None else min(c.B, max_obs)):
        x_t = c.noise[ob].float().clone()
        kc, vc = c.kctx[ob].float(), c.vctx[ob].float()
        for s in range(N):
            x = x_t @ c.w["w_ain"].float().T + b["b_ain"]
            for l in range(L):
                m = c.mods[s, l]
                xn = _mod(x, m[0, 0], m[0, 1])
                qkv = xn @ wq[l].T + b["b_qkv"][l]
                q, k, v = (qkv[:, i * D:(i + 1) * D].view(T, H, HD) for i in range(3))
                q, k = _rms(q), _rms(k)

                def rope(z):
                    z1, z2 = z[..., :48], z[..., 48:]
                    return torch.cat([z1 * cos[:, None] - z2 * sin[:, None], z1 * sin[:, None] + z2 * cos[:, None]], -1)
                q, k = rope(q), rope(k)
                p = torch.softmax(torch.einsum("thd,jhd->htj", q, k) * scl, -1)
                att = torch.einsum("htj,jhd->thd", p, v).reshape(T, D)
                x = x + m[0, 2] * (att @ wso[l].T + b["b_so"][l])
                xn = _mod(x, m[1, 0], m[1, 1])
                qc = _rms((xn @ wcq[l].T + b["b_cq"][l]).view(T, H, HD))
                kh, vh = kc[l].view(-1, H, HD), vc[l].view(-1, H, HD)
                p = torch.softmax(torch.einsum("thd,jhd->htj", qc, kh) * scl, -1)
                att = torch.einsum("htj,jhd->thd", p, vh).reshape(T, D)
                x = x + m[1, 2] * (att @ wco[l].T + b["b_co"][l])
                xn = _mod(x, m[2, 0], m[2, 1])
                h = torch.nn.functional.silu(xn @ wg[l].T + b["b_gate"][l]) * (xn @ wu[l].T + b["b_up"][l])
                x = x + m[2, 2] * (h @ wd[l].T + b["b_down"][l])
            xf = _mod(x, c.mod_final[s, 0], c.mod_final[s, 1])
            v = xf @ c.w["w_aout"].float().T + b["b_aout"]
            v[:, c.adim:] = 0
            x_t = x_t + (1.0 / N) * v
        outs.append(x_t)
    return torch.stack(outs)
