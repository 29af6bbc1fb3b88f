"""Runs the reference project's own CUDA kernels (built by oracle/build_ref.py into oracle/_ref)
on seeded synthetic inputs, packed the way the reference's host code packs them:
src/pi05/hybrid_model.py:76-133 (RoPE-pair interleave of W1, gate/up interleave of W2, per-row
FP8 E4M3 quantisation with scale amax/448) and benchmarks/molmoact2/eval_numerics.py:77-133.
Used by tests/test_ref_pin.py and tests/golden/make_ref_golden.py (GPU only)."""
import torch

from oracle import molmoact2_oracle as M
from oracle import pi05_oracle as O

D5, NL5, T5, AD5, F5 = 1024, 18, 16, 32, 4096
PI05_PIN = dict(seed=31, L=NL5, T=10, AD=AD5, Lp=300, B=1, num_steps=10)
MA2_PIN = dict(seed=41, L=36, T=30, AD=32, adim=6, Lk=493, B=1, num_steps=10)


def load(name):
    from oracle.build_ref import load_ref
    return load_ref(name)


def quant(w):
    """Per-output-row FP8 E4M3 with scale amax/448 (src/pi05/hybrid_model.py:105-110)."""
    s = w.float().abs().amax(dim=-1).clamp(min=1e-8) / 448.0
    q = (w.float() / s[..., None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, s


def pi05_dequantised_case(c):
    """The case with its GEMM weights replaced by their FP8-dequantised values and the prefix
    KV rounded to fp16, i.e. exactly what the reference kernel computes with."""
    c2 = O.Pi05Case(**{**c.__dict__})
    c2.w = dict(c.w)
    for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
        q, s = quant(c.w[n])
        c2.w[n] = q.float() * s[..., None]
    c2.k, c2.v = c.k.half().float(), c.v.half().float()
    return c2


def prepare_pi05_ref(ext, c):
    """Packs case c for the reference pi0.5 megakernel; returns (launch, read): launch() runs the
    kernel once from the initial noise, read() returns x_t [Tv][32]."""
    args, xt_d, x0 = pi05_ref_args(c)

    def launch():
        xt_d.copy_(x0)
        ext.launch(*args)

    return launch, lambda: xt_d[:c.T].cpu()


def pi05_ref_args(c):
    """The reference pi0.5 launch() arguments for case c (device tensors, packed like
    src/pi05/hybrid_model.py:76-133), its x_t tensor and x_t's initial value."""
    Tv, Lp, N = c.T, c.Lp, c.num_steps
    dev = torch.device("cuda")
    # quantise per original row (row permutations commute with per-row scales)
    deq = {}
    qs = {}
    for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
        q, s = quant(c.w[n])
        qs[n] = (q, s)
        deq[n] = q.float() * s[..., None]
    p_ = torch.arange(1024)
    qsrc = torch.stack([p_ // 128 * 256 + p_ % 128, p_ // 128 * 256 + p_ % 128 + 128], 1).reshape(-1)
    jk = torch.arange(128)
    ksrc = torch.stack([jk, jk + 128], 1).reshape(-1)

    qs = {n: (q.float(), s) for n, (q, s) in qs.items()}  # exact fp8 values, permuted in fp32

    def pack_rows(parts):
        q = torch.cat([x[0] for x in parts], 1).to(torch.float8_e4m3fn)
        s = torch.cat([x[1] for x in parts], 1)
        return q.view(torch.uint8).contiguous().to(dev), s.float().contiguous().to(dev)

    w1, s1 = pack_rows([(qs["wq"][0][:, qsrc], qs["wq"][1][:, qsrc]), (qs["wk"][0][:, ksrc], qs["wk"][1][:, ksrc]),
                        qs["wv"]])
    wo, so_ = pack_rows([qs["wo"]])
    gq = torch.stack([qs["w_gate"][0], qs["w_up"][0]], 2).reshape(NL5, 2 * F5, D5)
    gs = torch.stack([qs["w_gate"][1], qs["w_up"][1]], 2).reshape(NL5, 2 * F5)
    w2, s2 = gq.to(torch.float8_e4m3fn).view(torch.uint8).contiguous().to(dev), gs.float().contiguous().to(dev)
    w3, s3 = pack_rows([qs["w_down"]])
    mods, modf = O.modulations(c.w, NL5, N)
    cos, sin = O.rope_tables(Lp, T5)
    Lmax = (Lp + T5 + 15) // 16 * 16
    kc = torch.zeros(NL5, Lmax, 256, dtype=torch.float16)
    vt = torch.zeros(NL5, 256, Lmax, dtype=torch.float16)
    kc[:, :Lp] = c.k[0].half()
    vt[:, :, :Lp] = c.v[0].half().transpose(1, 2)
    x_t = torch.zeros(T5, AD5)
    x_t[:Tv] = c.noise[0]
    f32 = lambda *s: torch.zeros(*s, dtype=torch.float32, device=dev)
    f16 = lambda *s: torch.zeros(*s, dtype=torch.float16, device=dev)
    xt_d = x_t.to(dev)
    empty = torch.empty(0, dtype=torch.bfloat16, device=dev)
    x0 = xt_d.clone()

    args = [w1, wo, w2, w3, s1, so_, s2, s3, mods.contiguous().to(dev), modf.contiguous().to(dev),
                   cos.contiguous().to(dev), sin.contiguous().to(dev), c.w["ain_w"].float().contiguous().to(dev),
                   c.w["ain_b"].float().to(dev), c.w["aout_w"].float().contiguous().to(dev), c.w["aout_b"].float().to(dev),
                   empty, empty, 0, kc.to(dev), vt.to(dev), Lp, Lmax, N, Tv, xt_d, f32(2 * T5, D5), f32(4, T5, D5),
                   torch.zeros(16, dtype=torch.int64, device=dev), f16(T5, D5), f16(T5, 2048), f16(T5, 2048),
                   f16(T5, F5), f32(8, T5, Lmax), f16(8, T5, Lmax), 148, 256]  # device arguments, built once
    return args, xt_d, x0


def run_pi05_ref(ext, c):
    """Reference pi0.5 megakernel (18 layers, <= 16 tokens) on case c; returns x_t [Tv][32]."""
    launch, read = prepare_pi05_ref(ext, c)
    launch()
    torch.cuda.synchronize()
    return read()


def prepare_ma2_ref(ext, c):
    """Packs case c for the reference MolmoAct2 megakernel; returns (launch, read)."""
    args, xt_d, x0 = ma2_ref_args(c)

    def launch():
        xt_d.copy_(x0)
        ext.launch(*args)

    return launch, lambda: xt_d[:c.T].cpu()


def ma2_ref_args(c):
    """The reference MolmoAct2 launch() arguments for case c
    (benchmarks/molmoact2/eval_numerics.py:77-150 packing), its x_t tensor and initial value."""
    NL, T, D, F, AD = 36, 32, 768, 3072, 32
    dev = torch.device("cuda")
    bf = lambda t: t.to(torch.bfloat16).contiguous().to(dev)
    fp = lambda t: t.float().contiguous().to(dev)
    w_gu = torch.stack([c.w["w_gate"], c.w["w_up"]], 2).reshape(NL, 2 * F, D)
    b_gu = torch.stack([c.w["b_gate"], c.w["b_up"]], 2).reshape(NL, 2 * F)
    ws = [bf(c.w["w_qkv"]), bf(c.w["w_so"]), bf(c.w["w_cq"]), bf(c.w["w_co"]), bf(w_gu), bf(c.w["w_down"])]
    bs = [fp(c.w["b_qkv"]), fp(c.w["b_so"]), fp(c.w["b_cq"]), fp(c.w["b_co"]), fp(b_gu), fp(c.w["b_down"])]
    Lk = c.Lk
    Lkmax = (Lk + 15) // 16 * 16
    kctx = torch.zeros(NL, Lkmax, D)
    vtctx = torch.zeros(NL, D, Lkmax)
    kctx[:, :Lk] = c.kctx[0]
    vtctx[:, :, :Lk] = c.vctx[0].transpose(1, 2)
    cosf = torch.zeros(T, 48)
    sinf = torch.zeros(T, 48)
    cosf[:c.T], sinf[:c.T] = c.rope_cos, c.rope_sin
    x_t = torch.zeros(T, AD)
    x_t[:c.T] = c.noise[0]
    xt_d = x_t.to(dev)
    bufs = [torch.zeros(T, D, dtype=torch.bfloat16, device=dev) for _ in range(8)]
    bufs.append(torch.zeros(T, F, dtype=torch.bfloat16, device=dev))
    x0 = xt_d.clone()

    args = [ws, bs, fp(c.mods), fp(c.mod_final), fp(cosf), fp(sinf), fp(c.w["w_ain"]), fp(c.w["b_ain"]),
                   bf(c.w["w_aout"]), fp(c.w["b_aout"]), bf(kctx), bf(vtctx), Lk, Lkmax, c.T, c.adim, c.num_steps, xt_d,
                   torch.zeros(T, D, device=dev), torch.zeros(3, T, D, device=dev),
                   torch.zeros(16, dtype=torch.int64, device=dev), bufs, torch.zeros(8, T, Lkmax, device=dev),
                   torch.zeros(8, T, Lkmax, dtype=torch.bfloat16, device=dev), 148, 256]  # device arguments, built once
    return args, xt_d, x0


def run_ma2_ref(ext, c):
    """Reference MolmoAct2 megakernel (36 blocks, 32 tokens) on case c; returns x_t [Tv][32]."""
    launch, read = prepare_ma2_ref(ext, c)
    launch()
    torch.cuda.synchronize()
    return read()


def ma2_bf16_case(c):
    """The case as the reference MolmoAct2 kernel sees it: bf16 action-out weights and context."""
    c2 = M.Ma2Case(**{**c.__dict__})
    c2.w = {**c.w, "w_aout": c.w["w_aout"].to(torch.bfloat16).float()}
    c2.kctx, c2.vctx = c.kctx.to(torch.bfloat16).float(), c.vctx.to(torch.bfloat16).float()
    return c2
