"""CPU checks of the reference-launch drop-in's weight handling (flashact_b200/compat.py): the
reference packs pi0.5's FP8 codes and row scales in its own row order (src/pi05/hybrid_model.py:
100-110: Q / K rotary pairs interleaved, gate / up interleaved); compat must put both back in model
row order exactly, since the engine streams the codes as they are."""
import torch

from oracle import quant as Q


def _pack_like_reference(w):
    """The reference's packing of per-row FP8 codes + scales (the same permutations
    tests/ref_runner.py applies before launching the reference kernel)."""
    p_ = torch.arange(1024)
    qsrc = torch.stack([p_ // 128 * 256 + p_ % 128, p_ // 128 * 256 + p_ % 128 + 128], 1).reshape(-1)
    jk = torch.arange(128)
    ksrc = torch.stack([jk, jk + 128], 1).reshape(-1)
    q = {n: Q.fp8_rowwise(w[n]) for n in w}
    w1 = torch.cat([q["wq"][0][:, qsrc], q["wk"][0][:, ksrc], q["wv"][0]], 1)
    s1 = torch.cat([q["wq"][1][:, qsrc], q["wk"][1][:, ksrc], q["wv"][1]], 1)
    L = w["wq"].shape[0]
    w2 = torch.stack([q["w_gate"][0], q["w_up"][0]], 2).reshape(L, 2 * 4096, 1024)
    s2 = torch.stack([q["w_gate"][1], q["w_up"][1]], 2).reshape(L, 2 * 4096)
    return q, (w1, q["wo"][0], w2, q["w_down"][0], s1, q["wo"][1], s2, q["w_down"][1])


def test_compat_fp8_weights_back_in_model_order():
    from flashact_b200.compat import _pi05_weights
    g = torch.Generator().manual_seed(3)
    L = 1
    shapes = {"wq": (2048, 1024), "wk": (256, 1024), "wv": (256, 1024), "wo": (1024, 2048),
              "w_gate": (4096, 1024), "w_up": (4096, 1024), "w_down": (1024, 4096)}
    w = {n: torch.randn(L, *s, generator=g) * 0.02 for n, s in shapes.items()}
    q, packed = _pack_like_reference(w)
    extra = [torch.zeros(1024, 32), torch.zeros(1024), torch.zeros(32, 1024), torch.zeros(32)]
    weights, scales = _pi05_weights(*packed, *extra)
    for n in shapes:
        assert torch.equal(weights[n], q[n][0]), n
        assert torch.equal(scales[n], q[n][1]), n
        assert weights[n].is_contiguous() and scales[n].is_contiguous(), n
