"""Checkpoint loading by openpi key names (flashact_b200.pi05.weights_from_openpi), CPU only: a
synthetic two-layer state dict written as .safetensors and as a torch checkpoint must come back
as the engine's weight dict, per-layer tensors stacked in layer order."""
import torch

from flashact_b200.pi05 import OPENPI_EXPERT, weights_from_openpi


def _state_dict(L=2, AD=32):
    g = torch.Generator().manual_seed(1)
    r = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)
    sd = {}
    for i in range(L):
        p = f"{OPENPI_EXPERT}layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = r(2048, 1024)
        sd[p + "self_attn.k_proj.weight"] = r(256, 1024)
        sd[p + "self_attn.v_proj.weight"] = r(256, 1024)
        sd[p + "self_attn.o_proj.weight"] = r(1024, 2048)
        sd[p + "mlp.gate_proj.weight"] = r(4096, 1024)
        sd[p + "mlp.up_proj.weight"] = r(4096, 1024)
        sd[p + "mlp.down_proj.weight"] = r(1024, 4096)
        sd[p + "input_layernorm.dense.weight"] = r(3072, 1024)
        sd[p + "input_layernorm.dense.bias"] = r(3072)
        sd[p + "post_attention_layernorm.dense.weight"] = r(3072, 1024)
        sd[p + "post_attention_layernorm.dense.bias"] = r(3072)
    sd[OPENPI_EXPERT + "norm.dense.weight"] = r(3072, 1024)
    sd[OPENPI_EXPERT + "norm.dense.bias"] = r(3072)
    for n in ("time_mlp_in", "time_mlp_out"):
        sd[n + ".weight"], sd[n + ".bias"] = r(1024, 1024), r(1024)
    sd["action_in_proj.weight"], sd["action_in_proj.bias"] = r(1024, AD), r(1024)
    sd["action_out_proj.weight"], sd["action_out_proj.bias"] = r(AD, 1024), r(AD)
    return sd


def _check(w, sd, L):
    from flashact_b200._capi import PI05_WEIGHT_FIELDS
    assert set(w) == set(PI05_WEIGHT_FIELDS)
    assert w["wq"].shape == (L, 2048, 1024) and w["w_down"].shape == (L, 1024, 4096)
    assert torch.equal(w["wk"][1], sd[f"{OPENPI_EXPERT}layers.1.self_attn.k_proj.weight"])
    assert torch.equal(w["ln_post_b"][0], sd[f"{OPENPI_EXPERT}layers.0.post_attention_layernorm.dense.bias"])
    assert torch.equal(w["aout_w"], sd["action_out_proj.weight"]) and w["wq"].dtype == torch.bfloat16


def test_from_safetensors_and_torch_checkpoint(tmp_path):
    from safetensors.torch import save_file
    sd = _state_dict()
    save_file(sd, str(tmp_path / "model.safetensors"))
    _check(weights_from_openpi(tmp_path / "model.safetensors", num_layers=2), sd, 2)
    torch.save(sd, str(tmp_path / "model.pt"))
    _check(weights_from_openpi(str(tmp_path / "model.pt"), num_layers=2), sd, 2)
    _check(weights_from_openpi(sd, num_layers=2), sd, 2)
