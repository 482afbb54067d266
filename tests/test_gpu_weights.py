"""GPU: a layer loaded from per-expert checkpoint names (``UocrMoE.from_checkpoint``) computes the
same bits as the same weights loaded as stacks, bf16 and int8, decode and prefill."""

from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _checkpoint(state: dict, layer: int) -> dict:
    """The stacked state written back out under the model file's per-expert names."""
    ck = {f"model.layers.{layer}.mlp.gate.weight": state["gate.gate_score.weight"]}
    for p in ("gate_proj", "up_proj", "down_proj"):
        ck[f"model.layers.{layer}.mlp.shared_experts.{p}.weight"] = state[f"shared_experts.{p}.weight"]
        for e in range(state[f"experts.{p}"].shape[0]):
            ck[f"model.layers.{layer}.mlp.experts.{e}.{p}.weight"] = state[f"experts.{p}"][e].clone()
            if f"experts.{p}_scales" in state:
                ck[f"model.layers.{layer}.mlp.experts.{e}.{p}.weight_scales"] = state[f"experts.{p}_scales"][e].clone()
    ck["model.norm.weight"] = torch.ones(8, dtype=torch.bfloat16)  # a non-MoE tensor passes by
    return ck


@pytest.mark.parametrize("int8", [False, True])
def test_per_expert_checkpoint_equals_the_stacked_state(uocr, int8):
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    cfg = uocr.MoEConfig(int8_experts=int8)
    state = synth.layer_state(cfg, 77 + int(int8), device="cpu")
    stacked = uocr.UocrMoE(cfg, device=DEV).load_state_dict(state)
    loaded = uocr.UocrMoE.from_checkpoint(_checkpoint(state, 4), 4, device=DEV)
    assert loaded.config.int8_experts is int8
    x = synth.hidden_states(8, 1280, 9, device=DEV)
    assert torch.equal(loaded.decode_rows(x), stacked.decode_rows(x))
    xp = synth.hidden_states(300, 1280, 10, device=DEV)
    assert torch.equal(loaded.prefill(xp), stacked.prefill(xp))


@pytest.mark.parametrize("int8", [False, True])
def test_safetensors_file_equals_the_stacked_state(uocr, int8, tmp_path):
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    ck = importlib.import_module("unlimited-ocr-max_b200.checkpoint")
    cfg = uocr.MoEConfig(int8_experts=int8)
    state = synth.layer_state(cfg, 91 + int(int8), device="cpu")
    path = tmp_path / "model.safetensors"
    ck.write_safetensors(path, _checkpoint(state, 3), {"format": "pt"})
    stacked = uocr.UocrMoE(cfg, device=DEV).load_state_dict(state)
    loaded = ck.load_moe_layer(path, 3, device=DEV)
    assert loaded.config.int8_experts is int8
    x = synth.hidden_states(8, 1280, 12, device=DEV)
    assert torch.equal(loaded.decode_rows(x), stacked.decode_rows(x))


def test_quantise_on_load_equals_the_int8_checkpoint(uocr, tmp_path):
    """A bf16 file loaded with ``quantize="int8"`` computes the bits of the same layer loaded from
    the int8 checkpoint that the pinned oracle quantiser makes of it."""
    from oracle import moe_oracle as oracle

    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    ck = importlib.import_module("unlimited-ocr-max_b200.checkpoint")
    state = synth.layer_state(uocr.MoEConfig(), 93, device="cpu")
    path = tmp_path / "model.safetensors"
    ck.write_safetensors(path, _checkpoint(state, 2), {"format": "pt"})
    q8 = dict(state)
    for p in ("gate_proj", "up_proj", "down_proj"):
        q, s = oracle.quantize_per_group(state[f"experts.{p}"].float().numpy())
        q8[f"experts.{p}"], q8[f"experts.{p}_scales"] = torch.from_numpy(q), torch.from_numpy(s)
    want = uocr.UocrMoE(uocr.MoEConfig(int8_experts=True), device=DEV).load_state_dict(q8)
    got = ck.load_moe_layer(path, 2, device=DEV, quantize="int8")
    assert got.config.int8_experts is True
    x = synth.hidden_states(8, 1280, 13, device=DEV)
    assert torch.equal(got.decode_rows(x), want.decode_rows(x))
    xp = synth.hidden_states(300, 1280, 14, device=DEV)
    assert torch.equal(got.prefill(xp), want.prefill(xp))
