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
