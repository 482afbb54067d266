"""Checkpoint -> stacked MoE weights (``weights.py``), on the CPU: expert stacking, int8
detection, half-quantised files, one layer's selection under UocrMoE's names.

Mirrors the reference's model-free adapter tests (tests/test_weight_adapters.py:86-228 of
kthr/unlimited-ocr-max): tiny shapes, 4 experts, and every expert tensor filled with its own
expert index so that a misordered stack cannot pass.
"""

from __future__ import annotations

import importlib

import pytest
import torch

W = importlib.import_module("unlimited-ocr-max_b200.weights")
WeightMappingError = W.WeightMappingError

EXPERTS = 4
N, K = 6, 256  # two groups of 128
GROUPS = K // 128
PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def _expert(index: int, dtype: torch.dtype) -> torch.Tensor:
    return torch.full((N, K), index, dtype=dtype)


def _scales(index: int) -> torch.Tensor:
    return torch.full((N, GROUPS), float(index), dtype=torch.float32)


def bf16_checkpoint(layers=(1,), experts=EXPERTS) -> dict:
    out = {"model.norm.weight": torch.ones(N, dtype=torch.bfloat16)}
    for layer in layers:
        for e in range(experts):
            for p in PROJECTIONS:
                out[f"model.layers.{layer}.mlp.experts.{e}.{p}.weight"] = _expert(e, torch.bfloat16)
    return out


def int8_checkpoint(layers=(1,), experts=EXPERTS) -> dict:
    out = {"model.norm.weight": torch.ones(N, dtype=torch.bfloat16)}
    for layer in layers:
        for e in range(experts):
            for p in PROJECTIONS:
                stem = f"model.layers.{layer}.mlp.experts.{e}.{p}"
                out[f"{stem}.weight"] = _expert(e, torch.int8)
                out[f"{stem}.weight_scales"] = _scales(e)
    return out


def renamed(ck: dict) -> dict:
    return {k.removeprefix("model."): v for k, v in ck.items()}


# ---- stacking ---------------------------------------------------------------------------------


def test_bf16_stacking_puts_expert_j_at_slice_j():
    out = W.stack_expert_weights(renamed(bf16_checkpoint()), num_experts=EXPERTS)
    assert set(out) == {"norm.weight", *(f"layers.1.mlp.experts.{p}" for p in PROJECTIONS)}
    for p in PROJECTIONS:
        s = out[f"layers.1.mlp.experts.{p}"]
        assert (tuple(s.shape), s.dtype) == ((EXPERTS, N, K), torch.bfloat16)
        for e in range(EXPERTS):
            assert torch.all(s[e] == e)


def test_int8_stacking_groups_the_scales_into_their_own_stack():
    out = W.stack_expert_weights(renamed(int8_checkpoint(layers=(1, 2))), num_experts=EXPERTS)
    expected = {"norm.weight"}
    for layer in (1, 2):
        for p in PROJECTIONS:
            expected |= {f"layers.{layer}.mlp.experts.{p}", f"layers.{layer}.mlp.experts.{p}_scales"}
    assert set(out) == expected
    for layer in (1, 2):
        for p in PROJECTIONS:
            w, s = out[f"layers.{layer}.mlp.experts.{p}"], out[f"layers.{layer}.mlp.experts.{p}_scales"]
            assert (tuple(w.shape), w.dtype) == ((EXPERTS, N, K), torch.int8)
            assert (tuple(s.shape), s.dtype) == ((EXPERTS, N, GROUPS), torch.float32)
            for e in range(EXPERTS):
                assert torch.all(w[e] == e) and torch.all(s[e] == float(e))


def test_stacking_refuses_experts_that_disagree_on_dtype():
    state = renamed(bf16_checkpoint())
    state["layers.1.mlp.experts.2.up_proj.weight"] = _expert(2, torch.int8)
    with pytest.raises(WeightMappingError, match=r"up_proj: the experts disagree on dtype: \['bfloat16', 'int8'\]"):
        W.stack_expert_weights(state, num_experts=EXPERTS)


def test_stacking_refuses_experts_that_disagree_on_shape_and_names_the_stack():
    state = renamed(bf16_checkpoint())
    state["layers.1.mlp.experts.2.up_proj.weight"] = torch.zeros((N, K // 2), dtype=torch.bfloat16)
    with pytest.raises(WeightMappingError,
                       match=rf"up_proj: the experts disagree on shape: \[\({N}, {K // 2}\), \({N}, {K}\)\]"):
        W.stack_expert_weights(state, num_experts=EXPERTS)


def test_stacking_rejects_a_gap_in_the_scales():
    state = renamed(int8_checkpoint())
    del state["layers.1.mlp.experts.2.up_proj.weight_scales"]
    with pytest.raises(WeightMappingError, match=r"up_proj_scales: expert indices must be 0\.\.n-1"):
        W.stack_expert_weights(state, num_experts=EXPERTS)


def test_stacking_rejects_a_short_scales_stack():
    state = renamed(int8_checkpoint())
    del state[f"layers.1.mlp.experts.{EXPERTS - 1}.down_proj.weight_scales"]
    with pytest.raises(WeightMappingError, match=rf"down_proj_scales: expected {EXPERTS} experts, got {EXPERTS - 1}"):
        W.stack_expert_weights(state, num_experts=EXPERTS)


@pytest.mark.parametrize("name", [
    "layers.1.mlp.experts.0.up_proj.weight_zeros",
    "layers.1.mlp.experts.0.up_proj.weight_scale_inv",
    "layers.1.mlp.experts.0.up_proj.weight_scales2",
    "layers.1.mlp.experts.0.up_proj.weight_SCALES",
    "layers.1.self_attn.q_proj.weight_scales",
])
def test_an_unknown_weight_suffix_is_never_half_matched(name):
    state = renamed(bf16_checkpoint())
    state[name] = torch.zeros(N, GROUPS)
    state["layers.1.mlp.shared_experts.up_proj.weight"] = torch.zeros(N, K)
    out = W.stack_expert_weights(state, num_experts=EXPERTS)
    assert name in out
    assert "layers.1.mlp.shared_experts.up_proj.weight" in out
    assert not any(k.startswith("layers.1.mlp.experts.up_proj_") for k in out)


# ---- detection --------------------------------------------------------------------------------


def test_a_bf16_checkpoint_is_not_int8():
    assert W.is_int8_checkpoint(bf16_checkpoint()) is False
    assert W.is_int8_checkpoint(renamed(bf16_checkpoint())) is False


def test_an_int8_checkpoint_is_int8():
    assert W.is_int8_checkpoint(int8_checkpoint(layers=(1, 2))) is True
    assert W.is_int8_checkpoint(renamed(int8_checkpoint())) is True


def test_a_checkpoint_without_experts_is_not_int8():
    assert W.is_int8_checkpoint({"model.norm.weight": torch.ones(N, dtype=torch.bfloat16)}) is False


def test_int8_weights_without_scales_are_rejected():
    ck = {k: v for k, v in int8_checkpoint().items() if not k.endswith("_scales")}
    with pytest.raises(WeightMappingError, match="int8 expert weights without weight_scales"):
        W.is_int8_checkpoint(ck)


def test_scales_for_some_experts_but_not_all_are_rejected():
    ck = int8_checkpoint()
    del ck["model.layers.1.mlp.experts.3.gate_proj.weight_scales"]
    with pytest.raises(WeightMappingError, match="half-quantized checkpoint: no weight_scales for"):
        W.is_int8_checkpoint(ck)


def test_scales_for_some_projections_but_not_all_are_rejected():
    ck = int8_checkpoint()
    for e in range(EXPERTS):
        del ck[f"model.layers.1.mlp.experts.{e}.down_proj.weight_scales"]
    with pytest.raises(WeightMappingError, match="half-quantized checkpoint: no weight_scales for"):
        W.is_int8_checkpoint(ck)


def test_scales_next_to_bf16_weights_are_rejected():
    ck = int8_checkpoint()
    ck.update(bf16_checkpoint())
    with pytest.raises(WeightMappingError, match=r"expert weights are \['bfloat16'\], not int8"):
        W.is_int8_checkpoint(ck)


def test_scales_with_no_weight_to_scale_are_rejected():
    ck = int8_checkpoint()
    del ck["model.layers.1.mlp.experts.0.gate_proj.weight"]
    with pytest.raises(WeightMappingError, match="weight_scales without an expert weight to scale"):
        W.is_int8_checkpoint(ck)


# ---- one layer under UocrMoE's names -----------------------------------------------------------


def _full_layer(layer: int, int8: bool) -> dict:
    ck = int8_checkpoint(layers=(layer, layer + 1)) if int8 else bf16_checkpoint(layers=(layer, layer + 1))
    for l in (layer, layer + 1):
        ck[f"model.layers.{l}.mlp.gate.weight"] = torch.full((EXPERTS, K), l, dtype=torch.bfloat16)
        for p in PROJECTIONS:
            ck[f"model.layers.{l}.mlp.shared_experts.{p}.weight"] = torch.full((2 * N, K), 10 + l, dtype=torch.bfloat16)
    return ck


@pytest.mark.parametrize("int8", [False, True])
def test_moe_layer_state_selects_one_layer_under_the_module_names(int8):
    state, got_int8 = W.moe_layer_state(_full_layer(3, int8), 3, num_experts=EXPERTS)
    assert got_int8 is int8
    want = {"gate.gate_score.weight", *(f"experts.{p}" for p in PROJECTIONS),
            *(f"shared_experts.{p}.weight" for p in PROJECTIONS)}
    if int8:
        want |= {f"experts.{p}_scales" for p in PROJECTIONS}
    assert set(state) == want
    assert torch.all(state["gate.gate_score.weight"] == 3)  # layer 3's router, renamed
    assert torch.all(state["shared_experts.up_proj.weight"] == 13)
    for e in range(EXPERTS):
        assert torch.all(state["experts.down_proj"][e] == e)


def test_moe_layer_state_names_a_missing_projection():
    ck = _full_layer(3, False)
    del ck["model.layers.3.mlp.shared_experts.down_proj.weight"]
    with pytest.raises(WeightMappingError, match=r"missing \['shared_experts.down_proj.weight'\]"):
        W.moe_layer_state(ck, 3, num_experts=EXPERTS)


def test_moe_layer_state_refuses_a_half_quantised_file_before_stacking():
    ck = _full_layer(3, True)
    del ck["model.layers.4.mlp.experts.1.up_proj.weight_scales"]  # another layer's: still refused
    with pytest.raises(WeightMappingError, match="half-quantized checkpoint"):
        W.moe_layer_state(ck, 3, num_experts=EXPERTS)


def test_moe_layer_state_needs_the_layer():
    with pytest.raises(WeightMappingError, match="no MoE weights for layer 9"):
        W.moe_layer_state(_full_layer(3, False), 9, num_experts=EXPERTS)


def test_router_rename_matches_the_reference_rule():
    assert W.language_weight_name("model.layers.2.mlp.gate.weight") == "layers.2.mlp.gate.gate_score.weight"
    assert W.language_weight_name("model.layers.2.mlp.experts.5.up_proj.weight") == "layers.2.mlp.experts.5.up_proj.weight"
    assert W.language_weight_name("lm_head.weight") == "lm_head.weight"


# ---- the module's constructor keywords -----------------------------------------------------------


def test_uocr_moe_takes_the_reference_constructor_keywords(uocr):
    cfg = uocr.MoEConfig()

    class FakeMaxDType:  # a MAX DType spells its name on .name
        def __init__(self, name):
            self.name = name

    for dtype, router in ((None, None), (torch.bfloat16, torch.float32), ("bfloat16", "bfloat16"),
                          (FakeMaxDType("bfloat16"), FakeMaxDType("float32"))):
        m = uocr.UocrMoE(cfg, dtype=dtype, device="cuda", norm_router_dtype=router)
        assert m.dtype == torch.bfloat16
    with pytest.raises(uocr.ConfigError, match="dtype float16"):
        uocr.UocrMoE(cfg, dtype=torch.float16, device="cuda")
    with pytest.raises(uocr.ConfigError, match="norm_router_dtype int8"):
        uocr.UocrMoE(cfg, device="cuda", norm_router_dtype="int8")
    with pytest.raises(ValueError, match="CUDA device only"):
        uocr.UocrMoE(cfg, dtype=torch.bfloat16, device="cpu")


def test_rope_tables_follow_the_rotary_formula():
    """The rotary table (decoder.py:115-123): position 0 is the identity, each column pair repeats,
    angles grow as position x theta^(-2i/dim), cos^2 + sin^2 = 1."""
    import importlib

    import numpy as np

    dl = importlib.import_module("unlimited-ocr-max_b200.decode_layer")
    cos, sin = dl.rope_tables(head_dim=128, seq_len=64, theta=10000.0)
    assert cos.shape == sin.shape == (64, 128) and cos.dtype == np.float32
    assert np.array_equal(cos[0], np.ones(128, np.float32)) and np.array_equal(sin[0], np.zeros(128, np.float32))
    assert np.array_equal(cos[:, :64], cos[:, 64:]) and np.array_equal(sin[:, :64], sin[:, 64:])
    assert np.allclose(cos ** 2 + sin ** 2, 1.0, atol=1e-6)
    ang = np.arange(64)[:, None] * (10000.0 ** (-np.arange(0, 128, 2) / 128.0))[None, :]
    assert np.allclose(cos[:, :64], np.cos(ang), atol=2e-5) and np.allclose(sin[:, :64], np.sin(ang), atol=2e-5)
