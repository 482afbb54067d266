"""GPU parity of the MoE sublayer (UocrMoE, the reference's MoE surface) through the C ABI.

Bars (the reference's own, tests/test_decoder_int8.py:742-893): against the float64 evaluation
of the exact layer math -- fed the bit-exact fp32 routing, so a near-tie cannot move an expert
between the two sides -- cosine >= 0.99999 and max-abs/max-ref <= 1e-4, for bf16 and for int8
(the int8 math is q * scale, exact). Routing ids and weights are bit-exact with the oracle.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from golden import reference_inputs as ri

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


def small_cfg(uocr, int8: bool):
    return uocr.MoEConfig(hidden_size=256, moe_intermediate_size=128, n_routed_experts=8, n_shared_experts=2,
                          num_experts_per_tok=6, int8_experts=int8)


def declared(state):
    """The reference's declared form of a bare MoE's state (tests/test_decoder_int8.py:666-675):
    shared-expert projections K-blocked [K/16, N, 16]."""
    out = {}
    for name, w in state.items():
        if name.startswith("shared_experts."):
            w = w.reshape(w.shape[0], -1, 16).permute(1, 0, 2).contiguous()
        out[name] = w
    return out


def oracle_weights(oracle, state, int8):
    from test_oracle import weights_from_state

    return weights_from_state(oracle, state, int8)


@pytest.mark.parametrize("seed", [1, 2, 19])
@pytest.mark.parametrize("int8", [False, True])
def test_small_layer_matches_reference_fp64(uocr, oracle, seed, int8):
    """The reference's float64 MoE outputs (fixture) for its small decoder config."""
    g = np.load(GOLDEN / "moe_layer.npz")
    orig, q = ri.moe_weights(ri.SMALL_MOE, seed)
    state = q if int8 else orig
    moe = uocr.UocrMoE(small_cfg(uocr, int8)).load_state_dict(declared(state))
    x = g[f"seed{seed}_x"]
    got = moe.decode_rows(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ref = g[f"seed{seed}_ref_int8" if int8 else f"seed{seed}_ref_bf16"]
    for i in range(x.shape[0]):
        assert oracle.cosine(got[i], ref[i]) >= 0.99999
    assert oracle.rel_err(got, ref) <= 1e-4


@pytest.mark.parametrize("int8", [False, True])
def test_small_layer_rows_are_batch_independent(uocr, oracle, int8):
    orig, q = ri.moe_weights(ri.SMALL_MOE, 19)
    moe = uocr.UocrMoE(small_cfg(uocr, int8)).load_state_dict(q if int8 else orig)
    x = torch.from_numpy(np.random.default_rng(23).standard_normal((8, 256)).astype(np.float32)).to(DEV)
    rows = moe.decode_rows(x)
    for i in range(8):
        assert torch.equal(rows[i : i + 1], moe.decode_rows(x[i : i + 1])), i
    for b in (2, 5):
        assert torch.equal(rows[:b], moe.decode_rows(x[:b]))


def full_layer(oracle, int8: bool, seed: int):
    cfg = oracle.MoEConfig()
    return cfg, oracle.synth_weights(cfg, seed, int8=int8)


def to_state(w, cfg, int8):
    def b(a):
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)

    st = {
        "gate.gate_score.weight": b(w.router),
        "shared_experts.gate_proj.weight": b(w.shared_gate),
        "shared_experts.up_proj.weight": b(w.shared_up),
        "shared_experts.down_proj.weight": b(w.shared_down),
    }
    for name in ("gate", "up", "down"):
        a = getattr(w, name)
        st[f"experts.{name}_proj"] = torch.from_numpy(a) if int8 else b(a)
        if int8:
            st[f"experts.{name}_proj_scales"] = torch.from_numpy(getattr(w, f"{name}_scales"))
    return st


@pytest.mark.parametrize("int8", [False, True])
def test_full_size_decode_layer(uocr, oracle, int8):
    """hidden 1280, 64 experts top-6 + 2 shared, I = 896 at B = 1, 4, 8."""
    cfg, w = full_layer(oracle, int8, 0)
    moe = uocr.UocrMoE(uocr.MoEConfig(int8_experts=int8)).load_state_dict(to_state(w, cfg, int8))
    x_all = oracle.synth_hidden(8, cfg.hidden, 0)
    for B in (1, 4, 8):
        x = x_all[:B]
        ids = torch.empty((B, 6), dtype=torch.int32, device=DEV)
        wts = torch.empty((B, 6), dtype=torch.float32, device=DEV)
        got = moe.decode_rows(torch.from_numpy(x).to(DEV), ids=ids, wts=wts).cpu().numpy()
        r = oracle.route_fp32(x, w.router, None, 6)
        assert np.array_equal(ids.cpu().numpy(), r.ids)
        assert np.array_equal(wts.cpu().numpy().view(np.uint32), r.weights.view(np.uint32))
        ref = oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights)
        for i in range(B):
            assert oracle.cosine(got[i], ref[i]) >= 0.99999, (B, i)
        assert oracle.rel_err(got, ref) <= 1e-4, B
        # the north-star bar against the fp32 reference path
        assert np.max(np.abs(got - ref)) <= 2e-2 and oracle.rel_l2(got, ref) <= 1e-2


def test_decode_status_clean_and_repeatable(uocr, oracle):
    """The self-resetting control block: many calls in a row give identical bits and leave
    the device status word clear (no bounded wait expired)."""
    import ctypes

    orig, _ = ri.moe_weights(ri.SMALL_MOE, 2)
    moe = uocr.UocrMoE(small_cfg(uocr, False)).load_state_dict(orig)
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((6, 256)).astype(np.float32)).to(DEV)
    first = moe.decode_rows(x).clone()
    for _ in range(20):
        assert torch.equal(moe.decode_rows(x), first)
    lib = uocr.load()
    rc = lib.uocr_moe_device_status(moe.workspace(6).data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.uocr_last_error().decode()
