"""GPU parity of the prefill MoE (UocrMoE.prefill, the reference's MoE.__call__ with native
routing, decoder.py:606-614, 657-667) through the C ABI.

The expert products run as bf16 GEMMs (bf16 activations, fp32 accumulate), so the bar is the
north-star tolerance against the float64 evaluation of the exact layer math fed the bit-exact
fp32 routing: max-abs <= 2e-2 and relative L2 <= 1e-2 (plus a cosine floor). Routing ids and
weights are bit-exact with the oracle; the combine has a fixed order, so repeated calls are
bit-identical.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden import reference_inputs as ri
from test_gpu_moe import full_layer, small_cfg, to_state

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ABS = 2e-2
REL_L2 = 1e-2


def _check(oracle, got, ref):
    assert np.all(np.isfinite(got))
    assert np.max(np.abs(got - ref)) <= MAX_ABS, np.max(np.abs(got - ref))
    assert oracle.rel_l2(got, ref) <= REL_L2, oracle.rel_l2(got, ref)
    assert oracle.cosine(got, ref) >= 0.9999


def _small(uocr, int8, seed=19):
    orig, q = ri.moe_weights(ri.SMALL_MOE, seed)
    state = q if int8 else orig
    moe = uocr.UocrMoE(small_cfg(uocr, int8)).load_state_dict(state)
    return moe, state


def _small_oracle(oracle, state, int8):
    from test_oracle import weights_from_state

    cfg = oracle.MoEConfig(hidden=256, inter=128, n_routed=8, n_shared=2, top_k=6, group=128)
    return cfg, weights_from_state(oracle, state, int8)


@pytest.mark.parametrize("T", [1, 9, 130, 300])
@pytest.mark.parametrize("int8", [False, True])
def test_small_prefill_vs_fp64(uocr, oracle, T, int8):
    moe, state = _small(uocr, int8)
    cfg, w = _small_oracle(oracle, state, int8)
    x = oracle.synth_hidden(T, 256, 100 + T)
    ids = torch.empty((T, 6), dtype=torch.int32, device=DEV)
    wts = torch.empty((T, 6), dtype=torch.float32, device=DEV)
    got = moe.prefill(torch.from_numpy(x).to(DEV), ids=ids, wts=wts).cpu().numpy()
    r = oracle.route_fp32(x, w.router, None, 6)
    assert np.array_equal(ids.cpu().numpy(), r.ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), r.weights.view(np.uint32))
    _check(oracle, got, oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights))


def test_small_prefill_skewed_bias(uocr, oracle):
    """A logit bias that sends every token to the same six experts: two experts' groups span
    many 128-row tiles while the rest are empty (skipped groups, a ragged last tile)."""
    moe, state = _small(uocr, False, seed=2)
    cfg, w = _small_oracle(oracle, state, False)
    bias = np.zeros(8, np.float32)
    bias[[1, 2, 3, 5, 6, 7]] = 30.0
    moe.bias = torch.from_numpy(bias).to(DEV)
    T = 333
    x = oracle.synth_hidden(T, 256, 7)
    ids = torch.empty((T, 6), dtype=torch.int32, device=DEV)
    wts = torch.empty((T, 6), dtype=torch.float32, device=DEV)
    got = moe.prefill(torch.from_numpy(x).to(DEV), ids=ids, wts=wts).cpu().numpy()
    r = oracle.route_fp32(x, w.router, bias, 6)
    assert np.array_equal(ids.cpu().numpy(), r.ids)
    assert set(np.unique(r.ids)) == {1, 2, 3, 5, 6, 7}
    _check(oracle, got, oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights))


def test_prefill_repeatable_and_status_clean(uocr, oracle):
    moe, _ = _small(uocr, True, seed=1)
    x = torch.from_numpy(oracle.synth_hidden(257, 256, 3)).to(DEV)
    first = moe.prefill(x).clone()
    for _ in range(5):
        assert torch.equal(moe.prefill(x), first)
    lib = uocr.load()
    rc = lib.uocr_moe_device_status(moe.prefill_workspace(257).data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.uocr_last_error().decode()


def test_call_dispatches_by_length(uocr, oracle):
    """__call__: up to 8 rows take the decode kernels, longer inputs the prefill GEMMs."""
    moe, _ = _small(uocr, False, seed=19)
    x = torch.from_numpy(oracle.synth_hidden(40, 256, 11)).to(DEV)
    assert torch.equal(moe(x[:8]), moe.decode_rows(x[:8]))
    assert torch.equal(moe(x), moe.prefill(x))


@pytest.mark.parametrize("int8,T,biased", [(False, 4096, True), (True, 1000, False), (True, 4096, True)])
def test_full_size_prefill(uocr, oracle, int8, T, biased):
    """hidden 1280, 64 experts top-6 + 2 shared, I = 896; the bf16 case is BASELINE config 3
    (T = 4096 with an N(0, 1) logit bias skewing the expert loads). int8 at T = 1000 takes the
    single-CTA GEMMs, at T = 4096 the CTA-pair GEMMs, both after the dequant pass."""
    cfg, w = full_layer(oracle, int8, 0)
    moe = uocr.UocrMoE(uocr.MoEConfig(int8_experts=int8)).load_state_dict(to_state(w, cfg, int8))
    bias = np.random.default_rng(41).standard_normal(64).astype(np.float32) if biased else None
    if bias is not None:
        moe.bias = torch.from_numpy(bias).to(DEV)
    x = oracle.synth_hidden(T, cfg.hidden, 5)
    ids = torch.empty((T, 6), dtype=torch.int32, device=DEV)
    wts = torch.empty((T, 6), dtype=torch.float32, device=DEV)
    got = moe.prefill(torch.from_numpy(x).to(DEV), ids=ids, wts=wts).cpu().numpy()
    r = oracle.route_fp32(x, w.router, bias, 6)
    assert np.array_equal(ids.cpu().numpy(), r.ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), r.weights.view(np.uint32))
    _check(oracle, got, oracle.moe_layer_fp64(cfg, w, x, r.ids, r.weights))


def test_int8_prefill_equals_bf16_of_dequantised_weights(uocr, oracle):
    """The int8 layer dequantises the touched experts' int8 items to bf16_rne(f32(q) * scale)
    (int8_dequant_expert's bits) before the bf16 GEMMs: it equals, bit for bit, the bf16 layer
    whose routed experts are the reference dequant of the same int8 stacks (oracle.dequant_bits),
    routing, GEMM tiling and combine being the same."""
    cfg, w = full_layer(oracle, True, 0)
    st8 = to_state(w, cfg, True)
    st16 = {k: v for k, v in st8.items() if not k.endswith("_scales")}
    for name in ("gate", "up", "down"):
        q, sc = getattr(w, name), getattr(w, f"{name}_scales")
        bits = np.stack([oracle.dequant_bits(q, sc, e) for e in range(q.shape[0])])
        st16[f"experts.{name}_proj"] = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    moe8 = uocr.UocrMoE(uocr.MoEConfig(int8_experts=True)).load_state_dict(st8)
    moe16 = uocr.UocrMoE(uocr.MoEConfig()).load_state_dict(st16)
    bias = torch.from_numpy(np.random.default_rng(41).standard_normal(64).astype(np.float32)).to(DEV)
    moe8.bias = moe16.bias = bias
    x = torch.from_numpy(oracle.synth_hidden(4096, cfg.hidden, 6)).to(DEV)
    got8, got16 = moe8.prefill(x), moe16.prefill(x)
    assert torch.isfinite(got8).all()
    assert torch.equal(got8, got16)
    moe8.check_status()
