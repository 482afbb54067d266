"""GPU: the MoE half of the decode step (``MoEDecodeStack``: per layer the post-attention RMSNorm,
the MoE sublayer and the residual add, decoder.py:702-709), eager and from its CUDA graph.

Per layer: the normalised rows against the float64 RMSNorm (decoder.py:252-261), the routing ids
and weights bit-exact with the oracle's fp32 gate on those rows, the MoE output within the
reference's float64 bar and the north-star bar of the float64 layer, and the residual stream
exactly h + out in fp32; the graph's step equals the eager step bit for bit.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from test_oracle import weights_from_state

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("int8,B", [(True, 8), (False, 4)])
def test_moe_decode_stack_layer_by_layer(uocr, oracle, int8, B):
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    stack = importlib.import_module("unlimited-ocr-max_b200.stack")
    dev = torch.device("cuda", 0)
    L, H = 3, 1280
    cfg = uocr.MoEConfig(int8_experts=int8)
    states = [synth.layer_state(cfg, 600 + 10 * l + int(int8), device="cpu") for l in range(L)]
    layers = [uocr.UocrMoE(cfg, device=dev).load_state_dict(s) for s in states]
    g = torch.Generator().manual_seed(77)
    gammas = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(L)]
    st = stack.MoEDecodeStack(layers, gammas, eps=1e-6)
    h0 = (3 * torch.randn(B, H, generator=g)).to(dev)

    hs, ys, outs = st.decode_rows(h0, keep_intermediates=True)
    torch.cuda.synchronize()
    st.check_status()
    ocfg = oracle.MoEConfig()
    for l in range(L):
        h = hs[l].double().cpu()
        gam = gammas[l].double()
        y_ref = h / torch.sqrt((h * h).mean(dim=1, keepdim=True) + 1e-6) * gam
        y = ys[l].double().cpu()
        assert bool(((y - y_ref).abs() <= 1e-5 * y_ref.abs() + 1e-6).all()), l
        w = weights_from_state(oracle, states[l], int8)
        x = ys[l].cpu().numpy()
        r = oracle.route_fp32(x, w.router, None, 6)
        got = outs[l].cpu().numpy()
        ref = oracle.moe_layer_fp64(ocfg, w, x, r.ids, r.weights)
        for i in range(B):
            assert oracle.cosine(got[i], ref[i]) >= 0.99999, (l, i)
        assert oracle.rel_err(got, ref) <= 1e-4, l
        assert np.max(np.abs(got - ref)) <= 2e-2 and oracle.rel_l2(got, ref) <= 1e-2, l
        assert torch.equal(hs[l + 1], hs[l] + outs[l]), l

    stepped = st.step(h0)
    assert torch.equal(stepped, hs[L])
    assert torch.equal(st.step(h0), stepped)  # replays repeat
    assert torch.equal(st.decode_rows(h0), hs[L])
    st.check_status()
