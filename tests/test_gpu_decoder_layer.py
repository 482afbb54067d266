"""GPU: a decoder layer's decode step composed from the library's kernels (``DecoderLayerDecode``,
DecoderLayer.decode, decoder.py:702-709), checked stage by stage, each stage fed the previous
stage's device values: the input and post-attention norms against float64, the fused q|k|v and the
o projection within 1e-4 of sum |w x| of float64, RoPE bit for bit against the fp32 formula
(decoder.py:459-462), the attention against the float64 paged attention (the pool's new rows exact),
the MoE with bit-exact routing and within the float64 and north-star bars, both residual adds exact;
then two layers captured in one CUDA graph replay the eager step bit for bit."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from test_oracle import weights_from_state

pytestmark = pytest.mark.gpu
H, HEADS, DIM = 1280, 10, 128


def _layer(uocr, synth, dl, idx, seed, dev):
    cfg = uocr.MoEConfig(int8_experts=True)
    state = synth.layer_state(cfg, seed, device="cpu")
    moe = uocr.UocrMoE(cfg, device=dev).load_state_dict(state)
    g = torch.Generator().manual_seed(seed)
    ws = [(torch.randn(H, H, generator=g) * 0.02).to(torch.bfloat16) for _ in range(4)]
    gam = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(2)]
    layer = dl.DecoderLayerDecode(moe, layer_idx=idx, heads=HEADS, q_proj=ws[0], k_proj=ws[1], v_proj=ws[2],
                                  o_proj=ws[3], input_norm=gam[0], post_norm=gam[1], kblocked=False)
    return layer, state, ws, gam


def _step_inputs(B, layers, dev, seed):
    dl = importlib.import_module("unlimited-ocr-max_b200.decode_layer")
    rng = np.random.default_rng(seed)
    cols = 5
    pages = B * cols + 1
    pool = torch.from_numpy(rng.standard_normal((pages, 2, layers, 128, HEADS, DIM)).astype(np.float32)).to(dev)
    lut = torch.from_numpy(rng.permutation(B * cols).astype(np.int32).reshape(B, cols)).to(dev)
    attend = np.asarray([7, 130, 400, 640, 33, 512, 600, 200][:B], np.int32)
    write = attend - 1
    cos_t, sin_t = dl.rope_tables(head_dim=DIM, seq_len=1024, theta=10000.0)
    pos = attend - 1
    step = {"cos": torch.from_numpy(cos_t[pos]).to(dev), "sin": torch.from_numpy(sin_t[pos]).to(dev),
            "kv_pool": pool, "lut": lut, "write_index": torch.from_numpy(write).to(dev),
            "attend_len": torch.from_numpy(attend).to(dev)}
    h = torch.from_numpy((3 * rng.standard_normal((B, H))).astype(np.float32)).to(dev)
    return h, step


def _near(out, w, x, tol=1e-4):
    ref = x.double() @ w.double().T
    bound = x.double().abs() @ w.double().abs().T
    assert bool(((out.double() - ref).abs() <= tol * bound + 1e-6).all())


def _norm64(h, gamma):
    h = h.double().cpu()
    return h / torch.sqrt((h * h).mean(dim=1, keepdim=True) + 1e-6) * gamma.double()


def test_one_layer_stage_by_stage(uocr, oracle):
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    dl = importlib.import_module("unlimited-ocr-max_b200.decode_layer")
    dev = torch.device("cuda", 0)
    B = 4
    layer, state, ws, gam = _layer(uocr, synth, dl, 1, 900, dev)
    h, step = _step_inputs(B, 2, dev, 5)
    h0 = h.clone()
    pool0 = step["kv_pool"].clone()
    layer.decode(h, **step)
    torch.cuda.synchronize()
    layer.check_status()
    t = layer.buffers(B)

    y = t["y"].double().cpu()
    assert bool(((y - _norm64(h0, gam[0])).abs() <= 1e-5 * _norm64(h0, gam[0]).abs() + 1e-6).all())
    _near(t["qkv"], torch.cat(ws[:3]).to(dev), t["y"])
    # RoPE exactly as the fp32 formula: each product and the sum rounded
    x = t["qkv"].view(B, 3, HEADS, DIM)
    c, s = step["cos"].view(B, 1, DIM), step["sin"].view(B, 1, DIM)
    rot = lambda z: torch.cat([-z[..., DIM // 2:], z[..., :DIM // 2]], dim=-1)  # noqa: E731
    assert torch.equal(t["q"], x[:, 0] * c + rot(x[:, 0]) * s)
    assert torch.equal(t["k"], x[:, 1] * c + rot(x[:, 1]) * s)
    assert torch.equal(t["v"], x[:, 2])
    ref, pool_ref = oracle.paged_decode_attention_ref(
        t["q"].cpu().numpy(), t["k"].cpu().numpy(), t["v"].cpu().numpy(), pool0.cpu().numpy(), 1,
        step["lut"].cpu().numpy(), step["write_index"].cpu().numpy(), step["attend_len"].cpu().numpy(), DIM ** -0.5)
    assert np.max(np.abs(t["attn"].cpu().numpy() - ref)) <= 2e-5
    assert np.array_equal(step["kv_pool"].cpu().numpy().view(np.uint32), pool_ref.view(np.uint32))
    _near(t["o"], ws[3].to(dev), t["attn"].view(B, H))
    h1 = h0 + t["o"]
    y2 = t["y2"].double().cpu()
    assert bool(((y2 - _norm64(h1, gam[1])).abs() <= 1e-5 * _norm64(h1, gam[1]).abs() + 1e-6).all())
    w = weights_from_state(oracle, state, True)
    xm = t["y2"].cpu().numpy()
    r = oracle.route_fp32(xm, w.router, None, 6)
    got = t["m"].cpu().numpy()
    mref = oracle.moe_layer_fp64(oracle.MoEConfig(), w, xm, r.ids, r.weights)
    assert oracle.rel_err(got, mref) <= 1e-4
    assert np.max(np.abs(got - mref)) <= 2e-2 and oracle.rel_l2(got, mref) <= 1e-2
    assert torch.equal(h, h1 + t["m"])


def test_two_layers_in_one_graph_replay_the_eager_step(uocr):
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    dl = importlib.import_module("unlimited-ocr-max_b200.decode_layer")
    dev = torch.device("cuda", 0)
    B = 8
    layers = [_layer(uocr, synth, dl, i, 910 + i, dev)[0] for i in range(2)]
    stack = dl.DecoderDecodeStack(layers)
    h, step = _step_inputs(B, 2, dev, 6)
    h0, pool0 = h.clone(), step["kv_pool"].clone()
    eager = stack.decode(h, **step).clone()
    step["kv_pool"].copy_(pool0)
    h.copy_(h0)
    g = stack.graph(h, **step)
    step["kv_pool"].copy_(pool0)
    h.copy_(h0)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(h, eager)
    stack.check_status()
