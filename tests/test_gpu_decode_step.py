"""GPU: the whole decode step (``DecoderDecodeStep``: token ids -> embedding -> decoder layers ->
final norm -> lm_head -> n-gram guard) and its two elementwise kernels: the embedding bit for bit
against the table's rows (ids clamped), silu(g)*u against float64, layer 0's dense FFN
(``DenseFfn``) stage by stage, and the step: the final norm against float64, the guarded logits equal
to lm_head's output except exactly the oracle's banned ids, the CUDA-graph replay equal to the eager
step bit for bit."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
H, HEADS, DIM, I0 = 1280, 10, 128, 6848
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def mods():
    return (importlib.import_module("unlimited-ocr-max_b200.ops"),
            importlib.import_module("unlimited-ocr-max_b200.decode_layer"))


def _w(g, *shape, std=0.02):
    return (torch.randn(shape, generator=g) * std).to(torch.bfloat16)


def _near(out, w, x, tol=1e-4):
    ref = x.double() @ w.double().T
    bound = x.double().abs() @ w.double().abs().T
    assert bool(((out.double() - ref).abs() <= tol * bound + 1e-6).all())


def test_embedding_rows_and_clamped_ids(mods):
    ops, _ = mods
    g = torch.Generator().manual_seed(1)
    table = _w(g, 1000, 256, std=1.0).to(DEV)
    ids = torch.tensor([0, 999, 17, -3, 1005], dtype=torch.int32, device=DEV)
    out = ops.embed_rows(table, ids)
    want = table[ids.clamp(0, 999).long()].float()
    assert torch.equal(out, want)


def test_silu_mul_matches_float64(mods):
    ops, _ = mods
    g = torch.Generator().manual_seed(2)
    gu = (torch.randn(5, 2 * 300, generator=g) * 4).to(DEV)
    out = ops.silu_mul(gu).double().cpu()
    x = gu.double().cpu()
    gg, u = x[:, :300], x[:, 300:]
    ref = gg / (1 + torch.exp(-gg)) * u
    assert bool(((out - ref).abs() <= 2e-6 * ref.abs() + 1e-30).all())


def test_dense_ffn_stage_by_stage(mods):
    _, dl = mods
    g = torch.Generator().manual_seed(3)
    wg, wu, wd = _w(g, I0, H), _w(g, I0, H), _w(g, H, I0)
    ffn = dl.DenseFfn(wg, wu, wd, device=DEV, kblocked=False)
    x = torch.randn(4, H, generator=g).to(DEV)
    out = ffn.decode_rows(x)
    gu, act = ffn._bufs[4]
    _near(gu, torch.cat([wg, wu]).to(DEV), x)
    a64 = gu.double().cpu()
    ref_act = a64[:, :I0] / (1 + torch.exp(-a64[:, :I0])) * a64[:, I0:]
    assert bool(((act.double().cpu() - ref_act).abs() <= 2e-6 * ref_act.abs() + 1e-12).all())
    _near(out, wd.to(DEV), act)
    ffn.check_status()


def test_the_decode_step_ids_to_guarded_logits(uocr, oracle, mods):
    _, dl = mods
    synth = importlib.import_module("unlimited-ocr-max_b200.synth")
    g = torch.Generator().manual_seed(4)
    V, B, W, n = 8192, 4, 64, 3
    layers = []
    for idx in range(2):
        if idx == 0:
            mlp = dl.DenseFfn(_w(g, I0, H), _w(g, I0, H), _w(g, H, I0), device=DEV, kblocked=False)
        else:
            cfg = uocr.MoEConfig(int8_experts=True)
            mlp = uocr.UocrMoE(cfg, device=DEV).load_state_dict(synth.layer_state(cfg, 950, device="cpu"))
        gam = [(1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(2)]
        layers.append(dl.DecoderLayerDecode(mlp, layer_idx=idx, heads=HEADS, q_proj=_w(g, H, H), k_proj=_w(g, H, H),
                                            v_proj=_w(g, H, H), o_proj=_w(g, H, H), input_norm=gam[0],
                                            post_norm=gam[1], kblocked=False))
    final = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    step_fn = dl.DecoderDecodeStep(_w(g, V, H, std=1.0), layers, final, _w(g, V, H), kblocked=False)

    rng = np.random.default_rng(5)
    cols = 2
    pool = torch.from_numpy(rng.standard_normal((B * cols + 1, 2, 2, 128, HEADS, DIM)).astype(np.float32)).to(DEV)
    attend = np.asarray([9, 100, 200, 256], np.int32)
    cos_t, sin_t = dl.rope_tables(head_dim=DIM, seq_len=512, theta=10000.0)
    hist = rng.integers(0, V, size=(B, W)).astype(np.int32)
    hist[:, -2:] = hist[:, 10:12]  # the last two ids recur: each row bans hist[:, 12]
    step = {"cos": torch.from_numpy(cos_t[attend - 1]).to(DEV), "sin": torch.from_numpy(sin_t[attend - 1]).to(DEV),
            "kv_pool": pool, "lut": torch.from_numpy(rng.permutation(B * cols).astype(np.int32).reshape(B, cols)).to(DEV),
            "write_index": torch.from_numpy(attend - 1).to(DEV), "attend_len": torch.from_numpy(attend).to(DEV),
            "history": torch.from_numpy(hist).to(DEV), "ngram": torch.tensor([n], dtype=torch.int32, device=DEV)}
    ids = torch.tensor([5, 77, 8191, 1000], dtype=torch.int32, device=DEV)
    pool0 = pool.clone()

    logits = step_fn(ids, **step).clone()
    torch.cuda.synchronize()
    step_fn.check_status()
    t = step_fn.buffers(B)
    h = t["h"].double().cpu()
    y_ref = h / torch.sqrt((h * h).mean(dim=1, keepdim=True) + 1e-6) * final.double()
    assert bool(((t["y"].double().cpu() - y_ref).abs() <= 1e-5 * y_ref.abs() + 1e-6).all())
    plain = step_fn.lm_head.decode_rows(t["y"])
    want = oracle.ngram_block_rows(plain.cpu().numpy(), [list(r) for r in hist], n, W)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert all(logits[b, int(hist[b, 12])] == oracle.NGRAM_BLOCKED for b in range(B))
    assert bool(torch.isfinite(plain).all())

    pool.copy_(pool0)
    gr = step_fn.graph(ids, **step)
    pool.copy_(pool0)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(step_fn.buffers(B)["logits"], logits)
