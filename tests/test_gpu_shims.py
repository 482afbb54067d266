"""GPU parity of the reference's four custom ops, through the C ABI (ops.py wrappers).

Mirrors the reference's kernel tests (tests/test_kernels_bf16.py, tests/test_kernels_int8.py,
tests/test_kernels_dense_bf16.py): fp64 gates (bf16 qmv 1e-5, int8 qmv 1e-6), the int8 qmv's
bits against the reference's exact fma order, dequant bit for bit (incl. -0.0), clamped ids,
row independence, k = 0, misaligned inputs, and the real-shape smoke.
"""

from __future__ import annotations

from collections import Counter
from pathlib import Path

import numpy as np
import pytest
import torch

from golden import reference_inputs as ri

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return t(bits.view(np.int16)).view(torch.bfloat16)


def misaligned(x: torch.Tensor) -> torch.Tensor:
    """A copy of ``x`` one element past its buffer's (256-byte) aligned start."""
    buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=x.device)
    v = buf[1:].view(x.shape)
    v.copy_(x)
    assert v.data_ptr() % 16 != 0
    return v


# ---- moe_bf16_qmv ----------------------------------------------------------------------


def bf16_qmv(uocr, x, ids, w_bits):
    return uocr.ops.moe_bf16_qmv(t(x), t(ids), bf16_dev(w_bits)).cpu().numpy()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_bf16_qmv_random(uocr, oracle, seed):
    x, ids, w = ri.bf16_rand(seed)
    assert oracle.rel_err(bf16_qmv(uocr, x, ids, w), oracle.bf16_qmv_ref64(x, ids, w)) <= 1e-5


def test_bf16_qmv_scalar_path_k30(uocr, oracle):
    x, ids, w = ri.bf16_rand(3, kdim=ri.BF16_K_ODD)
    assert oracle.rel_err(bf16_qmv(uocr, x, ids, w), oracle.bf16_qmv_ref64(x, ids, w)) <= 1e-5


@pytest.mark.parametrize("k", [1, 6, 12, 24, 48])
def test_bf16_qmv_rows_sharing_experts_are_their_lone_values(uocr, oracle, k):
    x, _, w = ri.bf16_rand(40 + k, k=k)
    ids = np.random.default_rng(80 + k).integers(-2, ri.BF16_E + 2, size=k).astype(np.int32)
    if k >= 24:
        assert max(Counter(ids.tolist()).values()) > 4
    out = bf16_qmv(uocr, x, ids, w)
    assert oracle.rel_err(out, oracle.bf16_qmv_ref64(x, ids, w)) <= 1e-5
    for s in range(k):
        assert np.array_equal(out[s : s + 1], bf16_qmv(uocr, x[s : s + 1], ids[s : s + 1], w)), s


def test_bf16_qmv_one_hot_exact(uocr):
    E, N, K, k = 5, 8, 32, 6
    x = (np.arange(k * K, dtype=np.float32).reshape(k, K) + 1.0) * np.float32(0.5)
    ids = np.array([4, 0, 2, 3, 1, 4], dtype=np.int32)
    w = np.zeros((E, N, K), dtype=np.float32)
    for e in range(E):
        for n in range(N):
            w[e, n, (n + 3 * e) % K] = 1.0
    out = bf16_qmv(uocr, x, ids, ri.bf16_bits(w))
    want = np.array([[x[s, (n + 3 * ids[s]) % K] for n in range(N)] for s in range(k)], dtype=np.float32)
    assert np.array_equal(out, want)


def test_bf16_qmv_zero_weights_clamp_and_empty(uocr, oracle):
    x, ids, w = ri.bf16_rand(5)
    assert not np.any(bf16_qmv(uocr, x, ids, np.zeros_like(w)))
    raw = np.array([-1, 5, 7, -100, 2, 4], dtype=np.int32)
    assert np.array_equal(bf16_qmv(uocr, x, raw, w), bf16_qmv(uocr, x, np.clip(raw, 0, 4).astype(np.int32), w))
    out = uocr.ops.moe_bf16_qmv(torch.zeros((0, 32), device=DEV), torch.zeros(0, dtype=torch.int32, device=DEV),
                                bf16_dev(w))
    assert tuple(out.shape) == (0, 8)


@pytest.mark.parametrize("off", ["w", "x", "wx"])
def test_bf16_qmv_misaligned_gives_the_aligned_bits(uocr, off):
    x, ids, w = ri.bf16_rand(11)
    xt, wt = t(x), bf16_dev(w)
    ref = uocr.ops.moe_bf16_qmv(xt, t(ids), wt)
    got = uocr.ops.moe_bf16_qmv(misaligned(xt) if "x" in off else xt, t(ids), misaligned(wt) if "w" in off else wt)
    assert torch.equal(got, ref)


def test_bf16_qmv_rejects_a_k_mismatch(uocr):
    with pytest.raises(ValueError, match=r"moe_bf16_qmv: w and x disagree on K"):
        uocr.ops.moe_bf16_qmv(torch.zeros((2, 24), device=DEV), torch.zeros(2, dtype=torch.int32, device=DEV),
                              torch.zeros((3, 4, 32), dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("k", [6, 48])
@pytest.mark.parametrize("n,kdim", [(896, 1280), (1280, 896)])
def test_bf16_qmv_real_shape(uocr, oracle, n, kdim, k):
    rng = np.random.default_rng(20261003 + k)
    x = rng.standard_normal((k, kdim)).astype(np.float32)
    pool = rng.permutation(64)[:28]
    ids = np.concatenate([rng.choice(pool, 6, replace=False) for _ in range(k // 6)]).astype(np.int32)
    w = ri.bf16_bits((0.05 * rng.standard_normal((64, n, kdim))).astype(np.float32))
    out = bf16_qmv(uocr, x, ids, w)
    assert oracle.rel_err(out, oracle.bf16_qmv_ref64(x, ids, w)) <= 1e-5
    if k > 6:
        for s0 in range(0, k, 6):
            assert np.array_equal(out[s0 : s0 + 6], bf16_qmv(uocr, x[s0 : s0 + 6], ids[s0 : s0 + 6], w))


# ---- moe_int8_qmv ----------------------------------------------------------------------


def int8_qmv(uocr, x, ids, w, s):
    return uocr.ops.moe_int8_qmv(t(x), t(ids), t(w), t(s)).cpu().numpy()


def test_int8_qmv_bits_are_the_reference_order_on_every_fixture(uocr):
    """Bitwise the reference's ``_qmv_base_order_fp32`` outputs stored in the fixture."""
    g = np.load(GOLDEN / "int8_kernels.npz")
    for tag in g["cases"]:
        seed, k, kdim, id_seed = (int(v) for v in g[f"{tag}_meta"])
        x, _, w, scales = ri.int8_rand(seed, k=k, kdim=kdim)
        ids = np.random.default_rng(id_seed).integers(-2, ri.INT8_E + 2, size=k).astype(np.int32)
        out = int8_qmv(uocr, x, ids, w, scales)
        assert np.array_equal(out.view(np.uint32), g[f"{tag}_base_bits"]), tag


@pytest.mark.parametrize("k", [1, 6, 12, 24, 48])
def test_int8_qmv_rows_and_oracle_bits(uocr, oracle, k):
    x, _, w, scales = ri.int8_rand(40 + k, k=k)
    ids = np.random.default_rng(80 + k).integers(-2, ri.INT8_E + 2, size=k).astype(np.int32)
    out = int8_qmv(uocr, x, ids, w, scales)
    assert np.array_equal(out.view(np.uint32), oracle.int8_qmv_base_order(x, ids, w, scales).view(np.uint32))
    assert oracle.rel_err(out, oracle.int8_qmv_ref64(x, ids, w, scales)) <= 1e-6


def test_int8_qmv_zero_groups_and_edges(uocr, oracle):
    x, ids, w, scales = ri.int8_rand(5)
    w = w.copy()
    scales = scales.copy()
    w[:, :, 32:64] = 0
    scales[:, :, 2] = 0.0
    assert oracle.rel_err(int8_qmv(uocr, x, ids, w, scales), oracle.int8_qmv_ref64(x, ids, w, scales)) <= 1e-6
    assert not np.any(int8_qmv(uocr, x, ids, np.zeros_like(w), scales))
    edge = np.broadcast_to(np.where(np.arange(128) % 2 == 0, 127, -127)[None, None, :], w.shape).astype(np.int8)
    assert oracle.rel_err(int8_qmv(uocr, x, ids, edge, scales), oracle.int8_qmv_ref64(x, ids, edge, scales)) <= 1e-6


def test_int8_qmv_misaligned_and_clamp(uocr, oracle):
    x, ids, w, scales = ri.int8_rand(14)
    ref = uocr.ops.moe_int8_qmv(t(x), t(ids), t(w), t(scales))
    got = uocr.ops.moe_int8_qmv(misaligned(t(x)), t(ids), misaligned(t(w)), t(scales))
    assert torch.equal(got, ref)
    raw = np.array([-1, 5, 7, -100, 2, 4], dtype=np.int32)
    assert np.array_equal(int8_qmv(uocr, x, raw, w, scales), int8_qmv(uocr, x, np.clip(raw, 0, 4).astype(np.int32), w, scales))


def test_int8_qmv_rejects_a_group_miscount(uocr):
    with pytest.raises(ValueError, match=r"moe_int8_qmv: K must be a multiple of the group count"):
        uocr.ops.moe_int8_qmv(torch.zeros((2, 32), device=DEV), torch.zeros(2, dtype=torch.int32, device=DEV),
                              torch.zeros((3, 4, 32), dtype=torch.int8, device=DEV),
                              torch.zeros((3, 4, 5), device=DEV))


@pytest.mark.parametrize("k", [6, 48])
@pytest.mark.parametrize("n,kdim", [(896, 1280), (1280, 896)])
def test_int8_qmv_real_shape_bits(uocr, oracle, n, kdim, k):
    rng = np.random.default_rng(20260909 + k)
    x = rng.standard_normal((k, kdim)).astype(np.float32)
    pool = rng.permutation(64)[:28]
    ids = np.concatenate([rng.choice(pool, 6, replace=False) for _ in range(k // 6)]).astype(np.int32)
    w = rng.integers(-127, 128, size=(64, n, kdim)).astype(np.int8)
    scales = rng.uniform(1e-3, 3e-2, size=(64, n, kdim // 128)).astype(np.float32)
    out = int8_qmv(uocr, x, ids, w, scales)
    assert np.array_equal(out.view(np.uint32), oracle.int8_qmv_base_order(x, ids, w, scales).view(np.uint32))
    assert oracle.rel_err(out, oracle.int8_qmv_ref64(x, ids, w, scales)) <= 1e-6


# ---- int8_dequant_expert ------------------------------------------------------------------


def dequant(uocr, w, s, e):
    out = uocr.ops.int8_dequant_expert(t(w), t(s), t(np.array([e], np.int32)))
    return out.view(torch.int16).cpu().numpy().view(np.uint16)


def test_dequant_fixture_bits(uocr):
    g = np.load(GOLDEN / "int8_kernels.npz")
    _, _, w, scales = ri.int8_rand(8)
    for e in (-3, 0, 1, 2, 3, 4, ri.INT8_E, ri.INT8_E + 7):
        assert np.array_equal(dequant(uocr, w, scales, e), g[f"rand8_e{e}"]), e
    _, _, w, scales = ri.int8_rand(10)
    scales = scales.copy()
    scales[:, :, 1] = 0.0
    got = dequant(uocr, w, scales, 2)
    assert np.array_equal(got, g["zeroscale_e2"]) and np.any(got == 0x8000)
    rng = np.random.default_rng(15)
    w = rng.integers(-127, 128, size=(ri.INT8_E, ri.INT8_N, 30)).astype(np.int8)
    scales = (10.0 ** rng.uniform(-3.0, 1.0, size=(ri.INT8_E, ri.INT8_N, 5))).astype(np.float32)
    for e in (0, ri.INT8_E - 1):
        assert np.array_equal(dequant(uocr, w, scales, e), g[f"k30_e{e}"])


def test_dequant_real_shape(uocr, oracle):
    rng = np.random.default_rng(1)
    w = rng.integers(-127, 128, size=(64, 896, 1280)).astype(np.int8)
    scales = rng.uniform(1e-3, 3e-2, size=(64, 896, 10)).astype(np.float32)
    assert np.array_equal(dequant(uocr, w, scales, 37), oracle.dequant_bits(w, scales, 37))


# ---- dense_bf16_qmv --------------------------------------------------------------------------


@pytest.mark.parametrize("m", [1, 3, 8])
def test_dense_bf16_qmv(uocr, oracle, m):
    rng = np.random.default_rng(m)
    n, k = 1792, 1280
    W = ri.bf16_bits((0.05 * rng.standard_normal((n, k))).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = x.astype(np.float64) @ oracle.bf16_to_f32(W).astype(np.float64).T
    outs = [uocr.ops.dense_bf16_qmv(t(x), bf16_dev(oracle.kblocked(W)), tile=tile).cpu().numpy() for tile in (1, 4, 8)]
    assert oracle.rel_err(outs[0], ref) <= 1e-5
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
    assert np.array_equal(outs[0][:1], uocr.ops.dense_bf16_qmv(t(x[:1]), bf16_dev(oracle.kblocked(W))).cpu().numpy())


# ---- router ------------------------------------------------------------------------------------


@pytest.mark.parametrize("T", [1, 7, 8, 13, 597, 4096])
@pytest.mark.parametrize("E,H", [(64, 1280), (8, 256), (64, 1536), (40, 2048)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_route_bit_exact(uocr, oracle, T, E, H, with_bias):
    """H <= 1280: the persistent kernel with the router in shared memory (T = 597 leaves 149
    4-token tiles over 148 CTAs, 4096 wraps each CTA's token double buffer many times); 1536 and
    2048: the register-blocked kernels (16- and 8-token CTAs)."""
    rng = np.random.default_rng(T + E)
    x = oracle.synth_hidden(T, H, T)
    router = oracle.bf16_bits(rng.standard_normal((E, H)).astype(np.float32) * np.float32(0.02))
    bias = rng.standard_normal(E).astype(np.float32) if with_bias else None
    ids, wts = uocr.ops.route(t(x), bf16_dev(router), None if bias is None else t(bias), 6)
    ref = oracle.route_fp32(x, router, bias, 6)
    assert np.array_equal(ids.cpu().numpy(), ref.ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ref.weights.view(np.uint32))


def test_route_ties_lowest_index(uocr, oracle):
    rng = np.random.default_rng(3)
    H, E = 256, 8
    router = oracle.bf16_bits(rng.standard_normal((E, H)).astype(np.float32) * np.float32(0.05))
    router[5] = router[2]
    router[7] = router[2]
    x = oracle.synth_hidden(64, H, 9)
    ids, wts = uocr.ops.route(t(x), bf16_dev(router), None, 6)
    ref = oracle.route_fp32(x, router, None, 6)
    assert np.array_equal(ids.cpu().numpy(), ref.ids)
