"""Regenerate the inputs of the golden fixtures from their seeds (no reference code needed).

These restate the reference tests' input generators -- ``_rand`` of
``tests/test_kernels_int8.py:211-222`` and ``tests/test_kernels_bf16.py:125-133``, and
``_moe_weights`` of ``tests/test_decoder_int8.py:643-663`` -- so a test can rebuild the exact
arrays the fixtures were computed from; each fixture stores a sha256 of its inputs and the
tests check it before comparing outputs.
"""

from __future__ import annotations

import hashlib
import types

import numpy as np

# tests/test_kernels_int8.py:60-62 and tests/test_kernels_bf16.py:57-59
INT8_E, INT8_N, INT8_K, INT8_GROUPS = 5, 8, 128, 4
INT8_K_SHORT = 32
BF16_E, BF16_N, BF16_K, BF16_K_ODD = 5, 8, 32, 30

SMALL_MOE = types.SimpleNamespace(
    n_routed_experts=8, hidden_size=256, moe_intermediate_size=128, shared_experts_dim=256, num_experts_per_tok=6
)


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def bf16_bits(values: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    carry = ((bits & np.uint32(0xFFFF)) + ((bits >> 16) & np.uint32(1)) + np.uint32(0x7FFF)) >> 16
    return ((bits >> 16) + carry).astype(np.uint16)


def int8_rand(seed: int, k: int = 6, kdim: int = INT8_K):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((k, kdim)).astype(np.float32)
    ids = rng.integers(0, INT8_E, size=k).astype(np.int32)
    w = rng.integers(-127, 128, size=(INT8_E, INT8_N, kdim)).astype(np.int8)
    scales = (10.0 ** rng.uniform(-3.0, 1.0, size=(INT8_E, INT8_N, INT8_GROUPS))).astype(np.float32)
    return x, ids, w, scales


def bf16_rand(seed: int, k: int = 6, kdim: int = BF16_K, num_experts: int = BF16_E, n: int = BF16_N):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((k, kdim)).astype(np.float32)
    ids = rng.integers(0, num_experts, size=k).astype(np.int32)
    magnitude = 10.0 ** rng.uniform(-3.0, 1.0, size=(num_experts, n, kdim))
    w = (magnitude * rng.choice([-1.0, 1.0], size=magnitude.shape)).astype(np.float32)
    return x, ids, bf16_bits(w)


def moe_weights(cfg, seed: int):
    """``(bf16 originals, int8 stacks + scales)`` as the reference's ``_moe_weights`` draws them:
    numpy float64 normals, scaled, cast to fp32 then bf16 (RNE); int8 by the torch twin
    quantiser ``_quantize`` (tests/test_decoder_int8.py:627-640)."""
    import torch

    rng = np.random.default_rng(seed)
    e, hidden, ffn, shared = cfg.n_routed_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.shared_experts_dim

    def bf16(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)

    common = {
        "gate.gate_score.weight": bf16(rng.standard_normal((e, hidden)) * 0.1),
        "shared_experts.gate_proj.weight": bf16(rng.standard_normal((shared, hidden)) * 0.05),
        "shared_experts.up_proj.weight": bf16(rng.standard_normal((shared, hidden)) * 0.05),
        "shared_experts.down_proj.weight": bf16(rng.standard_normal((hidden, shared)) * 0.05),
    }
    shapes = {"gate_proj": (e, ffn, hidden), "up_proj": (e, ffn, hidden), "down_proj": (e, hidden, ffn)}
    original, int8 = dict(common), dict(common)
    for proj, shape in shapes.items():
        stack = bf16(rng.standard_normal(shape) * 0.05)
        w = stack.float()
        E_, n, k = w.shape
        grouped = w.reshape(E_, n, k // 128, 128)
        amax = grouped.abs().amax(dim=3)
        scales = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax)).contiguous()
        q = torch.round(grouped / scales[..., None]).clamp(-127, 127)
        original[f"experts.{proj}"] = stack
        int8[f"experts.{proj}"] = q.to(torch.int8).reshape(E_, n, k).contiguous()
        int8[f"experts.{proj}_scales"] = scales
    return original, int8


def state_sha(state) -> str:
    import torch

    return sha(*[state[k].view(torch.int16).numpy() if state[k].dtype == torch.bfloat16 else state[k].numpy() for k in sorted(state)])
