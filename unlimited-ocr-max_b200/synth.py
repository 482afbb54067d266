"""Seeded synthetic MoE layers generated on the device (random init stands in
for the checkpoint, which is not available offline).

Every matrix is N(0, std) rounded to bf16; int8 stacks are quantised from those bf16 values
with the int8 format of tools/quantize_int8.py:55-70 (per-group G=128 along K,
scale = amax / 127 as an fp32 division, 1.0 for an all-zero group,
q = clip(rint(w / scale), -127, 127) with half-to-even rounding), computed with torch ops
that round exactly as the format states.
"""

from __future__ import annotations

import torch

INT8_GROUP_SIZE = 128


def quantize_per_group(w: torch.Tensor, group: int = INT8_GROUP_SIZE) -> tuple[torch.Tensor, torch.Tensor]:
    """``[..., N, K]`` -> ``(int8 [..., N, K], fp32 [..., N, K/group])``."""
    w = w.float()
    *lead, n, k = w.shape
    if k % group:
        raise ValueError(f"K={k} is not divisible by the group size {group}")
    g = w.reshape(*lead, n, k // group, group)
    amax = torch.maximum(g.amax(dim=-1), -g.amin(dim=-1))
    scales = torch.where(amax == 0, torch.ones_like(amax), amax / 127.0)
    q = torch.round(g / scales[..., None]).clamp_(-127, 127).to(torch.int8)
    return q.reshape(*lead, n, k).contiguous(), scales.contiguous()


def hidden_states(T: int, H: int, seed: int, device="cuda") -> torch.Tensor:
    """N(0, 1) rows RMS-normalised (gamma 1, eps 1e-6): the MoE sublayer's input."""
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((T, H), generator=gen, device=device, dtype=torch.float32)
    return (x / torch.sqrt((x.double() ** 2).mean(dim=1, keepdim=True) + 1e-6).float()).contiguous()


def layer_state(cfg, seed: int, *, device="cuda", std: float = 0.02) -> dict[str, torch.Tensor]:
    """A reference-named state dict (decoder.py:305-313, 269-271, 507) for one MoE layer."""
    gen = torch.Generator(device=device).manual_seed(seed)
    E, H, I, SI = cfg.n_routed_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.shared_experts_dim

    def mat(*shape):
        return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)

    st = {
        "gate.gate_score.weight": mat(E, H),
        "shared_experts.gate_proj.weight": mat(SI, H),
        "shared_experts.up_proj.weight": mat(SI, H),
        "shared_experts.down_proj.weight": mat(H, SI),
    }
    for name, shape in (("gate_proj", (E, I, H)), ("up_proj", (E, I, H)), ("down_proj", (E, H, I))):
        w = mat(*shape)
        if cfg.int8_experts:
            q, s = quantize_per_group(w)
            del w
            st[f"experts.{name}"] = q
            st[f"experts.{name}_scales"] = s
        else:
            st[f"experts.{name}"] = w
    return st


def skew_bias(E: int, seed: int, *, zipf_s: float | None = None, device="cuda") -> torch.Tensor:
    """A per-expert logit bias: N(0, 1), or log p_e with p_e proportional to
    rank^-s over a seeded permutation of ranks (config 5's Zipf skew)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    if zipf_s is None:
        return torch.randn(E, generator=gen).to(device)
    ranks = torch.randperm(E, generator=gen).double() + 1.0
    p = ranks ** (-zipf_s)
    p = p / p.sum()
    return torch.log(p).float().to(device)
