"""Checkpoint tensors -> the MoE sublayer's stacked state dict (the MoE half of the reference's
weight adapter, unlimited_ocr_max/weight_adapters.py).

The checkpoint stores every routed expert's projection under its own name,
``model.layers.{L}.mlp.experts.{E}.{proj}.weight`` (bf16 ``[N, K]``, or int8 next to a
``...weight_scales`` fp32 ``[N, K / 128]``). The MoE sublayer reads them as stacks in ascending
expert index: ``experts.{proj}`` ``[E, N, K]`` and, for int8, ``experts.{proj}_scales``
``[E, N, K / 128]`` (weight_adapters.py:121-163). This module does that stacking with the
reference's completeness checks and messages, tells the two checkpoint forms apart and refuses a
half-quantised file (weight_adapters.py:187-219), and selects one layer's MoE tensors under the
names :class:`UocrMoE.load_state_dict` takes (the router renamed ``mlp.gate.weight`` ->
``gate.gate_score.weight`` as weight_adapters.py:115-119 does). The stacks are torch tensors on
whatever device the checkpoint tensors live on; the packing into the library's layout happens in
``UocrMoE.load_state_dict`` on the GPU.
"""

from __future__ import annotations

import re
from collections.abc import Mapping

import torch

__all__ = ["WeightMappingError", "EXPERT_WEIGHT_RE", "language_weight_name", "stack_expert_weights",
           "is_int8_checkpoint", "moe_layer_state"]


class WeightMappingError(RuntimeError):
    """The checkpoint and the layer's declared weights do not line up exactly
    (weight_adapters.py:97-98)."""


#: A per-expert weight after the ``model.`` prefix is stripped, or the group scales of an int8
#: one. Anchored at both ends: ``shared_experts`` never matches, and ``_scales`` is a whole
#: suffix (``weight_zeros``, ``weight_scale_inv`` or ``weight_scales2`` are no match at all), as
#: weight_adapters.py:87-90 specifies.
EXPERT_WEIGHT_RE = re.compile(
    r"^(?P<stem>layers\.(?P<layer>[0-9]+)\.mlp\.experts)\.(?P<expert>[0-9]+)\."
    r"(?P<proj>gate_proj|up_proj|down_proj)\.weight(?P<scales>_scales)?$")

_PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def _dtype_name(t: torch.Tensor) -> str:
    """A tensor's dtype as a bare name (``bfloat16``, ``int8``, ``float32``)."""
    return str(t.dtype).removeprefix("torch.")


def language_weight_name(checkpoint_name: str) -> str:
    """The decoder's name of a checkpoint tensor: ``model.`` stripped, the router's
    ``mlp.gate.weight`` renamed ``mlp.gate.gate_score.weight`` (weight_adapters.py:115-119)."""
    name = checkpoint_name.removeprefix("model.")
    if name.endswith(".mlp.gate.weight"):
        name = name[: -len(".weight")] + ".gate_score.weight"
    return name


def stack_expert_weights(state: Mapping[str, torch.Tensor], *, num_experts: int) -> dict[str, torch.Tensor]:
    """Collapse each MoE layer's per-expert tensors into one stack per projection.

    ``layers.{L}.mlp.experts.{E}.{proj}.weight`` becomes ``layers.{L}.mlp.experts.{proj}`` and
    ``...weight_scales`` becomes ``layers.{L}.mlp.experts.{proj}_scales``; every other name passes
    through. Each stack is checked before it is built (weight_adapters.py:145-162): expert indices
    0..n-1 with no gaps, exactly ``num_experts`` of them, one dtype (``torch.stack`` would promote
    a mixed set silently) and one shape (named here, where ``torch.stack`` would only say the sizes
    differ). Slice j of a stack is expert j.
    """
    out: dict[str, torch.Tensor] = {}
    grouped: dict[str, dict[int, torch.Tensor]] = {}
    for name, value in state.items():
        m = EXPERT_WEIGHT_RE.match(name)
        if m is None:
            out[name] = value
            continue
        grouped.setdefault(f"{m['stem']}.{m['proj']}{m['scales'] or ''}", {})[int(m["expert"])] = value
    for stacked, members in grouped.items():
        idx = sorted(members)
        if idx != list(range(len(idx))):
            raise WeightMappingError(f"{stacked}: expert indices must be 0..n-1 with no gaps, got {idx}")
        if len(idx) != num_experts:
            raise WeightMappingError(f"{stacked}: expected {num_experts} experts, got {len(idx)}")
        dtypes = sorted({_dtype_name(members[j]) for j in idx})
        if len(dtypes) != 1:
            raise WeightMappingError(f"{stacked}: the experts disagree on dtype: {dtypes}")
        shapes = sorted({tuple(int(d) for d in members[j].shape) for j in idx})
        if len(shapes) != 1:
            raise WeightMappingError(f"{stacked}: the experts disagree on shape: {shapes}")
        out[stacked] = torch.stack([members[j] for j in idx]).contiguous()
    return out


def _expert_tensors(checkpoint: Mapping[str, torch.Tensor]):
    """(weights, scales), each keyed by (layer, expert, proj), from checkpoint or decoder names."""
    weights, scales = {}, {}
    for name, value in checkpoint.items():
        m = EXPERT_WEIGHT_RE.match(name.removeprefix("model."))
        if m is not None:
            (scales if m["scales"] else weights)[(int(m["layer"]), int(m["expert"]), m["proj"])] = value
    return weights, scales


def _names(keys, suffix: str = "") -> list[str]:
    """The first 20 keys back as checkpoint names, for an error message."""
    return [f"model.layers.{l}.mlp.experts.{e}.{p}.weight{suffix}" for l, e, p in sorted(keys)[:20]]


def is_int8_checkpoint(checkpoint: Mapping[str, torch.Tensor]) -> bool:
    """Whether the routed experts are int8 with per-group ``weight_scales`` (False for the bf16
    form, which carries no scales at all). A half-quantised file raises
    :class:`WeightMappingError` instead of being read as either form (weight_adapters.py:187-219):
    int8 weights without scales, scales without a weight, scales next to weights that are not
    int8, or scales for some experts or projections but not all."""
    weights, scales = _expert_tensors(checkpoint)
    quantized = {k for k, v in weights.items() if v.dtype == torch.int8}
    if not scales:
        if quantized:
            raise WeightMappingError(f"int8 expert weights without weight_scales: {_names(quantized)}")
        return False
    orphans = set(scales) - set(weights)
    if orphans:
        raise WeightMappingError(
            f"weight_scales without an expert weight to scale: {_names(orphans, '_scales')}")
    unquantized = set(weights) - quantized
    if unquantized:
        found = sorted({_dtype_name(weights[k]) for k in unquantized})
        raise WeightMappingError(
            f"weight_scales are present but these expert weights are {found}, not int8: {_names(unquantized)}")
    bare = set(weights) - set(scales)
    if bare:
        raise WeightMappingError(f"half-quantized checkpoint: no weight_scales for {_names(bare)}")
    return True


def moe_layer_state(checkpoint: Mapping[str, torch.Tensor], layer: int, *, num_experts: int = 64
                    ) -> tuple[dict[str, torch.Tensor], bool]:
    """One decoder layer's MoE tensors from a checkpoint, under the names ``UocrMoE`` loads:
    ``gate.gate_score.weight``, ``experts.{proj}`` (+ ``_scales``) stacked in ascending expert
    index, and ``shared_experts.{proj}.weight``. Returns ``(state, int8)``; ``int8`` says which
    checkpoint form the layer is in. The whole checkpoint is checked for a half-quantised file
    first (as language_state_dict does, weight_adapters.py:278-292), then only this layer's
    tensors are stacked."""
    int8 = is_int8_checkpoint(checkpoint)
    prefix = f"layers.{layer}.mlp."
    mine = {}
    for name, value in checkpoint.items():
        dec = language_weight_name(name)
        if dec.startswith(prefix):
            mine[dec] = value
    if not mine:
        raise WeightMappingError(f"no MoE weights for layer {layer} in the checkpoint")
    stacked = stack_expert_weights(mine, num_experts=num_experts)
    state = {name[len(prefix):]: t for name, t in stacked.items()}
    want = {"gate.gate_score.weight", *(f"experts.{p}" for p in _PROJECTIONS),
            *(f"shared_experts.{p}.weight" for p in _PROJECTIONS)}
    if int8:
        want |= {f"experts.{p}_scales" for p in _PROJECTIONS}
    missing, extra = sorted(want - set(state)), sorted(set(state) - want)
    if missing or extra:
        raise WeightMappingError(
            f"layer {layer} MoE weights disagree with the checkpoint: missing {missing[:20]}, unexpected {extra[:20]}")
    return state, int8
