"""The MoE sublayer with the reference's call surface.

``UocrMoE`` is a drop-in for ``MoE`` (unlimited_ocr_max/decoder.py:517-667): the same
config fields, the same state-dict names (``gate.gate_score.weight``,
``experts.{gate,up,down}_proj`` [+ ``_scales``], ``shared_experts.{proj}.weight``), and the
same two entry points -- ``decode_rows(x [B, H])`` for the batched decode step and
``__call__(x [T, H])`` for prefill -- each fp32 in, fp32 out. The weights are re-laid out
once at load (``uocr_moe_pack_*``); every forward runs the CUDA kernels of
``libuocr_moe.so``. There is no CPU path.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Mapping

import torch

from . import ops
from ._lib import UocrMoeLayer, check, load

__all__ = ["MoEConfig", "UocrMoE", "ConfigError"]

#: the int8 checkpoint's group size along K (model_config.py:52)
INT8_GROUP_SIZE = 128
#: decode batches run through the decode kernels in chunks of this many rows (cli.py:34 MAX_BATCH_CAP)
DECODE_MAX_B = 8


class ConfigError(ValueError):
    """The MoE hyper-parameters are not the ones this block implements (model_config.py:40)."""


@dataclass(frozen=True)
class MoEConfig:
    """The MoE fields of ``DecoderConfig`` (unlimited_ocr_max/model_config.py:66-173)."""

    hidden_size: int = 1280
    moe_intermediate_size: int = 896
    n_routed_experts: int = 64
    n_shared_experts: int = 2
    num_experts_per_tok: int = 6
    int8_experts: bool = False
    scoring_func: str = "softmax"
    topk_method: str = "greedy"
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0

    def __post_init__(self) -> None:
        # model_config.py:135-160
        if self.scoring_func != "softmax":
            raise ConfigError(f"unsupported scoring_func {self.scoring_func!r}")
        if self.topk_method != "greedy":
            raise ConfigError(f"unsupported topk_method {self.topk_method!r}")
        if self.n_group != 1 or self.topk_group != 1:
            raise ConfigError("grouped expert routing is not implemented")
        if self.n_shared_experts <= 0:
            raise ConfigError("this port expects shared experts")
        if self.norm_topk_prob or self.routed_scaling_factor != 1.0:
            raise ConfigError("the router is implemented without top-k renormalisation or scaling")
        if self.int8_experts:
            for name in ("hidden_size", "moe_intermediate_size"):
                if getattr(self, name) % INT8_GROUP_SIZE:
                    raise ConfigError(f"int8 experts need {name} divisible by the group size {INT8_GROUP_SIZE}")
        if self.hidden_size % 128:
            raise ConfigError("hidden_size must be a multiple of 128 (packed weight blocks, 16-byte loads)")
        if self.moe_intermediate_size % 128:
            raise ConfigError("moe_intermediate_size must be a multiple of 128 (gate|up packing)")
        if not 1 <= self.num_experts_per_tok <= self.n_routed_experts <= 64:
            raise ConfigError("need 1 <= num_experts_per_tok <= n_routed_experts <= 64")

    @property
    def shared_experts_dim(self) -> int:
        return self.n_shared_experts * self.moe_intermediate_size


def _dtype_name(d) -> str | None:
    """A dtype given as a torch dtype, a name, or an object with ``.name`` -> its bare name."""
    if d is None:
        return None
    if isinstance(d, torch.dtype):
        return str(d).removeprefix("torch.")
    name = getattr(d, "name", d)
    return str(name).removeprefix("torch.").lower()


def _unkblock(w: torch.Tensor) -> torch.Tensor:
    """A shared-expert projection as ``[N, K]``: accepts the plain checkpoint form or the
    reference's K-blocked declaration ``[K/16, N, 16]`` (decoder.py:219-225)."""
    if w.dim() == 3:
        blocks, n, width = w.shape
        return w.permute(1, 0, 2).reshape(n, blocks * width)
    return w


class UocrMoE:
    """64 routed experts, top-6, plus the shared experts (decoder.py:517-554)."""

    def __init__(self, config: MoEConfig, *, dtype=None, device: str | torch.device = "cuda",
                 norm_router_dtype=None) -> None:
        """``MoE(config, *, dtype, device, norm_router_dtype=None)`` (decoder.py:533-535).

        ``dtype`` is the non-expert weights' dtype: bf16 (the checkpoint's), the only one this
        build takes. ``norm_router_dtype`` is the dtype the router weight is held in: bf16, or
        fp32 holding bf16 values exactly (the accelerator pipeline's upcast, pipeline.py:380-389);
        either way the logits are fp32 sums of the same products. Both accept a torch dtype, a
        name ("bfloat16"), or any object whose ``.name`` is one (a MAX ``DType``)."""
        self.config = config
        if _dtype_name(dtype) not in (None, "bfloat16"):
            raise ConfigError(f"UocrMoE: dtype {_dtype_name(dtype)} (this build holds the non-expert weights in bfloat16)")
        if _dtype_name(norm_router_dtype) not in (None, "bfloat16", "float32"):
            raise ConfigError(f"UocrMoE: norm_router_dtype {_dtype_name(norm_router_dtype)} (bfloat16 or float32)")
        self.dtype = torch.bfloat16
        self.norm_router_dtype = norm_router_dtype
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("UocrMoE runs on a CUDA device only (no CPU path)")
        self._layer: UocrMoeLayer | None = None
        self._tensors: dict[str, torch.Tensor] = {}
        self._ws: dict[int, torch.Tensor] = {}
        self.bias: torch.Tensor | None = None  # optional fp32 [E] logit bias (benchmark input)

    # ---- weights -----------------------------------------------------------------------
    def load_state_dict(self, state: Mapping[str, torch.Tensor]) -> "UocrMoE":
        """Load the reference's declared names (decoder.py:305-313, 269-271, 507) and pack them."""
        cfg = self.config
        E, H, I, S = cfg.n_routed_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_shared_experts
        dev = self.device
        want = {"gate.gate_score.weight", "experts.gate_proj", "experts.up_proj", "experts.down_proj",
                "shared_experts.gate_proj.weight", "shared_experts.up_proj.weight", "shared_experts.down_proj.weight"}
        if cfg.int8_experts:
            want |= {"experts.gate_proj_scales", "experts.up_proj_scales", "experts.down_proj_scales"}
        missing, extra = sorted(want - set(state)), sorted(set(state) - want)
        if missing or extra:
            raise ValueError(f"MoE weights disagree with the declaration: missing {missing}, unexpected {extra}")

        def on_dev(name: str, dtype: torch.dtype, shape: tuple) -> torch.Tensor:
            t = state[name]
            if tuple(t.shape) != shape:
                raise ValueError(f"{name}: shape {tuple(t.shape)} but the layer declares {shape}")
            if t.dtype != dtype:
                raise ValueError(f"{name}: dtype {t.dtype} but the layer declares {dtype}")
            return t.to(dev).contiguous()

        router = state["gate.gate_score.weight"]
        if router.dtype == torch.float32:  # the shared registry's exact fp32 upcast (pipeline.py:380-389)
            rb = router.to(torch.bfloat16)
            if not torch.equal(rb.float(), router):
                raise ValueError("gate.gate_score.weight: fp32 router values are not bf16-exact")
            router = rb
        if router.dtype != torch.bfloat16 or tuple(router.shape) != (E, H):
            raise ValueError(f"gate.gate_score.weight: expected bf16 [{E}, {H}], got {router.dtype} {tuple(router.shape)}")
        t = {"router": router.to(dev).contiguous()}
        wdt = torch.int8 if cfg.int8_experts else torch.bfloat16
        gate = on_dev("experts.gate_proj", wdt, (E, I, H))
        up = on_dev("experts.up_proj", wdt, (E, I, H))
        G = INT8_GROUP_SIZE
        L = load()
        stream = torch.cuda.current_stream(dev).cuda_stream
        i8 = int(cfg.int8_experts)
        scales = {}
        if cfg.int8_experts:
            scales["gate"] = on_dev("experts.gate_proj_scales", torch.float32, (E, I, H // G))
            scales["up"] = on_dev("experts.up_proj_scales", torch.float32, (E, I, H // G))
            scales["down"] = on_dev("experts.down_proj_scales", torch.float32, (E, H, I // G))
        down = on_dev("experts.down_proj", wdt, (E, H, I))
        ptr = lambda n: scales[n].data_ptr() if n in scales else None  # noqa: E731
        t["w13"] = torch.empty(L.uocr_moe_w13_bytes(E, I, H, G, i8), dtype=torch.uint8, device=dev)
        t["w2"] = torch.empty(L.uocr_moe_w2_bytes(E, H, I, G, i8), dtype=torch.uint8, device=dev)
        check(L.uocr_moe_pack_w13(gate.data_ptr(), up.data_ptr(), ptr("gate"), ptr("up"), E, I, H, G, i8,
                                  t["w13"].data_ptr(), stream))
        check(L.uocr_moe_pack_w2(down.data_ptr(), ptr("down"), E, H, I, G, i8, t["w2"].data_ptr(), stream))
        del scales, down
        sg = _unkblock(state["shared_experts.gate_proj.weight"]).to(dev, torch.bfloat16).contiguous()
        su = _unkblock(state["shared_experts.up_proj.weight"]).to(dev, torch.bfloat16).contiguous()
        sd = _unkblock(state["shared_experts.down_proj.weight"]).to(dev, torch.bfloat16).contiguous()
        if tuple(sg.shape) != (S * I, H) or tuple(su.shape) != (S * I, H) or tuple(sd.shape) != (H, S * I):
            raise ValueError("shared_experts: projections do not match shared_experts_dim")
        t["w13s"] = torch.empty(L.uocr_moe_w13_bytes(S, I, H, G, 0) // 2, dtype=torch.bfloat16, device=dev)
        t["w2s"] = torch.empty(L.uocr_moe_w2_bytes(S, H, I, G, 0) // 2, dtype=torch.bfloat16, device=dev)
        check(L.uocr_moe_pack_shared(sg.data_ptr(), su.data_ptr(), sd.data_ptr(), S, I, H,
                                     t["w13s"].data_ptr(), t["w2s"].data_ptr(), stream))
        torch.cuda.current_stream(dev).synchronize()
        self._tensors = t
        lay = UocrMoeLayer()
        lay.hidden, lay.inter, lay.n_routed, lay.n_shared = H, I, E, S
        lay.top_k, lay.group, lay.int8 = cfg.num_experts_per_tok, INT8_GROUP_SIZE, int(cfg.int8_experts)
        lay.router = t["router"].data_ptr()
        lay.w13, lay.w2 = t["w13"].data_ptr(), t["w2"].data_ptr()
        lay.w13_shared, lay.w2_shared = t["w13s"].data_ptr(), t["w2s"].data_ptr()
        self._layer = lay
        return self

    @classmethod
    def from_checkpoint(cls, checkpoint: Mapping[str, torch.Tensor], layer: int, config: MoEConfig | None = None,
                        *, device: str | torch.device = "cuda") -> "UocrMoE":
        """Decoder layer ``layer``'s MoE from checkpoint tensors named as in the model file
        (``model.layers.{L}.mlp.experts.{E}.{proj}.weight`` [+ ``_scales``], ``...mlp.gate.weight``,
        ``...mlp.shared_experts.{proj}.weight``): stacked and checked as the reference's weight
        adapter does (``weights.moe_layer_state``), then packed. The int8 form is detected from
        the checkpoint; ``config`` (default: the model's MoE fields) must agree with it."""
        from .weights import WeightMappingError, moe_layer_state

        cfg = config or MoEConfig()
        state, int8 = moe_layer_state(checkpoint, layer, num_experts=cfg.n_routed_experts)
        if config is None:
            cfg = MoEConfig(int8_experts=int8)
        elif cfg.int8_experts != int8:
            raise WeightMappingError(
                f"the checkpoint's experts are {'int8' if int8 else 'bfloat16'} but the config declares "
                f"{'int8' if cfg.int8_experts else 'bfloat16'}")
        return cls(cfg, device=device).load_state_dict(state)

    @property
    def layer(self) -> UocrMoeLayer:
        if self._layer is None:
            raise RuntimeError("UocrMoE: load_state_dict first")
        return self._layer

    def workspace(self, B: int) -> torch.Tensor:
        ws = self._ws.get(B)
        if ws is None:
            nbytes = load().uocr_moe_decode_workspace_bytes(ctypes.byref(self.layer), B)
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)  # the control block starts zeroed
            self._ws[B] = ws
        return ws

    # ---- forward ---------------------------------------------------------------------------
    def _check_x(self, x: torch.Tensor) -> torch.Tensor:
        if not isinstance(x, torch.Tensor) or not x.is_cuda:
            raise ValueError("UocrMoE: x must be a CUDA tensor")
        if x.dtype != torch.float32:
            raise TypeError(f"UocrMoE takes an fp32 activation, got {x.dtype}")
        if x.dim() != 2 or x.shape[1] != self.config.hidden_size:
            raise ValueError(f"UocrMoE: x must be [rows, {self.config.hidden_size}], got {tuple(x.shape)}")
        return x.contiguous()

    def check_status(self) -> None:
        """Synchronise and read (clearing) the device status of every workspace of this layer:
        raises :class:`UocrError` (code UOCR_EDEVICE) if a device-side bounded wait of any call
        since the last check gave up. Such a call wrote NaN over its output instead of a result."""
        L = load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for ws in list(self._ws.values()):
            check(L.uocr_moe_device_status(ws.data_ptr(), stream))

    def decode_rows(self, x: torch.Tensor, *, out: torch.Tensor | None = None, ids: torch.Tensor | None = None,
                    wts: torch.Tensor | None = None, check_status: bool = False) -> torch.Tensor:
        """MoE.decode_rows (decoder.py:641-655): routed top-k + shared experts for B rows.
        ``check_status=True`` synchronises after the call and raises if a device-side wait gave
        up (otherwise such a failure shows as NaN output and in :meth:`check_status`)."""
        x = self._check_x(x)
        B = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        if B == 0:
            return out
        stream = torch.cuda.current_stream(x.device).cuda_stream
        L = load()
        k = self.config.num_experts_per_tok
        for b0 in range(0, B, DECODE_MAX_B):
            b1 = min(B, b0 + DECODE_MAX_B)
            nb = b1 - b0
            ws = self.workspace(nb)
            check(L.uocr_moe_decode(
                ctypes.byref(self.layer), x[b0:b1].data_ptr(), nb,
                0 if self.bias is None else self.bias.data_ptr(), out[b0:b1].data_ptr(),
                0 if ids is None else ids[b0:b1].data_ptr(), 0 if wts is None else wts[b0:b1].data_ptr(),
                ws.data_ptr(), ws.numel(), stream))
        if check_status:
            self.check_status()
        return out

    def prefill_workspace(self, T: int) -> torch.Tensor:
        """The prefill scratch for up to ``T`` tokens (kept and grown; its status word starts zeroed)."""
        nbytes = load().uocr_moe_prefill_workspace_bytes(ctypes.byref(self.layer), T)
        if nbytes == 0:
            raise ValueError(f"UocrMoE: no prefill workspace for T={T}")
        ws = self._ws.get(-1)
        if ws is None or ws.numel() < nbytes:
            self._ws.pop(-1, None)
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[-1] = ws
        return ws

    def prefill(self, x: torch.Tensor, *, out: torch.Tensor | None = None, ids: torch.Tensor | None = None,
                wts: torch.Tensor | None = None) -> torch.Tensor:
        """The prefill MoE (decoder.py:657-667, routed part as _routed_native, decoder.py:606-614):
        tokens permuted by expert, grouped bf16 GEMMs on the tensor cores, weighted combine."""
        x = self._check_x(x)
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        if T == 0:
            return out
        ws = self.prefill_workspace(T)
        check(load().uocr_moe_prefill(
            ctypes.byref(self.layer), x.data_ptr(), T, 0 if self.bias is None else self.bias.data_ptr(),
            out.data_ptr(), 0 if ids is None else ids.data_ptr(), 0 if wts is None else wts.data_ptr(),
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream(x.device).cuda_stream))
        return out

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """MoE.__call__ (decoder.py:657-667): the MoE over ``x [T, H]``. Up to DECODE_MAX_B rows
        run the decode kernels (one weight read per selected expert; the activations enter the
        tensor cores as three int8 digit planes per 128-group for int8 experts, exact to 2^-21 of
        the group's largest value, and as two bf16 terms for bf16 weights, exact to about 2^-17
        relative; fp32 accumulation); longer inputs run :meth:`prefill` (bf16 activations into
        grouped bf16 GEMMs) when hidden_size is a multiple of 256."""
        if x.dim() == 2 and x.shape[0] > DECODE_MAX_B and self.config.hidden_size % 256 == 0:
            return self.prefill(x)
        return self.decode_rows(x)

    def route(self, x: torch.Tensor):
        """The gate alone: ``(ids i32[T,k], weights f32[T,k])``."""
        return ops.route(self._check_x(x), self._tensors["router"], self.bias, self.config.num_experts_per_tok)
