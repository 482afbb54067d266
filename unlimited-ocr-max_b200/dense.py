"""The decode step's dense bf16 projections on the tensor-core weight stream.

:class:`DenseProjection` mirrors the reference's ``Projection`` (decoder.py:189-238): a bias-free
``W [out_dim, in_dim]`` applied as ``x @ W.T`` to fp32 rows, its weight declared K-blocked as
``[in_dim / 16, out_dim, 16]`` (``kblocked=True``, the layout ``dense_bf16_qmv`` reads) or plain
``[out_dim, in_dim]``. ``load_state_dict`` packs the weight once into the library's streaming
layout (``uocr_dense_pack``); ``decode_rows`` -- the decode step's rows, the reference's
``dense_bf16_qmv`` call -- runs ``uocr_dense_stream``, which reads the weight once per 8 rows
through the tensor cores. The attention projections (q/k/v/o), the dense FFN of layer 0 and
lm_head of the decoder are all of this kind.
"""

from __future__ import annotations

from collections.abc import Mapping

import torch

from ._lib import check, load
from .moe import _dtype_name

KBLOCK = 16  # decoder.py:72


class DenseProjection:
    """``Projection.decode_rows`` (decoder.py:236-238) through ``uocr_dense_stream``."""

    def __init__(self, in_dim: int, out_dim: int, *, dtype=None, device: str | torch.device = "cuda",
                 kblocked: bool = True):
        if dtype is not None and _dtype_name(dtype) not in ("bfloat16", "bf16"):
            raise ValueError(f"DenseProjection: the weight is bf16, got dtype {dtype}")
        if in_dim % KBLOCK:
            raise ValueError(f"a K-blocked projection needs in_dim to be a multiple of {KBLOCK}, got {in_dim}")
        if out_dim < 1:
            raise ValueError(f"DenseProjection: out_dim must be >= 1, got {out_dim}")
        self.in_dim, self.out_dim, self.kblocked = int(in_dim), int(out_dim), bool(kblocked)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DenseProjection: the weight stream runs on a CUDA device (no CPU path)")
        self._packed: torch.Tensor | None = None
        self._ws: torch.Tensor | None = None

    @property
    def weight_shape(self) -> tuple[int, ...]:
        """The declared weight shape (decoder.py:225)."""
        if self.kblocked:
            return (self.in_dim // KBLOCK, self.out_dim, KBLOCK)
        return (self.out_dim, self.in_dim)

    def load_state_dict(self, state: Mapping[str, torch.Tensor]) -> "DenseProjection":
        w = state["weight"]
        if w.dtype != torch.bfloat16:
            raise TypeError(f"DenseProjection: weight must be bfloat16, got {w.dtype}")
        if tuple(w.shape) != self.weight_shape:
            raise ValueError(f"DenseProjection: weight of shape {tuple(w.shape)}, declared {self.weight_shape}")
        w = w.to(self.device).contiguous()
        self.device = w.device  # "cuda" resolved to the current device's index
        lib = load()
        n, k = self.out_dim, self.in_dim
        with torch.cuda.device(self.device):
            packed = torch.empty(lib.uocr_dense_packed_bytes(n, k), dtype=torch.uint8, device=self.device)
            stream = torch.cuda.current_stream(self.device)
            check(lib.uocr_dense_pack(w.data_ptr(), int(self.kblocked), n, k, packed.data_ptr(), stream.cuda_stream))
            self._ws = torch.zeros(lib.uocr_dense_stream_workspace_bytes(n, k), dtype=torch.uint8, device=self.device)
            stream.synchronize()
        self._packed = packed
        return self

    def decode_rows(self, x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        """``x @ W.T`` for fp32 ``x [M, in_dim]`` -> fp32 ``[M, out_dim]`` (8 rows per weight pass)."""
        if self._packed is None:
            raise RuntimeError("DenseProjection: load_state_dict first")
        if not isinstance(x, torch.Tensor) or x.device != self.device:
            raise ValueError(f"DenseProjection: x must be a tensor on {self.device}")
        if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != self.in_dim:
            raise ValueError(f"DenseProjection: x must be fp32 [M, {self.in_dim}], got {x.dtype} {tuple(x.shape)}")
        x = x.contiguous()
        if out is None:
            out = torch.empty((x.shape[0], self.out_dim), dtype=torch.float32, device=self.device)
        if out.dtype != torch.float32 or tuple(out.shape) != (x.shape[0], self.out_dim) or not out.is_contiguous():
            raise ValueError(f"DenseProjection: out must be a contiguous fp32 [{x.shape[0]}, {self.out_dim}]")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(load().uocr_dense_stream(self._packed.data_ptr(), self.out_dim, self.in_dim, x.data_ptr(), x.shape[0],
                                       out.data_ptr(), self._ws.data_ptr(), self._ws.numel(), stream))
        return out

    __call__ = decode_rows

    def check_status(self) -> None:
        """Raise if a device-side wait of the calls since the last check gave up (synchronises)."""
        if self._ws is not None:
            check(load().uocr_moe_device_status(self._ws.data_ptr(),
                                                torch.cuda.current_stream(self.device).cuda_stream))


class FusedProjection(DenseProjection):
    """Several projections of the same input in one weight stream: the decoder's q/k/v projections
    (decoder.py:141-238, three ``dense_bf16_qmv`` calls on one normalised row) or the dense FFN's
    gate and up projections. The weights are concatenated along ``out_dim`` at load, so one launch
    reads all of them; ``decode_rows`` returns one ``[M, out_dim_i]`` view per part."""

    def __init__(self, in_dim: int, out_dims, *, dtype=None, device: str | torch.device = "cuda",
                 kblocked: bool = True):
        self.out_dims = [int(d) for d in out_dims]
        if not self.out_dims or min(self.out_dims) < 1:
            raise ValueError(f"FusedProjection: need at least one positive out_dim, got {out_dims}")
        super().__init__(in_dim, sum(self.out_dims), dtype=dtype, device=device, kblocked=kblocked)

    def load_weights(self, weights) -> "FusedProjection":
        """One declared-shape weight per part (K-blocked ``[in_dim/16, out_dim_i, 16]`` or plain
        ``[out_dim_i, in_dim]``), in order."""
        if len(weights) != len(self.out_dims):
            raise ValueError(f"FusedProjection: {len(self.out_dims)} parts, got {len(weights)} weights")
        dim = 1 if self.kblocked else 0
        for w, d in zip(weights, self.out_dims):
            want = (self.in_dim // KBLOCK, d, KBLOCK) if self.kblocked else (d, self.in_dim)
            if tuple(w.shape) != want:
                raise ValueError(f"FusedProjection: weight of shape {tuple(w.shape)}, declared {want}")
        fused = torch.cat([w.to(self.device) for w in weights], dim=dim)
        return self.load_state_dict({"weight": fused})

    def decode_rows(self, x: torch.Tensor, *, out: torch.Tensor | None = None):
        full = super().decode_rows(x, out=out)
        return tuple(torch.split(full, self.out_dims, dim=1))

    __call__ = decode_rows
