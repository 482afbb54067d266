"""The MoE half of the decoder's decode step: every MoE layer's post-attention RMSNorm, the MoE
sublayer and the residual add, as one CUDA graph.

Per layer l (DecoderLayer.decode, decoder.py:702-709, after its attention):

    h = h + MoE_l.decode_rows(RmsNorm_l(h))

:class:`MoEDecodeStack` holds the layers' :class:`UocrMoE` and their ``post_attention_layernorm``
weights. One step is 3 launches per layer: the fused residual-add + RMSNorm
(``uocr_residual_rmsnorm``: the previous layer's output added into h, the next layer's input
normalised) and the MoE's two decode kernels; a last launch adds the final layer's output.
``graph(B)`` captures the whole step once for a batch size; ``step(h)`` replays it. The residual
stream is fp32, the norm weights are cast from bf16 to fp32 as RmsNorm does (decoder.py:261).
"""

from __future__ import annotations

import torch

from ._lib import check, load
from .moe import UocrMoE


class MoEDecodeStack:
    """``h -> h + MoE_l(RmsNorm_l(h))`` over the given layers, eager (``decode_rows``) or replayed
    from a CUDA graph (``graph`` / ``step``)."""

    def __init__(self, layers: list[UocrMoE], norm_weights: list[torch.Tensor], *, eps: float = 1e-6):
        if not layers or len(layers) != len(norm_weights):
            raise ValueError(f"MoEDecodeStack: {len(layers)} layers and {len(norm_weights)} norm weights")
        self.layers = list(layers)
        self.device = self.layers[0].device
        H = self.layers[0].config.hidden_size
        for m in self.layers:
            if m.config.hidden_size != H or m.device != self.device:
                raise ValueError("MoEDecodeStack: every layer needs the same hidden size and device")
        self.hidden = H
        self.eps = float(eps)
        self.gammas = []
        for g in norm_weights:
            if tuple(g.shape) != (H,):
                raise ValueError(f"MoEDecodeStack: a norm weight of shape {tuple(g.shape)}, expected ({H},)")
            self.gammas.append(g.to(self.device, torch.float32).contiguous())
        self._graphs: dict[int, tuple] = {}

    def _norm(self, h: torch.Tensor, add: torch.Tensor | None, gamma: torch.Tensor | None,
              y: torch.Tensor | None) -> None:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(load().uocr_residual_rmsnorm(h.data_ptr(), 0 if add is None else add.data_ptr(),
                                           0 if gamma is None else gamma.data_ptr(), h.shape[0], self.hidden,
                                           self.eps, 0 if y is None else y.data_ptr(), stream))

    def _run(self, hs: list[torch.Tensor], ys: list[torch.Tensor], outs: list[torch.Tensor]) -> None:
        """hs[0] -> hs[L]: ys[l] = RmsNorm_l(hs[l]), outs[l] = MoE_l(ys[l]), hs[l + 1] = hs[l] + outs[l]
        (the add and the next norm in one launch). The h buffers may all be one storage."""
        L = len(self.layers)
        self._norm(hs[0], None, self.gammas[0], ys[0])
        for l in range(L):
            self.layers[l].decode_rows(ys[l], out=outs[l])
            if hs[l + 1].data_ptr() != hs[l].data_ptr():
                hs[l + 1].copy_(hs[l])
            last = l + 1 == L
            self._norm(hs[l + 1], outs[l], None if last else self.gammas[l + 1], None if last else ys[l + 1])

    def _buffers(self, B: int, keep: bool):
        L, H, dev = len(self.layers), self.hidden, self.device
        if keep:
            hs = [torch.empty((B, H), device=dev) for _ in range(L + 1)]
        else:
            one = torch.empty((B, H), device=dev)
            hs = [one] * (L + 1)
        ys = [torch.empty((B, H), device=dev) for _ in range(L)]
        outs = [torch.empty((B, H), device=dev) for _ in range(L)]
        return hs, ys, outs

    def decode_rows(self, h: torch.Tensor, *, keep_intermediates: bool = False):
        """One step for fp32 rows ``h [B, H]``; returns the new h, or with ``keep_intermediates``
        ``(hs, ys, outs)``: every layer's residual input, normalised input and MoE output."""
        if h.dtype != torch.float32 or h.dim() != 2 or h.shape[1] != self.hidden or h.device != self.device:
            raise ValueError(f"MoEDecodeStack: h must be fp32 [B, {self.hidden}] on {self.device}")
        hs, ys, outs = self._buffers(h.shape[0], keep_intermediates)
        hs[0].copy_(h)
        self._run(hs, ys, outs)
        return (hs, ys, outs) if keep_intermediates else hs[-1].clone()

    def graph(self, B: int):
        """Capture (once per B) the whole step; returns ``(graph, h_in_out)``: copy the rows into
        ``h_in_out``, replay, read the new rows from it."""
        if B not in self._graphs:
            hs, ys, outs = self._buffers(B, False)
            hs[0].zero_()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self._run(hs, ys, outs)  # warm-up: workspaces allocated outside the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._run(hs, ys, outs)
            self._graphs[B] = (g, hs[0], ys, outs)
        g, h_io, _, _ = self._graphs[B]
        return g, h_io

    def step(self, h: torch.Tensor) -> torch.Tensor:
        """One step through the captured graph (captured on first use for this B)."""
        g, h_io = self.graph(h.shape[0])
        h_io.copy_(h)
        g.replay()
        return h_io.clone()

    def check_status(self) -> None:
        for m in self.layers:
            m.check_status()
