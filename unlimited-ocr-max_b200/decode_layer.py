"""A decoder layer's decode step on the library's kernels (DecoderLayer.decode, decoder.py:702-709):

    y  = input_layernorm(h)                                   uocr_residual_rmsnorm
    q|k|v = y @ [Wq; Wk; Wv]^T                                 one tensor-core weight stream
    q, k = RoPE(q, k) at each row's position                    uocr_rope_qkv
    a  = paged attention over the request's cached rows        uocr_paged_decode_attention (stores k, v)
    h  = h + a @ Wo^T ;  y2 = post_attention_layernorm(h)       dense stream, then one fused launch
    h  = h + MoE(y2)                                           the MoE decode kernels, then the add
                                                               (layer 0: the dense FFN, DenseFfn)

:class:`DecoderLayerDecode` holds one layer (its norms, projections and :class:`UocrMoE`, or
:class:`DenseFfn` for layer 0); :class:`DecoderDecodeStack` runs several in order and captures them
in one CUDA graph; :class:`DecoderDecodeStep` is the whole step from token ids to the n-gram-guarded
logits (embedding, every layer, the final norm, lm_head, the guard). The residual
stream, the attention and the KV page pool are fp32 (the reference keeps every activation in fp32);
the pool has the reference's layout ``[pages, 2, layers, 128, heads, head_dim]`` (kv_cache.py).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import ops
from ._lib import check, load
from .dense import DenseProjection
from .moe import UocrMoE


def rope_tables(*, head_dim: int, seq_len: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """``(cos, sin)`` ``[seq_len, head_dim]`` fp32 as the reference builds them (decoder.py:115-123):
    inverse frequencies theta^-(2i / head_dim) over the even indices, positions times those, the
    angles repeated over both halves, cos and sin in fp32."""
    exponent = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32)
    inv_freq = (1.0 / (np.float32(theta) ** (exponent / np.float32(head_dim)))).astype(np.float32)
    positions = np.arange(seq_len, dtype=np.int64).astype(np.float32)
    angles = positions[:, None] * inv_freq[None, :]
    emb = np.concatenate([angles, angles], axis=-1).astype(np.float32)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


class DenseFfn:
    """GatedMlp.decode_rows (decoder.py:276-278), the dense FFN of layer 0: gate and up in one
    weight stream, ``uocr_silu_mul``, then down. Weights bf16, K-blocked as declared
    (``kblocked=True``) or plain ``[out, in]``."""

    def __init__(self, gate_proj, up_proj, down_proj, *, device: str | torch.device = "cuda", kblocked: bool = True):
        dim = 1 if kblocked else 0
        inter = gate_proj.shape[dim]
        hidden = down_proj.shape[dim]
        self.gate_up = DenseProjection(hidden, 2 * inter, kblocked=kblocked, device=device).load_state_dict(
            {"weight": torch.cat([gate_proj.to(device), up_proj.to(device)], dim=dim)})
        self.device = self.gate_up.device
        self.down = DenseProjection(inter, hidden, kblocked=kblocked, device=self.device).load_state_dict(
            {"weight": down_proj})
        self.hidden_size, self.inter = hidden, inter
        self._bufs: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def decode_rows(self, x: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
        B = x.shape[0]
        if B not in self._bufs:
            self._bufs[B] = (torch.empty((B, 2 * self.inter), device=self.device),
                             torch.empty((B, self.inter), device=self.device))
        gu, act = self._bufs[B]
        self.gate_up.decode_rows(x, out=gu)
        ops.silu_mul(gu, out=act)
        return self.down.decode_rows(act, out=out)

    def check_status(self) -> None:
        self.gate_up.check_status()
        self.down.check_status()


class DecoderLayerDecode:
    """One decoder layer's decode step for B requests (decoder.py:702-709, the attention of
    Attention.decode, decoder.py:478-493). Weights: the four bf16 attention projections in the
    reference's K-blocked declaration (``kblocked=True``) or plain ``[out, in]``; the two norm
    weights ``[hidden]``; ``moe`` the layer's loaded :class:`UocrMoE` (or a :class:`DenseFfn`)."""

    def __init__(self, moe: UocrMoE | DenseFfn, *, layer_idx: int, heads: int, q_proj, k_proj, v_proj, o_proj,
                 input_norm: torch.Tensor, post_norm: torch.Tensor, eps: float = 1e-6, kblocked: bool = True):
        self.moe, self.layer_idx, self.heads = moe, int(layer_idx), int(heads)
        self.device = moe.device
        H = moe.hidden_size if isinstance(moe, DenseFfn) else moe.config.hidden_size
        if H % heads:
            raise ValueError("hidden_size is not divisible by the head count")
        self.hidden, self.head_dim, self.eps = H, H // heads, float(eps)
        self.scale = 1.0 / math.sqrt(self.head_dim)
        dim = 1 if kblocked else 0
        self.qkv = DenseProjection(H, 3 * H, kblocked=kblocked, device=self.device).load_state_dict(
            {"weight": torch.cat([w.to(self.device) for w in (q_proj, k_proj, v_proj)], dim=dim)})
        self.o = DenseProjection(H, H, kblocked=kblocked, device=self.device).load_state_dict({"weight": o_proj})
        self.device = self.qkv.device
        self.g_in = input_norm.to(self.device, torch.float32).contiguous()
        self.g_post = post_norm.to(self.device, torch.float32).contiguous()
        self._bufs: dict[int, dict[str, torch.Tensor]] = {}

    def buffers(self, B: int) -> dict[str, torch.Tensor]:
        """The step's intermediate rows for batch B (kept: the last call's values stay readable)."""
        if B not in self._bufs:
            H, dev = self.hidden, self.device
            e = lambda *s: torch.empty(s, device=dev)  # noqa: E731
            self._bufs[B] = {"y": e(B, H), "qkv": e(B, 3 * H), "q": e(B, self.heads, self.head_dim),
                             "k": e(B, self.heads, self.head_dim), "v": e(B, self.heads, self.head_dim),
                             "attn": e(B, self.heads, self.head_dim), "o": e(B, H), "y2": e(B, H), "m": e(B, H)}
        return self._bufs[B]

    def _norm(self, h, add, gamma, y) -> None:
        check(load().uocr_residual_rmsnorm(h.data_ptr(), 0 if add is None else add.data_ptr(),
                                           0 if gamma is None else gamma.data_ptr(), h.shape[0], self.hidden, self.eps,
                                           0 if y is None else y.data_ptr(),
                                           torch.cuda.current_stream(self.device).cuda_stream))

    def decode(self, h: torch.Tensor, *, cos: torch.Tensor, sin: torch.Tensor, kv_pool: torch.Tensor, lut: torch.Tensor,
               write_index: torch.Tensor, attend_len: torch.Tensor) -> torch.Tensor:
        """Advance the residual rows ``h`` (fp32 ``[B, hidden]``, updated in place) through this
        layer; ``cos`` / ``sin`` ``[B, head_dim]`` at each row's position; the page pool, lookup
        table, write indices and attend lengths as ``ops.paged_decode_attention`` takes them."""
        B = h.shape[0]
        t = self.buffers(B)
        self._norm(h, None, self.g_in, t["y"])
        self.qkv.decode_rows(t["y"], out=t["qkv"])
        check(load().uocr_rope_qkv(t["qkv"].data_ptr(), B, self.heads, self.head_dim, cos.data_ptr(), sin.data_ptr(),
                                   t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(),
                                   torch.cuda.current_stream(self.device).cuda_stream))
        ops.paged_decode_attention(t["q"], t["k"], t["v"], kv_pool, self.layer_idx, lut, write_index, attend_len,
                                   self.scale, out=t["attn"])
        self.o.decode_rows(t["attn"].view(B, self.hidden), out=t["o"])
        self._norm(h, t["o"], self.g_post, t["y2"])  # h += attention; y2 = post_attention_layernorm(h)
        self.moe.decode_rows(t["y2"], out=t["m"])
        self._norm(h, t["m"], None, None)  # h += MoE
        return h

    def check_status(self) -> None:
        self.qkv.check_status()
        self.o.check_status()
        self.moe.check_status()


class DecoderDecodeStack:
    """Several :class:`DecoderLayerDecode` in order, eager (``decode``) or from one CUDA graph per
    batch size (``graph``), all reading one page pool."""

    def __init__(self, layers: list[DecoderLayerDecode]):
        if not layers:
            raise ValueError("DecoderDecodeStack: no layers")
        self.layers = list(layers)
        self.device = self.layers[0].device
        self._graphs: dict[int, tuple] = {}

    def decode(self, h, **step) -> torch.Tensor:
        for layer in self.layers:
            layer.decode(h, **step)
        return h

    def graph(self, h: torch.Tensor, **step):
        """Capture (once per B) the step over these exact tensors (``h`` and the step's inputs are
        read and written in place by every replay); returns the graph."""
        B = h.shape[0]
        if B not in self._graphs:
            saved = h.clone()
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self.decode(h, **step)  # warm-up: workspaces and buffers allocated outside the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            h.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.decode(h, **step)
            self._graphs[B] = g
        return self._graphs[B]

    def check_status(self) -> None:
        for layer in self.layers:
            layer.check_status()


class DecoderDecodeStep:
    """The decode step from token ids to logits for B requests: the embedding (``uocr_embed_rows``),
    every decoder layer (UnlimitedOcrDecoder.decode, decoder.py:777-792), the final norm, lm_head
    (one weight stream) and the no-repeat-n-gram guard (``ngram_block``, n read from the device).
    ``graph`` captures it all once per batch size."""

    def __init__(self, embed: torch.Tensor, layers: list[DecoderLayerDecode], final_norm: torch.Tensor,
                 lm_head: torch.Tensor, *, eps: float = 1e-6, kblocked: bool = True):
        self.stack = DecoderDecodeStack(layers)
        self.device = self.stack.device
        self.embed = embed.to(self.device, torch.bfloat16).contiguous()
        self.vocab, self.hidden = self.embed.shape
        self.g_final = final_norm.to(self.device, torch.float32).contiguous()
        self.lm_head = DenseProjection(self.hidden, self.vocab, kblocked=kblocked, device=self.device).load_state_dict(
            {"weight": lm_head})
        self.eps = float(eps)
        self._bufs: dict[int, dict[str, torch.Tensor]] = {}
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def buffers(self, B: int) -> dict[str, torch.Tensor]:
        if B not in self._bufs:
            e = lambda *s: torch.empty(s, device=self.device)  # noqa: E731
            self._bufs[B] = {"h": e(B, self.hidden), "y": e(B, self.hidden), "logits": e(B, self.vocab)}
        return self._bufs[B]

    def __call__(self, ids: torch.Tensor, *, history: torch.Tensor, ngram: torch.Tensor, **step) -> torch.Tensor:
        """``ids [B]`` int32 -> guarded logits ``[B, vocab]`` (a buffer reused by the next call);
        ``history [B, W]`` int32 each request's last W token ids, ``ngram`` an int32 ``[1]`` device
        tensor; ``step`` the attention inputs of :meth:`DecoderLayerDecode.decode`."""
        B = ids.shape[0]
        t = self.buffers(B)
        ops.embed_rows(self.embed, ids, out=t["h"])
        self.stack.decode(t["h"], **step)
        check(load().uocr_residual_rmsnorm(t["h"].data_ptr(), 0, self.g_final.data_ptr(), B, self.hidden, self.eps,
                                           t["y"].data_ptr(), torch.cuda.current_stream(self.device).cuda_stream))
        self.lm_head.decode_rows(t["y"], out=t["logits"])
        ops.ngram_block(t["logits"], history, ngram, out=t["logits"])
        return t["logits"]

    def graph(self, ids: torch.Tensor, **step) -> torch.cuda.CUDAGraph:
        """Capture (once per B) the step over these exact tensors; replaying it reads ``ids`` and the
        step's inputs and writes the logits buffer (and the page pool) in place."""
        B = ids.shape[0]
        if B not in self._graphs:
            pool = step.get("kv_pool")
            saved = pool.clone() if pool is not None else None
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self(ids, **step)  # warm-up: every buffer and workspace allocated outside the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            if saved is not None:
                pool.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self(ids, **step)
            self._graphs[B] = g
        return self._graphs[B]

    def check_status(self) -> None:
        self.stack.check_status()
        self.lm_head.check_status()
