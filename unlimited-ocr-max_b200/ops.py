"""torch-tensor wrappers over the C ABI, one per reference op.

Each wrapper takes the same tensors as the reference's custom op (kernels/*.mojo
``@register``) or graph function, checks device and dtype, and passes raw device pointers
plus the current CUDA stream to ``libuocr_moe.so``. Shape errors come back from the library
with the reference op's message and are raised as ``ValueError``. Nothing here computes on
the host; a non-CUDA tensor is an error, never a CPU fallback.
"""

from __future__ import annotations

import torch

from ._lib import check, load

KBLOCK = 16  # decoder.py:72


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(op: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{op}: every tensor must be a CUDA tensor (no CPU path)")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"{op}: tensors on different devices ({dev} vs {t.device})")


def _need(op: str, t: torch.Tensor, name: str, dtype: torch.dtype, rank: int) -> torch.Tensor:
    if t.dtype != dtype:
        raise TypeError(f"{op}: {name} must be {dtype}, got {t.dtype}")
    if t.dim() != rank:
        raise ValueError(f"{op}: {name} must be rank {rank}, got shape {tuple(t.shape)}")
    return t if t.is_contiguous() else t.contiguous()


def moe_bf16_qmv(x: torch.Tensor, expert_ids: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``moe_bf16_qmv(x f32[k,K], ids i32[k], w bf16[E,N,K]) -> f32[k,N]`` (kernels/moe_bf16.mojo:264)."""
    op = "moe_bf16_qmv"
    _need_cuda(op, x, expert_ids, w)
    x = _need(op, x, "x", torch.float32, 2)
    expert_ids = _need(op, expert_ids, "expert_ids", torch.int32, 1)
    w = _need(op, w, "w", torch.bfloat16, 3)
    if out is None:
        out = torch.empty((x.shape[0], w.shape[1]), dtype=torch.float32, device=x.device)
    out = _need(op, out, "output", torch.float32, 2)
    check(load().uocr_moe_bf16_qmv(
        out.data_ptr(), out.shape[0], out.shape[1], x.data_ptr(), x.shape[0], x.shape[1],
        expert_ids.data_ptr(), expert_ids.shape[0], w.data_ptr(), *w.shape, _stream(x)))
    return out


def moe_int8_qmv(x: torch.Tensor, expert_ids: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """``moe_int8_qmv(x, ids, w i8[E,N,K], scales f32[E,N,K/G]) -> f32[k,N]`` (kernels/moe_int8.mojo:181)."""
    op = "moe_int8_qmv"
    _need_cuda(op, x, expert_ids, w, scales)
    x = _need(op, x, "x", torch.float32, 2)
    expert_ids = _need(op, expert_ids, "expert_ids", torch.int32, 1)
    w = _need(op, w, "w", torch.int8, 3)
    scales = _need(op, scales, "scales", torch.float32, 3)
    if out is None:
        out = torch.empty((x.shape[0], w.shape[1]), dtype=torch.float32, device=x.device)
    out = _need(op, out, "output", torch.float32, 2)
    check(load().uocr_moe_int8_qmv(
        out.data_ptr(), out.shape[0], out.shape[1], x.data_ptr(), x.shape[0], x.shape[1],
        expert_ids.data_ptr(), expert_ids.shape[0], w.data_ptr(), *w.shape, scales.data_ptr(), *scales.shape,
        _stream(x)))
    return out


def int8_dequant_expert(w: torch.Tensor, scales: torch.Tensor, expert_idx: torch.Tensor,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """``int8_dequant_expert(w, scales, idx i32[1]) -> bf16[N,K]`` (kernels/moe_int8.mojo:261)."""
    op = "int8_dequant_expert"
    _need_cuda(op, w, scales, expert_idx)
    w = _need(op, w, "w", torch.int8, 3)
    scales = _need(op, scales, "scales", torch.float32, 3)
    expert_idx = _need(op, expert_idx, "expert_idx", torch.int32, 1)
    if out is None:
        out = torch.empty((w.shape[1], w.shape[2]), dtype=torch.bfloat16, device=w.device)
    out = _need(op, out, "output", torch.bfloat16, 2)
    check(load().uocr_int8_dequant_expert(
        out.data_ptr(), out.shape[0], out.shape[1], w.data_ptr(), *w.shape, scales.data_ptr(), *scales.shape,
        expert_idx.data_ptr(), expert_idx.shape[0], _stream(w)))
    return out


def dense_bf16_qmv(x: torch.Tensor, w: torch.Tensor, *, tile: int | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """``dense_bf16_qmv[tile](x f32[M,K], w bf16[K/16,N,16]) -> f32[M,N]`` (kernels/dense_bf16.mojo:119)."""
    op = "dense_bf16_qmv"
    _need_cuda(op, x, w)
    x = _need(op, x, "x", torch.float32, 2)
    w = _need(op, w, "w", torch.bfloat16, 3)
    if out is None:
        out = torch.empty((x.shape[0], w.shape[1]), dtype=torch.float32, device=x.device)
    out = _need(op, out, "output", torch.float32, 2)
    check(load().uocr_dense_bf16_qmv(
        out.data_ptr(), out.shape[0], out.shape[1], x.data_ptr(), x.shape[0], x.shape[1],
        w.data_ptr(), *w.shape, 1 if tile is None else int(tile), _stream(x)))
    return out


class QuantizeError(RuntimeError):
    """A refusal of the int8 quantiser, with the reference tool's message
    (tools/quantize_int8.py:77-78)."""


def quantize_per_group(w: torch.Tensor, group: int = 128, *, q: torch.Tensor | None = None,
                       scales: torch.Tensor | None = None, check_finite: bool = True):
    """``[..., N, K]`` bf16 or fp32 -> ``(int8 [..., N, K], fp32 [..., N, K / 128])`` on the GPU.

    The symmetric per-group format of tools/quantize_int8.py:298-329 with its exact bits: amax =
    max|w| per 128 elements along K, scale = amax / 127 (1.0 for an all-zero group), q =
    clip(rint(w / scale), -127, 127). The reference takes one ``[N, K]`` weight; leading dims
    here are a stack of them. ``check_finite`` reads the device's non-finite flag (one
    synchronisation) and refuses a weight holding NaN or Inf as the reference does.
    """
    op = "quantize_per_group"
    _need_cuda(op, w)
    if w.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"{op}: w must be bf16 or fp32, got {w.dtype}")
    if w.dim() < 2:
        raise QuantizeError(f"expected a 2-D weight, got shape {tuple(w.shape)}")
    if group != 128:
        raise ValueError(f"{op}: this build quantises groups of 128, got {group}")
    k = w.shape[-1]
    if k % group:
        raise QuantizeError(f"K={k} is not divisible by the group size {group}")
    w = w if w.is_contiguous() else w.contiguous()
    rows = w.numel() // k if k else 0
    if q is None:
        q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    if scales is None:
        scales = torch.empty((*w.shape[:-1], k // group), dtype=torch.float32, device=w.device)
    if q.dtype != torch.int8 or tuple(q.shape) != tuple(w.shape) or not q.is_contiguous():
        raise ValueError(f"{op}: q must be a contiguous int8 tensor of shape {tuple(w.shape)}")
    if (scales.dtype != torch.float32 or tuple(scales.shape) != (*w.shape[:-1], k // group)
            or not scales.is_contiguous()):
        raise ValueError(f"{op}: scales must be a contiguous fp32 tensor of shape {(*w.shape[:-1], k // group)}")
    _need_cuda(op, w, q, scales)
    flag = torch.zeros(1, dtype=torch.int32, device=w.device)
    check(load().uocr_quantize_int8_g128(w.data_ptr(), 1 if w.dtype == torch.bfloat16 else 0, rows, k,
                                         q.data_ptr(), scales.data_ptr(), flag.data_ptr(), _stream(w)))
    if check_finite and int(flag.item()):
        raise QuantizeError("weight holds NaN or Inf; refusing to quantise it")
    return q, scales


def route(x: torch.Tensor, router: torch.Tensor, bias: torch.Tensor | None = None, top_k: int = 6):
    """MoEGate.__call__ (decoder.py:509-514): ``(ids i32[T,k], weights f32[T,k])`` in score order.

    ``router`` is the bf16 ``gate.gate_score.weight [E, H]``; ``bias`` an optional fp32 ``[E]``
    added to the logits before the softmax (a benchmark input; the reference has none).
    """
    op = "route"
    _need_cuda(op, x, router, *([] if bias is None else [bias]))
    x = _need(op, x, "x", torch.float32, 2)
    router = _need(op, router, "router", torch.bfloat16, 2)
    if bias is not None:
        bias = _need(op, bias, "bias", torch.float32, 1)
    T, H = x.shape
    E = router.shape[0]
    if router.shape[1] != H:
        raise ValueError(f"route: router and x disagree on the hidden size ({router.shape[1]} vs {H})")
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    wts = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    check(load().uocr_moe_route(x.data_ptr(), T, H, router.data_ptr(), E, 0 if bias is None else bias.data_ptr(),
                                top_k, ids.data_ptr(), wts.data_ptr(), _stream(x)))
    return ids, wts


def ngram_block(logits: torch.Tensor, history: torch.Tensor, ngram: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``ngram_block(logits f32[V] or [B,V], history i32[H] or [B,H], ngram i32[1])`` (kernels/
    ngram_block.mojo:51-151): row b's tokens that would repeat an n-gram of row b's history set
    to -3.0e38, every other logit copied bit for bit. ``out`` may be ``logits`` (in place)."""
    op = "ngram_block"
    _need_cuda(op, logits, history, ngram)
    if logits.dim() not in (1, 2):
        raise ValueError(f"{op} takes one row (V,) or B rows (B, V), got shape {tuple(logits.shape)}")
    rank = logits.dim()
    logits = _need(op, logits, "logits", torch.float32, rank)
    history = _need(op, history, "history", torch.int32, rank)
    ngram = _need(op, ngram, "ngram", torch.int32, 1)
    if ngram.shape[0] != 1:
        raise ValueError("ngram_block: `ngram` must be a single int32")
    if rank == 2 and history.shape[0] != logits.shape[0]:
        raise ValueError("ngram_block: history and logits disagree on the row count")
    if out is None:
        out = torch.empty_like(logits)
    if out.dtype != torch.float32 or out.shape != logits.shape or not out.is_contiguous():
        raise ValueError("ngram_block: logits and output disagree on shape")
    B = logits.shape[0] if rank == 2 else 1
    check(load().uocr_ngram_block(logits.data_ptr(), B, logits.shape[-1], history.data_ptr(), history.shape[-1],
                                  ngram.data_ptr(), out.data_ptr(), _stream(logits)))
    return out


_ATTN_WS: dict[tuple, torch.Tensor] = {}


def paged_decode_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, kv_pool: torch.Tensor,
                           layer: int, lut: torch.Tensor, write_index: torch.Tensor, attend_len: torch.Tensor,
                           scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """paged_decode_attention (decoder.py:425-437): store each request's new k/v row at its write
    index of ``layer`` in ``kv_pool`` fp32 ``[pages, 2, layers, 128, heads, 128]`` and attend ``q``
    ``[B, heads, 128]`` over its rows ``[0, attend_len)`` (``lut`` uint32/int32 ``[B, cols]`` page ids,
    ``write_index`` / ``attend_len`` ``[B]``). The workspace is kept per (device, B, heads, cols)."""
    op = "paged_decode_attention"
    _need_cuda(op, q, k_new, v_new, kv_pool, lut, write_index, attend_len)
    q = _need(op, q, "q", torch.float32, 3)
    k_new = _need(op, k_new, "k_new", torch.float32, 3)
    v_new = _need(op, v_new, "v_new", torch.float32, 3)
    kv_pool = _need(op, kv_pool, "kv_pool", torch.float32, 6)
    B, heads, dim = q.shape
    if k_new.shape != q.shape or v_new.shape != q.shape:
        raise ValueError(f"{op}: q, k_new and v_new disagree on shape")
    pages, two, layers, rows, ph, pd = kv_pool.shape
    if two != 2 or rows != 128 or ph != heads or pd != dim:
        raise ValueError(f"{op}: the pool must be [pages, 2, layers, 128, {heads}, {dim}], got {tuple(kv_pool.shape)}")
    for name, t in (("lut", lut), ("write_index", write_index), ("attend_len", attend_len)):
        if t.dtype not in (torch.int32, torch.uint32):
            raise TypeError(f"{op}: {name} must be int32 or uint32, got {t.dtype}")
    lut = lut.contiguous()
    if lut.dim() != 2 or lut.shape[0] != B or write_index.shape != (B,) or attend_len.shape != (B,):
        raise ValueError(f"{op}: lut [B, cols], write_index [B] and attend_len [B] expected")
    if out is None:
        out = torch.empty_like(q)
    key = (q.device, B, heads, lut.shape[1])
    ws = _ATTN_WS.get(key)
    if ws is None:
        ws = torch.zeros(load().uocr_paged_attention_workspace_bytes(B, heads, lut.shape[1]), dtype=torch.uint8,
                         device=q.device)
        _ATTN_WS[key] = ws
    check(load().uocr_paged_decode_attention(
        q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), B, heads, dim, kv_pool.data_ptr(), pages, layers, layer,
        lut.data_ptr(), lut.shape[1], write_index.contiguous().data_ptr(), attend_len.contiguous().data_ptr(),
        float(scale), out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(q)))
    return out


def embed_rows(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """The token embedding (EmbeddingTable, decoder.py:241-249): fp32 rows of the bf16 ``table
    [vocab, hidden]`` at ``ids [B]`` (int32, clamped into the vocabulary)."""
    op = "embed_rows"
    _need_cuda(op, table, ids)
    table = _need(op, table, "table", torch.bfloat16, 2)
    ids = _need(op, ids, "ids", torch.int32, 1)
    if out is None:
        out = torch.empty((ids.shape[0], table.shape[1]), dtype=torch.float32, device=table.device)
    check(load().uocr_embed_rows(table.data_ptr(), table.shape[0], table.shape[1], ids.data_ptr(), ids.shape[0],
                                 out.data_ptr(), _stream(table)))
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(g) * u on the fused gate|up rows ``[B, 2 x inter]`` (GatedMlp.decode_rows, decoder.py:276-278)."""
    op = "silu_mul"
    _need_cuda(op, gate_up)
    gate_up = _need(op, gate_up, "gate_up", torch.float32, 2)
    if gate_up.shape[1] % 2:
        raise ValueError(f"{op}: gate_up must hold gate and up halves, got {gate_up.shape[1]} columns")
    inter = gate_up.shape[1] // 2
    if out is None:
        out = torch.empty((gate_up.shape[0], inter), dtype=torch.float32, device=gate_up.device)
    check(load().uocr_silu_mul(gate_up.data_ptr(), gate_up.shape[0], inter, out.data_ptr(), _stream(gate_up)))
    return out
