"""The model file on disk: safetensors reading and writing, the MoE loader, and the int8 checkpoint
quantiser running on the GPU.

* :func:`read_header` / :class:`SafetensorsFile` read a ``.safetensors`` file (8 bytes of
  little-endian header length, a JSON header ``name -> {dtype, shape, data_offsets}`` plus
  ``__metadata__``, then the data buffer) with the format's invariants checked: known dtypes,
  byte spans equal to shape x item size, offsets ascending and gap-free from 0. Tensors are read
  one at a time through a memory map, so loading one decoder layer of the 6.7 GB file touches
  only that layer's bytes.
* :func:`load_moe_layer` builds :class:`UocrMoE` for one decoder layer straight from the file:
  the whole file's expert names and dtypes are checked for a half-quantised checkpoint from the
  header alone (weight_adapters.py:187-219, 278-292), then only that layer's tensors are read,
  stacked and packed. ``quantize="int8"`` turns a bf16 file's routed experts into the int8 form
  on the GPU, with the bits the published int8 file holds.
* :func:`quantize_checkpoint` is tools/quantize_int8.py's ``quantize_file`` (:490-640) with the
  quantisation on the GPU (``ops.quantize_per_group``): every routed expert weight
  ``model.layers.{L}.mlp.experts.{E}.{proj}.weight`` (bf16 ``[N, K]``) becomes int8 plus an fp32
  ``...weight_scales`` ``[N, K / 128]``, every other tensor is copied byte for byte, the output
  holds its tensors in sorted-name order with the source's metadata plus ``group_size``,
  ``scheme``, ``source_sha256`` and ``tool``, and the refusals are the tool's (an expert weight
  that is not bf16 or not 2-D, K not a multiple of 128, scales already present, nothing to
  quantise, a source whose sha256 is not the pinned one). Given the tool's name as ``tool``, the
  output file is byte-identical to the tool's.
"""

from __future__ import annotations

import hashlib
import json
import mmap
import os
import re
import struct
from collections.abc import Iterator, Mapping
from pathlib import Path

import numpy as np
import torch

from .ops import QuantizeError, quantize_per_group

__all__ = ["SafetensorsError", "read_header", "SafetensorsFile", "write_safetensors", "load_moe_layer",
           "quantize_checkpoint", "QuantizeError", "TOOL", "SCHEME", "GROUP_SIZE"]

TOOL = "uocr_moe quantize_checkpoint 1.0"
SCHEME = "symmetric-int8-per-group-k"
GROUP_SIZE = 128
SCALES_SUFFIX = "_scales"
MAX_HEADER_BYTES = 100_000_000
COPY_CHUNK = 2 << 20

#: safetensors dtype name -> (item size, torch dtype)
DTYPES: dict[str, tuple[int, torch.dtype]] = {
    "BOOL": (1, torch.bool), "U8": (1, torch.uint8), "I8": (1, torch.int8),
    "F8_E4M3": (1, torch.float8_e4m3fn), "F8_E5M2": (1, torch.float8_e5m2),
    "I16": (2, torch.int16), "U16": (2, torch.uint16), "F16": (2, torch.float16), "BF16": (2, torch.bfloat16),
    "I32": (4, torch.int32), "U32": (4, torch.uint32), "F32": (4, torch.float32),
    "I64": (8, torch.int64), "U64": (8, torch.uint64), "F64": (8, torch.float64),
}
_NAME_OF = {dt: name for name, (_, dt) in DTYPES.items()}

#: A routed expert's weight in the model file (the quantiser's selection rule: by name, never by
#: shape; ``shared_experts`` and stacked ``experts.{proj}`` names do not match).
CHECKPOINT_EXPERT_RE = re.compile(
    r"^model\.layers\.(?P<layer>\d+)\.mlp\.experts\.(?P<expert>\d+)\.(?P<proj>gate_proj|up_proj|down_proj)\.weight$")


class SafetensorsError(QuantizeError):
    """A file that is not a well-formed safetensors file."""


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def read_header(fh) -> tuple[dict, dict, int]:
    """``(metadata, {name: entry}, data_start)`` of an open binary file, validated."""
    raw = fh.read(8)
    if len(raw) != 8:
        raise SafetensorsError("not a safetensors file: shorter than 8 bytes")
    (size,) = struct.unpack("<Q", raw)
    if not 0 < size <= MAX_HEADER_BYTES:
        raise SafetensorsError(f"implausible safetensors header length {size}")
    blob = fh.read(size)
    if len(blob) != size:
        raise SafetensorsError(f"truncated safetensors header: wanted {size} bytes, got {len(blob)}")
    try:
        header = json.loads(blob)
    except json.JSONDecodeError as exc:
        raise SafetensorsError(f"safetensors header is not JSON: {exc}") from exc
    if not isinstance(header, dict):
        raise SafetensorsError("safetensors header is not a JSON object")
    metadata = header.pop("__metadata__", {})
    if not isinstance(metadata, dict):
        raise SafetensorsError("__metadata__ is not a JSON object")
    for name, entry in header.items():
        if not isinstance(entry, dict):
            raise SafetensorsError(f"{name}: header entry is not an object")
        dtype, shape, offs = entry.get("dtype"), entry.get("shape"), entry.get("data_offsets")
        if dtype not in DTYPES:
            raise SafetensorsError(f"{name}: unknown safetensors dtype {dtype!r}")
        if not isinstance(shape, list) or not all(isinstance(d, int) and d >= 0 for d in shape):
            raise SafetensorsError(f"{name}: bad shape {shape!r}")
        if (not isinstance(offs, list) or len(offs) != 2 or not all(isinstance(o, int) for o in offs)
                or offs[0] > offs[1]):
            raise SafetensorsError(f"{name}: bad data_offsets {offs!r}")
        want = DTYPES[dtype][0] * _numel(shape)
        if offs[1] - offs[0] != want:
            raise SafetensorsError(f"{name}: {dtype}{shape} needs {want} bytes but the header spans {offs[1] - offs[0]}")
    end = 0
    for name, entry in sorted(header.items(), key=lambda kv: kv[1]["data_offsets"]):
        start, stop = entry["data_offsets"]
        if start != end:
            raise SafetensorsError(f"{name}: data_offsets start at {start}, expected {end} "
                                   "(safetensors buffers are gap-free and ordered)")
        end = stop
    return metadata, header, 8 + size


class SafetensorsFile(Mapping):
    """A read-only ``name -> torch.Tensor`` view of a safetensors file; each lookup reads that
    tensor's bytes (a CPU tensor owning a copy, or one on ``device``). ``meta()`` gives every tensor
    as a data-less ``meta`` tensor (name, dtype and shape only)."""

    def __init__(self, path: str | os.PathLike, *, device: str | torch.device = "cpu"):
        self.path = Path(path)
        self.device = torch.device(device)
        with open(self.path, "rb") as fh:
            self.metadata, self.entries, self.data_start = read_header(fh)
            size = os.fstat(fh.fileno()).st_size
            end = max((e["data_offsets"][1] for e in self.entries.values()), default=0)
            if self.data_start + end > size:
                raise SafetensorsError(f"{self.path}: the header spans {self.data_start + end} bytes, the file has {size}")
            self._mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ) if size else None

    def __getitem__(self, name: str) -> torch.Tensor:
        entry = self.entries[name]
        _, dt = DTYPES[entry["dtype"]]
        start, stop = entry["data_offsets"]
        if stop == start:
            return torch.empty(entry["shape"], dtype=dt, device=self.device)
        raw = np.frombuffer(self._mm, dtype=np.uint8, count=stop - start, offset=self.data_start + start)
        t = torch.from_numpy(raw.copy()).view(dt).reshape(entry["shape"])
        return t if self.device.type == "cpu" else t.to(self.device)

    def raw_bytes(self, name: str) -> bytes:
        start, stop = self.entries[name]["data_offsets"]
        return bytes(self._mm[self.data_start + start: self.data_start + stop]) if stop > start else b""

    def meta(self) -> dict[str, torch.Tensor]:
        return {n: torch.empty(e["shape"], dtype=DTYPES[e["dtype"]][1], device="meta") for n, e in self.entries.items()}

    def __iter__(self) -> Iterator[str]:
        return iter(self.entries)

    def __len__(self) -> int:
        return len(self.entries)

    def close(self) -> None:
        if self._mm is not None:
            self._mm.close()
            self._mm = None

    def __enter__(self) -> "SafetensorsFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def _header_blob(entries: list[tuple[str, str, tuple, int, int]], metadata: dict) -> bytes:
    """The JSON header with sorted keys and compact separators, space-padded to a multiple of 8
    bytes so the data buffer starts 8-byte aligned: the same plan always gives the same bytes."""
    header: dict = {"__metadata__": metadata}
    for name, dtype, shape, start, stop in entries:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [start, stop]}
    blob = json.dumps(header, separators=(",", ":"), sort_keys=True).encode("utf-8")
    return blob + b" " * (-len(blob) % 8)


def _tensor_bytes(t: torch.Tensor) -> bytes:
    t = t.detach().contiguous().cpu()
    return t.view(torch.uint8).numpy().tobytes() if t.numel() else b""


def write_safetensors(path: str | os.PathLike, tensors: Mapping[str, torch.Tensor],
                      metadata: Mapping[str, str] | None = None) -> None:
    """Write ``tensors`` (any device) in sorted-name order with ``metadata`` (strings)."""
    names = sorted(tensors)
    entries, cursor = [], 0
    for n in names:
        t = tensors[n]
        if t.dtype not in _NAME_OF:
            raise SafetensorsError(f"{n}: dtype {t.dtype} has no safetensors name")
        nbytes = t.numel() * t.element_size()
        entries.append((n, _NAME_OF[t.dtype], tuple(t.shape), cursor, cursor + nbytes))
        cursor += nbytes
    head = _header_blob(entries, {str(k): str(v) for k, v in (metadata or {}).items()})
    with open(path, "wb") as out:
        out.write(struct.pack("<Q", len(head)))
        out.write(head)
        for n in names:
            out.write(_tensor_bytes(tensors[n]))


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for block in iter(lambda: fh.read(COPY_CHUNK), b""):
            h.update(block)
    return h.hexdigest()


def _plan(entries: dict) -> list[tuple[str, str, str, tuple]]:
    """``(name, kind, dtype, shape)`` in sorted-name order; kind ``copy``, ``quant`` or ``scales``.
    Reads no tensor data; raises the tool's refusals (tools/quantize_int8.py:412-488)."""
    plan = []
    for name in sorted(entries):
        e = entries[name]
        dtype, shape = e["dtype"], tuple(e["shape"])
        if name.endswith(SCALES_SUFFIX) and CHECKPOINT_EXPERT_RE.match(name[: -len(SCALES_SUFFIX)]):
            raise QuantizeError(f"{name}: the source already carries per-group scales -- this looks like an "
                                "already-quantised checkpoint")
        if CHECKPOINT_EXPERT_RE.match(name) is None:
            plan.append((name, "copy", dtype, shape))
            continue
        if dtype != "BF16":
            raise QuantizeError(f"{name}: routed expert weights must be BF16, header says {dtype}")
        if len(shape) != 2:
            raise QuantizeError(f"{name}: expected a per-expert 2-D [N,K] weight, header says {list(shape)} "
                                "(a stacked [E,N,K] tensor is not this format)")
        n, k = shape
        if k % GROUP_SIZE:
            raise QuantizeError(f"{name}: K={k} is not divisible by the group size {GROUP_SIZE}")
        plan.append((name, "quant", "I8", shape))
        plan.append((name + SCALES_SUFFIX, "scales", "F32", (n, k // GROUP_SIZE)))
    if [p[0] for p in plan] != sorted(p[0] for p in plan):
        raise QuantizeError("output layout is not in sorted-name order -- some tensor name sorts between a "
                            f"weight and its {SCALES_SUFFIX} companion")
    if not any(kind == "quant" for _, kind, _, _ in plan):
        raise QuantizeError("no expert weights matched the pattern -- refusing to write a byte-copy that only "
                            "looks quantised")
    return plan


def quantize_checkpoint(src: str | os.PathLike, dst: str | os.PathLike, *, expect_sha: str | None = None,
                        device: str | torch.device = "cuda", tool: str = TOOL) -> dict:
    """Write the int8 checkpoint of ``src`` to ``dst`` (through ``dst.partial``); returns a report.

    Every routed expert weight is read, moved to ``device`` and quantised there; the int8 bytes
    and, right after them, the scales are written as the plan reaches them.
    """
    src, dst = Path(src), Path(dst)
    src_sha = _sha256(src)
    if expect_sha is not None and src_sha != expect_sha.strip().lower():
        raise QuantizeError(f"source sha256 mismatch\n  expected {expect_sha.strip().lower()}\n  actual   {src_sha}\n"
                            "refusing to quantise a checkpoint that is not the one this run was pinned to")
    dev = torch.device(device)
    with SafetensorsFile(src) as f:
        plan = _plan(f.entries)
        entries, cursor = [], 0
        for name, kind, dtype, shape in plan:
            nbytes = DTYPES[dtype][0] * _numel(shape)
            entries.append((name, dtype, shape, cursor, cursor + nbytes))
            cursor += nbytes
        meta = {str(k): str(v) for k, v in sorted(f.metadata.items())}
        meta.update({"group_size": str(GROUP_SIZE), "scheme": SCHEME, "source_sha256": src_sha, "tool": tool})
        head = _header_blob(entries, meta)
        tmp = dst.with_name(dst.name + ".partial")
        pending: bytes | None = None
        quantized = 0
        digest = hashlib.sha256()
        with open(tmp, "wb") as out:
            def emit(block: bytes) -> None:
                out.write(block)
                digest.update(block)

            emit(struct.pack("<Q", len(head)))
            emit(head)
            for name, kind, _, _ in plan:
                if kind == "copy":
                    start, stop = f.entries[name]["data_offsets"]
                    for pos in range(start, stop, COPY_CHUNK):
                        emit(bytes(f._mm[f.data_start + pos: f.data_start + min(stop, pos + COPY_CHUNK)]))
                elif kind == "quant":
                    w = f[name].to(dev, non_blocking=False)
                    q, s = quantize_per_group(w)
                    emit(_tensor_bytes(q))
                    pending = _tensor_bytes(s)
                    quantized += 1
                else:
                    if pending is None:
                        raise QuantizeError(f"{name}: scales written before their weight")
                    emit(pending)
                    pending = None
            written = out.tell()
        expected = 8 + len(head) + cursor
        if written != expected:
            raise QuantizeError(f"wrote {written} bytes, planned {expected}")
    os.replace(tmp, dst)
    return {"tool": tool, "scheme": SCHEME, "group_size": GROUP_SIZE, "source": str(src), "source_sha256": src_sha,
            "output": str(dst), "output_sha256": digest.hexdigest(), "output_bytes": written,
            "quantized_tensors": quantized, "copied_tensors": sum(1 for p in plan if p[1] == "copy")}


def load_moe_layer(path: str | os.PathLike, layer: int, config=None, *, device: str | torch.device = "cuda",
                   quantize: str | None = None):
    """``UocrMoE`` of decoder layer ``layer`` read from a safetensors model file.

    The half-quantised check runs over the whole file's header (data-less ``meta`` tensors);
    then only ``model.layers.{layer}.mlp.*`` is read. ``quantize="int8"`` quantises a bf16 file's
    routed experts on the GPU first (the bits of the published int8 file).
    """
    from .moe import MoEConfig, UocrMoE
    from .weights import is_int8_checkpoint

    if quantize not in (None, "int8"):
        raise ValueError(f"load_moe_layer: quantize must be None or 'int8', got {quantize!r}")
    dev = torch.device(device)
    with SafetensorsFile(path) as f:
        file_int8 = is_int8_checkpoint(f.meta())
        prefix = f"model.layers.{layer}.mlp."
        mine = {n: f[n].to(dev) for n in f.entries if n.startswith(prefix)}
    if quantize == "int8" and not file_int8:
        for name in sorted(mine):
            if CHECKPOINT_EXPERT_RE.match(name):
                q, s = quantize_per_group(mine[name])
                mine[name] = q
                mine[name + SCALES_SUFFIX] = s
    if config is None:
        config = MoEConfig(int8_experts=file_int8 or quantize == "int8")
    return UocrMoE.from_checkpoint(mine, layer, config, device=dev)
