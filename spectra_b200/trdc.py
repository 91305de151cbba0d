"""Direct-to-device loader of SPECTRA's ``.trdc`` weight container.

The container (written by the reference's SpectraCompressor,
spectra/compressor.py:457-571) is the 8-byte magic ``TRDC4B01``, a
little-endian (manifest offset, manifest length) pair of u64, the raw tensor
records, and a JSON manifest.  Per quantised weight (type ``q4_g32_hdsq`` /
``q4_g32``) a record holds, back to back: packed codes u8 [N, K/2], fp16
scales [N, K/32], zero points (packed two per byte when ``zero_packed``),
outlier column indices (int32, int64 or uint16 per ``outlier_idx_dtype``) and
outlier weights [N, n_out]; other tensors are stored raw (``lossless_*``).

``load_container`` reads each record once into pinned host memory, copies it
to the device with one asynchronous copy, and builds there what the
reference engine binds to ``SpectraFusedLinear.set_weights``
(spectra/engine.py:999-1026): the zero points unpacked to one byte per group
by the CUDA kernel ``spectra_unpack_zeros`` (the reference does it with torch
ops, :1007-1012), the indices widened to int64, the outlier weights in their
stored dtype.  The same validity checks as the reference's loader are made
(:798-811): magic, size, manifest bounds.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Iterable, Optional, Union

import torch

from . import compress as C

MAGIC = b"TRDC4B01"
_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32, "int64": torch.int64,
           "int32": torch.int32, "int16": torch.int16, "int8": torch.int8, "uint8": torch.uint8, "bool": torch.bool}


class ContainerError(ValueError):
    """The file is not a valid TRDC container."""


@dataclass
class QuantizedWeight:
    """One quantised 2-D weight as ``SpectraFusedLinear.set_weights`` takes it."""
    packed: torch.Tensor        # u8 [N, K/2]
    scales: torch.Tensor        # fp16 [N, K/32]
    zeros: torch.Tensor         # u8 [N, K/32], unpacked
    outlier_idx: Optional[torch.Tensor]  # int64 [n_out]
    outlier_w: Optional[torch.Tensor]    # [N, n_out] in the stored dtype
    marlin_layout: bool
    shape: tuple


def read_manifest(path: Union[str, Path]) -> dict:
    """The container's JSON manifest, after the reference loader's checks."""
    path = Path(path)
    size = path.stat().st_size
    if size < 24:
        raise ContainerError(f"TRDC container '{path.name}' is corrupted or empty ({size} bytes)")
    with open(path, "rb") as f:
        magic = f.read(8)
        if magic != MAGIC:
            raise ContainerError(f"invalid container header: {magic!r}")
        off, length = struct.unpack("<QQ", f.read(16))
        if off < 24 or off + length > size:
            raise ContainerError(f"corrupted manifest table in '{path.name}': offset {off} + length {length} "
                                 f"exceeds the file size {size}")
        f.seek(off)
        return json.loads(f.read(length).decode("utf-8"))


def _record_bytes(meta: dict) -> int:
    if meta["type"] in ("q4_g32_hdsq", "q4_g32"):
        n = meta["packed_len"] + meta["scale_len"] + meta["zero_len"]
        if meta.get("outlier_idx_len", 0) > 0:
            n += meta["outlier_idx_len"] + meta["outlier_w_len"]
        return n
    return meta["total_len"]


def load_container(path: Union[str, Path], device: Union[str, torch.device] = "cuda",
                   names: Optional[Iterable[str]] = None) -> Dict[str, object]:
    """Every record (or those in ``names``) on ``device``: a ``QuantizedWeight``
    per quantised weight, a tensor per raw one."""
    path = Path(path)
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("spectra_b200.trdc loads to a CUDA device (the zero-point unpack runs there)")
    manifest = read_manifest(path)
    group = int(manifest.get("group_size", 32))
    if group != 32:
        raise ContainerError(f"group size {group} is not SPECTRA's 32")
    wanted = set(names) if names is not None else None
    size = path.stat().st_size
    out: Dict[str, object] = {}
    with open(path, "rb") as f:
        for name, meta in manifest["tensors"].items():
            if wanted is not None and name not in wanted:
                continue
            nbytes = _record_bytes(meta)
            if meta["offset"] < 24 or meta["offset"] + nbytes > size:
                raise ContainerError(f"record '{name}' lies outside the file")
            host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
            f.seek(meta["offset"])
            f.readinto(memoryview(host.numpy()))
            buf = host.to(dev, non_blocking=True)
            shape = tuple(meta["shape"])
            if meta["type"] in ("q4_g32_hdsq", "q4_g32"):
                out[name] = _quantized(buf, meta, shape)
            else:
                dt = _DTYPES.get(meta.get("dtype", "float16"), torch.float16)
                out[name] = buf.view(dt).reshape(shape)
            out.setdefault("__host_buffers__", []).append(host)  # alive until the copies are done
    torch.cuda.current_stream(dev).synchronize()
    out.pop("__host_buffers__", None)
    return out


def _quantized(buf: torch.Tensor, meta: dict, shape: tuple) -> QuantizedWeight:
    N, K = shape
    G = K // 32
    o = 0

    def take(n, align=1):
        """The next n bytes; copied to fresh (aligned) device memory when their
        offset in the record is not a multiple of the element size."""
        nonlocal o
        t = buf[o:o + n]
        if o % align:
            t = t.clone()
        o += n
        return t
    packed = take(meta["packed_len"]).view(N, K // 2)
    scales = take(meta["scale_len"], 2).view(torch.float16).view(N, G)
    zb = take(meta["zero_len"])
    if meta.get("zero_packed", False):
        zeros = C.unpack_zeros(zb.view(N, -1), K)
    else:
        zeros = zb.view(N, G)
    idx = ow = None
    if meta.get("outlier_idx_len", 0) > 0:
        idt = meta.get("outlier_idx_dtype", "int64")
        ib = take(meta["outlier_idx_len"], {"uint16": 2, "int32": 4}.get(idt, 8))
        if idt == "uint16":
            idx = ib.view(torch.int16).to(torch.int64) & 0xFFFF
        elif idt == "int32":
            idx = ib.view(torch.int32).to(torch.int64)
        else:
            idx = ib.view(torch.int64)
        owdt = _DTYPES.get(meta.get("outlier_w_dtype", "float16"), torch.float16)
        ow = take(meta["outlier_w_len"], torch.empty(0, dtype=owdt).element_size()).view(owdt).view(N, -1)
    return QuantizedWeight(packed, scales, zeros, idx, ow, bool(meta.get("marlin_layout", False)), shape)
