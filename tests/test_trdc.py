"""The .trdc container loader (spectra_b200/trdc.py) on the tiny Llama
container written by the reference compressor: the manifest and the validity
checks of the reference's loader on the CPU (spectra/engine.py:798-811), and
on the GPU the tensors it binds, checked against the sha256 of what the
reference engine's own loader bound (spectra/engine.py:952-1026), with the
zero points unpacked by the CUDA kernel."""
import json
import shutil
import struct

import pytest
import torch

from spectra_b200 import trdc
from tests import engine_helpers as H


def test_manifest_of_the_reference_container():
    m = trdc.read_manifest(H.TINY_TRDC)
    assert m["version"] == "TRDC4B01" and m["group_size"] == 32
    q = [n for n, t in m["tensors"].items() if t["type"] == "q4_g32_hdsq"]
    assert "model.embed_tokens.weight" in q and len(q) == 1 + 2 * 7
    assert all(m["tensors"][n]["zero_packed"] and m["tensors"][n]["marlin_layout"] for n in q)


def test_corrupted_containers_are_rejected(tmp_path):
    bad = tmp_path / "short.trdc"
    bad.write_bytes(b"TRDC4B01" + b"\0" * 8)
    with pytest.raises(trdc.ContainerError, match="corrupted or empty"):
        trdc.read_manifest(bad)
    magic = tmp_path / "magic.trdc"
    shutil.copy(H.TINY_TRDC, magic)
    with open(magic, "r+b") as f:
        f.write(b"XXXX4B01")
    with pytest.raises(trdc.ContainerError, match="header"):
        trdc.read_manifest(magic)
    table = tmp_path / "table.trdc"
    shutil.copy(H.TINY_TRDC, table)
    size = table.stat().st_size
    with open(table, "r+b") as f:
        f.seek(8)
        f.write(struct.pack("<QQ", size - 10, 100))
    with pytest.raises(trdc.ContainerError, match="manifest"):
        trdc.read_manifest(table)


def test_loader_needs_a_cuda_device():
    with pytest.raises(RuntimeError, match="CUDA"):
        trdc.load_container(H.TINY_TRDC, device="cpu")


@pytest.mark.gpu
def test_loaded_tensors_equal_what_the_reference_engine_binds():
    want = json.loads((H.TINY_DIR / "bound_tensors.json").read_text())
    got = trdc.load_container(H.TINY_TRDC, device="cuda")
    checked = 0
    for name, rec in want.items():
        if name not in got:  # the tied lm_head is bound to the embedding's tensors
            assert name == "lm_head.weight"
            name = "model.embed_tokens.weight"
        w = got[name]
        assert w.packed.is_cuda and w.zeros.dtype == torch.uint8 and w.outlier_idx.dtype == torch.int64
        assert w.marlin_layout == rec["marlin_layout"]
        for k in ("packed", "scales", "zeros", "outlier_idx", "outlier_w"):
            assert H.sha256(getattr(w, k)) == rec[k], f"{name}.{k}"
        checked += 1
    assert checked == len(want) == 2 * 7 + 2
    norm = got["model.layers.0.input_layernorm.weight"]
    assert norm.dtype == torch.bfloat16 and norm.shape == (256,) and norm.is_cuda
