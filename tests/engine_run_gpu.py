"""Runs the reference engine (spectra/engine.py, installed unchanged under
baseline/_ref) on the tiny Llama fixture on cuda:0, twice: with this
package's kernels bound as ``spectra.kernels`` (the drop-in), and with the
reference operator API restated in torch (oracle/engine_kernels.py) patched
into the same engine.  Prints one JSON record for tests/test_engine_gpu.py.

    python tests/engine_run_gpu.py <reference root>
"""
from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle import engine_kernels  # noqa: E402
from spectra_b200 import kernels as SK  # noqa: E402
from tests import engine_helpers as H  # noqa: E402

CALLS = {"gemv": 0, "gemm": 0}


def counting_module() -> types.ModuleType:
    m = types.ModuleType("spectra.kernels")

    def gemv(*a, **k):
        CALLS["gemv"] += 1
        return SK.fused_w4a16_gemv_hdsq(*a, **k)

    def gemm(*a, **k):
        CALLS["gemm"] += 1
        return SK.batched_w4a16_gemm(*a, **k)
    m.fused_w4a16_gemv_hdsq = gemv
    m.batched_w4a16_gemm = gemm
    return m


def main() -> None:
    ref_root = sys.argv[1]
    ours = counting_module()
    E = H.import_engine(ours, ref_root)
    engine = E.SpectraUniversalEngine.load(str(H.TINY_TRDC), model_dir=str(H.TINY_DIR), device_index=0)
    engine.tokenizer = H.IdTokenizer()
    gold = np.load(H.TINY_GOLDEN)
    ids = gold["prompt"].tolist()
    seq = ids + gold["tokens"].tolist()
    rec = {"plan": engine.plan.mode}

    def run(tag: str) -> None:
        toks, res = H.greedy(engine, ids)
        rec[f"{tag}_tokens"] = toks
        rec[f"{tag}_graph"] = bool(res.cuda_graph_accelerated)
        torch.cuda.synchronize()
        rec[f"{tag}_logits"] = H.teacher_forced_logits(E, engine, seq).numpy().tolist()

    run("ours")
    rec["ours_graph_calls"] = dict(CALLS)
    engine.plan.enable_cuda_graphs = False
    run("ours_eager")
    engine.plan.enable_cuda_graphs = True
    rec["ours_calls"] = dict(CALLS)
    # the same engine, the reference operator API restated in torch
    E.fused_w4a16_gemv_hdsq = engine_kernels.fused_w4a16_gemv_hdsq
    E.batched_w4a16_gemm = engine_kernels.batched_w4a16_gemm
    run("oracle")
    engine.plan.enable_cuda_graphs = False
    run("oracle_eager")
    engine.plan.enable_cuda_graphs = True
    rec["calls_after_oracle"] = dict(CALLS)
    print("ENGINE_RESULT " + json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
