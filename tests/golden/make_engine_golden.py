"""Writes the tiny-Llama engine fixtures under tests/golden/tiny_llama/:

* config.json      -- a 2-layer Llama (hidden 256, 4 heads / 2 KV heads,
                      SwiGLU 768, vocabulary 1024, tied embeddings, bf16);
* tiny_llama.trdc  -- its random-initialised weights (seed 1234) compressed by
                      the reference's own SpectraCompressor (container
                      TRDC4B01, spectra/compressor.py:393-571);
* bound_tensors.json -- sha256 of every tensor the reference engine's loader
                      bound to its quantised modules (packed codes, scales,
                      unpacked zero points, int64 outlier indices, outlier weights);
* engine_golden.npz -- the reference engine (spectra/engine.py) loading that
                      container on the CPU, with the reference's operator API
                      restated in torch (oracle/engine_kernels.py) injected as
                      spectra.kernels: the greedy tokens of its generate() loop
                      for a fixed prompt of token ids, and the teacher-forced
                      logits of the whole sequence.

    SPECTRA_REF=/path/to/SPECTRA python tests/golden/make_engine_golden.py

The reference is imported from SPECTRA_REF; nothing here runs at test time.
"""
from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
REF = os.environ.get("SPECTRA_REF")
if not REF:
    sys.exit("make_engine_golden.py: set SPECTRA_REF to the root of a NeuraCryption/SPECTRA checkout")

from oracle import engine_kernels  # noqa: E402
from tests import engine_helpers as H  # noqa: E402


def main() -> None:
    from transformers import LlamaConfig, LlamaForCausalLM
    E = H.import_engine(engine_kernels.as_module(), REF)
    from spectra.compressor import SpectraCompressor

    H.TINY_DIR.mkdir(parents=True, exist_ok=True)
    cfg = LlamaConfig(**H.TINY_CONFIG)
    cfg.torch_dtype = torch.bfloat16
    cfg.architectures = ["LlamaForCausalLM"]
    torch.manual_seed(1234)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    with tempfile.TemporaryDirectory() as td:
        src = Path(td) / "src"
        model.save_pretrained(str(src), safe_serialization=True)
        out = Path(td) / "tiny_llama.trdc"
        SpectraCompressor().compress(str(src), str(out), save_tokenizer=False)
        shutil.copy(out, H.TINY_TRDC)
        shutil.copy(src / "config.json", H.TINY_DIR / "config.json")

    engine = E.SpectraUniversalEngine.load(str(H.TINY_TRDC), model_dir=str(H.TINY_DIR), device_index=0)
    engine.tokenizer = H.IdTokenizer()
    # what the reference loader bound to each quantised module (sha256 of the
    # buffers SpectraFusedLinear / SpectraFusedEmbedding received)
    bound = {}
    for mname, mod in engine.model.named_modules():
        if isinstance(mod, (E.SpectraFusedLinear, E.SpectraFusedEmbedding)):
            rec = {k: H.sha256(getattr(mod, a)) for k, a in (("packed", "packed_weight"), ("scales", "scales"),
                                                             ("zeros", "zeros"), ("outlier_idx", "outlier_idx"),
                                                             ("outlier_w", "outlier_weight"))
                   if getattr(mod, a, None) is not None}
            rec["marlin_layout"] = bool(mod.marlin_layout)
            bound[mname + ".weight"] = rec
    (H.TINY_DIR / "bound_tensors.json").write_text(json.dumps(bound, indent=1, sort_keys=True))
    ids = H.prompt_ids()
    toks, res = H.greedy(engine, ids)
    assert len(toks) == H.NEW_TOKENS, toks
    logits = H.teacher_forced_logits(E, engine, ids + toks)
    np.savez_compressed(H.TINY_GOLDEN, prompt=np.array(ids, np.int64), tokens=np.array(toks, np.int64),
                        logits=logits.numpy().astype(np.float32))
    top2 = torch.topk(logits, 2, dim=-1).values
    margin = (top2[:, 0] - top2[:, 1]) / logits.abs().max()
    print(json.dumps({"tokens": toks, "mode": res.mode, "min_rel_margin": float(margin[H.PROMPT_LEN - 1:-1].min()),
                      "logits_absmax": float(logits.abs().max())}))


if __name__ == "__main__":
    main()
