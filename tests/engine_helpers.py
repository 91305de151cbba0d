"""Helpers for running the reference engine (spectra/engine.py) on a tiny
random Llama: the model configuration, a token-id "tokenizer" (no tokenizer
files exist for a random model), and the injection of an operator module as
``spectra.kernels`` before ``spectra.engine`` is imported -- the way a user
binds this package in place of the reference's Triton kernels."""
from __future__ import annotations

import hashlib
import sys
import types
from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
TINY_DIR = GOLDEN / "tiny_llama"           # config.json of the tiny model
TINY_TRDC = TINY_DIR / "tiny_llama.trdc"   # its container, written by the reference compressor
TINY_GOLDEN = TINY_DIR / "engine_golden.npz"

TINY_CONFIG = dict(
    vocab_size=1024, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
    num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=2048,
    rms_norm_eps=1e-5, rope_theta=500000.0, tie_word_embeddings=True, initializer_range=0.1,
    bos_token_id=None, eos_token_id=None, pad_token_id=None,
)
PROMPT_LEN = 24
NEW_TOKENS = 16


class IdTokenizer:
    """Prompts are space-separated token ids; decode joins them back."""
    eos_token_id = None
    pad_token_id = None
    unk_token_id = None
    chat_template = None

    class _Enc:
        def __init__(self, ids):
            self.input_ids = ids

        def to(self, dev):
            return IdTokenizer._Enc(self.input_ids.to(dev))

    def __call__(self, prompt, return_tensors="pt"):
        ids = torch.tensor([[int(t) for t in prompt.split()]], dtype=torch.int64)
        return IdTokenizer._Enc(ids)

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(i)) for i in ids)

    def convert_tokens_to_ids(self, name):
        raise KeyError(name)


def sha256(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (contiguous, on the host)."""
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def prompt_ids(seed: int = 11):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, TINY_CONFIG["vocab_size"], (PROMPT_LEN,), generator=g).tolist()


def import_engine(kernels_module: types.ModuleType, ref_root: str):
    """Import the reference engine with ``kernels_module`` bound as
    ``spectra.kernels`` (engine.py:26 imports both operators by name).  Never
    imports ``spectra.server`` (it writes files next to its source)."""
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    for name in [m for m in sys.modules if m == "spectra" or m.startswith("spectra.")]:
        del sys.modules[name]
    # bound before the package imports: spectra/__init__.py imports the engine,
    # whose ``from spectra.kernels import ...`` then finds this module
    sys.modules["spectra.kernels"] = kernels_module
    import spectra
    import spectra.engine as E
    spectra.kernels = kernels_module
    assert E.fused_w4a16_gemv_hdsq is kernels_module.fused_w4a16_gemv_hdsq
    return E


def greedy(engine, ids, new_tokens: int = NEW_TOKENS):
    """The engine's own generate loop, greedy, no sampling penalties."""
    res = engine.generate(" ".join(str(i) for i in ids), max_new_tokens=new_tokens, temperature=0.0,
                          repetition_penalty=1.0, frequency_penalty=0.0, no_repeat_ngram_size=0)
    return [int(t) for t in res.text.split()], res


def teacher_forced_logits(E, engine, ids):
    """Logits of every position of ``ids`` through the engine's model_forward_step (no cache)."""
    x = torch.tensor([ids], dtype=torch.int64, device=engine.target_device)
    with torch.no_grad():
        out = E.model_forward_step(engine.model, x, cache=None)
    return out.logits[0].float().cpu()
