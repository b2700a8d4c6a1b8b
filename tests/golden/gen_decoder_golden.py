"""Generate decoder golden vectors with the reference's OWN exporter.

Runs tools/export_decoder_llm.py of the reference project (the checkout named
by TMC_REFERENCE, else the default below) in-process: it builds the
reference's PyTorch DecoderOnlyLLM (workloads/pytorch/decoder_llm.py), seeds it,
runs the fp16 precision admission, and records prefill and per-step decode
logits, greedy next tokens and full KV caches (export_decoder_llm.py:453-551).
The tensors are saved as compressed .npz fixtures beside this script:

    python tests/golden/gen_decoder_golden.py

decoder_default_fp16.npz  the exporter's defaults (hidden 64, 4 heads, 2 layers,
                          intermediate 128, vocab 128, capacity 32, prefill 8,
                          decode 8), seed 11 as in run.sh:19, dtype fp16.
KV caches are kept after prefill and after the last decode step (the
intermediate steps' caches are prefixes of the last).
decoder_wide_fp16.npz     hidden 256, 8 heads (head_dim 32), 2 layers,
                          intermediate 512, vocab 512, capacity 64, prefill 19,
                          decode 12, seed 5, dtype fp16.
"""

import argparse
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("TMC_REFERENCE", Path(__file__).resolve().parents[2].parent / "reference"))


def load_exporter():
    path = REFERENCE / "tools" / "export_decoder_llm.py"
    spec = importlib.util.spec_from_file_location("reference_export_decoder_llm", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def export(name, seed, **overrides):
    exporter = load_exporter()
    args = argparse.Namespace(checkpoint=None, dtype="fp16", effective_dtype=None, seed=seed,
                              model_name="DecoderOnlyLLM", batch=None, hidden_size=None, heads=None,
                              layers=None, intermediate_size=None, vocabulary_size=None,
                              capacity=None, prefill_length=None, decode_count=None, epsilon=None)
    for k, v in overrides.items():
        setattr(args, k, v)
    config, tensors = exporter._make_workload(REFERENCE, args)
    assert config["storage_dtype"] == "fp16", config
    out = {}
    last = f"decode{config['decode_count'] - 1}."
    for key, tensor in tensors.items():
        # Keep the KV caches after prefill and after the last decode step only
        # (the intermediate ones are prefixes of the last).
        if "_cache" in key and not (key.startswith("prefill.") or key.startswith(last)):
            continue
        t = tensor.detach().cpu()
        if key.endswith(("tokens", "next_tokens")):
            out[key] = t.to(torch.int64).numpy().astype(np.int32)
        elif key.startswith("rope."):
            out[key] = t.to(torch.float32).numpy()
        else:
            # Every other tensor holds fp16 values (weights, fp16 logits, caches).
            out[key] = t.to(torch.float16).numpy()
    meta = {k: config[k] for k in ("batch", "hidden_size", "heads", "layers", "intermediate_size",
                                   "vocabulary_size", "capacity", "prefill_length",
                                   "decode_count", "epsilon", "storage_dtype")}
    meta["seed"] = seed
    meta["torch"] = torch.__version__
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / name, **out)
    print(f"{name}: {len(tensors)} tensors, torch {torch.__version__}")


def main():
    export("decoder_default_fp16.npz", 11)
    export("decoder_wide_fp16.npz", 5, hidden_size=256, heads=8, layers=2, intermediate_size=512,
           vocabulary_size=512, capacity=64, prefill_length=19, decode_count=12)


if __name__ == "__main__":
    sys.exit(main())
