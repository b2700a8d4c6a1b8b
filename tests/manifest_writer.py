"""Writes decoder-only manifests in the reference's export format
(export_decoder_llm.py:554-595: a "TMC_DECODER_LLM 2" text header and a
float32 payload beside it) from a golden fixture, for the importer tests."""

import json
import os

import numpy as np

CONFIG_KEYS = ("batch", "hidden_size", "heads", "intermediate_size", "vocabulary_size", "layers", "capacity",
               "prefill_length", "decode_count")


def write_manifest(path, meta, tensors, model="golden", version=2, dtypes=("F16", "F16"), extra_lines=(),
                   attention=None):
    """`attention` = (kv_heads, rope_theta) writes the optional ATTENTION line
    of this backend's grouped-query extension after CONFIG."""
    payload_name = os.path.basename(path) + ".bin"
    chunks, ranges, offset = [], [], 0
    for name, value in tensors.items():
        flat = np.ascontiguousarray(np.asarray(value, dtype=np.float32).reshape(-1))
        chunks.append(flat)
        ranges.append((name, offset, flat.size))
        offset += flat.size
    with open(os.path.join(os.path.dirname(path), payload_name), "wb") as f:
        for c in chunks:
            f.write(c.tobytes())
    lines = [f"TMC_DECODER_LLM {version}", f"MODEL {json.dumps(model)}", f"PAYLOAD {json.dumps(payload_name)}",
             "CONFIG " + " ".join(str(meta[k]) for k in CONFIG_KEYS) + f" {meta['epsilon']:.9g}"]
    if attention is not None:
        lines.append(f"ATTENTION {attention[0]} {attention[1]!r}")
    if dtypes:
        lines.append("DTYPE "+ " ".join(dtypes[:2] if version == 2 else dtypes[:1]))
    lines.append(f"TENSORS {len(ranges)}")
    lines += [f"TENSOR {json.dumps(n)} {o} {c}" for n, o, c in ranges]
    lines.append("END")
    lines += list(extra_lines)
    with open(path, "w", encoding="utf-8") as f:
        f.write("\n".join(lines) + "\n")
    return path


def golden_manifest(tmpdir, npz_path, **kw):
    g = np.load(npz_path)
    meta = json.loads(str(g["meta"]))
    tensors = {k: g[k] for k in g.files if k != "meta"}
    return write_manifest(os.path.join(str(tmpdir), "model.tmc"), meta, tensors, **kw), meta, g
