"""Decoder-only manifests in the reference's export format, read through the
C-ABI importer (tmc_manifest_*, DecoderManifest.cpp; reference
importDecoderLLMWorkload, DecoderLLMImporter.cpp:154-281), on the CPU: header
and config, every named tensor bit-exact, and the reference importer's
rejections."""

import os

import numpy as np
import pytest

from tests.manifest_writer import golden_manifest, write_manifest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_manifest_round_trips_the_exporter_format(tmp_path):
    import tmc_cuda
    path, meta, g = golden_manifest(tmp_path, os.path.join(GOLDEN, "decoder_default_fp16.npz"))
    m = tmc_cuda.Manifest(path)
    i = m.info
    assert (i["version"], i["batch"], i["hidden_size"], i["heads"], i["layers"], i["capacity"]) == \
        (2, meta["batch"], meta["hidden_size"], meta["heads"], meta["layers"], meta["capacity"])
    assert i["head_dim"] == meta["hidden_size"] // meta["heads"]
    assert (i["prefill_length"], i["decode_count"]) == (meta["prefill_length"], meta["decode_count"])
    assert i["epsilon"] == np.float32(meta["epsilon"]) and i["requested_dtype"] == "F16"
    for name in g.files:
        if name != "meta":
            assert np.array_equal(m.tensor(name), np.asarray(g[name], np.float32).reshape(-1)), name
    m.close()


@pytest.mark.parametrize("version,dtypes", [(1, ("F32",)), (1, None), (2, ("F16", "F32"))])
def test_manifest_versions_and_dtype_markers(tmp_path, version, dtypes):
    import tmc_cuda
    meta = dict(batch=1, hidden_size=8, heads=2, intermediate_size=16, vocabulary_size=10, layers=1, capacity=6,
                prefill_length=2, decode_count=3, epsilon=1e-5)
    path = write_manifest(str(tmp_path / "m.tmc"), meta, {"a": np.arange(4.0)}, version=version, dtypes=dtypes)
    m = tmc_cuda.Manifest(path)
    assert m.info["version"] == version
    assert m.info["requested_dtype"] == (dtypes[0] if dtypes else "F32")
    assert m.info["effective_dtype"] == (dtypes[-1] if dtypes else "F32")
    assert np.array_equal(m.tensor("a"), np.arange(4.0, dtype=np.float32))


@pytest.mark.parametrize("case", ["magic", "heads", "capacity", "duplicate", "trailing", "range", "missing"])
def test_manifest_rejections(tmp_path, case):
    import tmc_cuda
    meta = dict(batch=1, hidden_size=8, heads=2, intermediate_size=16, vocabulary_size=10, layers=1, capacity=6,
                prefill_length=2, decode_count=3, epsilon=1e-5)
    tensors = {"a": np.arange(4.0), "b": np.ones(2)}
    path = str(tmp_path / "m.tmc")
    if case == "heads":
        meta["heads"] = 3
    if case == "capacity":
        meta["decode_count"] = 5
    write_manifest(path, meta, tensors, extra_lines=("TENSOR",) if case == "trailing" else ())
    text = open(path).read()
    if case == "magic":
        text = text.replace("TMC_DECODER_LLM 2", "TMC_DECODER_LLM 3")
    if case == "duplicate":
        text = text.replace('TENSOR "b"', 'TENSOR "a"')
    if case == "range":
        text = text.replace('TENSOR "b" 4 2', 'TENSOR "b" 4 9')
    open(path, "w").write(text)
    if case == "missing":
        os.remove(path + ".bin")
    with pytest.raises(tmc_cuda.TmcError):
        tmc_cuda.Manifest(path)


def _small_meta():
    return dict(batch=1, hidden_size=8, heads=4, intermediate_size=16, vocabulary_size=10, layers=1, capacity=6,
                prefill_length=2, decode_count=3, epsilon=1e-5)


def test_manifest_attention_line_sets_kv_heads_and_theta(tmp_path):
    import tmc_cuda
    path = write_manifest(str(tmp_path / "m.tmc"), _small_meta(), {"a": np.arange(4.0)}, attention=(2, 500000.0))
    m = tmc_cuda.Manifest(path)
    assert (m.info["kv_heads"], m.info["rope_theta"], m.info["heads"]) == (2, 500000.0, 4)
    assert m.info["requested_dtype"] == "F16"
    assert np.array_equal(m.tensor("a"), np.arange(4.0, dtype=np.float32))


def test_manifest_without_attention_line_is_mha(tmp_path):
    import tmc_cuda
    path = write_manifest(str(tmp_path / "m.tmc"), _small_meta(), {"a": np.arange(4.0)})
    m = tmc_cuda.Manifest(path)
    assert (m.info["kv_heads"], m.info["rope_theta"]) == (4, 10000.0)


@pytest.mark.parametrize("attention", [(3, 10000.0), (0, 10000.0), (2, 0.0), (2, -1.0)])
def test_manifest_attention_line_rejections(tmp_path, attention):
    import tmc_cuda
    path = write_manifest(str(tmp_path / "m.tmc"), _small_meta(), {"a": np.arange(4.0)}, attention=attention)
    with pytest.raises(tmc_cuda.TmcError):
        tmc_cuda.Manifest(path)
