"""Model packages in the reference format: write, read back with integrity
checks, and reject tampering (npu_llm/runtime/model.py:84-154,
npu_llm/tests/test_model_integrity.py-style cases)."""

import json

import numpy as np
import pytest
from ml_dtypes import bfloat16

from runtime import synthetic
from runtime.model import PackageModel, open_model, write_package


@pytest.fixture(scope="module")
def package(tmp_path_factory):
    model = synthetic.build("tiny-qwen", seed=3)
    out = tmp_path_factory.mktemp("pkg") / "tiny-qwen"
    write_package(model, out)
    return model, out


def test_package_round_trips(package):
    model, path = package
    pkg = PackageModel(path)
    assert pkg.metadata["model_family"] == "qwen2"
    for name in model.tensors:
        leaf = name.split(".")[-1]
        if leaf in ("qkv", "o_proj", "gate_up", "down_proj") or name == "lm_head":
            assert np.array_equal(np.asarray(pkg.bf16_projection(name)).view(np.uint16),
                                  np.asarray(model.bf16_projection(name)).view(np.uint16))
            q = pkg.quantized(name)
            assert np.array_equal(np.asarray(q.weight), model.quantized(name).weight)
            assert np.array_equal(np.asarray(q.scale).view(np.uint32), model.quantized(name).scale.view(np.uint32))
        else:
            assert np.array_equal(np.asarray(pkg.raw(name)).view(np.uint8),
                                  np.asarray(model.raw(name)).view(np.uint8))
    assert np.asarray(pkg.raw("token_embedding")).dtype == np.dtype(bfloat16)


def test_open_model_passes_objects_through(package):
    model, path = package
    assert open_model(model) is model
    assert isinstance(open_model(path), PackageModel)


def test_tampered_file_is_rejected(package, tmp_path):
    _, path = package
    import shutil
    copy = tmp_path / "copy"
    shutil.copytree(path, copy)
    target = copy / "layer00.qkv.w8.bin"
    data = bytearray(target.read_bytes())
    data[0] ^= 1
    target.write_bytes(bytes(data))
    with pytest.raises(RuntimeError, match="checksum mismatch"):
        PackageModel(copy)


def test_tampered_metadata_is_rejected(package, tmp_path):
    _, path = package
    import shutil
    copy = tmp_path / "copy"
    shutil.copytree(path, copy)
    meta = json.loads((copy / "metadata.json").read_text())
    meta["layers"] = 3
    (copy / "metadata.json").write_text(json.dumps(meta))
    with pytest.raises(RuntimeError, match="metadata checksum"):
        PackageModel(copy)


def test_escaping_paths_are_rejected(package, tmp_path):
    _, path = package
    import shutil
    from runtime.model import _digest_metadata
    copy = tmp_path / "copy"
    shutil.copytree(path, copy)
    meta = json.loads((copy / "metadata.json").read_text())
    meta["tensors"]["final_norm"]["file"] = "../outside.bin"
    meta["metadata_sha256"] = _digest_metadata(meta)
    (copy / "metadata.json").write_text(json.dumps(meta))
    with pytest.raises(RuntimeError):
        PackageModel(copy)


def test_failed_write_keeps_previous_package(package, tmp_path, monkeypatch):
    model, _ = package
    out = tmp_path / "pkg"
    write_package(model, out)
    before = (out / "metadata.json").read_text()
    import runtime.model as m

    def boom(*args, **kwargs):
        raise OSError("simulated disk-full failure")

    monkeypatch.setattr(m, "_write_into", boom)
    with pytest.raises(OSError):
        write_package(model, out)
    assert (out / "metadata.json").read_text() == before
    assert not [p for p in tmp_path.iterdir() if p.name.startswith(".pkg.staging")]
