"""Model packages in the reference's on-disk format.

A package is a directory with ``metadata.json`` and one ``.bin`` file per
tensor, as written by the reference converter
(npu_llm/tools/convert_smollm2.py:174-337) and read by ``XDNA1Model``
(npu_llm/runtime/model.py:84-198).  ``PackageModel`` reads it with the same
integrity rules, so a converted checkpoint drops in unchanged:

* ``metadata_sha256`` is the SHA-256 of the metadata JSON without that key,
  serialised with ``sort_keys=True`` and separators ``(",", ":")``;
* ``files`` lists the size and SHA-256 of every file, all verified on load;
* every tensor file is covered by ``files`` and stays inside the package;
* projections carry ``weight`` (int8) + ``scale`` (float32) + ``bf16_file``.

``write_package`` writes a model with the package surface (e.g. a seeded
``SyntheticModel``) in that format and publishes it atomically.
"""

import hashlib
import json
import os
from pathlib import Path
import shutil
import tempfile

import numpy as np
from ml_dtypes import bfloat16

from runtime.synthetic import PROJECTIONS, QuantizedView

MAX_ELEMENTS = 1 << 31


def _digest_metadata(meta):
    body = {k: v for k, v in meta.items() if k != "metadata_sha256"}
    return hashlib.sha256(json.dumps(body, separators=(",", ":"), sort_keys=True).encode()).hexdigest()


def _file_sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            block = f.read(1 << 20)
            if not block:
                break
            h.update(block)
    return h.hexdigest()


def _inside(root, name):
    if not isinstance(name, str) or not name:
        raise RuntimeError("package manifest names a file with an empty or non-string path")
    p = Path(name)
    if p.is_absolute():
        raise RuntimeError(f"package files must use relative paths, got {name}")
    root = Path(root).resolve()
    full = (root / p).resolve()
    if root != full and root not in full.parents:
        raise RuntimeError(f"package file {name} resolves outside the package directory")
    return full


def _dims(shape, name):
    if not isinstance(shape, (list, tuple)) or not shape:
        raise RuntimeError(f"{name}: shape must be a non-empty list of dimensions")
    count = 1
    for d in shape:
        if isinstance(d, bool) or not isinstance(d, int):
            raise RuntimeError(f"{name}: every dimension must be an integer")
        if d <= 0:
            raise RuntimeError(f"{name}: every dimension must be at least 1")
        count *= d
        if count > MAX_ELEMENTS:
            raise RuntimeError(f"{name}: more than 2**31 elements")
    return tuple(shape), count


class PackageModel:
    """Read-only, integrity-checked view of a package directory."""

    def __init__(self, model_dir, verify=True):
        self.root = Path(model_dir).resolve()
        try:
            meta = json.loads(_inside(self.root, "metadata.json").read_text())
        except (OSError, json.JSONDecodeError) as exc:
            raise RuntimeError("metadata.json is missing or is not valid JSON") from exc
        if not isinstance(meta, dict):
            raise RuntimeError("metadata.json must hold a JSON object at the top level")
        if not isinstance(meta.get("tensors"), dict):
            raise RuntimeError("metadata.json lacks the 'tensors' table")
        digest = meta.get("metadata_sha256")
        if not isinstance(digest, str) or len(digest) != 64:
            raise RuntimeError("metadata.json carries no metadata_sha256 digest (written by an older converter?)")
        if _digest_metadata(meta) != digest:
            raise RuntimeError("metadata checksum mismatch: metadata.json was edited after conversion")
        self.metadata = meta
        self.tensors = meta["tensors"]
        self._files = meta.get("files")
        if verify:
            self._verify()

    def _verify(self):
        files = self._files
        if not isinstance(files, dict) or not files:
            raise RuntimeError("metadata.json lists no files with sizes and digests; convert the model again")
        for name, entry in files.items():
            path = _inside(self.root, name)
            size = entry.get("size") if isinstance(entry, dict) else None
            sha = entry.get("sha256") if isinstance(entry, dict) else None
            if isinstance(size, bool) or not isinstance(size, int) or size < 0 \
                    or not isinstance(sha, str) or len(sha) != 64:
                raise RuntimeError(f"files[{name!r}] needs an integer size and a 64-digit sha256")
            if not path.is_file() or path.stat().st_size != size:
                raise RuntimeError(f"{name}: absent, or its size differs from the manifest")
            if _file_sha256(path) != sha:
                raise RuntimeError(f"{name}: content checksum mismatch against the manifest")
        for tname, spec in self.tensors.items():
            if not isinstance(spec, dict):
                raise RuntimeError(f"tensors[{tname!r}] must be a JSON object")
            for field in ("file", "weight", "scale", "bf16_file"):
                fname = spec.get(field)
                if fname is not None and fname not in files:
                    raise RuntimeError(f"{fname} is referenced by a tensor but not listed under files")

    def _map(self, fname, dtype, shape):
        path = _inside(self.root, fname)
        dtype = np.dtype(dtype)
        shape, count = _dims(list(shape), fname)
        if path.stat().st_size != count * dtype.itemsize:
            raise RuntimeError(f"{fname}: byte size does not match the tensor's shape and dtype")
        if isinstance(self._files, dict) and fname not in self._files:
            raise RuntimeError(f"{fname} is referenced by a tensor but not listed under files")
        return np.memmap(path, mode="r", dtype=dtype, shape=shape)

    def raw(self, name):
        spec = self.tensors[name]
        try:
            dtype = np.dtype(bfloat16) if spec["dtype"] == "bfloat16" else np.dtype(spec["dtype"])
        except (KeyError, TypeError) as exc:
            raise RuntimeError(f"{name}: unknown or missing dtype") from exc
        return self._map(spec["file"], dtype, spec["shape"])

    def bf16_projection(self, name):
        spec = self.tensors[name]
        if "bf16_file" not in spec:
            raise RuntimeError(f"{name}: the package stores no BF16 copy of this projection")
        return self._map(spec["bf16_file"], bfloat16, spec["shape"])

    def quantized(self, name):
        spec = self.tensors[name]
        shape, _ = _dims(spec.get("shape"), name)
        if len(shape) != 2:
            raise RuntimeError("an int8 projection must be a 2-D [rows, columns] matrix")
        return QuantizedView(
            self._map(spec["weight"], np.int8, shape), self._map(spec["scale"], np.float32, shape[:1])
        )


def _write(out_dir, fname, array):
    np.ascontiguousarray(array).tofile(out_dir / fname)
    return fname


def _write_into(model, out_dir):
    meta = {k: v for k, v in model.metadata.items() if k != "tensors"}
    tensors = {}
    for name, spec in model.tensors.items():
        leaf = name.split(".")[-1]
        if leaf in PROJECTIONS or name == "lm_head":
            bf = np.asarray(model.bf16_projection(name)).astype(bfloat16, copy=False)
            q = model.quantized(name)
            tensors[name] = {
                "weight": _write(out_dir, f"{name}.w8.bin", np.asarray(q.weight, np.int8)),
                "scale": _write(out_dir, f"{name}.scale.f32.bin", np.asarray(q.scale, np.float32)),
                "shape": list(bf.shape),
                "layout": "row_major",
                "weight_dtype": "int8",
                "scale_dtype": "float32",
                "quantization": "symmetric_per_output_channel",
                "bf16_file": _write(out_dir, f"{name}.bf16.bin", bf),
                "bf16_dtype": "bfloat16",
            }
        else:
            arr = np.asarray(model.raw(name))
            dtype_name = "bfloat16" if arr.dtype == np.dtype(bfloat16) else arr.dtype.name
            tensors[name] = {
                "file": _write(out_dir, f"{name}.{dtype_name}.bin", arr),
                "shape": list(arr.shape),
                "dtype": dtype_name,
            }
    meta["tensors"] = tensors
    meta["files"] = {
        p.name: {"sha256": _file_sha256(p), "size": p.stat().st_size}
        for p in sorted(out_dir.iterdir())
        if p.is_file() and p.name != "metadata.json"
    }
    meta["metadata_sha256"] = _digest_metadata(meta)
    (out_dir / "metadata.json").write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n")
    return meta


def write_package(model, out_dir):
    """Write ``model`` as a package at ``out_dir``, replacing any previous
    package only once the new one is complete."""
    out_dir = Path(out_dir)
    out_dir.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{out_dir.name}.staging-", dir=out_dir.parent))
    try:
        meta = _write_into(model, staging)
        backup = None
        if out_dir.exists():
            backup = out_dir.with_name(f".{out_dir.name}.old-{os.getpid()}")
            os.replace(out_dir, backup)
        try:
            os.replace(staging, out_dir)
        except Exception:
            if backup is not None:
                os.replace(backup, out_dir)
            raise
        if backup is not None:
            shutil.rmtree(backup)
        return meta
    finally:
        if staging.exists():
            shutil.rmtree(staging)


def open_model(model_dir_or_model, verify=True):
    """A package directory, or any object that already has the package
    surface (``metadata`` + ``raw``/``bf16_projection``/``quantized``)."""
    if hasattr(model_dir_or_model, "metadata") and hasattr(model_dir_or_model, "bf16_projection"):
        return model_dir_or_model
    return PackageModel(model_dir_or_model, verify=verify)
