"""Reader for the `.so3lr` native model file (test infrastructure only).

ORACLE — test infrastructure. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` leg of `bench.py` may import this package. The shipped library
(`so3lr_b200`) parses model files with its own C++ loader and never calls
anything under `oracle/`.

Restates the reader of source/so3lr-lammps-native/src/native_model.cpp:338-405
(header, manifest and per-tensor integrity checks) and the layout documented in
source/so3lr-lammps-native/docs/FORMAT.md:14-41:

* 128-byte header: magic ``SO3LRN1\\0``, u32 version 1, u32 flags 0,
  u64 manifest bytes, u64 payload bytes, SHA-256(manifest), SHA-256(payload),
  32 zero bytes;
* canonical JSON manifest;
* payload of 64-byte aligned tensors, each with its own SHA-256.
"""
from __future__ import annotations

import hashlib
import json
import struct
from dataclasses import dataclass, field

import numpy as np

_DTYPES = {
    "float64": ("<f8", 8),
    "float32": ("<f4", 4),
    "int64": ("<i8", 8),
    "int32": ("<i4", 4),
    "uint8": ("u1", 1),
    "bool": ("u1", 1),
}


class ModelFormatError(RuntimeError):
    """Raised for every integrity violation (native_model.cpp:341-398)."""


@dataclass
class NativeModelFile:
    path: str
    manifest: dict
    tensors: dict = field(default_factory=dict)  # state_key -> np.ndarray

    @property
    def arch(self) -> dict:
        return self.manifest["architecture"]

    def t(self, key: str) -> np.ndarray:
        try:
            return self.tensors[key]
        except KeyError as exc:
            raise ModelFormatError(f"missing tensor {key}") from exc


def load_model(path: str) -> NativeModelFile:
    """Load and verify a `.so3lr` file (native_model.cpp:338-405)."""
    with open(path, "rb") as handle:
        data = handle.read()
    return load_model_bytes(data, path)


def load_model_bytes(data: bytes, origin: str = "<bytes>") -> NativeModelFile:
    header = 128
    if len(data) < header:
        raise ModelFormatError("file is shorter than fixed header")
    if data[:8] != b"SO3LRN1\x00":
        raise ModelFormatError("wrong magic")
    version, flags = struct.unpack_from("<II", data, 8)
    if version != 1 or flags != 0:
        raise ModelFormatError("unsupported version or flags")
    manifest_size, payload_size = struct.unpack_from("<QQ", data, 16)
    if manifest_size > len(data) - header or payload_size != len(data) - header - manifest_size:
        raise ModelFormatError("header length mismatch")
    if any(data[96:128]):
        raise ModelFormatError("nonzero reserved header bytes")
    manifest_bytes = data[header:header + manifest_size]
    payload = data[header + manifest_size:]
    if hashlib.sha256(manifest_bytes).digest() != data[32:64]:
        raise ModelFormatError("manifest SHA-256 mismatch")
    if hashlib.sha256(payload).digest() != data[64:96]:
        raise ModelFormatError("payload SHA-256 mismatch")
    try:
        manifest = json.loads(manifest_bytes.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ModelFormatError(f"malformed manifest JSON: {exc}") from exc
    canonical = json.dumps(manifest, sort_keys=True, separators=(",", ":"),
                           ensure_ascii=False).encode("utf-8")
    if canonical != manifest_bytes:
        raise ModelFormatError("noncanonical manifest JSON")
    if manifest.get("format") != "so3lr-native" or manifest.get("format_version") != 1:
        raise ModelFormatError("manifest format mismatch")
    if manifest.get("endianness") != "little" or manifest.get("tensor_alignment") != 64:
        raise ModelFormatError("manifest endianness/alignment mismatch")
    if manifest.get("model_family") != "SO3LR":
        raise ModelFormatError("wrong model family")

    result = NativeModelFile(path=origin, manifest=manifest)
    names, keys = set(), set()
    previous_end = 0
    total = 0
    for record in manifest["tensors"]:
        name, key, dtype = record["name"], record["state_key"], record["dtype"]
        if dtype not in _DTYPES:
            raise ModelFormatError(f"unsupported dtype {dtype}")
        np_dtype, width = _DTYPES[dtype]
        shape = [int(s) for s in record["shape"]]
        count = int(np.prod(shape)) if shape else 1
        offset, nbytes = int(record["offset"]), int(record["nbytes"])
        if name in names or key in keys:
            raise ModelFormatError("duplicate tensor name/state key")
        names.add(name)
        keys.add(key)
        if offset % 64 != 0 or nbytes != count * width:
            raise ModelFormatError("tensor alignment/size mismatch")
        if offset < previous_end or offset > payload_size or nbytes > payload_size - offset:
            raise ModelFormatError("tensor overlap/range error")
        if any(payload[previous_end:offset]):
            raise ModelFormatError("nonzero payload padding")
        blob = payload[offset:offset + nbytes]
        if hashlib.sha256(blob).hexdigest() != record["sha256"]:
            raise ModelFormatError("per-tensor SHA-256 mismatch")
        previous_end = offset + nbytes
        total += nbytes
        result.tensors[key] = np.frombuffer(blob, dtype=np_dtype).reshape(shape).copy()
    if previous_end != payload_size:
        raise ModelFormatError("unreferenced trailing payload bytes")
    if manifest["tensor_count"] != len(result.tensors) or manifest["tensor_bytes"] != total:
        raise ModelFormatError("tensor totals mismatch")
    return result
