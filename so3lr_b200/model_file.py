"""Read, check, dump and write `.so3lr` model files.

The container (format version 1) is the interface the reference defines in
source/so3lr-lammps-native/docs/FORMAT.md: a 128-byte header (magic
``SO3LRN1\\0``, u32 version 1, u32 flags 0, u64 manifest bytes, u64 payload
bytes, SHA-256 of the manifest, SHA-256 of the payload, 32 zero bytes), the
manifest as canonical JSON (sorted keys, no spaces, UTF-8), and a payload of
little-endian tensors at 64-byte aligned offsets with zero padding, each with
its own SHA-256 in the manifest. This module is the user-side counterpart of
the reference's tools/checkpoint_conversion/so3lr_native_format.py:

    python -m so3lr_b200.model_file MODEL [--manifest OUT.json]

checks MODEL with the library's own loader (every integrity rule plus the
capability negotiation that decides whether this build can run it) and prints
a summary; ``write_model`` writes a file from a manifest and tensors (for
example a model with edited tensors or flags), filling in offsets, sizes and
hashes.
"""
from __future__ import annotations

import argparse
import copy
import hashlib
import json
import pathlib
import struct
import sys

import numpy as np

MAGIC = b"SO3LRN1\x00"
HEADER_BYTES = 128
ALIGNMENT = 64
_NP = {"float64": "<f8", "float32": "<f4", "int64": "<i8", "int32": "<i4", "uint8": "u1", "bool": "u1"}


def canonical_json(manifest: dict) -> bytes:
    return json.dumps(manifest, sort_keys=True, separators=(",", ":"), ensure_ascii=False).encode("utf-8")


def read_manifest(path) -> tuple[dict, bytes]:
    """The manifest and the payload bytes of a model file (layout checks only;
    ``check`` runs the full integrity rules)."""
    raw = pathlib.Path(path).read_bytes()
    if len(raw) < HEADER_BYTES or raw[:8] != MAGIC:
        raise ValueError(f"{path}: not a .so3lr file (bad size or magic)")
    version, flags, msize, psize = struct.unpack_from("<IIQQ", raw, 8)
    if version != 1 or flags != 0 or HEADER_BYTES + msize + psize != len(raw):
        raise ValueError(f"{path}: unsupported version/flags or sizes that disagree with the file")
    manifest = json.loads(raw[HEADER_BYTES:HEADER_BYTES + msize].decode("utf-8"))
    return manifest, raw[HEADER_BYTES + msize:]


def tensors(path) -> dict:
    """state_key -> numpy array (little-endian, the manifest's shape)."""
    manifest, payload = read_manifest(path)
    out = {}
    for rec in manifest["tensors"]:
        blob = payload[rec["offset"]:rec["offset"] + rec["nbytes"]]
        out[rec["state_key"]] = np.frombuffer(blob, dtype=_NP[rec["dtype"]]).reshape(rec["shape"]).copy()
    return out


def write_model(path, manifest: dict, tensor_list: list) -> pathlib.Path:
    """Write a model file. tensor_list: (record, array) pairs in file order;
    each record holds name, state_key, dtype and role; shape, offset, nbytes and
    sha256 are filled in here, as are tensor_count, tensor_bytes and
    architecture.state_tensor_count."""
    manifest = copy.deepcopy(manifest)
    payload = bytearray()
    records = []
    for rec, arr in tensor_list:
        rec = dict(rec)
        arr = np.array(arr, dtype=_NP[rec["dtype"]], order="C")  # keeps 0-d tensors 0-d
        payload += bytes((-len(payload)) % ALIGNMENT)
        blob = arr.tobytes()
        rec["shape"] = [int(s) for s in arr.shape]
        rec["offset"] = len(payload)
        rec["nbytes"] = len(blob)
        rec["sha256"] = hashlib.sha256(blob).hexdigest()
        payload += blob
        records.append(rec)
    manifest["tensors"] = records
    manifest["tensor_count"] = len(records)
    manifest["tensor_bytes"] = sum(r["nbytes"] for r in records)
    if "architecture" in manifest:
        manifest["architecture"]["state_tensor_count"] = len(records)
    mbytes = canonical_json(manifest)
    header = bytearray(HEADER_BYTES)
    header[0:8] = MAGIC
    struct.pack_into("<IIQQ", header, 8, 1, 0, len(mbytes), len(payload))
    header[32:64] = hashlib.sha256(mbytes).digest()
    header[64:96] = hashlib.sha256(bytes(payload)).digest()
    path = pathlib.Path(path)
    path.write_bytes(bytes(header) + mbytes + bytes(payload))
    return path


def check(path) -> dict:
    """Full check by the library's loader: header, hashes, canonical manifest,
    tensor layout, architecture record and capability negotiation. Returns the
    architecture record; raises So3lrError with the loader's message."""
    from .runtime import inspect_model
    return inspect_model(str(path))


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description="check a .so3lr model file and print its summary")
    parser.add_argument("model", type=pathlib.Path)
    parser.add_argument("--manifest", type=pathlib.Path, help="write the manifest as indented JSON")
    args = parser.parse_args(argv)
    from .runtime import So3lrError
    try:
        info = check(args.model)
    except So3lrError as exc:
        print(f"native_model_check=FAIL\n{exc}")
        return 1
    manifest, payload = read_manifest(args.model)
    if args.manifest:
        args.manifest.write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    arch = manifest.get("architecture", {})
    print(f"format_version={manifest.get('format_version')}")
    print(f"model_family={manifest.get('model_family')}")
    print(f"tensor_count={manifest.get('tensor_count')}")
    print(f"tensor_bytes={manifest.get('tensor_bytes')}")
    print(f"payload_bytes={len(payload)}")
    print(f"short_range_cutoff={arch.get('short_range_cutoff_angstrom')}")
    print(f"long_range_cutoff={arch.get('long_range_cutoff_angstrom')}")
    print(f"architecture={info['summary']}")
    print("native_model_check=PASS")
    return 0


if __name__ == "__main__":
    sys.exit(main())
