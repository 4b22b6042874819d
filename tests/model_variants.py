"""Synthetic `.so3lr` model files exercising the optional operators a model
descriptor can ask for (src/so3lr_capabilities.cpp:46-80 in the reference):
RMSNorm without scale, no second block norm, query/key normalisation,
residual scalars and the NLH pair-table repulsion. No released checkpoint uses
them, so each variant is the shipped model with the manifest flags switched,
the tensors the operator needs added (seeded values) and the tensors it no
longer reads removed. The writer produces the container layout the loaders
check (native_model.cpp:338-405): 128-byte header, canonical JSON manifest,
64-byte aligned tensors with per-tensor SHA-256.
"""
from __future__ import annotations

import copy
import hashlib
import json
import pathlib
import struct

import numpy as np

from oracle.model_io import load_model

_NP = {"float64": "<f8", "float32": "<f4", "int64": "<i8", "int32": "<i4", "uint8": "u1", "bool": "u1"}


def write_model(path, manifest: dict, tensors: list) -> pathlib.Path:
    """tensors: list of (record, array) in file order; record holds name,
    state_key, dtype, role; shape, offset, nbytes and sha256 are filled here."""
    manifest = copy.deepcopy(manifest)
    payload = bytearray()
    records = []
    for rec, arr in tensors:
        rec = dict(rec)
        arr = np.array(arr, dtype=_NP[rec["dtype"]], order="C")  # keeps 0-d tensors 0-d
        while len(payload) % 64:
            payload.append(0)
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
    manifest["architecture"]["state_tensor_count"] = len(records)
    mbytes = json.dumps(manifest, sort_keys=True, separators=(",", ":"), ensure_ascii=False).encode("utf-8")
    header = bytearray(128)
    header[0:8] = b"SO3LRN1\x00"
    struct.pack_into("<IIQQ", header, 8, 1, 0, len(mbytes), len(payload))
    header[32:64] = hashlib.sha256(mbytes).digest()
    header[64:96] = hashlib.sha256(bytes(payload)).digest()
    path = pathlib.Path(path)
    path.write_bytes(bytes(header) + mbytes + bytes(payload))
    return path


def make_variant(base_path, out_path, *, rms_norm: bool = False, second_norm: bool = True, qk_norm: bool = False,
                 residual_scalars=None, nlh_capacity: int | None = None, attention_norm_factor: float = 1.0,
                 c6_keys: int | None = None, hirshfeld_keys: int | None = None, seed: int = 0) -> pathlib.Path:
    """The shipped model with optional operators switched on.

    residual_scalars: (resid, x0) lists of length interaction_blocks, or None.
    nlh_capacity: size of the NLH pair tables (elements 1..capacity), or None.
    c6_keys: add a C6 ratio head with this many keys (its first layer copied
    from the Hirshfeld head, the rest seeded so that ratios stay near 1).
    hirshfeld_keys: replace the Hirshfeld head's second layer by a seeded one
    with this many keys (K = 1 is the a0 head of C6-head models).
    attention_norm_factor: multiplies avg_num_neighbors (the attention
    normaliser). The shipped weights were not trained for query/key
    normalisation or without the second norm; there the features grow without
    bound through the blocks unless the attention is damped (x20 keeps water
    energies and forces in the normal range).
    """
    base = load_model(str(base_path))
    man = copy.deepcopy(base.manifest)
    arch = man["architecture"]
    layers = int(arch["interaction_blocks"])
    arch["avg_num_neighbors"] = float(arch["avg_num_neighbors"]) * attention_norm_factor
    by_key = {r["state_key"]: r for r in man["tensors"]}
    drop = set()
    tensors = []
    if rms_norm:
        arch["use_rms_norm"] = True
        # RMSNorm(use_scale=False) has no parameters
        for b in range(layers):
            for pos in (1, 2):
                for part in ("weight", "bias"):
                    drop.add(f"model.euclidean_transformers.{b}.layer_norm_inv_{pos}.{part}")
    if not second_norm:
        arch["layer_normalization_2"] = False
        for b in range(layers):
            for part in ("weight", "bias"):
                drop.add(f"model.euclidean_transformers.{b}.layer_norm_inv_2.{part}")
    if qk_norm:
        arch["qk_norm"] = True
    rng = np.random.default_rng(seed)

    def seeded_keys(prefix, keys):
        """second layer, key embeddings and shifts of a ratio head with `keys` keys"""
        out = {prefix + "transform_features.2.weight": 0.05 * rng.standard_normal((keys, 64)),
               prefix + "transform_features.2.bias": 0.05 * rng.standard_normal(keys),
               prefix + "q_embedding.weight": 0.5 * rng.standard_normal((100, keys)),
               prefix + "v_shift_embedding.weight": 1.0 + 0.1 * rng.standard_normal((100, 1))}
        return out

    replace = {}
    if hirshfeld_keys is not None:
        replace.update(seeded_keys("model.hirshfeld_output_block.", int(hirshfeld_keys)))
    for key, rec in by_key.items():
        if key not in drop:
            tensors.append((rec, replace.get(key, base.tensors[key])))
    if c6_keys is not None:
        arch["output_heads"] = list(arch["output_heads"]) + ["c6_ratios_output_block"]
        src = "model.hirshfeld_output_block."
        dst = "model.c6_ratios_output_block."
        new = {dst + "transform_features.0.weight": base.tensors[src + "transform_features.0.weight"],
               dst + "transform_features.0.bias": base.tensors[src + "transform_features.0.bias"]}
        new.update(seeded_keys(dst, int(c6_keys)))
        for key, vals in new.items():
            tensors.append(({"name": key, "state_key": key, "dtype": "float64", "role": "parameter"}, vals))
    if residual_scalars is not None:
        arch["use_residual_scalars"] = True
        resid, x0 = residual_scalars
        assert len(resid) == layers and len(x0) == layers
        for key, vals in (("model.resid_lambdas", resid), ("model.x0_lambdas", x0)):
            tensors.append(({"name": key, "state_key": key, "dtype": "float64", "role": "parameter"},
                            np.asarray(vals, dtype=np.float64)))
    if nlh_capacity is not None:
        arch["repulsion_type"] = "nlh"
        cap = int(nlh_capacity)
        amp = np.empty((cap, cap, 3))
        rate = np.empty((cap, cap, 3))
        for i in range(cap):
            for j in range(i, cap):
                a = np.array([0.25, 0.55, 0.20]) * (1.0 + 0.2 * rng.random(3))
                r = np.sort(2.0 + 10.0 * rng.random(3))[::-1]
                amp[i, j] = amp[j, i] = a
                rate[i, j] = rate[j, i] = r
        for key, vals in (("physical.nlh_a", amp), ("physical.nlh_b", rate)):
            tensors.append(({"name": key, "state_key": key, "dtype": "float64", "role": "physical_constant"}, vals))
    return write_model(out_path, man, tensors)
