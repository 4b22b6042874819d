"""Synthetic `.so3lr` model files exercising the optional operators a model
descriptor can ask for (src/so3lr_capabilities.cpp:46-80 in the reference):
RMSNorm without scale, no second block norm, query/key normalisation,
residual scalars and the NLH pair-table repulsion. No released checkpoint uses
them, so each variant is the shipped model with the manifest flags switched,
the tensors the operator needs added (seeded values) and the tensors it no
longer reads removed, written by so3lr_b200.model_file.write_model.
"""
from __future__ import annotations

import copy
import pathlib

import numpy as np

from oracle.model_io import load_model
from so3lr_b200.model_file import write_model

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
