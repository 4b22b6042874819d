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


# ---------------------------------------------------------------------------
# "l"-size model: F = 256 invariant features in 8 heads of 32, 64 radial
# functions, duplicated degrees {1,1,2,2,3,3,4,4} (48 equivariant channels).
# The reference accepts these widths (src/so3lr_capabilities.cpp:58-59, 74),
# but no checkpoint of that size is in this repository. The weights here are
# the shipped model's, widened: feature c = 32 h + j of the wide model stands
# for feature 32 (h // 2) + j of the shipped one (heads 2k and 2k+1 both come
# from head k, so the ev slot of head h has degree h // 2 + 1), radial function
# k for function k // 2 and ev-branch hidden unit j for unit j // 2. A weight
# whose input axis was widened is halved (both copies of an input feed it),
# and every weight is multiplied by 1 + 0.1 N(0, 1), so no two heads, slots or
# features of the wide model are equal.
# ---------------------------------------------------------------------------
L_FEATURES, L_HEADS, L_RBF = 256, 8, 64
L_REPEATS = [3, 3, 5, 5, 7, 7, 9, 9]


def _widen_index(width_new: int, width_old: int, group: int) -> np.ndarray:
    """old index of every new index when each `group`-wide block of the old axis
    appears twice in a row"""
    idx = np.arange(width_new)
    return (idx // (2 * group)) * group + idx % group


def make_l_variant(base_path, out_path, *, seed: int = 0) -> pathlib.Path:
    import math

    base = load_model(str(base_path))
    man = copy.deepcopy(base.manifest)
    arch = man["architecture"]
    F0 = int(arch["invariant_features"])
    H0 = int(arch["attention_heads"])
    R0 = int(arch["radial_basis_features"])
    assert (F0, H0, R0) == (128, 4, 32), "the base must be the shipped F=128 model"
    arch["invariant_features"] = L_FEATURES
    arch["attention_heads"] = L_HEADS
    arch["euclidean_degree_channels"] = L_HEADS
    arch["radial_basis_features"] = L_RBF
    rng = np.random.default_rng(seed)
    fmap = _widen_index(L_FEATURES, F0, 32)          # features by head blocks
    smap = np.arange(L_HEADS) // 2                    # degree slot / head
    imap = np.concatenate([fmap, F0 + smap])          # interaction layer: F features + H invariants
    rmap = np.arange(L_RBF) // 2                      # radial functions
    hmap = np.arange(2 * 32) // 2                     # ev-branch hidden units (F / 4)
    deg_of_channel = np.concatenate([[s] * r for s, r in enumerate(L_REPEATS)])
    degree_l = np.concatenate([[(r - 1) // 2] * r for r in L_REPEATS])

    def noisy(a):
        a = np.asarray(a, dtype=np.float64)
        return a * (1.0 + 0.1 * rng.standard_normal(a.shape))

    def widen(a, out_map=None, in_map=None):
        """rows by out_map, columns by in_map (halved), then noise"""
        a = np.asarray(a, dtype=np.float64)
        if out_map is not None:
            a = a[out_map]
        if in_map is not None:
            a = a[..., in_map] * 0.5
        return noisy(a)

    def block_tensor(key, a):
        part = key.split(".", 3)[3]  # after model.euclidean_transformers.<b>.
        if part.endswith("degree_repeats"):
            return np.asarray(L_REPEATS, dtype=np.int64)
        if part.endswith("so3_conv_invariants.cg_rep"):
            return 1.0 / np.sqrt(2.0 * degree_l + 1.0)
        if part.endswith("so3_conv_invariants.segment_ids"):
            return deg_of_channel.astype(np.int64)
        if part.endswith("so3_conv_invariants.segment_sum_matrix"):
            return np.eye(L_HEADS)[deg_of_channel]
        if part.split(".")[-1] in ("W_q_inv", "W_k_inv", "W_v_inv", "W_q_ev", "W_k_ev"):
            return noisy(np.asarray(a)[smap])
        if "mlp_rbf.0.weight" in part:
            return widen(a, fmap, rmap)
        if "mlp_rbf.0.bias" in part or "mlp_rbf_layer_1.0.bias" in part or "mlp_ev_layer_1.0.bias" in part:
            return widen(a, fmap)
        if "mlp_rbf_layer_1.0.weight" in part:
            return widen(a, fmap, fmap)
        if "mlp_ev.0.weight" in part:
            return widen(a, hmap, smap)
        if "mlp_ev.0.bias" in part:
            return widen(a, hmap)
        if "mlp_ev_layer_1.0.weight" in part:
            return widen(a, fmap, hmap)
        if part == "interaction_block.linear_layer.weight":
            return widen(a, imap, imap)
        if part == "interaction_block.linear_layer.bias":
            return widen(a, imap)
        if part.startswith("layer_norm_inv_") or part in ("mlp_1.1.bias", "mlp_1.3.bias"):
            return widen(a, fmap)
        if part in ("mlp_1.1.weight", "mlp_1.3.weight"):
            return widen(a, fmap, fmap)
        raise KeyError(f"no widening rule for block tensor {key}")

    def tensor(key, a):
        if key.startswith("model.euclidean_transformers."):
            return block_tensor(key, a)
        if key == "model.radial_embedding.radial_basis_fn.b":
            n = L_RBF - 1
            return np.array([math.lgamma(n + 1) - math.lgamma(k + 1) - math.lgamma(n - k + 1) for k in range(L_RBF)])
        if key == "model.radial_embedding.radial_basis_fn.k":
            return np.arange(L_RBF, dtype=np.int64)
        if key == "model.radial_embedding.radial_basis_fn.k_rev":
            return (L_RBF - 1 - np.arange(L_RBF)).astype(np.int64)
        if key in ("model.inv_feature_embedding.embedding.weight", "model.charge_embedding.Wq.weight",
                   "model.spin_embedding.Wq.weight"):
            return widen(a, fmap)
        if key in ("model.charge_embedding.Wk", "model.charge_embedding.Wv", "model.spin_embedding.Wk",
                   "model.spin_embedding.Wv"):
            return noisy(np.asarray(a)[:, fmap])
        if key.endswith("embedding.mlp.1.weight") or key.endswith("embedding.mlp.3.weight"):
            return widen(a, fmap, fmap)
        if key in ("model.atomic_energy_output_block.layers.0.weight",
                   "model.partial_charges_output_block.transform_inv_features.0.weight",
                   "model.hirshfeld_output_block.transform_features.0.weight"):
            return widen(a, None, fmap)
        return a

    tensors = []
    for rec in man["tensors"]:
        key = rec["state_key"]
        tensors.append((rec, tensor(key, base.tensors[key])))
    return write_model(out_path, man, tensors)
