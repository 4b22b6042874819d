"""Host side of the boundary, no GPU: the C-ABI library loads and exports every
declared symbol; the `.so3lr` loader verifies integrity and refuses models the
kernels do not implement; element tokens and charge/multiplicity validation
behave like the reference's.

Reference tests mirrored: tests/test_element_map.cpp,
source/so3lr-lammps-native/tests/test_capability_rejection.py (mutated
manifests must be refused), test_loader_and_inputs.cpp (integrity checks),
so3lr_charge_spin parity rules (src/so3lr_charge_spin.cpp:116-141).
"""
import hashlib
import json
import pathlib
import re
import struct

import numpy as np
import pytest

from conftest import MODEL, ROOT

HEADER = ROOT / "include" / "so3lr_b200.h"


@pytest.fixture(scope="module")
def lib():
    from so3lr_b200 import load_library
    return load_library()


def test_library_exports_every_declared_symbol(lib):
    text = HEADER.read_text()
    declared = set(re.findall(r"^\s*(?:int|void|long long)\s*\**\s*(so3lr_\w+)\s*\(", text, re.M))
    assert len(declared) >= 15
    from so3lr_b200.runtime import EXPORTED
    assert declared == set(EXPORTED), declared ^ set(EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name


def test_inspect_shipped_model():
    from so3lr_b200 import inspect_model
    info = inspect_model(MODEL)
    assert info["layers"] == 3 and info["features"] == 128 and info["heads"] == 4 and info["head_width"] == 32
    assert info["degrees"] == 4 and info["ev_width"] == 24 and info["rbf"] == 32
    assert info["sr_cutoff"] == 4.5 and info["lr_cutoff"] == 12.0
    assert abs(info["attention_norm"] - 13.168995780096482) < 1e-12
    assert "zbl_learned" in info["summary"]


def _rewrite(tmp_path: pathlib.Path, mutate_manifest=None, mutate_bytes=None) -> pathlib.Path:
    data = bytearray(MODEL.read_bytes())
    msize, psize = struct.unpack_from("<QQ", data, 16)
    manifest = json.loads(bytes(data[128:128 + msize]))
    payload = bytes(data[128 + msize:])
    if mutate_manifest:
        mutate_manifest(manifest)
        mbytes = json.dumps(manifest, sort_keys=True, separators=(",", ":")).encode()
        data = bytearray(data[:128]) + mbytes + payload
        struct.pack_into("<QQ", data, 16, len(mbytes), len(payload))
        data[32:64] = hashlib.sha256(mbytes).digest()
    if mutate_bytes:
        mutate_bytes(data)
    out = tmp_path / "mutated.so3lr"
    out.write_bytes(bytes(data))
    return out


@pytest.mark.parametrize("change, message", [
    (lambda m: m["architecture"].__setitem__("invariant_features", 256), "invariant_features"),
    (lambda m: m["architecture"].__setitem__("use_residual_scalars", True), "model.resid_lambdas"),
    (lambda m: m["architecture"].__setitem__("repulsion_type", "nlh"), "physical.nlh_a"),
    (lambda m: m["architecture"].__setitem__("repulsion_type", "none"), "repulsion_type"),
    (lambda m: m["architecture"].__setitem__("radial_basis_features", 64), "radial_basis_features"),
    (lambda m: m["architecture"].__setitem__("brand_new_flag", 1), "unknown architecture key"),
    (lambda m: m["architecture"]["output_heads"].append("c6_ratios_output_block"), "c6_ratios_output_block"),
    (lambda m: m["architecture"]["output_heads"].append("dipole_vec_output_block"), "output heads"),
    (lambda m: m["architecture"].__setitem__("message_normalization", "softmax"), "message_normalization"),
    (lambda m: m.__setitem__("schema", "so3lr-native-model-v1"), "schema"),
    (lambda m: m["architecture"].__setitem__("interaction_blocks", 9), "interaction_blocks"),
    # a shape whose element count wraps around 2^64 to the stored byte count
    (lambda m: m["tensors"][0].__setitem__("shape", [2 ** 52, 2 ** 12] + m["tensors"][0]["shape"]), "overflows"),
])
def test_capability_rejection(tmp_path, change, message):
    from so3lr_b200 import So3lrError, inspect_model
    path = _rewrite(tmp_path, mutate_manifest=change)
    with pytest.raises(So3lrError, match=message):
        inspect_model(path)


@pytest.mark.parametrize("corrupt, message", [
    (lambda d: d.__setitem__(slice(0, 8), b"SO3LRN2\x00"), "magic"),
    (lambda d: d.__setitem__(len(d) - 1, (d[-1] ^ 0x5A) or 1), "payload SHA-256"),
    (lambda d: d.__setitem__(200, d[200] ^ 0x01), "SHA-256|JSON"),
    (lambda d: d.__setitem__(100, 1), "reserved"),
    (lambda d: d.__setitem__(8, 2), "version"),
])
def test_integrity_checks(tmp_path, corrupt, message):
    from so3lr_b200 import So3lrError, inspect_model
    path = _rewrite(tmp_path, mutate_bytes=corrupt)
    with pytest.raises(So3lrError, match=message):
        inspect_model(path)


def _with_manifest_text(tmp_path: pathlib.Path, text: str) -> pathlib.Path:
    """The shipped model with its manifest replaced by `text` (header sizes and
    manifest SHA-256 recomputed, so only the parser can object)."""
    data = bytearray(MODEL.read_bytes())
    msize = struct.unpack_from("<Q", data, 16)[0]
    payload = bytes(data[128 + msize:])
    mbytes = text.encode()
    out = bytearray(data[:128]) + mbytes + payload
    struct.pack_into("<QQ", out, 16, len(mbytes), len(payload))
    out[32:64] = hashlib.sha256(mbytes).digest()
    path = tmp_path / "manifest.so3lr"
    path.write_bytes(bytes(out))
    return path


@pytest.mark.parametrize("text, message", [
    ("[" * 100000 + "]" * 100000, "nested too deeply"),
    ('{"format": NaN}', "malformed manifest JSON value"),
    ('{"format": Infinity}', "malformed manifest JSON value"),
    ('{"format": 0x10}', "expected"),
    ('{"format": 01}', "expected"),
    ('{"format": 1.}', "malformed manifest JSON number"),
    ('{"format": 2e}', "malformed manifest JSON number"),
    ('{"format": 1e999}', "out of range"),
    ('{"format": "\\uZZZZ"}', "unicode escape"),
    ('{"format": "abc', "unterminated"),
    ('{"format": 1} x', "trailing"),
    ('{"format": 1, "format": 2}', "duplicate JSON key"),
])
def test_manifest_parser_refuses_malformed_json(tmp_path, text, message):
    """The manifest is untrusted text: anything outside JSON's grammar, numbers
    that overflow, and nesting deep enough to exhaust a recursive parser's stack
    are refused with a message."""
    from so3lr_b200 import So3lrError, inspect_model
    with pytest.raises(So3lrError, match=message):
        inspect_model(_with_manifest_text(tmp_path, text))


def test_random_corruptions_are_refused(tmp_path):
    """A model file is untrusted input: any single flipped byte (header,
    manifest or any tensor) and any truncation is refused with an error, never
    accepted and never a crash."""
    from so3lr_b200 import So3lrError, inspect_model
    rng = np.random.default_rng(2024)
    good = MODEL.read_bytes()
    msize = struct.unpack_from("<Q", good, 16)[0]
    # a spread over the three regions: header, manifest, payload
    positions = list(rng.integers(0, 128, 8)) + list(rng.integers(128, 128 + msize, 16)) + \
        list(rng.integers(128 + msize, len(good), 24))
    path = tmp_path / "corrupt.so3lr"
    for pos in positions:
        data = bytearray(good)
        data[pos] ^= int(rng.integers(1, 256))
        path.write_bytes(bytes(data))
        with pytest.raises(So3lrError):
            inspect_model(path)
    for cut in rng.integers(0, len(good), 8):
        path.write_bytes(good[:int(cut)])
        with pytest.raises(So3lrError):
            inspect_model(path)


def test_truncated_and_missing_model(tmp_path):
    from so3lr_b200 import So3lrError, inspect_model
    short = tmp_path / "short.so3lr"
    short.write_bytes(MODEL.read_bytes()[:100])
    with pytest.raises(So3lrError, match="shorter"):
        inspect_model(short)
    with pytest.raises(So3lrError, match="cannot open"):
        inspect_model(tmp_path / "nope.so3lr")
    with pytest.raises(So3lrError, match="not a regular file"):
        inspect_model(tmp_path)  # a directory
    with pytest.raises(So3lrError, match="not a regular file"):
        inspect_model("/dev/zero")  # a device that never ends is not read


def test_python_and_native_loaders_agree():
    """Both readers accept the shipped model and see the same architecture."""
    from oracle.model_io import load_model
    from so3lr_b200 import inspect_model
    m = load_model(str(MODEL))
    info = inspect_model(MODEL)
    a = m.manifest["architecture"]
    assert a["interaction_blocks"] == info["layers"]
    assert a["invariant_features"] == info["features"]
    assert a["short_range_cutoff_angstrom"] == info["sr_cutoff"]


def test_element_tokens():
    from so3lr_b200 import element_from_token
    # reference tests/test_element_map.cpp: symbols are case-insensitive, numbers 1..99
    assert element_from_token("H") == 1 and element_from_token("o") == 8 and element_from_token("CL") == 17
    assert element_from_token("Es") == 99 and element_from_token("8") == 8 and element_from_token("99") == 99
    for bad in ("0", "100", "Xx", "", "-1", "Fm"):
        assert element_from_token(bad) == 0, bad


@pytest.mark.parametrize("z, q, m, ok", [
    ([8, 1, 1], 0, 1, True),
    ([8, 1, 1], 1, 2, True),       # H2O+ doublet
    ([8, 1, 1], 1, 1, False),      # 9 electrons cannot be a singlet
    ([8, 8], 0, 3, True),          # O2 triplet
    ([8, 8], 0, 2, False),
    ([6, 1, 1, 1], 0, 2, True),    # methyl radical
    ([1], 0, 3, False),            # more unpaired electrons than electrons
    ([1], 2, 1, False),            # negative electron count
    ([8, 1, 1], 0.5, 1, False),    # non-integer charge
    ([8, 1, 1], 0, 0, False),      # multiplicity below 1
    ([8, 1, 1], 0, 1.5, False),
    ([8, 1, 1], float("nan"), 1, False),
    ([8, 1, 1], 0, float("inf"), False),
    ([8, 1, 1], 1e300, 1, False),     # out of range, not an overflowed conversion
    ([8, 1, 1], 0, 1e300, False),
])
def test_charge_multiplicity_validation(z, q, m, ok):
    from so3lr_b200 import validate_charge_spin
    problem = validate_charge_spin(z, q, m)
    assert (problem == "") == ok, problem


def test_python_binding_refuses_mismatched_arrays():
    """The library reads and writes as many rows as the system has atoms, so
    the binding checks every array's shape first: a short array is a
    ValueError, never an overrun."""
    from so3lr_b200 import So3lrB200, So3lrError
    z = np.array([8, 1, 1])
    with pytest.raises(ValueError, match="positions"):
        So3lrB200._frame(np.zeros((2, 3)), z, None, None, 0.0, 1.0)
    with pytest.raises(ValueError, match="cell"):
        So3lrB200._frame(np.zeros((3, 3)), z, np.eye(3), None, 0.0, 1.0)
    with pytest.raises(ValueError, match="atomic numbers"):
        So3lrB200._frame(np.zeros((0, 3)), [], None, None, 0.0, 1.0)
    fr, _, _ = So3lrB200._frame(np.zeros((3, 3)), z, [10.0, 11.0, 12.0], [0.0, 0.0, 0.0], 1.0, 2.0)
    assert fr.natoms == 3 and fr.periodic == 1 and fr.boxlen[1] == 11.0 and fr.multiplicity == 2.0
    h = So3lrB200.__new__(So3lrB200)  # no GPU here: only the host-side checks run
    with pytest.raises(ValueError, match="image_charge"):
        h.compute_batch(np.zeros((3, 3)), z, [0, 3], [0.0, 1.0], [1.0])
    with pytest.raises(ValueError, match="positions"):
        h.compute_batch(np.zeros((2, 3)), z, [0, 3], [0.0], [1.0])
    with pytest.raises(ValueError, match="image_offsets"):
        h.compute_batch(np.zeros((3, 3)), z, [0], [], [])
    with pytest.raises(ValueError, match="velocities"):
        h.md_init(np.zeros((3, 3)), z, None, None, np.zeros((2, 3)), np.ones(3))
    with pytest.raises(ValueError, match="masses"):
        h.md_init(np.zeros((3, 3)), z, None, None, np.zeros((3, 3)), np.ones(4))
    with pytest.raises(So3lrError, match="no evaluation"):
        h.virial_atom()
    h._natoms = 3
    with pytest.raises(ValueError, match="last evaluation had 3 atoms"):
        h.virial_atom(5)
    with pytest.raises(ValueError, match="last evaluation had 3 atoms"):
        h.md_state(2)


def test_create_without_gpu_fails_cleanly():
    """On a host without a usable GPU the handle is refused with a message, never a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from so3lr_b200 import So3lrB200, So3lrError
    with pytest.raises(So3lrError, match="CUDA|device"):
        So3lrB200(MODEL, 0)
