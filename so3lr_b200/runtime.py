"""ctypes binding of the C ABI in include/so3lr_b200.h.

The library ``so3lr_b200/libso3lr_b200.so`` is the only compute path: if it is
missing, or a call fails, this module raises. There is no CPU fallback.

The class mirrors what the reference's pair styles do on the host
(plugins/lammps/pair_so3lr_native_mpi.cpp, plugins/lammps/pair_so3lr_turbo.cpp):
load a model, describe its architecture (cutoffs for init_style/init_one),
validate charge and multiplicity, and evaluate energy, forces, per-atom
energies and the virial once per step.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libso3lr_b200.so"
DEFAULT_MODEL = HERE.parent / "models" / "so3lr.so3lr"

# every function the header declares (checked by the CPU tests)
EXPORTED = (
    "so3lr_create", "so3lr_describe", "so3lr_validate_charge_spin", "so3lr_element_from_token",
    "so3lr_inspect_model", "so3lr_compute", "so3lr_compute_local", "so3lr_compute_device", "so3lr_compute_batch",
    "so3lr_md_init", "so3lr_md_run", "so3lr_md_thermostat", "so3lr_md_thermostat_energy", "so3lr_md_state", "so3lr_profile", "so3lr_profile_read",
    "so3lr_launch_count", "so3lr_set_precision", "so3lr_long_range_noalloc", "so3lr_virial_atom", "so3lr_stream", "so3lr_last_stats",
    "so3lr_destroy",
    "so3lr_nccl_unique_id", "so3lr_comm_init", "so3lr_owned_atoms", "so3lr_partition",
)

_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)
_lp = C.POINTER(C.c_longlong)


class ArchInfo(C.Structure):
    _fields_ = [("abi_version", C.c_int), ("layers", C.c_int), ("features", C.c_int), ("heads", C.c_int),
                ("head_width", C.c_int), ("degrees", C.c_int), ("ev_width", C.c_int), ("rbf", C.c_int),
                ("sr_cutoff", C.c_double), ("lr_cutoff", C.c_double), ("attention_norm", C.c_double),
                ("embedding_scale", C.c_double), ("parameter_count", C.c_longlong), ("summary", C.c_char * 512)]


class Frame(C.Structure):
    _fields_ = [("natoms", C.c_longlong), ("x", _dp), ("z", _ip), ("periodic", C.c_int),
                ("boxlo", C.c_double * 3), ("boxlen", C.c_double * 3), ("total_charge", C.c_double),
                ("multiplicity", C.c_double)]


class Result(C.Structure):
    _fields_ = [("f", _dp), ("eatom", _dp), ("charges", _dp), ("ratios", _dp), ("e_learned", _dp),
                ("e_zbl", _dp), ("e_lr", _dp), ("e_elec", _dp), ("e_disp", _dp), ("energy", C.c_double),
                ("virial", C.c_double * 6)]


class LocalFrame(C.Structure):
    _fields_ = [("natoms", C.c_longlong), ("nlocal", C.c_longlong), ("tag", _lp), ("x", _dp), ("z", _ip),
                ("periodic", C.c_int), ("boxlo", C.c_double * 3), ("boxlen", C.c_double * 3),
                ("total_charge", C.c_double), ("multiplicity", C.c_double)]


class LocalResult(C.Structure):
    _fields_ = [("f", _dp), ("eatom", _dp), ("vatom", _dp), ("energy", C.c_double), ("virial", C.c_double * 6)]


class Batch(C.Structure):
    _fields_ = [("natoms", C.c_longlong), ("nimages", C.c_int), ("x", _dp), ("z", _ip), ("image_offsets", _lp),
                ("image_charge", _dp), ("image_multiplicity", _dp)]


class BatchResult(C.Structure):
    _fields_ = [("f", _dp), ("eatom", _dp), ("charges", _dp), ("image_energy", _dp)]


class So3lrError(RuntimeError):
    pass


_LIB = None


def load_library(path: os.PathLike | str | None = None) -> C.CDLL:
    """Load libso3lr_b200.so (raises when it has not been built)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise So3lrError(f"{p} is missing: build it with `python -m so3lr_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(str(p))
    lib.so3lr_create.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
    lib.so3lr_describe.argtypes = [C.c_void_p, C.POINTER(ArchInfo)]
    lib.so3lr_inspect_model.argtypes = [C.c_char_p, C.POINTER(ArchInfo), C.c_char_p, C.c_size_t]
    lib.so3lr_validate_charge_spin.argtypes = [_lp, C.c_double, C.c_double, C.c_char_p, C.c_size_t]
    lib.so3lr_element_from_token.argtypes = [C.c_char_p]
    lib.so3lr_compute.argtypes = [C.c_void_p, C.POINTER(Frame), C.POINTER(Result), C.c_char_p, C.c_size_t]
    lib.so3lr_compute_local.argtypes = [C.c_void_p, C.POINTER(LocalFrame), C.POINTER(LocalResult), C.c_char_p,
                                        C.c_size_t]
    lib.so3lr_compute_device.argtypes = [C.c_void_p, C.POINTER(Frame), C.c_void_p, C.c_void_p, _dp, _dp,
                                         C.c_char_p, C.c_size_t]
    lib.so3lr_compute_batch.argtypes = [C.c_void_p, C.POINTER(Batch), C.POINTER(BatchResult), C.c_char_p,
                                        C.c_size_t]
    lib.so3lr_md_init.argtypes = [C.c_void_p, C.POINTER(Frame), _dp, _dp, C.c_char_p, C.c_size_t]
    lib.so3lr_md_run.argtypes = [C.c_void_p, C.c_int, C.c_double, C.c_char_p, C.c_size_t]
    lib.so3lr_md_thermostat.argtypes = [C.c_void_p, C.c_double, C.c_double, C.c_int, C.c_char_p, C.c_size_t]
    lib.so3lr_md_thermostat_energy.argtypes = [C.c_void_p, _dp, C.c_char_p, C.c_size_t]
    lib.so3lr_md_state.argtypes = [C.c_void_p, _dp, _dp, _dp, _dp, C.c_char_p, C.c_size_t]
    lib.so3lr_profile.argtypes = [C.c_void_p, C.c_int]
    lib.so3lr_profile_read.argtypes = [C.c_void_p, C.c_int, _dp, _lp, _dp, C.c_char_p, C.c_size_t]
    lib.so3lr_set_precision.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]
    lib.so3lr_launch_count.argtypes = []
    lib.so3lr_launch_count.restype = C.c_longlong
    lib.so3lr_long_range_noalloc.argtypes = [C.c_void_p, C.c_longlong] + [C.c_void_p] * 11 + [C.c_void_p, C.c_char_p,
                                                                                              C.c_size_t]
    lib.so3lr_nccl_unique_id.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
    lib.so3lr_comm_init.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_char_p, C.c_size_t]
    lib.so3lr_owned_atoms.argtypes = [C.c_void_p]
    lib.so3lr_partition.argtypes = [C.c_longlong, _dp, _dp, _dp, C.c_int, _ip]
    lib.so3lr_stream.argtypes = [C.c_void_p]
    lib.so3lr_stream.restype = C.c_void_p
    lib.so3lr_last_stats.argtypes = [C.c_void_p, _lp, _lp, _lp]
    lib.so3lr_virial_atom.argtypes = [C.c_void_p, _dp, C.c_char_p, C.c_size_t]
    lib.so3lr_destroy.argtypes = [C.c_void_p]
    lib.so3lr_destroy.restype = None
    if path is None:
        _LIB = lib
    return lib


def _ptr(a: np.ndarray | None, ctype=C.c_double):
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(ctype))


def _array(a, dtype, shape: tuple, what: str) -> np.ndarray:
    """C-contiguous copy-or-view of `a` with exactly `shape`: the library reads
    and writes as many elements as the system has, so a short array is refused
    here rather than overrun there."""
    out = np.ascontiguousarray(a, dtype=dtype)
    if out.shape != shape:
        raise ValueError(f"{what} must have shape {shape}, got {out.shape}")
    return out


def _check(rc: int, err: C.Array) -> None:
    if rc != 0:
        raise So3lrError(err.value.decode(errors="replace") or f"status {rc}")


def element_from_token(token: str) -> int:
    return int(load_library().so3lr_element_from_token(token.encode()))


def validate_charge_spin(z, total_charge: float, multiplicity: float) -> str:
    """'' when valid, else the reason (so3lr_charge_spin.cpp:116-141)."""
    counts = np.zeros(119, dtype=np.int64)
    for zi in np.asarray(z).ravel():
        counts[int(zi)] += 1
    err = C.create_string_buffer(512)
    rc = load_library().so3lr_validate_charge_spin(_ptr(counts, C.c_longlong), float(total_charge),
                                                   float(multiplicity), err, 512)
    return "" if rc == 0 else err.value.decode()


def partition(x, boxlo, boxlen, nranks: int) -> np.ndarray:
    """Owner rank of every atom under the library's spatial brick partition (host only)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    lo = np.ascontiguousarray(boxlo, dtype=np.float64)
    ln = np.ascontiguousarray(boxlen, dtype=np.float64)
    out = np.empty(len(x), dtype=np.int32)
    rc = load_library().so3lr_partition(len(x), _ptr(x), _ptr(lo), _ptr(ln), int(nranks), _ptr(out, C.c_int))
    if rc != 0:
        raise So3lrError("so3lr_partition: invalid arguments")
    return out


def inspect_model(path: os.PathLike | str = DEFAULT_MODEL) -> dict:
    """Load, verify and capability-check a model on the host only (no GPU needed)."""
    info = ArchInfo()
    err = C.create_string_buffer(4096)
    _check(load_library().so3lr_inspect_model(str(path).encode(), C.byref(info), err, 4096), err)
    return _arch_dict(info)


def _arch_dict(info: ArchInfo) -> dict:
    return {k: (getattr(info, k).decode() if k == "summary" else getattr(info, k)) for k, _ in ArchInfo._fields_}


class So3lrB200:
    """One model on one GPU (the drop-in evaluator behind the pair styles)."""

    def __init__(self, model_path: os.PathLike | str = DEFAULT_MODEL, device: int = 0):
        self._lib = load_library()
        self._natoms = None
        handle = C.c_void_p()
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_create(str(model_path).encode(), int(device), C.byref(handle), err, 4096), err)
        self._h = handle

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.so3lr_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def describe(self) -> dict:
        info = ArchInfo()
        self._lib.so3lr_describe(self._h, C.byref(info))
        return _arch_dict(info)

    @property
    def stream(self) -> int:
        return int(self._lib.so3lr_stream(self._h) or 0)

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        err = C.create_string_buffer(512)
        _check(load_library().so3lr_nccl_unique_id(buf, err, 512), err)
        return buf.raw

    def comm_init(self, nranks: int, rank: int, unique_id: bytes) -> None:
        """Join a group of GPUs for spatial decomposition (see include/so3lr_b200.h)."""
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_comm_init(self._h, int(nranks), int(rank), unique_id, err, 1024), err)

    def owned_atoms(self) -> int:
        return int(self._lib.so3lr_owned_atoms(self._h))

    def profile(self, enable: bool) -> None:
        self._lib.so3lr_profile(self._h, 1 if enable else 0)

    def profile_read(self, kernel: int) -> dict:
        ms, n, fl = C.c_double(), C.c_longlong(), C.c_double()
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_profile_read(self._h, int(kernel), C.byref(ms), C.byref(n), C.byref(fl), err, 1024),
               err)
        return {"ms": ms.value, "launches": n.value, "flops": fl.value}

    PRECISIONS = {"float64": 0, "mixed": 1}

    def set_precision(self, precision: str) -> None:
        """'float64' (default) or 'mixed': the pair-filter MLPs as three-pass
        TF32 tensor-core GEMMs with float32 accumulation, the rest float64."""
        if precision not in self.PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(self.PRECISIONS)}")
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_set_precision(self._h, self.PRECISIONS[precision], err, 1024), err)

    def launch_count(self) -> int:
        return int(self._lib.so3lr_launch_count())

    def _system_size(self, natoms) -> int:
        """The atom count of the handle's current system (the library writes
        that many rows); `natoms`, when given, must agree with it."""
        n = getattr(self, "_natoms", None)
        if n is None:
            raise So3lrError("no evaluation has run on this handle")
        if natoms is not None and int(natoms) != n:
            raise ValueError(f"natoms = {natoms} but the last evaluation had {n} atoms")
        return n

    def virial_atom(self, natoms: int | None = None) -> np.ndarray:
        """Per-atom virial (natoms x 6, xx yy zz xy xz yz) of the last evaluation."""
        out = np.empty((self._system_size(natoms), 6), dtype=np.float64)
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_virial_atom(self._h, _ptr(out), err, 1024), err)
        return out

    def stats(self) -> dict:
        e, p, b = C.c_longlong(), C.c_longlong(), C.c_longlong()
        self._lib.so3lr_last_stats(self._h, C.byref(e), C.byref(p), C.byref(b))
        return {"sr_edges": e.value, "sr_pairs": p.value, "device_bytes": b.value}

    @staticmethod
    def _frame(x, z, cell, boxlo, charge, multiplicity):
        z = np.ascontiguousarray(z, dtype=np.int32)
        if z.ndim != 1 or len(z) == 0:
            raise ValueError("atomic numbers must be a non-empty 1-D array")
        x = _array(x, np.float64, (len(z), 3), "positions")
        fr = Frame()
        fr.natoms = len(z)
        fr.x = _ptr(x)
        fr.z = _ptr(z, C.c_int)
        fr.periodic = 1 if cell is not None else 0
        lo = np.zeros(3) if boxlo is None else _array(boxlo, np.float64, (3,), "boxlo")
        ln = np.zeros(3) if cell is None else _array(cell, np.float64, (3,), "cell (orthorhombic box lengths)")
        for d in range(3):
            fr.boxlo[d] = float(lo[d])
            fr.boxlen[d] = float(ln[d])
        fr.total_charge = float(charge)
        fr.multiplicity = float(multiplicity)
        return fr, x, z

    def compute(self, x, z, cell=None, boxlo=None, charge: float = 0.0, multiplicity: float = 1.0,
                terms: bool = True, forces_out=None) -> dict:
        """forces_out: optional caller-owned (n, 3) float64 C-contiguous array
        (page-locked host memory makes the copy a direct DMA) that receives the
        forces; returned as out["forces"]."""
        fr, x, z = self._frame(x, z, cell, boxlo, charge, multiplicity)
        n = len(z)
        self._natoms = None  # unknown until the call succeeds
        out = {k: np.empty(n) for k in ("eatom", "charges", "ratios", "e_learned", "e_zbl", "e_lr", "e_elec",
                                        "e_disp")} if terms else {}
        if forces_out is not None:
            if (forces_out.shape != (n, 3) or forces_out.dtype != np.float64
                    or not forces_out.flags["C_CONTIGUOUS"]):
                raise ValueError("forces_out must be a C-contiguous float64 array of shape (natoms, 3)")
            out["forces"] = forces_out
        else:
            out["forces"] = np.empty((n, 3))
        res = Result()
        res.f = _ptr(out["forces"])
        for k in ("eatom", "charges", "ratios", "e_learned", "e_zbl", "e_lr", "e_elec", "e_disp"):
            setattr(res, k, _ptr(out.get(k)))
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_compute(self._h, C.byref(fr), C.byref(res), err, 4096), err)
        self._natoms = n
        out["energy"] = res.energy
        out["virial"] = np.array(res.virial[:])
        return out

    def compute_local(self, natoms: int, tags, x, z, cell=None, boxlo=None, charge: float = 0.0,
                      multiplicity: float = 1.0, eatom: bool = True, vatom: bool = False, forces_out=None) -> dict:
        """This rank's atoms only (global tags 1..natoms); collective on a
        multi-GPU handle. Returns forces (nlocal x 3), optionally per-atom
        energies and virials of these atoms, and the whole-system energy and
        virial."""
        tags = np.ascontiguousarray(tags, dtype=np.int64)
        z = np.ascontiguousarray(z, dtype=np.int32)
        nl = len(tags)
        if tags.ndim != 1 or z.shape != (nl,):
            raise ValueError("tags and atomic numbers must be 1-D arrays of the same length")
        x = _array(x, np.float64, (nl, 3), "positions")
        fr = LocalFrame()
        fr.natoms = int(natoms)
        fr.nlocal = nl
        fr.tag = _ptr(tags, C.c_longlong)
        fr.x = _ptr(x)
        fr.z = _ptr(z, C.c_int)
        fr.periodic = 1 if cell is not None else 0
        lo = np.zeros(3) if boxlo is None else _array(boxlo, np.float64, (3,), "boxlo")
        ln = np.zeros(3) if cell is None else _array(cell, np.float64, (3,), "cell (orthorhombic box lengths)")
        for d in range(3):
            fr.boxlo[d] = float(lo[d])
            fr.boxlen[d] = float(ln[d])
        fr.total_charge = float(charge)
        fr.multiplicity = float(multiplicity)
        if forces_out is not None:
            if (forces_out.shape != (nl, 3) or forces_out.dtype != np.float64
                    or not forces_out.flags["C_CONTIGUOUS"]):
                raise ValueError("forces_out must be a C-contiguous float64 array of shape (nlocal, 3)")
            out = {"forces": forces_out}
        else:
            out = {"forces": np.empty((nl, 3))}
        if eatom:
            out["eatom"] = np.empty(nl)
        if vatom:
            out["vatom"] = np.empty((nl, 6))
        res = LocalResult()
        res.f = _ptr(out["forces"])
        res.eatom = _ptr(out.get("eatom"))
        res.vatom = _ptr(out.get("vatom"))
        err = C.create_string_buffer(4096)
        self._natoms = None
        _check(self._lib.so3lr_compute_local(self._h, C.byref(fr), C.byref(res), err, 4096), err)
        self._natoms = int(natoms)
        out["energy"] = res.energy
        out["virial"] = np.array(res.virial[:])
        return out

    def compute_batch(self, x, z, image_offsets, image_charge, image_multiplicity) -> dict:
        z = np.ascontiguousarray(z, dtype=np.int32)
        off = np.ascontiguousarray(image_offsets, dtype=np.int64)
        if z.ndim != 1 or len(z) == 0 or off.ndim != 1 or len(off) < 2:
            raise ValueError("atomic numbers must be a non-empty 1-D array and image_offsets hold K + 1 entries")
        n, nimg = len(z), len(off) - 1
        x = _array(x, np.float64, (n, 3), "positions")
        q = _array(image_charge, np.float64, (nimg,), "image_charge")
        m = _array(image_multiplicity, np.float64, (nimg,), "image_multiplicity")
        self._natoms = None
        out = {"forces": np.empty((n, 3)), "eatom": np.empty(n), "charges": np.empty(n),
               "image_energy": np.empty(nimg)}
        b = Batch(natoms=n, nimages=nimg, x=_ptr(x), z=_ptr(z, C.c_int), image_offsets=_ptr(off, C.c_longlong),
                  image_charge=_ptr(q), image_multiplicity=_ptr(m))
        r = BatchResult(f=_ptr(out["forces"]), eatom=_ptr(out["eatom"]), charges=_ptr(out["charges"]),
                        image_energy=_ptr(out["image_energy"]))
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_compute_batch(self._h, C.byref(b), C.byref(r), err, 4096), err)
        self._natoms = n
        return out

    def compute_device(self, x_ptr: int, z, cell, boxlo, f_ptr: int, charge=0.0, multiplicity=1.0):
        """Positions/forces already in device memory of this handle's GPU."""
        z = np.ascontiguousarray(z, dtype=np.int32)
        if z.ndim != 1 or len(z) == 0:
            raise ValueError("atomic numbers must be a non-empty 1-D array")
        self._natoms = None
        fr = Frame()
        fr.natoms = len(z)
        fr.x = C.cast(C.c_void_p(x_ptr), _dp)
        fr.z = _ptr(z, C.c_int)
        fr.periodic = 1 if cell is not None else 0
        for d in range(3):
            fr.boxlo[d] = 0.0 if boxlo is None else float(boxlo[d])
            fr.boxlen[d] = 0.0 if cell is None else float(cell[d])
        fr.total_charge = float(charge)
        fr.multiplicity = float(multiplicity)
        e = C.c_double()
        vir = (C.c_double * 6)()
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_compute_device(self._h, C.byref(fr), C.c_void_p(f_ptr), None, C.byref(e),
                                              C.cast(vir, _dp), err, 4096), err)
        self._natoms = len(z)
        return e.value, np.array(vir[:])

    def long_range_noalloc(self, natoms: int, x_ptr: int, q_ptr: int, ratio_ptr: int, z_ptr: int, e_lr_ptr: int,
                           e_elec_ptr: int, e_disp_ptr: int, dq_ptr: int, dh_ptr: int, f_ptr: int, w_ptr: int,
                           stream: int = 0) -> None:
        """Allocation-free long-range step on device buffers (see include/so3lr_b200.h)."""
        err = C.create_string_buffer(1024)
        ptrs = [C.c_void_p(v) for v in (x_ptr, q_ptr, ratio_ptr, z_ptr, e_lr_ptr, e_elec_ptr, e_disp_ptr, dq_ptr,
                                        dh_ptr, f_ptr, w_ptr)]
        _check(self._lib.so3lr_long_range_noalloc(self._h, int(natoms), *ptrs, C.c_void_p(stream or None), err,
                                                  1024), err)

    def md_init(self, x, z, cell, boxlo, v, mass, charge=0.0, multiplicity=1.0):
        fr, x, z = self._frame(x, z, cell, boxlo, charge, multiplicity)
        v = _array(v, np.float64, (len(z), 3), "velocities")
        mass = _array(mass, np.float64, (len(z),), "masses")
        self._natoms = None
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_md_init(self._h, C.byref(fr), _ptr(v), _ptr(mass), err, 4096), err)
        self._natoms = len(z)

    def md_thermostat(self, t_target_k: float, t_damp_ps: float, chain: int = 3) -> None:
        """Nose-Hoover chain for the following md_run calls (t_damp_ps <= 0: NVE)."""
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_md_thermostat(self._h, float(t_target_k), float(t_damp_ps), int(chain), err, 1024), err)

    def md_thermostat_energy(self) -> float:
        e = C.c_double(0.0)
        err = C.create_string_buffer(1024)
        _check(self._lib.so3lr_md_thermostat_energy(self._h, C.byref(e), err, 1024), err)
        return e.value

    def md_run(self, nsteps: int, dt_ps: float) -> None:
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_md_run(self._h, int(nsteps), float(dt_ps), err, 4096), err)

    def md_state(self, n: int | None = None) -> dict:
        n = self._system_size(n)
        x, v, f = np.empty((n, 3)), np.empty((n, 3)), np.empty((n, 3))
        e = C.c_double()
        err = C.create_string_buffer(4096)
        _check(self._lib.so3lr_md_state(self._h, _ptr(x), _ptr(v), _ptr(f), C.byref(e), err, 4096), err)
        return {"x": x, "v": v, "f": f, "energy": e.value}
