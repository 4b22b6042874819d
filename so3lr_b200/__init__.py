"""B200-native SO3LR force evaluation (drop-in for the `so3lr/native/mpi` and
`so3lr/turbo` LAMMPS pair-style path of CPradaL/so3lrxlammps).

The compute path is the CUDA library `libso3lr_b200.so` behind the C ABI in
`include/so3lr_b200.h`; `so3lr_b200.runtime` binds it with ctypes.
"""
from .runtime import (So3lrB200, So3lrError, element_from_token, inspect_model, load_library,  # noqa: F401
                      validate_charge_spin)

__all__ = ["So3lrB200", "So3lrError", "element_from_token", "inspect_model", "load_library",
           "validate_charge_spin"]
