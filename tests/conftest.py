import json
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"
MODEL = ROOT / "models" / "so3lr.so3lr"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def load_golden(name: str) -> dict:
    return json.loads((GOLDEN / f"jaxref_{name}.json").read_text())


def golden_system(fx: dict):
    from oracle.so3lr_oracle import System
    return System(pos=np.array(fx["positions"]), z=np.array(fx["z"]),
                  cell=np.array(fx["cell"]) if fx["cell"] else None,
                  charge=fx["charge"], multiplicity=fx["multiplicity"])


@pytest.fixture(scope="session")
def oracle_model():
    from oracle.so3lr_oracle import OracleModel
    return OracleModel.load(str(MODEL))


@pytest.fixture(scope="session")
def gpu_model():
    from so3lr_b200 import So3lrB200
    m = So3lrB200(MODEL, 0)
    yield m
    m.close()
