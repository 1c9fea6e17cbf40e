import os
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE / "golden"))
sys.path.insert(0, str(HERE.parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")
    config.addinivalue_line("markers", "slow: larger CPU cases")


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle, build_oracle
    build_oracle(ref=True)
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle_lib import RefLib, ref_library_path
    if ref_library_path() is None:
        pytest.skip("oracle/_ref (the reference compiled here) is not built for this host")
    return RefLib()


@pytest.fixture(scope="session")
def tiny_model_path():
    import synth_model as sm
    return sm.cached_model("tiny", sm.tiny_hparams(), "Q4_K_M", seed=0)


@pytest.fixture(scope="session")
def tiny_q8_path():
    import synth_model as sm
    return sm.cached_model("tiny", sm.tiny_hparams(), "Q8_0", seed=1)


@pytest.fixture(autouse=True)
def _release_device_copies():
    yield
    gl = sys.modules.get("gpulib")
    if gl is not None and gl._KEEP:
        gl.release()
