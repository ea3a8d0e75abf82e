import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; compares the CUDA path with the oracle")


@pytest.fixture(scope="session")
def c1_config():
    from yue2_rs_b200 import synth
    return synth.config_c1()


@pytest.fixture(scope="session")
def c1_dir(tmp_path_factory, c1_config):
    """the reduced model as a safetensors checkpoint (seed 0)."""
    from yue2_rs_b200 import synth
    return synth.write_checkpoint(str(tmp_path_factory.mktemp("c1")), c1_config, seed=0)


@pytest.fixture(scope="session")
def c1u_dir(tmp_path_factory, c1_config):
    """The reduced model with unit-mean RMSNorm gains (1 + N(0, 0.02)): activations and
    logits of order one, the sensitive variant for numerical parity."""
    from yue2_rs_b200 import synth
    return synth.write_checkpoint(str(tmp_path_factory.mktemp("c1u")), c1_config, seed=0, norm_mean=1.0)


def _oracle(path, config):
    from oracle.oracle import OracleModel
    from yue2_rs_b200 import checkpoint
    return OracleModel.from_tensors(config, checkpoint.tensors(path))


@pytest.fixture(scope="session")
def c1_oracle(c1_dir, c1_config):
    return _oracle(c1_dir, c1_config)


@pytest.fixture(scope="session")
def c1u_oracle(c1u_dir, c1_config):
    return _oracle(c1u_dir, c1_config)


@pytest.fixture(scope="session")
def c1_device(c1_dir):
    from yue2_rs_b200 import Model
    m = Model.open(c1_dir)
    yield m
    m.close()


@pytest.fixture(scope="session")
def c1u_device(c1u_dir):
    from yue2_rs_b200 import Model
    m = Model.open(c1u_dir)
    yield m
    m.close()


@pytest.fixture(scope="session")
def c1_prompt(c1_config):
    """256 token ids uniform over the vocabulary (seeded) and 64 teacher-forced ids."""
    rng = np.random.default_rng(12345)
    return (rng.integers(0, c1_config.vocab_size, 256).tolist(), rng.integers(0, c1_config.vocab_size, 64).tolist())


@pytest.fixture(scope="session")
def nar_tiny_dir(tmp_path_factory):
    """The small real-vocabulary model (unit-mean gains) with its NAR tensors."""
    from yue2_rs_b200 import synth
    return synth.write_checkpoint(str(tmp_path_factory.mktemp("nar_tiny")), synth.config_nar_tiny(), seed=6,
                                  norm_mean=1.0)
