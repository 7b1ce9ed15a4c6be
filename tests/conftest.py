import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("4pe_u250_b200")


@pytest.fixture(scope="session")
def F():
    return importlib.import_module("4pe_u250_b200.formats")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("4pe_u250_b200.synth")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def rope_lut(F):
    return F.generate_rope_lut()


@pytest.fixture(scope="session")
def rope_tables(oracle, rope_lut):
    return oracle.rope_tables(rope_lut)
