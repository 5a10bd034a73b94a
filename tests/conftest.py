"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked ``gpu`` need a B200 and the built CUDA library; everything else
runs on the CPU (the oracle, the GGUF parsers, the host logic, and that the
C-ABI library loads and exports every declared symbol).
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libllmb200.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc

    orc.lib()
    orc.set_threads(min(8, os.cpu_count() or 1))
    return orc


@pytest.fixture(scope="session")
def model_path():
    """Returns a function: spec name -> path of its synthetic GGUF file."""
    from llm_b200 import synth

    return synth.ensure
