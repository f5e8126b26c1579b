"""Shared pytest setup: the `gpu` marker, import paths and built libraries."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "katgpt-rs_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libkgcuda.so")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def kg():
    import build as kgbuild
    kgbuild.build()
    import kgcuda
    kgcuda.lib()
    return kgcuda
