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



@pytest.fixture(scope="session")
def forced_oracle(orc):
    """forward_quantized in the oracle replaying the device's K/V codes.

    4-bit codes make the forward discontinuous: a rotated coordinate within
    rounding distance of a codebook boundary takes the neighbouring code, and
    at early positions (few attended rows) one flipped code moves the logits
    by a few percent (the oracle against itself, every weight of a 12-layer
    model at n_embd 768 perturbed by 1e-5 relative: 2.8e-2 at position 0,
    1.4e-2 to 2e-2 at positions 1..3). With the device's codes imposed on
    every store the two sides make the same quantization decisions and what
    remains is the continuous arithmetic, held to the 2e-2 bar at every
    position. Sequences run on parallel threads (the oracle call releases
    the GIL).
    """
    from concurrent.futures import ThreadPoolExecutor

    def run(be, cfg, w, toks, key_bits, val_bits):
        codes = [be.kv_codes_all(i, toks.shape[1]) for i in range(toks.shape[0])]
        c = orc.from_kg(cfg)
        with ThreadPoolExecutor(len(codes)) as ex:
            return list(ex.map(lambda i: orc.run_sequence_forced(c, w, toks[i], codes[i], key_bits, val_bits),
                               range(len(codes))))
    return run
