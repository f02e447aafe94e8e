"""Shared test setup: import paths, the `gpu` marker and model fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mbr-cuda-tile_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libmbr_b200.so")


@pytest.fixture(scope="session")
def csm_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("csm")


@pytest.fixture(scope="session")
def make_csm(csm_dir):
    """make_csm(preset, seed=0, **config_overrides) -> path (cached per session)."""
    import csm_tool

    cache = {}

    def _make(preset, seed=0, **ov):
        key = (preset, seed, tuple(sorted(ov.items())))
        if key not in cache:
            name = f"{preset}_{seed}_{abs(hash(key)) % 10**8}.csm"
            path = str(csm_dir / name)
            csm_tool.make_random_csm(path, preset, seed, **ov)
            cache[key] = path
        return cache[key]

    return _make
