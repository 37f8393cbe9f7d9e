"""pytest setup: the `gpu` marker, import paths and shared fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "seedvr2-2b-ncnn_b200"), ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def port():
    from oracle import pyoracle as po
    if not po.have_port():
        pytest.fail("oracle/_build/liboracle.so missing: run __graft_entry__.build()")
    return po.Port()


@pytest.fixture(scope="session")
def ref():
    from oracle import pyoracle as po
    if not po.have_ref():
        pytest.skip("reference library oracle/_ref/libref_dit.so not built here")
    return po.Ref()


@pytest.fixture(scope="session")
def m5_small(tmp_path_factory):
    """Synthetic m5 directory (seed 1234) with layers 0, 1, 30, 31."""
    import cases
    import s2b
    d = str(tmp_path_factory.mktemp("m5_small"))
    s2b.synth_write_m5(d, cases.DIT_SMALL["wseed"], 0, 2)
    s2b.synth_write_m5(d, cases.DIT_SMALL["wseed"], 30, 32)
    return d
