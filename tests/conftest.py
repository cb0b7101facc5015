"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200; run with -m gpu);
* imports the package directory ``comfyui-powershard_b200/`` as
  ``powershard_b200`` and puts the repository root on sys.path for
  ``oracle`` (the CPU checker);
* ``gloo_available`` reports a forbidden Gloo transport as a skip labelled
  NOT_RUN, never as a pass (like the reference's test_sequence_distributed).
"""
from __future__ import annotations

import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built libps_b200.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import ulysses_oracle
    return ulysses_oracle


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on a B200; fails (never skips) when it cannot load."""
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    from powershard_b200 import _lib, build_lib
    build_lib.build()
    return _lib.load()


@pytest.fixture(scope="session")
def gloo_available(tmp_path_factory):
    import torch.distributed as dist
    directory = tmp_path_factory.mktemp("gloo-probe")
    try:
        dist.init_process_group("gloo", init_method=(directory / "store").as_uri(), rank=0, world_size=1,
                                timeout=timedelta(seconds=10))
    except RuntimeError as error:
        if "Operation not permitted" in str(error):
            pytest.skip("NOT_RUN: environment forbids Gloo TCP transport")
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
