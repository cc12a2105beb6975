"""Shared fixtures.  ``-m gpu`` tests need a CUDA device and the built
``noetic_b200/libnoetic_gpu.so``; everything else runs on CPU."""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def nb():
    import noetic_b200

    if not os.path.exists(noetic_b200.LIB_PATH):
        noetic_b200.build()
    return noetic_b200


@pytest.fixture(scope="session")
def gpu(nb):
    """The product library with at least one visible device (gpu tests only)."""
    if nb.device_count() < 1:
        raise RuntimeError("gpu tests need a CUDA device")
    return nb


def tiny_cfg(L, vocab, **kw):
    """selftest.rs:25-27 tiny_cfg: d16 L2 expand2 k3 mlp2 tau8."""
    base = dict(vocab=vocab, d_model=16, n_layer=2, expand=2, conv_k=3, mlp_mult=2, eps=1e-5, tau_max=8.0)
    base.update(kw)
    return L(**base)


def c1_cfg(L):
    """The d=192 / 3-layer / vocab-1024 model (expand 1, conv 4, SwiGLU 3)."""
    return L(vocab=1024, d_model=192, n_layer=3, expand=1, conv_k=4, mlp_mult=3, eps=1e-5, tau_max=128.0)


def same_model(orc, nb, cfg_kw, seed):
    """The same seeded model in the oracle and in the product library."""
    om = orc.Model(orc.LmConfig(**cfg_kw), seed=seed)
    gm = nb.Model.new(nb.LmConfig(**cfg_kw), seed, device=0)
    return om, gm


def state_rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """max |a-b| / max(max|b|, 1e-6), the recurrent-state tolerance metric."""
    return float(np.abs(a - b).max() / max(float(np.abs(b).max()), 1e-6))
