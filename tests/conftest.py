"""Shared test setup: markers, import paths, seeded inputs."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.lib()
    return o


def rand_weights(rng, d_model, n_heads, scale=0.02, use_bias=True, out_bias=True):
    """Seeded rel-pos MHA parameters (N(0, scale^2)), the shapes of
    RelPositionMultiHeadAttention::new (attention.rs:367-406)."""
    dh = d_model // n_heads
    f = lambda *s: (rng.standard_normal(s) * scale).astype(np.float32)
    w = {
        "wq": f(d_model, d_model), "wk": f(d_model, d_model),
        "wv": f(d_model, d_model), "wo": f(d_model, d_model),
        "wp": f(d_model, d_model),
        "pos_bias_u": f(n_heads, dh), "pos_bias_v": f(n_heads, dh),
    }
    for name in ("bq", "bk", "bv"):
        w[name] = f(d_model) if use_bias else None
    w["bo"] = f(d_model) if (use_bias and out_bias) else None
    return w
