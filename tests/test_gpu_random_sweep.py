"""A seeded random sweep of the offline forward (RelPositionMultiHeadAttention
::forward, src/asr/modules/encoders/attention.rs:446-573) through the C ABI
against the CPU oracle: batch 1-4, 1-520 frames, random key-padding lengths,
no context / regular windows / chunked_limited contexts of random sizes,
d_model 256-1024, bf16 (tolerance 2e-2) and f32 (1e-4) modules, with the
bounds of tests/test_gpu_parity.py.  The cases are drawn once from fixed
seeds, so a failure names a reproducible case."""
import numpy as np
import pytest

from conftest import rand_weights
from test_gpu_parity import (TOL_BF16, TOL_F32, check_close, make_module,  # noqa: F401
                             run_forward, nrp)

pytestmark = pytest.mark.gpu

N_CASES = 64


def draw_case(i):
    rng = np.random.default_rng(90000 + i)
    f32 = i % 4 == 3
    D, H = (256, 2) if f32 else [(256, 2), (512, 4), (1024, 8)][int(rng.integers(0, 3))]
    B = int(rng.integers(1, 5))
    T = int(rng.integers(1, 521))
    lengths = None
    if rng.random() < 0.7:
        lengths = rng.integers(1, T + 1, B).astype(np.int32)
        if rng.random() < 0.5:
            lengths[int(rng.integers(0, B))] = T
        if (lengths == T).all():
            lengths = None  # no frame is padding: key_padding_mask gives None
    context = None
    u = rng.random()
    if u < 0.3:
        left, right = int(rng.integers(-1, 200)), int(rng.integers(-1, 200))
        if left >= 0 or right >= 0:
            context = (left, right, False)
    elif u < 0.6:
        context = (int(rng.integers(-1, 150)), int(rng.integers(-1, 21)), True)
    return dict(seed=90000 + i, f32=f32, D=D, H=H, B=B, T=T, lengths=lengths, context=context)


@pytest.mark.parametrize("i", range(N_CASES))
def test_random_offline_case(nrp, orc, i):
    c = draw_case(i)
    rng = np.random.default_rng(c["seed"] + 1)
    dtype = nrp.F32 if c["f32"] else nrp.BF16
    w = rand_weights(rng, c["D"], c["H"])
    x = rng.standard_normal((c["B"], c["T"], c["D"])).astype(np.float32)
    attn = make_module(nrp, w, c["D"], c["H"], dtype)
    got, pe = run_forward(nrp, attn, x, c["T"], c["lengths"], c["context"], dtype)
    assert np.isfinite(got).all(), c
    ref = orc.mha_forward(x, w, pe, c["H"], lengths=c["lengths"], context=c["context"],
                          bf16=not c["f32"])
    check_close(got, ref, c["lengths"], TOL_F32 if c["f32"] else TOL_BF16)
