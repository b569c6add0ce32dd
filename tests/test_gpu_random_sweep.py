"""A seeded random sweep of the offline forward (RelPositionMultiHeadAttention
::forward, src/asr/modules/encoders/attention.rs:446-573) through the C ABI
against the CPU oracle: batch 1-4, 1-520 frames, random key-padding lengths,
no context / regular windows / chunked_limited contexts of random sizes,
d_model 256-1024, bf16 (tolerance 2e-2) and f32 (1e-4) modules, with the
bounds of tests/test_gpu_parity.py; and forward_with_cache (606-816) over
six chunks of random cache, chunk, drop and context sizes.  The cases are drawn once from fixed
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


N_STREAM_CASES = 24


def draw_stream_case(i):
    rng = np.random.default_rng(95000 + i)
    bf = i % 4 != 3
    D, H = [(256, 2), (1024, 8)][int(rng.integers(0, 2))] if bf else [(64, 2), (256, 2)][
        int(rng.integers(0, 2))]
    B = int(rng.integers(1, 5))
    C = int(rng.integers(1, 121))
    T = int(rng.integers(1, 41))
    drop = int(rng.integers(0, min(3, T - 1) + 1)) if T > 1 else 0
    ctx = None
    if rng.random() < 0.7:
        ctx = (int(rng.integers(0, C + 1)), int(rng.integers(0, 16)), bool(rng.random() < 0.5))
    return dict(seed=95000 + i, bf=bf, D=D, H=H, B=B, C=C, T=T, drop=drop, ctx=ctx)


@pytest.mark.parametrize("i", range(N_STREAM_CASES))
def test_random_streaming_case(nrp, orc, i):
    """forward_with_cache (attention.rs:606-816) over six chunks of a random
    case: outputs and the exported attention-input cache against the
    oracle's streaming step, the last chunk with valid = T - 2."""
    import torch
    c = draw_stream_case(i)
    bf, D, H, B, C, T, drop, ctx = (c[k] for k in ("bf", "D", "H", "B", "C", "T", "drop", "ctx"))
    dtype = nrp.BF16 if bf else nrp.F32
    tol = TOL_BF16 if bf else TOL_F32
    rng = np.random.default_rng(c["seed"] + 1)
    w = rand_weights(rng, D, H, scale=0.02 if bf else 0.2)
    attn = make_module(nrp, w, D, H, dtype)
    attn.cache_drop_size = drop
    cache = nrp.AttentionCache(attn, B, C)
    pe = nrp.RelPositionalEncoding(D, 5000, False)
    pe.set_dtype(dtype)
    pos = pe.get_encoding(C + T)
    pos_h = pe.get_encoding_host(C + T)[0]
    context = nrp.AttentionContext.new(ctx[:2], "chunked_limited" if ctx[2] else "regular") \
        if ctx else None
    h_ref = np.zeros((B, C, D), np.float32)
    filled = 0
    tdt = torch.bfloat16 if bf else torch.float32
    for step in range(6):
        x = rng.standard_normal((B, T, D)).astype(np.float32)
        if bf:
            x = orc.bf16_round(x)
        valid = T if step < 5 else max(T - 2, 0)
        out = attn.forward_with_cache(torch.from_numpy(x).to("cuda", tdt), pos, cache, filled,
                                      valid, context)
        attn.ctx.check()
        got = out.float().cpu().numpy()
        l, r = (ctx[0], ctx[1]) if ctx else (-1, -1)
        ref, nxt = orc.stream_layer_step(x, w, pos_h, H, h_ref, filled, valid, l, r,
                                         bool(ctx and ctx[2]), drop, bf16=bf)
        if valid > 0:
            check_close(got, ref, [valid] * B, tol)
        hc = cache.export_h().cpu().numpy()
        assert np.abs(hc - h_ref).max() <= (1e-6 if bf else 0), (c, step)
        filled = nxt
