"""The CPU oracle of the streaming Conformer block (oracle.stream_block_step:
ConformerBlock::forward_with_cache with ConvolutionModule::forward_with_cache,
src/asr/modules/encoders/conformer.rs:1877-1967, 2332-2400, driven as
forward_streaming does, 883-1000).

The reference holds no test of it.  It is pinned to the offline block oracle
(itself checked against a torch composition) through two properties of a
causal block (left-padded depthwise conv):

- one chunk against an empty cache (fill level 0: the cache keys are hidden,
  the conv cache is zeros) equals the offline block on that chunk;
- a stream of chunks with a one-chunk cache and the chunked_limited context
  of a cache-aware model equals the offline block with that context over the
  concatenated chunks: every row sees the same keys and conv context.
"""
import numpy as np
import pytest

from conftest import rand_block


@pytest.fixture(scope="module")
def orc():
    from oracle import oracle
    return oracle


def offline(orc, x, bw, H, ff, K, conv_norm):
    T, D = x.shape[1], x.shape[2]
    return orc.block_forward(x, bw, orc.get_encoding(D, 5000, T), H, ff, K, causal=True,
                             conv_norm=conv_norm, bf16=False)


@pytest.mark.parametrize("conv_norm", [0, 1])
def test_first_chunk_equals_offline_causal_block(orc, conv_norm):
    rng = np.random.default_rng(31 + conv_norm)
    B, T, C, D, H, ff, K = 2, 14, 20, 64, 2, 128, 9
    bw, _ = rand_block(rng, D, H, ff, K, "batch_norm" if conv_norm == 0 else "layer_norm")
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    hc = np.zeros((B, C, D), np.float32)
    cc = np.zeros((B, K - 1, D), np.float32)
    got, nxt = orc.stream_block_step(x, bw, orc.get_encoding(D, 5000, C + T), H, ff, K, hc, cc,
                                     0, T, conv_norm=conv_norm, bf16=False)
    want = offline(orc, x, bw, H, ff, K, conv_norm)
    assert nxt == T
    assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("conv_norm", [0, 1])
def test_stream_equals_offline_chunked_context(orc, conv_norm):
    """Three chunks of T frames with a T-frame cache and chunked_limited
    [T, T-1]: each chunk sees itself and the chunk before.  The offline
    causal block over the concatenation with the same context gives the same
    rows (the conv cache carries the last K-1 GLU frames, the attention cache
    the previous chunk's inputs)."""
    rng = np.random.default_rng(7 + conv_norm)
    B, T, n, D, H, ff, K = 2, 10, 3, 64, 2, 128, 9
    bw, _ = rand_block(rng, D, H, ff, K, "batch_norm" if conv_norm == 0 else "layer_norm")
    x = rng.standard_normal((B, n * T, D)).astype(np.float32)
    C = T
    hc = np.zeros((B, C, D), np.float32)
    cc = np.zeros((B, K - 1, D), np.float32)
    pe = orc.get_encoding(D, 5000, C + T)
    f, outs = 0, []
    for k in range(n):
        y, f = orc.stream_block_step(np.ascontiguousarray(x[:, k * T:(k + 1) * T]), bw, pe, H,
                                     ff, K, hc, cc, f, T, T, T - 1, True, conv_norm=conv_norm,
                                     bf16=False)
        outs.append(y)
    got = np.concatenate(outs, axis=1)
    want = orc.block_forward(x, bw, orc.get_encoding(D, 5000, n * T), H, ff, K, causal=True,
                             conv_norm=conv_norm, context=(T, T - 1, True), bf16=False)
    assert f == C
    assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())


def test_conv_cache_holds_the_last_glu_frames_and_padding_is_zeroed(orc):
    """Frames past `valid` reach neither the conv cache nor the valid rows'
    depthwise inputs: changing them leaves the cache's valid part alone."""
    rng = np.random.default_rng(3)
    B, T, C, D, H, ff, K = 1, 14, 14, 64, 2, 128, 5
    bw, _ = rand_block(rng, D, H, ff, K)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    pe = orc.get_encoding(D, 5000, C + T)
    runs = []
    for scale in (1.0, 50.0):
        x2 = x.copy()
        x2[:, 10:] *= scale
        hc = np.zeros((B, C, D), np.float32)
        cc = np.zeros((B, K - 1, D), np.float32)
        orc.stream_block_step(x2, bw, pe, H, ff, K, hc, cc, 0, 10, bf16=True)
        runs.append(cc.copy())
    # the last K-1 = 4 frames are frames 10..13: all past valid -> zeros
    assert np.array_equal(runs[0], np.zeros_like(runs[0]))
    assert np.array_equal(runs[0], runs[1])


def test_bf16_close_to_f32(orc):
    rng = np.random.default_rng(12)
    B, T, C, D, H, ff, K = 2, 14, 28, 128, 2, 256, 9
    bw, _ = rand_block(rng, D, H, ff, K)
    pe = orc.get_encoding(D, 5000, C + T)
    outs = []
    for bf16 in (False, True):
        hc = np.zeros((B, C, D), np.float32)
        cc = np.zeros((B, K - 1, D), np.float32)
        f = 0
        for k in range(3):
            x = np.random.default_rng(100 + k).standard_normal((B, T, D)).astype(np.float32)
            y, f = orc.stream_block_step(x, bw, pe, H, ff, K, hc, cc, f, T, 28, 13, True,
                                         bf16=bf16)
        outs.append(y)
    assert np.abs(outs[0] - outs[1]).max() < 0.05 * np.abs(outs[0]).max()
