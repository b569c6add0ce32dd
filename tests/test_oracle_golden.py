"""Pins the CPU oracle to the reference's own unit tests.

Each test restates one test of animaslabs/mlx-nemo-rs against the values in
tests/golden/reference_kats.json (made by tests/golden/make_reference_kats.py);
the source file:line is in each fixture's "source" field.  The reference's
MLX-RNG inputs cannot be reproduced without MLX, so the invariance tests use
seeded numpy inputs of the same shapes and scales.
"""
import json
import math
import os

import numpy as np
import pytest

from conftest import rand_weights

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                   "reference_kats.json")))


def test_rel_shift_correctness(orc):
    k = KATS["rel_shift_correctness"]
    x = np.array(k["input"], np.float32).reshape(k["input_shape"])
    out = orc.rel_shift(x)
    assert out.shape == tuple(k["input_shape"])
    got = out[0, 0, :, :3]
    assert np.array_equal(got, np.array(k["expected_first3"], np.float32))


def test_rel_shift_shape(orc):
    k = KATS["rel_shift_shape"]
    assert orc.rel_shift(np.ones(k["input_shape"], np.float32)).shape == \
        tuple(k["expected_shape"])


def _verify_rel_shift(orc, seq_len, pos_len, num_keys):
    x = np.arange(seq_len * pos_len, dtype=np.float32).reshape(1, 1, seq_len, pos_len)
    out = orc.rel_shift(x)[0, 0]
    for i in range(seq_len):
        for j in range(num_keys):
            col = seq_len - 1 - i + j
            assert out[i, j] == i * pos_len + col, (seq_len, pos_len, i, j)


def test_rel_shift_property_standard(orc):
    for s in KATS["rel_shift_property_standard"]["seq_lens"]:
        _verify_rel_shift(orc, s, 2 * s - 1, s)


def test_rel_shift_property_streaming(orc):
    k = KATS["rel_shift_property_streaming"]
    for s in k["seq_lens"]:
        for c in k["cache_lens"]:
            total = s + c
            _verify_rel_shift(orc, s, 2 * total - 1, total)


def test_rel_shift_no_padding_zeros(orc):
    k = KATS["rel_shift_no_padding_zeros"]
    s, t = k["seq_len"], k["total_len"]
    p = 2 * t - 1
    x = (k["min_value"] + np.arange(s * p, dtype=np.float32)).reshape(1, 1, s, p)
    out = orc.rel_shift(x)[0, 0]
    assert (out[:, :t] >= k["min_value"]).all()


def test_pe_values(orc):
    k = KATS["pe_values"]
    enc = orc.get_encoding(k["d_model"], k["max_len"], k["seq_len"])
    assert (1,) + enc.shape == tuple(k["expected_shape"])
    assert np.abs(enc[0] - np.array(k["row0"], np.float32)).max() < k["tol"]
    assert np.abs(enc[2, :2] - np.array(k["row2_first2"], np.float32)).max() < k["tol"]


def test_pe_shape_and_streaming_dims(orc):
    k = KATS["pe_shape"]
    enc = orc.get_encoding(k["d_model"], k["max_len"], k["seq_len"])
    assert (1,) + enc.shape == tuple(k["expected_shape"])
    k = KATS["pe_streaming_dimensions"]
    enc = orc.get_encoding(k["d_model"], k["max_len"], k["cache"] + k["seq_len"])
    assert (1,) + enc.shape == tuple(k["expected_shape"])


def test_pe_extends_past_max_len(orc):
    k = KATS["pe_extends_past_max_len"]
    ext = orc.get_encoding(k["d_model"], k["short_max_len"], k["seq_len"])
    ref = orc.get_encoding(k["d_model"], k["long_max_len"], k["seq_len"])
    assert (1,) + ext.shape == tuple(k["expected_shape"])
    assert np.abs(ext - ref).max() < k["tol"]


def test_pe_empty_sequence_is_an_error(orc):
    with pytest.raises(ValueError):
        orc.get_encoding(16, 10, 0)


def test_context_mask_matches_nemo(orc):
    k = KATS["context_mask_matches_nemo"]

    def nemo(size, style, i, j):  # brute-force _create_masks, attention.rs:1109-1119
        left, right = size
        if style == "chunked_limited" and right >= 0:
            chunk = right + 1
            lc = left // chunk if left >= 0 else 10000
            diff = i // chunk - j // chunk
            return 0 <= diff <= lc
        right_ok = style == "chunked_limited" or right < 0 or j - i <= right
        return (left < 0 or j - i >= -left) and right_ok

    for size, style in k["cases"]:
        m = orc.block_mask(size[0], size[1], style == "chunked_limited",
                           k["start"], k["end"], k["seq_len"])
        assert m.shape == (k["end"] - k["start"], k["seq_len"])
        for i in range(k["start"], k["end"]):
            for j in range(k["seq_len"]):
                assert m[i - k["start"], j] == nemo(size, style, i, j), (size, style, i, j)


def test_query_block_size(orc):
    k = KATS["blocked_attention_matches_full"]
    b = orc.query_block_size(2 * 2, k["seq_len"], k["budget"])
    blocks = [min(b, k["seq_len"] - s) for s in range(0, k["seq_len"], b)]
    assert blocks == k["expected_blocks"]
    # the reference's clamp (attention.rs:202-206) at BASELINE config 1
    assert orc.query_block_size(16 * 8, 750, 1 << 26) == 349


def test_standard_linear_forward(orc):
    k = KATS["standard_linear_forward"]
    y = orc.linear(np.array(k["x"]), np.array(k["weight"]), np.array(k["bias"]))
    assert np.abs(y - np.array(k["expected"])).max() < k["tol"]


def test_dequantize_roundtrip(orc):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    wq, s, b = orc.quantize(w, 64, 8)
    assert wq.shape == (64, 64) and s.shape == (64, 4)
    wd = orc.dequantize(wq, s, b, 64, 8)
    # affine 8-bit: error at most half a step per group
    step = np.repeat(s, 64, axis=1)
    assert (np.abs(wd - w) <= 0.5 * step + 1e-7).all()
    # packing is lowest byte first (MLX layout, quantization.rs:4-8)
    q0 = int(np.rint((w[0, 0] - b[0, 0]) / s[0, 0]))
    assert int(wq[0, 0] & 0xFF) == q0


def _rand_attn_inputs(seed, d, h, t, scale):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, d, h, scale=scale, out_bias=False)
    x = rng.standard_normal((2, t, d)).astype(np.float32)
    return w, x


def test_padded_keys_are_ignored(orc):
    k = KATS["padded_keys_are_ignored"]
    d, h, t, valid = k["d_model"], k["n_heads"], k["seq_len"], k["valid"]
    w, x = _rand_attn_inputs(12, d, h, t, k["weight_scale"])
    x[1, valid:] = k["garbage"]
    for ctxd in k["contexts"]:
        ctx = None if ctxd is None else (ctxd[0][0], ctxd[0][1], ctxd[1] == "chunked_limited")
        for mode in (orc.ORC_DIRECT, orc.ORC_REFERENCE_ALGO):
            pe = orc.get_encoding(d, 64, t)
            masked = orc.mha_forward(x, w, pe, h, lengths=[t, valid], context=ctx, mode=mode)
            full = orc.mha_forward(x[:1], w, pe, h, context=ctx, mode=mode)
            short = orc.mha_forward(x[1:2, :valid], w, orc.get_encoding(d, 64, valid), h,
                                    context=ctx, mode=mode)
            assert np.abs(masked[:1] - full).max() < k["tol_full"]
            assert np.abs(masked[1:2, :valid] - short).max() < k["tol_short"]


def test_blocked_attention_matches_full(orc):
    k = KATS["blocked_attention_matches_full"]
    d, h, t = k["d_model"], k["n_heads"], k["seq_len"]
    w, x = _rand_attn_inputs(11, d, h, t, k["weight_scale"])
    pe = orc.get_encoding(d, 64, t)
    for ctxd in k["contexts"]:
        ctx = None if ctxd is None else (ctxd[0][0], ctxd[0][1], ctxd[1] == "chunked_limited")
        full = orc.mha_forward(x, w, pe, h, context=ctx, mode=orc.ORC_REFERENCE_ALGO,
                               max_score_elements=2 ** 62)
        blocked = orc.mha_forward(x, w, pe, h, context=ctx, mode=orc.ORC_REFERENCE_ALGO,
                                  max_score_elements=k["budget"])
        direct = orc.mha_forward(x, w, pe, h, context=ctx, mode=orc.ORC_DIRECT)
        assert np.abs(full - blocked).max() < k["tol"]
        # the direct (index-arithmetic) form equals the reference algorithm
        assert np.abs(full - direct).max() < k["tol"]


def test_streaming_mask_rules(orc):
    # chunked_limited [70,13] at cache 70, chunk 14
    m = orc.create_attention_mask(70, 13, True, 84, 70, 70, 14, 14)
    assert m.all()  # once the cache is full every key is visible -> no mask
    m = orc.create_attention_mask(70, 13, True, 84, 70, 14, 14, 14)
    assert not m[:, :56].any() and m[:, 56:].all()  # unfilled prefix hidden
    m = orc.create_attention_mask(70, 13, True, 84, 70, 70, 14, 10)
    assert not m[10:].any()  # rows past the valid length see nothing


def test_stream_step_cache_semantics(orc):
    """forward_with_cache's sliding window (attention.rs:661-684) and the
    encoder's fill update (conformer.rs:1027-1037), checked on the oracle
    against its own offline attention over concat(cache, x)."""
    rng = np.random.default_rng(5)
    d, h, C, T = 32, 2, 6, 3
    w = rand_weights(rng, d, h, scale=0.2)
    cache = np.zeros((2, C, d), np.float32)
    filled = 0
    hist = []
    for step in range(4):
        x = rng.standard_normal((2, T, d)).astype(np.float32)
        pe = orc.get_encoding(d, 5000, C + T)
        before = cache.copy()
        out, nxt = orc.stream_layer_step(x, w, pe, h, cache, filled, T, -1, -1, False)
        assert nxt == min(filled + T, C)
        # the cache holds the newest frames, zero-padded in front
        hist.append(x)
        allf = np.concatenate(hist, axis=1)[:, -C:]
        n = allf.shape[1]
        assert np.array_equal(cache[:, C - n:], allf)
        assert not cache[:, :C - n].any()
        # keys are concat(cache, x); the unfilled prefix is hidden by the mask
        kv = np.concatenate([before, x], axis=1)
        vis = orc.create_attention_mask(-1, -1, False, C + T, C, filled, T, T)
        q = orc.linear(x, w["wq"], w["bq"])
        k = orc.linear(kv, w["wk"], w["bk"])
        v = orc.linear(kv, w["wv"], w["bv"])
        p = orc.linear(pe, w["wp"])
        ctx = orc.relpos_attention(q, k, v, p, w["pos_bias_u"], w["pos_bias_v"], h, vis=vis)
        ref = orc.linear(ctx, w["wo"], w["bo"])
        assert np.abs(out - ref).max() < 1e-5
        filled = nxt
