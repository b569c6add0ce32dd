"""The CPU oracle of the dw_striding subsampling (oracle.subsampling_forward,
Subsampling::forward_frames, src/asr/modules/encoders/conformer.rs:1413-1555).

The reference's own test of this module (conformer.rs:2446-2488,
test_chunked_subsampling_matches_single_pass) runs the conv stack over time
chunks of 40 frames with its chunking rule (1345-1377) and requires the
single-pass result, for both padding styles, on a [1, 203, 16] input with 4
channels and d_model 8.  That property is restated here on the oracle, which
pins the oracle's padding, stride alignment and receptive field.  Beside it:

- in f32 the oracle equals the same stack composed from torch.nn.functional
  (conv2d with padding 1, or F.pad (2, 1) on both axes for the causal form;
  groups = C for the depthwise convs; NeMo's [B, C, T, F] -> [B, T, C*F]
  flattening) for subsampling factors 2, 4 and 8;
- the frequency and length formulas give the reference's documented values
  (compute_freq_output_size's doc, 1206-1219: 128 -> 65 -> 33 -> 17 causal).
"""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def orc():
    from oracle import oracle
    return oracle


def rand_sub(rng, C, F, d_model, factor, causal, bias=True, scale=0.3):
    from oracle import oracle
    S = oracle.subsampling_strides(factor)
    Fp = oracle.subsampling_feat_out(F, factor, causal)
    f = lambda *sh: (rng.standard_normal(sh) * scale).astype(np.float32)
    b = (lambda n: f(n)) if bias else (lambda n: None)
    return {
        "conv0": (f(C, 3, 3, 1), b(C)),
        "dw": [(f(C, 3, 3, 1), b(C)) for _ in range(S - 1)],
        "pw": [(f(C, 1, 1, C) / np.sqrt(C), b(C)) for _ in range(S - 1)],
        "out": (f(d_model, C * Fp) / np.sqrt(C * Fp), b(d_model)),
    }


def torch_sub(x, sw, factor, causal):
    import torch
    import torch.nn.functional as F
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))
    ob = lambda a: t(a) if a is not None else None
    conv_w = lambda w: t(w).permute(0, 3, 1, 2).contiguous()  # MLX [O,kH,kW,I] -> [O,I,kH,kW]
    X = t(x)[:, None]  # [B, 1, T, F]
    C = sw["conv0"][0].shape[0]

    def conv(v, w, b, groups):
        if causal:
            return F.conv2d(F.pad(v, (2, 1, 2, 1)), conv_w(w), ob(b), stride=2, groups=groups)
        return F.conv2d(v, conv_w(w), ob(b), stride=2, padding=1, groups=groups)

    X = F.relu(conv(X, *sw["conv0"], 1))
    for (dw, db), (pw, pb) in zip(sw["dw"], sw["pw"]):
        X = conv(X, dw, db, C)
        X = F.relu(F.conv2d(X, conv_w(pw), ob(pb)))
    B, _, Tp, Fp = X.shape
    X = X.permute(0, 2, 1, 3).reshape(B, Tp, C * Fp)
    w, b = sw["out"]
    return F.linear(X, t(w), ob(b)).numpy()


@pytest.mark.parametrize("factor", [2, 4, 8])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,T,F,C,D", [(2, 57, 80, 16, 24), (1, 203, 16, 4, 8), (1, 1, 9, 4, 8)])
def test_oracle_equals_torch_composition(orc, factor, causal, B, T, F, C, D):
    rng = np.random.default_rng(factor * 7 + causal + T)
    sw = rand_sub(rng, C, F, D, factor, causal)
    x = rng.standard_normal((B, T, F)).astype(np.float32)
    got = orc.subsampling_forward(x, sw, D, factor, causal, bf16=False)
    want = torch_sub(x, sw, factor, causal)
    assert got.shape == want.shape == (B, orc.subsampling_out_len(T, factor, causal), D)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_sizes_match_reference_formulas(orc):
    # compute_freq_output_size's doc: 128 mel bins, 3 causal stages
    assert orc.subsampling_feat_out(128, 8, True) == 17
    assert orc.subsampling_feat_out(128, 8, False) == 16
    assert orc.subsampling_feat_out(80, 8, False) == 10
    assert orc.subsampling_feat_out(80, 8, True) == 11
    assert orc.subsampling_strides(2) == 1 and orc.subsampling_strides(4) == 2
    assert orc.subsampling_strides(8) == 3 and orc.subsampling_strides(16) == 2
    # output_length: non-causal floor((len-1)/2)+1 per stage (0 stays 0);
    # causal floor(len/2)+1 per stage
    for n in range(0, 70):
        a, c = n, n
        for _ in range(3):
            a = (a - 1) // 2 + 1
            c = c // 2 + 1
        assert orc.subsampling_out_len(n, 8, False) == max(a, 0)
        assert orc.subsampling_out_len(n, 8, True) == c
    assert orc.subsampling_out_len(4000, 8, False) == 500


def chunked(orc, x, sw, d_model, factor, causal, chunk_frames):
    """forward_frames_chunked (conformer.rs:1345-1377) over the oracle."""
    total = x.shape[1]
    chunk = max(chunk_frames, factor) // factor * factor
    if total <= chunk:
        return orc.subsampling_forward(x, sw, d_model, factor, causal, bf16=False)
    rf = 1 + (3 - 1) * (factor - 1)
    context = -(-(2 * rf) // factor) * factor
    outs, start = [], 0
    while start < total:
        end = min(start + chunk, total)
        left, right = min(context, start), min(context, total - end)
        out = orc.subsampling_forward(x[:, start - left:end + right], sw, d_model, factor,
                                      causal, bf16=False)
        first = left // factor
        outs.append(out[:, first:] if end == total
                    else out[:, first:first + (end - start) // factor])
        start = end
    return np.concatenate(outs, axis=1)


@pytest.mark.parametrize("causal", [False, True])
def test_chunked_matches_single_pass(orc, causal):
    """The reference's test_chunked_subsampling_matches_single_pass."""
    rng = np.random.default_rng(3)
    sw = rand_sub(rng, 4, 16, 8, 8, causal, scale=0.5)
    sw["out"] = (sw["out"][0], None)
    x = rng.standard_normal((1, 203, 16)).astype(np.float32)
    single = orc.subsampling_forward(x, sw, 8, 8, causal, bf16=False)
    got = chunked(orc, x, sw, 8, 8, causal, 40)
    assert got.shape == single.shape
    assert np.abs(single).max() > 1e-3
    assert np.abs(got - single).max() < 1e-5


def test_bf16_close_to_f32(orc):
    rng = np.random.default_rng(11)
    sw = rand_sub(rng, 32, 80, 64, 8, False)
    x = rng.standard_normal((2, 64, 80)).astype(np.float32)
    a = orc.subsampling_forward(x, sw, 64, 8, False, bf16=False)
    b = orc.subsampling_forward(x, sw, 64, 8, False, bf16=True)
    assert np.abs(a - b).max() < 0.05 * np.abs(a).max()
