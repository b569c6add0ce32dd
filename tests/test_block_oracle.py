"""The CPU oracle of the Conformer block (oracle.block_forward,
ConformerBlock::forward, src/asr/modules/encoders/conformer.rs:1693-1870).

The reference holds no test of the block, so the oracle's block is checked
by an independent composition and by properties of the reference's design:

- in f32 it equals the same block composed from torch.nn.functional ops
  (layer_norm, linear, silu, glu, depthwise conv1d, batch_norm in eval mode)
  around the oracle's pinned attention;
- frames past an utterance's length never reach its valid frames (padded
  keys are masked, padded frames are zeroed before the depthwise conv);
- with every linear, the depthwise conv and the attention projections zero,
  the block reduces to its final LayerNorm.
"""
import numpy as np
import pytest

from conftest import rand_block


def torch_block(orc, x, bw, pe, H, ff, K, causal, conv_norm, lengths, context):
    import torch
    import torch.nn.functional as F
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))
    X = t(x)
    B, T, D = x.shape

    def ln(v, name):
        g, b = bw["norms"][name]
        return F.layer_norm(v, (D,), t(g), t(b), eps=1e-5)

    def lin(v, name):
        w, b = bw[name]
        return F.linear(v, t(w), t(b) if b is not None else None)

    valid = torch.ones(B, T, 1)
    if lengths is not None:
        valid = (torch.arange(T)[None, :, None] < torch.as_tensor(lengths)[:, None, None]).float()
    X = X + 0.5 * lin(F.silu(lin(ln(X, "ff1"), "ff1_1")), "ff1_2")
    att = orc.mha_forward(ln(X, "att").numpy(), bw["attn"], pe, H,
                          lengths=lengths, context=context)
    X = X + t(att)
    g = F.glu(lin(ln(X, "conv"), "pw1"), dim=-1) * valid
    g = g.transpose(1, 2)
    pad = (K - 1, 0) if causal else ((K - 1) // 2, (K - 1) // 2)
    dw_w, dw_b = bw["dw"]
    c = F.conv1d(F.pad(g, pad), t(dw_w)[:, None, :], t(dw_b), groups=D)
    cg, cb, cm, cv = bw["conv_norm"]
    if conv_norm == "batch_norm":
        c = F.batch_norm(c, t(cm), t(cv), t(cg), t(cb), training=False, eps=1e-5)
        c = c.transpose(1, 2)
    else:
        c = F.layer_norm(c.transpose(1, 2), (D,), t(cg), t(cb), eps=1e-5)
    X = X + lin(F.silu(c), "pw2")
    X = X + 0.5 * lin(F.silu(lin(ln(X, "ff2"), "ff2_1")), "ff2_2")
    return ln(X, "out").numpy()


def run_oracle(orc, x, bw, pe, H, ff, K, causal, conv_norm, lengths, context, bf16=False):
    return orc.block_forward(x, bw, pe, H, ff, K, causal=causal,
                             conv_norm=0 if conv_norm == "batch_norm" else 1,
                             lengths=lengths, context=context, bf16=bf16)


@pytest.mark.parametrize("causal,conv_norm,lengths,context", [
    (False, "batch_norm", [40, 27], None),
    (True, "batch_norm", None, (8, 4, False)),
    (False, "layer_norm", [40, 1], (6, 1, True)),
])
def test_block_oracle_matches_torch_composition(orc, causal, conv_norm, lengths, context):
    rng = np.random.default_rng(17)
    B, T, D, H, ff, K = 2, 40, 64, 2, 128, 9
    bw, _ = rand_block(rng, D, H, ff, K, conv_norm)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    pe = orc.get_encoding(D, 5000, T)
    ln = np.array(lengths, np.int32) if lengths is not None else None
    got = run_oracle(orc, x, bw, pe, H, ff, K, causal, conv_norm, ln, context)
    want = torch_block(orc, x, bw, pe, H, ff, K, causal, conv_norm, ln, context)
    rows = lengths or [T] * B
    for b, L in enumerate(rows):
        assert np.abs(got[b, :L] - want[b, :L]).max() < 1e-4 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("bf16", [False, True])
def test_padded_frames_do_not_reach_valid_frames(orc, bf16):
    rng = np.random.default_rng(5)
    B, T, D, H, ff, K = 2, 32, 64, 2, 128, 9
    bw, _ = rand_block(rng, D, H, ff, K)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    lengths = np.array([32, 19], np.int32)
    pe = orc.get_encoding(D, 5000, T)
    a = run_oracle(orc, x, bw, pe, H, ff, K, False, "batch_norm", lengths, None, bf16)
    x2 = x.copy()
    x2[1, 19:] = rng.standard_normal((T - 19, D)) * 100
    b = run_oracle(orc, x2, bw, pe, H, ff, K, False, "batch_norm", lengths, None, bf16)
    assert np.array_equal(a[1, :19], b[1, :19])
    assert np.array_equal(a[0], b[0])


def test_zero_parameters_reduce_to_the_final_norm(orc):
    rng = np.random.default_rng(9)
    B, T, D, H, ff, K = 1, 24, 64, 2, 128, 9
    bw, _ = rand_block(rng, D, H, ff, K)
    for name in ("ff1_1", "ff1_2", "pw1", "pw2", "ff2_1", "ff2_2"):
        w, b = bw[name]
        bw[name] = (np.zeros_like(w), np.zeros_like(b))
    bw["dw"] = (np.zeros_like(bw["dw"][0]), np.zeros_like(bw["dw"][1]))
    for k in ("wq", "wk", "wv", "wo", "wp", "bq", "bk", "bv", "bo"):
        bw["attn"][k] = np.zeros_like(bw["attn"][k])
    cg, cb, cm, cv = bw["conv_norm"]
    bw["conv_norm"] = (cg, np.zeros_like(cb), np.zeros_like(cm), cv)  # BN(0) = 0, silu(0) = 0
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    got = run_oracle(orc, x, bw, orc.get_encoding(D, 5000, T), H, ff, K, False, "batch_norm",
                     None, None)
    g, b = bw["norms"]["out"]
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    want = (x - mu) / np.sqrt(var + 1e-5) * g + b
    assert np.abs(got - want).max() < 1e-5
