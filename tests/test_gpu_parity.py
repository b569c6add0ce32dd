"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances: f32 modules 1e-4, bf16 modules 2e-2, as
max-abs error relative to the output's scale: rel = max|got - ref| /
max|ref| over the valid query rows (padded rows are unspecified in the reference,
src/asr/modules/encoders/conformer.rs:1590-1593), and per element
|got - ref| <= tol * (|ref| + 4 * rms(ref)), so that a wrong small element
cannot hide behind the largest one.  The bf16 oracle rounds to bf16 where the
reference's bf16 graph does -- among them the positional scores bd * scale
before the softmax (attention.rs:530-556), which the device keeps in f32.
That rounding moves a whole row's probabilities, so its effect on an output
element scales with the row's magnitude, not the element's: the 4 * rms(ref)
term (0.08 rms at tol 2e-2).
"""
import numpy as np
import pytest

from conftest import rand_weights
from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-4
TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def weight_dict(w, prefix="l"):
    m = {"linear_q": ("wq", "bq"), "linear_k": ("wk", "bk"), "linear_v": ("wv", "bv"),
         "linear_out": ("wo", "bo"), "linear_pos": ("wp", None)}
    d = {}
    for name, (wk, bk) in m.items():
        d[f"{prefix}.{name}.weight"] = w[wk]
        if bk and w.get(bk) is not None:
            d[f"{prefix}.{name}.bias"] = w[bk]
    d[f"{prefix}.pos_bias_u"] = w["pos_bias_u"]
    d[f"{prefix}.pos_bias_v"] = w["pos_bias_v"]
    return d


def rel_err(got, ref, lengths=None):
    """(max abs err, max abs err / max |ref|) over valid rows."""
    if lengths is None:
        lengths = [got.shape[1]] * got.shape[0]
    g = np.concatenate([got[b, :L].ravel() for b, L in enumerate(lengths)])
    r = np.concatenate([ref[b, :L].ravel() for b, L in enumerate(lengths)])
    a = float(np.abs(g - r).max())
    return a, a / max(float(np.abs(r).max()), 1e-12)


def check_close(got, ref, lengths, tol):
    """Asserts both bounds of the module docstring over the valid rows
    (lengths None: all rows) and returns (max abs err, max-normalised err,
    worst per-element ratio)."""
    if lengths is None:
        lengths = [got.shape[1]] * got.shape[0]
    g = np.concatenate([got[b, :L].ravel() for b, L in enumerate(lengths)]).astype(np.float64)
    r = np.concatenate([ref[b, :L].ravel() for b, L in enumerate(lengths)]).astype(np.float64)
    d = np.abs(g - r)
    a = float(d.max())
    rel = a / max(float(np.abs(r).max()), 1e-12)
    rms = float(np.sqrt(np.mean(r * r)))
    worst = float((d / (tol * (4.0 * rms + np.abs(r)) + 1e-30)).max())
    assert rel < tol and worst <= 1.0, (a, rel, worst)
    return a, rel, worst


def make_module(nrp, w, D, H, dtype, use_bias=True):
    attn = nrp.RelPositionMultiHeadAttention(D, H, use_bias)
    attn.load_weights(weight_dict(w), "l")
    attn.set_dtype(dtype)
    return attn


def run_forward(nrp, attn, x, T, lengths, context, dtype):
    import torch
    pe = nrp.RelPositionalEncoding(x.shape[2], 5000, False)
    pe.set_dtype(dtype)
    tdt = torch.bfloat16 if dtype == nrp.BF16 else torch.float32
    xd = torch.from_numpy(x).to("cuda", tdt)
    mask = nrp.key_padding_mask(lengths, T) if lengths is not None else None
    ctx = nrp.AttentionContext.new(context[:2], "chunked_limited" if context[2] else "regular") \
        if context is not None else None
    out = attn.forward(xd, pe.get_encoding(T), ctx, mask)
    attn.ctx.check()
    return out.float().cpu().numpy(), pe.get_encoding_host(T)[0]


# ---------------------------------------------------------------- linears
# (896, 1024, 3072) and (1000, 1024, 3072) take the 192-wide tiles (128-wide
# ones would overflow one wave of 148 SMs)
@pytest.mark.parametrize("M,K,N", [(300, 1024, 3072), (1499, 1024, 1024), (7, 512, 256),
                                   (128, 64, 32), (896, 1024, 3072), (1000, 1024, 3072)])
def test_linear_bf16_tcgen05(nrp, orc, M, K, N):
    import torch
    rng = np.random.default_rng(M + N)
    x = orc.bf16_round(rng.standard_normal((M, K)))
    w = orc.bf16_round(rng.standard_normal((N, K)) * 0.02)
    b = orc.bf16_round(rng.standard_normal(N) * 0.02)
    dev = lambda a: torch.from_numpy(a).to("cuda", torch.bfloat16)
    y = nrp.linear(dev(x), dev(w), dev(b)).float().cpu().numpy()
    ref = orc.linear(x, w, b)
    check_close(y[None], ref[None], None, 1e-2)  # bf16 output rounding only


def test_linear_f32(nrp, orc):
    import torch
    rng = np.random.default_rng(1)
    x = rng.standard_normal((249, 1024)).astype(np.float32)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(1024) * 0.02).astype(np.float32)
    y = nrp.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                   torch.from_numpy(b).cuda()).cpu().numpy()
    a, _, _ = check_close(y[None], orc.linear(x, w, b)[None], None, TOL_F32)
    assert a < TOL_F32


@pytest.mark.parametrize("M", [1, 14, 16, 17, 33, 64, 65, 128, 200, 255, 256, 257, 300, 896, 2500])
@pytest.mark.parametrize("K,N", [(1024, 1024), (1024, 4096), (4096, 1024)])
def test_qlinear_mlx_affine_8bit(nrp, orc, M, K, N):
    """Up to 256 rows: the small-M kernel (codes dequantised in registers
    into bf16 MMA fragments; 1, 14, 16, 17, 64: one 64-row chunk with 1, 2
    or 4 m tiles, full and ragged; 128, 200, 255, 256: two to four chunks);
    from 257 rows: the weight dequantised once per call (caller-owned
    weights are never kept), then the bf16 tcgen05 GEMM."""
    import torch
    rng = np.random.default_rng(M * 7 + N)
    wm = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    wq, s, z = orc.quantize(wm, 64, 8)
    s, z = orc.bf16_round(s), orc.bf16_round(z)   # LinearLayer::cast to bf16
    x = orc.bf16_round(rng.standard_normal((M, K)))
    bias = orc.bf16_round(rng.standard_normal(N) * 0.02)
    dev = lambda a: torch.from_numpy(a).to("cuda", torch.bfloat16)
    y = nrp.qlinear(dev(x), torch.from_numpy(wq.view(np.int32)).cuda(), dev(s), dev(z),
                    dev(bias)).float().cpu().numpy()
    ref = orc.linear(x, orc.dequantize(wq, s, z, 64, 8), bias)
    check_close(y[None], ref[None], None, 1e-2)


# ------------------------------------------------------- offline, f32
@pytest.mark.parametrize("context", [None, (3, 2, False), (4, 1, True), (-1, 2, True),
                                     (4, -1, True)])
def test_f32_reference_test_shapes(nrp, orc, context):
    """attention.rs:1026-1104 shapes (d_model 16, 2 heads, T 13, a row
    padded to 9) at f32 parity."""
    rng = np.random.default_rng(12)
    D, H, T = 16, 2, 13
    w = rand_weights(rng, D, H, scale=0.3)
    x = rng.standard_normal((2, T, D)).astype(np.float32)
    x[1, 9:] = 50.0
    lengths = np.array([T, 9], np.int32)
    attn = make_module(nrp, w, D, H, nrp.F32)
    got, pe = run_forward(nrp, attn, x, T, lengths, context, nrp.F32)
    ref = orc.mha_forward(x, w, pe, H, lengths=lengths, context=context,
                          mode=orc.ORC_REFERENCE_ALGO)
    check_close(got, ref, lengths, TOL_F32)


def test_f32_config0(nrp, orc):
    """[1,125,1024] f32, 8 heads, no mask."""
    rng = np.random.default_rng(0)
    D, H, T = 1024, 8, 125
    w = rand_weights(rng, D, H)
    x = rng.standard_normal((1, T, D)).astype(np.float32)
    attn = make_module(nrp, w, D, H, nrp.F32)
    got, pe = run_forward(nrp, attn, x, T, None, None, nrp.F32)
    ref = orc.mha_forward(x, w, pe, H, mode=orc.ORC_REFERENCE_ALGO)
    a, _, _ = check_close(got, ref, None, TOL_F32)
    assert a < TOL_F32  # outputs are O(0.1): the absolute bound holds too


# ------------------------------------------------------ offline, bf16
@pytest.mark.parametrize("B,T,lengths,context", [
    (1, 13, None, None),
    (2, 128, None, None),
    (2, 129, [129, 60], None),
    (2, 300, [300, 1], None),
    (3, 750, [750, 375, 500], None),
    (2, 400, None, (128, 128, False)),
    (2, 300, [300, 200], (4, 1, True)),
    (1, 520, None, (70, 13, True)),
    (1, 260, None, (-1, 0, False)),
    (1, 260, None, (16, -1, True)),
])
def test_bf16_offline(nrp, orc, B, T, lengths, context):
    rng = np.random.default_rng(B * 1000 + T)
    D, H = 256, 2
    w = rand_weights(rng, D, H)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    ln = np.array(lengths, np.int32) if lengths is not None else None
    attn = make_module(nrp, w, D, H, nrp.BF16)
    got, pe = run_forward(nrp, attn, x, T, ln, context, nrp.BF16)
    assert np.isfinite(got).all()
    ref = orc.mha_forward(x, w, pe, H, lengths=ln, context=context, bf16=True)
    check_close(got, ref, ln, TOL_BF16)


def test_bf16_config1_shape(nrp, orc):
    """BASELINE config 1 layer: [16,750,1024] bf16, lengths U[375,750]; the
    oracle checks all 16 utterances."""
    rng = np.random.default_rng(1)
    B, T, D, H = 16, 750, 1024, 8
    w = rand_weights(rng, D, H)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    ln = rng.integers(375, 751, B).astype(np.int32)
    attn = make_module(nrp, w, D, H, nrp.BF16)
    got, pe = run_forward(nrp, attn, x, T, ln, None, nrp.BF16)
    assert np.isfinite(got).all()
    ref = orc.mha_forward(x, w, pe, H, lengths=ln, bf16=True)
    check_close(got, ref, ln, TOL_BF16)


def test_bf16_quantized_projections(nrp, orc):
    """All five projections MLX 8-bit (group 64) quantised, bf16 module."""
    rng = np.random.default_rng(3)
    B, T, D, H = 2, 300, 1024, 8
    w = rand_weights(rng, D, H)
    wd = weight_dict(w)
    deq = dict(w)
    for name, key in (("linear_q", "wq"), ("linear_k", "wk"), ("linear_v", "wv"),
                      ("linear_out", "wo"), ("linear_pos", "wp")):
        wq, s, z = orc.quantize(w[key], 64, 8)
        wd[f"l.{name}.weight"] = wq
        wd[f"l.{name}.scales"] = s
        wd[f"l.{name}.biases"] = z
        deq[key] = orc.dequantize(wq, orc.bf16_round(s), orc.bf16_round(z), 64, 8)
    attn = nrp.RelPositionMultiHeadAttention(D, H, True)
    attn.load_weights(wd, "l", nrp.QuantizationConfig(8, 64))
    attn.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    ln = np.array([300, 211], np.int32)
    got, pe = run_forward(nrp, attn, x, T, ln, None, nrp.BF16)
    ref = orc.mha_forward(x, deq, pe, H, lengths=ln, bf16=True)
    check_close(got, ref, ln, TOL_BF16)


# ---------------------------------------------------------- streaming
@pytest.mark.parametrize("dtype_name,D,H,C,T,ctx,drop", [
    ("f32", 16, 2, 6, 3, None, 0),
    ("f32", 256, 2, 10, 4, (10, 3, True), 0),
    ("f32", 64, 2, 8, 5, (6, 1, False), 2),
    ("bf16", 256, 2, 70, 14, (70, 13, True), 0),
    ("bf16", 1024, 8, 70, 14, (70, 13, True), 0),
    ("bf16", 256, 2, 40, 20, (40, 3, False), 3),
    ("bf16", 256, 2, 100, 12, None, 2),
    ("bf16", 256, 2, 240, 16, None, 0),
    ("bf16", 256, 2, 200, 33, (200, 10, False), 0),
    ("bf16", 256, 2, 1, 1, None, 0),
    ("bf16", 256, 2, 16, 16, (16, 15, True), 0),
])
def test_streaming_chunks(nrp, orc, dtype_name, D, H, C, T, ctx, drop):
    """forward_with_cache over consecutive chunks (attention.rs:606-816,
    conformer.rs:883-1037): outputs and the exported attention-input cache
    against the oracle's streaming step, including the warm-up where the
    unfilled cache prefix is masked and a last chunk with valid < T."""
    import torch
    dtype = nrp.F32 if dtype_name == "f32" else nrp.BF16
    bf = dtype == nrp.BF16
    tol = TOL_BF16 if bf else TOL_F32
    rng = np.random.default_rng(D + C)
    B = 3
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
    for step in range(8):
        x = rng.standard_normal((B, T, D)).astype(np.float32)
        if bf:
            x = orc.bf16_round(x)
        valid = T if step < 7 else max(T - 2, 0)
        out = attn.forward_with_cache(torch.from_numpy(x).to("cuda", tdt), pos, cache, filled,
                                      valid, context)
        attn.ctx.check()
        got = out.float().cpu().numpy()
        l, r = (ctx[0], ctx[1]) if ctx else (-1, -1)
        ref, nxt = orc.stream_layer_step(x, w, pos_h, H, h_ref, filled, valid, l, r,
                                         bool(ctx and ctx[2]), drop, bf16=bf)
        if valid > 0:
            check_close(got, ref, [valid] * B, tol)
        if valid < T:
            # rows that see no key have a zero context, so linear_out leaves
            # exactly its bias there (attention.rs:786-789, 807)
            bo = orc.bf16_round(w["bo"]) if bf else w["bo"]
            assert np.abs(got[:, valid:] - bo).max() <= (1e-2 if bf else 1e-6)
        hc = cache.export_h().cpu().numpy()
        assert np.abs(hc - h_ref).max() <= (0 if not bf else 1e-6), step
        filled = nxt


def test_cache_import_roundtrip(nrp, orc):
    """Importing an exported cache and continuing equals not interrupting."""
    import torch
    rng = np.random.default_rng(9)
    D, H, C, T, B = 256, 2, 12, 4, 2
    w = rand_weights(rng, D, H)
    a1 = make_module(nrp, w, D, H, nrp.BF16)
    a2 = make_module(nrp, w, D, H, nrp.BF16)
    c1 = nrp.AttentionCache(a1, B, C)
    c2 = nrp.AttentionCache(a2, B, C)
    pe = nrp.RelPositionalEncoding(D, 5000, False)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(C + T)
    xs = [torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).cuda().bfloat16()
          for _ in range(5)]
    filled = 0
    for x in xs[:3]:
        a1.forward_with_cache(x, pos, c1, filled)
        filled = min(filled + T, C)
    c2.import_h(c1.export_h())
    o1 = a1.forward_with_cache(xs[3], pos, c1, filled).float()
    o2 = a2.forward_with_cache(xs[3], pos, c2, filled).float()
    a1.ctx.check()
    assert torch.allclose(o1, o2, atol=2e-2, rtol=0)
    assert torch.equal(c1.export_h(), c2.export_h())
