"""Device parity of the streaming Conformer block (nrp_block_forward_with_cache:
ConformerBlock::forward_with_cache with ConvolutionModule::forward_with_cache,
src/asr/modules/encoders/conformer.rs:1877-1967, 2332-2400) against the CPU
oracle (oracle.stream_block_step, pinned to the offline block in
tests/test_stream_block_oracle.py), chunk by chunk through the cache's
warm-up and full cycles, a short last chunk (valid < T) included.  Outputs,
the conv cache and the attention's h cache are compared after every chunk.
bf16 tolerance 2e-2 of the output scale."""
import numpy as np
import pytest

from conftest import rand_block
from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def rel(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6))


@pytest.mark.parametrize("B,T,C,D,H,ff,K,conv_norm,quant,ctx,chunks", [
    (3, 14, 28, 256, 2, 1024, 9, "batch_norm", False, (28, 13, True), 6),
    (2, 14, 70, 512, 4, 1024, 9, "layer_norm", True, (70, 13, True), 7),
    (2, 8, 16, 256, 2, 768, 5, "batch_norm", True, None, 5),
])
def test_stream_block_matches_oracle(nrp, orc, B, T, C, D, H, ff, K, conv_norm, quant, ctx,
                                     chunks):
    import torch
    rng = np.random.default_rng(B * 10 + T + K)
    bw, wd = rand_block(rng, D, H, ff, K, conv_norm, quant=quant, orc=orc)
    blk = nrp.ConformerBlock(D, H, ff, K, True, conv_norm)
    blk.load_weights(wd, "b", nrp.QuantizationConfig(8, 64) if quant else None)
    blk.set_dtype(nrp.BF16)
    cache = nrp.AttentionCache(blk.self_attn, B, C)
    conv_cache = blk.new_conv_cache(B)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(C + T)
    pos_h = pe.get_encoding_host(C + T)[0]
    actx = nrp.AttentionContext.new(ctx[:2], "chunked_limited" if ctx[2] else "regular") \
        if ctx is not None else None
    left, right, chunked = ctx if ctx is not None else (-1, -1, False)
    hc = np.zeros((B, C, D), np.float32)
    cc = np.zeros((B, K - 1, D), np.float32)
    filled = 0
    cn = 0 if conv_norm == "batch_norm" else 1
    for k in range(chunks):
        valid = T if k < chunks - 1 else T - 5
        x = orc.bf16_round(rng.standard_normal((B, T, D)).astype(np.float32))
        xd = torch.from_numpy(x).cuda().bfloat16()
        got = blk.forward_with_cache(xd, pos, cache, conv_cache, filled, valid, actx)
        blk.ctx.check()
        ref, nxt = orc.stream_block_step(x, bw, pos_h, H, ff, K, hc, cc, filled, valid, left,
                                         right, chunked, conv_norm=cn, bf16=True)
        g = got.float().cpu().numpy()
        assert np.isfinite(g).all()
        err = rel(g[:, :valid], ref[:, :valid])
        assert err < TOL_BF16, (k, err)
        cerr = rel(conv_cache.float().cpu().numpy(), cc) if np.abs(cc).max() > 0 else \
            float(np.abs(conv_cache.float().cpu().numpy()).max())
        assert cerr < TOL_BF16, (k, cerr)
        herr = rel(cache.export_h().cpu().numpy(), hc)
        assert herr < TOL_BF16, (k, herr)
        filled = nxt


def test_stream_block_in_place_and_repeat(nrp, orc):
    """out == x in place gives the same bits as out-of-place, and the same
    chunk sequence from reset caches repeats bit for bit."""
    import torch
    rng = np.random.default_rng(4)
    B, T, C, D, H, ff, K = 2, 14, 28, 256, 2, 1024, 9
    _, wd = rand_block(rng, D, H, ff, K)
    blk = nrp.ConformerBlock(D, H, ff, K, True)
    blk.load_weights(wd, "b")
    blk.set_dtype(nrp.BF16)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(C + T)
    xs = [torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).cuda().bfloat16()
          for _ in range(4)]

    def run(in_place):
        cache = nrp.AttentionCache(blk.self_attn, B, C)
        cc = blk.new_conv_cache(B)
        outs, f = [], 0
        for x in xs:
            if in_place:
                y = x.clone()
                blk.forward_with_cache(y, pos, cache, cc, f, T, out=y)
            else:
                y = blk.forward_with_cache(x, pos, cache, cc, f, T)
            outs.append(y)
            f = min(f + T, C)
        return outs, cc

    a, ca = run(False)
    b, cb = run(True)
    c, cc_ = run(False)
    blk.ctx.check()
    for u, v, w in zip(a, b, c):
        assert torch.equal(u, v) and torch.equal(u, w)
    assert torch.equal(ca, cb) and torch.equal(ca, cc_)
