"""Device parity of ConformerEncoder::forward_streaming
(nrp_encoder_forward_streaming, src/asr/modules/encoders/conformer.rs:840-1047)
against the CPU oracle's composition: the subsampling of each mel chunk (no
mel mask), the pre-encoded frames dropped, x * sqrt(d_model), every layer's
streaming block step (oracle.stream_block_step) with the fill level and
valid length of the first stream, chunk after chunk through the caches'
warm-up.  Also: the fill level, the output lengths, the caches in the
reference's EncoderCache layout, and a reset stream repeating bit for bit.
bf16 tolerance 2e-2 of the output scale."""
import numpy as np
import pytest

from conftest import rand_block
from test_gpu_subsampling import sub_weights
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


def build(nrp, orc, rng, L, D, H, ff, K, F, quant):
    enc = nrp.ConformerEncoder(L, D, H, ff, K, causal_conv=True, feat_in=F, subsampling_factor=8,
                               subsampling_conv_channels=256, causal_downsampling=True)
    sw, wd = sub_weights(orc, rng, 256, F, D, 8, True, quant)
    bws = []
    for i in range(L):
        bw, w = rand_block(rng, D, H, ff, K, quant=quant, orc=orc, prefix=f"encoder.layers.{i}")
        bws.append(bw)
        wd.update(w)
    enc.load_weights(wd, nrp.QuantizationConfig(8, 64) if quant else None)
    enc.set_dtype(nrp.BF16)
    return enc, sw, bws


def test_stream_encoder_matches_oracle(nrp, orc):
    import torch
    rng = np.random.default_rng(21)
    L, D, H, ff, K, F = 2, 256, 2, 1024, 9, 80
    B, T, C = 2, 14, 42  # encoder frames per chunk, attention cache
    enc, sw, bws = build(nrp, orc, rng, L, D, H, ff, K, F, True)
    cache = enc.new_stream_cache(B, C)
    actx = nrp.AttentionContext.new((C, T - 1), "chunked_limited")
    pe_h = orc.get_encoding(D, 5000, C + T)
    hcs = [np.zeros((B, C, D), np.float32) for _ in range(L)]
    ccs = [np.zeros((B, K - 1, D), np.float32) for _ in range(L)]
    filled = 0
    # causal subsampling: 8 t mel frames give t + 1 encoder frames; with
    # drop_extra_pre_encoded = 1, 8 T mel frames give T frames
    steps = [(8 * T, 1, None), (8 * T, 1, None), (8 * T, 1, None), (8 * T, 1, None),
             (8 * T, 1, [8 * T - 40, 8 * T])]
    for k, (frames, drop, lengths) in enumerate(steps):
        mel = rng.standard_normal((B, F, frames)).astype(np.float32)
        feats = torch.from_numpy(mel).cuda()
        ln = np.array(lengths, np.int32) if lengths is not None else None
        out, out_len = enc.forward_streaming(feats, ln, cache, drop, actx)
        enc.ctx.check()
        # oracle
        x = orc.subsampling_forward(np.ascontiguousarray(mel.transpose(0, 2, 1)), sw, D, 8, True,
                                    bf16=True)[:, drop:]
        assert x.shape[1] == T
        x = orc.bf16_round(x * np.float32(np.sqrt(D)))
        lens = [frames] * B if lengths is None else lengths
        want_len = [orc.subsampling_out_len(v, 8, True) - drop for v in lens]
        assert list(out_len) == want_len
        valid = min(want_len[0], T)
        nxt = filled
        for i, bw in enumerate(bws):
            x, nxt = orc.stream_block_step(x, bw, pe_h, H, ff, K, hcs[i], ccs[i], filled, valid,
                                           C, T - 1, True, bf16=True)
        filled = nxt
        got = out.float().cpu().numpy().transpose(0, 2, 1)
        assert np.isfinite(got).all()
        err = rel(got[:, :valid], x[:, :valid])
        assert err < TOL_BF16, (k, err)
        assert cache.filled == filled
    # the caches in EncoderCache's layout
    lc = cache.last_channel().cpu().numpy()
    lt = cache.last_time().cpu().numpy()
    assert lc.shape == (L, B, C, D) and lt.shape == (L, B, D, K - 1)
    for i in range(L):
        assert rel(lc[i], hcs[i]) < TOL_BF16
        assert rel(lt[i], ccs[i].transpose(0, 2, 1)) < TOL_BF16


def test_stream_encoder_reset_repeats_bitwise(nrp, orc):
    import torch
    rng = np.random.default_rng(5)
    L, D, H, ff, K, F = 2, 256, 2, 1024, 9, 80
    B, T, C = 3, 14, 28
    enc, _, _ = build(nrp, orc, rng, L, D, H, ff, K, F, False)
    cache = enc.new_stream_cache(B, C)
    actx = nrp.AttentionContext.new((C, T - 1), "chunked_limited")
    mels = [torch.from_numpy(rng.standard_normal((B, F, 8 * T)).astype(np.float32)).cuda()
            for _ in range(4)]

    def run():
        outs = []
        for m in mels:
            y, _ = enc.forward_streaming(m, None, cache, 1, actx)
            outs.append(y.clone())
        return outs

    a = run()
    assert cache.filled == C
    saved_t = cache.last_time()
    cache.reset()
    assert cache.filled == 0
    b = run()
    enc.ctx.check()
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    # last_time round-trips through set_last_time
    cache.set_last_time(saved_t)
    assert torch.equal(cache.last_time(), saved_t)
