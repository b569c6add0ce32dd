"""StreamingStepGraphs: a stack of cached attention layers driven chunk by
chunk through CUDA graphs equals the same calls made one by one, bit for bit,
through the warm-up (fill 0 .. cache_len) and two full cycles of the ring."""
import numpy as np
import pytest

from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def _stack(nrp, rng, L, D, H, B, C):
    layers, caches = [], []
    f = lambda *sh: (rng.standard_normal(sh).astype(np.float32) * 0.05)
    for _ in range(L):
        a = nrp.RelPositionMultiHeadAttention(D, H, True)
        for which, bias in ((nrp.LINEAR_Q, True), (nrp.LINEAR_K, True), (nrp.LINEAR_V, True),
                            (nrp.LINEAR_OUT, True), (nrp.LINEAR_POS, False)):
            a.set_linear(which, nrp.LinearLayer.standard(f(D, D), f(D) if bias else None))
        a.set_pos_bias(f(H, D // H), f(H, D // H))
        a.set_dtype(nrp.BF16)
        layers.append(a)
        caches.append(nrp.AttentionCache(a, B, C))
    return layers, caches


def test_graph_driven_stream_equals_eager(nrp):
    import torch
    L, D, H, B, C, T, chunks = 3, 256, 2, 4, 28, 7, 16
    seed = np.random.default_rng(5)
    chunk_x = [torch.from_numpy(seed.standard_normal((B, T, D)).astype(np.float32))
               .cuda().bfloat16() for _ in range(chunks)]
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(C + T)
    actx = nrp.AttentionContext.new((C, T - 1), "chunked_limited")

    def run(use_graphs):
        layers, caches = _stack(nrp, np.random.default_rng(9), L, D, H, B, C)
        x = torch.empty((B, T, D), dtype=torch.bfloat16, device="cuda")
        bufs = [torch.empty_like(x) for _ in range(L)]

        def step(filled):
            h = x
            for i, a in enumerate(layers):
                a.forward_with_cache(h, pos, caches[i], filled, T, actx, out=bufs[i])
                h = bufs[i]

        drive = nrp.StreamingStepGraphs(step, caches) if use_graphs else step
        outs = []
        for k in range(chunks):
            x.copy_(chunk_x[k])
            drive(min(k * T, C))
            outs.append(bufs[-1].clone())
        layers[0].ctx.check()
        return outs, [c.export_h() for c in caches], drive

    eager, h_eager, _ = run(False)
    graphed, h_graph, drive = run(True)
    # fill 0, 7, 14, 21, then 28 with the ring cycling over 4 slots: the
    # full-cache keys are captured on their second chunk and replayed on their
    # third
    assert len(drive.graphs) == 4
    for k, (a, b) in enumerate(zip(eager, graphed)):
        assert torch.equal(a, b), k
    for a, b in zip(h_eager, h_graph):
        assert torch.equal(a, b)


def test_graph_driven_encoder_stream_equals_eager(nrp, orc):
    """ConformerEncoder.forward_streaming (subsampling, conv caches,
    attention rings, fill level) driven through StreamingStepGraphs over the
    encoder cache's rings equals eager calls bit for bit, caches included."""
    import torch
    from test_gpu_stream_encoder import build
    rng = np.random.default_rng(8)
    L, D, H, ff, K, F = 2, 256, 2, 1024, 9, 80
    B, T, C, chunks = 2, 7, 21, 12
    enc, _, _ = build(nrp, orc, rng, L, D, H, ff, K, F, True)
    actx = nrp.AttentionContext.new((C, T - 1), "chunked_limited")
    mels = [torch.from_numpy(rng.standard_normal((B, F, 8 * T)).astype(np.float32)).cuda()
            for _ in range(chunks)]

    def run(use_graphs):
        cache = enc.new_stream_cache(B, C)
        x = torch.empty_like(mels[0])
        out = torch.empty((B, D, T), dtype=torch.bfloat16, device="cuda")

        def step(filled):
            cache.filled = filled
            enc.forward_streaming(x, None, cache, 1, actx, out=out)

        drive = nrp.StreamingStepGraphs(step, cache.rings()) if use_graphs else step
        outs = []
        for k in range(chunks):
            x.copy_(mels[k])
            drive(min(k * T, C))
            outs.append(out.clone())
        enc.ctx.check()
        return outs, cache.last_channel(), cache.last_time(), drive

    eager, ch_e, t_e, _ = run(False)
    graphed, ch_g, t_g, drive = run(True)
    assert len(drive.graphs) >= 1
    for k, (a, b) in enumerate(zip(eager, graphed)):
        assert torch.equal(a, b), k
    assert torch.equal(ch_e, ch_g) and torch.equal(t_e, t_g)
