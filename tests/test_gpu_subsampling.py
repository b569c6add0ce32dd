"""Device parity of the dw_striding subsampling (Subsampling::forward_frames,
src/asr/modules/encoders/conformer.rs:1413-1555) and of the encoder's
mel-input forward (ConformerEncoder::forward, 475-560) against the CPU
oracle (oracle.subsampling_forward, itself checked against a torch
composition and the reference's chunking test), through the C ABI.  bf16
tolerance 2e-2 of the output scale over every output frame."""
import numpy as np
import pytest

from conftest import rand_block
from test_subsampling_oracle import rand_sub
from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def sub_weights(orc, rng, C, F, D, factor, causal, quant, prefix="encoder.pre_encode"):
    """(oracle dict, NeMo-named MLX-layout weight dict)."""
    sw = rand_sub(rng, C, F, D, factor, causal)
    wd = {f"{prefix}.conv.0.weight": sw["conv0"][0], f"{prefix}.conv.0.bias": sw["conv0"][1]}
    for i, ((dw, db), (pw, pb)) in enumerate(zip(sw["dw"], sw["pw"])):
        wd[f"{prefix}.conv.{2 + 3 * i}.weight"], wd[f"{prefix}.conv.{2 + 3 * i}.bias"] = dw, db
        wd[f"{prefix}.conv.{3 + 3 * i}.weight"], wd[f"{prefix}.conv.{3 + 3 * i}.bias"] = pw, pb
    w, b = sw["out"]
    if quant:
        wq, s, z = orc.quantize(w, 64, 8)
        s = s.astype(np.float16).astype(np.float32)
        z = z.astype(np.float16).astype(np.float32)
        wd[f"{prefix}.out.weight"], wd[f"{prefix}.out.scales"] = wq, s
        wd[f"{prefix}.out.biases"] = z
        sw["out"] = (orc.dequantize(wq, orc.bf16_round(s), orc.bf16_round(z), 64, 8), b)
    else:
        wd[f"{prefix}.out.weight"] = w
    wd[f"{prefix}.out.bias"] = b
    return sw, wd


def masked(x_btf, lengths):
    x = x_btf.copy()
    if lengths is not None:
        for b, L in enumerate(lengths):
            x[b, L:] = 0.0
    return x


def rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("B,T,F,C,D,factor,causal,layout,lengths,quant", [
    (2, 203, 80, 256, 512, 8, False, "btf", None, False),
    (2, 203, 80, 256, 512, 8, True, "bft", [203, 120], False),
    (3, 400, 128, 256, 1024, 8, False, "bft", [400, 1, 257], False),
    (2, 160, 80, 256, 512, 8, False, "bft", [160, 90], True),
    (2, 97, 80, 128, 256, 4, False, "btf", None, False),
    (2, 97, 80, 128, 256, 4, True, "btf", [97, 50], False),
    (1, 64, 80, 64, 256, 2, False, "btf", None, False),
    (1, 64, 80, 64, 256, 2, True, "bft", [40], False),
    (1, 1, 80, 256, 512, 8, False, "btf", None, False),
    (2, 37, 128, 256, 512, 8, True, "btf", [0, 37], False),
])
def test_subsampling_matches_oracle(nrp, orc, B, T, F, C, D, factor, causal, layout, lengths,
                                    quant):
    import torch
    rng = np.random.default_rng(T * 10 + F + factor + causal)
    sw, wd = sub_weights(orc, rng, C, F, D, factor, causal, quant)
    sub = nrp.Subsampling(F, D, factor, C, causal)
    sub.load_weights(wd, quant=nrp.QuantizationConfig(8, 64) if quant else None)
    sub.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, F)).astype(np.float32)
    if layout == "btf":
        xd = torch.from_numpy(x).cuda()
        lay = nrp.FEATURES_BTF
    else:
        xd = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
        lay = nrp.FEATURES_BFT
    ln = np.array(lengths, np.int32) if lengths is not None else None
    out, out_len = sub.forward(xd, ln, layout=lay)
    sub.ctx.check()
    got = out.float().cpu().numpy()
    ref = orc.subsampling_forward(masked(x, lengths), sw, D, factor, causal, bf16=True)
    assert got.shape == ref.shape
    assert np.isfinite(got).all()
    err = rel(got, ref)
    assert err < TOL_BF16, err
    if ln is not None:
        assert list(out_len) == [orc.subsampling_out_len(v, factor, causal) for v in ln]


def test_subsampling_repeat_is_bitwise(nrp, orc):
    """The same input twice, and a batch of one, give the same bits (no
    state kept between calls, no cross-utterance reads)."""
    import torch
    rng = np.random.default_rng(21)
    sw, wd = sub_weights(orc, rng, 256, 80, 512, 8, False, False)
    sub = nrp.Subsampling(80, 512, 8, 256, False)
    sub.load_weights(wd)
    sub.set_dtype(nrp.BF16)
    x = torch.from_numpy(rng.standard_normal((3, 80, 333)).astype(np.float32)).cuda()
    a, _ = sub.forward(x, [333, 200, 17], layout=nrp.FEATURES_BFT)
    b, _ = sub.forward(x, [333, 200, 17], layout=nrp.FEATURES_BFT)
    c, _ = sub.forward(x[1:2].contiguous(), [200], layout=nrp.FEATURES_BFT)
    sub.ctx.check()
    assert torch.equal(a, b)
    assert torch.equal(a[1:2], c)


def test_encoder_forward_from_mel(nrp, orc):
    """ConformerEncoder::forward: mel [B, F, T] masked past each length, the
    subsampling, x * sqrt(d_model), the blocks with the subsampled lengths,
    the [B, D, T'] transpose.  Equals the subsampling followed by
    forward_from_embeddings bit for bit, and the oracle's composition."""
    import torch
    rng = np.random.default_rng(8)
    B, T, F, D, H, ff, K, L = 2, 403, 80, 256, 2, 1024, 9, 2
    enc = nrp.ConformerEncoder(L, D, H, ff, K, feat_in=F, subsampling_factor=8,
                               subsampling_conv_channels=256)
    sw, wd = sub_weights(orc, rng, 256, F, D, 8, False, True)
    bws = []
    for i in range(L):
        bw, w = rand_block(rng, D, H, ff, K, quant=True, orc=orc, prefix=f"encoder.layers.{i}")
        bws.append(bw)
        wd.update(w)
    enc.load_weights(wd, nrp.QuantizationConfig(8, 64))
    enc.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, F)).astype(np.float32)
    lengths = np.array([403, 250], np.int32)
    feats = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
    out, out_len = enc.forward(feats, lengths)
    emb, emb_len = enc.subsampling.forward(feats, lengths, layout=nrp.FEATURES_BFT)
    parts, _ = enc.forward_from_embeddings(emb, emb_len)
    enc.ctx.check()
    Tp = orc.subsampling_out_len(T, 8, False)
    assert tuple(out.shape) == (B, D, Tp)
    assert list(out_len) == [orc.subsampling_out_len(v, 8, False) for v in lengths]
    assert torch.equal(out, parts)
    got = out.float().cpu().numpy().transpose(0, 2, 1)
    h = orc.subsampling_forward(masked(x, lengths), sw, D, 8, False, bf16=True)
    h = orc.bf16_round(h * np.float32(np.sqrt(D)))
    pe = orc.get_encoding(D, 5000, Tp)
    for bw in bws:
        h = orc.block_forward(h, bw, pe, H, ff, K, lengths=out_len, bf16=True)
    err = max(rel(got[b, :n], h[b, :n]) for b, n in enumerate(out_len))
    assert err < TOL_BF16, err


@pytest.mark.parametrize("B,T,factor,causal,layout,lengths,chunk", [
    # lengths ending inside a chunk, on a chunk edge, and inside the context
    (3, 1300, 8, False, "btf", [1300, 700, 1030], 512),
    (2, 1300, 8, True, "bft", [1300, 517], 512),
    (2, 901, 4, False, "bft", None, 256),
    (2, 901, 4, True, "btf", [901, 260], 256),
    (1, 330, 2, False, "btf", [300], 64),
    (2, 4100, 8, False, "bft", [4100, 4096], 4096),  # the reference's chunk size
])
def test_chunked_subsampling_equals_single_pass(nrp, orc, B, T, factor, causal, layout, lengths,
                                                 chunk):
    """forward_frames_chunked (conformer.rs:1334-1377) on the device gives the
    single pass's output bit for bit: every output frame is computed from the
    same input frames by the same arithmetic."""
    import torch
    F, C, D = 80, 256 if factor == 8 else 128, 512
    rng = np.random.default_rng(T + factor + 7 * causal)
    sw, wd = sub_weights(orc, rng, C, F, D, factor, causal, False)
    sub = nrp.Subsampling(F, D, factor, C, causal)
    sub.load_weights(wd)
    sub.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, F)).astype(np.float32)
    if layout == "btf":
        xd, lay = torch.from_numpy(x).cuda(), nrp.FEATURES_BTF
    else:
        xd = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1))).cuda()
        lay = nrp.FEATURES_BFT
    whole, _ = sub.forward(xd, lengths, layout=lay)
    sub.set_chunk_frames(chunk)
    chunked, _ = sub.forward(xd, lengths, layout=lay)
    sub.set_chunk_frames(0)
    sub.ctx.check()
    assert chunked.shape == whole.shape == (B, sub.output_length(T), D)
    assert torch.equal(chunked.view(torch.int16), whole.view(torch.int16))
    if T <= 1300:  # and the single pass against the oracle
        ref = orc.subsampling_forward(masked(x, lengths), sw, D, factor, causal, bf16=True)
        assert rel(whole.float().cpu().numpy(), ref) < TOL_BF16
