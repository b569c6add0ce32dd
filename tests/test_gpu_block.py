"""Device parity of the Conformer block and encoder (BASELINE config 3's
layer: macaron FF 1024->4096->1024 with SiLU, rel-pos MHA 8x128, conv module
with depthwise kernel 9, GLU and BatchNorm, all linears MLX 8-bit) against
the CPU oracle (oracle.block_forward, conformer.rs:1693-1870), through the
C ABI.  bf16 tolerance 2e-2 of the output scale over valid rows, and per
element |got - ref| <= 2e-2 * (|ref| + 4 rms(ref))."""
import numpy as np
import pytest

from conftest import rand_block
from __graft_entry__ import load_package
from test_gpu_parity import check_close

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def rel_err(got, ref, lengths):
    """Max-normalised error over the valid rows; also asserts the
    per-element bound of check_close."""
    return check_close(got, ref, lengths, TOL_BF16)[1]


def make_block(nrp, wd, D, H, ff, K, causal, conv_norm, quant):
    blk = nrp.ConformerBlock(D, H, ff, K, causal, conv_norm)
    blk.load_weights(wd, "b", nrp.QuantizationConfig(8, 64) if quant else None)
    blk.set_dtype(nrp.BF16)
    return blk


@pytest.mark.parametrize("B,T,D,H,ff,K,causal,conv_norm,quant,lengths,context", [
    (3, 300, 256, 2, 1024, 9, False, "batch_norm", False, [300, 171, 245], None),
    (2, 260, 256, 2, 1024, 9, False, "batch_norm", True, [260, 130], None),
    (2, 200, 256, 2, 512, 5, True, "layer_norm", False, None, (64, 0, False)),
    (1, 129, 512, 4, 2048, 31, False, "batch_norm", True, None, (70, 13, True)),
    (2, 150, 512, 4, 1024, 9, True, "layer_norm", False, [150, 77], None),
    (3, 70, 256, 2, 768, 9, False, "batch_norm", True, [70, 1, 33], None),
    (2, 500, 1024, 8, 4096, 9, False, "batch_norm", True, [500, 313], None),
    (3, 500, 1024, 8, 4096, 9, False, "batch_norm", True, [500, 250, 421], None),
])
def test_block_matches_oracle(nrp, orc, B, T, D, H, ff, K, causal, conv_norm, quant, lengths,
                              context):
    import torch
    rng = np.random.default_rng(B * 100 + T + D)
    bw, wd = rand_block(rng, D, H, ff, K, conv_norm, quant=quant, orc=orc)
    blk = make_block(nrp, wd, D, H, ff, K, causal, conv_norm, quant)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    ln = np.array(lengths, np.int32) if lengths is not None else None
    mask = nrp.key_padding_mask(ln, T) if ln is not None else None
    ctx = nrp.AttentionContext.new(context[:2], "chunked_limited" if context[2] else "regular") \
        if context is not None else None
    xd = torch.from_numpy(x).cuda().bfloat16()
    got = blk.forward(xd, pe.get_encoding(T), ctx, mask)
    blk.ctx.check()
    got = got.float().cpu().numpy()
    ref = orc.block_forward(x, bw, pe.get_encoding_host(T)[0], H, ff, K, causal=causal,
                            conv_norm=0 if conv_norm == "batch_norm" else 1, lengths=ln,
                            context=context, bf16=True)
    rows = lengths or [T] * B
    assert all(np.isfinite(got[b, :L]).all() for b, L in enumerate(rows))
    err = rel_err(got, ref, rows)
    assert err < TOL_BF16, err


def test_block_in_place_equals_out_of_place(nrp, orc):
    import torch
    rng = np.random.default_rng(2)
    B, T, D, H, ff, K = 2, 150, 256, 2, 1024, 9
    _, wd = rand_block(rng, D, H, ff, K)
    blk = make_block(nrp, wd, D, H, ff, K, False, "batch_norm", False)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    x = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).cuda().bfloat16()
    a = blk.forward(x, pos)
    y = x.clone()
    blk.forward(y, pos, out=y)
    blk.ctx.check()
    assert torch.equal(a, y)


def test_encoder_forward_from_embeddings(nrp, orc):
    """Three layers of forward_from_embeddings (conformer.rs:694-722): x *
    sqrt(d_model), the blocks, the [B, D, T] transpose.  The quantised
    weights of each next layer are dequantised on a second stream into one
    of two slots, so three layers reuse a slot; a second forward reuses both
    and must give the same bits."""
    import torch
    rng = np.random.default_rng(4)
    B, T, D, H, ff, K, L = 2, 180, 256, 2, 1024, 9, 3
    enc = nrp.ConformerEncoder(L, D, H, ff, K)
    bws, wd = [], {}
    for i in range(L):
        bw, w = rand_block(rng, D, H, ff, K, quant=True, orc=orc, prefix=f"encoder.layers.{i}")
        bws.append(bw)
        wd.update(w)
    enc.load_weights(wd, nrp.QuantizationConfig(8, 64))
    enc.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    lengths = np.array([180, 97], np.int32)
    xd = torch.from_numpy(x).cuda().bfloat16()
    out, out_len = enc.forward_from_embeddings(xd, lengths)
    again, _ = enc.forward_from_embeddings(xd, lengths)
    enc.ctx.check()
    assert torch.equal(out, again)
    assert tuple(out.shape) == (B, D, T) and np.array_equal(out_len, lengths)
    got = out.float().cpu().numpy().transpose(0, 2, 1)
    h = orc.bf16_round(orc.bf16_round(x) * np.float32(np.sqrt(D)))
    pe = orc.get_encoding(D, 5000, T)
    for bw in bws:
        h = orc.block_forward(h, bw, pe, H, ff, K, lengths=lengths, bf16=True)
    err = rel_err(got, h, lengths)
    assert err < TOL_BF16, err


@pytest.mark.parametrize("form", ["mlx_dir", "nemo"])
def test_encoder_from_checkpoint_equals_dict(nrp, orc, tmp_path, form):
    """ConformerEncoder.load_checkpoint (weights.rs, checkpoint.rs): an MLX
    8-bit model directory, or a .nemo archive with PyTorch-layout float
    weights, gives the same bits as loading the same arrays from a dict."""
    import json
    import tarfile
    import torch
    from test_checkpoint import _pytorch_layout
    rng = np.random.default_rng(11)
    B, T, D, H, ff, K, L = 2, 140, 256, 2, 1024, 9, 2
    quant = form == "mlx_dir"
    wd = {}
    for i in range(L):
        _, w = rand_block(rng, D, H, ff, K, quant=quant, orc=orc, prefix=f"encoder.layers.{i}")
        wd.update(w)
    wd = {k: np.asarray(v) for k, v in wd.items()}
    if form == "mlx_dir":
        path = tmp_path / "model"
        path.mkdir()
        nrp.write_safetensors(str(path / "model.safetensors"), wd, metadata={"format": "mlx"})
        (path / "config.json").write_text(json.dumps({"quantization": {"bits": 8,
                                                                       "group_size": 64}}))
    else:
        st = tmp_path / "w.safetensors"
        nrp.write_safetensors(str(st), _pytorch_layout(wd))
        path = tmp_path / "m.nemo"
        with tarfile.open(path, "w") as tar:
            tar.add(str(st), arcname="model_weights.safetensors")
            cfg = tmp_path / "model_config.yaml"
            cfg.write_text("encoder: {}\n")
            tar.add(str(cfg), arcname="model_config.yaml")
    a = nrp.ConformerEncoder(L, D, H, ff, K)
    a.load_weights(wd, nrp.QuantizationConfig(8, 64) if quant else None)
    b = nrp.ConformerEncoder(L, D, H, ff, K)
    q = b.load_checkpoint(str(path))
    assert (q is not None) == quant
    a.set_dtype(nrp.BF16)
    b.set_dtype(nrp.BF16)
    x = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).cuda().bfloat16()
    lengths = np.array([140, 77], np.int32)
    ya, _ = a.forward_from_embeddings(x, lengths)
    yb, _ = b.forward_from_embeddings(x, lengths)
    a.ctx.check()
    assert torch.equal(ya, yb)


def test_weight_cache_equals_per_call_dequant_and_follows_reloads(nrp, orc):
    """The kept bf16 copies of quantised weights give the same bits as the
    per-call dequantisation, and re-loading a block's weights replaces its
    copies (the output follows the new weights, checked against the
    oracle)."""
    import torch
    rng = np.random.default_rng(31)
    B, T, D, H, ff, K = 2, 300, 256, 2, 1024, 9
    ctx = nrp.Context(0)
    bw1, wd1 = rand_block(rng, D, H, ff, K, quant=True, orc=orc)
    bw2, wd2 = rand_block(rng, D, H, ff, K, quant=True, orc=orc)
    blk = nrp.ConformerBlock(D, H, ff, K, ctx=ctx)
    blk.load_weights(wd1, "b", nrp.QuantizationConfig(8, 64))
    blk.set_dtype(nrp.BF16)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    xd = torch.from_numpy(x).cuda().bfloat16()
    a = blk.forward(xd, pe.get_encoding(T))  # makes the copies
    b = blk.forward(xd, pe.get_encoding(T))  # uses them
    ctx.set_weight_cache(False)
    c = blk.forward(xd, pe.get_encoding(T))  # scratch per call
    ctx.set_weight_cache(True)
    ctx.check()
    assert torch.equal(a, b) and torch.equal(a, c)
    blk.load_weights(wd2, "b", nrp.QuantizationConfig(8, 64))
    blk.set_dtype(nrp.BF16)
    y = blk.forward(xd, pe.get_encoding(T)).float().cpu().numpy()
    ctx.check()
    ref = orc.block_forward(x, bw2, pe.get_encoding_host(T)[0], H, ff, K, bf16=True)
    assert rel_err(y, ref, [T] * B) < TOL_BF16
