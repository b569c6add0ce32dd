"""Device parity of the sequence-split forward (nrp_attn_forward_seq_sharded):
long-form windowed attention cut along the sequence, one segment per GPU,
with the K/V halo exchanged over NCCL.

- one rank: the time-major halo buffer, the row-tiled projection and the
  attention geometry give nrp_attn_forward's result;
- two ranks (two GPUs, skipped with fewer): the gathered segments match the
  oracle's single-device forward (bf16 tolerance 2e-2) and, at BASELINE
  config 4's shape ([4, 12500, 1024], window (128, 128)), nrp_attn_forward
  on one GPU.

Each rank is its own process on its own GPU (gloo carries the NCCL id and the
gathered results); no two ranks share a GPU.
"""
import numpy as np
import pytest

from conftest import rand_weights
from __graft_entry__ import load_package
from test_seq_split_host import _spawn

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _module(nrp, w, D, H, ctx=None):
    attn = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
    for which, (wk, bk) in enumerate((("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo"),
                                      ("wp", None))):
        attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(nrp.BF16)
    return attn


def _rel(got, ref, lengths):
    err = 0.0
    for b, L in enumerate(lengths):
        err = max(err, float(np.abs(got[b, :L] - ref[b, :L]).max() / np.abs(ref[b, :L]).max()))
    return err


def test_one_rank_matches_forward():
    if _gpus() < 1:
        pytest.skip("needs a CUDA device")
    import torch
    nrp = load_package()
    rng = np.random.default_rng(3)
    B, T, D, H = 3, 700, 256, 2
    w = rand_weights(rng, D, H)
    attn = _module(nrp, w, D, H)
    lengths = np.array([700, 500, 650], np.int32)
    mask = nrp.key_padding_mask(lengths, T)
    ctx = nrp.AttentionContext.new((128, 128), "regular")
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    x = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).cuda().bfloat16()
    halo = nrp.HaloComm(0, 1, nrp.HaloComm.unique_id())
    try:
        got = attn.forward_seq_sharded(x, pos, T, halo, ctx, mask)
        halo.check()
        ref = attn.forward(x, pos, ctx, mask)
        attn.ctx.check()
    finally:
        halo.close()
    err = _rel(got.float().cpu().numpy(), ref.float().cpu().numpy(), lengths)
    assert err < 1e-3, err


def _rank(rank, world, B, T, D, H, context, lengths, seed, check):
    import torch
    from __graft_entry__ import load_package
    nrp = load_package()
    torch.cuda.set_device(rank)
    dev = nrp.Context(rank)
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, D, H)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    attn = _module(nrp, w, D, H, ctx=dev)
    ctx = nrp.AttentionContext.new(context[:2], "chunked_limited" if context[2] else "regular")
    mask = nrp.key_padding_mask(lengths, T)  # lengths on the current device
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=rank)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    halo = nrp.HaloComm.from_process_group(ctx=dev, timeout_ms=60000)
    try:
        p = halo.plan(T, ctx)
        xl = torch.from_numpy(x[:, p.start:p.start + p.len]).to(f"cuda:{rank}").bfloat16()
        for _ in range(2):  # the second step reuses the halo buffer
            got = attn.forward_seq_sharded(xl, pos, T, halo, ctx, mask)
        halo.check()
        dev.check()
        mine = got.float().cpu().numpy()
    finally:
        halo.close()
    import torch.distributed as dist
    parts = [None] * world
    dist.all_gather_object(parts, (p.start, mine))
    if rank != 0:
        return None
    full = np.zeros((B, T, D), np.float32)
    for s, o in parts:
        full[:, s:s + o.shape[1]] = o
    if check == "oracle":
        from oracle import oracle as orc
        ref = orc.mha_forward(x, w, pe.get_encoding_host(T)[0], H, lengths=lengths,
                              context=context, bf16=True)
    else:  # the single-device forward on this GPU
        xd = torch.from_numpy(x).to(f"cuda:{rank}").bfloat16()
        ref = attn.forward(xd, pos, ctx, mask).float().cpu().numpy()
        dev.check()
    return _rel(full, ref, lengths)


@pytest.mark.parametrize("B,T,D,H,context,lengths", [
    (2, 3000, 256, 2, (128, 128, False), [3000, 2100]),
    (1, 1000, 256, 2, (70, 13, True), [1000]),
    (2, 777, 256, 2, (16, 0, False), [777, 400]),
])
def test_two_ranks_match_oracle(B, T, D, H, context, lengths):
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    err = _spawn(_rank, 2, B, T, D, H, context, np.array(lengths, np.int32), 11, "oracle")[0]
    assert err < TOL_BF16, err


def test_two_ranks_config4_shape_match_one_device():
    """[4, 12500, 1024] bf16, 8 heads, window (128, 128)."""
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    err = _spawn(_rank, 2, 4, 12500, 1024, 8, (128, 128, False),
                 np.array([12500] * 4, np.int32), 4, "device")[0]
    assert err < TOL_BF16, err
