"""Host side of the sequence-split forward (long-form
windowed attention cut along the sequence, one segment per GPU, with a K/V
halo exchanged between neighbours).  CPU only:

- the halo plan (nrp_seq_shard_plan) is consistent between neighbours and
  covers the sequence;
- two gloo ranks that follow the plan -- project their own frames, swap the
  halo rows with their neighbour, attend over [segment + halo] with global
  frame indices -- reproduce the oracle's single-device forward
  (RelPositionMultiHeadAttention::forward, attention.rs:446-573);
- HaloComm.share_unique_id hands every rank the same NCCL id over
  torch.distributed.

The device path runs in test_gpu_seq_split.py (two GPUs).
"""
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

from conftest import ROOT, rand_weights
from __graft_entry__ import load_package

CONTEXTS = [(128, 128, False), (5, 3, False), (4, 1, True), (70, 13, True), (16, 0, False)]


@pytest.fixture(scope="module")
def nrp():
    return load_package()


def _ctx(nrp, c):
    return nrp.AttentionContext.new(c[:2], "chunked_limited" if c[2] else "regular")


@pytest.mark.parametrize("context", CONTEXTS)
@pytest.mark.parametrize("T,n", [(12500, 2), (12500, 4), (12500, 8), (1001, 3), (700, 5)])
def test_plan_is_consistent_between_neighbours(nrp, context, T, n):
    ctx = _ctx(nrp, context)
    plans = [nrp.seq_shard_plan(T, n, r, ctx) for r in range(n)]
    assert plans[0].start == 0 and plans[-1].start + plans[-1].len == T
    for r in range(n):
        p = plans[r]
        assert p.len > 0
        if r + 1 < n:
            q = plans[r + 1]
            assert q.start == p.start + p.len
            assert p.send_next == q.halo_left and q.send_prev == p.halo_right
        # the halo covers every key the segment's rows can see
        vis = nrp.AttentionContext.block_mask(ctx, p.start, p.start + p.len, T)
        cols = np.nonzero(vis.any(axis=0))[0]
        assert cols.min() >= p.start - p.halo_left
        assert cols.max() < p.start + p.len + p.halo_right
    assert plans[0].halo_left == 0 and plans[0].send_prev == 0
    assert plans[-1].halo_right == 0 and plans[-1].send_next == 0


def test_plan_rejects_windows_wider_than_a_segment(nrp):
    ctx = _ctx(nrp, (128, 128, False))
    with pytest.raises(nrp.NrpError) as e:
        nrp.seq_shard_plan(300, 8, 3, ctx)
    assert e.value.code == nrp.NRP_ERR_UNSUPPORTED
    with pytest.raises(nrp.NrpError):
        nrp.seq_shard_plan(9, 8, 0, None)  # ranks without frames


# ----------------------------------------------------- two gloo ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args):
    """Runs target(rank, world, *args) in `world` spawned processes joined
    in a gloo group; returns rank 0's result or raises a rank's error."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(target, r, world, port, q, args))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, ok, val = q.get(timeout=240)
            if not ok:
                raise AssertionError(f"rank {r}: {val}")
            results[r] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def _rank_main(target, rank, world, port, q, args):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        try:
            q.put((rank, True, target(rank, world, *args)))
        finally:
            dist.destroy_process_group()
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _share_id(rank, world):
    from __graft_entry__ import load_package
    return load_package().HaloComm.share_unique_id()


def test_unique_id_reaches_every_rank():
    ids = _spawn(_share_id, 2)
    assert len(ids[0]) == 128 and ids[0] == ids[1]


def _shard_forward(rank, world, T, B, D, H, context, lengths, seed):
    """One rank of the sequence split, in numpy (f32), following the plan
    the library computes: project the segment's frames, swap halo rows with
    the neighbours, attend with global frame indices, project out."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle as orc
    nrp = load_package()
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, D, H)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    pe = orc.get_encoding(D, 5000, T)
    ctx = nrp.AttentionContext.new(context[:2], "chunked_limited" if context[2] else "regular")
    p = nrp.seq_shard_plan(T, world, rank, ctx)
    s, e = p.start, p.start + p.len
    wqkv = np.concatenate([w["wq"], w["wk"], w["wv"]], 0)
    bqkv = np.concatenate([w["bq"], w["bk"], w["bv"]], 0)
    mine = x[:, s:e] @ wqkv.T + bqkv  # [B, len, 3D]
    # halo rows: first send_prev frames to rank-1, last send_next to rank+1
    left = np.zeros((B, p.halo_left, 3 * D), np.float32)
    right = np.zeros((B, p.halo_right, 3 * D), np.float32)
    ops = []
    if rank > 0:
        ops.append(dist.P2POp(dist.isend, torch.from_numpy(
            np.ascontiguousarray(mine[:, :p.send_prev])), rank - 1))
        lt = torch.from_numpy(left)
        ops.append(dist.P2POp(dist.irecv, lt, rank - 1))
    if rank + 1 < world:
        ops.append(dist.P2POp(dist.isend, torch.from_numpy(
            np.ascontiguousarray(mine[:, p.len - p.send_next:])), rank + 1))
        rt = torch.from_numpy(right)
        ops.append(dist.P2POp(dist.irecv, rt, rank + 1))
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    buf = np.concatenate([left, mine, right], 1)  # frames [base, base + tbuf)
    base = s - p.halo_left
    tbuf = buf.shape[1]
    q, k, v = buf[..., :D], buf[..., D:2 * D], buf[..., 2 * D:]
    q = q[:, p.halo_left:p.halo_left + p.len]
    dh = D // H
    vis = orc.block_mask(*context, s, e, T)[:, base:base + tbuf]  # [len, tbuf]
    ii = np.arange(s, e)[:, None]
    jj = np.arange(base, base + tbuf)[None, :]
    rows = T - 1 - ii + jj  # P row of each (i, j)
    proj_p = pe @ w["wp"].T  # [2T-1, D] (only rows[vis] are used)
    ctx_out = np.zeros((B, p.len, D), np.float32)
    for b in range(B):
        keep = vis & (jj < max(int(lengths[b]), 1))
        for h in range(H):
            sl = slice(h * dh, (h + 1) * dh)
            qu = q[b, :, sl] + w["pos_bias_u"][h]
            qv = q[b, :, sl] + w["pos_bias_v"][h]
            ac = qu @ k[b, :, sl].T
            bd = np.einsum("id,ijd->ij", qv, proj_p[rows][:, :, sl])
            sc = np.where(keep, (ac + bd) / np.sqrt(dh), -np.inf)
            sc -= sc.max(1, keepdims=True)
            pr = np.exp(sc)
            pr /= pr.sum(1, keepdims=True)
            ctx_out[b, :, sl] = pr @ v[b, :, sl]
    out = ctx_out @ w["wo"].T + w["bo"]
    gathered = [None] * world
    dist.all_gather_object(gathered, (s, out))
    if rank != 0:
        return None
    full = np.zeros((B, T, D), np.float32)
    for s0, o in gathered:
        full[:, s0:s0 + o.shape[1]] = o
    ref = orc.mha_forward(x, w, pe, H, lengths=lengths, context=context)
    err = 0.0
    for b in range(B):
        L = int(lengths[b])
        err = max(err, float(np.abs(full[b, :L] - ref[b, :L]).max() / np.abs(ref[b, :L]).max()))
    return err


@pytest.mark.parametrize("T,context,lengths", [
    (300, (128, 128, False), [300, 300]),
    (97, (5, 3, False), [97, 60]),
    (120, (4, 1, True), [120, 33]),
])
def test_two_ranks_with_halo_match_single_device_forward(T, context, lengths):
    err = _spawn(_shard_forward, 2, T, 2, 64, 2, context, np.array(lengths, np.int32), 7)[0]
    assert err < 1e-4, err


# Middle ranks exchange halos with both neighbours (world > 2).
@pytest.mark.parametrize("world,T,context,lengths", [
    (3, 120, (4, 1, True), [120, 33]),
    (4, 600, (128, 128, False), [600, 421]),
])
def test_middle_ranks_with_halo_match_single_device_forward(world, T, context, lengths):
    err = _spawn(_shard_forward, world, T, 2, 64, 2, context, np.array(lengths, np.int32), 11)[0]
    assert err < 1e-4, err
