"""copy_frames: the valid frames of each utterance, one copy per utterance,
padded frames untouched (the host side of a serving loop that moves only
valid frames across PCIe); unpack_frames / pack_frames: the same frames
packed back to back on the host, one copy per direction plus a device
scatter or gather.  CPU tensors, except the GPU round trips."""
import numpy as np
import pytest

from __graft_entry__ import load_package


def test_copies_valid_frames_only():
    import torch
    nrp = load_package()
    rng = np.random.default_rng(3)
    B, T, D = 5, 9, 6
    src = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).bfloat16()
    dst = torch.full((B, T, D), 7.0, dtype=torch.bfloat16)
    lengths = np.array([9, 0, 4, 1, 12], np.int32)  # 12 clips to T
    n = nrp.copy_frames(dst, src, lengths, non_blocking=False)
    assert n == (9 + 0 + 4 + 1 + 9) * D * 2
    for b, L in enumerate(lengths):
        L = min(int(L), T)
        assert torch.equal(dst[b, :L], src[b, :L])
        assert bool((dst[b, L:] == 7.0).all())


def test_rejects_mismatched_tensors():
    import torch
    nrp = load_package()
    a = torch.zeros((2, 3, 4))
    with pytest.raises(ValueError):
        nrp.copy_frames(a, torch.zeros((2, 3, 5)), [3, 3])
    with pytest.raises(ValueError):
        nrp.copy_frames(a, torch.zeros((2, 3, 4)), [3])


@pytest.mark.gpu
def test_host_device_round_trip():
    """Pinned host -> device -> pinned host through nrp_copy_frames."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nrp = load_package()
    rng = np.random.default_rng(4)
    B, T, D = 4, 33, 256
    src = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).bfloat16()
    src = src.pin_memory()
    lengths = np.array([33, 7, 0, 20], np.int32)
    dev = torch.full((B, T, D), 3.0, dtype=torch.bfloat16, device="cuda")
    back = torch.full((B, T, D), 5.0, dtype=torch.bfloat16).pin_memory()
    n_in = nrp.copy_frames(dev, src, lengths)
    n_out = nrp.copy_frames(back, dev, lengths, non_blocking=False)
    assert n_in == n_out == int(lengths.sum()) * D * 2
    d = dev.cpu()
    for b, L in enumerate(lengths):
        assert torch.equal(back[b, :L], src[b, :L]) and torch.equal(d[b, :L], src[b, :L])
        assert bool((back[b, L:] == 5.0).all()) and bool((d[b, L:] == 3.0).all())


def _packed(src, lengths):
    import torch
    return torch.cat([src[b, :L] for b, L in enumerate(lengths)])


def test_pack_rejects_bad_arguments():
    """Python checks, then the C ABI's own (no device work is queued)."""
    import ctypes as C
    import torch
    nrp = load_package()
    pad = torch.zeros((2, 3, 4))
    with pytest.raises(ValueError):  # the padded side must live on the device
        nrp.unpack_frames(pad, torch.zeros((6, 4)), [3, 3])
    ln = np.array([2, 4], np.int32)  # 4 > T = 3
    buf = (C.c_uint8 * 64)()
    rc = nrp.lib().nrp_unpack_frames(C.addressof(buf), C.addressof(buf), ln.ctypes.data, 2, 3,
                                     8, None, None, None, None)
    assert rc == nrp.NRP_ERR_INVALID and b"lengths[1]" in nrp.lib().nrp_last_error()
    rc = nrp.lib().nrp_pack_frames(None, C.addressof(buf), ln.ctypes.data, 2, 3, 8, None, None,
                                   None)
    assert rc == nrp.NRP_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,D,dtype", [(4, 33, 256, "bf16"), (130, 5, 64, "f32"),
                                         (3, 17, 3, "bf16")])
def test_packed_round_trip(B, T, D, dtype):
    """Pinned host packed rows -> device [B, T, D] -> pinned host packed rows
    through nrp_unpack_frames / nrp_pack_frames (one link copy each way),
    the device-packed path, and the lengths written to a device array.
    (130 utterances: two launches; D = 3 bf16: 6-byte rows, the byte path.)"""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nrp = load_package()
    rng = np.random.default_rng(B)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    src = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).to(tdt)
    lengths = rng.integers(0, T + 1, B).astype(np.int32)
    lengths[0] = T
    packed = _packed(src, lengths).pin_memory()
    nb = packed.numel() * packed.element_size()
    staging = torch.empty(nb + 16, dtype=torch.uint8, device="cuda")
    dev = torch.full((B, T, D), 3.0, dtype=tdt, device="cuda")
    dev_len = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    assert nrp.unpack_frames(dev, packed, lengths, staging, dev_len) == nb
    back = torch.full_like(packed, 5.0).pin_memory()
    assert nrp.pack_frames(back, dev, lengths, staging) == nb
    torch.cuda.synchronize()
    d = dev.cpu()
    assert torch.equal(back, packed)
    assert np.array_equal(dev_len.cpu().numpy(), lengths)
    for b, L in enumerate(lengths):
        assert torch.equal(d[b, :L], src[b, :L]) and bool((d[b, L:] == 3.0).all())
    # packed rows already on the device: no staging
    dev2 = torch.zeros_like(dev)
    assert nrp.unpack_frames(dev2, packed.cuda(), lengths) == nb
    back2 = torch.empty_like(packed, device="cuda")
    assert nrp.pack_frames(back2, dev2, lengths) == nb
    assert torch.equal(back2.cpu(), packed)
