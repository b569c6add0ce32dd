"""copy_frames: the valid frames of each utterance, one copy per utterance,
padded frames untouched (the host side of a serving loop that moves only
valid frames across PCIe).  CPU tensors."""
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
