"""nrp_attn_forward_noalloc: the rel-pos MHA forward for callers that cannot
let the library allocate device memory (for instance an audio thread with a
real-time deadline, which cannot wait on cudaMalloc's device synchronisation,
or a process whose device memory belongs to another runtime's allocator).

Its intermediates live in a fixed 32 MiB array in the library's device
memory instead of buffers grown with cudaMalloc.  These tests call it
through the C ABI and check it against nrp_attn_forward, the allocating
entry point, on two calls in a row (the second call reuses the array the
first one left behind); they also check its size limit and that it refuses
to run before the module's parameters are on the device.

This file is collected last so that a run stopping at the first failure has
run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rand_weights
from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu

TOL = {0: 1e-4, 1: 2e-2}  # f32, bf16: the parity tolerances of test_gpu_parity.py


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    m = load_package()
    f = m.lib().nrp_attn_forward_noalloc
    f.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int] + [C.c_void_p] * 4
    f.restype = C.c_int
    return m


def _module(nrp, D, H, dtype, seed):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, D, H)
    attn = nrp.RelPositionMultiHeadAttention(D, H, True)
    for which, (wk, bk) in enumerate((("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo"),
                                      ("wp", None))):
        attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(dtype)
    return attn, rng


def _noalloc(nrp, attn, x, pos, lengths, out):
    B, T, _ = x.shape
    return nrp.lib().nrp_attn_forward_noalloc(
        attn.handle, nrp._stream(), x.data_ptr(), B, T, pos.data_ptr(),
        lengths.data_ptr() if lengths is not None else None, None, out.data_ptr())


@pytest.mark.parametrize("dtype_name,D,H", [("bf16", 1024, 8), ("f32", 256, 2)])
def test_noalloc_matches_forward_on_two_calls(nrp, dtype_name, D, H):
    import torch
    dtype = nrp.BF16 if dtype_name == "bf16" else nrp.F32
    tdt = torch.bfloat16 if dtype == nrp.BF16 else torch.float32
    attn, rng = _module(nrp, D, H, dtype, seed=21)
    B, T = 3, 300
    lengths_h = np.array([300, 171, 245], np.int32)
    mask = nrp.key_padding_mask(lengths_h, T)
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(dtype)
    pos = pe.get_encoding(T)
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).to("cuda", tdt)
        ref = attn.forward(x, pos, None, mask)  # the allocating entry point
        out = torch.full_like(x, float("nan"))
        assert _noalloc(nrp, attn, x, pos, mask.lengths, out) == 0, nrp.lib().nrp_last_error()
        attn.ctx.check()
        got = out.float().cpu().numpy()
        want = ref.float().cpu().numpy()
        for b, L in enumerate(lengths_h):
            err = np.abs(got[b, :L] - want[b, :L]).max() / np.abs(want[b, :L]).max()
            assert err < TOL[dtype], (call, b, err)
        assert np.isfinite(got).all()


def test_noalloc_rejects_sizes_beyond_its_scratch(nrp):
    import torch
    attn, _ = _module(nrp, 1024, 8, nrp.BF16, seed=5)
    pe = nrp.RelPositionalEncoding(1024, 5000, True)
    pe.set_dtype(nrp.BF16)
    small = torch.zeros((1, 16, 1024), dtype=torch.bfloat16, device="cuda")
    attn.forward(small, pe.get_encoding(16))  # makes the parameters resident
    T = 2000  # 2 x 2000 frames need ~39 MB of intermediates, more than 32 MiB
    x = torch.zeros((2, T, 1024), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    rc = _noalloc(nrp, attn, x, pe.get_encoding(T), None, out)
    assert rc == nrp.NRP_ERR_INVALID
    assert b"static scratch" in nrp.lib().nrp_last_error()


def test_noalloc_needs_parameters_on_the_device(nrp):
    import torch
    attn, _ = _module(nrp, 256, 2, nrp.BF16, seed=6)
    pe = nrp.RelPositionalEncoding(256, 5000, True)
    pe.set_dtype(nrp.BF16)
    x = torch.zeros((1, 8, 256), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    rc = _noalloc(nrp, attn, x, pe.get_encoding(8), None, out)
    assert rc == nrp.NRP_ERR_INVALID
    assert b"parameters" in nrp.lib().nrp_last_error()
