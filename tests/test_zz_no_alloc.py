"""nrp_attn_forward_noalloc: the rel-pos MHA forward for callers that cannot
let the library allocate device memory (for instance an audio thread with a
real-time deadline, which cannot wait on cudaMalloc's device synchronisation,
or a process whose device memory belongs to another runtime's allocator).

Its intermediates live in a fixed 32 MiB array in the library's device
memory instead of buffers grown with cudaMalloc.  These tests call it
through the C ABI and check it against nrp_attn_forward, the allocating
entry point, on two calls in a row (the second call reuses the array the
first one left behind).  Both run the same kernels on the same inputs, so
the valid rows must be bit-identical: full context, a (128, 128) window,
and 8-bit weights (the bf16 copies the allocating forward kept at >= 256
rows, and the GEMV at <= 16 rows).  They also check that the second call
changes the device's free memory by nothing, the size limit, and that it
refuses to run before the module's parameters are on the device.

This file is collected last so that a run stopping at the first failure has
run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rand_weights
from __graft_entry__ import load_package

pytestmark = pytest.mark.gpu


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


LINEARS = (("linear_q", "wq", "bq"), ("linear_k", "wk", "bk"), ("linear_v", "wv", "bv"),
           ("linear_out", "wo", "bo"), ("linear_pos", "wp", None))


def _module(nrp, orc, D, H, dtype, seed, quant=False):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, D, H)
    attn = nrp.RelPositionMultiHeadAttention(D, H, True)
    if quant:
        wd = {}
        for name, wk, bk in LINEARS:
            wq, s, z = orc.quantize(w[wk], 64, 8)
            wd[f"l.{name}.weight"], wd[f"l.{name}.scales"], wd[f"l.{name}.biases"] = wq, s, z
            if bk:
                wd[f"l.{name}.bias"] = w[bk]
        wd["l.pos_bias_u"], wd["l.pos_bias_v"] = w["pos_bias_u"], w["pos_bias_v"]
        attn.load_weights(wd, "l", nrp.QuantizationConfig(8, 64))
    else:
        for which, (_, wk, bk) in enumerate(LINEARS):
            attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
        attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(dtype)
    return attn, rng


def _noalloc(nrp, attn, x, pos, lengths, context, out):
    B, T, _ = x.shape
    cs = None
    if context is not None:
        cs = nrp._AttCtx(context[0], context[1], int(context[2]))
    return nrp.lib().nrp_attn_forward_noalloc(
        attn.handle, nrp._stream(), x.data_ptr(), B, T, pos.data_ptr(),
        lengths.data_ptr() if lengths is not None else None,
        C.addressof(cs) if cs is not None else None, out.data_ptr())


@pytest.mark.parametrize("dtype_name,D,H,B,T,lengths,context,quant", [
    ("bf16", 1024, 8, 3, 300, [300, 171, 245], None, False),
    ("f32", 256, 2, 3, 300, [300, 171, 245], None, False),
    ("bf16", 1024, 8, 2, 600, [600, 433], (128, 128, False), False),
    ("bf16", 1024, 8, 3, 300, [300, 171, 245], None, True),
    ("bf16", 1024, 8, 1, 12, None, None, True),
])
def test_noalloc_equals_forward_on_two_calls(nrp, orc, dtype_name, D, H, B, T, lengths,
                                             context, quant):
    import torch
    dtype = nrp.BF16 if dtype_name == "bf16" else nrp.F32
    tdt = torch.bfloat16 if dtype == nrp.BF16 else torch.float32
    attn, rng = _module(nrp, orc, D, H, dtype, seed=21 + T, quant=quant)
    lengths_h = np.array(lengths if lengths else [T] * B, np.int32)
    mask = nrp.key_padding_mask(lengths_h, T) if lengths else None
    ctx = nrp.AttentionContext.new(context[:2], "chunked_limited" if context[2] else "regular") \
        if context else None
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(dtype)
    pos = pe.get_encoding(T)
    xs = [torch.from_numpy(rng.standard_normal((B, T, D)).astype(np.float32)).to("cuda", tdt)
          for _ in range(2)]
    refs = [attn.forward(x, pos, ctx, mask) for x in xs]  # the allocating entry point
    outs = [torch.full_like(x, float("nan")) for x in xs]
    attn.ctx.check()
    torch.cuda.synchronize()
    for call in range(2):
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(nrp, attn, xs[call], pos, mask.lengths if mask else None, context,
                      outs[call])
        assert rc == 0, nrp.lib().nrp_last_error()
        torch.cuda.synchronize()
        if call == 1:  # nothing allocated (nor a module loaded) by a call
            assert torch.cuda.mem_get_info()[0] == free_before
        attn.ctx.check()
        for b, L in enumerate(lengths_h):
            assert torch.equal(outs[call][b, :L], refs[call][b, :L]), (call, b)
        assert torch.isfinite(outs[call].float()).all()


def test_noalloc_rejects_sizes_beyond_its_scratch(nrp, orc):
    import torch
    attn, _ = _module(nrp, orc, 1024, 8, nrp.BF16, seed=5)
    pe = nrp.RelPositionalEncoding(1024, 5000, True)
    pe.set_dtype(nrp.BF16)
    small = torch.zeros((1, 16, 1024), dtype=torch.bfloat16, device="cuda")
    attn.forward(small, pe.get_encoding(16))  # makes the parameters resident
    T = 2000  # 2 x 2000 frames need ~39 MB of intermediates, more than 32 MiB
    x = torch.zeros((2, T, 1024), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    rc = _noalloc(nrp, attn, x, pe.get_encoding(T), None, None, out)
    assert rc == nrp.NRP_ERR_INVALID
    assert b"static scratch" in nrp.lib().nrp_last_error()
    # with a (128, 128) window only 257 positions are projected: 2 x 1900
    # frames fit (29.7 MB + 0.5 MB), where the 3799 positions of full context
    # would not (+7.4 MB)
    T = 1900
    x = torch.zeros((2, T, 1024), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    pos = pe.get_encoding(T)
    assert _noalloc(nrp, attn, x, pos, None, None, out) == nrp.NRP_ERR_INVALID
    assert _noalloc(nrp, attn, x, pos, None, (128, 128, False), out) == 0, \
        nrp.lib().nrp_last_error()
    attn.ctx.check()


def test_noalloc_needs_parameters_on_the_device(nrp, orc):
    import torch
    attn, _ = _module(nrp, orc, 256, 2, nrp.BF16, seed=6)
    pe = nrp.RelPositionalEncoding(256, 5000, True)
    pe.set_dtype(nrp.BF16)
    x = torch.zeros((1, 8, 256), dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    rc = _noalloc(nrp, attn, x, pe.get_encoding(8), None, None, out)
    assert rc == nrp.NRP_ERR_INVALID
    assert b"parameters" in nrp.lib().nrp_last_error()
