"""The bounded-wait failure path on the device, without a fault: a kernel
waits on an mbarrier that nothing arrives on, gives up at its deadline and
records an error in the context's device word; nrp_context_check reports
NRP_ERR_DEVICE once and clears it, and the same context then runs a forward
whose output matches a second context's bit for bit."""
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
    return load_package()


def _forward(nrp, ctx, w, x, pos, D, H):
    attn = nrp.RelPositionMultiHeadAttention(D, H, True, ctx=ctx)
    for which, (wk, bk) in zip((nrp.LINEAR_Q, nrp.LINEAR_K, nrp.LINEAR_V, nrp.LINEAR_OUT,
                                nrp.LINEAR_POS),
                               (("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo"),
                                ("wp", None))):
        attn.set_linear(which, nrp.LinearLayer.standard(w[wk], w[bk] if bk else None))
    attn.set_pos_bias(w["pos_bias_u"], w["pos_bias_v"])
    attn.set_dtype(nrp.BF16)
    return attn.forward(x, pos, None, None)


def test_expired_wait_is_reported_once_and_context_stays_usable(nrp):
    import torch
    ctx = nrp.Context(0)
    ctx.check()
    ctx.selftest_wait_expiry(20000)  # 20 ms
    with pytest.raises(nrp.NrpError) as e:
        ctx.check()
    assert e.value.code == nrp.NRP_ERR_DEVICE
    ctx.check()  # cleared
    with pytest.raises(nrp.NrpError):
        ctx.selftest_wait_expiry(0)  # outside [1, 10^6] us
    D, H, T = 256, 2, 70
    rng = np.random.default_rng(3)
    w = rand_weights(rng, D, H)
    x = torch.from_numpy(rng.standard_normal((1, T, D)).astype(np.float32)).cuda().bfloat16()
    pe = nrp.RelPositionalEncoding(D, 5000, True, device=0)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    got = _forward(nrp, ctx, w, x, pos, D, H)
    ctx.check()
    other = nrp.Context(0)
    ref = _forward(nrp, other, w, x, pos, D, H)
    other.check()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
