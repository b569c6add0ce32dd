"""The CTA-pair GEMM (two SMs share 256 x 256 tiles through cta_group::2
MMAs), which the bf16 linears take from 128 row tiles on, at its edges:

- a flat linear with an odd number of 128-row tiles (the last pair's second
  CTA has no rows: it loads zeros and writes nothing) against a float32
  product of the same bf16 operands (tolerance 1e-2 of the output scale,
  and the per-element bound of tests/test_gpu_parity.py);
- config 3's batch shape (B = 32, T = 500, lengths U[250, 500]: per-utterance
  row tiles, 128 of them, with tiles past each utterance's length that only
  write zeros) through two 8-bit Conformer layers, whose linears run the
  SiLU, GLU and residual epilogues on pairs; three utterances are checked
  against the oracle block by block (bf16 tolerance 2e-2).
"""
import numpy as np
import pytest

from conftest import rand_block
from __graft_entry__ import load_package
from test_gpu_parity import check_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nrp():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_package()


def test_flat_linear_odd_row_tiles(nrp):
    import torch
    M, K, N = 129 * 128 - 5, 1024, 512  # 129 row tiles, the last one ragged
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).bfloat16()
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).bfloat16()
    y = nrp.linear(x, w, b)
    ref = (x.float() @ w.float().t() + b.float()).cpu().numpy()
    check_close(y.float().cpu().numpy()[None], ref[None], None, 1e-2)


def test_encoder_layers_config3_batch(nrp, orc):
    import torch
    L, D, H, ff, K = 2, 1024, 8, 4096, 9
    B, T = 32, 500
    rng = np.random.default_rng(32)
    lengths = rng.integers(250, T + 1, B).astype(np.int32)
    lengths[0] = T
    seeds = [4100 + i for i in range(L)]
    enc = nrp.ConformerEncoder(L, D, H, ff, K)
    wd = {}
    for i, sd in enumerate(seeds):
        _, w = rand_block(np.random.default_rng(sd), D, H, ff, K, quant=True, orc=orc,
                          prefix=f"encoder.layers.{i}", scale=0.02)
        wd.update(w)
    enc.load_weights(wd, nrp.QuantizationConfig(8, 64))
    del wd
    enc.set_dtype(nrp.BF16)
    x = np.random.default_rng(7).standard_normal((B, T, D)).astype(np.float32)
    xd = torch.from_numpy(x).cuda().bfloat16()
    pe = nrp.RelPositionalEncoding(D, 5000, True)
    pe.set_dtype(nrp.BF16)
    pos = pe.get_encoding(T)
    mask = nrp.key_padding_mask(lengths, T)
    h = (xd.float() * np.float32(np.sqrt(D))).bfloat16()
    inputs = []
    for blk in enc.layers:  # the whole batch per block: 128 row tiles per linear
        inputs.append(h)
        h = blk.forward(h, pos, None, mask)
    enc.ctx.check()
    outs = inputs[1:] + [h]
    pe_h = orc.get_encoding(D, 5000, T)
    pick = [0, int(np.argmin(lengths)), B - 1]
    for i, sd in enumerate(seeds):
        bw, _ = rand_block(np.random.default_rng(sd), D, H, ff, K, quant=True, orc=orc,
                           prefix="b", scale=0.02)
        xin = inputs[i].float().cpu().numpy()[pick]
        ref = orc.block_forward(xin, bw, pe_h, H, ff, K, lengths=lengths[pick], bf16=True)
        got = outs[i].float().cpu().numpy()[pick]
        check_close(got, ref, lengths[pick], 2e-2)
