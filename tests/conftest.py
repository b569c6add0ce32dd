"""Shared test setup: markers, import paths, seeded inputs."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.lib()
    return o


def rand_weights(rng, d_model, n_heads, scale=0.02, use_bias=True, out_bias=True):
    """Seeded rel-pos MHA parameters (N(0, scale^2)), the shapes of
    RelPositionMultiHeadAttention::new (attention.rs:367-406)."""
    dh = d_model // n_heads
    f = lambda *s: (rng.standard_normal(s) * scale).astype(np.float32)
    w = {
        "wq": f(d_model, d_model), "wk": f(d_model, d_model),
        "wv": f(d_model, d_model), "wo": f(d_model, d_model),
        "wp": f(d_model, d_model),
        "pos_bias_u": f(n_heads, dh), "pos_bias_v": f(n_heads, dh),
    }
    for name in ("bq", "bk", "bv"):
        w[name] = f(d_model) if use_bias else None
    w["bo"] = f(d_model) if (use_bias and out_bias) else None
    return w


# ------------------------------------------------------- conformer block
BLOCK_LIN_KEYS = {"ff1_1": "feed_forward1.linear1", "ff1_2": "feed_forward1.linear2",
                  "pw1": "conv.pointwise_conv1", "pw2": "conv.pointwise_conv2",
                  "ff2_1": "feed_forward2.linear1", "ff2_2": "feed_forward2.linear2"}
BLOCK_NORM_KEYS = {"ff1": "norm_feed_forward1", "att": "norm_self_att", "conv": "norm_conv",
                   "ff2": "norm_feed_forward2", "out": "norm_out"}
ATTN_LIN_KEYS = {"wq": ("linear_q", "bq"), "wk": ("linear_k", "bk"), "wv": ("linear_v", "bv"),
                 "wo": ("linear_out", "bo"), "wp": ("linear_pos", None)}


def rand_block(rng, D, H, ff, K, conv_norm="batch_norm", quant=False, orc=None, prefix="b",
               scale=None):
    """One Conformer block's parameters as (oracle dict for
    oracle.block_forward, NeMo-named weight dict for ConformerBlock.load_weights,
    conformer.rs:1978-2028).  Linears ~ N(0, 1/fan_in) unless `scale` is given,
    so that every branch moves the output.  quant: every linear MLX 8-bit,
    group 64, with fp16 scales/biases (the oracle gets the dequantised
    weights from their bf16-rounded values, as the device does)."""
    g = lambda sd, *s: (rng.standard_normal(s) * sd).astype(np.float32)
    shapes = {"ff1_1": (ff, D), "ff1_2": (D, ff), "pw1": (2 * D, D), "pw2": (D, D),
              "ff2_1": (ff, D), "ff2_2": (D, ff)}
    bw, wd = {}, {}

    def add_linear(key, w, b):
        if quant:
            wq, s, z = orc.quantize(w, 64, 8)
            s = s.astype(np.float16).astype(np.float32)
            z = z.astype(np.float16).astype(np.float32)
            wd[f"{key}.weight"], wd[f"{key}.scales"], wd[f"{key}.biases"] = wq, s, z
            w = orc.dequantize(wq, orc.bf16_round(s), orc.bf16_round(z), 64, 8)
        else:
            wd[f"{key}.weight"] = w
        if b is not None:
            wd[f"{key}.bias"] = b
        return w

    for name, (n, k) in shapes.items():
        w = g(scale or 1 / np.sqrt(k), n, k)
        b = g(0.1 if scale is None else scale, n)
        bw[name] = (add_linear(f"{prefix}.{BLOCK_LIN_KEYS[name]}", w, b), b)
    dw_w = g(scale or 1 / np.sqrt(K), D, K)
    dw_b = g(0.1 if scale is None else scale, D)
    wd[f"{prefix}.conv.depthwise_conv.weight"] = dw_w.reshape(D, K, 1)
    wd[f"{prefix}.conv.depthwise_conv.bias"] = dw_b
    bw["dw"] = (dw_w, dw_b)
    sd = 0.1 if scale is None else scale
    cg, cb = 1 + g(sd, D), g(sd, D)
    cm, cv = (g(sd, D), 1 + np.abs(g(2 * sd, D))) if conv_norm == "batch_norm" else (None, None)
    bn = f"{prefix}.conv.batch_norm"
    wd[f"{bn}.weight"], wd[f"{bn}.bias"] = cg, cb
    if cm is not None:
        wd[f"{bn}.running_mean"], wd[f"{bn}.running_var"] = cm, cv
    bw["conv_norm"] = (cg, cb, cm, cv)
    bw["norms"] = {}
    for name, key in BLOCK_NORM_KEYS.items():
        ng_, nb_ = 1 + g(sd, D), g(sd, D)
        bw["norms"][name] = (ng_, nb_)
        wd[f"{prefix}.{key}.weight"], wd[f"{prefix}.{key}.bias"] = ng_, nb_
    attn = rand_weights(rng, D, H, scale=scale or 1 / np.sqrt(D))
    for wk, (name, bk) in ATTN_LIN_KEYS.items():
        key = f"{prefix}.self_attn.{name}"
        attn[wk] = add_linear(key, attn[wk], attn[bk] if bk else None)
    wd[f"{prefix}.self_attn.pos_bias_u"] = attn["pos_bias_u"]
    wd[f"{prefix}.self_attn.pos_bias_v"] = attn["pos_bias_v"]
    bw["attn"] = attn
    return bw, wd
