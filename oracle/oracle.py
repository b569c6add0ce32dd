"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module;
the product library never does.  Every function restates the reference
(animaslabs/mlx-nemo-rs) at the file:line cited in relpos_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

ORC_DIRECT = 0
ORC_REFERENCE_ALGO = 1
MAX_SCORE_ELEMENTS = 1 << 26  # attention.rs:198


class _Weights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "wp",
                 "pos_bias_u", "pos_bias_v")]


class _Lin(C.Structure):
    _fields_ = [("w", C.c_void_p), ("b", C.c_void_p)]


class _BlockWeights(C.Structure):
    _fields_ = ([(n, _Lin) for n in ("ff1_1", "ff1_2", "pw1", "pw2", "ff2_1", "ff2_2")] +
                [(n, C.c_void_p) for n in ("dw_w", "dw_b", "cn_g", "cn_b", "cn_m", "cn_v")] +
                [("norm_g", C.c_void_p * 5), ("norm_b", C.c_void_p * 5), ("attn", _Weights)])


class _Ctx(C.Structure):
    _fields_ = [("has", C.c_int), ("left", C.c_int), ("right", C.c_int),
                ("chunked", C.c_int)]


def build():
    """Compile liboracle.so in place (make)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.orc_create_pe.argtypes = [C.c_int, C.c_int, _f32p]
        L.orc_get_encoding.argtypes = [C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_get_encoding.restype = C.c_int
        L.orc_rel_shift.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_block_mask.argtypes = [C.c_int] * 6 + [_u8p]
        L.orc_query_block_size.argtypes = [C.c_int, C.c_int, C.c_int64]
        L.orc_query_block_size.restype = C.c_int
        L.orc_create_attention_mask.argtypes = [C.c_int] * 8 + [_u8p]
        L.orc_linear.argtypes = [_f32p, C.c_int, C.c_int, _f32p, C.c_int,
                                 C.c_void_p, _f32p]
        L.orc_dequantize.argtypes = [_u32p, _f32p, _f32p, C.c_int, C.c_int,
                                     C.c_int, C.c_int, _f32p]
        L.orc_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   _u32p, _f32p, _f32p]
        L.orc_mha_forward.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.POINTER(_Weights), _f32p, C.c_void_p,
                                      C.c_void_p, C.c_int, C.c_int, C.c_int64,
                                      _f32p]
        L.orc_mha_forward.restype = C.c_int
        L.orc_relpos_attention.argtypes = [
            _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int,
            C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
            C.c_int, _f32p]
        L.orc_stream_layer_step.argtypes = [
            _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_Weights),
            _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
            C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_stream_layer_step.restype = C.c_int
        L.orc_block_forward.argtypes = [
            _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
            C.POINTER(_BlockWeights), _f32p, C.c_void_p, C.c_void_p, C.c_int, _f32p]
        L.orc_block_forward.restype = C.c_int
        L.orc_bf16_round_array.argtypes = [_f32p, C.c_int64]
        L.orc_subsampling_forward.argtypes = [_f32p] + [C.c_int] * 7 + [C.c_void_p, C.c_int,
                                                                         _f32p]
        L.orc_subsampling_forward.restype = C.c_int
        L.orc_stream_block_step.argtypes = (
            [_f32p] + [C.c_int] * 7 + [C.c_void_p, _f32p, _f32p, C.c_int, _f32p] +
            [C.c_int] * 7 + [_f32p])
        L.orc_stream_block_step.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _LIB = L
    return _LIB


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int):
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return lib().orc_get_threads()


def bf16_round(a):
    a = _f32(a).copy()
    lib().orc_bf16_round_array(a, a.size)
    return a


def create_pe(d_model, max_len):
    out = np.empty((2 * max_len - 1, d_model), np.float32)
    lib().orc_create_pe(d_model, max_len, out)
    return out


def get_encoding(d_model, max_len, seq_len):
    if seq_len <= 0:
        raise ValueError("positional encoding requested for an empty sequence")
    out = np.empty((2 * seq_len - 1, d_model), np.float32)
    rc = lib().orc_get_encoding(d_model, max_len, seq_len, out)
    assert rc == 0
    return out


def rel_shift(x):
    x = _f32(x)
    *lead, s, p = x.shape
    bh = int(np.prod(lead)) if lead else 1
    out = np.empty_like(x)
    lib().orc_rel_shift(x, bh, s, p, out)
    return out


def block_mask(left, right, chunked, start, end, seq_len):
    out = np.empty((end - start, seq_len), np.uint8)
    lib().orc_block_mask(left, right, int(chunked), start, end, seq_len, out)
    return out.astype(bool)


def query_block_size(batch_heads, seq_len, budget):
    return lib().orc_query_block_size(batch_heads, seq_len, budget)


def create_attention_mask(left, right, chunked, max_audio_length, cache_len,
                          filled, tensor_seq_len, valid_seq_len):
    out = np.empty((tensor_seq_len, max_audio_length), np.uint8)
    lib().orc_create_attention_mask(left, right, int(chunked), max_audio_length,
                                    cache_len, filled, tensor_seq_len,
                                    valid_seq_len, out)
    return out.astype(bool)


def linear(x, w, bias=None):
    x = _f32(x)
    w = _f32(w)
    lead = x.shape[:-1]
    K = x.shape[-1]
    N = w.shape[0]
    M = int(np.prod(lead)) if lead else 1
    y = np.empty((M, N), np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_linear(x.reshape(M, K), M, K, w, N,
                     b.ctypes.data if b is not None else None, y)
    return y.reshape(*lead, N)


def dequantize(wq, scales, biases, group_size=64, bits=8):
    wq = np.ascontiguousarray(wq, np.uint32)
    N = wq.shape[0]
    K = wq.shape[1] * (32 // bits)
    out = np.empty((N, K), np.float32)
    lib().orc_dequantize(wq, _f32(scales), _f32(biases), N, K, group_size, bits,
                         out)
    return out


def quantize(w, group_size=64, bits=8):
    w = _f32(w)
    N, K = w.shape
    wq = np.empty((N, K // (32 // bits)), np.uint32)
    s = np.empty((N, K // group_size), np.float32)
    b = np.empty((N, K // group_size), np.float32)
    lib().orc_quantize(w, N, K, group_size, bits, wq, s, b)
    return wq, s, b


def _weights_struct(w, keep):
    st = _Weights()
    for name in ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "wp",
                 "pos_bias_u", "pos_bias_v"):
        a = w.get(name)
        if a is None:
            setattr(st, name, None)
        else:
            a = _f32(a)
            keep.append(a)
            setattr(st, name, a.ctypes.data)
    return st


def _ctx_struct(context):
    if context is None:
        return None
    left, right, chunked = context
    return _Ctx(1, int(left), int(right), int(chunked))


def mha_forward(x, w, pos_emb, n_heads, lengths=None, context=None,
                mode=ORC_DIRECT, bf16=False, max_score_elements=MAX_SCORE_ELEMENTS):
    """RelPositionMultiHeadAttention::forward (attention.rs:446-573).

    w: dict with wq,bq,wk,bk,wv,bv,wo,bo,wp,pos_bias_u,pos_bias_v (float32,
    weights [out,in]); context: (left, right, chunked) or None."""
    x = _f32(x)
    B, T, D = x.shape
    keep = []
    st = _weights_struct(w, keep)
    out = np.empty_like(x)
    ln = np.ascontiguousarray(lengths, np.int32) if lengths is not None else None
    cs = _ctx_struct(context)
    rc = lib().orc_mha_forward(
        x, B, T, D, n_heads, C.byref(st), _f32(pos_emb),
        ln.ctypes.data if ln is not None else None,
        C.cast(C.pointer(cs), C.c_void_p) if cs is not None else None,
        mode, int(bool(bf16)), int(max_score_elements), out)
    assert rc == 0
    return out


def relpos_attention(q, k, v, p, u, vb, n_heads, vis=None, key_len=None,
                     context=None, q_offset=0):
    """Attention core on projected tensors; rows with no visible key are 0."""
    q, k, v, p = _f32(q), _f32(k), _f32(v), _f32(p)
    B, Tq, D = q.shape
    Tk = k.shape[1]
    out = np.empty_like(q)
    vis_a = np.ascontiguousarray(vis, np.uint8) if vis is not None else None
    kl = np.ascontiguousarray(key_len, np.int32) if key_len is not None else None
    cs = _ctx_struct(context)
    lib().orc_relpos_attention(
        q, k, v, p, _f32(u), _f32(vb), B, Tq, Tk, D, n_heads,
        vis_a.ctypes.data if vis_a is not None else None,
        kl.ctypes.data if kl is not None else None,
        C.cast(C.pointer(cs), C.c_void_p) if cs is not None else None,
        q_offset, out)
    return out


def stream_layer_step(x, w, pos_emb, n_heads, h_cache, filled, valid, left,
                      right, chunked, cache_drop_size=0, bf16=False):
    """One attention layer of ConformerEncoder::forward_streaming
    (conformer.rs:883-1037).  h_cache [B,C,D] is updated in place; returns
    (out, next_filled)."""
    x = _f32(x)
    B, T, D = x.shape
    assert h_cache.dtype == np.float32 and h_cache.flags["C_CONTIGUOUS"]
    Cc = h_cache.shape[1]
    keep = []
    st = _weights_struct(w, keep)
    out = np.empty_like(x)
    nxt = lib().orc_stream_layer_step(
        x, B, T, D, n_heads, C.byref(st), _f32(pos_emb), h_cache, Cc, filled,
        valid, left, right, int(chunked), cache_drop_size, int(bool(bf16)), out)
    return out, nxt


BLOCK_LINEARS = ("ff1_1", "ff1_2", "pw1", "pw2", "ff2_1", "ff2_2")
BLOCK_NORMS = ("ff1", "att", "conv", "ff2", "out")


def _block_struct(bw, D, kernel, keep):
    def ptr(a):
        if a is None:
            return None
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    st = _BlockWeights()
    for name in BLOCK_LINEARS:
        w, b = bw[name]
        setattr(st, name, _Lin(ptr(w), ptr(b)))
    st.dw_w, st.dw_b = ptr(np.asarray(bw["dw"][0]).reshape(D, kernel)), ptr(bw["dw"][1])
    g, b, m, v = bw["conv_norm"]
    st.cn_g, st.cn_b, st.cn_m, st.cn_v = ptr(g), ptr(b), ptr(m), ptr(v)
    for i, name in enumerate(BLOCK_NORMS):
        st.norm_g[i] = ptr(bw["norms"][name][0])
        st.norm_b[i] = ptr(bw["norms"][name][1])
    st.attn = _weights_struct(bw["attn"], keep)
    return st


def stream_block_step(x, bw, pos_emb, n_heads, ff_dim, kernel, h_cache, conv_cache, filled,
                      valid, left=-1, right=-1, chunked=False, cache_drop_size=0, conv_norm=0,
                      bf16=True):
    """ConformerBlock::forward_with_cache (conformer.rs:1877-1967) as
    forward_streaming drives it.  h_cache [B,C,D] and conv_cache [B,K-1,D]
    (f32, C-contiguous) are updated in place; returns (out, next_filled)."""
    x = _f32(x)
    B, T, D = x.shape
    assert h_cache.dtype == np.float32 and h_cache.flags["C_CONTIGUOUS"]
    assert conv_cache.dtype == np.float32 and conv_cache.flags["C_CONTIGUOUS"]
    assert conv_cache.shape == (B, kernel - 1, D)
    keep = []
    st = _block_struct(bw, D, kernel, keep)
    out = np.empty_like(x)
    nxt = lib().orc_stream_block_step(
        x, B, T, D, n_heads, ff_dim, kernel, int(conv_norm), C.byref(st), _f32(pos_emb),
        h_cache, h_cache.shape[1], conv_cache, filled, valid, left, right, int(bool(chunked)),
        cache_drop_size, int(bool(bf16)), out)
    assert nxt >= 0
    return out, nxt


def block_forward(x, bw, pos_emb, n_heads, ff_dim, kernel, causal=False, conv_norm=0,
                  lengths=None, context=None, bf16=True):
    """ConformerBlock::forward (conformer.rs:1693-1870).

    bw: {"ff1_1": (w, b), ... (BLOCK_LINEARS, f32 weights [out, in]; a
    quantised layer gives its dequantised weights), "dw": (w [D, K], b),
    "conv_norm": (gamma, beta, mean, var) (mean/var None for a layer norm),
    "norms": {name: (gamma, beta)} for BLOCK_NORMS, "attn": the mha_forward
    weight dict}."""
    x = _f32(x)
    B, T, D = x.shape
    keep = []
    st = _block_struct(bw, D, kernel, keep)
    ln = np.ascontiguousarray(lengths, np.int32) if lengths is not None else None
    cs = _ctx_struct(context)
    out = np.empty_like(x)
    rc = lib().orc_block_forward(
        x, B, T, D, n_heads, ff_dim, kernel, int(bool(causal)), int(conv_norm), C.byref(st),
        _f32(pos_emb), ln.ctypes.data if ln is not None else None,
        C.cast(C.pointer(cs), C.c_void_p) if cs is not None else None, int(bool(bf16)), out)
    assert rc == 0
    return out


class _SubWeights(C.Structure):
    _fields_ = [("conv0_w", C.c_void_p), ("conv0_b", C.c_void_p),
                ("dw_w", C.c_void_p * 2), ("dw_b", C.c_void_p * 2),
                ("pw_w", C.c_void_p * 2), ("pw_b", C.c_void_p * 2),
                ("out_w", C.c_void_p), ("out_b", C.c_void_p)]


def subsampling_strides(factor):
    return lib().orc_subsampling_strides(int(factor))


def subsampling_out_len(length, factor, causal):
    """Subsampling::output_length (conformer.rs:1315-1327)."""
    return lib().orc_subsampling_out_len(int(length), int(factor), int(bool(causal)))


def subsampling_feat_out(feat_in, factor, causal):
    """compute_freq_output_size (conformer.rs:1220-1244)."""
    return lib().orc_subsampling_feat_out(int(feat_in), int(factor), int(bool(causal)))


def subsampling_forward(x, sw, d_model, factor=8, causal=False, bf16=True):
    """Subsampling::forward_frames (conformer.rs:1413-1555) on x [B, T, F].

    sw: {"conv0": (w [C, 3, 3, 1], b), "dw": [(w [C, 3, 3, 1], b), ...],
    "pw": [(w [C, 1, 1, C], b), ...], "out": (w [d_model, C * F'], b)}
    (MLX layouts; biases may be None)."""
    x = _f32(x)
    B, T, F = x.shape
    Cc = np.asarray(sw["conv0"][0]).shape[0]
    keep = []

    def ptr(a):
        if a is None:
            return None
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    st = _SubWeights()
    st.conv0_w, st.conv0_b = ptr(sw["conv0"][0]), ptr(sw["conv0"][1])
    for i, ((dw, db), (pw, pb)) in enumerate(zip(sw.get("dw", []), sw.get("pw", []))):
        st.dw_w[i], st.dw_b[i] = ptr(dw), ptr(db)
        st.pw_w[i], st.pw_b[i] = ptr(pw), ptr(pb)
    st.out_w, st.out_b = ptr(sw["out"][0]), ptr(sw["out"][1])
    Tp = subsampling_out_len(T, factor, causal)
    out = np.empty((B, Tp, d_model), np.float32)
    rc = lib().orc_subsampling_forward(x, B, T, F, Cc, int(factor), int(bool(causal)),
                                       int(d_model), C.byref(st), int(bool(bf16)), out)
    assert rc == 0
    return out
