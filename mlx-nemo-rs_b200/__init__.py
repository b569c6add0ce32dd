"""B200 rel-pos MHA for FastConformer -- Python mirror of the reference API.

A thin ctypes layer over libnemo_relpos.so (include/nemo_relpos.h) whose
names, argument meanings and errors follow the `internals` API of
animaslabs/mlx-nemo-rs that the library replaces:

    src/asr/modules/encoders/attention.rs  RelPositionalEncoding,
        AttentionContext, key_padding_mask, RelPositionMultiHeadAttention
    src/core/quantization.rs               QuantizationConfig, LinearLayer
    src/asr/streaming/core.rs              EncoderCache, StreamingConfig,
        compute_streaming_config, StreamingModeInfo

Tensors are torch CUDA tensors (torch is the device-memory and stream
plumbing; every computation runs in the library's kernels).  There is no
CPU fallback: without the built library or a B200 the calls raise.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnemo_relpos.so")

NRP_OK = 0
NRP_ERR_INVALID = -1
NRP_ERR_CUDA = -2
NRP_ERR_UNSUPPORTED = -3
NRP_ERR_NOMEM = -4
NRP_ERR_DEVICE = -5

F32 = 0
BF16 = 1
LINEAR_Q, LINEAR_K, LINEAR_V, LINEAR_OUT, LINEAR_POS = range(5)
_LINEAR_NAMES = ("linear_q", "linear_k", "linear_v", "linear_out", "linear_pos")

MAX_SCORE_ELEMENTS = 1 << 26  # attention.rs:198 (no blocking is needed here)


class NrpError(RuntimeError):
    """Error from the library; `code` is the NRP_ERR_* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class _AttCtx(C.Structure):
    _fields_ = [("left", C.c_int32), ("right", C.c_int32), ("chunked", C.c_int32)]


class _SeqPlan(C.Structure):
    _fields_ = [("start", C.c_int32), ("len", C.c_int32), ("halo_left", C.c_int32),
                ("halo_right", C.c_int32), ("send_prev", C.c_int32), ("send_next", C.c_int32)]


class _StreamCfg(C.Structure):
    _fields_ = [("chunk_size", C.c_int32 * 2), ("shift_size", C.c_int32 * 2),
                ("cache_drop_size", C.c_int32), ("last_channel_cache_size", C.c_int32),
                ("last_time_cache_size", C.c_int32), ("valid_out_len", C.c_int32),
                ("pre_encode_cache_size", C.c_int32 * 2), ("drop_extra_pre_encoded", C.c_int32),
                ("lookahead_frames", C.c_int32), ("mode_idx", C.c_int32),
                ("left_context", C.c_int32), ("right_context", C.c_int32)]


_lib = None


def lib():
    """The loaded C library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NrpError(NRP_ERR_UNSUPPORTED,
                           f"{LIB_PATH} is missing: run python mlx-nemo-rs_b200/build.py")
        L = C.CDLL(LIB_PATH)
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        sig = {
            "nrp_abi_version": ([], i),
            "nrp_last_error": ([], C.c_char_p),
            "nrp_pe_encoding_host": ([i, i, i, vp], i),
            "nrp_pe_xscale": ([i, i], f),
            "nrp_att_context_new": ([i, i, C.c_char_p, vp], i),
            "nrp_block_mask_host": ([vp, i, i, i, vp], i),
            "nrp_key_padding_mask_host": ([vp, i, i, vp], i),
            "nrp_streaming_mask_host": ([vp, i, i, i, i, i, vp], i),
            "nrp_streaming_config_compute": ([i] * 9 + [vp], i),
            "nrp_context_create": ([i, vp], i),
            "nrp_context_destroy": ([vp], i),
            "nrp_context_check": ([vp, vp], i),
            "nrp_context_selftest_wait_expiry": ([vp, vp, i], i),
            "nrp_pe_encoding": ([vp, i, i, i, i, vp, vp], i),
            "nrp_attn_create": ([vp, i, i, i, vp], i),
            "nrp_attn_destroy": ([vp], i),
            "nrp_attn_set_dtype": ([vp, i], i),
            "nrp_attn_set_cache_drop_size": ([vp, i], i),
            "nrp_attn_load_linear": ([vp, i, vp, vp], i),
            "nrp_attn_load_linear_quantized": ([vp, i, i, i, vp, vp, vp, vp], i),
            "nrp_attn_load_pos_bias": ([vp, vp, vp], i),
            "nrp_attn_forward": ([vp, vp, vp, i, i, vp, vp, vp, vp], i),
            "nrp_attn_forward_noalloc": ([vp, vp, vp, i, i, vp, vp, vp, vp], i),
            "nrp_cache_create": ([vp, i, i, vp], i),
            "nrp_cache_destroy": ([vp], i),
            "nrp_cache_reset": ([vp, vp], i),
            "nrp_cache_get_head": ([vp, vp], i),
            "nrp_cache_set_head": ([vp, i], i),
            "nrp_cache_import_h": ([vp, vp, vp], i),
            "nrp_cache_export_h": ([vp, vp, vp], i),
            "nrp_attn_forward_with_cache": ([vp, vp, vp, i, i, vp, vp, i, i, vp, vp], i),
            "nrp_linear": ([vp, vp, i, vp, i, i, vp, i, vp, vp], i),
            "nrp_qlinear": ([vp, vp, vp, i, i, vp, vp, vp, i, i, i, vp, vp], i),
            "nrp_seq_shard": ([i, i, i, vp, vp], i),
            "nrp_partition_utterances": ([vp, i, i, i, vp, vp], i),
            "nrp_copy_frames": ([vp, vp, vp, i, i, C.c_int64, vp, vp], i),
            "nrp_unpack_frames": ([vp, vp, vp, i, i, C.c_int64, vp, vp, vp, vp], i),
            "nrp_pack_frames": ([vp, vp, vp, i, i, C.c_int64, vp, vp, vp], i),
            "nrp_seq_shard_plan": ([i, i, i, vp, vp], i),
            "nrp_halo_unique_id": ([vp], i),
            "nrp_halo_comm_create": ([vp, vp, i, i, i, vp], i),
            "nrp_halo_comm_destroy": ([vp], i),
            "nrp_halo_comm_check": ([vp, vp], i),
            "nrp_attn_forward_seq_sharded": ([vp, vp, vp, vp, i, i, vp, vp, vp, vp], i),
            "nrp_block_create": ([vp, i, i, i, i, i, i, i, vp], i),
            "nrp_block_destroy": ([vp], i),
            "nrp_block_set_dtype": ([vp, i], i),
            "nrp_block_attn": ([vp, vp], i),
            "nrp_block_load_linear": ([vp, i, vp, vp], i),
            "nrp_block_load_linear_quantized": ([vp, i, i, i, vp, vp, vp, vp], i),
            "nrp_block_load_norm": ([vp, i, vp, vp], i),
            "nrp_block_load_depthwise": ([vp, vp, vp], i),
            "nrp_block_load_conv_norm": ([vp, vp, vp, vp, vp], i),
            "nrp_block_forward": ([vp, vp, vp, i, i, vp, vp, vp, vp], i),
            "nrp_encoder_create": ([vp] + [i] * 10 + [vp], i),
            "nrp_encoder_destroy": ([vp], i),
            "nrp_encoder_block": ([vp, i, vp], i),
            "nrp_encoder_set_dtype": ([vp, i], i),
            "nrp_encoder_forward_from_embeddings": ([vp, vp, vp, i, i, vp, vp, vp], i),
            "nrp_encoder_add_subsampling": ([vp, i, i, i, i, vp], i),
            "nrp_block_forward_with_cache": ([vp, vp, vp, i, i, vp, vp, vp, i, i, vp, vp], i),
            "nrp_encoder_cache_create": ([vp, i, i, vp], i),
            "nrp_encoder_cache_destroy": ([vp], i),
            "nrp_encoder_cache_reset": ([vp, vp], i),
            "nrp_encoder_cache_get_filled": ([vp, vp], i),
            "nrp_encoder_cache_set_filled": ([vp, i], i),
            "nrp_encoder_cache_layer": ([vp, i, vp, vp], i),
            "nrp_encoder_cache_copy_conv": ([vp, i, vp, i, vp], i),
            "nrp_encoder_forward_streaming": ([vp, vp, vp, i, i, vp, vp, i, vp, vp, vp, vp], i),
            "nrp_encoder_forward": ([vp, vp, vp, i, i, vp, vp, vp, vp], i),
            "nrp_subsampling_create": ([vp, i, i, i, i, i, vp], i),
            "nrp_subsampling_destroy": ([vp], i),
            "nrp_subsampling_set_dtype": ([vp, i], i),
            "nrp_subsampling_feat_out": ([vp, vp], i),
            "nrp_subsampling_output_length": ([vp, i, vp], i),
            "nrp_subsampling_load_conv": ([vp, i, vp, vp], i),
            "nrp_subsampling_load_out": ([vp, vp, vp], i),
            "nrp_subsampling_load_out_quantized": ([vp, i, i, vp, vp, vp, vp], i),
            "nrp_subsampling_forward": ([vp, vp, vp, i, i, i, vp, vp], i),
            "nrp_subsampling_set_chunk_frames": ([vp, i], i),
            "nrp_context_set_weight_cache": ([vp, i], i),
            "nrp_profile_enable": ([vp, i], i),
            "nrp_profile_reset": ([vp], i),
            "nrp_profile_read": ([vp, i, vp, vp], i),
            "nrp_profile_launches": ([vp, vp, vp, C.c_int64, vp], i),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _check(rc: int):
    if rc < 0:
        raise NrpError(rc, lib().nrp_last_error().decode())
    return rc


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _np_f32(a) -> np.ndarray:
    if hasattr(a, "detach"):
        a = a.detach().float().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _torch_dtype(dtype: int):
    import torch
    return torch.bfloat16 if dtype == BF16 else torch.float32


# ----------------------------------------------------------------- context
class Context:
    """One CUDA device (nrp_context)."""

    _default: Dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().nrp_context_create(device, C.byref(h)))
        self.handle = h
        self.device = device

    @classmethod
    def default(cls, device: int = 0) -> "Context":
        if device not in cls._default:
            cls._default[device] = Context(device)
        return cls._default[device]

    def set_weight_cache(self, enable: bool = True):
        """Keep each quantised weight's bf16 copy for linears of >= 256 rows
        (default on), or remake it every call."""
        _check(lib().nrp_context_set_weight_cache(self.handle, int(bool(enable))))

    def check(self, stream=None):
        """Synchronise and raise NrpError(NRP_ERR_DEVICE) if a kernel gave up
        on a bounded wait."""
        _check(lib().nrp_context_check(self.handle, stream if stream is not None else _stream()))

    def selftest_wait_expiry(self, budget_us: int = 20000, stream=None):
        """Queues a kernel whose bounded wait (on a barrier nothing arrives
        on) gives up after budget_us; the next check() raises NRP_ERR_DEVICE
        and the context stays usable."""
        _check(lib().nrp_context_selftest_wait_expiry(
            self.handle, stream if stream is not None else _stream(), int(budget_us)))

    KERNELS = ("gemm_bf16", "gemm_q8", "qgemv", "gemm_f32", "attn_sm100", "attn_simt",
               "attn_stream", "ring_append", "layernorm", "dwconv", "elementwise", "dequant",
               "subsample")

    def profile(self, enable: bool = True):
        _check(lib().nrp_profile_enable(self.handle, int(enable)))

    def profile_reset(self):
        _check(lib().nrp_profile_reset(self.handle))

    def profile_launches(self):
        """[(kernel, ms)] of every recorded launch since the last reset, in
        the order the host issued them."""
        n = C.c_int64()
        _check(lib().nrp_profile_launches(self.handle, None, None, 0, C.byref(n)))
        kinds = (C.c_int * max(n.value, 1))()
        ms = (C.c_float * max(n.value, 1))()
        _check(lib().nrp_profile_launches(self.handle, kinds, ms, n.value, C.byref(n)))
        return [(self.KERNELS[kinds[i]], float(ms[i])) for i in range(n.value)]

    def profile_read(self) -> Dict[str, Tuple[int, float]]:
        """{kernel: (launches, total ms)} for kernels that ran."""
        res = {}
        for k, name in enumerate(self.KERNELS):
            n = C.c_int64()
            ms = C.c_double()
            _check(lib().nrp_profile_read(self.handle, k, C.byref(n), C.byref(ms)))
            if n.value:
                res[name] = (n.value, ms.value)
        return res

    def __del__(self):
        try:
            if self.handle:
                lib().nrp_context_destroy(self.handle)
        except Exception:
            pass


# ---------------------------------------------------- positional encoding
class RelPositionalEncoding:
    """attention.rs:19-194.  get_encoding returns a device tensor
    [1, 2*seq_len-1, d_model] in the table's dtype."""

    def __init__(self, d_model: int, max_len: int, xscaling: bool, device: int = 0):
        self._d_model = d_model
        self.max_len = max_len
        self._xscale = float(lib().nrp_pe_xscale(d_model, int(bool(xscaling))))
        self.dtype = F32
        self.device = device

    def xscale(self) -> float:
        return self._xscale

    def d_model(self) -> int:
        return self._d_model

    def set_dtype(self, dtype: int):
        self.dtype = dtype

    def get_encoding_host(self, seq_len: int) -> np.ndarray:
        out = np.empty((2 * max(seq_len, 1) - 1, self._d_model), np.float32)
        _check(lib().nrp_pe_encoding_host(self._d_model, self.max_len, seq_len,
                                          out.ctypes.data))
        return out[None]

    def get_encoding(self, seq_len: int):
        import torch
        if seq_len <= 0:
            _check(lib().nrp_pe_encoding_host(self._d_model, self.max_len, seq_len, None))
        out = torch.empty((1, 2 * seq_len - 1, self._d_model), dtype=_torch_dtype(self.dtype),
                          device=f"cuda:{self.device}")
        _check(lib().nrp_pe_encoding(Context.default(self.device).handle, self._d_model,
                                     self.max_len, seq_len, self.dtype, out.data_ptr(),
                                     _stream()))
        return out


# ------------------------------------------------------------------ masks
@dataclass(frozen=True)
class AttentionContext:
    """attention.rs:210-273."""
    left: int
    right: int
    chunked: bool

    @staticmethod
    def new(size: Tuple[int, int], style: str) -> Optional["AttentionContext"]:
        c = _AttCtx()
        some = _check(lib().nrp_att_context_new(int(size[0]), int(size[1]), style.encode(),
                                                C.byref(c)))
        return AttentionContext(c.left, c.right, bool(c.chunked)) if some else None

    def _c(self) -> _AttCtx:
        return _AttCtx(self.left, self.right, int(self.chunked))

    def block_mask(self, start: int, end: int, seq_len: int) -> np.ndarray:
        vis = np.empty((end - start, seq_len), np.uint8)
        c = self._c()
        _check(lib().nrp_block_mask_host(C.byref(c), start, end, seq_len, vis.ctypes.data))
        return vis.astype(bool)


class KeyPaddingMask:
    """key_padding_mask's value (attention.rs:280-294), kept as the device
    lengths the kernels read; `additive()` is the reference's [B,1,1,T] form."""

    def __init__(self, lengths, seq_len: int):
        import torch
        self.seq_len = seq_len
        self.lengths = torch.as_tensor(np.asarray(lengths, np.int32)).cuda()
        self._host = np.asarray(lengths, np.int32)

    def additive(self) -> np.ndarray:
        m = np.empty((len(self._host), self.seq_len), np.float32)
        _check(lib().nrp_key_padding_mask_host(self._host.ctypes.data, len(self._host),
                                               self.seq_len, m.ctypes.data))
        return m[:, None, None, :]


def key_padding_mask(lengths, seq_len: int) -> Optional[KeyPaddingMask]:
    h = np.ascontiguousarray(lengths, np.int32)
    some = _check(lib().nrp_key_padding_mask_host(h.ctypes.data, len(h), seq_len, None))
    return KeyPaddingMask(h, seq_len) if some else None


def create_attention_mask(att_context_size, att_context_style, max_audio_length, cache_len,
                          filled_cache_len, tensor_seq_len, valid_seq_len) -> np.ndarray:
    """conformer.rs:97-221 (visibility, [tensor_seq_len, max_audio_length])."""
    vis = np.empty((tensor_seq_len, max_audio_length), np.uint8)
    ctx = None
    if att_context_size is not None:
        ctx = _AttCtx(att_context_size[0], att_context_size[1],
                      int(att_context_style == "chunked_limited"))
    _check(lib().nrp_streaming_mask_host(C.byref(ctx) if ctx is not None else None,
                                         max_audio_length, cache_len, filled_cache_len,
                                         tensor_seq_len, valid_seq_len, vis.ctypes.data))
    return vis.astype(bool)


# ------------------------------------------------------------ quantization
@dataclass
class QuantizationConfig:
    """quantization.rs:20-32."""
    bits: int = 8
    group_size: int = 64


class LinearLayer:
    """quantization.rs:36-163: Standard {weight, bias} or Quantized {weight
    (u32 packed), scales, biases, bias, bits, group_size}; host arrays."""

    def __init__(self, weight, bias=None, scales=None, biases=None, bits=8, group_size=64):
        self.weight = weight
        self.bias = bias
        self.scales = scales
        self.biases = biases
        self.bits = bits
        self.group_size = group_size

    @staticmethod
    def standard(weight, bias=None) -> "LinearLayer":
        return LinearLayer(weight, bias)

    @staticmethod
    def quantized(weight, scales, biases, bias, bits, group_size) -> "LinearLayer":
        return LinearLayer(weight, bias, scales, biases, bits, group_size)

    def is_quantized(self) -> bool:
        return self.scales is not None


def load_linear_layer(weights: Dict[str, object], prefix: str,
                      quant: Optional[QuantizationConfig]) -> Optional[LinearLayer]:
    """quantization.rs:289-349: `.scales` + `.biases` mean quantized,
    default (8, 64); 3-D pointwise weights [O,1,I] are squeezed."""
    w = weights.get(f"{prefix}.weight")
    s = weights.get(f"{prefix}.scales")
    b = weights.get(f"{prefix}.biases")
    bias = weights.get(f"{prefix}.bias")
    if w is not None and s is not None and b is not None:
        bits, gs = (quant.bits, quant.group_size) if quant else (8, 64)
        return LinearLayer.quantized(w, s, b, bias, bits, gs)
    if w is not None:
        w = np.asarray(w.detach().cpu() if hasattr(w, "detach") else w)
        if w.ndim == 3 and w.shape[1] == 1:
            w = w[:, 0, :]
        return LinearLayer.standard(w, bias)
    return None


# ------------------------------------------------------- the attention
class RelPositionMultiHeadAttention:
    """attention.rs:328-894 on the B200 kernels."""

    def __init__(self, d_model: int, n_heads: int, use_bias: bool = True,
                 ctx: Optional[Context] = None):
        self.ctx = ctx or Context.default()
        h = C.c_void_p()
        _check(lib().nrp_attn_create(self.ctx.handle, d_model, n_heads, int(bool(use_bias)),
                                     C.byref(h)))
        self.handle = h
        self._owned = True
        self.d_model = d_model
        self._n_heads = n_heads
        self.dtype = F32
        self._cache_drop_size = 0
        self.att_context_size: Optional[Tuple[int, int]] = None

    @classmethod
    def _view(cls, handle, d_model: int, n_heads: int, ctx: Context, owner=None):
        """A module owned by a ConformerBlock (not freed by this object; it
        keeps the block alive while the view, or a cache made from it, is)."""
        self = cls.__new__(cls)
        self.ctx = ctx
        self.handle = handle
        self._owned = False
        self._owner = owner
        self.d_model = d_model
        self._n_heads = n_heads
        self.dtype = F32
        self._cache_drop_size = 0
        self.att_context_size = None
        return self

    def __del__(self):
        try:
            if self.handle and self._owned:
                lib().nrp_attn_destroy(self.handle)
        except Exception:
            pass

    def head_dim(self) -> int:
        return self.d_model // self._n_heads

    def n_heads(self) -> int:
        return self._n_heads

    @property
    def cache_drop_size(self) -> int:
        return self._cache_drop_size

    @cache_drop_size.setter
    def cache_drop_size(self, n: int):
        _check(lib().nrp_attn_set_cache_drop_size(self.handle, int(n)))
        self._cache_drop_size = int(n)

    def set_dtype(self, dtype: int):
        _check(lib().nrp_attn_set_dtype(self.handle, dtype))
        self.dtype = dtype

    def set_linear(self, which: int, layer: LinearLayer):
        if layer.is_quantized():
            wq = np.ascontiguousarray(np.asarray(layer.weight), np.uint32)
            s = _np_f32(layer.scales)
            b = _np_f32(layer.biases)
            bias = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_attn_load_linear_quantized(
                self.handle, which, layer.bits, layer.group_size, wq.ctypes.data,
                s.ctypes.data, b.ctypes.data, bias.ctypes.data if bias is not None else None))
        else:
            w = _np_f32(layer.weight)
            bias = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_attn_load_linear(self.handle, which, w.ctypes.data,
                                              bias.ctypes.data if bias is not None else None))

    def set_pos_bias(self, u, v):
        u = _np_f32(u)
        v = _np_f32(v)
        _check(lib().nrp_attn_load_pos_bias(self.handle, u.ctypes.data, v.ctypes.data))

    def load_weights(self, weights: Dict[str, object], prefix: str,
                     quant: Optional[QuantizationConfig] = None):
        """attention.rs:863-893."""
        for which, name in enumerate(_LINEAR_NAMES):
            layer = load_linear_layer(weights, f"{prefix}.{name}", quant)
            if layer is not None:
                self.set_linear(which, layer)
        u = weights.get(f"{prefix}.pos_bias_u")
        v = weights.get(f"{prefix}.pos_bias_v")
        if u is not None or v is not None:
            n = self.d_model
            cur_u = _np_f32(u) if u is not None else np.zeros(n, np.float32)
            cur_v = _np_f32(v) if v is not None else np.zeros(n, np.float32)
            self.set_pos_bias(cur_u, cur_v)

    def forward(self, x, pos_emb, context: Optional[AttentionContext] = None,
                key_mask: Optional[KeyPaddingMask] = None, out=None):
        """attention.rs:446-454.  x [B,T,D], pos_emb [1 or none, 2T-1, D]."""
        import torch
        B, T, D = x.shape
        pe = pos_emb.reshape(-1, D)
        if out is None:
            out = torch.empty_like(x)
        c = context._c() if context is not None else None
        _check(lib().nrp_attn_forward(
            self.handle, _stream(), x.data_ptr(), B, T, pe.data_ptr(),
            key_mask.lengths.data_ptr() if key_mask is not None else None,
            C.byref(c) if c is not None else None, out.data_ptr()))
        return out

    def forward_with_cache(self, x, pos_emb, cache: "AttentionCache", cache_filled_len: int,
                           valid_len: Optional[int] = None,
                           context: Optional[AttentionContext] = None, out=None):
        """attention.rs:606-816 as driven per layer by
        ConformerEncoder::forward_streaming (conformer.rs:883-1000).
        Returns the output; `cache` slides in place."""
        import torch
        B, T, D = x.shape
        pe = pos_emb.reshape(-1, D)
        if out is None:
            out = torch.empty_like(x)
        c = context._c() if context is not None else None
        _check(lib().nrp_attn_forward_with_cache(
            self.handle, _stream(), x.data_ptr(), B, T, pe.data_ptr(), cache.handle,
            int(cache_filled_len), T if valid_len is None else int(valid_len),
            C.byref(c) if c is not None else None, out.data_ptr()))
        return out


    def forward_seq_sharded(self, x_local, pos_emb, seq_len: int, halo: "HaloComm",
                            context: Optional[AttentionContext] = None,
                            key_mask: Optional[KeyPaddingMask] = None, out=None):
        """This rank's rows of forward() on a sequence of seq_len frames cut
        into one segment per rank (seq_shard): x_local [B, len, D] holds the
        segment's frames, pos_emb the whole [2*seq_len-1, D] table, key_mask
        the whole-sequence lengths.  No reference counterpart (the reference
        runs on one device); every rank calls it in the same order."""
        import torch
        B, T, D = x_local.shape
        pe = pos_emb.reshape(-1, D)
        if out is None:
            out = torch.empty_like(x_local)
        c = context._c() if context is not None else None
        _check(lib().nrp_attn_forward_seq_sharded(
            self.handle, halo.handle, _stream(), x_local.data_ptr(), B, int(seq_len),
            pe.data_ptr(), key_mask.lengths.data_ptr() if key_mask is not None else None,
            C.byref(c) if c is not None else None, out.data_ptr()))
        return out


# ------------------------------------------------------- conformer block
BLOCK_LINEARS = ("feed_forward1.linear1", "feed_forward1.linear2", "conv.pointwise_conv1",
                 "conv.pointwise_conv2", "feed_forward2.linear1", "feed_forward2.linear2")
BLOCK_NORMS = ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2",
               "norm_out")


class ConformerBlock:
    """ConformerBlock (src/asr/modules/encoders/conformer.rs:1617-2028): the
    macaron feed-forwards, the rel-pos attention, the convolution module and
    the final norm, in bf16 on the device.  conv_norm: "batch_norm" or
    "layer_norm"."""

    def __init__(self, d_model: int, n_heads: int, ff_dim: int, conv_kernel: int = 9,
                 causal_conv: bool = False, conv_norm: str = "batch_norm",
                 use_bias: bool = True, ctx: Optional[Context] = None, _handle=None,
                 _owner=None):
        self.ctx = ctx or Context.default()
        self.d_model, self.n_heads, self.ff_dim, self.conv_kernel = d_model, n_heads, ff_dim, \
            conv_kernel
        self.conv_norm = conv_norm
        self._owner = _owner
        if _handle is None:
            h = C.c_void_p()
            _check(lib().nrp_block_create(self.ctx.handle, d_model, n_heads, ff_dim, conv_kernel,
                                          int(causal_conv), int(conv_norm == "layer_norm"),
                                          int(use_bias), C.byref(h)))
            self.handle, self._owned = h, True
        else:
            self.handle, self._owned = _handle, False
        a = C.c_void_p()
        _check(lib().nrp_block_attn(self.handle, C.byref(a)))
        self.self_attn = RelPositionMultiHeadAttention._view(a, d_model, n_heads, self.ctx,
                                                             owner=self)

    def __del__(self):
        try:
            if self._owned and self.handle:
                lib().nrp_block_destroy(self.handle)
        except Exception:
            pass

    def set_dtype(self, dtype: int):
        _check(lib().nrp_block_set_dtype(self.handle, dtype))
        self.self_attn.dtype = dtype

    def set_linear(self, which: int, layer: LinearLayer):
        if layer.is_quantized():
            wq = np.ascontiguousarray(layer.weight, np.uint32)
            sc, bi = _np_f32(layer.scales), _np_f32(layer.biases)
            b = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_block_load_linear_quantized(
                self.handle, which, layer.bits, layer.group_size, wq.ctypes.data, sc.ctypes.data,
                bi.ctypes.data, b.ctypes.data if b is not None else None))
        else:
            w = _np_f32(layer.weight)
            b = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_block_load_linear(self.handle, which, w.ctypes.data,
                                               b.ctypes.data if b is not None else None))

    def set_norm(self, which: int, gamma, beta):
        g, b = _np_f32(gamma), _np_f32(beta)
        _check(lib().nrp_block_load_norm(self.handle, which, g.ctypes.data, b.ctypes.data))

    def set_depthwise(self, weight, bias=None):
        """weight in the MLX Conv1d layout [d_model, kernel, 1] (or [d_model, kernel])."""
        w = _np_f32(weight).reshape(self.d_model, self.conv_kernel)
        b = _np_f32(bias) if bias is not None else None
        _check(lib().nrp_block_load_depthwise(self.handle, w.ctypes.data,
                                              b.ctypes.data if b is not None else None))

    def set_conv_norm(self, gamma, beta, running_mean=None, running_var=None):
        g, b = _np_f32(gamma), _np_f32(beta)
        m = _np_f32(running_mean) if running_mean is not None else None
        v = _np_f32(running_var) if running_var is not None else None
        _check(lib().nrp_block_load_conv_norm(self.handle, g.ctypes.data, b.ctypes.data,
                                              m.ctypes.data if m is not None else None,
                                              v.ctypes.data if v is not None else None))

    def load_weights(self, weights: Dict[str, object], prefix: str,
                     quant: Optional[QuantizationConfig] = None):
        """ConformerBlock::load_weights (conformer.rs:1978-2028) with the
        NeMo key names."""
        for which, name in enumerate(BLOCK_LINEARS):
            layer = load_linear_layer(weights, f"{prefix}.{name}", quant)
            if layer is not None:
                self.set_linear(which, layer)
        for which, name in enumerate(BLOCK_NORMS):
            g = weights.get(f"{prefix}.{name}.weight")
            b = weights.get(f"{prefix}.{name}.bias")
            if g is not None or b is not None:
                n = self.d_model
                self.set_norm(which, g if g is not None else np.ones(n, np.float32),
                              b if b is not None else np.zeros(n, np.float32))
        self.self_attn.load_weights(weights, f"{prefix}.self_attn", quant)
        w = weights.get(f"{prefix}.conv.depthwise_conv.weight")
        if w is not None:
            self.set_depthwise(w, weights.get(f"{prefix}.conv.depthwise_conv.bias"))
        bn = f"{prefix}.conv.batch_norm"
        g = weights.get(f"{bn}.weight")
        if g is not None:
            self.set_conv_norm(g, weights[f"{bn}.bias"], weights.get(f"{bn}.running_mean"),
                               weights.get(f"{bn}.running_var"))

    def forward(self, x, pos_emb, context: Optional[AttentionContext] = None,
                lengths=None, out=None):
        """conformer.rs:1693-1870.  x [B, T, D] bf16; lengths: device int32
        [B] (a KeyPaddingMask's) or None."""
        import torch
        B, T, D = x.shape
        pe = pos_emb.reshape(-1, D)
        if out is None:
            out = torch.empty_like(x)
        if isinstance(lengths, KeyPaddingMask):
            lengths = lengths.lengths
        c = context._c() if context is not None else None
        _check(lib().nrp_block_forward(self.handle, _stream(), x.data_ptr(), B, T, pe.data_ptr(),
                                       _ptr(lengths), C.byref(c) if c is not None else None,
                                       out.data_ptr()))
        return out

    def forward_with_cache(self, x, pos_emb, cache: "AttentionCache", conv_cache,
                           cache_filled_len: int, valid_len: int,
                           context: Optional[AttentionContext] = None, out=None):
        """ConformerBlock::forward_with_cache (conformer.rs:1877-1967) as
        forward_streaming drives it (883-1000).  x [B, T, D] bf16; pos_emb the
        table for C + T frames; cache the block attention's AttentionCache;
        conv_cache device bf16 [B, conv_kernel - 1, D] (new_conv_cache()),
        replaced in place by the last conv_kernel - 1 GLU frames; frames >=
        valid_len are zeroed before the depthwise conv."""
        import torch
        B, T, D = x.shape
        assert tuple(conv_cache.shape) == (B, self.conv_kernel - 1, D)
        assert conv_cache.dtype == torch.bfloat16 and conv_cache.is_contiguous()
        pe = pos_emb.reshape(-1, D)
        if out is None:
            out = torch.empty_like(x)
        c = context._c() if context is not None else None
        _check(lib().nrp_block_forward_with_cache(
            self.handle, _stream(), x.data_ptr(), B, T, pe.data_ptr(), cache.handle,
            conv_cache.data_ptr(), int(cache_filled_len), int(valid_len),
            C.byref(c) if c is not None else None, out.data_ptr()))
        return out

    def new_conv_cache(self, batch: int, device=None):
        """A zero conv cache [batch, conv_kernel - 1, d_model] bf16 (NeMo starts
        streams with zeros: conformer.rs:960-963)."""
        import torch
        return torch.zeros((batch, self.conv_kernel - 1, self.d_model), dtype=torch.bfloat16,
                           device=device or torch.device("cuda", self.ctx.device))


FEATURES_BFT = 0  # [batch, feat_in, frames]
FEATURES_BTF = 1  # [batch, frames, feat_in]


class Subsampling:
    """The dw_striding Subsampling (src/asr/modules/encoders/conformer.rs:
    1058-1588), the encoder's pre_encode: mel frames -> [B, T', d_model] in
    bf16 on the device."""

    def __init__(self, feat_in: int, d_model: int, subsampling_factor: int = 8,
                 conv_channels: int = 256, causal_downsampling: bool = False,
                 ctx: Optional[Context] = None, _handle=None, _owner=None,
                 host_only: bool = False):
        self.ctx = None if host_only else (ctx or Context.default())
        self.feat_in, self.d_model = feat_in, d_model
        self.factor, self.conv_channels = subsampling_factor, conv_channels
        self.causal = bool(causal_downsampling)
        if _handle is None:
            h = C.c_void_p()
            _check(lib().nrp_subsampling_create(self.ctx.handle if self.ctx else None,
                                                feat_in, d_model,
                                                subsampling_factor, conv_channels,
                                                int(self.causal), C.byref(h)))
            self.handle, self._owned = h, True
        else:
            self.handle, self._owned = _handle, False
        self._owner = _owner
        n = C.c_int()
        _check(lib().nrp_subsampling_feat_out(self.handle, C.byref(n)))
        self.feat_out = n.value
        self.n_strides = {2: 1, 4: 2, 8: 3}.get(subsampling_factor, 2)

    def __del__(self):
        try:
            if self._owned and self.handle:
                lib().nrp_subsampling_destroy(self.handle)
        except Exception:
            pass

    def set_dtype(self, dtype: int):
        _check(lib().nrp_subsampling_set_dtype(self.handle, dtype))

    def set_chunk_frames(self, frames: int):
        """forward_frames_chunked (conformer.rs:1334-1377): inputs longer than
        `frames` mel frames run in time chunks (same output, bounded memory);
        0, the default, runs the whole input at once.  The reference uses
        4096."""
        _check(lib().nrp_subsampling_set_chunk_frames(self.handle, int(frames)))

    def output_length(self, frames: int) -> int:
        """Subsampling::output_length (conformer.rs:1315-1327)."""
        n = C.c_int()
        _check(lib().nrp_subsampling_output_length(self.handle, int(frames), C.byref(n)))
        return n.value

    def output_lengths(self, lengths) -> np.ndarray:
        """Subsampling::output_lengths (conformer.rs:1387-1411)."""
        return np.array([self.output_length(max(int(v), 0)) for v in np.asarray(lengths)],
                        np.int32)

    def set_conv(self, index: int, weight, bias=None):
        """pre_encode.conv.{index} in MLX's layout [O, kH, kW, I]: 0 = conv.0,
        2 + 3i the depthwise convs, 3 + 3i the pointwise ones."""
        w = _np_f32(weight)
        b = _np_f32(bias) if bias is not None else None
        _check(lib().nrp_subsampling_load_conv(self.handle, index, w.ctypes.data,
                                               b.ctypes.data if b is not None else None))

    def set_out(self, layer: "LinearLayer"):
        if layer.is_quantized():
            wq = np.ascontiguousarray(layer.weight, np.uint32)
            sc, bi = _np_f32(layer.scales), _np_f32(layer.biases)
            b = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_subsampling_load_out_quantized(
                self.handle, layer.bits, layer.group_size, wq.ctypes.data, sc.ctypes.data,
                bi.ctypes.data, b.ctypes.data if b is not None else None))
        else:
            w = _np_f32(layer.weight)
            b = _np_f32(layer.bias) if layer.bias is not None else None
            _check(lib().nrp_subsampling_load_out(self.handle, w.ctypes.data,
                                                  b.ctypes.data if b is not None else None))

    def load_weights(self, weights: Dict[str, object], prefix: str = "encoder.pre_encode",
                     quant: Optional[QuantizationConfig] = None):
        """Subsampling::load_weights (conformer.rs:1557-1588)."""
        idx = [0] + [j for i in range(self.n_strides - 1) for j in (2 + 3 * i, 3 + 3 * i)]
        for k in idx:
            w = weights.get(f"{prefix}.conv.{k}.weight")
            if w is not None:
                self.set_conv(k, w, weights.get(f"{prefix}.conv.{k}.bias"))
        layer = load_linear_layer(weights, f"{prefix}.out", quant)
        if layer is not None:
            self.set_out(layer)

    def forward(self, features, lengths=None, layout: int = FEATURES_BTF, out=None):
        """forward_frames (conformer.rs:1413-1555) on device f32 features
        ([B, T, F] by default, or [B, F, T]); lengths: host int32 [B], a
        device int32 tensor, or None; frames past a length read as zero (the
        encoder's mel mask).  Returns ([B, T', d_model] bf16, the output
        lengths for host lengths, else None)."""
        import torch
        if layout == FEATURES_BTF:
            B, T, F = features.shape
        else:
            B, F, T = features.shape
        assert F == self.feat_in and features.dtype == torch.float32 and features.is_contiguous()
        Tp = self.output_length(T)
        if out is None:
            out = torch.empty((B, Tp, self.d_model), dtype=torch.bfloat16,
                              device=features.device)
        dl, out_len = None, None
        if isinstance(lengths, torch.Tensor) and lengths.is_cuda:
            assert lengths.dtype == torch.int32 and lengths.numel() == B
            dl = lengths  # (output lengths: self.output_lengths of the host copy)
        elif lengths is not None:
            ln = np.ascontiguousarray(lengths, np.int32)
            dl = torch.from_numpy(ln).to(features.device)
            out_len = self.output_lengths(ln)
        _check(lib().nrp_subsampling_forward(self.handle, _stream(), features.data_ptr(), layout,
                                             B, T, dl.data_ptr() if dl is not None else None,
                                             out.data_ptr()))
        return out, out_len


class ConformerEncoder:
    """ConformerEncoder (conformer.rs:381-722): the conformer stack, with
    forward_from_embeddings on post-subsampling embeddings, and, given
    feat_in, the dw_striding pre_encode and forward on mel features."""

    def __init__(self, n_layers: int, d_model: int, n_heads: int, ff_dim: int,
                 conv_kernel: int = 9, causal_conv: bool = False,
                 conv_norm: str = "batch_norm", use_bias: bool = True, xscaling: bool = True,
                 max_len: int = 5000, ctx: Optional[Context] = None,
                 feat_in: Optional[int] = None, subsampling_factor: int = 8,
                 subsampling_conv_channels: int = 256, causal_downsampling: bool = False):
        self.ctx = ctx or Context.default()
        self.d_model = d_model
        h = C.c_void_p()
        _check(lib().nrp_encoder_create(self.ctx.handle, n_layers, d_model, n_heads, ff_dim,
                                        conv_kernel, int(causal_conv),
                                        int(conv_norm == "layer_norm"), int(use_bias),
                                        int(xscaling), max_len, C.byref(h)))
        self.handle = h
        self.layers = []
        for i in range(n_layers):
            b = C.c_void_p()
            _check(lib().nrp_encoder_block(h, i, C.byref(b)))
            self.layers.append(ConformerBlock(d_model, n_heads, ff_dim, conv_kernel, causal_conv,
                                              conv_norm, use_bias, self.ctx, _handle=b,
                                              _owner=self))
        self.subsampling = None
        if feat_in is not None:
            sh = C.c_void_p()
            _check(lib().nrp_encoder_add_subsampling(h, feat_in, subsampling_factor,
                                                     subsampling_conv_channels,
                                                     int(causal_downsampling), C.byref(sh)))
            self.subsampling = Subsampling(feat_in, d_model, subsampling_factor,
                                           subsampling_conv_channels, causal_downsampling,
                                           self.ctx, _handle=sh, _owner=self)

    def __del__(self):
        try:
            if self.handle:
                lib().nrp_encoder_destroy(self.handle)
        except Exception:
            pass

    def set_dtype(self, dtype: int):
        _check(lib().nrp_encoder_set_dtype(self.handle, dtype))

    def load_weights(self, weights: Dict[str, object],
                     quant: Optional[QuantizationConfig] = None):
        """conformer.rs:590-605: pre_encode from encoder.pre_encode, layer i
        from encoder.layers.{i}."""
        if self.subsampling is not None:
            self.subsampling.load_weights(weights, "encoder.pre_encode", quant)
        for i, layer in enumerate(self.layers):
            layer.load_weights(weights, f"encoder.layers.{i}", quant)

    def load_checkpoint(self, path: str) -> Optional[QuantizationConfig]:
        """Weights from a .nemo archive (NemoCheckpoint), a model directory
        (SafetensorsLoader.from_directory) or one .safetensors file; the
        convolution weights are brought to MLX's layout first.  Returns the
        quantization config applied (None: standard linears)."""
        from .checkpoint import NemoCheckpoint, SafetensorsLoader, load_safetensors_weights
        quant = None
        if os.path.isdir(path):
            loader = SafetensorsLoader.from_directory(path)
            weights, quant = loader.load_weights(), loader.quantization
        elif path.endswith(".safetensors"):
            weights = load_safetensors_weights(path)
        else:
            weights = NemoCheckpoint.open(path).load_weights()
        self.load_weights(weights, quant)
        return quant

    def forward_from_embeddings(self, x, lengths, context: Optional[AttentionContext] = None,
                                out=None):
        """conformer.rs:694-722: returns ([B, D, T] bf16, lengths)."""
        import torch
        B, T, D = x.shape
        if out is None:
            out = torch.empty((B, D, T), dtype=x.dtype, device=x.device)
        mask = key_padding_mask(np.asarray(lengths, np.int32), T)
        c = context._c() if context is not None else None
        _check(lib().nrp_encoder_forward_from_embeddings(
            self.handle, _stream(), x.data_ptr(), B, T,
            mask.lengths.data_ptr() if mask is not None else None,
            C.byref(c) if c is not None else None, out.data_ptr()))
        return out, lengths

    def new_stream_cache(self, batch: int, cache_len: int) -> EncoderStreamCache:
        """Device caches for forward_streaming (after set_dtype(BF16))."""
        return EncoderStreamCache(self, batch, cache_len)

    def forward_streaming(self, features, lengths, cache: EncoderStreamCache,
                          drop_extra_pre_encoded: int = 0,
                          context: Optional[AttentionContext] = None, out=None):
        """ConformerEncoder::forward_streaming (conformer.rs:840-1047):
        features device f32 [B, feat_in, frames] (the chunk with its
        pre-encode cache frames in front); lengths host int32 [B] or None.
        Returns ([B, D, T] bf16, output lengths int32 [B]); cache.filled
        advances."""
        import torch
        if self.subsampling is None:
            raise NrpError(NRP_ERR_INVALID, "the encoder was built without feat_in")
        B, F, T = features.shape
        assert features.dtype == torch.float32 and features.is_contiguous()
        Tp = self.subsampling.output_length(T) - drop_extra_pre_encoded
        if out is None:
            out = torch.empty((B, self.d_model, Tp), dtype=torch.bfloat16,
                              device=features.device)
        ln = np.ascontiguousarray(lengths, np.int32) if lengths is not None else None
        out_len = np.empty(B, np.int32)
        c = context._c() if context is not None else None
        _check(lib().nrp_encoder_forward_streaming(
            self.handle, _stream(), features.data_ptr(), B, T,
            ln.ctypes.data if ln is not None else None, cache.handle,
            int(drop_extra_pre_encoded), C.byref(c) if c is not None else None, out.data_ptr(),
            out_len.ctypes.data, None))
        return out, out_len

    def forward(self, features, lengths=None, context: Optional[AttentionContext] = None,
                out=None):
        """ConformerEncoder::forward (conformer.rs:475-560): features device
        f32 [B, feat_in, frames], lengths host int32 [B] (mel frames) or None.
        Returns ([B, D, T'] bf16, subsampled lengths int32 [B])."""
        import torch
        if self.subsampling is None:
            raise NrpError(NRP_ERR_INVALID, "the encoder was built without feat_in")
        B, F, T = features.shape
        assert features.dtype == torch.float32 and features.is_contiguous()
        Tp = self.subsampling.output_length(T)
        if out is None:
            out = torch.empty((B, self.d_model, Tp), dtype=torch.bfloat16,
                              device=features.device)
        ln = np.ascontiguousarray(lengths, np.int32) if lengths is not None else None
        out_len = np.empty(B, np.int32)
        c = context._c() if context is not None else None
        _check(lib().nrp_encoder_forward(
            self.handle, _stream(), features.data_ptr(), B, T,
            ln.ctypes.data if ln is not None else None, C.byref(c) if c is not None else None,
            out.data_ptr(), out_len.ctypes.data))
        return out, out_len


class EncoderStreamCache:
    """An encoder's streaming caches on the device (EncoderCache,
    streaming/core.rs:117-185): per layer the attention ring and the conv
    cache, and the shared fill level (last_channel_len)."""

    def __init__(self, encoder: "ConformerEncoder", batch: int, cache_len: int):
        h = C.c_void_p()
        _check(lib().nrp_encoder_cache_create(encoder.handle, batch, cache_len, C.byref(h)))
        self.handle = h
        self.encoder = encoder
        self.batch, self.cache_len = batch, cache_len
        self.conv_kernel = encoder.layers[0].conv_kernel if encoder.layers else 1

    def __del__(self):
        try:
            if self.handle:
                lib().nrp_encoder_cache_destroy(self.handle)
        except Exception:
            pass

    def reset(self):
        _check(lib().nrp_encoder_cache_reset(self.handle, _stream()))

    @property
    def filled(self) -> int:
        n = C.c_int()
        _check(lib().nrp_encoder_cache_get_filled(self.handle, C.byref(n)))
        return n.value

    @filled.setter
    def filled(self, v: int):
        _check(lib().nrp_encoder_cache_set_filled(self.handle, int(v)))

    class _Ring:
        """A layer's attention ring: its slot of the oldest frame (`head`)."""

        def __init__(self, handle):
            self.handle = handle

        @property
        def head(self) -> int:
            h = C.c_int()
            _check(lib().nrp_cache_get_head(self.handle, C.byref(h)))
            return h.value

        @head.setter
        def head(self, v: int):
            _check(lib().nrp_cache_set_head(self.handle, int(v)))

    def rings(self):
        """The layers' attention rings, for StreamingStepGraphs (whose keys
        and restores follow their slots)."""
        out = []
        for i in range(len(self.encoder.layers)):
            a = C.c_void_p()
            _check(lib().nrp_encoder_cache_layer(self.handle, i, C.byref(a), None))
            out.append(EncoderStreamCache._Ring(a))
        return out

    def last_channel(self):
        """[layers, B, C, D] f32 (oldest frame first), as EncoderCache.last_channel."""
        import torch
        outs = []
        for i in range(len(self.encoder.layers)):
            a = C.c_void_p()
            _check(lib().nrp_encoder_cache_layer(self.handle, i, C.byref(a), None))
            out = torch.empty((self.batch, self.cache_len, self.encoder.d_model),
                              dtype=torch.float32, device="cuda")
            _check(lib().nrp_cache_export_h(a, out.data_ptr(), _stream()))
            outs.append(out)
        return torch.stack(outs)

    def last_time(self):
        """[layers, B, D, conv_kernel - 1] f32, as EncoderCache.last_time."""
        import torch
        outs = []
        for i in range(len(self.encoder.layers)):
            buf = torch.empty((self.batch, self.conv_kernel - 1, self.encoder.d_model),
                              dtype=torch.bfloat16, device="cuda")
            _check(lib().nrp_encoder_cache_copy_conv(self.handle, i, buf.data_ptr(), 0,
                                                     _stream()))
            outs.append(buf.float().transpose(1, 2))
        return torch.stack(outs)

    def set_last_time(self, t):
        """Load [layers, B, D, conv_kernel - 1] (EncoderCache.last_time)."""
        import torch
        for i in range(len(self.encoder.layers)):
            buf = t[i].permute(0, 2, 1).to(torch.bfloat16).contiguous().cuda()
            _check(lib().nrp_encoder_cache_copy_conv(self.handle, i, buf.data_ptr(), 1,
                                                     _stream()))


# ------------------------------------------- sequence split (several GPUs)
@dataclass
class SeqPlan:
    """A rank's segment [start, start + len) and its halo: frames received
    from rank-1 / rank+1 and frames sent to them (nrp_seq_shard_plan)."""
    start: int
    len: int
    halo_left: int
    halo_right: int
    send_prev: int
    send_next: int


def copy_frames(dst, src, lengths, non_blocking: bool = True) -> int:
    """dst[b, :lengths[b]] = src[b, :lengths[b]] for every utterance b: one
    copy per utterance (its valid frames are contiguous in a [B, T, ...]
    tensor) on the current stream, e.g. pinned host <-> device around a
    forward.  Padded frames are left as they are: the reference leaves a
    forward's padded rows unspecified (conformer.rs:1590-1593) and padded
    input rows reach no valid output row.  Returns the bytes copied."""
    if dst.shape != src.shape or dst.dtype != src.dtype or dst.dim() < 2:
        raise ValueError("copy_frames: dst and src need the same [B, T, ...] shape and dtype")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("copy_frames: contiguous tensors only")
    B, T = dst.shape[0], dst.shape[1]
    ln = np.ascontiguousarray(
        lengths.detach().cpu().numpy() if hasattr(lengths, "detach") else lengths, np.int32)
    if ln.shape != (B,):
        raise ValueError("copy_frames: one length per utterance")
    row = dst[0, 0].numel() * dst.element_size() if T else 0
    if not (dst.is_cuda or src.is_cuda):  # host to host: no device involved
        total = 0
        for b, L in enumerate(ln.tolist()):
            L = min(max(L, 0), T)
            if L:
                dst[b, :L].copy_(src[b, :L])
                total += L * row
        return total
    if B == 0 or T == 0:
        return 0
    nbytes = C.c_int64(0)
    _check(lib().nrp_copy_frames(dst.data_ptr(), src.data_ptr(),
                                 ln.ctypes.data, B, T, row, _stream(), C.byref(nbytes)))
    if not non_blocking:
        import torch
        torch.cuda.current_stream().synchronize()
    return int(nbytes.value)


def _frames_args(name, padded, packed, lengths, staging):
    """Checks shared by unpack_frames / pack_frames; returns (lengths as
    int32, row bytes, packed bytes)."""
    if padded.dim() < 2 or packed.dim() != padded.dim() - 1:
        raise ValueError(f"{name}: padded [B, T, ...] and packed [rows, ...] tensors")
    if padded.dtype != packed.dtype or padded.shape[2:] != packed.shape[1:]:
        raise ValueError(f"{name}: padded and packed rows differ in shape or dtype")
    if not (padded.is_contiguous() and packed.is_contiguous()):
        raise ValueError(f"{name}: contiguous tensors only")
    if not padded.is_cuda:
        raise ValueError(f"{name}: the padded tensor lives on the device")
    B, T = padded.shape[0], padded.shape[1]
    ln = np.ascontiguousarray(
        lengths.detach().cpu().numpy() if hasattr(lengths, "detach") else lengths, np.int32)
    if ln.shape != (B,) or (ln < 0).any() or (ln > T).any():
        raise ValueError(f"{name}: one length in [0, T] per utterance")
    if packed.shape[0] < int(ln.sum()):
        raise ValueError(f"{name}: the packed tensor has fewer rows than sum(lengths)")
    row = padded[0, 0].numel() * padded.element_size() if T else 0
    nbytes = int(ln.sum()) * row
    if packed.is_cuda:
        if staging is not None:
            raise ValueError(f"{name}: staging is for a packed tensor in host memory")
    else:
        if staging is None or not staging.is_cuda or not staging.is_contiguous() or \
                staging.numel() * staging.element_size() < nbytes:
            raise ValueError(f"{name}: a host packed tensor needs a device staging buffer of "
                             f"{nbytes} bytes")
        if not packed.is_pinned():
            raise ValueError(f"{name}: the host packed tensor must be pinned")
    return ln, row, nbytes


def unpack_frames(dst, src, lengths, staging=None, dev_lengths=None) -> int:
    """dst[b, :lengths[b]] = the packed rows of utterance b in src
    ([sum(lengths), ...], utterances back to back) -- nrp_unpack_frames.
    A pinned host src crosses the link in one copy into `staging` (a device
    buffer of at least the packed bytes), then a kernel scatters the rows;
    a device src is scattered directly.  dev_lengths (an int32 device
    tensor of B, may be None, e.g. a KeyPaddingMask's lengths) also
    receives the lengths.  Stream ordered; returns the packed bytes."""
    ln, row, nbytes = _frames_args("unpack_frames", dst, src, lengths, staging)
    B, T = dst.shape[0], dst.shape[1]
    if dev_lengths is not None and (not dev_lengths.is_cuda or dev_lengths.dtype.itemsize != 4
                                    or dev_lengths.numel() < B):
        raise ValueError("unpack_frames: dev_lengths is an int32 device tensor of B")
    if B == 0 or T == 0:
        return 0
    out = C.c_int64(0)
    _check(lib().nrp_unpack_frames(dst.data_ptr(), src.data_ptr(), ln.ctypes.data, B, T, row,
                                   staging.data_ptr() if staging is not None else None,
                                   dev_lengths.data_ptr() if dev_lengths is not None else None,
                                   _stream(), C.byref(out)))
    return int(out.value)


def pack_frames(dst, src, lengths, staging=None) -> int:
    """The rows src[b, :lengths[b]] of every utterance, back to back into
    dst ([sum(lengths), ...]) -- nrp_pack_frames.  For a pinned host dst a
    kernel gathers the rows into `staging` (device, at least the packed
    bytes) and one copy crosses the link; a device dst is gathered into
    directly.  Stream ordered; returns the packed bytes."""
    ln, row, nbytes = _frames_args("pack_frames", src, dst, lengths, staging)
    B, T = src.shape[0], src.shape[1]
    if B == 0 or T == 0:
        return 0
    out = C.c_int64(0)
    _check(lib().nrp_pack_frames(dst.data_ptr(), src.data_ptr(), ln.ctypes.data, B, T, row,
                                 staging.data_ptr() if staging is not None else None,
                                 _stream(), C.byref(out)))
    return int(out.value)


def partition_utterances(lengths, nranks: int, d_model: int = 1024):
    """Utterance-parallel split of a batch over nranks GPUs
    (nrp_partition_utterances): returns (per-rank index arrays in batch
    order, per-rank cost)."""
    ln = np.ascontiguousarray(lengths, np.int32)
    rank_of = np.empty(len(ln), np.int32)
    cost = np.empty(nranks, np.float64)
    _check(lib().nrp_partition_utterances(ln.ctypes.data, len(ln), nranks, d_model,
                                          rank_of.ctypes.data, cost.ctypes.data))
    return [np.nonzero(rank_of == r)[0] for r in range(nranks)], cost


def seq_shard(seq_len: int, nranks: int, rank: int) -> Tuple[int, int]:
    """(start, len) of rank's segment: ceil(seq_len / nranks) frames each,
    the last one ragged."""
    s, n = C.c_int(), C.c_int()
    _check(lib().nrp_seq_shard(seq_len, nranks, rank, C.byref(s), C.byref(n)))
    return s.value, n.value


def seq_shard_plan(seq_len: int, nranks: int, rank: int,
                   context: Optional[AttentionContext] = None) -> SeqPlan:
    p = _SeqPlan()
    c = context._c() if context is not None else None
    _check(lib().nrp_seq_shard_plan(seq_len, nranks, rank, C.byref(c) if c is not None else None,
                                    C.byref(p)))
    return SeqPlan(p.start, p.len, p.halo_left, p.halo_right, p.send_prev, p.send_next)


class HaloComm:
    """The NCCL communicator of a sequence split (nrp_halo): one rank per
    process and GPU.  Every host-side wait is bounded by timeout_ms; a peer
    that does not join or answer in time aborts the communicator and raises
    NrpError(NRP_ERR_DEVICE)."""

    ID_BYTES = 128

    def __init__(self, rank: int, nranks: int, unique_id: bytes,
                 ctx: Optional[Context] = None, timeout_ms: int = 30000):
        self.handle = None
        self.ctx = ctx or Context.default()
        if len(unique_id) != self.ID_BYTES:
            raise NrpError(NRP_ERR_INVALID, "unique id must be 128 bytes")
        uid = (C.c_ubyte * self.ID_BYTES).from_buffer_copy(unique_id)
        h = C.c_void_p()
        _check(lib().nrp_halo_comm_create(self.ctx.handle, uid, rank, nranks, timeout_ms,
                                          C.byref(h)))
        self.handle = h
        self.rank, self.nranks = rank, nranks

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_ubyte * HaloComm.ID_BYTES)()
        _check(lib().nrp_halo_unique_id(buf))
        return bytes(buf)

    @staticmethod
    def share_unique_id(group=None) -> bytes:
        """Makes the id on the group's first rank and broadcasts it over
        torch.distributed (any backend)."""
        import torch.distributed as dist
        first = dist.get_global_rank(group, 0) if group is not None else 0
        obj = [HaloComm.unique_id() if dist.get_rank() == first else None]
        dist.broadcast_object_list(obj, src=first, group=group)
        return obj[0]

    @classmethod
    def from_process_group(cls, ctx: Optional[Context] = None, group=None,
                           timeout_ms: int = 30000) -> "HaloComm":
        import torch.distributed as dist
        uid = cls.share_unique_id(group)
        return cls(dist.get_rank(group), dist.get_world_size(group), uid, ctx, timeout_ms)

    def plan(self, seq_len: int, context: Optional[AttentionContext] = None) -> SeqPlan:
        return seq_shard_plan(seq_len, self.nranks, self.rank, context)

    def check(self, stream=None):
        """Waits (bounded) for `stream`; raises NRP_ERR_DEVICE if a peer never
        answered (the communicator is then aborted)."""
        _check(lib().nrp_halo_comm_check(self.handle,
                                         stream if stream is not None else _stream()))

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            _check(lib().nrp_halo_comm_destroy(h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class AttentionCache:
    """One layer's EncoderCache.last_channel (streaming/core.rs:117-127) as a
    device ring with derived K/V rings."""

    def __init__(self, attn: RelPositionMultiHeadAttention, batch: int, cache_len: int):
        h = C.c_void_p()
        _check(lib().nrp_cache_create(attn.handle, batch, cache_len, C.byref(h)))
        self.handle = h
        self.attn = attn
        self.batch = batch
        self.cache_len = cache_len

    def __del__(self):
        try:
            if self.handle:
                lib().nrp_cache_destroy(self.handle)
        except Exception:
            pass

    def reset(self):
        _check(lib().nrp_cache_reset(self.handle, _stream()))

    @property
    def head(self) -> int:
        """Ring slot of the oldest cached frame (host state)."""
        h = C.c_int()
        _check(lib().nrp_cache_get_head(self.handle, C.byref(h)))
        return h.value

    @head.setter
    def head(self, value: int):
        _check(lib().nrp_cache_set_head(self.handle, int(value)))

    def export_h(self):
        import torch
        out = torch.empty((self.batch, self.cache_len, self.attn.d_model), dtype=torch.float32,
                          device="cuda")
        _check(lib().nrp_cache_export_h(self.handle, out.data_ptr(), _stream()))
        return out

    def import_h(self, h):
        h = h.float().contiguous().cuda()
        _check(lib().nrp_cache_import_h(self.handle, h.data_ptr(), _stream()))


class StreamingStepGraphs:
    """A streaming chunk step replayed as CUDA graphs, with no host work per
    layer (the sync-free driver the reference's forward_streaming lacks:
    conformer.rs:840-1047 rebuilds masks and caches on the host every chunk).

    `step(filled, *args)` enqueues one chunk of work on the current stream: calls of
    `forward_with_cache` on the `caches`, reading and writing device buffers
    that stay the same from chunk to chunk (the caller copies each new chunk
    into the step's input buffer; `args`, hashable, may pick among several
    such buffers).  The launches of a step depend on the fill level and on
    each cache's ring slot, so a graph is kept per (filled, ring slots, args)
    key: once the cache is full the slots cycle with
    period cache_len / gcd(cache_len, frames appended per chunk), so a few
    graphs serve a whole stream.  The first step with a key runs as it is
    (sizing every workspace), the second is captured and replayed, later ones
    are replayed.  Capturing runs the calls' host logic without their device
    work, so the ring slots that logic leaves are restored after each replay.
    """

    def __init__(self, step, caches):
        self.step = step
        self.caches = list(caches)
        self.graphs = {}   # key -> (graph, ring slots after the step)
        self.seen = set()

    def __call__(self, filled: int, *args):
        import torch
        key = (int(filled), tuple(c.head for c in self.caches), args)
        if key in self.graphs:
            g, after = self.graphs[key]
            g.replay()
        elif key in self.seen:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.step(filled, *args)
            after = tuple(c.head for c in self.caches)
            self.graphs[key] = (g, after)
            g.replay()
        else:
            self.seen.add(key)
            self.step(filled, *args)
            return
        for c, h in zip(self.caches, after):
            c.head = h


class EncoderCache:
    """streaming/core.rs:117-187: dimensions of the three cache tensors and
    the host fill level last_channel_len."""

    def __init__(self, num_layers, batch_size, channel_cache_size, time_cache_size, d_model):
        self._dims = (num_layers, batch_size, channel_cache_size, time_cache_size, d_model)
        self.last_channel_len = np.zeros(batch_size, np.int64)

    def batch_size(self):
        return self._dims[1]

    def num_layers(self):
        return self._dims[0]

    def channel_cache_size(self):
        return self._dims[2]

    def time_cache_size(self):
        return self._dims[3]


@dataclass
class StreamingConfig:
    """streaming/core.rs:27-108."""
    chunk_size: Tuple[int, int]
    shift_size: Tuple[int, int]
    cache_drop_size: int
    last_channel_cache_size: int
    last_time_cache_size: int
    valid_out_len: int
    pre_encode_cache_size: Tuple[int, int]
    drop_extra_pre_encoded: int
    lookahead_frames: int
    mode_idx: int
    left_context: int
    right_context: int

    def chunk_size_for_step(self, is_first):
        return self.chunk_size[0] if is_first else self.chunk_size[1]

    def shift_size_for_step(self, is_first):
        return self.shift_size[0] if is_first else self.shift_size[1]

    def pre_encode_cache_for_step(self, is_first):
        return self.pre_encode_cache_size[0] if is_first else self.pre_encode_cache_size[1]

    def drop_extra_for_step(self, is_first):
        return 0 if is_first else self.drop_extra_pre_encoded


def compute_streaming_config(left: int, right: int, style: str, n_layers: int,
                             subsampling_factor: int = 8, conv_kernel_size: int = 9,
                             causal_conv: bool = True, mode_idx: int = 0,
                             max_context: int = 10000) -> StreamingConfig:
    """streaming/core.rs:247-362 for one (left, right) mode."""
    c = _StreamCfg()
    _check(lib().nrp_streaming_config_compute(left, right, int(style == "chunked_limited"),
                                              n_layers, subsampling_factor, conv_kernel_size,
                                              int(causal_conv), mode_idx, max_context,
                                              C.byref(c)))
    return StreamingConfig(tuple(c.chunk_size), tuple(c.shift_size), c.cache_drop_size,
                           c.last_channel_cache_size, c.last_time_cache_size, c.valid_out_len,
                           tuple(c.pre_encode_cache_size), c.drop_extra_pre_encoded,
                           c.lookahead_frames, c.mode_idx, c.left_context, c.right_context)


@dataclass
class StreamingModeInfo:
    """streaming/core.rs:190-243."""
    mode_idx: int
    left_context: int
    right_context: int
    latency_ms: float
    description: str

    @staticmethod
    def from_context(mode_idx, left_context, right_context, frame_duration_ms):
        latency = right_context * frame_duration_ms if right_context >= 0 else math.inf
        if right_context == 0:
            d = f"Zero lookahead (lowest latency), left={left_context}"
        elif right_context < 0:
            d = f"Unlimited lookahead, left={left_context}"
        else:
            d = f"Lookahead={right_context} frames (~{latency:.0f}ms), left={left_context}"
        return StreamingModeInfo(mode_idx, left_context, right_context, latency, d)


# ----------------------------------------------------- linear primitives
def linear(x, w, bias=None, ctx: Optional[Context] = None, out=None):
    """LinearLayer::forward Standard arm on device tensors (f32 or bf16)."""
    import torch
    ctx = ctx or Context.default()
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], N), dtype=x.dtype, device=x.device)
    dt = BF16 if x.dtype == torch.bfloat16 else F32
    _check(lib().nrp_linear(ctx.handle, _stream(), dt, x.data_ptr(), M, K, w.data_ptr(), N,
                            _ptr(bias), out.data_ptr()))
    return out


def qlinear(x, wq, scales, biases, bias=None, group_size=64, bits=8,
            ctx: Optional[Context] = None, out=None):
    """LinearLayer::forward Quantized arm (bf16 activations, u32 packed W)."""
    import torch
    ctx = ctx or Context.default()
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = wq.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], N), dtype=torch.bfloat16, device=x.device)
    _check(lib().nrp_qlinear(ctx.handle, _stream(), x.data_ptr(), M, K, wq.data_ptr(),
                             scales.data_ptr(), biases.data_ptr(), N, group_size, bits,
                             _ptr(bias), out.data_ptr()))
    return out


# weight ingestion (safetensors, .nemo archives, model directories)
from .checkpoint import (CheckpointError, NemoCheckpoint, SafetensorsLoader,  # noqa: E402
                         WeightFormat, load_safetensors_weights, read_safetensors,
                         read_safetensors_metadata, transform_weights_to_mlx, write_safetensors)
