"""C ABI without a GPU: the library loads, exports every symbol that
include/nemo_relpos.h declares, and its host-side logic (positional table,
masks, streaming config) matches the oracle and the reference's tests."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

from __graft_entry__ import load_package, ROOT

KATS = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_kats.json")))


@pytest.fixture(scope="module")
def nrp():
    from __graft_entry__ import _load_build_script
    _load_build_script().build()
    return load_package()


def _declared_functions():
    src = open(os.path.join(ROOT, "include", "nemo_relpos.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nrp_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol(nrp):
    names = _declared_functions()
    assert len(names) >= 25
    lib = ctypes.CDLL(nrp.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert nrp.lib().nrp_abi_version() == 1


def test_rust_binding_declares_every_function():
    """The Rust FFI block in the integration notes names every function the
    header declares, and no other: a maintainer can paste it as is."""
    names = set(_declared_functions())
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = set(re.findall(r"\bpub fn (nrp_[a-z0-9_]+)\(", doc))
    assert names - bound == set(), sorted(names - bound)
    assert bound - names == set(), sorted(bound - names)


RUST = os.path.join(ROOT, "mlx-nemo-rs_b200", "rust")


def test_rust_sys_crate_matches_header():
    """The -sys crate (mlx-nemo-rs_b200/rust/nemo-relpos-sys, not compiled
    here: no Rust toolchain) declares every function and constant of the
    header, and only those, with the header's values."""
    names = set(_declared_functions())
    src = open(os.path.join(RUST, "nemo-relpos-sys", "src", "lib.rs")).read()
    bound = set(re.findall(r"\bpub fn (nrp_[a-z0-9_]+)\(", src))
    assert bound == names, (sorted(names - bound), sorted(bound - names))
    hdr = open(os.path.join(ROOT, "include", "nemo_relpos.h")).read()
    consts = dict(re.findall(r"^#define (NRP_[A-Z0-9_]+) (-?\d+)", hdr, re.M))
    consts.update(re.findall(r"\b(NRP_[A-Z0-9_]+) = (-?\d+)", hdr))
    rust = dict(re.findall(r"pub const (NRP_[A-Z0-9_]+): \w+ = (-?\d+);", src))
    assert rust == consts
    build = open(os.path.join(RUST, "nemo-relpos-sys", "build.rs")).read()
    srcs = set(re.findall(r'"([a-z0-9_]+\.(?:cu|cpp))"', build))
    csrc = {f for f in os.listdir(os.path.join(ROOT, "mlx-nemo-rs_b200", "csrc"))
            if f.endswith((".cu", ".cpp"))}
    assert srcs == csrc, (sorted(csrc - srcs), sorted(srcs - csrc))


def test_rust_safe_crate_keeps_reference_signatures():
    """The safe crate calls only functions the -sys crate declares and keeps
    the reference's method names and argument lists
    (attention.rs:35-188, 220, 280, 367, 409, 446, 606, 863)."""
    sys_src = open(os.path.join(RUST, "nemo-relpos-sys", "src", "lib.rs")).read()
    declared = set(re.findall(r"\bpub fn ([a-zA-Z0-9_]+)\(", sys_src))
    src = open(os.path.join(RUST, "nemo-relpos", "src", "lib.rs")).read()
    called = set(re.findall(r"\bsys::(?:cuda::)?([a-zA-Z0-9_]+)\(", src))
    assert called and called <= declared, sorted(called - declared)
    for sig in [
        r"pub fn new\(d_model: i32, max_len: i32, xscaling: bool\) -> Self",
        r"pub fn get_encoding\(&self, seq_len: i32\) -> Result<Array>",
        r"pub fn new\(size: \(i32, i32\), style: &str\) -> Option<Self>",
        r"pub fn key_padding_mask\(lengths: &\[i32\], max_len: i32\) -> Result<Option<Array>>",
        r"pub fn new\(d_model: i32, n_heads: i32, use_bias: bool\) -> Result<Self>",
        r"pub fn set_dtype\(&mut self, dtype: Dtype\) -> Result<\(\)>",
        r"pub fn forward\(&mut self, x: &Array, pos_emb: &Array, context: Option<AttentionContext>,"
        r"\s+key_mask: Option<&Array>\) -> Result<Array>",
        r"pub fn forward_with_cache\(&mut self, x: &Array, pos_emb: &Array, cache: Option<&Array>,"
        r"\s+filled: i32, att_mask: Option<&Array>\)\s+-> Result<\(Array, Option<Array>\)>",
        r"pub fn load_weights\(&mut self, weights: &Weights, prefix: &str,"
        r"\s+quant: Option<&QuantizationConfig>\) -> Result<\(\)>",
        r"pub cache_drop_size: i32", r"pub att_context_size: Option<AttentionContext>",
    ]:
        assert re.search(sig, src), sig


def test_python_mirror_declares_every_function():
    """The Python mirror gives ctypes argument and return types for every
    function the header declares."""
    names = set(_declared_functions())
    src = open(os.path.join(ROOT, "mlx-nemo-rs_b200", "__init__.py")).read()
    table = set(re.findall(r'"(nrp_[a-z0-9_]+)":\s*\(', src))
    assert names - table == set(), sorted(names - table)


def test_pe_matches_oracle_and_kats(nrp, orc):
    for d, max_len, seq in [(4, 3, 3), (512, 100, 50), (16, 10, 25), (1024, 5000, 750),
                            (1024, 5000, 84)]:
        pe = nrp.RelPositionalEncoding(d, max_len, True)
        got = pe.get_encoding_host(seq)
        assert got.shape == (1, 2 * seq - 1, d)
        ref = orc.get_encoding(d, max_len, seq)
        assert np.array_equal(got[0], ref)  # same f32 arithmetic, bit-exact
    k = KATS["pe_values"]
    got = nrp.RelPositionalEncoding(4, 3, False).get_encoding_host(3)[0]
    assert np.abs(got[0] - np.array(k["row0"], np.float32)).max() < k["tol"]
    k = KATS["pe_xscale"]
    assert abs(nrp.RelPositionalEncoding(512, 100, True).xscale() - k["expected"]) < k["tol"]
    assert nrp.RelPositionalEncoding(512, 100, False).xscale() == 1.0
    with pytest.raises(nrp.NrpError):
        nrp.RelPositionalEncoding(16, 10, False).get_encoding_host(0)


def test_context_masks_match_oracle(nrp, orc):
    k = KATS["context_mask_matches_nemo"]
    for size, style in k["cases"]:
        c = nrp.AttentionContext.new(tuple(size), style)
        got = c.block_mask(k["start"], k["end"], k["seq_len"])
        ref = orc.block_mask(size[0], size[1], style == "chunked_limited", k["start"], k["end"],
                             k["seq_len"])
        assert np.array_equal(got, ref), (size, style)
    assert nrp.AttentionContext.new(tuple(k["none_case"][0]), k["none_case"][1]) is None


def test_key_padding_mask(nrp):
    k = KATS["key_padding_mask"]
    lib = nrp.lib()
    full = np.array(k["full_lengths"], np.int32)
    assert lib.nrp_key_padding_mask_host(full.ctypes.data, 2, k["seq_len"], None) == 0
    pad = np.array(k["padded_lengths"] + [0], np.int32)
    m = np.empty((3, k["seq_len"]), np.float32)
    assert lib.nrp_key_padding_mask_host(pad.ctypes.data, 3, k["seq_len"], m.ctypes.data) == 1
    assert (m[0] == 0).all()
    assert (m[1, :9] == 0).all() and np.isinf(m[1, 9:]).all()
    assert m[2, 0] == 0 and np.isinf(m[2, 1:]).all()  # len 0 keeps one key


def test_streaming_masks_match_oracle(nrp, orc):
    cases = [((70, 13), "chunked_limited", 84, 70, f, 14, v) for f in (0, 14, 42, 70)
             for v in (14, 10)]
    cases += [((5, 2), "regular", 12, 6, 3, 6, 6), ((4, -1), "chunked_limited", 9, 5, 5, 4, 4),
              (None, "regular", 10, 6, 2, 4, 3)]
    for size, style, total, cache, filled, T, valid in cases:
        got = nrp.create_attention_mask(size, style, total, cache, filled, T, valid)
        l, r = size if size is not None else (-1, -1)
        ref = orc.create_attention_mask(l, r, style == "chunked_limited", total, cache, filled,
                                        T, valid)
        assert np.array_equal(got, ref), (size, style, filled, valid)


def test_streaming_config_and_mode_info(nrp):
    cfg = nrp.compute_streaming_config(70, 13, "chunked_limited", 24, 8, 9, True)
    assert cfg.cache_drop_size == 0 and cfg.lookahead_frames == 13
    assert cfg.last_channel_cache_size == 70 and cfg.last_time_cache_size == 8
    assert cfg.chunk_size == (1 + 8 * 13, 8 + 8 * 13)
    assert cfg.valid_out_len == 14  # a 14-frame encoder chunk
    assert cfg.pre_encode_cache_size == (0, 9) and cfg.drop_extra_pre_encoded == 2
    reg = nrp.compute_streaming_config(70, 2, "regular", 4, 8, 9, False)
    assert reg.cache_drop_size == reg.lookahead_frames == 2 * 4 + 4 * 4
    k = KATS["streaming_mode_info"]
    m = nrp.StreamingModeInfo.from_context(k["mode_idx"], k["left"], k["right"], k["frame_ms"])
    assert abs(m.latency_ms - k["expected_latency_ms"]) < k["tol"]
    k = KATS["streaming_config_chunk_sizes"]
    sc = nrp.StreamingConfig(tuple(k["chunk_size"]), tuple(k["shift_size"]), 0, 70, 8, 10,
                             tuple(k["pre_encode_cache_size"]), 2, 13, 0, 70, 13)
    assert sc.chunk_size_for_step(True) == 100 and sc.chunk_size_for_step(False) == 120
    assert sc.shift_size_for_step(True) == 80 and sc.shift_size_for_step(False) == 100
    assert sc.pre_encode_cache_for_step(True) == 0 and sc.pre_encode_cache_for_step(False) == 9
    k = KATS["encoder_cache_creation"]
    ec = nrp.EncoderCache(k["num_layers"], k["batch"], k["channel_cache"], k["time_cache"],
                          k["d_model"])
    assert (ec.num_layers(), ec.batch_size(), ec.channel_cache_size(), ec.time_cache_size()) == \
        (24, 1, 70, 8)


def test_load_linear_layer_detection(nrp):
    w = np.zeros((8, 16), np.float32)
    assert not nrp.load_linear_layer({"p.weight": w}, "p", None).is_quantized()
    q = nrp.load_linear_layer({"p.weight": np.zeros((8, 4), np.uint32),
                               "p.scales": np.ones((8, 1)), "p.biases": np.zeros((8, 1))},
                              "p", None)
    assert q.is_quantized() and (q.bits, q.group_size) == (8, 64)  # default (8,64)
    assert nrp.load_linear_layer({}, "p", None) is None
    w3 = np.zeros((8, 1, 16), np.float32)
    assert nrp.load_linear_layer({"p.weight": w3}, "p", None).weight.shape == (8, 16)


def test_no_gpu_calls_fail_loudly(nrp):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(nrp.NrpError):
        nrp.Context(0)


def test_subsampling_sizes_match_oracle(nrp, orc):
    """Subsampling::output_length and compute_freq_output_size through the C
    ABI (a handle without a device context) against the oracle's."""
    from oracle import oracle
    for factor in (2, 4, 8, 16):
        for causal in (False, True):
            for feat in (16, 80, 128):
                s = nrp.Subsampling(feat, 64, factor, 64, causal, host_only=True)
                assert s.feat_out == oracle.subsampling_feat_out(feat, factor, causal)
                for n in list(range(0, 40)) + [4000, 4001, 120000]:
                    assert s.output_length(n) == oracle.subsampling_out_len(n, factor, causal)
    s = nrp.Subsampling(80, 64, 8, 64, False, host_only=True)
    with pytest.raises(nrp.NrpError):
        s.set_conv(1, np.zeros((64, 3, 3, 1), np.float32))  # conv.1 is the ReLU
    with pytest.raises(nrp.NrpError):
        nrp.Subsampling(80, 64, 8, 96, False, host_only=True)  # channels not a power of two


def test_subsampling_chunk_frames_argument(nrp):
    """nrp_subsampling_set_chunk_frames takes 0 (the whole input at once) or a
    chunk size, and rejects a negative one (forward_frames_chunked,
    conformer.rs:1334-1377)."""
    s = nrp.Subsampling(80, 64, 8, 64, False, host_only=True)
    s.set_chunk_frames(4096)
    s.set_chunk_frames(0)
    with pytest.raises(nrp.NrpError) as e:
        s.set_chunk_frames(-1)
    assert e.value.code == nrp.NRP_ERR_INVALID


def test_chunk_plan_frames_match_output_length(nrp):
    """The reference's time-chunk plan (forward_frames_chunked,
    conformer.rs:1344-1377: chunks of a multiple of the factor, context of
    twice the receptive field rounded up to the factor, the first left/factor
    frames of each piece cropped, the last piece kept whole) yields exactly
    Subsampling::output_length(T) frames, so the chunked device path writes
    the same frames as the single pass."""
    for factor in (2, 4, 8):
        for causal in (False, True):
            s = nrp.Subsampling(80, 64, factor, 64, causal, host_only=True)
            for chunk in (64, 512, 4096):
                for T in list(range(1, 700, 7)) + [4095, 4096, 4097, 8200, 12001]:
                    c = max(chunk, factor) // factor * factor
                    if T <= c:
                        continue
                    rf = 1 + (3 - 1) * (factor - 1)
                    ctx = -(-2 * rf // factor) * factor
                    total, start = 0, 0
                    while start < T:
                        end = min(start + c, T)
                        left, right = min(ctx, start), min(ctx, T - end)
                        n = s.output_length(end + right - (start - left))
                        total += n - left // factor if end == T else (end - start) // factor
                        start = end
                    assert total == s.output_length(T), (factor, causal, chunk, T)
