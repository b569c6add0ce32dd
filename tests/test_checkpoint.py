"""Weight ingestion (src/core/weights.rs, src/core/checkpoint.rs): the
safetensors format, the PyTorch/MLX layout detection and conv transposes,
.nemo archives (plain and gzip TAR, .safetensors or .ckpt weights) and model
directories with their quantization config.  Host only."""
import io
import json
import os
import struct
import tarfile

import numpy as np
import pytest

from conftest import rand_block
from __graft_entry__ import load_package

nrp = load_package()
ck = nrp.checkpoint


def _header_bytes(header):
    hj = json.dumps(header).encode()
    return struct.pack("<Q", len(hj)) + hj


def test_reads_a_hand_built_file(tmp_path):
    # the format, independent of this package's writer: u64 LE header size,
    # JSON header, data section
    a = np.array([1.0, -2.5], "<f4").tobytes()
    b = struct.pack("<HH", 0x3F80, 0xBF00)  # bf16 1.0, -0.5
    c = struct.pack("<I", 0xDEADBEEF)
    header = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
              "b": {"dtype": "BF16", "shape": [1, 2], "data_offsets": [8, 12]},
              "c": {"dtype": "U32", "shape": [], "data_offsets": [12, 16]},
              "__metadata__": {"format": "mlx", "n": "3"}}
    p = tmp_path / "h.safetensors"
    p.write_bytes(_header_bytes(header) + a + b + c)
    t = nrp.read_safetensors(str(p))
    assert sorted(t) == ["a", "b", "c"]
    assert t["a"].dtype == np.float32 and list(t["a"]) == [1.0, -2.5]
    assert t["b"].shape == (1, 2) and list(t["b"][0]) == [1.0, -0.5]
    assert t["c"].dtype == np.uint32 and int(t["c"]) == 0xDEADBEEF
    assert nrp.read_safetensors_metadata(str(p)) == {"format": "mlx", "n": "3"}


def test_write_read_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    ts = {
        "f32": rng.standard_normal((3, 5)).astype(np.float32),
        "f16": rng.standard_normal(7).astype(np.float16),
        "bf": rng.standard_normal((2, 2, 3)).astype(np.float32),
        "u32": rng.integers(0, 2**32, (4, 3), dtype=np.uint64).astype(np.uint32),
        "i64": rng.integers(-5, 5, 6).astype(np.int64),
        "u8": rng.integers(0, 255, 9).astype(np.uint8),
        "flag": np.array([True, False]),
        "scalar": np.array(3.5, np.float32),
        "empty": np.zeros((0, 4), np.float32),
    }
    p = str(tmp_path / "w.safetensors")
    nrp.write_safetensors(p, ts, metadata={"format": "pt"}, bf16=("bf",))
    with open(p, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
    assert n % 8 == 0  # data section 8-byte aligned
    back = nrp.read_safetensors(p)
    assert set(back) == set(ts)
    for k, v in ts.items():
        if k == "bf":
            # rounded to bf16 (nearest even), read back exactly
            want = ck._bf16_to_f32(ck._f32_to_bf16_bits(v))
            assert np.array_equal(back[k], want) and back[k].dtype == np.float32
            assert np.max(np.abs(back[k] - v)) <= np.max(np.abs(v)) * 2.0 ** -8
        elif k == "f16":
            assert back[k].dtype == np.float32 and np.array_equal(back[k], v.astype(np.float32))
        else:
            assert back[k].dtype == v.dtype and np.array_equal(back[k], v)
    assert nrp.read_safetensors_metadata(p) == {"format": "pt"}


def test_malformed_files_are_rejected(tmp_path):
    p = tmp_path / "big.safetensors"
    p.write_bytes(struct.pack("<Q", 200_000_000) + b"{}")
    with pytest.raises(nrp.CheckpointError, match="too large"):
        nrp.read_safetensors(str(p))
    p = tmp_path / "off.safetensors"
    p.write_bytes(_header_bytes({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}})
                  + b"\0" * 8)
    with pytest.raises(nrp.CheckpointError, match="do not match"):
        nrp.read_safetensors(str(p))
    p = tmp_path / "json.safetensors"
    p.write_bytes(struct.pack("<Q", 3) + b"{x}")
    with pytest.raises(nrp.CheckpointError, match="invalid"):
        nrp.read_safetensors(str(p))


def test_weight_format_from_metadata():
    # weights.rs test_weight_format_from_metadata
    WF = nrp.WeightFormat
    assert WF.from_safetensors_metadata({}) is WF.PYTORCH
    assert WF.from_safetensors_metadata({"format": "mlx"}) is WF.MLX
    assert WF.from_safetensors_metadata({"format": "MLX"}) is WF.MLX
    assert WF.from_safetensors_metadata({"format": "pytorch"}) is WF.PYTORCH
    assert WF.PYTORCH.needs_conv1d_transpose() and not WF.MLX.needs_conv1d_transpose()


def test_weight_format_from_shapes():
    WF = nrp.WeightFormat
    z = np.zeros
    assert WF.detect_from_weights({"encoder.pre_encode.conv.0.weight": z((256, 1, 3, 3))}) \
        is WF.PYTORCH
    assert WF.detect_from_weights({"encoder.pre_encode.conv.0.weight": z((256, 3, 3, 1))}) is WF.MLX
    assert WF.detect_from_weights({"x.conv.3.weight": z((256, 1, 1, 256))}) is WF.MLX
    assert WF.detect_from_weights({"x.conv.3.weight": z((256, 256, 1, 1))}) is WF.PYTORCH
    assert WF.detect_from_weights({"encoder.layers.0.norm_out.weight": z(8)}) is WF.PYTORCH


def test_transform_weights_to_mlx():
    rng = np.random.default_rng(1)
    w = {
        "l.conv.depthwise_conv.weight": rng.standard_normal((6, 1, 9)),   # (O, I, K)
        "l.conv.pointwise_conv1.weight": rng.standard_normal((12, 6, 1)),
        "pre_encode.conv.0.weight": rng.standard_normal((4, 1, 3, 3)),    # (O, I, H, W)
        "l.self_attn.linear_q.weight": rng.standard_normal((6, 6)),
        "l.conv.depthwise_conv.bias": rng.standard_normal(6),
        "l.conv.batch_norm.weight": rng.standard_normal(6),
    }
    t = nrp.transform_weights_to_mlx(w)
    assert np.array_equal(t["l.conv.depthwise_conv.weight"], w["l.conv.depthwise_conv.weight"]
                          .transpose(0, 2, 1))
    assert t["l.conv.pointwise_conv1.weight"].shape == (12, 1, 6)
    assert np.array_equal(t["pre_encode.conv.0.weight"], w["pre_encode.conv.0.weight"]
                          .transpose(0, 2, 3, 1))
    for k in ("l.self_attn.linear_q.weight", "l.conv.depthwise_conv.bias",
              "l.conv.batch_norm.weight"):
        assert t[k] is w[k]


def test_load_safetensors_weights_detects_the_layout(tmp_path):
    rng = np.random.default_rng(2)
    pt = {"encoder.pre_encode.conv.0.weight": rng.standard_normal((4, 1, 3, 3)).astype(np.float32),
          "encoder.layers.0.conv.depthwise_conv.weight":
              rng.standard_normal((6, 1, 9)).astype(np.float32)}
    p = str(tmp_path / "pt.safetensors")
    nrp.write_safetensors(p, pt)
    got = nrp.load_safetensors_weights(p)
    assert got["encoder.layers.0.conv.depthwise_conv.weight"].shape == (6, 9, 1)
    assert got["encoder.pre_encode.conv.0.weight"].shape == (4, 3, 3, 1)
    # MLX metadata: no transpose, even though the shapes look like PyTorch's
    q = str(tmp_path / "mlx.safetensors")
    nrp.write_safetensors(q, pt, metadata={"format": "mlx"})
    got = nrp.load_safetensors_weights(q)
    assert got["encoder.layers.0.conv.depthwise_conv.weight"].shape == (6, 1, 9)


def _pytorch_layout(wd):
    """An MLX-layout weight dict as NeMo stores it (conv weights (O, I, K))."""
    out = {}
    for k, v in wd.items():
        v = np.asarray(v)
        if k.endswith("depthwise_conv.weight"):
            v = np.ascontiguousarray(v.transpose(0, 2, 1))          # (D, K, 1) -> (D, 1, K)
        elif "pointwise_conv" in k and k.endswith(".weight") and v.ndim == 2:
            v = np.ascontiguousarray(v[:, :, None])                  # (O, I) -> (O, I, 1)
        out[k] = v
    return out


def _tar(path, files, gz=False):
    with tarfile.open(path, "w:gz" if gz else "w") as tar:
        for name, data in files.items():
            info = tarfile.TarInfo(name)
            info.size = len(data)
            tar.addfile(info, io.BytesIO(data))


@pytest.mark.parametrize("gz", [False, True])
def test_nemo_archive_with_safetensors(tmp_path, orc, gz):
    rng = np.random.default_rng(3)
    _, wd = rand_block(rng, 64, 2, 128, 9, prefix="encoder.layers.0")
    wst = str(tmp_path / "w.safetensors")
    nrp.write_safetensors(wst, _pytorch_layout(wd))
    files = {"model_config.yaml": b"encoder:\n  d_model: 64\n  n_heads: 2\n",
             "model_weights.safetensors": open(wst, "rb").read(),
             "tokenizer/tokenizer.model": b"\x0a\x01x"}
    nemo = str(tmp_path / ("m.nemo"))
    _tar(nemo, files, gz)
    cp = nrp.NemoCheckpoint.open(nemo)
    assert cp.load_config()["encoder"]["d_model"] == 64
    assert cp.artifact_names() == ["tokenizer/tokenizer.model"]
    assert cp.find_tokenizer().endswith("tokenizer.model")
    got = cp.load_weights()
    assert set(got) == set(wd)
    for k, v in wd.items():
        v = np.asarray(v)
        g = got[k]
        if "pointwise_conv" in k and k.endswith(".weight"):
            assert g.shape == (v.shape[0], 1, v.shape[1])  # MLX (O, 1, I): squeezed on load
            g = g[:, 0, :]
        assert np.array_equal(g, v.astype(g.dtype)), k


def test_nemo_archive_with_ckpt(tmp_path):
    torch = pytest.importorskip("torch")
    sd = {"encoder.layers.0.conv.depthwise_conv.weight": torch.randn(6, 1, 9).bfloat16(),
          "encoder.layers.0.norm_out.weight": torch.randn(6)}
    buf = io.BytesIO()
    torch.save(sd, buf)
    nemo = str(tmp_path / "c.nemo")
    _tar(nemo, {"./model_config.yaml": b"x: 1\n", "./model_weights.ckpt": buf.getvalue()})
    got = nrp.NemoCheckpoint.open(nemo).load_weights()
    dw = got["encoder.layers.0.conv.depthwise_conv.weight"]
    assert dw.shape == (6, 9, 1) and dw.dtype == np.float32
    assert np.array_equal(dw[:, :, 0], sd["encoder.layers.0.conv.depthwise_conv.weight"]
                          .float()[:, 0, :].numpy())
    assert np.array_equal(got["encoder.layers.0.norm_out.weight"],
                          sd["encoder.layers.0.norm_out.weight"].numpy())


def test_missing_pieces_are_errors(tmp_path):
    with pytest.raises(nrp.CheckpointError, match="not found"):
        nrp.NemoCheckpoint.open(str(tmp_path / "none.nemo"))
    nemo = str(tmp_path / "nocfg.nemo")
    _tar(nemo, {"model_weights.safetensors": b""})
    with pytest.raises(nrp.CheckpointError, match="model_config.yaml"):
        nrp.NemoCheckpoint.open(nemo)
    d = tmp_path / "d"
    d.mkdir()
    with pytest.raises(nrp.CheckpointError, match="No safetensors"):
        nrp.SafetensorsLoader.from_directory(str(d))


def test_model_directory_quantized_round_trip(tmp_path, orc):
    """An MLX 8-bit model directory: weights with `format: mlx` metadata,
    the quantization block in config.json, the file names found by
    priority; the loaded dict equals the one written, bit for bit."""
    rng = np.random.default_rng(4)
    _, wd = rand_block(rng, 64, 2, 128, 9, quant=True, orc=orc, prefix="encoder.layers.0")
    d = tmp_path / "model"
    d.mkdir()
    nrp.write_safetensors(str(d / "model.safetensors"), {k: np.asarray(v) for k, v in wd.items()},
                          metadata={"format": "mlx"})
    nrp.write_safetensors(str(d / "other.safetensors"), {"x": np.zeros(1, np.float32)})
    (d / "model_config.yaml").write_text("encoder:\n  n_layers: 1\n")
    (d / "config.json").write_text(json.dumps({"quantization": {"bits": 8, "group_size": 64}}))
    ld = nrp.SafetensorsLoader.from_directory(str(d))
    assert ld.weights_path.endswith("model.safetensors")
    assert ld.weight_format is nrp.WeightFormat.MLX
    assert ld.is_quantized() and (ld.quantization.bits, ld.quantization.group_size) == (8, 64)
    assert ld.load_config()["encoder"]["n_layers"] == 1
    got = ld.load_weights()
    assert set(got) == set(wd)
    for k, v in wd.items():
        v = np.asarray(v)
        assert got[k].dtype == v.dtype and np.array_equal(got[k], v), k
    # the quantization block may also sit in the main config, YAML or JSON
    (d / "config.yaml").write_text("quantization:\n  bits: 8\n  group_size: 32\n")
    assert nrp.SafetensorsLoader.from_directory(str(d)).quantization.group_size == 32
