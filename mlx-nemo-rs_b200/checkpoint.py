"""Weight ingestion: safetensors files, .nemo archives and model directories.

The host side of the reference's loaders (src/core/weights.rs,
src/core/checkpoint.rs): read the tensors, detect whether they are laid out
as PyTorch or MLX stores them, transpose convolution weights to MLX's layout,
and hand the arrays (with the quantization config, when the model has one)
to `ConformerEncoder.load_weights` / `ConformerBlock.load_weights` /
`RelPositionMultiHeadAttention.load_weights`, which copy them to the device.

Arrays come back as numpy: bf16 and f16 tensors as float32 (exact), u32
(MLX's packed quantized weights) as uint32.  The safetensors reader needs no
third-party package; `.ckpt` files inside .nemo archives are PyTorch pickles
and are read with `torch.load(weights_only=True)`.
"""
from __future__ import annotations

import enum
import json
import os
import struct
import tarfile
import tempfile
from typing import Dict, Optional, Tuple

import numpy as np

# safetensors dtype names -> (numpy dtype as stored, numpy dtype returned)
_ST_DTYPES = {
    "F64": (np.float64, np.float64),
    "F32": (np.float32, np.float32),
    "F16": (np.float16, np.float32),
    "BF16": (np.uint16, np.float32),
    "I64": (np.int64, np.int64),
    "I32": (np.int32, np.int32),
    "I16": (np.int16, np.int16),
    "I8": (np.int8, np.int8),
    "U64": (np.uint64, np.uint64),
    "U32": (np.uint32, np.uint32),
    "U16": (np.uint16, np.uint16),
    "U8": (np.uint8, np.uint8),
    "BOOL": (np.bool_, np.bool_),
}

# a header larger than this is rejected (weights.rs:255-261)
_MAX_HEADER = 100_000_000


class CheckpointError(ValueError):
    """A file that is not a readable checkpoint (Error::Checkpoint)."""


def _bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(f, np.float32).view(np.uint32)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, (u >> 16) | 0x40, r).astype(np.uint16)


def read_safetensors_header(path: str) -> Tuple[dict, int]:
    """The JSON header (tensor entries and `__metadata__`) and the offset of
    the data section (weights.rs:237-279: u64 little-endian header size, then
    the JSON)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise CheckpointError(f"{path}: not a safetensors file (too short)")
        (n,) = struct.unpack("<Q", raw)
        if n > _MAX_HEADER:
            raise CheckpointError(f"{path}: safetensors header size too large: {n} bytes")
        try:
            header = json.loads(f.read(n))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise CheckpointError(f"{path}: invalid safetensors header: {e}") from e
    if not isinstance(header, dict):
        raise CheckpointError(f"{path}: invalid safetensors header")
    return header, 8 + n


def read_safetensors_metadata(path: str) -> Dict[str, str]:
    """`__metadata__` (string values only), or {} (weights.rs:237-279)."""
    header, _ = read_safetensors_header(path)
    meta = header.get("__metadata__")
    if not isinstance(meta, dict):
        return {}
    return {k: v for k, v in meta.items() if isinstance(v, str)}


def read_safetensors(path: str) -> Dict[str, np.ndarray]:
    """Every tensor of a safetensors file (Array::load_safetensors)."""
    header, base = read_safetensors_header(path)
    size = os.path.getsize(path) - base
    out: Dict[str, np.ndarray] = {}
    with open(path, "rb") as f:
        for name, ent in header.items():
            if name == "__metadata__":
                continue
            try:
                dt, shape, (lo, hi) = ent["dtype"], ent["shape"], ent["data_offsets"]
            except (KeyError, TypeError, ValueError) as e:
                raise CheckpointError(f"{path}: bad entry for {name!r}") from e
            if dt not in _ST_DTYPES:
                raise CheckpointError(f"{path}: {name!r} has unsupported dtype {dt}")
            stored, _ = _ST_DTYPES[dt]
            count = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if not (0 <= lo <= hi <= size) or hi - lo != count * np.dtype(stored).itemsize:
                raise CheckpointError(f"{path}: {name!r} data offsets {lo}..{hi} do not "
                                      f"match shape {shape} of {dt}")
            f.seek(base + lo)
            a = np.frombuffer(f.read(hi - lo), dtype=stored).reshape(shape)
            if dt == "BF16":
                a = _bf16_to_f32(a)
            elif dt == "F16":
                a = a.astype(np.float32)
            else:
                a = a.copy()
            out[name] = a
    return out


def write_safetensors(path: str, tensors: Dict[str, np.ndarray],
                      metadata: Optional[Dict[str, str]] = None,
                      bf16: Tuple[str, ...] = ()) -> None:
    """Write tensors (numpy) as safetensors; names in `bf16` are stored as
    BF16 (rounded to nearest even) instead of their own dtype."""
    rev = {np.dtype(v[0]): k for k, v in _ST_DTYPES.items() if k != "BF16"}
    header: Dict[str, object] = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        a = np.asarray(tensors[name])
        if name in bf16:
            data, dt = _f32_to_bf16_bits(a.astype(np.float32)), "BF16"
        else:
            if a.dtype not in rev:
                raise CheckpointError(f"{name!r}: dtype {a.dtype} has no safetensors name")
            data, dt = a, rev[a.dtype]
        b = np.ascontiguousarray(data).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = dict(metadata)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * (-len(hj) % 8)  # the data section starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


class WeightFormat(enum.Enum):
    """How convolution weights are laid out (weights.rs:13-127)."""
    PYTORCH = "pytorch"  # Conv1d (O, I, K), Conv2d (O, I, H, W)
    MLX = "mlx"          # Conv1d (O, K, I), Conv2d (O, H, W, I)

    @staticmethod
    def from_safetensors_metadata(metadata: Dict[str, str]) -> "WeightFormat":
        """MLX when metadata `format` contains "mlx" (any case), else PyTorch."""
        fmt = metadata.get("format")
        if isinstance(fmt, str) and "mlx" in fmt.lower():
            return WeightFormat.MLX
        return WeightFormat.PYTORCH

    @staticmethod
    def detect_from_weights(weights: Dict[str, np.ndarray]) -> "WeightFormat":
        """From the first subsampling conv's single input channel, else a
        pointwise (1x1) conv2d; PyTorch when neither decides."""
        def conv4(name, w):
            n = name.lower()
            return np.ndim(w) == 4 and "conv" in n and n.endswith(".weight")
        for name, w in weights.items():
            n = name.lower()
            if conv4(name, w) and ("pre_encode" in n or "subsampling" in n):
                s = np.shape(w)
                if s[1] == 1 and s[2] > 1 and s[3] > 1:
                    return WeightFormat.PYTORCH
                if s[3] == 1 and s[1] > 1 and s[2] > 1:
                    return WeightFormat.MLX
        for name, w in weights.items():
            if conv4(name, w):
                s = np.shape(w)
                if s[1] == 1 and s[2] == 1 and s[3] > 1:
                    return WeightFormat.MLX
                if s[2] == 1 and s[3] == 1 and s[1] > 1:
                    return WeightFormat.PYTORCH
        return WeightFormat.PYTORCH

    def needs_conv1d_transpose(self) -> bool:
        return self is WeightFormat.PYTORCH


def _is_conv_weight(name: str) -> bool:
    n = name.lower()
    return n.endswith(".weight") and ("conv" in n or "depthwise" in n or "pointwise" in n)


def transform_weights_to_mlx(weights: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """PyTorch -> MLX layout (weights.rs:130-213): Conv1d weights (O, I, K) ->
    (O, K, I), Conv2d weights (O, I, H, W) -> (O, H, W, I); the rest as is."""
    out = {}
    for name, w in weights.items():
        if _is_conv_weight(name) and np.ndim(w) == 3:
            w = np.ascontiguousarray(np.transpose(w, (0, 2, 1)))
        elif _is_conv_weight(name) and np.ndim(w) == 4:
            w = np.ascontiguousarray(np.transpose(w, (0, 2, 3, 1)))
        out[name] = w
    return out


def load_safetensors_weights(path: str,
                             fmt: Optional[WeightFormat] = None) -> Dict[str, np.ndarray]:
    """weights.rs:215-236: load, detect the format (metadata first, then the
    weight shapes) unless given, and transpose PyTorch-layout convs."""
    weights = read_safetensors(path)
    if fmt is None:
        try:
            fmt = WeightFormat.from_safetensors_metadata(read_safetensors_metadata(path))
        except CheckpointError:
            fmt = WeightFormat.PYTORCH
        if fmt is not WeightFormat.MLX:
            fmt = WeightFormat.detect_from_weights(weights)
    return transform_weights_to_mlx(weights) if fmt.needs_conv1d_transpose() else weights


def _torch_ckpt(path: str) -> Dict[str, np.ndarray]:
    import torch
    sd = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(sd, dict) and "state_dict" in sd and isinstance(sd["state_dict"], dict):
        sd = sd["state_dict"]
    out = {}
    for k, v in sd.items():
        if not hasattr(v, "detach"):
            continue
        v = v.detach()
        if v.dtype in (torch.bfloat16, torch.float16):
            v = v.float()
        out[k] = v.numpy().copy()
    return out


def _find_by_suffix(root: str, suffix: str) -> Optional[str]:
    direct = os.path.join(root, suffix)
    if os.path.exists(direct):
        return direct
    for d, _, files in sorted(os.walk(root)):
        for f in sorted(files):
            if f == suffix or f.endswith(suffix):
                return os.path.join(d, f)
    return None


class NemoCheckpoint:
    """A .nemo archive (checkpoint.rs:18-335): a TAR (gzip-compressed in older
    files) holding model_config.yaml, the weights (model_weights.safetensors
    or model_weights.ckpt, PyTorch layout) and artifacts (tokenizers, vocab)."""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise CheckpointError(f"File not found: {path}")
        self._tmp = tempfile.TemporaryDirectory(prefix="nemo_")
        root = self._tmp.name
        try:
            with tarfile.open(path, "r:*") as tar:  # plain or gzip
                tar.extractall(root, filter="data")
        except tarfile.TarError as e:
            raise CheckpointError(f"Failed to extract .nemo archive {path}: {e}") from e
        cfg = _find_by_suffix(root, "model_config.yaml")
        if cfg is None:
            raise CheckpointError(f"{path}: no model_config.yaml")
        with open(cfg) as f:
            self.config_yaml = f.read()
        self.weights_path = None
        for name in ("model_weights.safetensors", "model_weights.ckpt"):
            if os.path.exists(os.path.join(root, name)):
                self.weights_path = os.path.join(root, name)
                break
        if self.weights_path is None:
            for f in sorted(os.listdir(root)):
                if f.endswith(".safetensors") or f.endswith(".ckpt"):
                    self.weights_path = os.path.join(root, f)
                    break
        self.artifacts: Dict[str, bytes] = {}
        for d, _, files in os.walk(root):
            for f in files:
                full = os.path.join(d, f)
                rel = os.path.relpath(full, root)
                if rel == "model_config.yaml" or f.endswith(".ckpt") or f.endswith(".safetensors"):
                    continue
                with open(full, "rb") as fh:
                    self.artifacts[rel] = fh.read()

    @staticmethod
    def open(path: str) -> "NemoCheckpoint":
        return NemoCheckpoint(path)

    def load_config(self) -> dict:
        import yaml
        return yaml.safe_load(self.config_yaml)

    def load_weights(self) -> Dict[str, np.ndarray]:
        """The weights in MLX layout (.nemo files hold PyTorch layout)."""
        if self.weights_path is None:
            raise CheckpointError("No weights file found in checkpoint")
        if self.weights_path.endswith(".safetensors"):
            raw = read_safetensors(self.weights_path)
        elif self.weights_path.endswith(".ckpt"):
            raw = _torch_ckpt(self.weights_path)
        else:
            raise CheckpointError(f"Unknown weights format: {self.weights_path}")
        return transform_weights_to_mlx(raw)

    def artifact_names(self):
        return sorted(self.artifacts)

    def find_tokenizer(self) -> Optional[str]:
        for name in self.artifact_names():
            base = os.path.basename(name)
            if base.endswith(".model") or base in ("tokenizer.json", "vocab.txt"):
                return os.path.join(self._tmp.name, name)
        return None


def _parse_quantization(content: str):
    """{"quantization": {"bits", "group_size"}} in JSON or YAML, defaults
    (8, 64) (checkpoint.rs:532-570)."""
    from . import QuantizationConfig
    q = None
    try:
        doc = json.loads(content)
        if isinstance(doc, dict):
            q = doc.get("quantization")
    except json.JSONDecodeError:
        doc = None
    if q is None and doc is None:
        try:
            import yaml
            y = yaml.safe_load(content)
            if isinstance(y, dict):
                q = y.get("quantization")
        except Exception:
            q = None
    if not isinstance(q, dict):
        return None
    return QuantizationConfig(int(q.get("bits", 8)), int(q.get("group_size", 64)))


class SafetensorsLoader:
    """A safetensors model (checkpoint.rs:457-784): the weights file, its
    config (YAML or JSON), an optional tokenizer, the weight format (MLX when
    the file's metadata says so, else detected from the shapes on load) and
    the quantization config."""

    def __init__(self, weights_path: str, config_path: str,
                 tokenizer_path: Optional[str] = None):
        if not os.path.exists(weights_path):
            raise CheckpointError(f"Weights file not found: {weights_path}")
        if not os.path.exists(config_path):
            raise CheckpointError(f"Config file not found: {config_path}")
        self.weights_path = weights_path
        with open(config_path) as f:
            self.config_content = f.read()
        self.tokenizer_path = tokenizer_path
        try:
            fmt = WeightFormat.from_safetensors_metadata(read_safetensors_metadata(weights_path))
        except CheckpointError:
            fmt = WeightFormat.PYTORCH
        self.weight_format: Optional[WeightFormat] = fmt if fmt is WeightFormat.MLX else None
        self.quantization = _parse_quantization(self.config_content)

    @staticmethod
    def with_format(weights_path: str, config_path: str, tokenizer_path: Optional[str],
                    fmt: WeightFormat) -> "SafetensorsLoader":
        ld = SafetensorsLoader(weights_path, config_path, tokenizer_path)
        ld.weight_format = fmt
        return ld

    @staticmethod
    def from_directory(d: str) -> "SafetensorsLoader":
        if not os.path.isdir(d):
            raise CheckpointError(f"Not a directory: {d}")
        weights = None
        for name in ("model.safetensors", "weights.safetensors", "model_weights.safetensors",
                     os.path.join("weights", "model.safetensors")):
            if os.path.exists(os.path.join(d, name)):
                weights = os.path.join(d, name)
                break
        if weights is None:
            found = sorted(f for f in os.listdir(d) if f.endswith(".safetensors"))
            if not found:
                raise CheckpointError(f"No safetensors file found in directory {d}")
            weights = os.path.join(d, found[0])
        config = None
        for name in ("config.yaml", "model_config.yaml", "config.json", "model_config.json"):
            if os.path.exists(os.path.join(d, name)):
                config = os.path.join(d, name)
                break
        if config is None:
            raise CheckpointError(f"No config file found in directory {d}")
        tok = None
        for name in ("tokenizer.model", "tokenizer.json", "vocab.txt"):
            if os.path.exists(os.path.join(d, name)):
                tok = os.path.join(d, name)
                break
        ld = SafetensorsLoader(weights, config, tok)
        # MLX keeps the quantization block in config.json
        if ld.quantization is None and os.path.exists(os.path.join(d, "config.json")):
            with open(os.path.join(d, "config.json")) as f:
                ld.quantization = _parse_quantization(f.read())
        return ld

    def load_weights(self) -> Dict[str, np.ndarray]:
        return load_safetensors_weights(self.weights_path, self.weight_format)

    def load_weights_raw(self) -> Dict[str, np.ndarray]:
        return read_safetensors(self.weights_path)

    def load_config(self) -> dict:
        import yaml
        try:
            return yaml.safe_load(self.config_content)
        except Exception:
            return json.loads(self.config_content)

    def is_quantized(self) -> bool:
        return self.quantization is not None
