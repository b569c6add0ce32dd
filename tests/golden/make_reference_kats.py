"""Writes tests/golden/reference_kats.json: the known-answer values the
reference's own unit tests assert, transcribed with their file:line.

The reference (animaslabs/mlx-nemo-rs) is Rust over MLX/Metal and cannot run
in this container or on the GPU box, so its golden values are the literal
expectations in its test code plus the closed forms those tests compute
(sin/cos of known angles).  Run:  python tests/golden/make_reference_kats.py
"""
import json
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    kats = {}
    # attention.rs:927-998 test_rel_shift_correctness: seq_len 3, pos_len 5,
    # input row i = [5i .. 5i+4]; first three columns after rel_shift.
    kats["rel_shift_correctness"] = {
        "source": "src/asr/modules/encoders/attention.rs:927-998",
        "input_shape": [1, 1, 3, 5],
        "input": list(range(15)),
        "expected_first3": [[2.0, 3.0, 4.0], [6.0, 7.0, 8.0], [10.0, 11.0, 12.0]],
    }
    # attention.rs:918-924 test_rel_shift: shape preserved.
    kats["rel_shift_shape"] = {
        "source": "src/asr/modules/encoders/attention.rs:918-924",
        "input_shape": [1, 1, 4, 7],
        "expected_shape": [1, 1, 4, 7],
    }
    # attention.rs:1170-1246 test_rel_positional_encoding_values: d_model 4,
    # max_len 3, seq_len 3 -> [1,5,4]; row 0 is position 2, row 2 position 0.
    div1 = np.float32(math.exp(np.float32(-2.0) * np.float32(math.log(10000.0)) / np.float32(4.0)))
    pos = np.float32(2.0)
    kats["pe_values"] = {
        "source": "src/asr/modules/encoders/attention.rs:1170-1246",
        "d_model": 4, "max_len": 3, "seq_len": 3,
        "expected_shape": [1, 5, 4],
        "row0": [float(np.sin(pos)), float(np.cos(pos)),
                 float(np.sin(pos * div1)), float(np.cos(pos * div1))],
        "row2_first2": [0.0, 1.0],
        "tol": 1e-5,
    }
    kats["pe_shape"] = {
        "source": "src/asr/modules/encoders/attention.rs:908-915",
        "d_model": 512, "max_len": 100, "seq_len": 50,
        "expected_shape": [1, 99, 512],
    }
    kats["pe_xscale"] = {
        "source": "src/asr/modules/encoders/attention.rs:901-905",
        "d_model": 512, "expected": math.sqrt(512.0), "tol": 1e-5,
    }
    kats["pe_extends_past_max_len"] = {
        "source": "src/asr/modules/encoders/attention.rs:1151-1167",
        "d_model": 16, "short_max_len": 10, "long_max_len": 40, "seq_len": 25,
        "expected_shape": [1, 49, 16], "tol": 1e-6,
    }
    kats["pe_streaming_dimensions"] = {
        "source": "src/asr/modules/encoders/attention.rs:1338-1357",
        "d_model": 512, "max_len": 5000, "cache": 70, "seq_len": 14,
        "expected_shape": [1, 167, 512],
    }
    kats["rel_shift_property_standard"] = {
        "source": "src/asr/modules/encoders/attention.rs:1285-1291",
        "seq_lens": list(range(1, 9)),
    }
    kats["rel_shift_property_streaming"] = {
        "source": "src/asr/modules/encoders/attention.rs:1294-1303",
        "seq_lens": list(range(1, 7)), "cache_lens": list(range(1, 7)),
    }
    kats["rel_shift_no_padding_zeros"] = {
        "source": "src/asr/modules/encoders/attention.rs:1306-1335",
        "seq_len": 4, "total_len": 7, "min_value": 100.0,
    }
    kats["context_mask_matches_nemo"] = {
        "source": "src/asr/modules/encoders/attention.rs:1107-1148",
        "seq_len": 23, "start": 7, "end": 19,
        "cases": [[[56, 3], "chunked_limited"], [[5, 1], "chunked_limited"],
                  [[-1, 2], "chunked_limited"], [[4, -1], "chunked_limited"],
                  [[3, 2], "regular"], [[-1, 0], "regular"]],
        "none_case": [[-1, -1], "chunked_limited"],
    }
    kats["key_padding_mask"] = {
        "source": "src/asr/modules/encoders/attention.rs:1038-1040",
        "seq_len": 13, "padded_lengths": [13, 9], "full_lengths": [13, 13],
    }
    kats["padded_keys_are_ignored"] = {
        "source": "src/asr/modules/encoders/attention.rs:1026-1064",
        "d_model": 16, "n_heads": 2, "seq_len": 13, "valid": 9,
        "garbage": 50.0, "weight_scale": 0.3,
        "contexts": [None, [[3, 2], "regular"]],
        "tol_full": 1e-5, "tol_short": 1e-4,
    }
    kats["blocked_attention_matches_full"] = {
        "source": "src/asr/modules/encoders/attention.rs:1067-1104",
        "d_model": 16, "n_heads": 2, "seq_len": 13, "weight_scale": 0.3,
        "budget": 2 * 2 * 2 * 13 * 5, "expected_blocks": [5, 5, 3],
        "contexts": [None, [[4, 1], "chunked_limited"], [[3, 2], "regular"]],
        "tol": 1e-5,
    }
    kats["standard_linear_forward"] = {
        "source": "src/core/quantization.rs:414-430",
        "weight": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], "bias": [0.1, 0.2],
        "x": [[1.0, 1.0, 1.0]], "expected": [[6.1, 15.2]], "tol": 1e-5,
    }
    kats["quantization_config"] = {
        "source": "src/core/quantization.rs:463-468 and default (8,64) at 307",
        "bits": 8, "group_size": 64,
    }
    kats["encoder_cache_creation"] = {
        "source": "src/asr/streaming/core.rs:395-402",
        "num_layers": 24, "batch": 1, "channel_cache": 70, "time_cache": 8,
        "d_model": 1024,
    }
    kats["streaming_mode_info"] = {
        "source": "src/asr/streaming/core.rs:404-411",
        "mode_idx": 0, "left": 70, "right": 13, "frame_ms": 10.0,
        "expected_latency_ms": 130.0, "tol": 0.1,
    }
    kats["streaming_config_chunk_sizes"] = {
        "source": "src/asr/streaming/core.rs:413-436",
        "chunk_size": [100, 120], "shift_size": [80, 100],
        "pre_encode_cache_size": [0, 9],
    }
    path = os.path.join(HERE, "reference_kats.json")
    with open(path, "w") as f:
        json.dump(kats, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
