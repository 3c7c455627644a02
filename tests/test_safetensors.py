"""The safetensors reader behind cppinf_qwen3_load_safetensors, host side (no GPU): the reference's own test cases
(tests/files/safetensors_file_test.cpp) and the reference's real Qwen3-0.6B logits file when the reference tree is
present."""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import pytest

from cppinf_b200 import capi


def write_raw(path: Path, header: str, data: bytes) -> Path:
    h = header.encode()
    path.write_bytes(struct.pack("<Q", len(h)) + h + data)
    return path


def test_valid_file_with_metadata(tmp_path):
    # safetensors_file_test.cpp:32-57
    header = ('{"__metadata__":{"format":"pt"},"embed":{"dtype":"BF16","shape":[2,4],"data_offsets":[0,16]},'
              '"tail":{"dtype":"F32","shape":[1],"data_offsets":[16,20]}}')
    path = write_raw(tmp_path / "w.safetensors", header, bytes(range(0x10, 0x24)))
    count, offset = capi.safetensors_info(path)
    assert count == 2 and offset == 8 + len(header)


def test_invalid_range_and_unsupported_dtype(tmp_path):
    # safetensors_file_test.cpp:106-127
    with pytest.raises(ValueError, match="extends beyond the file data"):
        capi.safetensors_info(write_raw(tmp_path / "a", '{"weights":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}',
                                        b"\x00\x01"))
    with pytest.raises(ValueError, match="Unsupported dtype"):
        capi.safetensors_info(write_raw(tmp_path / "b", '{"weights":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}',
                                        b"\x00\x01\x02\x03"))


@pytest.mark.parametrize("header,data,message", [
    ('{"w":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', b"\x00" * 8, "does not match dtype and shape"),
    ('{"w":{"dtype":"F32","shape":[1],"data_offsets":[4,0]}}', b"\x00" * 8, "non-negative and ordered"),
    ('{"w":{"dtype":"F32","shape":[1],"data_offsets":[0]}}', b"\x00" * 4, "exactly two integers"),
    ('{"w":{"dtype":"F32","shape":1,"data_offsets":[0,4]}}', b"\x00" * 4, "shape must be an array"),
    ('{"w":[1,2]}', b"", "Tensor entries must be JSON objects"),
    ('[1,2]', b"", "must be a JSON object"),
    ('{"__metadata__":{"a":1}}', b"", "values must be strings"),
    ('{"w":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},"w":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}',
     b"\x00" * 4, "Duplicate tensor names"),
    ('{"w":', b"", "Failed to parse safetensors header"),
])
def test_header_errors(tmp_path, header, data, message):
    with pytest.raises(ValueError, match=message):
        capi.safetensors_info(write_raw(tmp_path / "x", header, data))


def test_short_files(tmp_path):
    (tmp_path / "short").write_bytes(b"\x01\x02")
    with pytest.raises(ValueError, match="8-byte header length"):
        capi.safetensors_info(tmp_path / "short")
    (tmp_path / "long").write_bytes(struct.pack("<Q", 100) + b"{}")
    with pytest.raises(ValueError, match="extends beyond the file size"):
        capi.safetensors_info(tmp_path / "long")


def test_writer_round_trip(tmp_path):
    from cppinf_b200.qwen3 import write_safetensors

    path = tmp_path / "rt.safetensors"
    write_safetensors(path, {"a": np.arange(6, dtype=np.uint16).reshape(2, 3), "b": np.ones(5, np.float32)},
                      {"format": "pt"})
    assert capi.safetensors_info(path)[0] == 2


def test_reference_real_logits_file():
    # The reference's own safetensors asset (tests/models/qwen3/qwen3_real_model_oracle.py writes it): one bf16
    # tensor of the 151,936 last-token logits.
    from oracle.oracle import reference_tree

    tree = reference_tree()
    if tree is None:
        pytest.skip("reference tree not present")
    path = tree / "tests/models/qwen3/qwen3_real_last_token_logits.safetensors"
    count, offset = capi.safetensors_info(path)
    assert count == 1
    assert path.stat().st_size - offset == 151936 * 2
