"""Extracts the golden cases of the reference's attention and decoder-block tests into tests/golden/ref_blocks.npz.

    python tests/golden/make_block_golden.py [reference tree]

Reads tests/nn/qwen_attention_test.cpp and tests/nn/qwen_decoder_block_test.cpp of the reference as text (the values
there come from the reference's Hugging Face oracles, tests/nn/qwen_attention_oracle.py and
qwen_decoder_block_oracle.py) and stores, per test case that has expected values:

    <case>/meta      [kind (0 attention, 1 decoder block), dtype (0 f32, 1 bf16), heads, kv_heads, head_dim,
                      seq_len, eps, tolerance]
    <case>/<tensor>  every make_f32_tensor / make_bf16_tensor of the case, as f32 with its dims
    <case>/expected  the values expect_float_values_near checks ([seq_len, hidden] of batch row 0)
"""

from __future__ import annotations

import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
TENSOR = re.compile(r'make_(f32|bf16)_tensor\(\s*"(\w+)"\s*,\s*\{([^}]*)\}\s*,\s*\{([^}]*)\}\s*\)', re.S)
CALL = re.compile(r'qwen_(attention|decoder_block)_with_cache\([^,]+,\s*sequence_lengths,\s*weights,\s*cache,\s*'
                  r'(\d+),\s*(\d+),\s*(\d+),\s*([0-9.e+-]+)f\s*\)', re.S)
EXPECT = re.compile(r'expect_float_values_near\(\s*squeeze\(result\.view\(\),\s*0\),\s*\{([^}]*)\}\s*,\s*([0-9.e+-]+)f',
                    re.S)
SEQ = re.compile(r'sequence_lengths\s*=\s*\{(\d+)\}')


def numbers(text: str) -> list[float]:
    return [float(v.rstrip("f")) for v in re.findall(r"-?\d+(?:\.\d*)?(?:e[+-]?\d+)?f?", text)]


def cases(path: Path, kind: int):
    text = path.read_text()
    parts = re.split(r"\nTEST_F\(\w+,\s*(\w+)\)", text)
    for name, body in zip(parts[1::2], parts[2::2]):
        expect = EXPECT.search(body)
        call = CALL.search(body)
        if expect is None or call is None:
            continue  # error-path tests: no golden values
        tensors = {}
        dtype = 0
        for kind_s, tname, dims, values in TENSOR.findall(body):
            d = [int(v) for v in numbers(dims)]
            v = np.array(numbers(values), np.float32)
            assert v.size == int(np.prod(d)), (name, tname)
            tensors[tname] = v.reshape(d)
            dtype = 1 if kind_s == "bf16" else dtype
        heads, kv_heads, head_dim, eps = int(call.group(2)), int(call.group(3)), int(call.group(4)), float(call.group(5))
        seq = int(SEQ.search(body).group(1))
        meta = np.array([kind, dtype, heads, kv_heads, head_dim, seq, eps, float(expect.group(2))], np.float64)
        yield name, meta, tensors, np.array(numbers(expect.group(1)), np.float32)


def main() -> None:
    sys.path.insert(0, str(HERE.parent.parent))
    from oracle.oracle import reference_tree

    tree = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_tree()
    if tree is None:
        sys.exit("usage: make_block_golden.py <reference tree> (or set CPPINF_REFERENCE_DIR)")
    out = {}
    for rel, kind in (("tests/nn/qwen_attention_test.cpp", 0), ("tests/nn/qwen_decoder_block_test.cpp", 1)):
        for name, meta, tensors, expected in cases(tree / rel, kind):
            out[f"{name}/meta"] = meta
            out[f"{name}/expected"] = expected
            for tname, arr in tensors.items():
                out[f"{name}/{tname}"] = arr
            print(name, "kind", kind, "tensors", sorted(tensors))
    np.savez_compressed(HERE / "ref_blocks.npz", **out)
    print("wrote", HERE / "ref_blocks.npz")


if __name__ == "__main__":
    main()
