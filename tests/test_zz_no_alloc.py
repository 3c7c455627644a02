"""cppinf_linear_argmax_noalloc (static device scratch) against cppinf_linear_argmax (caller-provided scratch).

The no-alloc variant serves callers that cannot allocate device memory themselves (an allocator that owns the whole
device budget, an FFI binding without device buffers); its output must equal the scratch version's bit for bit.

Collected last on purpose: the static scratch is process-wide state on the device, so this file runs after every
other GPU test. Two calls in a row check that each call leaves the static counter re-armed for the next one.
"""

from __future__ import annotations

import numpy as np
import pytest

from _dev import seeded_bf16, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k,n", [(1024, 151936), (256, 5000)])
def test_noalloc_matches_scratch_version_twice(cuda, k, n):
    from cppinf_b200 import ops

    rng = np.random.default_rng(k + n)
    x1, x2 = to_dev(seeded_bf16(rng, (1, k))), to_dev(seeded_bf16(rng, (1, k)))
    w = to_dev(seeded_bf16(rng, (n, k), std=0.02))
    for x in (x1, x2):  # two calls in a row on the same static scratch
        want_token, want_logits = ops.linear_argmax(x, w, with_logits=True)
        got_token, got_logits = ops.linear_argmax_noalloc(x, w, with_logits=True)
        assert int(got_token.item()) == int(want_token.item())
        assert (to_host(got_logits) == to_host(want_logits)).all()
    assert int(ops.linear_argmax_noalloc(x1, w).item()) == int(ops.linear_argmax(x1, w).item())


def test_static_scratch_covers_the_largest_grid(cuda):
    from cppinf_b200 import capi

    lib = capi.load()
    # The argmax grid is capped at two CTAs per SM, so on this device every vocabulary size fits the static scratch
    # (16-byte header + 8 bytes per CTA, 1024 CTAs).
    assert lib.cppinf_linear_argmax_scratch_bytes(1 << 30, 1024) <= 16 + 8 * 1024
