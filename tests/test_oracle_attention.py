"""The oracle's decode attention against the reference's own golden test
(src/tensor.rs:7-83, cached_attention_covers_long_context_and_append)."""
import os

import numpy as np
import pytest

from golden.make_golden import attention_inputs
from oracle.oracle import attention

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_ref.npz")


def cases():
    for dim in (64, 128, 256):
        for keys in (4096, 4097, 7169, 24576):
            for append in (0, 1) if keys < 24576 else (0,):
                yield dim, keys, append


@pytest.mark.parametrize("dim,keys,append", list(cases()))
def test_oracle_attention_matches_reference_test(dim, keys, append):
    heads, kv = 4, 2
    q, k, v = attention_inputs(heads, kv, dim, keys, append)
    want = np.load(GOLDEN)[f"d{dim}_k{keys}_a{append}"]
    got = attention(q, k, v, heads, kv, dim)
    assert np.all(np.abs(got - want) <= 5e-5 + np.abs(want) * 0.008)
