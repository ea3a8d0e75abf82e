"""Properties of the oracle's model.rs restatement on config 0 (the reduced model)."""
import numpy as np
import pytest

from oracle.oracle import OracleError


def test_chunked_prefill_equals_token_by_token(c1_oracle, c1_prompt):
    ids = c1_prompt[0][:24]
    a = c1_oracle.cache(64)
    la = c1_oracle.prefill(ids, a)
    b = c1_oracle.cache(64)
    for t in ids[:-1]:
        c1_oracle.forward([t], b)
    lb = c1_oracle.forward([ids[-1]], b)
    assert (la.view(np.uint32) == lb.view(np.uint32)).all()
    for layer in range(c1_oracle.config.num_hidden_layers):
        ka, va = a.read(layer)
        kb, vb = b.read(layer)
        assert (ka == kb).all() and (va == vb).all()


def test_logits_are_bf16_valued_and_finite(c1_oracle, c1_prompt):
    c = c1_oracle.cache(300)
    x = c1_oracle.prefill(c1_prompt[0][:8], c)
    assert np.isfinite(x).all()
    assert (x.view(np.uint32) & 0xFFFF == 0).all()
    assert 0.003 < float(np.std(x)) < 0.1  # config 0: every weight N(0, 0.02), gains included


def test_capacity_token_and_phase_errors(c1_oracle):
    c = c1_oracle.cache(2)
    c1_oracle.forward([1, 2], c)
    with pytest.raises(OracleError, match="exceeds cache"):
        c1_oracle.forward([3], c)
    with pytest.raises(OracleError, match="outside model vocabulary"):
        c1_oracle.forward([c1_oracle.config.vocab_size], c1_oracle.cache(4))
    with pytest.raises(OracleError, match="native music protocol"):
        c1_oracle.forward([1], c1_oracle.cache(4), phase=1)
