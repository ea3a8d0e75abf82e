"""Decode passes of three or more rows (several songs per GPU): the forward runs as
tensor-core GEMMs over all rows (gemm_rows.cu) instead of the weight-streaming GEMV.

  * logits against the oracle's decode path within the north_star tolerance, at 18 rows
    (cuBLASLt GEMMs) and 6 rows (the skinny tcgen05 GEMMs);
  * logits against the GEMV path on the same caches and ids (two passes of 10 rows);
  * the codec-window phase: window + stop row equal to the GEMV path's, -inf elsewhere;
  * generate_batch with 10 songs and CFG (20 rows) replays exactly against forward_rows
    (the same wide pass), the oracle's CFG mix and the oracle's choose.
"""
import numpy as np
import pytest

from oracle.oracle import OracleRng, cfg_mix
from oracle.oracle import choose as ochoose
from yue2_rs_b200 import Model, Phase, Request, Sampling, generate_batch, synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def _prompts(c1_prompt, n):
    p = c1_prompt[0]
    return [p[7 * i: 7 * i + 9 + (i % 5)] for i in range(n)]


def _caches(model, prompts, extra, phase=Phase.VOCAB):
    cs = [model.new_cache(len(q) + extra) for q in prompts]
    for c, q in zip(cs, prompts):
        model.forward_phase(q, c, phase)
    return cs


@pytest.mark.parametrize("rows", [18, 6])  # 6: the skinny tcgen05 GEMMs (default up to 16 rows)
def test_wide_rows_match_oracle(c1_device, c1_oracle, c1_prompt, rows):
    prompts = _prompts(c1_prompt, rows)
    teacher = c1_prompt[1]
    cs = _caches(c1_device, prompts, 3)
    ocs = [c1_oracle.cache(len(q) + 3) for q in prompts]
    for oc, q in zip(ocs, prompts):
        c1_oracle.prefill(q, oc, logits=False)
    for step in range(3):
        ids = [teacher[(step * rows + r) % len(teacher)] for r in range(rows)]
        dev = c1_device.forward_rows(cs, ids)
        for r in range(rows):
            ref = c1_oracle.forward([ids[r]], ocs[r])
            d = np.abs(dev[r].astype(np.float64) - ref)
            assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (step, r, d.max(), d.mean())


def test_wide_rows_match_gemv_rows(c1u_device, c1_prompt):
    prompts = _prompts(c1_prompt, 20)
    teacher = c1_prompt[1]
    wide = _caches(c1u_device, prompts, 4)
    narrow = _caches(c1u_device, prompts, 4)
    for step in range(4):
        ids = [teacher[(step * 20 + r) % len(teacher)] for r in range(20)]
        a = c1u_device.forward_rows(wide, ids)
        b = np.concatenate([c1u_device.forward_rows(narrow[:10], ids[:10]),
                            c1u_device.forward_rows(narrow[10:], ids[10:])])
        assert np.isfinite(a).all()
        # same roundings, other f32 summation order (unit gains: most logits within an ulp)
        assert np.abs(a - b).max() <= 0.08 and np.abs(a - b).mean() <= 1e-2
        assert (a.argmax(-1) == b.argmax(-1)).mean() >= 0.9


def test_wide_rows_codec_window():
    c = synth.config_c1()
    c.vocab_size, c.num_hidden_layers = 184704, 1
    m = Model.synthetic(c, seed=5, std=0.02, norm_mean=1.0)
    try:
        prompts = [[3 + i, 40 + i, 700 + 3 * i] for i in range(18)]
        wide = _caches(m, prompts, 2, Phase.SEMANTIC)
        narrow = _caches(m, prompts, 2, Phase.SEMANTIC)
        ids = [151900 + 13 * r for r in range(18)]
        a = m.forward_rows(wide, ids, Phase.SEMANTIC)
        b = np.concatenate([m.forward_rows(narrow[:9], ids[:9], Phase.SEMANTIC),
                            m.forward_rows(narrow[9:], ids[9:], Phase.SEMANTIC)])
        keep = np.zeros(c.vocab_size, dtype=bool)
        keep[151853:151853 + 32768] = True
        keep[151852] = True
        assert np.isneginf(a[:, ~keep]).all() and np.isfinite(a[:, keep]).all()
        assert np.abs(a[:, keep] - b[:, keep]).max() <= 0.08
        assert np.abs(a[:, keep] - b[:, keep]).mean() <= 1e-2
    finally:
        m.close()


def _replay(model, reqs, s, phase):
    """The batched loop step by step with every row in each pass (as on the device)."""
    rows, owner = [], []
    for i, r in enumerate(reqs):
        rows.append(model.new_cache(len(r.prefix) + s.max_tokens))
        owner.append((i, 0))
        rows.append(model.new_cache(len(r.negative) + s.max_tokens))
        owner.append((i, 1))
    logits = [model.forward_phase(reqs[i].negative if k else reqs[i].prefix, c, phase) for c, (i, k) in zip(rows, owner)]
    rngs = [OracleRng(r.seed) for r in reqs]
    toks = [[] for _ in reqs]
    done = [False] * len(reqs)
    last = [0] * len(reqs)
    for step in range(s.max_tokens):
        for i, r in enumerate(reqs):
            if done[i]:
                continue
            mix = cfg_mix(logits[2 * i], logits[2 * i + 1], r.scale)
            t = ochoose(mix, s, toks[i], step, int(phase), r.legacy, rngs[i])
            if t == phase.end():
                done[i] = True
                continue
            toks[i].append(t)
            last[i] = t
            if step + 1 >= s.max_tokens:
                done[i] = True
        if all(done):
            break
        out = model.forward_rows(rows, [last[i] for i, _ in owner], phase)
        logits = [out[j] for j in range(len(rows))]
    return toks


def test_generate_ten_songs_with_cfg_matches_replay(c1u_device, c1_prompt):
    p = c1_prompt[0]
    s = Sampling(1.0, 0.93, 50, 1.1, 20, 0, 8)
    reqs = [Request(p[9 * i: 9 * i + 10 + i], 60 + i, p[180 + 5 * i: 190 + 5 * i], 1.5) for i in range(10)]
    outs = generate_batch(c1u_device, reqs, s, Phase.VOCAB)
    want = _replay(c1u_device, reqs, s, Phase.VOCAB)
    for o, w in zip(outs, want):
        assert o.tokens == w and len(o.tokens) == 8


def test_wide_rows_on_skinny_tcgen05_gemms():
    """The oracle, GEMV-agreement and replay cases above with every GEMM of <= 256 rows on
    the skinny tcgen05 kernel (YUE2_CUDA_SKINNY=1: q|k|v, o, gate|up with the SwiGLU
    epilogue, down and the LM head). The switch is read when a model is created, so the
    cases rerun in a child process."""
    import os
    import subprocess
    import sys
    if os.environ.get("YUE2_CUDA_SKINNY"):
        pytest.skip("this process already runs with the switch set")
    env = dict(os.environ, YUE2_CUDA_SKINNY="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", os.path.abspath(__file__),
                        "-m", "gpu", "-k", "match_oracle or match_gemv_rows or matches_replay"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "4 passed" in r.stdout, r.stdout[-2000:]
