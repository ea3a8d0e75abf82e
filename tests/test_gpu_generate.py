"""sampling::generate on the device (one CUDA graph per token) against a step-by-step
replay: the same device logits (forward_rows), the oracle's CFG mix and the oracle's
choose with its own MT19937 -- tokens must match exactly."""
import numpy as np
import pytest

from oracle.oracle import OracleRng, cfg_mix
from oracle.oracle import choose as ochoose
from yue2_rs_b200 import Model, Phase, Request, Sampling, generate, generate_batch
from yue2_rs_b200 import synth

pytestmark = pytest.mark.gpu


def replay(model, prefix, negative, scale, s, seed, phase, legacy=False):
    cond = model.new_cache(len(prefix) + s.max_tokens)
    lc = model.forward_phase(prefix, cond, phase)
    uncond = lu = None
    if scale != 1.0:
        uncond = model.new_cache(len(negative) + s.max_tokens)
        lu = model.forward_phase(negative, uncond, phase)
    rng = OracleRng(seed)
    toks = []
    for step in range(s.max_tokens):
        mix = cfg_mix(lc, lu, scale) if uncond is not None else lc
        t = ochoose(mix, s, toks, step, int(phase), legacy, rng)
        if t == phase.end():
            return toks, False
        toks.append(t)
        if step + 1 < s.max_tokens:
            if uncond is not None:
                lc, lu = model.forward_rows([cond, uncond], [t, t], phase)
            else:
                lc = model.forward_rows([cond], [t], phase)[0]
    return toks, True


@pytest.mark.parametrize("temperature", [1.0, 0.0])
def test_generate_cfg_matches_replay(c1u_device, c1_prompt, temperature):
    prompt = c1_prompt[0][:40]
    negative = c1_prompt[0][200:230]
    s = Sampling(temperature, 0.93, 50, 1.2, 50, 0, 24)
    g = generate(c1u_device, prompt, s, 77, Phase.VOCAB, negative, 1.5)
    want, trunc = replay(c1u_device, prompt, negative, 1.5, s, 77, Phase.VOCAB)
    assert g.tokens == want and g.truncated and trunc and len(g.tokens) == 24


def replay_batch(model, reqs, s, phase):
    """The batched decode loop step by step: every row of every song stays in the weight
    pass until the last song ends (as on the device), so each row goes through the same
    GEMV path as in generate_batch."""
    rows, owner = [], []
    for i, r in enumerate(reqs):
        rows.append(model.new_cache(len(r.prefix) + s.max_tokens))
        owner.append((i, 0))
        if r.scale != 1.0:
            rows.append(model.new_cache(len(r.negative) + s.max_tokens))
            owner.append((i, 1))
    logits = [model.forward_phase(reqs[i].negative if k else reqs[i].prefix, c, phase)
              for c, (i, k) in zip(rows, owner)]
    rngs = [OracleRng(r.seed) for r in reqs]
    toks = [[] for _ in reqs]
    done = [False] * len(reqs)
    last = [0] * len(reqs)
    for step in range(s.max_tokens):
        for i, r in enumerate(reqs):
            if done[i]:
                continue
            lc = logits[owner.index((i, 0))]
            mix = cfg_mix(lc, logits[owner.index((i, 1))], r.scale) if r.scale != 1.0 else lc
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


def test_generate_without_cfg_and_batch(c1u_device, c1_prompt):
    p = c1_prompt[0]
    s = Sampling(1.0, 0.9, 40, 1.1, 20, 0, 12)
    reqs = [Request(p[:17], 5), Request(p[30:50], 6, p[60:70], 1.5), Request(p[80:90], 7, p[90:99], 2.0, True)]
    outs = generate_batch(c1u_device, reqs, s, Phase.VOCAB)
    want = replay_batch(c1u_device, reqs, s, Phase.VOCAB)
    for o, w in zip(outs, want):
        assert o.tokens == w


def test_generate_eight_songs_with_cfg(c1u_device, c1_prompt):
    """Eight songs with CFG: sixteen rows in every weight pass (the batched configuration)."""
    p = c1_prompt[0]
    s = Sampling(1.0, 0.93, 50, 1.1, 20, 0, 10)
    reqs = [Request(p[10 * i: 10 * i + 12 + i], 40 + i, p[150 + 7 * i: 160 + 7 * i], 1.5) for i in range(8)]
    outs = generate_batch(c1u_device, reqs, s, Phase.VOCAB)
    want = replay_batch(c1u_device, reqs, s, Phase.VOCAB)
    for o, w in zip(outs, want):
        assert o.tokens == w and len(o.tokens) == 10


def test_stop_token_ends_generation():
    """A zero LM head makes every logit 0: greedy picks the lowest eligible id, which is
    MUSIC_END (151852) as soon as step >= min_tokens, else CODEC_OFFSET."""
    c = synth.config_c1()
    c.vocab_size, c.num_hidden_layers = 184704, 1
    m = Model(c)
    from yue2_rs_b200 import _lib
    _lib.check(_lib.lib().yue2_model_init_synthetic(m._h, 3, 0.02, 1.0))
    m.set_tensor("lm_head.weight", np.zeros((c.vocab_size, c.hidden_size), dtype=np.uint16))
    m.finalize()
    s = Sampling(0.0, 0.95, 100, 1.2, 50, 5, 50)
    g = generate(m, [1, 2, 3, 4], s, 1, Phase.SEMANTIC, [5, 6], 1.5)
    assert g.tokens == [151853] * 5 and not g.truncated
    m.close()
