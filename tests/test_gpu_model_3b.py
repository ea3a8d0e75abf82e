"""The 3B-shaped AR model of the headline benchmark (hidden 3072, 24 query / 8 KV heads, so
G = 3, intermediate 8192, vocabulary 84,000) with 2 of its 28 layers, decoded two rows per
weight pass exactly as the benchmark runs a CFG pair: each row its own cache, both rows
through the GEMVs, the fused QK norm + RoPE + KV append inside attention, and the LM head.
Teacher-forced logits are compared with the oracle's restatement of the reference decode
path (src/model.rs:523-591, src/model.rs:465-468) on bit-identical weights and KV.

  * short context (~300 positions after a GEMM prefill): the SIMT split-K attention;
  * long context (KV filled with seeded N(0,1) bf16 to 4,097 and 24,560 positions, the
    same values written into the oracle's caches): at 4,097 the cluster form of attention
    that the engine picks there, and with the cluster form turned off the pipelined
    tensor-core split-K loop (attn_mma_kernel) that also serves 24,560;
  * BASELINE's initialisation (every weight N(0, 0.02)) at the north_star tolerance,
    and unit-mean RMSNorm gains (logits of order one) at the noise-floor criterion.
"""
import copy
import os

import numpy as np
import pytest

from devoracle import copy_cache_to_oracle, floor_check, oracle_from_device, within_tolerance
from oracle import oracle as orc
from yue2_rs_b200 import Model, synth

pytestmark = pytest.mark.gpu


def config_3b_2layers():
    c = copy.copy(synth.config_c2())
    c.num_hidden_layers = 2
    return c


def pipelined_for(keys, rows, kvh):
    """The engine's choice of attention loop (attn_pipe_for_keys with splits_for): the
    pipelined tile loop once a warp streams about 1.5 tiles of 32 keys. Splits where
    kvh * rows >= 8: 8 up to 8,192 positions, 16 beyond; else two CTAs per SM's worth."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if kvh * rows >= 8:
        splits = 8 if keys <= 8192 else 16
    else:
        splits = max(1, min(64, (2 * sms) // (kvh * rows)))
    return 2 * keys >= 3 * 32 * 4 * splits


@pytest.fixture(scope="module")
def rng_ids():
    rng = np.random.default_rng(2024)
    v = synth.config_c2().vocab_size
    return rng.integers(0, v, 300).tolist(), rng.integers(0, v, 277).tolist(), rng.integers(0, v, 16).tolist()


def _models(norm_mean):
    cfg = config_3b_2layers()
    dev = Model.synthetic(cfg, seed=1, std=0.02, norm_mean=norm_mean, device=0)
    return cfg, dev, oracle_from_device(dev, cfg)


def _teacher_steps(dev, orcm, dcs, ocs, teacher, steps):
    """`steps` two-row device passes and the oracle's two single-row forwards per step."""
    out_dev, out_ref = [], []
    for s in range(steps):
        ids = [teacher[2 * s], teacher[2 * s + 1]]
        out_dev.append(dev.forward_rows(dcs, ids))
        out_ref.append(np.stack([orcm.forward([ids[r]], ocs[r]) for r in range(2)]))
    return np.array(out_dev), np.array(out_ref)


def test_short_context_two_rows_baseline_init(rng_ids):
    cond, uncond, teacher = rng_ids
    cfg, dev, orcm = _models(0.0)
    try:
        assert not pipelined_for(len(cond) + 8, 2, cfg.num_key_value_heads)
        dcs = [dev.new_cache(len(p) + 8) for p in (cond, uncond)]
        ocs = [orcm.cache(len(p) + 8) for p in (cond, uncond)]
        for p, dc, oc in zip((cond, uncond), dcs, ocs):
            within_tolerance(dev.forward(p, dc), orcm.prefill(p, oc), "prefill")
        a, b = _teacher_steps(dev, orcm, dcs, ocs, teacher, 6)
        for s in range(len(a)):
            for r in range(2):
                within_tolerance(a[s, r], b[s, r], (s, r))
        # the K/V rows agree with the oracle's up to bf16 rounding flips: another f32
        # summation order moves a rounded value by an ulp (K passes three more roundings
        # in the QK norm and RoPE). Layer 0 sees identical inputs; deeper layers also carry
        # the earlier layers' flips, so there only the relative distance is bounded.
        to_f = lambda x: (x.astype(np.uint32) << 16).view(np.float32)
        for layer in range(cfg.num_hidden_layers):
            kd, vd = dcs[0].read(layer, 0, dcs[0].length)
            ko, vo = ocs[0].read(layer)
            for dev_kv, ref_kv in ((to_f(kd), ko), (to_f(vd), vo)):
                rel = np.linalg.norm(dev_kv - ref_kv) / np.linalg.norm(ref_kv)
                assert rel <= 1e-2, (layer, rel)
                if layer == 0:
                    mag = np.maximum(np.abs(dev_kv), np.abs(ref_kv))
                    ulp = np.exp2(np.floor(np.log2(np.maximum(mag, 1e-30))) - 7)
                    assert np.mean(np.abs(dev_kv - ref_kv) <= 2 * ulp) >= 0.99
    finally:
        dev.close()
        orcm.close()


@pytest.mark.parametrize("length,cluster", [(4097, None), (4097, "0"), (24560, None)])
def test_long_context_two_rows_pipelined_attention(rng_ids, length, cluster):
    _, _, teacher = rng_ids
    old = os.environ.get("YUE2_CUDA_ATTN_CLUSTER")
    if cluster is not None:
        os.environ["YUE2_CUDA_ATTN_CLUSTER"] = cluster
    try:
        cfg, dev, orcm = _models(0.0)
    finally:
        if old is None:
            os.environ.pop("YUE2_CUDA_ATTN_CLUSTER", None)
        else:
            os.environ["YUE2_CUDA_ATTN_CLUSTER"] = old
    try:
        assert pipelined_for(length + 1, 2, cfg.num_key_value_heads)
        dcs = [dev.new_cache(length + 4) for _ in range(2)]
        ocs = [orcm.cache(length + 4) for _ in range(2)]
        for i, (dc, oc) in enumerate(zip(dcs, ocs)):
            dc.fill_normal(length, seed=31 + i)
            copy_cache_to_oracle(dc, oc, cfg, length)
        a, b = _teacher_steps(dev, orcm, dcs, ocs, teacher, 3)
        for s in range(len(a)):
            for r in range(2):
                within_tolerance(a[s, r], b[s, r], (length, s, r))
    finally:
        dev.close()
        orcm.close()


@pytest.mark.parametrize("length", [0, 4097])
def test_unit_gains_noise_floor(rng_ids, length):
    cond, uncond, teacher = rng_ids
    cfg, dev, orcm = _models(1.0)
    try:
        if length:
            dcs = [dev.new_cache(length + 8) for _ in range(2)]
            ocs = [orcm.cache(length + 8) for _ in range(2)]
            alts = [orcm.cache(length + 8) for _ in range(2)]
            for i in range(2):
                dcs[i].fill_normal(length, seed=41 + i)
                copy_cache_to_oracle(dcs[i], ocs[i], cfg, length)
                copy_cache_to_oracle(dcs[i], alts[i], cfg, length)
        else:
            dcs = [dev.new_cache(len(p) + 8) for p in (cond, uncond)]
            ocs = [orcm.cache(len(p) + 8) for p in (cond, uncond)]
            alts = [orcm.cache(len(p) + 8) for p in (cond, uncond)]
            for p, dc, oc, al in zip((cond, uncond), dcs, ocs, alts):
                dev.forward(p, dc)
                orcm.prefill(p, oc, logits=False)
                orc.set_dot_order(1)
                try:
                    orcm.prefill(p, al, logits=False)
                finally:
                    orc.set_dot_order(0)
        a, b = _teacher_steps(dev, orcm, dcs, ocs, teacher, 5)
        # the same steps through the oracle with strictly sequential dot products
        alt = []
        orc.set_dot_order(1)
        try:
            for s in range(5):
                alt.append(np.stack([orcm.forward([teacher[2 * s + r]], alts[r]) for r in range(2)]))
        finally:
            orc.set_dot_order(0)
        floor_check(a.reshape(-1, a.shape[-1]), b.reshape(-1, b.shape[-1]), np.array(alt).reshape(-1, a.shape[-1]))
    finally:
        dev.close()
        orcm.close()
