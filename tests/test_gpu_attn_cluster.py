"""The cluster form of decode attention (thread-block clusters that merge their partials in
distributed shared memory) against the oracle's restatement of the reference decode path
(src/model.rs:314-397 attention, src/model.rs:523-591 hidden), on the 3B shape's grouped
heads (24 query / 8 KV heads, G = 3, head_dim 128) with 2 of its 28 layers, two rows per
weight pass as in the CFG pair.

YUE2_CUDA_ATTN_CLUSTER forces the CTAs per (kv head, row) when the model is created, so each
case runs one cluster size over:
  * decode positions that cross a 32-key tile edge and a 64-position page edge (the new
    position's K and V come from shared memory, the rest of its tile from the cache);
  * more CTAs than tiles (ranks whose partial is empty);
  * more tiles than warps in a CTA (warps that take a second tile after the first).
Logits must meet the north_star tolerance at every step, and the split-K kernel (cluster
form off) must agree with the same oracle. Two cases use head_dim 64 with G = 4, the
kernel's other tile width: a forced size over tile and page edges, and the engine's own
choice of size."""
import copy
import os

import numpy as np
import pytest

from devoracle import copy_cache_to_oracle, oracle_from_device, within_tolerance
from yue2_rs_b200 import Model, synth

pytestmark = pytest.mark.gpu


def _config():
    c = copy.copy(synth.config_c2())
    c.num_hidden_layers = 2
    return c


def _config_d64():
    """head_dim 64 and G = 4 (16 query / 4 KV heads), the cluster kernel's other tile width."""
    return synth.Config(hidden_size=1024, num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=4,
                        head_dim=64, intermediate_size=2048, vocab_size=8192, rms_norm_eps=1e-6,
                        rope_theta=10000.0, max_position_embeddings=4096, max_latent_frames=4)


def _model(cluster, cfg=None):
    old = os.environ.get("YUE2_CUDA_ATTN_CLUSTER")
    os.environ["YUE2_CUDA_ATTN_CLUSTER"] = str(cluster)
    try:
        cfg = cfg or _config()
        return cfg, Model.synthetic(cfg, seed=1, std=0.02, norm_mean=0.0, device=0)
    finally:
        if old is None:
            del os.environ["YUE2_CUDA_ATTN_CLUSTER"]
        else:
            os.environ["YUE2_CUDA_ATTN_CLUSTER"] = old


# (cluster size, how each row's cache is made, decode steps): ("prompt", n) prefills n ids on
# both sides; ("fill", n) fills n positions with seeded N(0, 1) bf16 K/V and copies them to
# the oracle's caches
CASES = [
    (6, (("prompt", 60), ("prompt", 29)), 6),  # positions 60..65, 29..34: tile and page edges; empty ranks
    (2, (("prompt", 95), ("prompt", 63)), 4),  # 3 and 2 tiles over two CTAs
    (1, (("prompt", 300), ("prompt", 281)), 3),  # 10 tiles in one CTA: warps 0 and 1 take a second tile
    (6, (("fill", 1030), ("fill", 1009)), 3),  # the headline context: one tile per warp
    (6, (("fill", 2040), ("fill", 1985)), 3),  # 64 tiles over six CTAs: second tiles per warp
    (0, (("prompt", 60), ("prompt", 29)), 6),  # the split-K ticket kernel on the same positions
]


D64 = [
    (3, (("prompt", 62), ("prompt", 31)), 4),  # head_dim 64: tile and page edges over three CTAs
    (-1, (("fill", 700), ("fill", 650)), 3),   # the engine's own choice of cluster size
]


@pytest.mark.parametrize("cluster,rows,steps,d64", [c + (False,) for c in CASES] + [c + (True,) for c in D64])
def test_cluster_attention_matches_oracle(cluster, rows, steps, d64):
    cfg, dev = _model(cluster, _config_d64() if d64 else None)
    orcm = oracle_from_device(dev, cfg)
    try:
        rng = np.random.default_rng(cluster * 31 + rows[0][1])
        teacher = rng.integers(0, cfg.vocab_size, 2 * steps).tolist()
        dcs = [dev.new_cache(n + steps + 2) for _, n in rows]
        ocs = [orcm.cache(n + steps + 2) for _, n in rows]
        for i, ((kind, n), dc, oc) in enumerate(zip(rows, dcs, ocs)):
            if kind == "fill":
                dc.fill_normal(n, seed=71 + i)
                copy_cache_to_oracle(dc, oc, cfg, n)
            else:
                p = rng.integers(0, cfg.vocab_size, n).tolist()
                within_tolerance(dev.forward(p, dc), orcm.prefill(p, oc), "prefill")
        for s in range(steps):
            pair = [teacher[2 * s], teacher[2 * s + 1]]
            got = dev.forward_rows(dcs, pair)
            for r in range(2):
                want = orcm.forward([pair[r]], ocs[r])
                within_tolerance(got[r], want, f"cluster {cluster} step {s} row {r}")
    finally:
        dev.close()
        orcm.close()
