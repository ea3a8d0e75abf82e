"""Tensor parallelism on the device (yue2_model_create_tp, yue2_tp_connect).

  * one GPU: a rank's synthetic shard holds exactly the unsharded model's values at the
    positions yue2_rs_b200.tp.shard_slices gives it, and a filled KV cache holds the
    unsharded fill of its heads;
  * two GPUs (skipped with fewer): two ranks decode a CFG pair through the peer-memory
    exchanges; both ranks' logits are identical, and within the north_star tolerance of the
    unsharded model's on the same weights and ids (the o and down sums take another f32
    order), and generation through sessions runs on both ranks in step.
"""
import json
import os
import socket

import numpy as np
import pytest

from yue2_rs_b200 import synth

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def _config():
    c = synth.config_c1()  # 2 layers, hidden 1024, 8/2 heads of 128, intermediate 2816, vocab 84,000
    return c


def test_shard_holds_the_unsharded_values():
    from yue2_rs_b200 import Model
    from yue2_rs_b200.tp import shard_slices
    c = _config()
    full = Model.synthetic(c, seed=9, std=0.02, norm_mean=1.0, device=0)
    try:
        specs = {n: s for n, s, _ in synth.tensor_specs(c)}
        for rank in range(2):
            part = Model.synthetic(c, seed=9, std=0.02, norm_mean=1.0, device=0, tp=(rank, 2))
            try:
                for name, (r0, nr, c0, nc) in shard_slices(c, rank, 2).items():
                    shape = specs[name] if len(specs[name]) == 2 else (1, specs[name][0])
                    whole = full.get_tensor(name, int(np.prod(shape))).reshape(shape)
                    got = part.get_tensor(name, nr * nc).reshape(nr, nc)
                    assert np.array_equal(got, whole[r0:r0 + nr, c0:c0 + nc]), name
                # a filled cache holds the unsharded fill of this rank's KV heads
                fc, pc = full.new_cache(70), part.new_cache(70)
                fc.fill_normal(70, seed=3)
                pc.fill_normal(70, seed=3)
                w = c.num_key_value_heads // 2 * c.head_dim
                for layer in range(c.num_hidden_layers):
                    kf, vf = fc.read(layer, 0, 70)
                    kp, vp = pc.read(layer, 0, 70)
                    assert np.array_equal(kp, kf[:, rank * w:(rank + 1) * w])
                    assert np.array_equal(vp, vf[:, rank * w:(rank + 1) * w])
            finally:
                part.close()
    finally:
        full.close()


def _two_gpus():
    import torch
    return torch.cuda.device_count() >= 2


def _rank_main(rank, world, port, path):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from yue2_rs_b200 import Model, Phase, Request, Sampling, generate_batch, tp
    c = _config()
    m = Model.synthetic(c, seed=9, std=0.02, device=rank, tp=(rank, world))
    tp.connect(m)
    rng = np.random.default_rng(4)
    cond, unc, teacher = (rng.integers(0, c.vocab_size, 7).tolist(), rng.integers(0, c.vocab_size, 5).tolist(),
                          rng.integers(0, c.vocab_size, 8).tolist())
    cc, uc = m.new_cache(32), m.new_cache(32)
    out = [m.forward(cond, cc).tolist(), m.forward(unc, uc).tolist()]
    for s in range(4):
        out.append(m.forward_rows([cc, uc], [teacher[2 * s], teacher[2 * s + 1]]).tolist())
    g = generate_batch(m, [Request(cond, seed=5, negative=unc, scale=1.5)], Sampling(1.0, 0.93, 50, 1.0, 50, 0, 12),
                       Phase.VOCAB)
    res = {"logits": out, "tokens": g[0].tokens}
    dist.barrier()
    m.close()
    dist.destroy_process_group()
    with open(f"{path}.{rank}", "w") as f:
        json.dump(res, f)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not _two_gpus(), reason="tensor parallelism needs two GPUs")
def test_two_ranks_match_the_unsharded_model(tmp_path):
    import torch.multiprocessing as mp

    from yue2_rs_b200 import Model
    path = str(tmp_path / "tp")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    res = [json.load(open(f"{path}.{r}")) for r in range(2)]
    assert res[0]["logits"] == res[1]["logits"] and res[0]["tokens"] == res[1]["tokens"]
    assert len(res[0]["tokens"]) == 12
    c = _config()
    m = Model.synthetic(c, seed=9, std=0.02, device=0)
    try:
        rng = np.random.default_rng(4)
        cond, unc, teacher = (rng.integers(0, c.vocab_size, 7).tolist(), rng.integers(0, c.vocab_size, 5).tolist(),
                              rng.integers(0, c.vocab_size, 8).tolist())
        cc, uc = m.new_cache(32), m.new_cache(32)
        want = [m.forward(cond, cc), m.forward(unc, uc)]
        for s in range(4):
            want.extend(m.forward_rows([cc, uc], [teacher[2 * s], teacher[2 * s + 1]]))
    finally:
        m.close()
    got = [np.array(x, dtype=np.float32) for x in res[0]["logits"][:2]]
    for x in res[0]["logits"][2:]:
        got.extend(np.array(x, dtype=np.float32))
    for a, b in zip(got, want):
        d = np.abs(a.astype(np.float64) - b)
        assert np.isfinite(a).all() and d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (d.max(), d.mean())
