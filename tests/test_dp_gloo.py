"""Data parallelism over songs on CPU: two gloo ranks, as bench.py --gpus 2 runs them with
NCCL. Checks the song partition, the timing reductions (max over ranks) and the whole-job
throughput, and that sharding songs over ranks does not change any song's tokens: each
rank decodes its songs with the oracle (standing in for the device; the decode path has
no data-path collective), and the union equals one rank decoding all songs."""
import json
import os
import socket

import pytest
import torch.multiprocessing as mp

N_SONGS, STEPS = 5, 4


def _config():
    from yue2_rs_b200 import synth
    c = synth.config_c1()
    c.vocab_size, c.hidden_size, c.intermediate_size = 512, 128, 256
    c.num_attention_heads, c.num_key_value_heads, c.head_dim = 4, 2, 64
    c.num_hidden_layers = 1
    return c


def _decode_songs(indices):
    """Tokens of songs `indices` (CFG, sampled), decoded with the oracle."""
    import numpy as np

    from oracle import oracle as orc
    from yue2_rs_b200 import Phase, Sampling
    m = orc.OracleModel.synthetic(_config(), seed=3)
    s = Sampling(1.0, 0.9, 20, 1.1, 8, 0, STEPS)
    out = {}
    for i in indices:
        rng_ids = np.random.default_rng(100 + i)
        prefix, negative = rng_ids.integers(0, 512, 6).tolist(), rng_ids.integers(0, 512, 4).tolist()
        c, u = m.cache(len(prefix) + STEPS), m.cache(len(negative) + STEPS)
        lc, lu = m.forward(prefix, c), m.forward(negative, u)
        g, toks = orc.OracleRng(7 + i), []
        for step in range(STEPS):
            t = orc.choose(orc.cfg_mix(lc, lu, 1.5), s, toks, step, int(Phase.VOCAB), False, g)
            toks.append(t)
            if step + 1 < STEPS:
                lc, lu = m.forward([t], c), m.forward([t], u)
        out[i] = toks
    m.close()
    return out


def _rank_main(rank, world, port, path):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from yue2_rs_b200.dp import DataParallel
    dp = DataParallel("gloo")
    mine = dp.songs(N_SONGS)
    toks = _decode_songs(mine)
    seconds = 1.0 + rank  # stand-in for this rank's timed region
    res = {"rank": dp.rank, "world": dp.world, "songs": mine, "tokens": {str(k): v for k, v in toks.items()},
           "max": dp.max(seconds), "sum": dp.sum(len(mine) * STEPS),
           "throughput": dp.throughput(len(mine) * STEPS, seconds)}
    dp.barrier()
    dp.close()
    with open(f"{path}.{rank}", "w") as f:
        json.dump(res, f)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_songs_shard_over_two_gloo_ranks(tmp_path):
    world, path = 2, str(tmp_path / "dp")
    mp.start_processes(_rank_main, args=(world, _free_port(), path), nprocs=world, join=True, start_method="spawn")
    res = [json.load(open(f"{path}.{r}")) for r in range(world)]
    songs = sorted(i for r in res for i in r["songs"])
    assert songs == list(range(N_SONGS))  # every song exactly once
    assert res[0]["songs"] == [0, 2, 4] and res[1]["songs"] == [1, 3]
    for r in res:
        assert r["world"] == world and r["max"] == 2.0 and r["sum"] == N_SONGS * STEPS
        assert abs(r["throughput"] - N_SONGS * STEPS / 2.0) < 1e-9
    sharded = {int(k): v for r in res for k, v in r["tokens"].items()}
    assert sharded == _decode_songs(range(N_SONGS))
