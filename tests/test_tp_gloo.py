"""Tensor parallelism's arithmetic on CPU with two gloo ranks, against the oracle's unsharded
layer math (Linear::apply/finish src/tensor.rs:946-1118, Mlp::apply src/model.rs:206-214,
the residual adds src/model.rs:586-587, the LM head src/model.rs:465-468).

Each rank holds the slices yue2_rs_b200.tp.shard_slices gives it. The o and down
projections leave f32 partial sums over the rank's input columns; gathered and added in
rank order, rounded once and added to the residual, they must match the oracle's rounded
full projection up to f32 summation order. The gate|up rows and the LM head's vocabulary
rows are whole on one rank, so those results must match bit for bit."""
import json
import os
import socket

import numpy as np
import torch.multiprocessing as mp

WORLD = 2


def _config():
    from yue2_rs_b200 import synth
    c = synth.config_c1()
    c.vocab_size, c.hidden_size, c.intermediate_size = 1000, 256, 512
    c.num_attention_heads, c.num_key_value_heads, c.head_dim = 4, 2, 64
    c.num_hidden_layers = 1
    return c


def _weights(c):
    rng = np.random.default_rng(5)
    bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32) * 0.05).view(np.uint32) >> 16
    return {"o": bits((c.hidden_size, c.num_attention_heads * c.head_dim)).astype(np.uint16),
            "gate": bits((c.intermediate_size, c.hidden_size)).astype(np.uint16),
            "up": bits((c.intermediate_size, c.hidden_size)).astype(np.uint16),
            "down": bits((c.hidden_size, c.intermediate_size)).astype(np.uint16),
            "head": bits((c.vocab_size, c.hidden_size)).astype(np.uint16)}


def _inputs(c):
    rng = np.random.default_rng(6)
    rb = lambda a: (a.astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
    return (rb(rng.standard_normal((2, c.num_attention_heads * c.head_dim))),  # attention output
            rb(rng.standard_normal((2, c.hidden_size))))                      # residual


def _f(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _rb(a):
    from refmath import round_bf16_np
    return round_bf16_np(np.asarray(a, dtype=np.float32))


def _rank_main(rank, world, port, path):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from oracle import oracle as orc
    from yue2_rs_b200.tp import shard_slices
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = _config()
    w = _weights(c)
    h, x = _inputs(c)
    sl = shard_slices(c, rank, world)
    blk = lambda a, name: a[sl[name][0]:sl[name][0] + sl[name][1], sl[name][2]:sl[name][2] + sl[name][3]]
    p = "model.layers.0."

    def allreduce_residual(part, resid):
        parts = [torch.zeros_like(torch.from_numpy(part)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        s = np.zeros_like(part)
        for q in range(world):  # rank order, as the device exchange adds them
            s += parts[q].numpy()
        return _rb(resid + _rb(s))

    # o: this rank's heads' columns of the attention output
    o0, _, oc0, ocs = sl[p + "self_attn.o_proj.weight"]
    part = h[:, oc0:oc0 + ocs] @ _f(blk(w["o"], p + "self_attn.o_proj.weight")).T
    x1 = allreduce_residual(part.astype(np.float32), x)
    # gate|up rows of this rank, SwiGLU with the oracle's rounding, then the down partial
    n = x1  # (the post-attention norm is whole on every rank; the identity keeps the test on the split)
    g = orc.linear(blk(w["gate"], p + "mlp.gate_proj.weight"), n)
    u = orc.linear(blk(w["up"], p + "mlp.up_proj.weight"), n)
    silu = _rb(g / (1.0 + np.exp(-g.astype(np.float64))).astype(np.float32))
    s_loc = _rb(silu * u)
    dpart = s_loc @ _f(blk(w["down"], p + "mlp.down_proj.weight")).T
    x2 = allreduce_residual(dpart.astype(np.float32), x1)
    # LM head: this rank's vocabulary rows, gathered
    v0, vr, _, _ = sl.get("lm_head.weight", (0, c.vocab_size, 0, c.hidden_size))
    lg = orc.linear(w["head"][v0:v0 + vr], x2)
    parts = [None] * world
    dist.all_gather_object(parts, lg.tolist())
    logits = np.concatenate([np.array(q, dtype=np.float32) for q in parts], axis=1)
    # silu for the unsharded reference as well, with the same expression
    res = {"x1": x1.tolist(), "x2": x2.tolist(), "logits": logits.tolist(), "g": g.tolist()}
    dist.barrier()
    dist.destroy_process_group()
    with open(f"{path}.{rank}", "w") as f:
        json.dump(res, f)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tensor_parallel_layer_matches_unsharded_oracle(tmp_path):
    from oracle import oracle as orc
    path = str(tmp_path / "tp")
    mp.start_processes(_rank_main, args=(WORLD, _free_port(), path), nprocs=WORLD, join=True, start_method="spawn")
    res = [json.load(open(f"{path}.{r}")) for r in range(WORLD)]
    c = _config()
    w = _weights(c)
    h, x = _inputs(c)
    x1 = _rb(x + orc.linear(w["o"], h))
    g = orc.linear(w["gate"], x1)
    u = orc.linear(w["up"], x1)
    silu = _rb(g / (1.0 + np.exp(-g.astype(np.float64))).astype(np.float32))
    x2 = _rb(x1 + orc.linear(w["down"], _rb(silu * u)))
    logits = orc.linear(w["head"], x2)
    for r in res:  # every rank ends with the same residual and logits
        for key, want, tol in (("x1", x1, 2 ** -7), ("x2", x2, 2 ** -6)):
            got = np.array(r[key], dtype=np.float32)
            rel = np.linalg.norm(got - want) / np.linalg.norm(want)
            assert rel <= tol, (key, rel)
            assert np.mean(got == want) > 0.9, key  # only f32 summation order differs
        got = np.array(r["logits"], dtype=np.float32)
        assert got.shape == logits.shape
        assert np.abs(got - logits).max() <= 0.05 * np.abs(logits).max()
    assert res[0]["x2"] == res[1]["x2"] and res[0]["logits"] == res[1]["logits"]
    # the vocabulary split is exact: rows never straddle ranks, so given the same input the
    # gathered logits equal the unsharded head's
    x2_tp = np.array(res[0]["x2"], dtype=np.float32)
    assert np.array_equal(np.array(res[0]["logits"], dtype=np.float32), orc.linear(w["head"], x2_tp))


def test_shard_slices_cover_every_tensor_once():
    from yue2_rs_b200.synth import tensor_specs
    from yue2_rs_b200.tp import shard_slices
    c = _config()
    c.num_hidden_layers = 2
    specs = {n: s for n, s, _ in tensor_specs(c) if n in shard_slices(c, 0, 1)}
    for world in (1, 2):
        cover = {n: np.zeros(s if len(s) == 2 else (1, s[0]), dtype=int) for n, s in specs.items()}
        for r in range(world):
            for n, (r0, nr, c0, nc) in shard_slices(c, r, world).items():
                cover[n][r0:r0 + nr, c0:c0 + nc] += 1
        for n, cv in cover.items():
            whole = n.startswith("model.embed") or "norm" in n
            assert (cv == (world if whole else 1)).all(), (n, world)
