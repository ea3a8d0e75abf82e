"""Tensor parallelism across processes, one GPU each (yue2_model_create_tp).

    model = Model.synthetic(cfg, seed, device=local_rank, tp=(rank, world))
    tp.connect(model, group)    # every rank, after construction

`connect` exchanges the ranks' CUDA IPC handles over a torch.distributed process group (any
backend; the handles are 128 bytes per rank) and maps every peer's exchange and logits
buffers. From then on every rank makes the same decode calls in the same order; each holds
identical logits and samples identical tokens.
"""
import ctypes

from . import _lib


def export_handles(model):
    buf = ctypes.create_string_buffer(128)
    _lib.check(_lib.lib().yue2_tp_export(model._h, buf))
    return buf.raw


def connect_handles(model, handles):
    """handles: one 128-byte string per rank, in rank order."""
    assert len(handles) == model.tp[1] and all(len(h) == 128 for h in handles)
    blob = ctypes.create_string_buffer(b"".join(handles), 128 * len(handles))
    _lib.check(_lib.lib().yue2_tp_connect(model._h, blob))


def connect(model, group=None):
    import torch.distributed as dist
    mine = export_handles(model)
    world = model.tp[1]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine, group=group)
    connect_handles(model, gathered)


def shard_slices(config, rank, world):
    """The block of every full AR tensor that rank `rank` of `world` holds, as
    {name: (row0, rows, col0, cols)} over the full [rows, cols] tensor (norm gains and the
    embedding whole): q|k|v and gate|up split by output rows (heads, MLP rows), o and down
    by input columns, the LM head by vocabulary rows. Use it to slice checkpoint tensors
    for Model.set_tensor on a tensor-parallel model."""
    c = config
    H, D, V = c.hidden_size, c.head_dim, c.vocab_size
    qd, kd, I = c.num_attention_heads * D // world, c.num_key_value_heads * D // world, c.intermediate_size // world
    out = {"model.embed_tokens.weight": (0, V, 0, H), "model.norm.weight": (0, 1, 0, H)}
    v0, v1 = V * rank // world, V * (rank + 1) // world
    if not c.tie_word_embeddings:
        out["lm_head.weight"] = (v0, v1 - v0, 0, H)
    for l in range(c.num_hidden_layers):
        p = f"model.layers.{l}."
        out[p + "self_attn.q_proj.weight"] = (rank * qd, qd, 0, H)
        out[p + "self_attn.k_proj.weight"] = (rank * kd, kd, 0, H)
        out[p + "self_attn.v_proj.weight"] = (rank * kd, kd, 0, H)
        out[p + "self_attn.o_proj.weight"] = (0, H, rank * qd, qd)
        out[p + "mlp.gate_proj.weight"] = (rank * I, I, 0, H)
        out[p + "mlp.up_proj.weight"] = (rank * I, I, 0, H)
        out[p + "mlp.down_proj.weight"] = (0, H, rank * I, I)
        for n in ("input_layernorm", "post_attention_layernorm"):
            out[p + n + ".weight"] = (0, 1, 0, H)
        for n in ("self_attn.q_norm", "self_attn.k_norm"):
            out[p + n + ".weight"] = (0, 1, 0, D)
    return out
