"""Seeded synthetic YuE2 checkpoints under the reference's tensor names
(src/model.rs:76-93,103-114,176-200,250-270,418-451), written as safetensors.

Matrices and embeddings are bf16(std * z), RMSNorm gains bf16(norm_mean + std * z) (norm_mean
0 follows the benchmark configurations literally: every weight N(0, std)), biases zero,
z standard normal from numpy's PCG64 generator seeded with `seed`, drawn tensor by tensor
in the order of `tensor_specs`. NAR and latent tensors are included so that the
reference's own Model::open would accept the directory.
"""
import json
import os

import numpy as np

from . import checkpoint
from .model import Config


def tensor_specs(c):
    """(name, shape, kind) with kind in {"matrix", "norm", "bias"} in generation order."""
    H, D, I = c.hidden_size, c.head_dim, c.intermediate_size
    qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D
    out = [("model.embed_tokens.weight", (c.vocab_size, H), "matrix")]
    if not c.tie_word_embeddings:
        out.append(("lm_head.weight", (c.vocab_size, H), "matrix"))
    out.append(("model.norm.weight", (H,), "norm"))
    for l in range(c.num_hidden_layers):
        p = f"model.layers.{l}."
        for pre, attn, mlp, n1, n2 in (("", "self_attn", "mlp", "input_layernorm", "post_attention_layernorm"),
                                       ("nar_", "nar_self_attn", "nar_mlp", "nar_input_layernorm",
                                        "nar_pre_mlp_layernorm")):
            out += [
                (p + n1 + ".weight", (H,), "norm"),
                (p + attn + ".q_proj.weight", (qd, H), "matrix"),
                (p + attn + ".k_proj.weight", (kd, H), "matrix"),
                (p + attn + ".v_proj.weight", (kd, H), "matrix"),
                (p + attn + ".o_proj.weight", (H, qd), "matrix"),
                (p + attn + ".q_norm.weight", (D,), "norm"),
                (p + attn + ".k_norm.weight", (D,), "norm"),
                (p + n2 + ".weight", (H,), "norm"),
                (p + mlp + ".gate_proj.weight", (I, H), "matrix"),
                (p + mlp + ".up_proj.weight", (I, H), "matrix"),
                (p + mlp + ".down_proj.weight", (H, I), "matrix"),
            ]
    out += [
        ("latent_pos_embed.pe", (c.max_latent_frames, H), "matrix"),
        ("vae2llm.weight", (H, c.latent_dim), "matrix"), ("vae2llm.bias", (H,), "bias"),
        ("llm2vae.weight", (c.latent_dim, H), "matrix"), ("llm2vae.bias", (c.latent_dim,), "bias"),
        ("time_embedder.mlp.0.weight", (H, 256), "matrix"), ("time_embedder.mlp.0.bias", (H,), "bias"),
        ("time_embedder.mlp.2.weight", (H, H), "matrix"), ("time_embedder.mlp.2.bias", (H,), "bias"),
    ]
    return out


def bf16_bits(x):
    """float32 -> bf16 bits, round to nearest even (tensor.rs:645-652)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def generate(config, seed, std=0.02, norm_mean=0.0):
    """Yields (name, shape, bf16 bits) for every tensor."""
    rng = np.random.default_rng(seed)
    for name, shape, kind in tensor_specs(config):
        n = int(np.prod(shape))
        if kind == "bias":
            bits = np.zeros(n, dtype=np.uint16)
        else:
            z = rng.standard_normal(n, dtype=np.float32)
            z *= np.float32(std)
            if kind == "norm":
                z += np.float32(norm_mean)
            bits = bf16_bits(z)
        yield name, shape, bits.reshape(shape)


def write_checkpoint(path, config, seed, std=0.02, norm_mean=0.0):
    """Writes config.json + model.safetensors; returns the directory."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config.json(), f, indent=1)
    named = {name: ("BF16", shape, bits) for name, shape, bits in generate(config, seed, std, norm_mean)}
    checkpoint.write(os.path.join(path, "model.safetensors"), named, {"format": "pt", "synthetic_seed": str(seed)})
    return path


# The configurations of the benchmark (BASELINE.json configs 0..1).
def config_c1():
    """Reduced CPU-runnable AR model: 2 layers, hidden 1024, 8/2 heads, intermediate 2816."""
    return Config(hidden_size=1024, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                  intermediate_size=2816, vocab_size=84000, rms_norm_eps=1e-6, rope_theta=10000.0,
                  max_position_embeddings=24576, max_latent_frames=16)


def config_nar_tiny():
    """A small model with the real 184,704-id vocabulary (the codec ids of the acoustic
    stage) and a 160-position context, so that a song of a few hundred frames spans several
    synthesize chunks: 2 layers, hidden 256, 4/2 heads of 64, intermediate 512."""
    return Config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                  intermediate_size=512, vocab_size=184704, rms_norm_eps=1e-6, rope_theta=10000.0,
                  max_position_embeddings=160, max_latent_frames=16)


def config_c2():
    """3B-shaped AR model: 28 layers, hidden 3072, 24/8 heads, intermediate 8192."""
    return Config(hidden_size=3072, num_hidden_layers=28, num_attention_heads=24, num_key_value_heads=8,
                  head_dim=128, intermediate_size=8192, vocab_size=84000, rms_norm_eps=1e-6, rope_theta=10000.0,
                  max_position_embeddings=24576, max_latent_frames=16)
