"""The native checkpoint loader (yue2_model_load_checkpoint) against the numpy reader +
set_tensor: identical device weights, so identical logits; and a sharded checkpoint with
F32 layer matrices (bf16-exact values) loads to the same model."""
import json
import os

import numpy as np
import pytest

from yue2_rs_b200 import Model, checkpoint

pytestmark = pytest.mark.gpu


def _logits(m, prompt):
    c = m.new_cache(len(prompt) + 4)
    out = [m.forward(prompt, c)] + [m.forward([t], c) for t in (5, 77, 901)]
    c.close()
    return np.array(out)


def test_native_loader_matches_python_loader(c1_dir, c1_prompt):
    prompt = c1_prompt[0][:100]
    a = Model.open(c1_dir, loader="native")
    b = Model.open(c1_dir, loader="python")
    try:
        la, lb = _logits(a, prompt), _logits(b, prompt)
        assert np.array_equal(la, lb)
        shapes = {name: shape for name, _, shape, _ in checkpoint.tensors(c1_dir)}
        for name in ("model.layers.1.mlp.down_proj.weight", "model.layers.0.self_attn.k_proj.weight",
                     "model.norm.weight", "model.layers.0.self_attn.q_norm.weight"):
            n = int(np.prod(shapes[name]))
            assert np.array_equal(a.get_tensor(name, n), b.get_tensor(name, n))
    finally:
        a.close()
        b.close()


def test_sharded_f32_checkpoint(tmp_path, c1_dir, c1_prompt):
    shards = ({}, {})
    weight_map = {}
    for name, code, shape, arr in checkpoint.tensors(c1_dir):
        dt = {0: "BF16", 1: "F32", 2: "F16"}[code]
        arr = np.asarray(arr)
        if ".layers." in name and code == 0 and len(shape) == 2:
            arr = (arr.astype(np.uint32) << 16).view(np.float32)  # bf16-exact F32
            dt = "F32"
        k = 0 if "layers.0." in name or "embed" in name else 1
        shards[k][name] = (dt, shape, arr)
        weight_map[name] = f"part-{k}.safetensors"
    for k in range(2):
        checkpoint.write(str(tmp_path / f"part-{k}.safetensors"), shards[k])
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    with open(os.path.join(c1_dir, "config.json")) as f:
        (tmp_path / "config.json").write_text(f.read())
    prompt = c1_prompt[0][:70]
    a = Model.open(str(tmp_path), loader="native")
    b = Model.open(c1_dir, loader="native")
    try:
        assert np.array_equal(_logits(a, prompt), _logits(b, prompt))
    finally:
        a.close()
        b.close()
