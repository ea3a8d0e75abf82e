"""Test helpers: an oracle model holding exactly the weights of a device model, device KV
copied into oracle caches, and the logits criteria the parity tests share."""
import numpy as np

from oracle.oracle import OracleModel
from yue2_rs_b200.synth import tensor_specs

MAX_ABS, MEAN_ABS = 2e-2, 1e-3  # north_star logits tolerance


def oracle_from_device(dev, cfg):
    """The AR tensors of `dev` (a Model) read back through yue2_model_get_tensor and loaded
    into the oracle, so both hold bit-identical bf16 weights."""
    items = []
    for name, shape, kind in tensor_specs(cfg):
        if "nar_" in name or kind == "bias" or name.startswith(("latent", "vae2", "llm2", "time_")):
            continue
        n = int(np.prod(shape))
        items.append((name, 0, shape if len(shape) > 1 else (n,), dev.get_tensor(name, n)))
    return OracleModel.from_tensors(cfg, items)


def copy_cache_to_oracle(dev_cache, orc_cache, cfg, length):
    """Positions [0, length) of every layer of a device cache into an oracle cache."""
    w = cfg.num_key_value_heads * cfg.head_dim
    bits = np.empty((cfg.num_hidden_layers, 2, length, w), dtype=np.uint16)
    for layer in range(cfg.num_hidden_layers):
        bits[layer, 0], bits[layer, 1] = dev_cache.read(layer, 0, length)
    orc_cache.write(length, bits)


def within_tolerance(dev, ref, what):
    d = np.abs(dev.astype(np.float64) - ref)
    assert np.isfinite(dev).all(), what
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (what, float(d.max()), float(d.mean()))


def floor_check(dev, ref, alt):
    """The noise-floor criterion: the device's relative L2 and mean-abs distance to the
    oracle within 2.5x of the oracle's own distance under another valid f32 summation
    order (`alt`), and argmax agreement on at least 90% of rows."""
    d = np.abs(dev.astype(np.float64) - ref)
    f = np.abs(alt.astype(np.float64) - ref)
    rel_dev = np.linalg.norm(dev.astype(np.float64) - ref) / np.linalg.norm(ref)
    rel_floor = np.linalg.norm(alt.astype(np.float64) - ref) / np.linalg.norm(ref)
    assert np.isfinite(dev).all()
    assert rel_dev <= 2.5 * rel_floor + 1e-6, (rel_dev, rel_floor)
    assert d.mean() <= 2.5 * f.mean() + 1e-7, (d.mean(), f.mean())
    assert (np.argmax(dev, -1) == np.argmax(ref, -1)).mean() >= 0.9
    return d, rel_dev, rel_floor
