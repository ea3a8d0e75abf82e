"""Regenerates the committed golden fixtures in this folder.

* mt19937_kat.json  -- first 2000 outputs of std::mt19937 for six seeds (the C++
  standard library restates the reference's Generator, sampling.rs:10-42).
* attention_ref.npz -- the reference's only hot-path golden test
  (src/tensor.rs:7-83, `cached_attention_covers_long_context_and_append`):
  deterministic integer-hash Q/K/V for heads 4, kv 2, dims {64,128,256},
  keys {4096,4097,7169,24576} (+1 appended key below 24576) and the f64
  softmax*V expectation rounded to bf16, exactly as that test computes it.

Run:  python tests/golden/make_golden.py
"""
import json
import os
import subprocess
import sys
import tempfile
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, ".."))
from refmath import round_bf16_np, f32lit  # noqa: E402,F401


def make_mt():
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "kat")
        subprocess.check_call(["g++", "-O2", "-o", exe, os.path.join(HERE, "make_mt_kat.cpp")])
        out = subprocess.check_output([exe]).decode()
    data = json.loads(out)
    with open(os.path.join(HERE, "mt19937_kat.json"), "w") as f:
        json.dump(data, f)


def attention_inputs(heads, kv, dim, keys, append):
    """Inputs of tensor.rs:12-38 as float32 arrays (bf16-valued)."""
    n = keys * kv * dim
    i = np.arange(n, dtype=np.int64)
    k = round_bf16_np(((i * 17 % 101).astype(np.float32) - f32lit("50")) * f32lit("0.06"))
    v = round_bf16_np(((i * 31 % 137).astype(np.float32) - f32lit("68")) * f32lit("0.007"))
    iq = np.arange(heads * dim, dtype=np.int64)
    q = round_bf16_np(((iq * 23 % 97).astype(np.float32) - f32lit("48")) * f32lit("0.04"))
    k = k.reshape(keys, kv * dim)
    v = v.reshape(keys, kv * dim)
    if append:
        ia = np.arange(kv * dim, dtype=np.int64).astype(np.float32)
        k = np.concatenate([k, round_bf16_np(ia * f32lit("0.002") - f32lit("0.3"))[None]], 0)
        v = np.concatenate([v, round_bf16_np(f32lit("0.4") - ia * f32lit("0.001"))[None]], 0)
    return q, k, v


def attention_expected(q, k, v, heads, kv, dim):
    """tensor.rs:42-77: f64 scores, f64 softmax, f64 P.V, then bf16."""
    groups = heads // kv
    scale = float(np.float32(1.0) / np.sqrt(np.float32(dim)))
    out = np.zeros(heads * dim, dtype=np.float32)
    for h in range(heads):
        kh = h // groups
        kk = k[:, kh * dim:(kh + 1) * dim].astype(np.float64)
        vv = v[:, kh * dim:(kh + 1) * dim].astype(np.float64)
        s = kk @ q[h * dim:(h + 1) * dim].astype(np.float64) * scale
        e = np.exp(s - s.max())
        out[h * dim:(h + 1) * dim] = round_bf16_np(((e @ vv) / e.sum()).astype(np.float32))
    return out


def make_attention():
    heads, kv = 4, 2
    arrays = {}
    for dim in (64, 128, 256):
        for keys in (4096, 4097, 7169, 24576):
            for append in (0, 1) if keys < 24576 else (0,):
                q, k, v = attention_inputs(heads, kv, dim, keys, append)
                arrays[f"d{dim}_k{keys}_a{append}"] = attention_expected(q, k, v, heads, kv, dim)
    np.savez_compressed(os.path.join(HERE, "attention_ref.npz"), **arrays)


if __name__ == "__main__":
    make_mt()
    make_attention()
    print("wrote", os.listdir(HERE))
