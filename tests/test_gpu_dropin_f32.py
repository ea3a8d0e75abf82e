"""The reference's f32 Metal imports as CUDA drop-ins (include/yue2_cuda.h):
yue2_cuda_gemm, yue2_cuda_linear, yue2_cuda_attention and yue2_cuda_stack, against a
float64 numpy restatement of what the reference's metal.m and attention.metal compute
(metal.m:164-237,330-362,429-538; attention.metal:9-157): f32 products, bf16 roundings
exactly where the shaders round. Products differ from f64 only by f32 summation, so the
bounds are f32-level for the GEMMs and one bf16 rounding (plus f32 noise) where the
reference rounds its outputs.
"""
import ctypes

import numpy as np
import pytest

from yue2_rs_b200 import _lib

pytestmark = pytest.mark.gpu

def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _bf(x):
    """round to nearest even bf16, NaN quieted (attention.metal:73-78, tensor.rs:645-652)"""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = np.where(nan, (u & 0xFFFF0000) | 0x00400000, (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000)
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def _bf16_bytes(x):
    return (_bf(x).view(np.uint32) >> 16).astype(np.uint16)


def test_gemm_matches_f64_with_strides_and_beta():
    lib = _lib.lib()
    rng = np.random.default_rng(1)
    for trans in (0, 1):
        for beta in (0.0, 0.5):
            m, n, k = 70, 90, 130
            lda, ldb, ldc = k + 3, (k if trans else n) + 5, n + 7
            a = rng.standard_normal((m, lda)).astype(np.float32)
            b = rng.standard_normal(((n if trans else k), ldb)).astype(np.float32)
            c = rng.standard_normal((m, ldc)).astype(np.float32)
            c0 = c.copy()
            assert lib.yue2_cuda_gemm(_p(a), _p(b), _p(c), m, n, k, trans, lda, ldb, ldc, beta) == 1, \
                lib.yue2_last_error()
            bb = b[:, :k].astype(np.float64).T if trans else b[:, :n].astype(np.float64)
            ref = a[:, :k].astype(np.float64) @ bb + beta * c0[:, :n]
            assert np.allclose(c[:, :n], ref, rtol=1e-5, atol=1e-4)
            assert np.array_equal(c[:, n:], c0[:, n:])  # past n untouched
    # m == 0: nothing to do
    z = np.zeros(4, np.float32)
    assert lib.yue2_cuda_gemm(_p(z), _p(z), _p(z), 0, 2, 2, 0, 2, 2, 2, 0.0) == 1


@pytest.mark.parametrize("dtype,rnd", [(0, 0), (1, 0), (1, 1), (2, 1)])
def test_linear_matches_f64(dtype, rnd):
    lib = _lib.lib()
    rng = np.random.default_rng(2 + dtype)
    m, n, k = 40, 72, 96
    a = rng.standard_normal((m, k)).astype(np.float32)
    w32 = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    if dtype == 0:
        raw = _bf16_bytes(w32)
        w = (raw.astype(np.uint32) << 16).view(np.float32)
    elif dtype == 1:
        raw = w32
        w = _bf(w32) if rnd else w32
    else:
        raw = w32.astype(np.float16)
        w = raw.astype(np.float32)
        w = _bf(w) if rnd else w
    raw = np.ascontiguousarray(raw)
    c = np.zeros((m, n), np.float32)
    assert lib.yue2_cuda_linear(_p(a), _p(raw), 7000 + dtype * 10 + rnd, dtype, rnd, _p(c), m, n, k) == 1, \
        lib.yue2_last_error()
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.allclose(c, ref, rtol=1e-5, atol=1e-4)


def _attention_ref(q, k, v, heads, kv, dim, causal, scale):
    """pack -> f32 scores -> attention_softmax -> P.V -> unpack_attention (bf16)."""
    rows, keys, G = q.shape[0], k.shape[0], heads // kv
    out = np.zeros((rows, heads * dim), np.float32)
    for h in range(heads):
        g = h // G
        s = q[:, h * dim:(h + 1) * dim].astype(np.float64) @ k[:, g * dim:(g + 1) * dim].astype(np.float64).T
        for r in range(rows):
            vis = keys if causal < 0 else min(keys, causal + r + 1)
            x = s[r, :vis] * scale
            p = np.exp(x - x.max())
            p /= p.sum()
            out[r, h * dim:(h + 1) * dim] = p @ v[:vis, g * dim:(g + 1) * dim].astype(np.float64)
    return _bf(out)


@pytest.mark.parametrize("rows,keys,causal", [(70, 100, -1), (70, 100, 20), (300, 333, 33), (5, 2000, -1)])
def test_attention_matches_reference_algorithm(rows, keys, causal):
    lib = _lib.lib()
    heads, kv, dim = 4, 2, 64
    rng = np.random.default_rng(rows + keys)
    q = _bf(rng.standard_normal((rows, heads * dim)).astype(np.float32))
    k = _bf(rng.standard_normal((keys, kv * dim)).astype(np.float32))
    v = _bf(rng.standard_normal((keys, kv * dim)).astype(np.float32))
    out = np.full((rows, heads * dim), np.nan, np.float32)
    scale = 1.0 / np.sqrt(dim)
    assert lib.yue2_cuda_attention(_p(q), _p(k), _p(v), _p(out), rows, keys, heads, kv, dim,
                                   ctypes.c_int64(causal), ctypes.c_float(scale)) == 1, lib.yue2_last_error()
    ref = _attention_ref(q, k, v, heads, kv, dim, causal, scale)
    assert np.isfinite(out).all()
    assert (np.abs(out - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-6).all()
    assert (out == ref).mean() >= 0.95


def _stack_ref(x, W, norms, pre_k, pre_v, heads, kv, dim, eps, cos, sin):
    """yue2_metal_stack (metal.m:429-538) in numpy: f32 products, shader roundings."""
    rows, H = x.shape
    x = x.astype(np.float32).copy()

    def lin(a, w):
        return (a.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)

    def rms(a, g):
        s = (a.astype(np.float64) ** 2).sum(1, keepdims=True)
        sc = _bf((1.0 / np.sqrt(s / a.shape[1] + eps)).astype(np.float32))
        return _bf(_bf(a * sc) * g)

    def rot(t, nh, g):
        t = _bf(t).reshape(rows, nh, dim)
        s = (t.astype(np.float64) ** 2).sum(2, keepdims=True)
        sc = _bf((1.0 / np.sqrt(s / dim + eps)).astype(np.float32))
        half = dim // 2
        a = _bf(_bf(t[:, :, :half] * sc) * g[:half])
        b = _bf(_bf(t[:, :, half:] * sc) * g[half:])
        c, s_ = cos[:, None, :], sin[:, None, :]
        return np.concatenate([_bf(_bf(a * c) - _bf(b * s_)), _bf(_bf(b * c) + _bf(a * s_))], 2).reshape(rows, nh * dim)

    for l in range(len(W)):
        q, k, v, o, gate, up, down = W[l]
        n0, n1, n2, n3 = norms[l]
        h = rms(x, n0)
        qq = rot(lin(h, q), heads, n1)
        kk = rot(lin(h, k), kv, n2)
        vv = _bf(lin(h, v))
        keys_k = np.concatenate([pre_k[l], kk]) if pre_k[l].size else kk
        keys_v = np.concatenate([pre_v[l], vv]) if pre_v[l].size else vv
        att = _attention_ref(qq, keys_k, keys_v, heads, kv, dim, -1, 1.0 / np.sqrt(dim))
        x = _bf(x + _bf(lin(att, o)))
        h = rms(x, n3)
        gg = _bf(lin(h, gate))
        act = _bf(gg / (1.0 + np.exp(-gg.astype(np.float64))).astype(np.float32))
        hh = _bf(act * _bf(lin(h, up)))
        x = _bf(x + _bf(lin(hh, down)))
    return x


def test_stack_matches_reference_algorithm():
    lib = _lib.lib()
    rng = np.random.default_rng(11)
    L, H, heads, kv, dim, I, rows, prefix, eps = 2, 128, 4, 2, 32, 256, 20, 12, 1e-6
    shapes = [(heads * dim, H), (kv * dim, H), (kv * dim, H), (H, heads * dim), (I, H), (I, H), (H, I)]
    keep = []
    W, norms, pre_k, pre_v = [], [], [], []
    layers = (_lib.GpuLayer * L)()
    for l in range(L):
        ws = []
        for j, (r, c) in enumerate(shapes):
            w = _bf((rng.standard_normal((r, c)) * 0.08).astype(np.float32))
            raw = np.ascontiguousarray(_bf16_bytes(w))
            keep.append(raw)
            ws.append(w)
            wd = layers[l].weights[j]
            wd.raw, wd.mapping, wd.rows, wd.cols, wd.dtype, wd.rounded = raw.ctypes.data, 9000 + 10 * l + j, r, c, 0, 1
        W.append(ws)
        ns = [_bf((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)) for n in (H, dim, dim, H)]
        norms.append(ns)
        keep.extend(ns)
        for j in range(4):
            layers[l].norms[j] = ns[j].ctypes.data
        pk = _bf(rng.standard_normal((prefix, kv * dim)).astype(np.float32))
        pv = _bf(rng.standard_normal((prefix, kv * dim)).astype(np.float32))
        keep.extend([pk, pv])
        pre_k.append(pk)
        pre_v.append(pv)
        layers[l].key, layers[l].value = pk.ctypes.data, pv.ctypes.data
    x = _bf(rng.standard_normal((rows, H)).astype(np.float32))
    pos = prefix + np.arange(rows)
    inv = 1.0 / (10000.0 ** (np.arange(0, dim, 2) / dim))
    ang = pos[:, None] * inv[None, :]
    cos, sin = _bf(np.cos(ang).astype(np.float32)), _bf(np.sin(ang).astype(np.float32))
    out = np.zeros_like(x)
    assert lib.yue2_cuda_stack(_p(x), _p(out), ctypes.cast(layers, ctypes.c_void_p), L, rows, H, heads, kv, dim, I,
                               prefix, 77, ctypes.c_float(eps), _p(cos), _p(sin)) == 1, lib.yue2_last_error()
    ref = _stack_ref(x, W, norms, pre_k, pre_v, heads, kv, dim, eps, cos, sin)
    assert np.isfinite(out).all()
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel <= 1e-2, rel
    assert (out == ref).mean() >= 0.9
    lib.yue2_cuda_release_cache(77)
    # a wrong weight shape is refused before any work
    layers[0].weights[0].rows = 3
    assert lib.yue2_cuda_stack(_p(x), _p(out), ctypes.cast(layers, ctypes.c_void_p), L, rows, H, heads, kv, dim, I,
                               prefix, 77, ctypes.c_float(eps), _p(cos), _p(sin)) == 0
    assert b"wrong shape" in lib.yue2_last_error()
