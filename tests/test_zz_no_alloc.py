"""yue2_attention_noalloc: the decode attention for callers that cannot allocate device
memory (hosts that own every allocation through their own pool, forbid cudaMalloc/cudaFree
after start-up because those synchronise the device, or run threads that may not block in
the allocator). Its split-K scratch is a fixed static device array instead of a workspace.

Checked through the C ABI against the existing entry point, yue2_cuda_cached_attention, on
the reference's own attention inputs (src/tensor.rs:12-38), for two calls in a row, with
the tolerance the attention tests use. This file sorts last so that a run stopping at the
first failure has already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from golden.make_golden import attention_inputs
from yue2_rs_b200 import _lib

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def bits(a):
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


# (heads, kv): the reference test's 4/2 (G=2), the reduced model's 8/2 (G=4) and the
# 3B-shaped model's 24/8 (G=3)
@pytest.mark.parametrize("dim,keys,heads,kv", [(128, 4097, 4, 2), (64, 24576, 4, 2), (256, 333, 4, 2),
                                               (128, 4097, 8, 2), (128, 2049, 24, 8), (128, 24576, 24, 8)])
def test_noalloc_attention_matches_existing_entry_point(dim, keys, heads, kv):
    import torch
    L = _lib.lib()
    q, k, v = attention_inputs(heads, kv, dim, keys - 1, 1)  # the reference inputs with one appended key
    want = np.empty(heads * dim, dtype=np.float32)
    cache = 777000 + dim * 100000 + keys + heads * 10_000_000
    assert L.yue2_cuda_cached_attention(_p(q), _p(k), _p(v), _p(want), k.shape[0], heads, kv, dim, cache, 0) == 1, \
        _lib.last_error()
    L.yue2_cuda_release_cache(cache)
    dev = torch.device("cuda", 0)
    dq = torch.from_numpy(bits(q).view(np.int16)).to(dev)
    dk = torch.from_numpy(bits(k).view(np.int16)).to(dev)
    dv = torch.from_numpy(bits(v).view(np.int16)).to(dev)
    stream = torch.cuda.current_stream(dev)
    for call in range(2):  # the second call reuses the shared scratch left by the first
        out = torch.full((heads * dim,), -1, dtype=torch.int16, device=dev)
        rc = L.yue2_attention_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), k.shape[0],
                                      heads, kv, dim, stream.cuda_stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize(dev)
        got = (out.cpu().numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        assert np.all(np.abs(got - want) <= 5e-5 + np.abs(want) * 0.008), (call, float(np.abs(got - want).max()))


def test_noalloc_rejects_sizes_beyond_the_static_scratch():
    import torch
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    buf = torch.zeros(1 << 20, dtype=torch.int16, device=dev)
    p = buf.data_ptr()
    # 512 heads of dim 256 over 64 kv heads use 5 splits on 148 SMs: 512 * 258 * 5 * 4 B of
    # partials, more than the 2 MiB array; the call is refused before any launch
    rc = L.yue2_attention_noalloc(p, p, p, p, 64, 512, 64, 256, None)
    assert rc == -1
    assert "static scratch" in _lib.last_error()
