"""The tcgen05 GEMM (TMEM accumulators, TMA-fed 128B-swizzled tiles) against a torch f32
reference of the same bf16 operands and against cuBLASLt: Y = bf16(X . W^T) with f32
accumulation, so every output lies within one bf16 rounding (plus f32 summation order) of
the reference. Shapes cover one tile and one K block, partial row/column tiles, a K loop
longer than the stage ring, and the prefill's q|k|v shape; the gate|up form with the
SwiGLU epilogue is checked against the unfused GEMM put through the same roundings. The
skinny form (3..256 rows, the decode passes of several songs) is held to the same bounds
over row counts on both sides of every padding step, ragged N, K loops that cut tiles
between CTAs and a vocabulary-sized N where each CTA owns several whole tiles, and must
repeat bit for bit."""
import ctypes

import pytest
import torch

from yue2_rs_b200 import Model, _lib, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    m = Model.synthetic(synth.config_c1(), seed=2)
    yield m
    m.close()


def _run(m, x, w, impl):
    C, K = x.shape
    N = w.shape[0] // (2 if impl in (2, 4) else 1)
    y = torch.full((C, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()  # the library works on its own non-blocking stream
    ms = ctypes.c_double()
    _lib.check(_lib.lib().yue2_bench_gemm(m._h, x.data_ptr(), w.data_ptr(), y.data_ptr(), C, N, K, impl, 2,
                                          ctypes.byref(ms)))
    torch.cuda.synchronize()
    return y, ms.value


@pytest.mark.parametrize("C,N,K", [(128, 256, 64), (200, 384, 1024), (96, 520, 320), (1024, 5120, 3072)])
def test_tcgen05_gemm_matches_reference(model, C, N, K):
    g = torch.Generator(device="cuda").manual_seed(C * 7 + N + K)
    x = (torch.randn(C, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    tc, _ = _run(model, x, w, 1)
    lt, _ = _run(model, x, w, 0)
    assert torch.isfinite(tc.float()).all()
    # within one bf16 ulp of the f32 reference (rounding) plus f32 summation-order noise
    tol = ref.abs() * 2.0 ** -7 + 1e-3
    assert ((tc.float() - ref).abs() <= tol).all()
    assert ((tc.float() - lt.float()).abs() <= tol).all()
    # the bf16 rounding of the exact sum is the same in most places
    assert (tc == ref.to(torch.bfloat16)).float().mean() >= 0.95


def _bf(t):
    return t.float().to(torch.bfloat16).float()


def test_tcgen05_gate_up_swiglu_epilogue(model):
    """The gate|up form: h = bf16(bf16(silu(bf16 g)) * bf16 u) straight from TMEM, against
    the unfused tcgen05 GEMM output put through the same roundings in torch (torch's exp
    may differ from the kernel's correctly rounded one by an ulp: at most a bf16 ulp off)."""
    C, I, K = 256, 384, 512
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn(C, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    h, _ = _run(model, x, w, 2)
    gu, _ = _run(model, x, w, 1)
    gt, ut = gu[:, :I].float(), gu[:, I:].float()
    a = _bf(gt / (1.0 + torch.exp(-gt)))
    ref = _bf(a * ut)
    assert torch.isfinite(h.float()).all()
    assert ((h.float() - ref).abs() <= ref.abs() * 2.0 ** -7 + 1e-6).all()
    assert (h.float() == ref).float().mean() >= 0.99


# ---- the skinny form (decode passes of 3..256 rows): weight rows on the MMA's M side,
# (tile, K block) work split evenly over one CTA per SM, cut tiles summed in CTA order

@pytest.mark.parametrize("C,N,K", [(3, 384, 256), (16, 5120, 3072), (17, 520, 320), (33, 3072, 3072),
                                   (64, 3072, 8192), (100, 1000, 1024), (128, 16384, 3072), (256, 3072, 3072),
                                   (48, 84000, 3072), (18, 1024, 2816), (18, 1536, 1024), (18, 1024, 1024)])
def test_skinny_gemm_matches_reference(model, C, N, K):
    g = torch.Generator(device="cuda").manual_seed(C * 13 + N + K)
    x = (torch.randn(C, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    ref = x.float() @ w.float().T
    sk, _ = _run(model, x, w, 3)
    assert torch.isfinite(sk.float()).all()
    tol = ref.abs() * 2.0 ** -7 + 1e-3
    assert ((sk.float() - ref).abs() <= tol).all()
    assert (sk == ref.to(torch.bfloat16)).float().mean() >= 0.95
    # the partial sums of cut tiles are added in a fixed order: the same bits every run
    again, _ = _run(model, x, w, 3)
    assert torch.equal(sk, again)


@pytest.mark.parametrize("C,I,K", [(5, 384, 512), (32, 8192, 3072), (130, 1024, 3072), (256, 2816, 1024),
                                   (18, 2816, 1024)])
def test_skinny_gate_up_swiglu_epilogue(model, C, I, K):
    g = torch.Generator(device="cuda").manual_seed(C + I)
    x = (torch.randn(C, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    h, _ = _run(model, x, w, 4)
    gu = (x.float() @ w.float().T).to(torch.bfloat16).float()
    gt, ut = gu[:, :I], gu[:, I:]
    ref = _bf(_bf(gt / (1.0 + torch.exp(-gt))) * ut)
    assert torch.isfinite(h.float()).all()
    # gate and up sums may round to the neighbouring bf16 value (f32 order): a few ulps
    assert ((h.float() - ref).abs() <= ref.abs() * 2.0 ** -5 + 1e-3).all()
    assert (h.float() == ref).float().mean() >= 0.95
