"""teacher-forced per-step logits of the CUDA path against the oracle's
restatement of the reference decode path.

Two criteria:
  * the north_star tolerance (2e-2 max-abs, 1e-3 mean-abs) on config 0 as specified
    (every weight, RMSNorm gains included, bf16 N(0, 0.02), seed 0);
  * a noise-floor criterion on config 0 and on a unit-gain variant (gains 1 + N(0, 0.02)):
    the reference rounds to bf16 after every op, so a change of f32 summation order alone
    moves ~70% of unit-gain logits by an ulp. The oracle evaluated with two valid orders
    (16 interleaved partial sums, strictly sequential) measures that floor; the CUDA path,
    which has its own order, must stay within 2.5x of it.
"""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def run_oracle(model, prompt, teacher, order):
    orc.set_dot_order(order)
    try:
        c = model.cache(len(prompt) + len(teacher))
        return np.array([model.prefill(prompt, c)] + [model.forward([t], c) for t in teacher])
    finally:
        orc.set_dot_order(0)


def run_device(model, prompt, teacher):
    c = model.new_cache(len(prompt) + len(teacher))
    out = [model.forward(prompt, c)] + [model.forward([t], c) for t in teacher]
    assert c.length == len(prompt) + len(teacher)
    return np.array(out), c


def floor_check(dev, ref, alt):
    d = np.abs(dev.astype(np.float64) - ref)
    f = np.abs(alt.astype(np.float64) - ref)
    rel_dev = np.linalg.norm(dev.astype(np.float64) - ref) / np.linalg.norm(ref)
    rel_floor = np.linalg.norm(alt.astype(np.float64) - ref) / np.linalg.norm(ref)
    assert np.isfinite(dev).all()
    assert rel_dev <= 2.5 * rel_floor + 1e-6, (rel_dev, rel_floor)
    assert d.mean() <= 2.5 * f.mean() + 1e-7, (d.mean(), f.mean())
    assert (np.argmax(dev, 1) == np.argmax(ref, 1)).mean() >= 0.9
    return d, rel_dev, rel_floor


def test_teacher_forced_logits_config0(c1_device, c1_oracle, c1_prompt):
    prompt, teacher = c1_prompt
    dev, dc = run_device(c1_device, prompt, teacher)
    ref = run_oracle(c1_oracle, prompt, teacher, 0)
    for step in range(len(dev)):
        d = np.abs(dev[step].astype(np.float64) - ref[step])
        assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (step, d.max(), d.mean())
    alt = run_oracle(c1_oracle, prompt, teacher, 1)
    floor_check(dev, ref, alt)
    # the KV caches agree except for rare bf16 rounding flips
    oc = c1_oracle.cache(len(prompt) + len(teacher))
    c1_oracle.prefill(prompt + teacher, oc, logits=False)
    to_f = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
    for layer in range(c1_oracle.config.num_hidden_layers):
        kd, vd = dc.read(layer, 0, dc.length)
        ko, vo = oc.read(layer)
        assert np.mean(to_f(kd) == ko) > 0.9 and np.mean(to_f(vd) == vo) > 0.9


def test_teacher_forced_logits_unit_gains(c1u_device, c1u_oracle, c1_prompt):
    prompt, teacher = c1_prompt
    dev, _ = run_device(c1u_device, prompt, teacher[:24])
    ref = run_oracle(c1u_oracle, prompt, teacher[:24], 0)
    alt = run_oracle(c1u_oracle, prompt, teacher[:24], 1)
    floor_check(dev, ref, alt)


def _batch_cases(model, prompt, teacher):
    def caches(n, off):
        cs = [model.new_cache(64) for _ in range(n)]
        for i, c in enumerate(cs):
            j = (i + off) % 3
            model.forward(prompt[j * 5: j * 5 + 7], c)
        return cs

    ids = lambda n, off: [teacher[(i + off) % 3] for i in range(n)]
    return caches, ids


def test_batched_rows_equal_single_rows_gemv(c1u_dir, c1_prompt):
    """Rows in one weight pass do not interact. On the GEMV passes (forced for every row
    count with YUE2_CUDA_WIDE_MIN=17): one or two rows share the SIMT GEMV, so R=2 gives the
    R=1 logits bit for bit; three to sixteen rows share the tensor-core GEMV, so a row gives
    the same logits at R=3 and R=8 whatever its companions hold."""
    import os

    from yue2_rs_b200 import Model
    prompt, teacher = c1_prompt
    old = os.environ.get("YUE2_CUDA_WIDE_MIN")
    os.environ["YUE2_CUDA_WIDE_MIN"] = "17"
    try:
        m = Model.open(c1u_dir)
    finally:
        if old is None:
            del os.environ["YUE2_CUDA_WIDE_MIN"]
        else:
            os.environ["YUE2_CUDA_WIDE_MIN"] = old
    try:
        caches, ids = _batch_cases(m, prompt, teacher)
        two = m.forward_rows(caches(2, 0), ids(2, 0))
        for i in range(2):
            one = m.forward([teacher[i]], caches(1, i)[0])
            assert (two[i].view(np.uint32) == one.view(np.uint32)).all()
        three = m.forward_rows(caches(3, 0), ids(3, 0))
        eight = m.forward_rows(caches(8, 0), ids(8, 0))
        for i in range(3):
            assert (three[i].view(np.uint32) == eight[i].view(np.uint32)).all()
            assert (three[i].view(np.uint32) == eight[i + 3].view(np.uint32)).all()
    finally:
        m.close()


def test_batched_rows_gemm_passes(c1u_device, c1_prompt):
    """Passes of three or more rows run as GEMMs (the default): rows with the same cache
    contents and id give the same logits in one pass, and other row counts (another
    cuBLASLt algorithm, another summation order) stay within an order-only difference."""
    prompt, teacher = c1_prompt
    caches, ids = _batch_cases(c1u_device, prompt, teacher)
    three = c1u_device.forward_rows(caches(3, 0), ids(3, 0))
    eight = c1u_device.forward_rows(caches(8, 0), ids(8, 0))
    for i in range(3):
        assert (eight[i].view(np.uint32) == eight[i + 3].view(np.uint32)).all()
        d = np.abs(three[i].astype(np.float64) - eight[i])
        assert d.max() <= 0.08 and d.mean() <= 1e-2


def test_capacity_and_token_errors(c1_device):
    from yue2_rs_b200 import Phase, Yue2Error
    c = c1_device.new_cache(2)
    c1_device.forward([1, 2], c)
    with pytest.raises(Yue2Error, match="exceeds cache"):
        c1_device.forward([3], c)
    with pytest.raises(Yue2Error, match="outside model vocabulary"):
        c1_device.forward([c1_device.config.vocab_size], c1_device.new_cache(4))
    with pytest.raises(Yue2Error, match="native music protocol"):
        c1_device.forward_phase([1], c1_device.new_cache(4), Phase.SEMANTIC)
