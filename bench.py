#!/usr/bin/env python
"""AR decode benchmark: tokens/s of YuE2's CFG decode loop on B200.

Product arm (default): BASELINE config 1 -- the 3B-shaped AR model (28 layers, hidden
3072, 24/8 heads, intermediate 8192, vocab 84,000, synthetic bf16 N(0, 0.02) weights,
seed 1), CFG on (scale 1.5), 1,024-id cond and uncond prompts, sampling T 1.0 / top-k 50 /
top-p 0.93. One step = one decode token: both CFG rows through every layer in one weight
pass, LM head, on-device CFG mix + choose (one CUDA-graph launch). W untimed steps, then
K timed steps between barriers; time = CUDA events on the decode stream, max over ranks.
Data-parallel over songs: every rank runs its own song (weak scaling, no collective).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

`--impl reference` times the reference's CPU decode math (the scalar host build in
oracle/, all host threads) on a bounded sample of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "AR decode tokens/s/GPU (CFG, 4k & 24k ctx) and % of HBM roofline; 1/2/4/8 GPU"
UNIT = "tokens/s"
PROMPT = 1024
SCALE = 1.5


def c2_sampling(max_tokens):
    from yue2_rs_b200 import Sampling
    # config 1: T 1.0, top-k 50, top-p 0.93; repetition penalty 1.0 (window 50), min_tokens 0
    return Sampling(1.0, 0.93, 50, 1.0, 50, 0, max_tokens)


def prompts(seed, vocab):
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, PROMPT).tolist(), rng.integers(0, vocab, PROMPT).tolist()


def weight_bytes(c):
    H, I, V, D = c.hidden_size, c.intermediate_size, c.vocab_size, c.head_dim
    qd, kd = c.num_attention_heads * D, c.num_key_value_heads * D
    per_layer = 2 * (qd * H + 2 * kd * H + H * qd + 3 * I * H)
    return c.num_hidden_layers * per_layer + V * H * 2 + (2 * c.num_hidden_layers + 1) * H * 2


def kv_bytes_per_token(c):
    return c.num_hidden_layers * 2 * c.num_key_value_heads * c.head_dim * 2


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_bf16_tflops():
    """The burst cuBLAS bf16 GEMM peak (TFLOP/s) for a kernel timed alone, and its source."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed region."""

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def host_cores():
    """Host threads this process may run on (its CPU affinity), whatever OMP_NUM_THREADS
    says: torchrun sets that to 1 for every rank."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_baseline(config, min_tokens=120, max_s=60.0):
    """The oracle (scalar host build of the reference's decode math) on all host cores:
    the config-1 decode step (two forwards -- cond and uncond, as sampling.rs:281-285
    runs them -- CFG mix and choose) at a 1,024-position synthetic context, timed over
    `min_tokens` tokens (fewer only if that takes more than `max_s` seconds). The rate is
    one host's: the GPU count of the run does not change it."""
    from oracle import oracle as orc
    from yue2_rs_b200 import Phase
    orc.set_threads(host_cores())
    cores = orc.lib().orc_max_threads()
    t0 = time.perf_counter()
    m = orc.OracleModel.synthetic(config, seed=1, std=0.02)
    setup = time.perf_counter() - t0
    c = config
    kvw = c.num_key_value_heads * c.head_dim
    rng = np.random.default_rng(0)
    caches = []
    for side in range(2):
        bits = (rng.standard_normal((c.num_hidden_layers, 2, PROMPT, kvw), dtype=np.float32).view(np.uint32) >> 16)
        oc = m.cache(PROMPT + min_tokens + 8)
        oc.write(PROMPT, bits.astype(np.uint16))
        caches.append(oc)
    s = c2_sampling(min_tokens)
    g = orc.OracleRng(1)
    tok, toks, n = 0, [], 0
    t0 = time.perf_counter()
    while True:
        lc = m.forward([tok], caches[0])
        lu = m.forward([tok], caches[1])
        tok = orc.choose(orc.cfg_mix(lc, lu, SCALE), s, toks, n, int(Phase.VOCAB), False, g)
        toks.append(tok)
        n += 1
        el = time.perf_counter() - t0
        if n >= min_tokens or (el >= max_s and n >= 8):
            break
    m.close()
    return {"value": n / el, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} config-1 decode tokens (2 forwards + CFG mix + choose each) at a 1,024-position "
                      f"synthetic context in {el:.1f} s on {cores} host threads; weights seeded N(0,0.02) (setup "
                      f"{setup:.1f}s untimed); scalar host build of the reference decode math, not Accelerate; "
                      f"one host's rate, independent of the run's GPU count"}


def velocity_flops(config, n, keys):
    """FLOPs of one Model::velocity call over n rows (latent frames + 2) seeing `keys` keys:
    the linears 2 n L H (q + k + v + o + 3 I) and the attention 4 n keys heads dim L."""
    c = config
    qd, kd = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
    lin = 2.0 * n * c.num_hidden_layers * c.hidden_size * (qd + 2 * kd + qd + 3 * c.intermediate_size)
    att = 4.0 * n * keys * c.num_attention_heads * c.head_dim * c.num_hidden_layers
    return lin, att


def cpu_velocity_baseline(config, length, frames, sample_frames=24, layers=4):
    """The oracle's Model::velocity (scalar host build of src/model.rs:611-697) on the host
    cores, on a bounded sample of the bench's velocity workload: `sample_frames` latent
    frames over the same `length`-position cached prefix (seeded N(0,1) K/V), through
    `layers` of the layers (same shapes; velocity never reads the vocabulary, so a 256-row
    one keeps the setup short). The FLOP rate is counted like the device's; the full call's
    time is at that rate."""
    import copy
    from oracle import oracle as orc
    c = copy.copy(config)
    c.num_hidden_layers, c.vocab_size = layers, 256
    cores = orc.lib().orc_max_threads()
    t0 = time.perf_counter()
    m = orc.OracleModel.synthetic(c, seed=4, std=0.02, norm_mean=1.0, nar=True)
    kvw = c.num_key_value_heads * c.head_dim
    rng = np.random.default_rng(5)
    bits = np.empty((layers, 2, length, kvw), dtype=np.uint16)
    for li in range(layers):
        bits[li] = rng.standard_normal((2, length, kvw), dtype=np.float32).view(np.uint32) >> 16
    oc = m.cache(length)
    oc.write(length, bits)
    del bits
    setup = time.perf_counter() - t0
    st = rng.standard_normal((sample_frames, c.latent_dim), dtype=np.float32)
    st = ((st.view(np.uint32).astype(np.uint64) + 0x7FFF + ((st.view(np.uint32) >> 16) & 1)) &
          0xFFFF0000).astype(np.uint32).view(np.float32)
    t0 = time.perf_counter()
    m.velocity(st, oc, 0.5)
    el = time.perf_counter() - t0
    oc.close()
    m.close()
    n = sample_frames + 2
    flop = sum(velocity_flops(c, n, length + n))
    full = sum(velocity_flops(config, frames + 2, length + frames + 2))
    rate = flop / el
    return {"value": rate / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "full_call_seconds": full / rate,
            "sample": f"one velocity call of {sample_frames} frames over the same {length}-position prefix "
                      f"through {layers} of the {config.num_hidden_layers} layers (same shapes; {flop / 1e9:.0f} "
                      f"GFLOP in {el:.1f} s; setup {setup:.1f} s untimed); scalar host build of the "
                      f"reference's velocity math"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from yue2_rs_b200 import synth
    cb = cpu_baseline(synth.config_c2())
    line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 1: 3B-shaped AR decode, CFG 1.5, T1.0/top-k50/top-p0.93, 1,024 ctx",
                       "parallelism": "host threads"},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_tp(args, dp, local):
    """the 3B-shaped model split over the world's ranks (heads, MLP rows and
    LM-head vocabulary rows; peer-memory exchanges after o, down and the head), one song with
    CFG 1.5 at a 4,096-position context (seeded N(0,1) KV fill ahead of 2-id prompts), 256
    decode steps, each timed alone with CUDA events on the session's stream. world 1 is the
    unsharded model on the same workload."""
    import torch
    from yue2_rs_b200 import Model, Phase, Request, Session, synth, tp
    rank, world = dp.rank, dp.world
    cfg = synth.config_c2()
    model = Model.synthetic(cfg, seed=1, std=0.02, device=local, tp=(rank, world) if world > 1 else None)
    if world > 1:
        tp.connect(model, dp.group if hasattr(dp, "group") else None)
    steps, W = 256, max(args.warmup, 3)
    ctx = 4096
    cond, uncond = prompts(1000, cfg.vocab_size)
    req = Request(cond[:2], seed=7, negative=uncond[:2], scale=SCALE, context_fill=ctx - 2)
    sess = Session(model, [req], c2_sampling(W + steps + 1), Phase.VOCAB)
    st = torch.cuda.ExternalStream(sess.cuda_stream)
    sess.step(W)
    sess.sync()
    dp.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(st)
    for i in range(steps):
        sess.step(1)
        ev[i + 1].record(st)
    sess.sync()
    dp.barrier()
    clk = clocks.stop()
    per = np.array([ev[i].elapsed_time(ev[i + 1]) for i in range(steps)])
    toks, _ = sess.collect()[0]
    sess.close()
    model.close()
    p50, p99, total = dp.max(float(np.percentile(per, 50))), dp.max(float(np.percentile(per, 99))), dp.max(float(per.sum()))
    line = {"metric": "single-song per-token decode latency (BASELINE config 5)", "tp": world, "n_gpus": world,
            "p50_ms": p50, "p99_ms": p99, "mean_ms": total / steps, "tokens_per_s": steps / (total / 1000.0),
            "unit": "ms", "higher_is_better": False, "steps": steps, "warmup": W, "tokens": len(toks),
            "config": {"workload": "config 5: 3B-shaped AR decode, CFG 1.5, T1.0/top-k50/top-p0.93, 4,096-position "
                                   "context (seeded KV fill + 2-id prompts), one song",
                       "parallelism": f"tp{world}: q|k|v and gate|up by output rows, o and down by input columns, "
                                      "LM head by vocabulary rows; peer-memory all-reduce after o and down, "
                                      "all-gather after the head" if world > 1 else "tp1 (unsharded)"},
            "clocks": clk, "data": "synthetic"}
    dp.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="product", choices=["product", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="decode steps only (16-id prompts; no sweep, e2e, kernel hook or CPU baseline): "
                         "the command line for ncu launch lists")
    ap.add_argument("--profile-songs", type=int, default=1, metavar="B",
                    help="with --profile: B songs (2B CFG rows) of 16-id prompts after a synthetic "
                         "1,008-position context")
    ap.add_argument("--profile-context", type=int, default=0, metavar="L",
                    help="with --profile: 16-id prompts after a synthetic (L - 16)-position context")
    ap.add_argument("--profile-layers", type=int, default=0, metavar="N",
                    help="with --profile: a model of N layers (same shapes otherwise), for ncu captures "
                         "that must stay small")
    ap.add_argument("--prefill-profile", type=int, default=0, metavar="N",
                    help="one N-id prefill of the config-1 model and exit: the command line for the "
                         "prefill's ncu launch list")
    ap.add_argument("--tp", action="store_true",
                    help="BASELINE config 5: one song's decode split over the torchrun ranks (tensor "
                         "parallel), 4,096-position context, 256 steps; per-token latency p50/p99")
    ap.add_argument("--velocity-profile", type=int, default=0, metavar="F",
                    help="one Model::velocity call of F latent frames after a synthetic 1,025-position "
                         "prefix (3B-shaped NAR model; --profile-layers N for a smaller one) and exit")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    from yue2_rs_b200 import Model, Phase, Request, Sampling, Session, generate_batch, synth, _lib

    from yue2_rs_b200.dp import DataParallel
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dp = DataParallel("nccl")
    rank, world = dp.rank, dp.world

    def barrier():
        dp.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return dp.max(x)

    if args.tp:
        return run_tp(args, dp, local)
    cfg = synth.config_c2()
    if (args.profile or args.velocity_profile) and args.profile_layers > 0:
        cfg.num_hidden_layers = args.profile_layers
    if args.velocity_profile:
        nm = Model.synthetic(cfg, seed=4, std=0.02, norm_mean=1.0, device=local, nar=True)
        frames = args.velocity_profile
        nc = nm.new_cache(PROMPT + 1 + frames + 2)
        nc.fill_normal(PROMPT + 1, seed=5)
        st = np.random.default_rng(0).standard_normal((frames, cfg.latent_dim)).astype(np.float32)
        nm.velocity(st, nc, 0.5)  # first call per shape: cuBLASLt candidate timing
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        v = nm.velocity(st, nc, 0.5)
        ms = (time.perf_counter() - t0) * 1000.0
        print(json.dumps({"velocity_profile": True, "frames": frames, "layers": cfg.num_hidden_layers,
                          "ms": ms, "finite": bool(np.isfinite(v).all())}), flush=True)
        nc.close()
        nm.close()
        dp.close()
        return 0
    model = Model.synthetic(cfg, seed=1, std=0.02, device=local)
    if args.prefill_profile:
        ids = np.random.default_rng(5).integers(0, cfg.vocab_size, args.prefill_profile).tolist()
        c = model.new_cache(args.prefill_profile + 8)
        model.forward(ids, c)
        torch.cuda.synchronize()
        c.close()
        model.close()
        dp.close()
        return 0
    W, K = max(args.warmup, 3), args.steps
    max_tokens = W + K + 1 if args.profile else max(512, W + K + 1)
    cond, uncond = prompts(1000 + rank, cfg.vocab_size)
    reqs = [Request(cond, seed=rank, negative=uncond, scale=SCALE)]
    if args.profile:
        B = max(1, args.profile_songs)
        fill = max(0, args.profile_context - 16) if args.profile_context else (PROMPT - 16 if B > 1 else 0)
        reqs = [Request(cond[16 * i: 16 * i + 16], seed=rank + i, negative=uncond[16 * i: 16 * i + 16], scale=SCALE,
                        context_fill=fill) for i in range(B)]
        args.no_sweep = args.no_cpu_baseline = True
    s = c2_sampling(max_tokens)

    # ---- device-resident timed region: K decode steps of one song per rank
    sess = Session(model, reqs, s, Phase.VOCAB)
    stream = torch.cuda.ExternalStream(sess.cuda_stream)
    sess.step(W)
    sess.sync()
    barrier()
    clocks = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launched = sess.step(K)
    e1.record(stream)
    sess.sync()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    assert launched == K, launched
    kps = sess.kernels_per_step
    toks, _ = sess.collect()[0]
    assert len(toks) == W + K + 1
    sess.close()
    value = world * K / (ms / 1000.0)
    ctx_avg = PROMPT + 1 + W + K / 2.0
    step_bytes = weight_bytes(cfg) + 2 * kv_bytes_per_token(cfg) * ctx_avg
    peak, peak_kind = measured_peaks()

    if args.profile:
        model.close()
        print(json.dumps({"profile_run": True, "ms_per_step": ms / K, "steps": K}), flush=True)
        return 0
    # ---- dominant kernel live: the gate|up GEMV (fused RMSNorm prologue + SwiGLU epilogue)
    import ctypes
    avg = ctypes.c_double()
    per = ctypes.c_double()
    _lib.check(_lib.lib().yue2_bench_gemv(model._h, 0, 2, 10 * cfg.num_hidden_layers, ctypes.byref(avg),
                                          ctypes.byref(per)))
    kern_gbs = per.value / (avg.value * 1e-3) / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", "gemv_gateup_c2_traffic.json")
    if os.path.exists(prof):
        with open(prof) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")

    # ---- long-context sweep (config 2): decode at 4,096, 8,192, 16,384 and 24,576 positions
    sweep = {}
    if not args.no_sweep:
        for L in (4096, 8192, 16384, 24576):
            ks = 128  # config 2: 128 timed decode steps at each length
            mt = 4 + ks + 1
            fill = L - 8 - mt - 1 if L == 24576 else L - 8
            r = Request(cond[:8], seed=rank, negative=uncond[:8], scale=SCALE, context_fill=fill)
            ss = Session(model, [r], c2_sampling(mt), Phase.VOCAB)
            st = torch.cuda.ExternalStream(ss.cuda_stream)
            ss.step(4)
            ss.sync()
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            ss.step(ks)
            b.record(st)
            ss.sync()
            barrier()
            sms = max_over_ranks(a.elapsed_time(b))
            ss.close()
            ctx = fill + 8 + 5 + ks / 2.0
            sb = weight_bytes(cfg) + 2 * kv_bytes_per_token(cfg) * ctx
            sweep[str(L)] = {"tokens_per_s": world * ks / (sms / 1000.0), "ms_per_step": sms / ks,
                             "context_mid": ctx, "step_bytes": sb,
                             "hbm_frac_of_measured": sb / (sms / ks * 1e-3) / 1e9 / peak,
                             "hbm_frac_of_8TBs": sb / (sms / ks * 1e-3) / 8e12}

    # ---- config 3 (batched songs): B songs of one rank in every pass (2B CFG rows; GEMV up to
    # 16 rows, tensor-core GEMMs beyond) at a ~1,024-position context (synthetic KV fill
    # ahead of 8-id prompts)
    batched = {}
    for B in ((8, 32, 64) if not args.no_sweep else ()):
        ks = 24
        mt = 4 + ks + 1
        reqs = [Request(cond[8 * i: 8 * i + 8], seed=100 * rank + i, negative=uncond[8 * i: 8 * i + 8], scale=SCALE,
                        context_fill=PROMPT - 8) for i in range(B)]
        ss = Session(model, reqs, c2_sampling(mt), Phase.VOCAB)
        st = torch.cuda.ExternalStream(ss.cuda_stream)
        ss.step(4)
        ss.sync()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        ss.step(ks)
        b.record(st)
        ss.sync()
        barrier()
        bms = max_over_ranks(a.elapsed_time(b))
        ss.close()
        ctx = PROMPT + 5 + ks / 2.0
        sb = weight_bytes(cfg) + 2 * B * kv_bytes_per_token(cfg) * ctx
        batched[str(B)] = {"songs_per_gpu": B, "rows": 2 * B, "tokens_per_s": world * B * ks / (bms / 1000.0),
                           "ms_per_step": bms / ks, "context_mid": ctx, "step_bytes": sb,
                           "hbm_frac_of_measured": sb / (bms / ks * 1e-3) / 1e9 / peak,
                           "forward": "gemm"}

    # ---- the real vocabulary (184,704 ids) in the Semantic phase: the LM head reads only the
    # 32,768-row codec window and the stop row (project_phase), a sixth of the full head
    semantic = {}
    if not args.no_sweep:
        import copy
        cs = copy.copy(cfg)
        cs.vocab_size = 184704
        ms_model = Model.synthetic(cs, seed=3, std=0.02, device=local)
        ks, wu = 24, 4
        sem = Sampling(1.0, 0.93, 50, 1.0, 50, wu + ks + 1, wu + ks + 1)  # no stop before the end
        codec_ids = lambda ids: [151853 + (t % 32768) for t in ids]
        ss = Session(ms_model, [Request(codec_ids(cond[:8]), seed=rank + 11, negative=codec_ids(uncond[:8]), scale=SCALE,
                                        context_fill=PROMPT - 8)], sem, Phase.SEMANTIC)
        st = torch.cuda.ExternalStream(ss.cuda_stream)
        ss.step(wu)
        ss.sync()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        ss.step(ks)
        b.record(st)
        ss.sync()
        barrier()
        sms = max_over_ranks(a.elapsed_time(b))
        ss.close()
        ms_model.close()
        ctx = PROMPT + wu + ks / 2.0
        H = cs.hidden_size
        sb = weight_bytes(cs) - cs.vocab_size * H * 2 + (32768 + 1) * H * 2 + 2 * kv_bytes_per_token(cs) * ctx
        semantic = {"vocab": cs.vocab_size, "phase": "semantic (codec window + MUSIC_END)",
                    "tokens_per_s": world * ks / (sms / 1000.0), "ms_per_step": sms / ks, "context_mid": ctx,
                    "step_bytes": sb, "hbm_frac_of_measured": sb / (sms / ks * 1e-3) / 1e9 / peak,
                    "lm_head_bytes_read": (32768 + 1) * H * 2, "lm_head_bytes_full": cs.vocab_size * H * 2}

    # ---- the NAR flow-matching velocity (Model::velocity) at the reference's largest acoustic
    # chunk: a 1,024-id prefix, then (CONTEXT - 1,024 - 3) / 2 = 11,774 latent frames whose
    # codec ids fill the cache, and one velocity call over all frames (non-causal attention
    # to the prefix, the codec ids and every frame)
    nar = {}
    if not args.no_sweep:
        import copy
        cn = copy.copy(cfg)
        cn.vocab_size = 184704  # the codec ids synthesize prefills
        nm = Model.synthetic(cn, seed=4, std=0.02, norm_mean=1.0, device=local, nar=True)
        frames = (24576 - PROMPT - 3) // 2
        length = PROMPT + frames + 1
        nc = nm.new_cache(24576)
        nc.fill_normal(length, seed=rank + 5)
        st = np.random.default_rng(rank).standard_normal((frames, cfg.latent_dim)).astype(np.float32)
        st = ((st.view(np.uint32).astype(np.uint64) + 0x7FFF + ((st.view(np.uint32) >> 16) & 1)) &
              0xFFFF0000).astype(np.uint32).view(np.float32)
        for _ in range(2):
            nm.velocity(st, nc, 0.5)
        reps = 3
        barrier()
        t0 = time.perf_counter()
        for _ in range(reps):
            vel = nm.velocity(st, nc, 0.5)
        vms = max_over_ranks((time.perf_counter() - t0) * 1000.0 / reps)
        assert np.isfinite(vel).all()
        n = frames + 2
        lin, att = velocity_flops(cfg, n, length + n)
        nc.close()
        # one song through Model::synthesize: a 1,024-id prefix, 4,096 codec frames (one
        # chunk), 4 midpoint steps = 8 velocity calls, host ids in / latents out
        rs = np.random.default_rng(rank + 1)
        sp = rs.integers(0, 151851, PROMPT).tolist()
        sc = rs.integers(0, 32768, 4096).tolist()
        nm.synthesize(sp, sc, seed=1, steps=1)
        barrier()
        t0 = time.perf_counter()
        lat = nm.synthesize(sp, sc, seed=2, steps=4)
        syn_s = max_over_ranks(time.perf_counter() - t0)
        assert np.isfinite(lat).all()
        nm.close()
        tf_peak, tf_kind = measured_bf16_tflops()
        nar = {"frames": frames, "prefix_positions": length, "ms_per_velocity": vms,
               "frames_per_s": world * frames / (vms / 1000.0), "linear_tflop": lin / 1e12,
               "attention_tflop": att / 1e12, "achieved_tflops": (lin + att) / (vms * 1e-3) / 1e12,
               "roofline": {"bound": "tensor", "peak": tf_peak, "unit": "TFLOP/s", "peak_kind": tf_kind,
                            "frac": (lin + att) / (vms * 1e-3) / 1e12 / tf_peak},
               "what": "yue2_velocity with host state in / velocity out, 3B-shaped NAR layers (synthetic), "
                       "one call = every frame through 28 layers; synthesize makes 2 per ODE step",
               "synthesize": {"prefix": PROMPT, "frames": 4096, "steps": 4, "seconds": syn_s,
                              "frames_per_s": world * 4096 / syn_s,
                              "what": "yue2_synthesize: prefill of 5,121 ids + 8 velocity calls of 4,098 rows"}}

    # ---- end to end through the public C ABI with host buffers (prefill included). One
    # untimed call first: the first generate of a process pays one-time costs (library
    # algorithm selection for the prefill GEMM shapes, lazy kernel loading, allocator growth)
    # that a serving process pays once, not per song.
    generate_batch(model, [Request(cond, seed=rank + 5, negative=uncond, scale=SCALE)], c2_sampling(512), Phase.VOCAB)
    barrier()
    t0 = time.perf_counter()
    outs = generate_batch(model, [Request(cond, seed=rank + 7, negative=uncond, scale=SCALE)], c2_sampling(512),
                          Phase.VOCAB)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_tokens = len(outs[0].tokens) * world
    h2d = 2 * PROMPT * 4
    d2h = 512 * 4

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,0.02) bf16 weights, uniform random prompt ids",
        "config": {"workload": "config 1: 3B-shaped AR decode (28L, H3072, 24/8 heads, I8192, V84000), CFG 1.5, "
                               "T1.0 top-k50 top-p0.93, 1,024-id cond+uncond prompts",
                   "global_batch": world, "context": f"{PROMPT + W + 1}..{PROMPT + W + K + 1}",
                   "parallelism": f"dp{world} (one song per GPU, no collective)",
                   "l2": "inputs larger than L2: 6.15 GB of weights streamed per step (126 MB L2), no flush",
                   "phase": "vocabulary-generic choose (vocab 84,000 has no codec window)"},
        "gpu_launches": kps * K,
        "clocks": clk,
        "roofline": {"bound": "hbm", "achieved": kern_gbs, "peak": peak, "unit": "GB/s", "frac": kern_gbs / peak,
                     "traffic": traffic, "kernel": "gemv gate|up + SwiGLU, 2 rows (CFG), 100.7 MB per launch; launches back to back over the 28 layers as programmatic dependents, as in the decode chain",
                     "peak_kind": peak_kind},
        "step_roofline": {"step_bytes": step_bytes, "achieved_gbs": step_bytes / (ms / K * 1e-3) / 1e9,
                          "frac_of_measured": step_bytes / (ms / K * 1e-3) / 1e9 / peak,
                          "frac_of_8TBs": step_bytes / (ms / K * 1e-3) / 8e12},
        "ctx_sweep": sweep,
        "batched": batched,
        "semantic_real_vocab": semantic,
        "nar_velocity": nar,
        "e2e": {"value": e2e_tokens / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "prefill_seconds": outs[0].prefill_seconds, "library_seconds": outs[0].seconds,
                "decode_ms": outs[0].decode_ms,
                "what": "yue2_generate: 512 tokens per song incl. both 1,024-id prefills, host buffers in/out; "
                        "timed after one untimed call of the same shape"},
    }
    model.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
        if nar:
            try:
                nar["cpu_baseline"] = cpu_velocity_baseline(cfg, nar["prefix_positions"], nar["frames"])
            except Exception as e:  # the headline line must still print
                nar["cpu_baseline"] = {"unavailable": f"{type(e).__name__}: {e}"}
    dp.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
