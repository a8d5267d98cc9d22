#!/usr/bin/env python
"""Benchmark of the denoising hot path (BASELINE.json metric: denoised tok/s per B200,
LLaDA-8B Q4_K_M, B=256, 16 steps; ms per step).

One bench "step" = one diffuse_generate call of the headline configuration (config 2):
LLaDA-8B architecture, seeded random-init weights quantized to Q4_K_M by the reference's
type policy, 64 uniform prompt ids, a 256-token masked block, 16 denoising steps,
entropy_exit remasking with tau = 0 (so every step runs), inter-step K/V cache on.

  value   tokens/s from the device time of the denoising steps (CUDA events on the
          engine's stream; the model and prompt are already resident)
  e2e     tokens/s through the public API call with host buffers (prompt in, tokens out,
          per-step stats), wall clock
  roofline the dequant-fused GEMMs (the dominant kernels) from a per-launch CUDA-event
          pass after the timed region
  cpu_baseline  the CPU oracle (a restatement of the reference's algorithm, OpenMP on
          all host cores) on a bounded sample, extrapolated by FLOPs

Multi-GPU (torchrun): every rank runs its own sequence (data parallel over independent
sequences, no collective on the data path); the timed region is bracketed by barriers and
the slowest rank's time sets the aggregate.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
MEASURED = ROOT / "MEASURED_PEAKS.json"

# DRAM bytes (read + write) over algorithmic bytes for dq_gemm_kernel, from one ncu
# capture of three launches (QKV, output, gate/up) of one LLaDA-8B-width layer over 192
# rows: 134.65 MB measured against 137.63 MB algorithmic.  Traffic per launch is
# proportional to the weight bytes streamed, so the bench scales its own algorithmic
# bytes per launch by this ratio.
NCU_GEMM_TRAFFIC_RATIO = 153.21 / 162.27


def load_pkg():
    name = "diffuse_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "diffuse-cpp_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    if MEASURED.exists():
        d = json.loads(MEASURED.read_text())
        return dict(hbm=d["hbm_gbs"], tf_burst=d["bf16_tflops"], tf_sust=d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                    src="measured")
    return dict(hbm=6650.0, tf_burst=1590.0, tf_sust=1400.0, src="fallback")


CONFIGS = {
    "c2": dict(arch="llada", scheme="q4_k_m", prompt=64, block=256, steps=16, remasking=2, tau=0.0, cache=1,
               desc="LLaDA-8B Q4_K_M random-init, prompt 64, block 256, 16 steps, entropy_exit tau=0, cache on"),
    "c1": dict(arch="llada", scheme="q4_k_m", prompt=16, block=64, steps=16, remasking=0, tau=1.5, cache=0,
               desc="LLaDA-8B Q4_K_M random-init, prompt 16, block 64, 16 steps, low_confidence, no cache"),
    # 64 independent sequences sharded over the ranks (dp.shard); one bench step generates all of
    # this rank's sequences, one after another on its GPU
    "c4": dict(arch="llada", scheme="q8_0", prompt=512, block=256, steps=16, remasking=2, tau=0.0, cache=1, n_seq=64,
               desc="LLaDA-8B Q8_0 random-init, 64 sequences x (prompt 512, block 256), 16 steps, entropy_exit tau=0, "
                    "cache on, sequences sharded over the ranks, each rank's stepped together"),
    "c4f16": dict(arch="llada", scheme="f16", prompt=512, block=256, steps=16, remasking=2, tau=0.0, cache=1, n_seq=64,
                  desc="LLaDA-8B F16 random-init, 64 sequences x (prompt 512, block 256), 16 steps, entropy_exit tau=0, "
                       "cache on, sequences sharded over the ranks, each rank's stepped together"),
    "c3": dict(arch="dream", scheme="q4_k_m", prompt=128, block=64, steps=16, remasking=2, tau=1.5, cache=1,
               desc="Dream-7B Q4_K_M random-init, prompt 128, block 64, 16 steps, entropy_exit tau=1.5, cache on"),
}


def model_file(pkg, cfg, workdir):
    arch = pkg.LLADA_8B if cfg["arch"] == "llada" else pkg.DREAM_7B
    path = pathlib.Path(workdir) / f"{cfg['arch']}_{cfg['scheme']}_seed0.gguf"
    if not path.exists():
        tmp = path.with_suffix(".tmp")
        pkg.synth_model(tmp, arch, cfg["scheme"], seed=0)
        tmp.rename(path)
    return str(path), arch


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def c2_algorithmic_flops(hp, n_active_per_step, n_keys):
    """FLOPs the reference's graph performs for these active-row counts (linears for all
    active rows, lm_head for all active rows, attention over all keys)."""
    d, ff, V, L = hp.n_embd, hp.n_ff, hp.n_vocab, hp.n_layer
    kvd = hp.n_head_kv * (d // hp.n_head)
    per_row = L * 2 * (2 * d * d + 2 * d * kvd + 3 * d * ff) + 2 * d * V
    att = L * 4 * n_keys * hp.n_head * (d // hp.n_head)
    return sum(m * (per_row + att) for m in n_active_per_step)


# Architectures of BASELINE.json's configs, for the reference arm (which imports nothing
# from the product package); the product's copies are diffuse-cpp_b200/__init__.py's.
ARCH = {
    "llada": dict(is_dream=0, n_vocab=126464, n_embd=4096, n_head=32, n_head_kv=32, n_layer=32, n_ff=12288,
                  n_ctx=4096, mask_token_id=126336, rope_theta=500000.0, rms_norm_eps=1e-5, with_bias=0),
    "dream": dict(is_dream=1, n_vocab=152064, n_embd=3584, n_head=28, n_head_kv=4, n_layer=28, n_ff=18944,
                  n_ctx=131072, mask_token_id=151666, rope_theta=1000000.0, rms_norm_eps=1e-6, with_bias=1),
}


def host_threads():
    """Host cores this process may use (torchrun's OMP_NUM_THREADS=1 does not apply here)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_model_file(cfg, workdir):
    """The config's model written by the CPU oracle's own synthesizer (byte-identical to the
    product's, tests/test_host_cpu.py), so the reference arm loads no product library."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle
    path = pathlib.Path(workdir) / f"{cfg['arch']}_{cfg['scheme']}_seed0.gguf"
    if not path.exists():
        tmp = path.with_suffix(".otmp")
        oracle.synth_model(tmp, ARCH[cfg["arch"]], cfg["scheme"], seed=0, n_threads=host_threads())
        tmp.rename(path)
    return str(path)


def step_flops(arch, n_active, n_keys):
    """Algorithmic FLOPs of one denoising step of the reference's graph: linears and
    lm_head for the active rows, attention of the active rows over all keys."""
    d, ff, V, L, H = arch["n_embd"], arch["n_ff"], arch["n_vocab"], arch["n_layer"], arch["n_head"]
    kvd = arch["n_head_kv"] * (d // H)
    return n_active * (L * 2 * (2 * d * d + 2 * d * kvd + 3 * d * ff) + 2 * d * V + L * 4 * n_keys * d)


_ORACLE_MODELS = {}


def reference_sample(path, cfg, prompt, threads):
    """The reference's loop (the CPU oracle's session: full forward of step 0, then the
    sampler, then the cached forward of step 1, all layers) on the host cores; returns
    (seconds of the two forwards, their algorithmic FLOPs, rows of step 1)."""
    from oracle import oracle
    om = _ORACLE_MODELS.get(path)
    if om is None:  # loaded once per process: every bench step samples the same file
        om = _ORACLE_MODELS[path] = oracle.OracleModel(path)
    prm = oracle.SamplerParams(n_steps=cfg["steps"], remasking=cfg["remasking"], entropy_threshold=cfg["tau"],
                               use_cache=cfg["cache"])
    sess = oracle.OracleSession(om, prompt, cfg["block"], prm, n_threads=threads)
    n = cfg["prompt"] + cfg["block"]
    t0 = time.perf_counter()
    rows0 = sess.forward(0)
    t1 = time.perf_counter()
    sess.sample(0)
    t2 = time.perf_counter()
    rows1 = sess.forward(1)
    t3 = time.perf_counter()
    sess.close()
    arch = ARCH[cfg["arch"]]
    return (t1 - t0) + (t3 - t2), step_flops(arch, rows0, n) + step_flops(arch, rows1, n), rows1


def run_reference(args, cfg):
    """--impl reference: the reference's algorithm on the host cores.  The reference itself
    cannot be built (its ggml submodule is empty), so this is the CPU oracle, which
    restates it; no product library is loaded.  One bench step = the first two denoising
    steps of one generation at full depth (a full and a cached forward), timed, and the
    whole 16-step generation extrapolated from them by algorithmic FLOPs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    work = pathlib.Path(os.environ.get("DFB_BENCH_DIR", tempfile.gettempdir())) / "dfb_bench"
    work.mkdir(parents=True, exist_ok=True)
    path = oracle_model_file(cfg, work)
    arch = ARCH[cfg["arch"]]
    rows = c2_active_rows(cfg)
    n_keys = cfg["prompt"] + cfg["block"]
    total_flops = sum(step_flops(arch, m, n_keys) for m in rows)
    rng = np.random.default_rng(1234)
    rates, dts = [], []
    for i in range(args.warmup + args.steps):
        prompt = rng.integers(0, min(arch["mask_token_id"], arch["n_vocab"]) - 1, cfg["prompt"]).astype(np.int32)
        dt, fl, _ = reference_sample(path, cfg, prompt, threads)
        if i >= args.warmup:
            rates.append(fl / dt)
            dts.append(dt)
    rate = statistics.median(rates)
    t_run = total_flops / rate
    tok_s = cfg["block"] / t_run
    metric = ("denoised tok/s per B200 (LLaDA-8B Q4_K_M, B=256, 16 steps)" if args.config == "c2"
              else f"denoised tok/s ({args.config})")
    sample = (f"full-depth forwards of denoising steps 0 (full, {n_keys} rows) and 1 (cached, {rows[1]} active rows) "
              f"of the reference's loop, {threads} threads; the 16-step run extrapolated by algorithmic FLOPs "
              f"({rate / 1e9:.0f} GFLOP/s)")
    line = {"impl": "reference", "metric": metric, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            # a bench step is the timed sample (two denoising steps at full depth); the
            # generation it stands for is extrapolated
            "ms_per_step": statistics.median(dts) * 1e3, "extrapolated_ms_per_generation": t_run * 1e3,
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg["desc"]}, "extrapolated": True, "sampled_denoising_steps": 2,
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def layer_probe(args):
    """Small profiling case (a few hundred MB on the device): one layer of LLaDA-8B width
    (Dream-7B width with --probe-arch dream: GQA 28 / 4),
    `--warmup` untimed forwards, then `--steps` forwards with the engine's per-launch
    CUDA-event profiler on; prints calls, average launch time, TFLOP/s and algorithmic
    GB/s per kernel class.  Launch order of one forward: embed, norm, QKV GEMM, attention,
    output GEMM, norm, gate/up GEMM, down GEMM (Q6_K: first FFN), final norm, lm_head.
    --probe-vocab sets the vocabulary (126464: LLaDA-8B's, so the sampler kernels read
    full-size logits rows); --probe-generate then runs one denoising step of a ROWS-token
    block (the sampler kernels: candidate statistics, commit) after the forwards."""
    import ctypes as C
    pkg = load_pkg()
    os.environ.setdefault("DIFFUSE_LOG_LEVEL", "0")
    work = pathlib.Path(os.environ.get("DFB_BENCH_DIR", tempfile.gettempdir())) / "dfb_bench"
    work.mkdir(parents=True, exist_ok=True)
    arch = pkg.DREAM_7B if args.probe_arch == "dream" else pkg.LLADA_8B
    V = args.probe_vocab
    path = work / f"{args.probe_arch}_q4_k_m_1layer_v{V}.gguf"
    if not path.exists():
        tmp = path.with_suffix(".tmp")
        pkg.synth_model(tmp, arch, "q4_k_m", seed=0, n_layer=1, n_vocab=V)
        tmp.rename(path)
    model = pkg.Model(str(path))
    M = args.layer_probe
    ctx = pkg.Context(model, max(M, 512))
    dfb, _ = pkg.native()

    class Prof(C.Structure):
        _fields_ = [("calls", C.c_int32), ("ms", C.c_double), ("flops", C.c_double), ("bytes", C.c_double)]
    dfb.dfb_ctx_profile.argtypes = [C.c_void_p, C.c_int]
    dfb.dfb_ctx_profile_read.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    toks = np.random.default_rng(0).integers(0, min(V, 16000), M).astype(np.int32)
    for _ in range(args.warmup):
        ctx.forward(toks)
    dfb.dfb_ctx_profile(ctx.engine, 1)
    for _ in range(args.steps):
        ctx.forward(toks)
    prof = (Prof * 7)()
    dfb.dfb_ctx_profile_read(ctx.engine, prof, 7)
    dfb.dfb_ctx_profile(ctx.engine, 0)
    for i, n in enumerate(["gemm_all", "q4_k", "q6_k", "q8_0", "f16", "lm_head", "attention"]):
        p = prof[i]
        if p.calls:
            print(f"rows {M:4d} {n:9s} calls {p.calls:4d} avg {p.ms / p.calls * 1e3:8.1f} us "
                  f"{p.flops / (p.ms * 1e-3) / 1e12:7.1f} TFLOP/s {p.bytes / (p.ms * 1e-3) / 1e9:7.1f} GB/s", flush=True)
    if args.probe_generate:
        P = 16
        hp = model.hparams
        prompt = np.random.default_rng(1).integers(0, min(hp.mask_token_id, V) - 1, P).astype(np.int32)
        out, tr = ctx.generate(prompt, M - P, pkg.SamplerParams(n_steps=1, remasking=0, use_cache=0), trace=True)
        print(f"generate: one step over {M} rows, {int(tr['n_unmasked'][0])} committed, {float(tr['step_ms'][0]):.3f} ms", flush=True)
    ctx.close()
    model.close()
    return 0


def c2_active_rows(cfg):
    """Active rows per denoising step of the reference's cached loop when no position
    changes except the committed ones (step 0 full, then masked + just committed)."""
    from math import cos, pi
    B, S, P = cfg["block"], cfg["steps"], cfg["prompt"]
    rows, masked, prev_commit = [], B, 0
    for s in range(S):
        if masked == 0:
            break
        rows.append(P + B if (s == 0 or not cfg["cache"]) else masked + prev_commit)
        t0, t1 = s / S, (s + 1) / S
        c0, c1 = np.float32(cos(np.float32(t0) * pi * 0.5)), np.float32(cos(np.float32(t1) * pi * 0.5))
        k = int(round(float(np.float32((c0 - c1) / c0) * masked)))
        k = max(1, min(k, masked))
        prev_commit = k
        masked -= k
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", action="store_true",
                    help="under torchrun: the ranks run one sequence tensor-parallel instead of one each")
    ap.add_argument("--probe-arch", default="llada", choices=["llada", "dream"])
    ap.add_argument("--probe-vocab", type=int, default=16384)
    ap.add_argument("--probe-generate", action="store_true")
    ap.add_argument("--layer-probe", type=int, default=0, metavar="ROWS",
                    help="profiling case instead of the benchmark: forwards of ROWS tokens through one "
                         "LLaDA-8B-width Q4_K_M layer (vocab 16384), per-kernel-class CUDA-event timings")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.layer_probe:
        return layer_probe(args)
    if args.impl == "reference":
        return run_reference(args, cfg)

    pkg = load_pkg()
    # one process per GPU (torchrun); each rank generates its own sequences, nothing
    # crosses ranks on the data path (diffuse-cpp_b200/dp.py)
    dp = pkg.dp.DataParallel.from_env(timeout_s=600, backend="nccl")
    world, rank, local = dp.world, dp.rank, dp.local
    os.environ["DIFFUSE_DEVICE"] = str(local)
    os.environ.setdefault("DIFFUSE_LOG_LEVEL", "0")
    barrier, reduce_max = dp.barrier, dp.max_over_ranks

    work = pathlib.Path(os.environ.get("DFB_BENCH_DIR", tempfile.gettempdir())) / "dfb_bench"
    work.mkdir(parents=True, exist_ok=True)
    t_synth = time.perf_counter()
    if rank == 0:
        path, arch = model_file(pkg, cfg, work)
    barrier()
    if rank != 0:
        path, arch = model_file(pkg, cfg, work)
    t_synth = time.perf_counter() - t_synth
    # --tp: the ranks form one tensor-parallel group over a single sequence (heads, FFN features
    # and vocabulary split; NCCL all-reduce after O and down) instead of independent replicas
    tp = bool(args.tp) and world > 1
    if tp and cfg.get("n_seq"):
        raise SystemExit("--tp runs the single-sequence configurations (c1, c2, c3)")
    if tp:
        nid = dp.broadcast_bytes(pkg.tp_unique_id() if rank == 0 else b"")
        model = pkg.Model(path, tp=(rank, world, nid))
    else:
        model = pkg.Model(path)
    hp = model.hparams
    P, B = cfg["prompt"], cfg["block"]
    params = pkg.SamplerParams(n_steps=cfg["steps"], remasking=cfg["remasking"], entropy_threshold=cfg["tau"],
                               use_cache=cfg["cache"])
    rng = np.random.default_rng(1234 if tp else 1234 + rank)  # one shared sequence under --tp
    # sequences of one bench step on this rank: one (configs 1-3) or this rank's share of
    # n_seq, all stepped together in one forward per denoising step (generate_batch)
    batched = bool(cfg.get("n_seq"))
    my_seq = pkg.dp.shard(cfg["n_seq"], rank, world) if batched else range(1)
    n_seq_total = cfg["n_seq"] if batched else (1 if tp else world)
    ctx = pkg.Context(model, (P + B) * len(my_seq))
    prompts = [[rng.integers(0, min(hp.mask_token_id, hp.n_vocab) - 1, P).astype(np.int32) for _ in my_seq]
               for _ in range(args.warmup + args.steps)]

    def run(prs):
        """One bench step: device ms of its denoising steps and the active rows per step."""
        if batched:
            _, tr = ctx.generate_batch(prs, B, params, trace=True)
            n = tr["steps_run"]
            return float(tr["step_ms"][:n].sum()), tr["n_active"][:n].sum(axis=1).tolist()
        _, tr = ctx.generate(prs[0], B, params, trace=True)
        n = tr["steps_run"]
        return float(tr["step_ms"][:n].sum()), tr["n_active"][:n].tolist()

    for i in range(args.warmup):
        run(prompts[i])
    barrier()
    dev_ms, wall_ms, actives = [], [], []
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            t0 = time.perf_counter()
            d, actives = run(prompts[args.warmup + i])
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            dev_ms.append(d)
    barrier()
    tot_dev = reduce_max(sum(dev_ms))
    tot_wall = reduce_max(sum(wall_ms))

    # roofline pass: per-launch CUDA events around every GEMM of one more bench step
    dfb, _ = pkg.native()
    import ctypes as C

    class Prof(C.Structure):
        _fields_ = [("calls", C.c_int32), ("ms", C.c_double), ("flops", C.c_double), ("bytes", C.c_double)]
    dfb.dfb_ctx_profile.argtypes = [C.c_void_p, C.c_int]
    dfb.dfb_ctx_profile_read.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    dfb.dfb_ctx_profile(ctx.engine, 1)
    run(prompts[-1])
    prof = (Prof * 7)()
    dfb.dfb_ctx_profile_read(ctx.engine, prof, 7)
    dfb.dfb_ctx_profile(ctx.engine, 0)
    g = prof[0]
    pk = peaks()
    gemm_tflops = g.flops / (g.ms * 1e-3) / 1e12 if g.ms > 0 else 0.0
    per_launch_bytes = g.bytes / max(g.calls, 1)
    roofline = {"bound": "tensor", "achieved": gemm_tflops, "peak": pk["tf_burst"], "unit": "TFLOP/s",
                "frac": gemm_tflops / pk["tf_burst"], "frac_of_sustained": gemm_tflops / pk["tf_sust"],
                "traffic": NCU_GEMM_TRAFFIC_RATIO * per_launch_bytes,
                "traffic_source": "ncu dram bytes / algorithmic bytes on a small capture of the same kernel, "
                                  "x this run's algorithmic bytes per launch",
                "peak_source": f"{pk['src']} bf16 burst (cuBLAS 8192^3); f16 operands run at the bf16 rate",
                "tensor_work_per_algorithmic_flop": 2.0,
                "tensor_work_note": "each product is an f16 MMA plus one E4M3 MMA over twice the K (the two "
                                    "precision corrections) at twice the f16 rate: 2x the algorithmic f16 work",
                "kernel": "dq_gemm_kernel (all linears of one bench step)", "launches": g.calls,
                "avg_launch_us": g.ms * 1e3 / max(g.calls, 1), "algorithmic_bytes_per_launch": per_launch_bytes,
                "hbm_gbs_achieved": g.bytes / (g.ms * 1e-3) / 1e9 if g.ms > 0 else 0.0,
                "breakdown": {name: {"calls": prof[i].calls, "ms": prof[i].ms,
                                     "tflops": prof[i].flops / (prof[i].ms * 1e-3) / 1e12 if prof[i].ms else 0}
                              for i, name in [(1, "q4_k"), (2, "q6_k"), (3, "q8_0"), (4, "f16"), (5, "lm_head"),
                                              (6, "attention")]}}

    tokens_all = B * args.steps * n_seq_total
    value = tokens_all / (tot_dev * 1e-3)
    e2e = tokens_all / (tot_wall * 1e-3)
    flops_run = c2_algorithmic_flops(hp, actives, P + B)
    launches_per_denoise_step = 7 * hp.n_layer + 6
    T, S = (P + B) * len(my_seq), len(my_seq)
    h2d = 4 * T * 3 + T + len(actives) * 5 * S      # seq, prev_seq, last_changed, masks; per step schedule + flags
    d2h = len(actives) * (4 * 8 * (S + 1) + 4) + 4 * T  # per-step counters + error flag, final tokens
    line = {
        "metric": "denoised tok/s per B200 (LLaDA-8B Q4_K_M, B=256, 16 steps)" if args.config == "c2" else
        f"denoised tok/s ({args.config})",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_dev / args.steps, "higher_is_better": True, "scaling": "strong" if tp else "weak",
        "vs_baseline": None,
        "dtype": "f32-exact products (f16 hi x f16 hi + e4m3 corrections, f32 accumulation); f32 attention",
        "data": "synthetic",
        "config": {"workload": cfg["desc"], "prompt_len": P, "block": B, "denoise_steps": cfg["steps"],
                   "step_definition": ("one generate_batch call: this rank's sequences stepped together"
                                       if batched else "one diffuse_generate call (all denoising steps of one sequence)"),
                   "sequences_per_rank": len(my_seq),
                   "l2": "inputs larger than L2: the weights (4.4-15 GB) stream from HBM every denoising step",
                   "parallelism": (f"tp{world} (one sequence; NCCL all-reduce after O and down)" if tp
                                   else f"dp{world} (independent sequences)"),
                   "value_scope": "tokens of all ranks / the slowest rank's device time",
                   "active_rows_per_denoising_step": actives,
                   "denoising_step_ms": (tot_dev / args.steps) / max(len(actives), 1),
                   "algorithmic_tflop_per_step": flops_run / 1e12,
                   "model_synth_s": round(t_synth, 1)},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": tot_wall / args.steps},
        "roofline": roofline,
        "gpu_launches": launches_per_denoise_step * len(actives) * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not batched:
        try:
            threads = host_threads()
            dt, fl, rows1 = reference_sample(path, cfg, prompts[-1][0], threads)
            t_run = flops_run / (fl / dt)
            line["cpu_baseline"] = {"value": B / t_run, "unit": "tok/s", "cores": threads, "kind": "port",
                                    "sample": f"CPU oracle (the reference's algorithm) on the same model: full-depth "
                                              f"forwards of denoising steps 0 and 1 ({dt:.1f} s, "
                                              f"{fl / dt / 1e9:.0f} GFLOP/s), the run extrapolated by its FLOPs",
                                    "extrapolated": True}
        except Exception as e:  # the baseline is context, never a reason to lose the line
            line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"failed: {e}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    model.close()
    dp.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
