"""Benchmark of the B200 Lunelette decoder backend (one JSON line on rank 0).

Workload ("C0"): the Ministral-3-3B-shaped decoder with a
seeded random-init checkpoint, batch 1, a 32-token prompt of ids ~ U[1000,
131072), greedy decode at context profile 256. A "step" is one greedy decode
token. The timed region is R rounds of: restore the 32-token prompt checkpoint
(host-only, no device work) and decode 31 greedy tokens on the device
(lunelette_cuda_decode_loop: one launch of the persistent decode kernel for the
31 tokens, argmax fed back on the GPU). `value` = decode tokens/s from CUDA
events (max over ranks, all ranks' tokens summed); `e2e` = the same metric
through the drop-in C-ABI with host buffers (lunelette_metal_decode + host
greedy each token: one persistent-kernel launch per token, H2D of the step
parameters and D2H of the 131072 logits inside the timed region). `roofline`
is the persistent kernel's: the algorithmic bytes of a launch (FP8 linears,
BF16 head, norm gains and the FP32 KV rows read) over its CUDA-event time.

Multi-GPU: one process per GPU (torchrun), each an independent weight replica
and session ("replicas only": the model has no collective), so scaling is weak.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tok/s (batch 1 and aggregate) + prefill tok/s, % of HBM/FP8 roofline"
PROMPT = 32
CONTEXT = 256
WEIGHT_BYTES_PER_TOKEN = 3026190336 + 805306368 + 53 * 3072 * 4  # FP8 linears + BF16 head + norms
KV_BYTES_PER_POSITION = 26 * 2 * 1024 * 4                         # FP32 K and V, all layers
GATEUP_BYTES = 18432 * 3072                                       # one fused gate/up launch
HEAD_BYTES = 131072 * 3072 * 2
# DRAM read + write bytes of one C0 decode token: ncu capture of a one-token
# launch of decode_mega_kernel at context 34 (profiles/decode_mega_c0_token.md:
# 3,839,687,168 read + 7,772,160 written)
DRAM_BYTES_PER_TOKEN = 3854483968 + 8470272


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q, "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def ensure_checkpoint(path, rank, world, barrier):
    import lunelette_b200 as L
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".partial%d" % os.getpid()
        L.synth_checkpoint(tmp, 0)
        os.replace(tmp, path)
    barrier()
    return path


def safetensors_slice(path, name):
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
        begin, end = header[name]["data_offsets"]
        f.seek(8 + n + begin)
        return np.frombuffer(f.read(end - begin), np.uint8)


def gateup_roofline(lib, torch, checkpoint, launches=40):
    """Average CUDA-event duration of the fused norm+gate/up+SwiGLU GEMV on the
    launching stream, rotating over 4 layers' weights (226 MB > L2)."""
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    copies = []
    for layer in range(4):
        gate = safetensors_slice(checkpoint, "language_model.model.layers.%d.mlp.gate_proj.weight" % layer)
        up = safetensors_slice(checkpoint, "language_model.model.layers.%d.mlp.up_proj.weight" % layer)
        raw = torch.from_numpy(np.concatenate([gate, up])).cuda()
        tiled = torch.empty(raw.numel(), dtype=torch.uint8, device="cuda")
        assert lib.lunelette_cuda_tile_fp8(raw.data_ptr(), 18432, 3072, 2, tiled.data_ptr(), s) == 0
        torch.cuda.synchronize()
        copies.append(tiled)
    x = torch.randn(3072, device="cuda")
    gain = torch.ones(3072, device="cuda")
    act = torch.empty(9216, device="cuda")

    def launch(i):
        rc = lib.lunelette_cuda_gateup_swiglu(copies[i % 4].data_ptr(), 2e-4, 2e-4, gain.data_ptr(),
                                              x.data_ptr(), 1, act.data_ptr(), s)
        assert rc == 0

    for i in range(8):
        launch(i)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(launches):
        launch(i)
    stop.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / launches
    algorithmic = GATEUP_BYTES + 3072 * 4 * 2 + 9216 * 4  # weights + x + gain + act out
    return ms, algorithmic


def traffic_per_launch(steps):
    """DRAM bytes (read + write) of a persistent-kernel launch of `steps` tokens,
    from the ncu capture summarised in profiles/ (one single-token launch on the
    C0 workload, scaled by the token count: the kernel's traffic is per token),
    or None when no capture has been summarised."""
    per_token = DRAM_BYTES_PER_TOKEN
    return None if per_token is None else per_token * steps


def prefill_gemm_roofline(lib, torch, count=256, reps=20):
    """Device time of the tcgen05 prefill GEMM (prefill_gemm_pair_kernel) for
    the gate/up projection of a 256-token block, from CUDA events on its
    stream (lunelette_cuda_gemm_fp8_timed, back-to-back launches rotating 5
    weight copies: 283 MB > L2). FLOPs: `issued` counts the tensor core's work
    (hi and lo passes, 256-token pair tiles), `useful` the projection's own
    2 * rows * cols * count."""
    import ctypes
    rows, cols, copies = 18432, 3072, 5
    gen = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randint(0, 256, (copies * rows * cols,), device="cuda", dtype=torch.uint8, generator=gen)
    w[(w & 127) == 127] = 0
    x = torch.randn(count, cols, device="cuda", generator=gen)
    y = torch.empty(count, rows, device="cuda")
    ms = (ctypes.c_float * 3)()
    s = torch.cuda.current_stream().cuda_stream
    for n in (copies, reps):
        assert lib.lunelette_cuda_gemm_fp8_timed(w.data_ptr(), copies, rows, cols, 1.0, x.data_ptr(), count,
                                                 y.data_ptr(), n, ms, s) == 0
    tiles = (count + 255) // 256
    issued = 2 * 2 * ((rows + 511) // 512 * 512) * cols * 256 * tiles
    useful = 2 * rows * cols * count
    return {"split_ms": ms[0], "gemm_ms": ms[1], "finish_ms": ms[2], "issued_flops": issued,
            "useful_flops": useful}


def config_lines(L, torch, checkpoint, seed, barrier, max_over_ranks, world):
    """BASELINE configs 2-4 on one batch context (64 sessions x 4352 positions,
    a paged FP32 KV pool of 59 GB): wall clock around host-synchronous calls.
      C2: 4096 seeded ids in 16 chunks of 256 at context 4352, then 128 greedy
          decode steps (persistent kernel);
      C3: a 512-token prefix, then 8 turns of 200 appended ids + 64 greedy tokens
          on the same session (its KV kept between turns); TTFT = the append;
      C4: 64 sessions, prompts ~ U[256, 4096] (seeded), prefilled in 256-token
          chunks, then 128 batched greedy decode steps over all 64 sessions.
    Aggregates sum the ranks' work over the slowest rank's time."""
    rng = np.random.default_rng(seed + 99)
    out = {}
    with L.Batch(checkpoint, max_sessions=64, context=4352, pool_positions=64 * 4352, block=256) as b:
        # C2
        s = b.open()
        ids = rng.integers(1000, 131072, 4096).astype(np.int64)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for c in range(16):
            logits = b.append(s, ids[256 * c:256 * (c + 1)])
        t_prefill = max_over_ranks(time.perf_counter() - t0)
        tok = int(np.argmax(logits))
        t0 = time.perf_counter()
        for _ in range(128):
            tok = int(np.argmax(b.append(s, [tok])))
        t_decode = max_over_ranks(time.perf_counter() - t0)
        b.close_session(s)
        out["c2"] = {"prefill_tok_s": world * 4096 / t_prefill, "decode_tok_s": world * 128 / t_decode,
                     "note": "4096-token prompt in 16 x 256 chunks at context 4352, then 128 greedy steps"}
        # C3
        s = b.open()
        prefix = rng.integers(1000, 131072, 512).astype(np.int64)
        b.append(s, prefix[:256])
        b.append(s, prefix[256:])
        ttft, dec = [], []
        for turn in range(8):
            user = rng.integers(1000, 131072, 200).astype(np.int64)
            t0 = time.perf_counter()
            tok = int(np.argmax(b.append(s, user)))
            ttft.append(time.perf_counter() - t0)
            t0 = time.perf_counter()
            for _ in range(63):
                tok = int(np.argmax(b.append(s, [tok])))
            dec.append(64 / (time.perf_counter() - t0))
        b.close_session(s)
        out["c3"] = {"ttft_ms_mean": 1e3 * max_over_ranks(float(np.mean(ttft))),
                     "ttft_ms_last_turn": 1e3 * max_over_ranks(ttft[-1]),
                     "decode_tok_s_per_turn_mean": float(np.mean(dec)),
                     "note": "512-token prefix, 8 turns of 200 appended ids + 64 greedy tokens, KV kept"}
        # C4
        lengths = rng.integers(256, 4097, 64)
        sessions = [b.open() for _ in range(64)]
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        toks = []
        for s, n in zip(sessions, lengths):
            ids = rng.integers(1000, 131072, int(n)).astype(np.int64)
            for c0 in range(0, int(n), 256):
                logits = b.append(s, ids[c0:c0 + 256])
            toks.append(int(np.argmax(logits)))
        t_prefill = max_over_ranks(time.perf_counter() - t0)
        t0 = time.perf_counter()
        for _ in range(128):
            toks = b.decode(sessions, toks).tolist()
        t_decode = max_over_ranks(time.perf_counter() - t0)
        out["c4"] = {"decode_tok_s_aggregate": world * 64 * 128 / t_decode,
                     "prefill_tok_s_aggregate": world * float(lengths.sum()) / t_prefill,
                     "ms_per_batched_step": 1e3 * t_decode / 128, "sessions_per_gpu": 64,
                     "mean_prompt": float(lengths.mean()),
                     "note": "64 ragged sessions per GPU, prompts U[256,4096], 128 batched greedy steps"}
    return out


def cpu_baseline(checkpoint, prompt, decode_steps=6):
    """The CPU oracle (C restatement of the reference kernels, OpenMP) on this
    box's host cores: the C0 prompt, then `decode_steps` greedy decode steps."""
    from tests import oracle_lib
    o = oracle_lib.load()
    m = o.open_model(checkpoint, CONTEXT)
    try:
        t0 = time.perf_counter()
        logits, _, _ = m.forward(prompt)
        t1 = time.perf_counter()
        tok = int(np.argmax(logits))
        for _ in range(decode_steps):
            logits, _, _ = m.forward([tok])
            tok = int(np.argmax(logits))
        t2 = time.perf_counter()
    finally:
        m.close()
    return {"value": decode_steps / (t2 - t1), "unit": "tok/s", "cores": o.threads(), "kind": "port",
            "sample": "C0 prompt of %d ids prefilled (%.2f s = %.1f tok/s), then %d greedy decode steps "
                      "timed; oracle/oracle.c FP32, OpenMP" % (len(prompt), t1 - t0, len(prompt) / (t1 - t0),
                                                                decode_steps),
            "prefill_tok_s": len(prompt) / (t1 - t0)}


class Ranks:
    """Rank plumbing of the bench: one process per GPU, replicas only (no
    data-path collective). `barrier` lines the ranks up around timed regions and
    `max` takes the slowest rank's time; with no process group (N = 1) both are
    no-ops. `device` is where the reduction tensor lives ("cuda" under NCCL,
    "cpu" under gloo in the tests)."""

    def __init__(self, dist=None, device="cpu"):
        self.dist = dist
        self.device = device

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, v):
        if self.dist is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def aggregate_rate(world, units_per_rank, slowest_seconds):
    """Whole-job throughput: the units every rank processed over the slowest
    rank's time (weak scaling: per-rank work is fixed)."""
    return world * units_per_rank / slowest_seconds


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path: this repo's oracle port of
    its Metal kernels (the Metal runtime itself cannot run off Apple hardware)."""
    if rank != 0:
        return 0
    import lunelette_b200 as L  # only for the synthetic checkpoint writer
    checkpoint = ensure_checkpoint(args.checkpoint, 0, 1, lambda: None)
    from tests import oracle_lib
    o = oracle_lib.load()
    prompt = np.random.default_rng(args.seed).integers(1000, 131072, PROMPT).astype(np.int64)
    # each step is one greedy token of the FP32 oracle on the host cores
    # (~0.18 s): at most 256 timed steps keep the run within a few minutes
    steps = min(args.steps, 256)
    warmup = min(max(args.warmup, 3), 5)
    m = o.open_model(checkpoint, CONTEXT)
    try:
        logits, _, _ = m.forward(prompt)
        first = int(np.argmax(logits))
        per_round = min(CONTEXT - PROMPT - 1, 31)

        def decode(n):
            # rounds of 31 greedy tokens from the prompt, as our arm's rounds
            tok = first
            m.rewind(PROMPT)
            for i in range(n):
                if i and i % per_round == 0:
                    m.rewind(PROMPT)
                    tok = first
                logits, _, _ = m.forward([tok])
                tok = int(np.argmax(logits))

        decode(warmup)
        t0 = time.perf_counter()
        decode(steps)
        elapsed = time.perf_counter() - t0
    finally:
        m.close()
    value = steps / elapsed
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": 1000 * elapsed / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init checkpoint, seeded token ids)",
            "config": {"workload": "C0: batch-1 greedy decode after a 32-token prompt, context 256",
                       "prompt": PROMPT, "context": CONTEXT},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": o.threads(), "kind": "port",
                             "sample": "%d greedy decode steps in rounds of 31 after the 32-token prompt "
                                       "(bounded sample of C0); oracle/oracle.c FP32 restatement of the "
                                       "reference's Metal kernels, OpenMP" % steps},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def run_ours(args, rank, world, local_rank):
    import torch
    import lunelette_b200 as L
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    ranks = Ranks(dist, "cuda")
    barrier, max_over_ranks = ranks.barrier, ranks.max

    lib = L.library()
    checkpoint = ensure_checkpoint(args.checkpoint, rank, world, barrier)
    rt = L.Runtime(checkpoint)  # default options, profile C=256/B=256
    prompt = np.random.default_rng(args.seed + rank).integers(1000, 131072, PROMPT).astype(np.int64)
    per_round = CONTEXT - PROMPT - 1
    per_round = min(per_round, 31)  # C0: 32 greedy tokens, the first from the prefill
    rounds = max(1, (args.steps + per_round - 1) // per_round)
    steps = rounds * per_round

    # ---- warm-up: untimed decode steps (also captures the decode graph)
    rt.reset()
    first = int(np.argmax(rt.prefill(prompt)))
    cp = rt.checkpoint_create()
    rt.decode_loop(first, max(args.warmup, 3))
    rt.checkpoint_restore(cp)

    # ---- value: device-resident decode, CUDA events
    barrier()
    torch.cuda.synchronize()
    device_ms = 0.0
    launches = 0
    tokens_seen = None
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        for r in range(rounds):
            tokens, ms, n = rt.decode_loop(first, per_round)
            device_ms += ms
            launches += n
            rt.checkpoint_restore(cp)
            tokens_seen = tokens
        torch.cuda.synchronize()
        wall_ms = 1000 * (time.perf_counter() - t0)
    barrier()
    device_ms = max_over_ranks(device_ms)
    value = aggregate_rate(world, steps, device_ms / 1000)

    # ---- e2e: the drop-in C-ABI with host buffers, host greedy each token
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_tokens = []
    for r in range(rounds):
        logits = rt.checkpoint_restore(cp)
        tok = int(np.argmax(logits))
        for i in range(per_round):
            logits = rt.decode(tok)
            e2e_tokens.append(tok)
            tok = int(np.argmax(logits))
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = aggregate_rate(world, steps, e2e_s)
    # the device loop and the host loop must generate the same greedy tokens
    same_tokens = list(e2e_tokens[1:per_round]) == [int(t) for t in tokens_seen[:per_round - 1]]

    # ---- prefill: 256-token chunk and the 32-token prompt through the C-ABI
    chunk = np.random.default_rng(args.seed + 17).integers(1000, 131072, 256).astype(np.int64)
    for _ in range(2):
        rt.reset()
        rt.prefill(chunk)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        rt.reset()
        rt.prefill(chunk)
    prefill_256 = max_over_ranks((time.perf_counter() - t0) / reps)
    t0 = time.perf_counter()
    for _ in range(reps):
        rt.reset()
        rt.prefill(prompt)
    prefill_32 = max_over_ranks((time.perf_counter() - t0) / reps)
    cp.destroy()
    rt.close()

    configs = None if args.no_configs else config_lines(L, torch, checkpoint, args.seed + rank, barrier,
                                                         max_over_ranks, world)
    hbm, bf16, peak_kind = measured_peaks()
    gemv_ms, gemv_bytes = gateup_roofline(lib, torch, checkpoint)
    pg = prefill_gemm_roofline(lib, torch)
    ms_per_step = device_ms / steps
    mean_ctx = PROMPT + (per_round + 1) / 2
    step_bytes = WEIGHT_BYTES_PER_TOKEN + KV_BYTES_PER_POSITION * mean_ctx
    launch_ms = device_ms / launches            # one persistent-kernel launch per round
    launch_bytes = step_bytes * steps / launches
    achieved = launch_bytes / (launch_ms / 1000) / 1e9

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 weights, fp32 activations/accumulation/kv",
            "data": "synthetic (seeded random-init checkpoint in the reference's tensor layout, seeded ids)",
            "config": {"workload": "C0: batch-1 greedy decode after a 32-token prompt, context profile 256",
                       "prompt": PROMPT, "decode_per_round": per_round, "rounds": rounds,
                       "parallelism": "replicas (one weight replica and session per GPU)",
                       "l2": "inputs larger than L2: each step streams %.2f GB of weights" % (step_bytes / 1e9)},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 1040,
                    "d2h_bytes_per_step": 131072 * 4 + 4,
                    "note": "lunelette_metal_decode per token, host greedy on the borrowed logits"},
            "prefill_tok_s": {"chunk_256": 256 / prefill_256, "prompt_32": PROMPT / prefill_32,
                              "note": "lunelette_metal_prefill wall time, host ids and logits"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic_per_launch(per_round), "peak_kind": peak_kind,
                         "kernel": "decode_mega_kernel (persistent: %d greedy tokens per launch)" % per_round,
                         "algorithmic_bytes": launch_bytes, "avg_launch_ms": launch_ms,
                         "bytes_per_token": step_bytes},
            "gemv_roofline": {"kernel": "gemv_tiled_kernel<1,kEpiSwiGLU> (fused norm + gate/up + SwiGLU, "
                                        "standalone launches, weights > L2)",
                              "achieved": gemv_bytes / (gemv_ms / 1000) / 1e9, "unit": "GB/s",
                              "frac": gemv_bytes / (gemv_ms / 1000) / 1e9 / hbm, "algorithmic_bytes": gemv_bytes,
                              "avg_launch_ms": gemv_ms},
            "prefill_roofline": {
                "kernel": "prefill_gemm_pair_kernel (tcgen05 cta_group::2, FP16 hi + lo passes, gate/up "
                          "18432x3072, 256 tokens, weights > L2)",
                "bound": "tensor", "unit": "TFLOP/s", "peak": bf16, "peak_kind": peak_kind,
                "achieved": pg["issued_flops"] / (pg["gemm_ms"] / 1e3) / 1e12,
                "frac": pg["issued_flops"] / (pg["gemm_ms"] / 1e3) / 1e12 / bf16,
                "useful_tflops": pg["useful_flops"] / (pg["gemm_ms"] / 1e3) / 1e12,
                "avg_launch_ms": pg["gemm_ms"], "split_ms": pg["split_ms"], "finish_ms": pg["finish_ms"],
                "note": "issued = 2 FP16 passes (hi, lo) x 2 x rows x cols x 256; useful = half of it"},
            "configs": configs,
            "clocks": clocks.summary(),
            "gpu_launches": launches,
            "greedy_device_matches_host": same_tokens,
            "wall_ms_timed_region": wall_ms,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(checkpoint, prompt)
        print(json.dumps(line))
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=496)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--checkpoint", default=os.path.join(tempfile.gettempdir(),
                                                         "lunelette_synth_seed0.safetensors"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 2-4 lines (batch context)")
    args = ap.parse_args()
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
