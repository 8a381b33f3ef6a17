"""Benchmark of the B200 Lunelette decoder backend (one JSON line on rank 0).

Workload ("C0"): the Ministral-3-3B-shaped decoder with a
seeded random-init checkpoint, batch 1, a 32-token prompt of ids ~ U[1000,
131072), then greedy decoding at context profile 256. One benchmark STEP is one
C0 generation's decode phase: starting from the prompt's checkpoint (a host-only
restore), 31 greedy decode tokens (the 32nd generated token comes from the
prompt's logits). `--steps K` times exactly K such passes. `value` = decode
tokens/s from CUDA events around lunelette_cuda_decode_loop (one launch of the
persistent decode kernel per pass, argmax fed back on the GPU), all ranks'
tokens over the slowest rank's device time. `e2e` = the same metric through
the drop-in C-ABI with host buffers (lunelette_metal_decode + host greedy each
token: H2D of the step parameters and D2H of the 131072 logits per token inside
the timed region). `roofline` is the persistent kernel's: the algorithmic
bytes of a launch (FP8 linears, BF16 head, norm gains and the FP32 KV rows
read) over its CUDA-event time; `traffic` scales the ncu DRAM bytes of one
token (profiles/decode_mega_c0_token.json) to a launch.

`--impl reference` times the CPU reference of the same path (the oracle's FP32
restatement of the reference's Metal kernels, all host threads) on the same
`config`: each step is a bounded sample of the pass (REF_TOKENS_PER_STEP greedy
tokens), and it never loads the product library (its checkpoint writer is
oracle/libsynth.so).

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
PER_PASS = 31            # greedy decode tokens in one C0 pass (one bench step)
REF_TOKENS_PER_STEP = 3  # CPU reference: greedy tokens sampled per step
WEIGHT_BYTES_PER_TOKEN = 3026190336 + 805306368 + 53 * 3072 * 4  # FP8 linears + BF16 head + norms
KV_BYTES_PER_POSITION = 26 * 2 * 1024 * 4                         # FP32 K and V, all layers
GATEUP_BYTES = 18432 * 3072                                       # one fused gate/up launch
HEAD_BYTES = 131072 * 3072 * 2
TRAFFIC_FILE = os.path.join(REPO, "profiles", "decode_mega_c0_token.json")

# The workload both arms report (identical dicts, so the two lines compare).
C0_CONFIG = {
    "workload": "C0: batch-1 greedy decode after a 32-token prompt, context profile 256",
    "prompt": PROMPT, "context": CONTEXT, "decode_tokens_per_step": PER_PASS,
    "step": "one C0 generation's decode phase: restore the prompt checkpoint, then 31 greedy tokens",
    "parallelism": "replicas (one weight replica and session per GPU)",
    "l2": "inputs larger than L2: every token streams 3.83 GB of weights",
}


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


def ensure_checkpoint(path, rank, barrier, writer):
    """The seeded synthetic checkpoint at `path`, written once by rank 0 with
    `writer(path, seed)` when absent (both arms' writers give identical bytes)."""
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".partial%d" % os.getpid()
        writer(tmp, 0)
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


def traffic_per_launch(tokens):
    """DRAM bytes (read + write) of a persistent-kernel launch of `tokens` tokens:
    the ncu capture of one single-token launch on the C0 workload, stored as data
    in profiles/decode_mega_c0_token.json, times the tokens of the launch (every
    token re-reads the weights); None when no capture is stored."""
    try:
        with open(TRAFFIC_FILE) as f:
            d = json.load(f)
        per_token = (int(d["dram_bytes_read"]) + int(d["dram_bytes_write"])) / int(d["tokens_per_launch"])
    except Exception:
        return None
    return per_token * tokens


def c0_bytes_per_token(context_before):
    """Algorithmic bytes of one decode token at `context_before` positions:
    weights, norms and the FP32 K/V rows of every position attended (the new one
    included)."""
    return WEIGHT_BYTES_PER_TOKEN + KV_BYTES_PER_POSITION * (context_before + 1)


def c1_gemv(peak):
    """every linear shape at token batch M = 1, 2, 4, 8 (the
    BF16 head at M = 1) through the kernels the runtime runs for that many
    tokens (the GEMV up to 4, the tcgen05 GEMM beyond), GB/s of algorithmic
    bytes and the fraction of the measured HBM peak, per shape and M."""
    from lunelette_b200 import microbench
    rows = microbench.run(list(microbench.SHAPES), [1, 2, 4, 8], iters=30)
    out = {}
    for r in rows:
        out.setdefault(r["shape"], {})["m%d" % r["m"]] = {"us": round(r["us"], 2), "gbs": round(r["gbs"], 1),
                                                          "frac": round(r["gbs"] / peak, 3)}
    return out


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


def config_lines(L, torch, checkpoint, seed, barrier, max_over_ranks, world, hbm):
    """BASELINE configs 2-4 on one batch context (64 sessions x 4352 positions,
    a paged FP32 KV pool of 59 GB): wall clock around host-synchronous calls,
    plus a device-timed C2 decode on a single-sequence context.
      C2: 4096 seeded ids in 16 chunks of 256 at context 4352, then 128 greedy
          decode steps (persistent kernel); `decode_device` repeats the decode
          with lunelette_cuda_decode_loop (CUDA events, one launch) and carries
          the roofline fraction of its algorithmic bytes;
      C3: a 512-token prefix, then 8 turns of 200 appended ids + 64 greedy tokens
          on the same session (its KV kept between turns); TTFT = the append;
      C4: 64 sessions, prompts ~ U[256, 4096] (seeded), prefilled in 256-token
          chunks, then 128 batched greedy decode steps over all 64 sessions; the
          step's roofline counts the weights once plus every session's FP32 K/V
          rows, over the wall-clock step time.
    Aggregates sum the ranks' work over the slowest rank's time."""
    rng = np.random.default_rng(seed + 99)
    out = {}
    ids_c2 = rng.integers(1000, 131072, 4096).astype(np.int64)
    with L.Batch(checkpoint, max_sessions=64, context=4352, pool_positions=64 * 4352, block=256) as b:
        # C2
        s = b.open()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for c in range(16):
            logits = b.append(s, ids_c2[256 * c:256 * (c + 1)])
        t_prefill = max_over_ranks(time.perf_counter() - t0)
        first_c2 = tok = int(np.argmax(logits))
        t0 = time.perf_counter()
        for _ in range(128):
            tok = int(np.argmax(b.append(s, [tok])))
        t_decode = max_over_ranks(time.perf_counter() - t0)
        b.close_session(s)
        out["c2"] = {"prefill_tok_s": world * 4096 / t_prefill, "decode_tok_s": world * 128 / t_decode,
                     "note": "4096-token prompt in 16 x 256 chunks at context 4352, then 128 greedy steps "
                             "(wall clock around lunelette_cuda_batch_append)"}
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
        step_s = t_decode / 128
        # mean positions attended per session over the 128 steps (the new one included)
        kv_positions = float(np.sum(lengths + 64.5))
        step_bytes = WEIGHT_BYTES_PER_TOKEN + KV_BYTES_PER_POSITION * kv_positions
        out["c4"] = {"decode_tok_s_aggregate": world * 64 * 128 / t_decode,
                     "prefill_tok_s_aggregate": world * float(lengths.sum()) / t_prefill,
                     "ms_per_batched_step": 1e3 * step_s, "sessions_per_gpu": 64,
                     "mean_prompt": float(lengths.mean()),
                     "roofline": {"bound": "hbm", "unit": "GB/s", "algorithmic_bytes_per_step": step_bytes,
                                  "achieved": step_bytes / step_s / 1e9, "peak": hbm,
                                  "frac": step_bytes / step_s / 1e9 / hbm,
                                  "timing": "wall clock per batched step (host-synchronous calls)"},
                     "note": "64 ragged sessions per GPU, prompts U[256,4096], 128 batched greedy steps"}
    # C2 decode on the device: the same prompt on a single-sequence context
    with L.Runtime(checkpoint, limits=(4352, 256)) as rt:
        rt.prefill(ids_c2[:256])
        for c in range(1, 16):
            rt.append(ids_c2[256 * c:256 * (c + 1)])
        cp = rt.checkpoint_create()
        rt.decode_loop(first_c2, 8)  # warm-up at this context
        rt.checkpoint_restore(cp)
        tokens, ms, launches = rt.decode_loop(first_c2, 128)
        cp.destroy()
    ms = max_over_ranks(ms)
    launch_bytes = sum(c0_bytes_per_token(4096 + i) for i in range(128))
    out["c2"]["decode_device"] = {
        "tok_s": world * 128 / (ms / 1e3), "ms_per_token": ms / 128, "launches": launches,
        "roofline": {"bound": "hbm", "unit": "GB/s", "algorithmic_bytes": launch_bytes,
                     "achieved": launch_bytes / (ms / 1e3) / 1e9, "peak": hbm,
                     "frac": launch_bytes / (ms / 1e3) / 1e9 / hbm,
                     "kernel": "decode_mega_kernel, 128 greedy tokens at context 4096..4223 in one launch"}}
    return out


def cpu_passes(oracle, checkpoint, prompt, steps, warmup, tokens_per_step):
    """The CPU reference of a C0 pass on this box's host cores: the oracle's FP32
    restatement of the reference kernels (OpenMP over all host threads). Each
    step continues the greedy generation from the prompt by `tokens_per_step`
    tokens, rewinding to the prompt after each pass of 31. Returns (seconds for
    the timed steps, prefill seconds of the prompt)."""
    m = oracle.open_model(checkpoint, CONTEXT)
    try:
        t0 = time.perf_counter()
        logits, _, _ = m.forward(prompt)
        prefill_s = time.perf_counter() - t0
        first = int(np.argmax(logits))
        state = {"tok": first, "done": 0}

        def step():
            for _ in range(tokens_per_step):
                if state["done"] == PER_PASS:
                    m.rewind(len(prompt))
                    state["tok"], state["done"] = first, 0
                out, _, _ = m.forward([state["tok"]])
                state["tok"] = int(np.argmax(out))
                state["done"] += 1

        for _ in range(warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        elapsed = time.perf_counter() - t0
    finally:
        m.close()
    return elapsed, prefill_s


def cpu_baseline(checkpoint, prompt, steps=2):
    """cpu_baseline of our arm's line: a bounded sample of the C0 pass on the
    host cores (rank 0 at N = 1)."""
    from tests import oracle_lib
    o = oracle_lib.load()
    elapsed, prefill_s = cpu_passes(o, checkpoint, prompt, steps, 1, REF_TOKENS_PER_STEP)
    n = steps * REF_TOKENS_PER_STEP
    return {"value": n / elapsed, "unit": "tok/s", "cores": o.threads(), "kind": "port",
            "sample": "%d greedy decode tokens of the C0 pass after the 32-token prompt (prefill %.2f s); "
                      "oracle/oracle.c FP32 restatement of the reference's Metal kernels, OpenMP"
                      % (n, prefill_s)}


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
    """The reference's CPU implementation of the path: this repository's oracle
    port of its Metal kernels (the Metal runtime cannot run off Apple hardware),
    on all host threads of rank 0. Loads only oracle/ libraries."""
    if rank != 0:
        return 0
    from tests import oracle_lib
    checkpoint = ensure_checkpoint(args.checkpoint, 0, lambda: None, oracle_lib.synth_checkpoint)
    o = oracle_lib.load()
    prompt = np.random.default_rng(args.seed).integers(1000, 131072, PROMPT).astype(np.int64)
    steps, warmup = args.steps, max(args.warmup, 3)
    elapsed, prefill_s = cpu_passes(o, checkpoint, prompt, steps, warmup, REF_TOKENS_PER_STEP)
    tokens = steps * REF_TOKENS_PER_STEP
    value = tokens / elapsed
    sample = ("each step: %d greedy decode tokens of the C0 pass (a bounded sample of the 31-token pass), "
              "continuing from the 32-token prompt; oracle/oracle.c FP32 restatement of the reference's "
              "Metal kernels, OpenMP; prompt prefill %.2f s untimed" % (REF_TOKENS_PER_STEP, prefill_s))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": 1000 * elapsed / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init checkpoint in the reference's tensor layout, seeded ids)",
            "config": dict(C0_CONFIG),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": o.threads(), "kind": "port",
                             "sample": sample},
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
    checkpoint = ensure_checkpoint(args.checkpoint, rank, barrier, L.synth_checkpoint)
    # checkpoint load: parse + FP8 admission of every payload byte + upload and
    # re-tiling (the file is in the page cache after its first read)
    t0 = time.perf_counter()
    rt = L.Runtime(checkpoint)  # default options, profile C=256/B=256
    load_s = time.perf_counter() - t0
    prompt = np.random.default_rng(args.seed + rank).integers(1000, 131072, PROMPT).astype(np.int64)
    steps, warmup = args.steps, max(args.warmup, 3)

    # ---- warm-up: untimed passes
    rt.reset()
    first = int(np.argmax(rt.prefill(prompt)))
    cp = rt.checkpoint_create()
    for _ in range(warmup):
        rt.decode_loop(first, PER_PASS)
        rt.checkpoint_restore(cp)

    # ---- value: K passes on the device (one persistent launch each), CUDA events
    barrier()
    torch.cuda.synchronize()
    device_ms = 0.0
    launches = 0
    tokens_seen = None
    with ClockSampler(local_rank) as clocks:
        t0 = time.perf_counter()
        for _ in range(steps):
            tokens, ms, n = rt.decode_loop(first, PER_PASS)
            device_ms += ms
            launches += n
            rt.checkpoint_restore(cp)
            tokens_seen = tokens
        torch.cuda.synchronize()
        wall_ms = 1000 * (time.perf_counter() - t0)
    barrier()
    device_ms = max_over_ranks(device_ms)
    value = aggregate_rate(world, steps * PER_PASS, device_ms / 1000)

    # ---- e2e: K passes through the drop-in C-ABI with host buffers, host greedy each token
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_tokens = []
    for _ in range(steps):
        logits = rt.checkpoint_restore(cp)
        tok = int(np.argmax(logits))
        e2e_tokens = []
        for i in range(PER_PASS):
            logits = rt.decode(tok)
            e2e_tokens.append(tok)
            tok = int(np.argmax(logits))
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = aggregate_rate(world, steps * PER_PASS, e2e_s)
    # the device loop and the host loop must generate the same greedy tokens
    same_tokens = list(e2e_tokens[1:]) == [int(t) for t in tokens_seen[:PER_PASS - 1]]

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

    hbm, bf16, peak_kind = measured_peaks()
    configs = None if args.no_configs else config_lines(L, torch, checkpoint, args.seed + rank, barrier,
                                                         max_over_ranks, world, hbm)
    gemv = c1_gemv(hbm) if not args.no_configs else None
    gemv_ms, gemv_bytes = gateup_roofline(lib, torch, checkpoint)
    pg = prefill_gemm_roofline(lib, torch)
    ms_per_step = device_ms / steps
    launch_bytes = sum(c0_bytes_per_token(PROMPT + i) for i in range(PER_PASS))
    launch_ms = device_ms / launches            # one persistent-kernel launch per pass
    achieved = launch_bytes / (launch_ms / 1000) / 1e9

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 weights, fp32 activations/accumulation/kv",
            "data": "synthetic (seeded random-init checkpoint in the reference's tensor layout, seeded ids)",
            "config": dict(C0_CONFIG),
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 1040 * PER_PASS,
                    "d2h_bytes_per_step": (131072 * 4 + 4) * PER_PASS,
                    "note": "lunelette_metal_decode per token, host greedy on the borrowed logits; bytes per "
                            "31-token step"},
            "prefill_tok_s": {"chunk_256": 256 / prefill_256, "prompt_32": PROMPT / prefill_32,
                              "note": "lunelette_metal_prefill wall time, host ids and logits"},
            "load": {"seconds": load_s, "file_bytes": os.path.getsize(checkpoint),
                     "gbs": os.path.getsize(checkpoint) / load_s / 1e9,
                     "note": "lunelette_metal_create: header parse, FP8 admission of every code, parallel reads "
                             "into pinned staging, upload and re-tiling"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic_per_launch(PER_PASS), "peak_kind": peak_kind,
                         "kernel": "decode_mega_kernel (persistent: %d greedy tokens per launch)" % PER_PASS,
                         "algorithmic_bytes": launch_bytes, "avg_launch_ms": launch_ms,
                         "bytes_per_token": launch_bytes / PER_PASS,
                         "traffic_source": "ncu DRAM read+write of one token (profiles/decode_mega_c0_token.json)"
                                           " x the launch's tokens"},
            "c1_gemv": gemv,
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
    ap.add_argument("--steps", type=int, default=20, help="C0 passes of 31 greedy tokens to time")
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
