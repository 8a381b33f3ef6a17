"""Decode GEMV microbenchmark on the current GPU, and the
prefill GEMM microbenchmark (--prefill-gemm).

Shapes: the model's FP8 linears q 3072->4096, k/v 3072->1024, o 4096->3072,
gate/up 3072->9216, down 9216->3072, and the BF16 lm_head 3072->131072, at token
batch M = 1, 2, 4, 8. Weights are random E4M3 codes, read as the tiled layout
the runtime stores (any random bytes are a valid tiled matrix of the same
size); several copies rotate so that the working set exceeds L2; activations
N(0,1). Time per launch from CUDA
events on the launching stream; GB/s counts weight bytes + activations in and
outputs once per launch (the algorithmic bytes), against the measured HBM peak.
M <= 4 runs the GEMV kernel; M = 8 runs the path the runtime takes for blocks
of more than four tokens: the activation split, the tcgen05 GEMM with the
weights as tensor-memory A and the ordered K-range finish (the sum of the three
kernels' device times, lunelette_cuda_gemm_fp8_timed).

    python -m lunelette_b200.microbench [--shapes q,gate,...] [--m 1,2,4,8] [--iters N]
    python -m lunelette_b200.microbench --accumulation-probe   # tensor-core accumulation rounding
"""
import argparse
import json
import os

import numpy as np

SHAPES = {
    "q": (4096, 3072), "k": (1024, 3072), "v": (1024, 3072), "o": (3072, 4096),
    "gate": (9216, 3072), "up": (9216, 3072), "down": (3072, 9216), "lm_head": (131072, 3072),
}
L2_BYTES = 126 << 20


def hbm_peak():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def run(shapes, ms_list, iters, warmup=3):
    import torch
    import lunelette_b200 as L
    lib = L.library()
    stream = torch.cuda.current_stream()
    peak, kind = hbm_peak()
    rows_out = []
    gen = torch.Generator(device="cuda").manual_seed(0)
    for name in shapes:
        rows, cols = SHAPES[name]
        bf16 = name == "lm_head"
        wbytes = rows * cols * (2 if bf16 else 1)
        copies = max(1, min(128, (2 * L2_BYTES) // wbytes + 1))  # rotated copies > 2x L2
        ws = []
        for _ in range(copies):
            if bf16:
                w = (torch.randn(rows, cols, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
            else:
                w = torch.randint(0, 256, (rows, cols), device="cuda", dtype=torch.uint8, generator=gen)
                w[(w & 127) == 127] = 0
            ws.append(w)
        gain = torch.ones(cols, device="cuda")
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        for m in ms_list:
            if bf16 and m != 1:
                continue
            x = torch.randn(m, cols, device="cuda", generator=gen)
            y = torch.empty(m, rows, device="cuda")
            if m > GEMV_MAX_TOKENS and not bf16:
                rows_out.append(gemm_row(lib, torch, name, rows, cols, m, copies, x, y, iters, peak, kind, gen))
                continue

            def launch(i):
                w = ws[i % copies]
                if bf16:
                    rc = lib.lunelette_cuda_head_bf16(w.data_ptr(), rows, cols, x.data_ptr(), gain.data_ptr(),
                                                      y.data_ptr(), flag.data_ptr(), stream.cuda_stream)
                else:
                    rc = lib.lunelette_cuda_gemv_fp8(w.data_ptr(), rows, cols, 1e-3, x.data_ptr(), None, m,
                                                     y.data_ptr(), stream.cuda_stream)
                assert rc == 0

            for i in range(warmup):
                launch(i)
            torch.cuda.synchronize()
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for i in range(iters):
                launch(i)
            stop.record(stream)
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / iters
            nbytes = wbytes + m * cols * 4 + m * rows * 4
            gbs = nbytes / (ms / 1000) / 1e9
            rows_out.append({"shape": name, "rows": rows, "cols": cols, "m": m, "us": ms * 1000,
                             "algorithmic_bytes": nbytes, "gbs": gbs, "frac_hbm": gbs / peak,
                             "peak_gbs": peak, "peak_kind": kind})
    return rows_out


GEMV_MAX_TOKENS = 4  # blocks of more tokens run the tcgen05 GEMM (kGemvMaxTokens in csrc/kernels.h)


def gemm_row(lib, torch, name, rows, cols, m, copies, x, y, iters, peak, kind, gen):
    """One C1 row on the tcgen05 path: split + GEMM + finish device time."""
    import ctypes
    w = torch.randint(0, 256, (copies * rows * cols,), device="cuda", dtype=torch.uint8, generator=gen)
    w[(w & 127) == 127] = 0
    ms = (ctypes.c_float * 3)()
    stream = torch.cuda.current_stream().cuda_stream
    for reps in (copies, iters):
        assert lib.lunelette_cuda_gemm_fp8_timed(w.data_ptr(), copies, rows, cols, 1e-3, x.data_ptr(), m,
                                                 y.data_ptr(), reps, ms, stream) == 0
    ms_total = ms[0] + ms[1] + ms[2]
    nbytes = rows * cols + m * cols * 4 + m * rows * 4
    gbs = nbytes / (ms_total / 1000) / 1e9
    return {"shape": name, "rows": rows, "cols": cols, "m": m, "us": ms_total * 1000, "algorithmic_bytes": nbytes,
            "gbs": gbs, "frac_hbm": gbs / peak, "peak_gbs": peak, "peak_kind": kind,
            "path": "split %.2f + tcgen05 GEMM %.2f + finish %.2f us" % (ms[0] * 1e3, ms[1] * 1e3, ms[2] * 1e3)}


PHASE_BYTES = {"attn_o": (6144 + 4096) * 3072, "ffn": 18432 * 3072 + 3072 * 9216, "head": 131072 * 3072 * 2}


def decode_phases(checkpoint, steps=8, prompt=32):
    """Phase durations of the persistent decode kernel (single-token steps through
    lunelette_metal_decode), from its %globaltimer timeline, as means over `steps`
    steps and 26 layers. Barrier phases, from CTA 0 leaving one barrier to
    leaving the next: `attn_o` (qkv, attention, o), `ffn` (gate/up, SwiGLU and
    down of every act slice), `head` (head GEMV and greedy pick); with
    `<phase>_spread`, first to last CTA arriving, and `<phase>_release`, last
    arrival to CTA 0 leaving. Milestones within a layer, measured from the
    barrier that opened the phase to the last CTA reaching them (`@max`) and to
    the median CTA (`@med`): row staged, items done, q/k/v published, attention
    published, act slice stored."""
    import torch
    import lunelette_b200 as L
    peak, kind = hbm_peak()
    ctas = torch.cuda.get_device_properties(0).multi_processor_count
    barriers, per_layer = 53, 13
    marks = 26 * per_layer + 1
    milestones = {0: "qkv_staged", 1: "qkv_items", 2: "qkv_published", 3: "attention", 4: "o_staged",
                  5: "o_items", 7: "gate_up_staged", 8: "gate_up_items", 9: "act_stored", 11: "down_items"}
    closing = {6: "attn_o", 12: "ffn"}
    rows = {}

    def add(name, v):
        rows.setdefault(name, []).append(v)

    # prompts beyond 248 ids run on the (4352, 256) profile, prefilled in 256-id chunks
    with L.Runtime(checkpoint, limits=(4352, 256) if prompt > 248 else None) as rt:
        ids = np.random.default_rng(7).integers(1000, 131072, prompt)
        logits = rt.prefill(ids[:256])
        for c in range(256, prompt, 256):
            logits = rt.append(ids[c:c + 256])
        tok = int(np.argmax(logits))
        rt.timeline(True)
        for _ in range(steps):
            tok = int(np.argmax(rt.decode(tok)))
            full = rt.timeline_copy(1 + barriers + marks * ctas).astype(np.float64) / 1000.0  # us
            start, exits = full[0], full[1:1 + barriers]
            mark = full[1 + barriers:].reshape(marks, ctas)
            opened = start
            for layer in range(26):
                base = layer * per_layer
                for k in range(per_layer):
                    arr = mark[base + k]
                    if k in milestones:
                        arr = arr[arr > 0]
                        add(milestones[k] + "@max", arr.max() - opened)
                        add(milestones[k] + "@med", float(np.median(arr)) - opened)
                    elif k in closing:
                        b = 2 * layer + (k == 12)
                        name = closing[k]
                        add(name, exits[b] - opened)
                        add(name + "_spread", arr.max() - arr.min())
                        add(name + "_release", exits[b] - arr.max())
                        opened = exits[b]
            arr = mark[marks - 1]
            add("head", exits[barriers - 1] - opened)
            add("head_spread", arr.max() - arr.min())
            add("head_release", exits[barriers - 1] - arr.max())
            add("step", exits[barriers - 1] - start)
        rt.timeline(False)
    out = []
    for name, vals in rows.items():
        us = float(np.mean(vals))
        nbytes = PHASE_BYTES.get(name, 0)
        rec = {"phase": name, "mean_us": us, "min_us": float(np.min(vals)), "max_us": float(np.max(vals))}
        if nbytes:
            rec["weight_bytes"] = nbytes
            rec["gbs"] = nbytes / (us * 1e-6) / 1e9
            rec["frac_hbm"] = rec["gbs"] / peak
        out.append(rec)
    return out


PREFILL_SHAPES = {"qkv": (6144, 3072), "o": (3072, 4096), "gateup": (18432, 3072), "down": (3072, 9216)}


def tensor_peak():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def prefill_gemm(counts, iters):
    """The tcgen05 prefill projections at the model's four shapes: mean device
    time of the split, GEMM and finish kernels (CUDA events), weights rotated
    over copies larger than 2x L2. `issued` TFLOP/s counts what the tensor core
    executes (hi and lo passes over 128-token tiles and 256-row tiles),
    `useful` the projection's own 2 * rows * cols * count."""
    import ctypes
    import torch
    import lunelette_b200 as L
    lib = L.library()
    stream = torch.cuda.current_stream().cuda_stream
    peak, kind = tensor_peak()
    gen = torch.Generator(device="cuda").manual_seed(0)
    out = []
    for name, (rows, cols) in PREFILL_SHAPES.items():
        copies = max(1, min(8, (2 * L2_BYTES) // (rows * cols) + 1))
        w = torch.randint(0, 256, (copies * rows * cols,), device="cuda", dtype=torch.uint8, generator=gen)
        w[(w & 127) == 127] = 0
        for count in counts:
            x = torch.randn(count, cols, device="cuda", generator=gen)
            y = torch.empty(count, rows, device="cuda")
            ms = (ctypes.c_float * 3)()
            # one warm-up pass, then the timed back-to-back runs
            for reps in (copies, iters):
                rc = lib.lunelette_cuda_gemm_fp8_timed(w.data_ptr(), copies, rows, cols, 1.0, x.data_ptr(), count,
                                                       y.data_ptr(), reps, ms, stream)
                assert rc == 0, (name, count)
            tot = [ms[0], ms[1], ms[2]]
            tt = (count + 127) // 128
            # a CTA pair covers 256 tokens (two 128-token tiles) x 512 rows
            issued = 2 * 2 * ((rows + 511) // 512 * 512) * ((cols + 63) // 64 * 64) * 256 * ((tt + 1) // 2)
            useful = 2 * rows * cols * count
            out.append({
                "projection": name, "rows": rows, "cols": cols, "count": count,
                "split_us": tot[0] * 1e3, "gemm_us": tot[1] * 1e3, "finish_us": tot[2] * 1e3,
                "gemm_issued_tflops": issued / (tot[1] * 1e-3) / 1e12,
                "gemm_useful_tflops": useful / (tot[1] * 1e-3) / 1e12,
                "tensor_frac_issued": issued / (tot[1] * 1e-3) / 1e12 / peak,
                "tensor_frac_useful": 2 * useful / (tot[1] * 1e-3) / 1e12 / peak, "peak_tflops": peak,
                "peak_kind": kind,
                "weight_gbs": rows * cols / (tot[1] * 1e-3) / 1e9,
            })
    return out


def prefill_tokens(checkpoint, count):
    """A profiling target: prefill `count` seeded ids once (warm-up), then again
    between cudaProfilerStart and cudaProfilerStop (ncu --profile-from-start off).
    Prompts longer than 256 ids go in 256-id chunks (prefill, then appends) at a
    context of the prompt plus one chunk, as in config 2."""
    import torch
    import lunelette_b200 as L
    if not os.path.exists(checkpoint):
        L.synth_checkpoint(checkpoint, 0)
    context = 256 if count <= 256 else (count + 63) // 64 * 64 + 256
    with L.Runtime(checkpoint, limits=(context, 256)) as rt:
        ids = np.random.default_rng(3).integers(1000, 131072, count).astype(np.int64)

        def run():
            rt.reset()
            logits = rt.prefill(ids[:256])
            for c in range(256, count, 256):
                logits = rt.append(ids[c:c + 256])
            return logits

        run()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        tok = int(np.argmax(run()))
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    return tok


def attention_block(length, count, reps=20):
    """Blocks of `count` query rows at positions length..length+count-1 (the
    prefill/append attention) through lunelette_cuda_attention on a random
    paged pool: mean device time (CUDA events) of `reps` back-to-back calls after
    one untimed call (an ncu target with -s 1 -c 1). FLOPs: QK and PV per query
    row and causally visible key (`useful`), times 3 for the hi/lo terms the
    tensor cores execute (`issued`)."""
    import torch
    import lunelette_b200 as L
    lib = L.library()
    total = length + count
    num_pages = (total + 63) // 64
    gen = torch.Generator(device="cuda").manual_seed(0)
    pool = torch.randn(num_pages * 2 * 8 * 64 * 128, device="cuda", generator=gen)
    table = torch.arange(num_pages, dtype=torch.int32, device="cuda")
    q = torch.randn(count, 4096, device="cuda", generator=gen)
    out = torch.empty(count, 4096, device="cuda")
    slots = 65536
    acc = torch.empty(slots * 128, device="cuda")
    ml = torch.empty(slots * 2, device="cuda")
    stream = torch.cuda.current_stream()

    def call():
        assert lib.lunelette_cuda_attention(q.data_ptr(), pool.data_ptr(), table.data_ptr(), num_pages, 0, length,
                                            count, out.data_ptr(), acc.data_ptr(), ml.data_ptr(), slots,
                                            stream.cuda_stream) == 0

    call()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        call()
    stop.record(stream)
    torch.cuda.synchronize()
    us = start.elapsed_time(stop) * 1000 / reps
    keys = sum(length + t + 1 for t in range(count))
    useful = 2 * 2 * 32 * 128 * keys
    peak, kind = tensor_peak()
    return {"length": length, "count": count, "us": us, "useful_tflops": useful / us / 1e6,
            "issued_tflops": 3 * useful / us / 1e6, "frac_issued": 3 * useful / us / 1e6 / peak,
            "peak_tflops": peak, "peak_kind": kind}


def batch_step(checkpoint, sessions=64, seed=5, pool=None):
    """A profiling target for config 4: `sessions` sessions with prompts ~
    U[256, 4096] (seeded) prefilled, one warm-up batched decode step, then one
    step between cudaProfilerStart and cudaProfilerStop."""
    import torch
    import lunelette_b200 as L
    if not os.path.exists(checkpoint):
        L.synth_checkpoint(checkpoint, 0)
    rng = np.random.default_rng(seed)
    pool = pool if pool is not None else sessions * 4352
    with L.Batch(checkpoint, max_sessions=sessions, context=4352, pool_positions=pool, block=256) as b:
        ss = [b.open() for _ in range(sessions)]
        toks = []
        for s in ss:
            ids = rng.integers(1000, 131072, int(rng.integers(256, 4097))).astype(np.int64)
            for c0 in range(0, ids.size, 256):
                logits = b.append(s, ids[c0:c0 + 256])
            toks.append(int(np.argmax(logits)))
        toks = b.decode(ss, toks).tolist()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        toks = b.decode(ss, toks).tolist()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    return toks[0]


def e4m3_values():
    """The 256 E4M3FN codes as float64 (sign, 4 exponent bits with bias 7, 3
    mantissa bits; exponent 0 subnormal; S.1111.111 NaN)."""
    v = np.empty(256)
    for c in range(256):
        sign, e, m = (-1.0 if c & 0x80 else 1.0), (c >> 3) & 15, c & 7
        if e == 15 and m == 7:
            v[c] = np.nan
        elif e == 0:
            v[c] = sign * m / 8 * 2.0 ** -6
        else:
            v[c] = sign * (1 + m / 8) * 2.0 ** (e - 7)
    return v


def accumulation_probe(rows=18432, cols=9216, seed=3):
    """How the tensor cores round the FP32 accumulation, measured through the
    FP8 projection entry points on operands whose every product is exact:
    positive codes 0x30..0x4F (0.5 .. 7.5), scale 1, activations k / 1024 with
    k in [1024, 2048) (exact FP16 after the kernels' power-of-two row scale, so
    the lo part is zero). The float64 dot product is then exact, and each
    output's signed error in units of its FP32 ulp shows the rounding:
    truncation toward zero leaves every error <= 0 and a mean of minus about
    half an ulp per accumulation step; round to nearest, errors of both signs
    around zero. Shapes: the small-block tcgen05 GEMM (16 tokens: one K range
    per CTA, 144 chunks of 64 over two alternating accumulators), the CTA-pair
    GEMM (128 tokens: two K ranges added in FP32 by the finish kernel) and the
    mma.sync GEMV (4 tokens)."""
    import torch
    import lunelette_b200 as L
    lib = L.library()
    rng = np.random.default_rng(seed)
    codes = rng.integers(0x30, 0x50, (rows, cols)).astype(np.uint8)
    w = e4m3_values()[codes]
    stream = torch.cuda.current_stream().cuda_stream
    raw = torch.from_numpy(codes).cuda()
    tiled = torch.zeros(-(-rows // 8) * 8 * (-(-cols // 128) * 128), dtype=torch.uint8, device="cuda")
    assert lib.lunelette_cuda_tile_fp8(raw.data_ptr(), rows, cols, 0, tiled.data_ptr(), stream) == 0
    out = {}
    for name, entry, count in (("tcgen05 small-block GEMM", "lunelette_cuda_gemm_fp8", 16),
                               ("tcgen05 CTA-pair GEMM", "lunelette_cuda_gemm_fp8", 128),
                               ("mma.sync GEMV", "lunelette_cuda_gemv_fp8", 4)):
        x = (rng.integers(1024, 2048, (count, cols)) / 1024.0).astype(np.float32)
        d_x = torch.from_numpy(x).cuda()
        y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
        assert getattr(lib, entry)(tiled.data_ptr(), rows, cols, 1.0, d_x.data_ptr(), None, count, y.data_ptr(),
                                   stream) == 0
        torch.cuda.synchronize()
        exact = x.astype(np.float64) @ w.T
        got = y.cpu().numpy().astype(np.float64)
        ulp = np.spacing(exact.astype(np.float32)).astype(np.float64)
        err = (got - exact) / ulp
        out[name] = {"tokens": count, "outputs": int(err.size), "mean_ulp": float(err.mean()),
                     "min_ulp": float(err.min()), "max_ulp": float(err.max()),
                     "below": float((err < 0).mean()), "above": float((err > 0).mean())}
    return out


def batch_head_ab(checkpoint, sessions=64, steps=20, seed=9):
    """Batched decode steps of `sessions` sessions with 8-token prompts (short
    contexts: the step is the projections and the head) with the mma.sync head
    and with the tcgen05 head (LUNELETTE_HEAD_TC, read when the context is
    created); wall-clock ms per step after three warm-up steps."""
    import time
    import lunelette_b200 as L
    if not os.path.exists(checkpoint):
        L.synth_checkpoint(checkpoint, 0)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(1000, 131072, 8) for _ in range(sessions)]
    out = {}
    for name, head in (("mma_ms", "0"), ("tc_ms", "1")):
        os.environ["LUNELETTE_HEAD_TC"] = head
        with L.Batch(checkpoint, max_sessions=sessions, context=4352, pool_positions=sessions * 128,
                     block=256) as b:
            ss = [b.open() for _ in range(sessions)]
            toks = [int(np.argmax(b.append(s, p))) for s, p in zip(ss, prompts)]
            for _ in range(3):
                toks = b.decode(ss, toks).tolist()
            t0 = time.perf_counter()
            for _ in range(steps):
                toks = b.decode(ss, toks).tolist()
            out[name] = (time.perf_counter() - t0) / steps * 1e3
    os.environ.pop("LUNELETTE_HEAD_TC", None)
    return out


def decode_tokens(checkpoint, steps, prompt=32):
    """A small profiling target: the C0 prompt, then `steps` greedy tokens through
    lunelette_metal_decode (one persistent-kernel launch each)."""
    import lunelette_b200 as L
    with L.Runtime(checkpoint) as rt:
        ids = np.random.default_rng(7).integers(1000, 131072, prompt)
        tok = int(np.argmax(rt.prefill(ids)))
        for _ in range(steps):
            tok = int(np.argmax(rt.decode(tok)))
    return tok


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--m", default="1,2,4,8")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--decode-tokens", nargs=2, metavar=("CHECKPOINT", "N"), default=None,
                    help="run the C0 prompt and N single-token decode launches (a profiling target)")
    ap.add_argument("--decode-phases", metavar="CHECKPOINT", default=None,
                    help="time the persistent decode kernel's phases on this checkpoint instead")
    ap.add_argument("--phases-prompt", type=int, default=32,
                    help="prompt length before the timed decode steps of --decode-phases (4096: config 2)")
    ap.add_argument("--prefill-tokens", nargs=2, metavar=("CHECKPOINT", "N"), default=None,
                    help="prefill N ids twice, the second between cudaProfilerStart/Stop (a profiling target)")
    ap.add_argument("--attention", metavar="LENGTH,COUNT", default=None,
                    help="time the block attention (tcgen05 kernel) of COUNT queries at LENGTH positions")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--batch-step", metavar="CHECKPOINT", default=None,
                    help="one batched decode step of ragged sessions between cudaProfilerStart/Stop")
    ap.add_argument("--batch-sessions", type=int, default=64)
    ap.add_argument("--accumulation-probe", action="store_true",
                    help="signed errors of the FP8 projections on exact-product operands (accumulation rounding)")
    ap.add_argument("--batch-head", metavar="CHECKPOINT", default=None,
                    help="batched step with the mma.sync and the tcgen05 head, ms per step")
    ap.add_argument("--prefill-gemm", metavar="COUNTS", default=None,
                    help="time the tcgen05 prefill projections at these token counts (e.g. 256,32)")
    args = ap.parse_args()
    if args.accumulation_probe:
        print(json.dumps(accumulation_probe()))
        return
    if args.batch_head:
        print(json.dumps(batch_head_ab(args.batch_head, args.batch_sessions)))
        return
    if args.batch_step:
        n = args.batch_sessions
        # the pool holds the sessions' prompts plus the two steps (pages of 64)
        print(json.dumps({"first_token": batch_step(args.batch_step, n, pool=None if n >= 64 else n * 4160)}))
        return
    if args.attention:
        length, count = (int(v) for v in args.attention.split(","))
        print(json.dumps(attention_block(length, count, args.reps)))
        return
    if args.prefill_tokens:
        print(json.dumps({"first_token": prefill_tokens(args.prefill_tokens[0], int(args.prefill_tokens[1]))}))
        return
    if args.prefill_gemm:
        for r in prefill_gemm([int(v) for v in args.prefill_gemm.split(",")], args.iters):
            print(json.dumps(r))
        return
    if args.decode_tokens:
        print(json.dumps({"last_token": decode_tokens(args.decode_tokens[0], int(args.decode_tokens[1]))}))
        return
    if args.decode_phases:
        for r in decode_phases(args.decode_phases, prompt=args.phases_prompt):
            print(json.dumps(r))
        return
    out = run(args.shapes.split(","), [int(v) for v in args.m.split(",")], args.iters, args.warmup)
    for r in out:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
