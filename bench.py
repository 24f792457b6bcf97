#!/usr/bin/env python
"""Benchmark of the Gemma-3-1B Q4_0 forward pass (BASELINE.json's metric).

A step is one greedy decode token of BASELINE config 1's model (26 layers,
Q4_0, seed-0 random init, batch 1 per GPU after a 32-token prefill), through
the C ABI.  `value` is decode tokens/s over all ranks with the inputs resident
(steps enqueued back to back); `e2e` is the same through the public step API
with each step's 16-byte record read back to the host before the next;
`prefill_tokens_per_s` times the 32-token prefill; `roofline` times the
dominant kernel, the 262144 x 1152 Q4_0 head matvec, alone.

N > 1 (torchrun): independent sequences, one per GPU (a 1B model has no
tensor-parallel split), with a final NCCL gather of each rank's last logits;
weak scaling.  `--impl reference` times the CPU restatement of the
reference's arithmetic (the WGSL path needs a WebGPU device, unavailable here).
"""
import argparse
import ctypes as C
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Gemma-3-1B q4_0 decode tok/s, prefill tok/s; q4 matvec HBM GB/s vs peak"
PROMPT = 32
HEAD_N, HEAD_K = 262144, 1152
LAUNCHES_PER_DECODE_STEP = 5   # embed, the persistent decode step (26 layers), head, select x2
DECODE_BYTES = 562_360_320 + 537_088           # Q4_0 weights + F32 gains a decode token reads
LAYER_BYTES = 392_491_008 + 532_480            # the 26 layers' Q4_0 weights + their norm gains (no head)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, ordinal):
        self.ordinal = ordinal
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.ordinal), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx.append(float(f[2]))
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU legs

def host_threads():
    """The host cores this process may run on (not OMP_NUM_THREADS, which a
    launcher such as torchrun sets to 1)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_decode_sample(path, decode_tokens=2, prefill=4, warmup=0):
    """The oracle's decode tokens/s on this host's cores (all of them): a
    `prefill`-token prompt, `warmup` untimed decode steps, then
    `decode_tokens` timed decode steps of the full model."""
    import numpy as np
    import oracle
    from frizzle_b200 import synth
    oracle.lib().oracle_set_threads(host_threads())
    orc = oracle.OracleModel(path, context=max(256, prefill + warmup + decode_tokens + 1))
    ids = np.random.default_rng(0).integers(2, synth.GEMMA3_1B.vocab, size=prefill).astype(np.uint32)
    logits, _ = orc.step(0, ids, logits=True)
    pos = prefill
    for _ in range(warmup):
        tok = int(np.argmax(logits))
        logits, _ = orc.step(pos, [tok], logits=True)
        pos += 1
    t0 = time.perf_counter()
    for i in range(decode_tokens):
        tok = int(np.argmax(logits))
        logits, _ = orc.step(pos + i, [tok], logits=True)
    dt = time.perf_counter() - t0
    threads = oracle.lib().oracle_threads()
    orc.close()
    return decode_tokens / dt, threads, f"{decode_tokens} timed greedy decode tokens of the 26-layer model after a " \
                                        f"{prefill}-token prompt and {warmup} untimed ones, oracle port on " \
                                        f"{threads} host threads"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from frizzle_b200 import synth
    path = synth.model_path(synth.GEMMA3_1B, 0)
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    # Config 1's 32-token prompt, the warm-up decode tokens untimed, then every
    # claimed step timed (about 50 ms a token on 16 host threads).
    value, threads, sample = cpu_decode_sample(path, decode_tokens=steps, prefill=PROMPT, warmup=warmup)
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init Q4_0 weights, seeded ids)",
            "config": config(args.gpus), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's WGSL forward pass needs a WebGPU device (Dawn), unavailable on this box; "
                    "this is the oracle's C restatement of its arithmetic"}
    print(json.dumps(line))
    return 0


def config(n):
    return {"workload": "BASELINE config 1: Gemma-3-1B-shaped Q4_0 model (26 layers, hidden 1152, vocab 262144, "
                        "seed 0), batch-1 greedy decode after a 32-token prefill, one sequence per GPU; every timed "
                        "pass (device-timed, end to end, the decode kernel's) decodes positions 32 .. 32 + steps - 1, "
                        "the cache cut back to the prompt between passes",
            "batch_per_gpu": 1, "prompt_tokens": PROMPT,
            "l2": "inputs larger than L2: each decode step streams 562.9 MB of weights (L2 is 126 MB)",
            "parallelism": f"independent sequences x{n}, final NCCL gather of logits" if n > 1 else "single GPU"}


# ------------------------------------------------------------------ GPU leg

def head_roofline(torch, lib, native, reps=20):
    """The dominant kernel (262144 x 1152 Q4_0 head, M = 1) timed alone with CUDA
    events on its stream; two weight copies alternate so L2 holds neither."""
    import numpy as np
    n, k = HEAD_N, HEAD_K
    rng = np.random.default_rng(1)
    mats = []
    for c in range(2):
        blocks = np.empty((n * k // 32, 18), dtype=np.uint8)
        d = np.abs(rng.standard_normal(n * k // 32).astype(np.float32) * np.float32(0.005)).astype(np.float16)
        blocks[:, :2] = d.view(np.uint8).reshape(-1, 2)
        blocks[:, 2:] = rng.integers(0, 256, size=(n * k // 32, 16), dtype=np.uint8)
        src = torch.from_numpy(blocks.reshape(-1)).cuda()
        codes = torch.empty(lib.fz_q4_0_codes_bytes(n, k), dtype=torch.uint8, device="cuda")
        scales = torch.empty(lib.fz_q4_0_scales_bytes(n, k), dtype=torch.uint8, device="cuda")
        native.check(lib.fz_q4_0_repack(src.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream))
        del src
        mats.append((codes, scales))
    x = torch.randn(1, k, device="cuda")
    logits = torch.empty(1, n, device="cuda")
    am = torch.zeros(1, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for i in range(4):
        c, sc = mats[i % 2]
        native.check(lib.fz_q4_0_head(c.data_ptr(), sc.data_ptr(), n, k, x.data_ptr(), 1, logits.data_ptr(),
                                      am.data_ptr(), s))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(reps):
        c, sc = mats[i % 2]
        native.check(lib.fz_q4_0_head(c.data_ptr(), sc.data_ptr(), n, k, x.data_ptr(), 1, logits.data_ptr(),
                                      am.data_ptr(), s))
    end.record()
    torch.cuda.synchronize()
    secs = start.elapsed_time(end) / 1000.0 / reps
    bytes_ = n * k * 9 // 16 + 4 * k + 4 * n
    del mats
    torch.cuda.empty_cache()
    return bytes_, secs


def formats_roofline(torch, lib, native, reps=20):
    """The pinned file's other block formats at the head's shape (262144 x 1152,
    M = 1): Q8_0 (its tied embedding/head) and Q4_1, each timed alone with CUDA
    events on its stream, two weight copies alternating so L2 holds neither.
    Algorithmic bytes: codes + scales + x + y."""
    from frizzle_b200 import synth
    n, k = HEAD_N, HEAD_K
    s = torch.cuda.current_stream().cuda_stream
    x = torch.randn(1, k, device="cuda")
    y = torch.empty(1, n, device="cuda")
    out = {}
    for name, gen, cb, sb, repack, matvec in (
            ("q8_0", synth.random_q8_0, lib.fz_q8_0_codes_bytes, lib.fz_q8_0_scales_bytes, lib.fz_q8_0_repack,
             lib.fz_q8_0_matvec),
            ("q4_1", synth.random_q4_1, lib.fz_q4_1_codes_bytes, lib.fz_q4_1_scales_bytes, lib.fz_q4_1_repack,
             lib.fz_q4_1_matvec)):
        mats = []
        for c in range(2):
            src = torch.from_numpy(gen(n, k, seed=c)).cuda()
            codes = torch.empty(cb(n, k), dtype=torch.uint8, device="cuda")
            scales = torch.empty(sb(n, k), dtype=torch.uint8, device="cuda")
            native.check(repack(src.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(), s))
            torch.cuda.synchronize()
            del src
            mats.append((codes, scales))
        for i in range(4):
            c, sc = mats[i % 2]
            native.check(matvec(c.data_ptr(), sc.data_ptr(), n, k, x.data_ptr(), 1, y.data_ptr(), s))
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(reps):
            c, sc = mats[i % 2]
            native.check(matvec(c.data_ptr(), sc.data_ptr(), n, k, x.data_ptr(), 1, y.data_ptr(), s))
        end.record()
        torch.cuda.synchronize()
        secs = start.elapsed_time(end) / 1000.0 / reps
        bytes_ = cb(n, k) + sb(n, k) + 4 * k + 4 * n
        hbm, _, which = peaks()
        out[name] = {"kernel": f"{name} matvec 262144 x 1152, M=1", "us": secs * 1e6, "algorithmic_bytes": bytes_,
                     "achieved_gbs": bytes_ / secs / 1e9, "frac": bytes_ / secs / 1e9 / hbm, "peak": hbm,
                     "peak_source": which}
        del mats
        torch.cuda.empty_cache()
    return out


def gemm_roofline(torch, lib, native, m=4096, reps=10):
    """The prefill's dominant product (gate and up, 1152 -> 2 x 6912, GELU and
    the f16 hand-off) on the tensor cores at m rows, timed alone."""
    import numpy as np
    from frizzle_b200 import synth
    f, k = 6912, 1152
    mats = []
    for seed in (1, 2):
        blocks = synth.random_q4_0(f, k, seed=seed)
        src = torch.from_numpy(blocks).cuda()
        codes = torch.empty(lib.fz_q4_0_codes_bytes(f, k), dtype=torch.uint8, device="cuda")
        scales = torch.empty(lib.fz_q4_0_scales_bytes(f, k), dtype=torch.uint8, device="cuda")
        native.check(lib.fz_q4_0_repack(src.data_ptr(), f, k, codes.data_ptr(), scales.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream))
        mats.append((codes, scales))
    x = torch.randn(m, k, device="cuda") * 0.05
    hi = torch.empty(m, k, dtype=torch.float16, device="cuda")
    lo = torch.empty(m, k, dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    native.check(lib.fz_split_f16(x.data_ptr(), m * k, hi.data_ptr(), lo.data_ptr(), s))
    ahi = torch.empty(m, f, dtype=torch.float16, device="cuda")
    alo = torch.empty(m, f, dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    (gc, gs), (uc, us) = mats
    f16 = []
    for codes, scales in mats:
        whi = torch.empty(f, k, dtype=torch.float16, device="cuda")
        wlo = torch.empty(f, k, dtype=torch.float16, device="cuda")
        native.check(lib.fz_q4_0_to_f16(codes.data_ptr(), scales.data_ptr(), f, k, whi.data_ptr(), wlo.data_ptr(), s))
        f16.append((whi, wlo))
    (ghi, glo), (uhi, ulo) = f16
    out = {}
    for key in ("3", "2", "1", "tma3", "tma2", "tma1"):
        passes, tma = int(key[-1]), key.startswith("tma")

        def run():
            xl = lo.data_ptr() if passes >= 2 else None
            al = alo.data_ptr() if passes >= 2 else None
            ex = 1 if passes == 3 else 0
            if tma:
                native.check(lib.fz_f16_gemm_gated(ghi.data_ptr(), glo.data_ptr(), uhi.data_ptr(), ulo.data_ptr(), f,
                                                   k, hi.data_ptr(), xl, ex, m, None, 0, 0, None, ahi.data_ptr(), al,
                                                   err.data_ptr(), s))
            else:
                native.check(lib.fz_q4_0_gemm_gated(gc.data_ptr(), gs.data_ptr(), uc.data_ptr(), us.data_ptr(), f, k,
                                                    hi.data_ptr(), xl, ex, m, None, 0, 0, None, ahi.data_ptr(), al,
                                                    err.data_ptr(), s))
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            run()
        b.record()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        secs = a.elapsed_time(b) / 1000.0 / reps
        out[key] = secs
    flops = 2.0 * m * (2 * f) * k
    return flops, out


def traffic_from_profile(name):
    """DRAM bytes (read + write) a launch of the kernel moved under ncu, from a
    committed one-launch summary (profiles/<name>), or None."""
    p = os.path.join(ROOT, "profiles", name)
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except (OSError, ValueError):
            return None
    return None


def kv_bytes(shape, positions):
    """Key and value bytes the decode attention reads over one-token steps at
    `positions`: each layer reads the keys it attends (the window's for the
    sliding-window layers, every earlier one for the global layers), f16 keys
    and values of its KV heads."""
    per_key = 2 * shape.kv_heads * shape.head_dim * 2
    total = 0
    for p in positions:
        for layer in range(shape.layers):
            glob = layer % shape.pattern == shape.pattern - 1
            total += (p + 1 if glob else min(p + 1, shape.window)) * per_key
    return total


C2_SHAPES = (("q", 1152, 1024), ("k", 1152, 256), ("v", 1152, 256), ("o", 1024, 1152), ("gate_up", 1152, 6912),
             ("down", 6912, 1152), ("head", 1152, 262144))


def c2_sweep(torch, lib, native, reps=5):
    """the isolated Q4_0 product over Gemma-3-1B's linear
    shapes (K -> N) at M = 1, 8, 64 and 512 rows: codes uniform in [0, 15],
    fp16 scales |N(0, 0.005)|, X ~ N(0, 1) f32, seeded.  M <= 16 runs the
    skinny matvec (fz_q4_0_matvec; the head's shape fz_q4_0_head), more rows
    the tcgen05 GEMM on the Q4_0 codes (fz_q4_0_gemm, f32-level, with X split
    into f16 part and remainder by fz_split_f16 in the same timed sequence).
    Each point's launches run back to back from a CUDA graph, each on its own
    copy of the weights, with enough copies (over 320 MB) that L2 holds none
    of them between uses; the time is the graph's replay over its launches
    (CUDA events, median of `reps` replays).  The roofline is whichever bound
    is slower: algorithmic bytes N K 9/16 + 4 M K + 4 M N at the measured HBM
    rate, or 2 M N K flops at the measured bf16 rate; frac = that time over
    the measured time."""
    import numpy as np
    from frizzle_b200 import synth
    hbm, bf16, which = peaks()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows = []
    for name, k, n in C2_SHAPES:
        cb, sb = lib.fz_q4_0_codes_bytes(n, k), lib.fz_q4_0_scales_bytes(n, k)
        copies = int(min(2048, max(2, -(-(320 << 20) // (cb + sb)))))
        codes = torch.empty(copies * cb, dtype=torch.uint8, device="cuda")
        scales = torch.empty(copies * sb, dtype=torch.uint8, device="cuda")
        src = torch.from_numpy(synth.random_q4_0(n, k, seed=2)).cuda()
        s0 = torch.cuda.current_stream().cuda_stream
        native.check(lib.fz_q4_0_repack(src.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(), s0))
        del src
        for c in range(1, copies):   # every copy the same matrix, at its own address
            codes[c * cb:(c + 1) * cb].copy_(codes[:cb])
            scales[c * sb:(c + 1) * sb].copy_(scales[:sb])
        head = n >= 65536
        for m in (1, 8, 64, 512):
            g = torch.Generator(device="cuda").manual_seed(m)
            x = torch.randn(m, k, device="cuda", generator=g)
            y = torch.empty(m, n, device="cuda")
            xh = torch.empty(m, k, dtype=torch.float16, device="cuda")
            xl = torch.empty(m, k, dtype=torch.float16, device="cuda")
            am = torch.zeros(m, dtype=torch.int64, device="cuda")

            def run(c, st):
                cp, sp = codes.data_ptr() + c * cb, scales.data_ptr() + c * sb
                if m <= 16 and head:
                    native.check(lib.fz_q4_0_head(cp, sp, n, k, x.data_ptr(), m, y.data_ptr(), am.data_ptr(), st))
                elif m <= 16:
                    native.check(lib.fz_q4_0_matvec(cp, sp, n, k, x.data_ptr(), m, y.data_ptr(), st))
                else:
                    native.check(lib.fz_split_f16(x.data_ptr(), m * k, xh.data_ptr(), xl.data_ptr(), st))
                    native.check(lib.fz_q4_0_gemm(cp, sp, n, k, xh.data_ptr(), xl.data_ptr(), 1, m, y.data_ptr(),
                                                  err.data_ptr(), st))
            run(0, torch.cuda.current_stream().cuda_stream)   # (first use: lazy set-up outside the capture)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                st = torch.cuda.current_stream().cuda_stream
                for c in range(copies):
                    run(c, st)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            times = []
            for _ in range(reps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                graph.replay()
                b.record()
                torch.cuda.synchronize()
                times.append(a.elapsed_time(b) / 1000.0 / copies)
            assert int(err.item()) == 0
            del graph
            t = float(np.median(times))
            bytes_ = n * k * 9 // 16 + 4 * m * k + 4 * m * n
            flops = 2.0 * m * n * k
            t_hbm, t_tc = bytes_ / (hbm * 1e9), flops / (bf16 * 1e12)
            kern = ("fz_q4_0_head" if head else "fz_q4_0_matvec") if m <= 16 else \
                "fz_split_f16 + fz_q4_0_gemm (tcgen05, f32-level)"
            rows.append({"shape": name, "k": k, "n": n, "m": m, "us": t * 1e6, "kernel": kern,
                         "weight_copies": copies, "algorithmic_bytes": bytes_, "flops": flops,
                         "achieved_gbs": bytes_ / t / 1e9, "achieved_tflops": flops / t / 1e12,
                         "bound": "hbm" if t_hbm >= t_tc else "tensor", "frac": max(t_hbm, t_tc) / t})
            del x, y, xh, xl, am
        del codes, scales
        torch.cuda.empty_cache()
    return {"workload": "BASELINE config 2: isolated Q4_0 products, Gemma-3-1B's linear shapes x M in "
                        "{1, 8, 64, 512}; launches back to back from a CUDA graph over rotating weight copies "
                        "(over 320 MB, larger than L2)", "peak_hbm_gbs": hbm, "peak_bf16_tflops": bf16,
            "peak_source": which, "points": rows}


def run_ours(args):
    import numpy as np
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from frizzle_b200 import _native, engine, synth
    if rank == 0:
        path = synth.model_path(synth.GEMMA3_1B, 0)
    if dist:
        dist.barrier()
    path = synth.model_path(synth.GEMMA3_1B, 0)
    dev = engine.Device(local)
    model = engine.Model.from_file(dev, path)
    batch = engine.Batch(model, 1, 4096)
    lib = _native.load()
    stream = torch.cuda.ExternalStream(dev.stream)
    ids = np.random.default_rng([rank, PROMPT]).integers(2, synth.GEMMA3_1B.vocab, size=PROMPT).astype(np.uint32)

    def prefill():
        # The 32-token prompt in one step (more than 16 rows: the tensor-core path).
        batch.step(0, ids, tokens=PROMPT, logits=True)

    # Prefill timing (two blocks of 16 tokens), after a warm-up prefill.
    prefill()
    batch.wait()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    with torch.cuda.stream(stream):
        ev[0].record()
    prefill()
    with torch.cuda.stream(stream):
        ev[1].record()
    batch.wait()
    prefill_s = ev[0].elapsed_time(ev[1]) / 1000.0

    pos = PROMPT
    for _ in range(args.warmup):
        batch.step(pos, fed=True, tokens=1, logits=True)
        batch.wait()
        pos += 1
    if args.profile_steps:
        # Only the decode steps run between the profiler marks (for ncu --profile-from-start off).
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for i in range(args.profile_steps):
            batch.step(pos + i, fed=True, tokens=1, logits=True)
        batch.wait()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        batch.free()
        model.free()
        dev.close()
        return 0
    K = args.steps

    def rewind():
        # Every timed pass decodes the same positions, from the end of config 1's prompt: the cache
        # is cut back to the prompt (KvCache::truncate) and the next fed step continues from there.
        batch.wait()
        kept = batch.truncate(PROMPT)
        assert kept == PROMPT, kept
        return PROMPT

    pos = rewind()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    with clocks:
        with torch.cuda.stream(stream):
            ev[2].record()
        for i in range(K):
            batch.step(pos + i, fed=True, tokens=1, logits=True)
        with torch.cuda.stream(stream):
            ev[3].record()
        batch.wait()
        torch.cuda.synchronize()
        pos = rewind()
        # End to end: every step's inputs copied in and its records read back, two steps in
        # flight (the next enqueued before the previous one's records are read, as the
        # reference's step order keeps two outstanding), records reported in order.
        with torch.cuda.stream(stream):
            ev[4].record()
        batch.step(pos, fed=True, tokens=1, logits=True)
        for i in range(K):
            if i + 1 < K:
                batch.step(pos + i + 1, fed=True, tokens=1, logits=True)
            batch.wait_oldest()
        with torch.cuda.stream(stream):
            ev[5].record()
        torch.cuda.synchronize()
    pos = rewind()
    dec_s = ev[2].elapsed_time(ev[3]) / 1000.0
    e2e_s = ev[4].elapsed_time(ev[5]) / 1000.0
    # The dominant kernel, the persistent decode step, untraced: CUDA events recorded around its launch on
    # the step's stream (fz_batch_time_decode), K ordinary decode steps, each kernel's duration summed.  Its
    # algorithmic bytes: the 26 layers' Q4_0 weights and norm gains plus the keys and values the steps'
    # attention reads (1 KiB a key a layer).
    import ctypes as C
    engine.check(lib.fz_batch_time_decode(batch.handle, 1))
    for i in range(3):
        batch.step(pos + i, fed=True, tokens=1, logits=True)
        batch.wait()
    pos = rewind()
    dk_us = []
    us = C.c_float()
    for i in range(K):
        batch.step(pos + i, fed=True, tokens=1, logits=True)
        batch.wait()
        engine.check(lib.fz_batch_decode_time(batch.handle, C.byref(us)))
        dk_us.append(us.value)
    engine.check(lib.fz_batch_time_decode(batch.handle, 0))
    dk_secs = float(np.mean(dk_us)) * 1e-6
    dk_bytes = LAYER_BYTES + kv_bytes(synth.GEMMA3_1B, range(pos, pos + K)) / K
    pos += K
    # The capture step and prefix reuse (rank 0): config 1's 32-token prompt as one step with and without
    # the per-layer capture (weights, statistics and 25 readouts through the head), and a second turn
    # that extends a 1024-token first turn's conversation by 16 tokens, prefilled fresh or after the cache
    # keeps the 1039 tokens it already holds.
    extras = None
    if rank == 0:
        def timed(fn, reps=5):
            out = []
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    e0.record()
                fn()
                with torch.cuda.stream(stream):
                    e1.record()
                torch.cuda.synchronize()
                out.append(e0.elapsed_time(e1))
            return float(np.median(out))
        cb = engine.Batch(model, 1, 4096)

        def pre(capture):
            cb.step(0, ids, tokens=PROMPT, logits=True, capture=capture)
            cb.wait()
        pre(False)
        pre(True)
        plain_ms, capture_ms = timed(lambda: pre(False)), timed(lambda: pre(True))
        sess = engine.Session(cb)
        long_ids = np.random.default_rng([rank, 1024]).integers(2, synth.GEMMA3_1B.vocab, size=1024)
        first = sess.run([long_ids], 16)
        convo = list(long_ids) + first.tokens[0][:15] + list(
            np.random.default_rng([rank, 16]).integers(2, synth.GEMMA3_1B.vocab, size=16))
        held = len(convo) - 16
        fresh = engine.Batch(model, 1, 4096)
        full = np.asarray(convo, dtype=np.uint32)

        def fresh_prefill():
            fresh.step(0, full, tokens=len(full), logits=True)
            fresh.wait()

        def reuse_prefill():
            assert cb.truncate(held) == held
            cb.step(held, full[held:], tokens=len(full) - held, logits=True)
            cb.wait()
        fresh_ms, reuse_ms = timed(fresh_prefill), timed(reuse_prefill)
        fresh.free()
        cb.free()
        extras = {"capture_step": {"workload": "config 1's 32-token prompt in one step", "plain_ms": plain_ms,
                                   "with_capture_ms": capture_ms},
                  "prefix_reuse": {"workload": "a second turn: the first turn's 1024-token prompt and 15 fed reply "
                                               "tokens, then 16 new tokens",
                                   "prompt_tokens": len(full), "reused_tokens": held, "fresh_prefill_ms": fresh_ms,
                                   "reused_prefill_ms": reuse_ms}}
    long_line = None
    if not args.no_long:
        # 8 sequences, each a seeded prompt prefilled into the KV cache, then 256 greedy
        # decode steps; sequences sharded across the ranks.  The prompt is 32,512 tokens so that the last
        # step's position is the model's 32,768-token trained context.
        from frizzle_b200 import sweep as _sw
        n_seq, p_len, l_steps, chunk = 8, 32768 - 256, 256, 4096
        mine = list(_sw.shard(n_seq, world, rank))
        lb = engine.Batch(model, len(mine), 32768) if mine else None
        prompts = np.stack([np.random.default_rng([s, 32768]).integers(2, synth.GEMMA3_1B.vocab, size=p_len)
                            for s in mine]).astype(np.uint32) if mine else None
        if dist:
            dist.barrier()
        lv = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        with torch.cuda.stream(stream):
            lv[0].record()
        if lb:
            for p0 in range(0, p_len, chunk):
                t = min(chunk, p_len - p0)
                lb.step(p0, np.ascontiguousarray(prompts[:, p0:p0 + t]), tokens=t, logits=p0 + t == p_len)
        with torch.cuda.stream(stream):
            lv[1].record()
        if lb:
            for i in range(l_steps - 1):
                lb.step(p_len + i, fed=True, tokens=1, logits=True)
            lb.wait()
        with torch.cuda.stream(stream):
            lv[2].record()
        torch.cuda.synchronize()
        l_pre, l_dec = lv[0].elapsed_time(lv[1]) / 1000.0, lv[1].elapsed_time(lv[2]) / 1000.0
        if lb:
            lb.free()
        if dist:
            t = torch.tensor([l_pre, l_dec], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            l_pre, l_dec = [float(v) for v in t.cpu()]
        long_line = {"workload": "BASELINE config 5: 8 sequences x 32,512-token seeded prompt (prefilled in 4096-token "
                                 "steps), then 256 greedy decode steps each (the last at the 32,768 trained context); "
                                 "sequences sharded over the GPUs",
                     "prefill_tokens_per_s": n_seq * p_len / l_pre, "prefill_s": l_pre,
                     "decode_tokens_per_s": n_seq * (l_steps - 1) / l_dec, "decode_s": l_dec,
                     "sequences_per_gpu": len(mine), "scaling": "strong"}
    sweep_line = None
    if not args.no_sweep:
        # 64 steered/unsteered pairs over one 256-token prompt, 128 sampled tokens each
        # (temperature 1, top-k 64), pairs sharded across the ranks; device-timed, max over ranks.
        from frizzle_b200 import sweep
        n_pairs, s_steps, s_layer = 64, 128, 13
        pairs = sweep.make_pairs(n_pairs, synth.GEMMA3_1B.ffn, seed=0)
        mine = [pairs[i] for i in sweep.shard(n_pairs, world, rank)]
        s_prompt = np.random.default_rng([0, 256]).integers(2, synth.GEMMA3_1B.vocab, size=256).astype(np.uint32)
        # Warm-up (untimed): one group of 8 sequences makes the batch and captures its step graphs, which
        # the timed sweep then reuses, as a serving process would.
        warm = {}
        sweep.run(model, s_prompt, mine[:4], 8, s_layer, batch_seqs=8, context=1024, temperature=1.0,
                  batches=warm)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        sv = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        with torch.cuda.stream(stream):
            sv[0].record()
        res = sweep.run(model, s_prompt, mine, s_steps, s_layer, batch_seqs=8, context=1024, temperature=1.0,
                        batches=warm)
        with torch.cuda.stream(stream):
            sv[1].record()
        torch.cuda.synchronize()
        for wb in warm.values():
            wb.free()
        sweep_s = sv[0].elapsed_time(sv[1]) / 1000.0
        full = sweep.gather(res, n_pairs, s_steps, dist, device=torch.device("cuda", local)) if dist else None
        if dist:
            t = torch.tensor([sweep_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sweep_s = float(t.item())
        else:
            full = np.stack([res[i] for i in range(n_pairs)])
        if rank == 0:
            differ = float(np.mean(np.any(full[:, 0] != full[:, 1], axis=1)))
            sweep_line = {"workload": "BASELINE config 4: 64 steered + 64 unsteered twins (same seed), one 256-token "
                                      "prompt, layer-13 pins (k in 1..8, values in [-10, 10]), 128 tokens each at "
                                      "temperature 1, top-k 64; 8 sequences a batch; pairs sharded over the GPUs",
                          "sequences": 2 * n_pairs, "tokens_per_sequence": s_steps, "seconds": sweep_s,
                          "tokens_per_s": 2 * n_pairs * s_steps / sweep_s, "scaling": "strong",
                          "pairs_whose_twins_differ": differ}
    if dist:
        # The job's final exchange: rank 0 gathers every sequence's last logits.
        last = torch.from_numpy(batch.logits(0)).cuda()
        gathered = [torch.empty_like(last) for _ in range(world)] if rank == 0 else None
        dist.gather(last, gathered, dst=0)
        t = torch.tensor([dec_s, e2e_s, prefill_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dec_s, e2e_s, prefill_s = [float(v) for v in t.cpu()]
    value = world * K / dec_s
    e2e = world * K / e2e_s
    line = None
    if rank == 0:
        head_bytes, head_secs = head_roofline(torch, lib, _native)
        hbm, _, which = peaks()
        achieved = head_bytes / head_secs / 1e9
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
                "warmup": args.warmup, "ms_per_step": 1000.0 * dec_s / K, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init Q4_0 weights, seeded prompt ids)",
                "config": config(world),
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 64 + 8, "d2h_bytes_per_step": 16},
                "gpu_launches": LAUNCHES_PER_DECODE_STEP * K,
                "prefill_tokens_per_s": world * PROMPT / prefill_s,
                "decode_step_hbm_gbs": DECODE_BYTES / (dec_s / K) / 1e9,
                "decode_step_hbm_frac": DECODE_BYTES / (dec_s / K) / 1e9 / hbm,
                "roofline": {"bound": "hbm", "kernel": "decode_kernel<1>: the persistent decode step, 26 layers "
                                                        "(the step's dominant launch by time)",
                             "achieved": dk_bytes / dk_secs / 1e9, "peak": hbm, "unit": "GB/s",
                             "frac": dk_bytes / dk_secs / 1e9 / hbm, "peak_source": which,
                             "algorithmic_bytes": dk_bytes, "launch_us": dk_secs * 1e6,
                             "traffic": traffic_from_profile("decode_kernel_traffic.json"),
                             "timing": "CUDA events recorded around the kernel's launch on its stream in each step "
                                       "(fz_batch_time_decode: the step launched directly, not from its graph), "
                                       "untraced, mean of K decode steps",
                             "bytes": "26 layers' Q4_0 weights + norm gains (392,491,008 + 532,480 B) + the keys "
                                      "and values the steps' attention reads (1 KiB a key a layer)"},
                "head_roofline": {"bound": "hbm", "kernel": "q4_0 head matvec 262144 x 1152, M=1, timed alone",
                                  "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                                  "peak_source": which, "algorithmic_bytes": head_bytes,
                                  "launch_us": head_secs * 1e6,
                                  "traffic": traffic_from_profile("head_matvec_traffic.json")},
                "clocks": clocks.summary()}
        if extras:
            line.update(extras)
        if sweep_line:
            line["steering_sweep"] = sweep_line
        if long_line:
            line["long_context"] = long_line
        # a 4096-token prompt prefilled in one step (the tcgen05 path).
        pre = engine.Batch(model, 1, 8192)
        ids4k = np.random.default_rng([rank, 4096]).integers(2, synth.GEMMA3_1B.vocab, size=4096).astype(np.uint32)
        pre.step(0, ids4k, tokens=4096, logits=True)
        pre.wait()
        pstream = torch.cuda.ExternalStream(dev.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(pstream):
            e0.record()
        pre.step(0, ids4k, tokens=4096, logits=True)
        with torch.cuda.stream(pstream):
            e1.record()
        pre.wait()
        p4k = e0.elapsed_time(e1) / 1000.0
        pre.free()
        line["formats_matvec"] = formats_roofline(torch, lib, _native)
        if not args.no_c2:
            line["c2_sweep"] = c2_sweep(torch, lib, _native)
        gflops, gsecs = gemm_roofline(torch, lib, _native)
        _, bf16, _ = peaks()
        line["prefill_4096"] = {"tokens_per_s": 4096 / p4k, "ms": 1000.0 * p4k,
                                "workload": "BASELINE config 3: 4096 seeded ids in one step, 26 layers, "
                                            "f32-level products (X and the weights each as f16 hi + lo, three "
                                            "tcgen05 MMAs a k-slice: the engine's default)",
                                "tflops_algorithmic": 6.03e12 / p4k / 1e12}

        def mode(p, mmas):
            return {"achieved": gflops / gsecs[p] / 1e12, "frac": gflops / gsecs[p] / 1e12 / bf16,
                    "us": gsecs[p] * 1e6, "mmas_per_k_slice": mmas, "tensor_pipe_frac": gflops * mmas / gsecs[p] /
                    1e12 / bf16}
        line["prefill_gemm_roofline"] = {
            "bound": "tensor", "kernel": "tcgen05 gated product 1152 -> 2 x 6912 at M = 4096, weight tiles by TMA "
                                         "from f16 copies (the engine's prefill)",
            "unit": "TFLOP/s", "peak": bf16, "algorithmic_flops": gflops,
            "achieved": gflops / gsecs["tma3"] / 1e12, "frac": gflops / gsecs["tma3"] / 1e12 / bf16,
            "f32_level": mode("tma3", 3), "x_split": mode("tma2", 2), "f16_one_pass": mode("tma1", 1),
            "in_kernel_dequant": {"f32_level": mode("3", 3), "x_split": mode("2", 2), "f16_one_pass": mode("1", 1)},
            "note": "f32_level is the engine's default: with one f16 rounding of X (x_split rounds W) or of both "
                    "(one pass), config 1's logits land at 1.1-1.6e-3 relative RMS from the fp32 oracle, above "
                    "the 1e-3 parity bar; tensor_pipe_frac counts the MMAs the tensor pipe runs"}
        if world == 1 and not args.no_cpu_baseline:
            v, threads, sample = cpu_decode_sample(path, decode_tokens=8, prefill=PROMPT, warmup=1)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    batch.free()
    model.free()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if line:
        print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the tensor-core gated product at M = 4096 and print its numbers")
    ap.add_argument("--formats-only", action="store_true",
                    help="time only the Q8_0 and Q4_1 matvecs at the head's shape and print their numbers")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="run only this many decode steps between cudaProfilerStart/Stop, print nothing")
    ap.add_argument("--no-sweep", action="store_true", help="skip the config-4 steering sweep")
    ap.add_argument("--no-long", action="store_true", help="skip the config-5 long-context run")
    ap.add_argument("--no-c2", action="store_true", help="skip the config-2 product sweep")
    ap.add_argument("--c2-only", action="store_true", help="run only the config-2 product sweep and print it")
    ap.add_argument("--profile-prefill-tokens", type=int, default=4096,
                    help="the prompt length --profile-prefill steps (4096: config 3; 32: config 1's prompt)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="run one config-3 4096-token prefill step between cudaProfilerStart/Stop (after a warm-up one)")
    ap.add_argument("--seqs", type=int, default=1, help="sequences a batch in --trace")
    ap.add_argument("--trace-prompt", type=int, default=PROMPT,
                    help="prompt tokens a sequence before the traced steps (prefilled in 4096-token steps)")
    ap.add_argument("--trace", action="store_true",
                    help="print the decode kernel's phase timeline (device timestamps), averaged over steps")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.gemm_only:
        import torch
        from frizzle_b200 import _native
        flops, secs = gemm_roofline(torch, _native.load(), _native, reps=args.steps)
        _, bf16, _ = peaks()
        print(json.dumps({"kernel": "tcgen05 gated product 1152 -> 2 x 6912, M = 4096",
                          "tflops": {p: flops / t / 1e12 for p, t in secs.items()},
                          "frac": {p: flops / t / 1e12 / bf16 for p, t in secs.items()},
                          "us": {p: t * 1e6 for p, t in secs.items()}}))
        return 0
    if args.formats_only:
        import torch
        from frizzle_b200 import _native
        print(json.dumps(formats_roofline(torch, _native.load(), _native, reps=args.steps)))
        return 0
    if args.c2_only:
        import torch
        from frizzle_b200 import _native
        print(json.dumps(c2_sweep(torch, _native.load(), _native)))
        return 0
    if args.trace:
        return run_trace(args)
    if args.profile_prefill:
        import numpy as np
        import torch
        from frizzle_b200 import engine, synth
        dev = engine.Device(0)
        model = engine.Model.from_file(dev, synth.model_path(synth.GEMMA3_1B, 0))
        b = engine.Batch(model, 1, 8192)
        n = args.profile_prefill_tokens
        ids = np.random.default_rng([0, n]).integers(2, synth.GEMMA3_1B.vocab, size=n).astype(np.uint32)
        b.step(0, ids, tokens=n, logits=True)
        b.wait()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        b.step(0, ids, tokens=n, logits=True)
        b.wait()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        b.free()
        model.free()
        dev.close()
        return 0
    return run_ours(args)


PHASES = ("qkv", "attention", "o", "gate_up", "down", "head")


def run_trace(args):
    """The persistent decode kernel's timeline: per phase, the time from the
    previous phase's last CTA finishing to this phase's last CTA having its
    inputs (hand-off: counter, wait, prologue) and from then to its last CTA
    finishing (work), in microseconds, the mean over layers and steps."""
    import ctypes as C
    import numpy as np
    from frizzle_b200 import engine, synth
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, synth.model_path(synth.GEMMA3_1B, 0))
    S, P = args.seqs, args.trace_prompt
    context = max(4096, P + args.warmup + args.steps + 1)
    batch = engine.Batch(model, S, context)
    ids = np.random.default_rng([0, P]).integers(2, synth.GEMMA3_1B.vocab, size=P).astype(np.uint32)
    for p0 in range(0, P, 4096):
        t = min(4096, P - p0)
        batch.step(p0, np.ascontiguousarray(np.tile(ids[p0:p0 + t], (S, 1))), tokens=t, logits=p0 + t == P)
    batch.wait()
    lib = batch.lib
    engine.check(lib.fz_batch_trace(batch.handle, 1))
    ctas, events = C.c_uint32(), C.c_uint32()
    engine.check(lib.fz_batch_read_trace(batch.handle, None, 0, C.byref(ctas), C.byref(events)))
    L = synth.GEMMA3_1B.layers
    hand = np.zeros((L, 6)), np.zeros((L, 6))
    spread = [{k: [] for k in ("work_median", "work_max", "ready_first", "ready_last", "counter_seen_last",
                               "prologue_median", "compute_median", "finish_median")} for _ in range(6)]
    totals = []
    tails = []
    pos, n = P, 0
    for i in range(args.warmup + args.steps):
        batch.step(pos, fed=True, tokens=1, logits=True)
        batch.wait()
        pos += 1
        if i < args.warmup:
            continue
        buf = np.zeros(ctas.value * events.value, dtype=np.uint64)
        engine.check(lib.fz_batch_read_trace(batch.handle, buf.ctypes.data, buf.size, None, None))
        body = L * 6 * 5
        tail = buf.reshape(ctas.value, events.value)[:, body:].astype(np.float64)
        tails.append(tail)
        t = buf.reshape(ctas.value, events.value)[:, :body].reshape(ctas.value, L, 6, 5).astype(np.float64)
        t[t == 0] = np.nan
        t0 = np.nanmin(t)
        t = (t - t0) / 1000.0
        prev = 0.0
        for l in range(L):
            for ph in range(6):
                if ph == 5 and l != L - 1:
                    continue
                if np.all(np.isnan(t[:, l, ph, 4])):
                    continue
                seen = np.nanmax(t[:, l, ph, 1])
                ready = np.nanmax(t[:, l, ph, 2])
                done = np.nanmax(t[:, l, ph, 4])
                per = t[:, l, ph, 4] - t[:, l, ph, 2]
                spread[ph]["compute_median"].append(np.nanmedian(t[:, l, ph, 3] - t[:, l, ph, 2]))
                spread[ph]["finish_median"].append(np.nanmedian(t[:, l, ph, 4] - t[:, l, ph, 3]))
                spread[ph]["counter_seen_last"].append(seen - prev)
                spread[ph]["prologue_median"].append(np.nanmedian(t[:, l, ph, 2] - t[:, l, ph, 1]))
                spread[ph]["work_median"].append(np.nanmedian(per))
                spread[ph]["work_max"].append(np.nanmax(per))
                spread[ph]["ready_first"].append(np.nanmin(t[:, l, ph, 2]) - prev)
                spread[ph]["ready_last"].append(ready - prev)
                hand[0][l, ph] += ready - prev
                hand[1][l, ph] += done - ready
                prev = done
        totals.append(prev)
        n += 1
    out = {"steps": n, "kernel_us": float(np.mean(totals)), "phases": {}}
    tl = np.mean(np.stack(tails), axis=0)  # [ctas][9], ns
    out["tile_wait_us_per_cta"] = {name: float(np.mean(tl[:, i]) / 1000.0) for i, name in enumerate(PHASES)}
    out["issuer"] = {"wait_us": float(np.mean(tl[:, 6]) / 1000.0), "issue_us": float(np.mean(tl[:, 7]) / 1000.0),
                     "tiles": float(np.mean(tl[:, 8]))}
    out["cta_span_us"] = {"entry_spread": float(np.ptp(tl[:, 9]) / 1000.0),
                          "exit_spread": float(np.ptp(tl[:, 10]) / 1000.0),
                          "first_entry_to_last_exit": float((tl[:, 10].max() - tl[:, 9].min()) / 1000.0)}
    for ph, name in enumerate(PHASES):
        rows = range(L - 1, L) if ph == 5 else range(L)
        if not spread[ph]["work_max"]:
            continue
        out["phases"][name] = {"handoff_us": float(np.mean([hand[0][l, ph] for l in rows]) / n),
                               "work_us": float(np.mean([hand[1][l, ph] for l in rows]) / n)}
        out["phases"][name].update({k: float(np.mean(v)) for k, v in spread[ph].items()})
    # Each layer's phases (hand-off + work, us): the global layers stand out at long contexts.
    out["layers"] = [[round(float((hand[0][l, ph] + hand[1][l, ph]) / n), 2) for ph in range(5)] for l in range(L)]
    print(json.dumps(out))
    batch.free()
    model.free()
    dev.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
