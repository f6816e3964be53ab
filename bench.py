#!/usr/bin/env python
"""Benchmark: Q4_K GEMV HBM throughput on B200 (the reference's headline metric).

One step = one decode-matvec pass over the Q4_K shape sweep of the benchmark
configuration (out x in = 4096x4096, 4096x12288, 12288x4096, 151936x4096),
weights in native GGUF Q4_K blocks resident in HBM, fp32 activations
~N(0,1), through the C ABI entry point gncx_xfold_universal_matvec.  The four
weight tensors total 417 MB per step, larger than the 126 MB L2, so every step
streams from HBM.

value     = algorithmic bytes (weights + x + y) of all steps on all ranks /
            device time (CUDA events, max over ranks).
e2e       = the same through the same entry point with host buffers: each
            step copies every x from pinned host memory and reads every y back.
roofline  = the 151936x4096 launch (84% of the bytes) against the measured
            HBM copy bandwidth in MEASURED_PEAKS.json.
Multi-GPU: one process per GPU, each streaming its own copy of the sweep
(the GEMV shards by rows with no exchange): weak scaling.

``--impl reference`` times the reference's own CPU kernels (oracle/_ref, built
from its sources) on the same sweep with all host threads its pool uses.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q4_K GEMV HBM GB/s"
SHAPES = [(4096, 4096), (4096, 12288), (12288, 4096), (151936, 4096)]  # (out, in)
SWEEP_TYPES = [2, 8, 12, 14]


def algo_bytes(t: int, out_dim: int, in_dim: int) -> int:
    from gncx_b200.core import row_bytes
    return out_dim * row_bytes(t, in_dim) + 4 * in_dim + 4 * out_dim


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50", "-i",
                 str(device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        time.sleep(0.12)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def host_info() -> dict:
    """The host the CPU baseline runs on: CPU model, the ISA extensions that
    matter to the reference's kernels, logical CPUs, the CPUs this process
    may use, and the reference pool's thread cap (clamp(hw, 2, 12),
    csrc/gncx_llm_kernels.cpp:141)."""
    model, flags = "unknown", set()
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name") and model == "unknown":
                model = line.split(":", 1)[1].strip()
            elif line.startswith("flags") and not flags:
                flags = set(line.split(":", 1)[1].split())
    except OSError:
        pass
    isa = [f for f in ("sse4_2", "avx", "avx2", "fma", "avx512f", "avx512bw", "avx512_vnni", "avx_vnni", "amx_int8")
           if f in flags]
    logical = os.cpu_count() or 1
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = logical
    from oracle.oracle import ref_build_flags, timing_reference_so
    return {"cpu_model": model, "isa": isa, "logical_cpus": logical, "usable_cpus": usable,
            "reference_pool_threads": max(2, min(usable, 12)), "reference_build": ref_build_flags(timing_reference_so())}


def gen_weights_gpu(torch, t: int, out_dim: int, in_dim: int, seed: int):
    """Seeded random blocks generated on the device (same distributions as gncx_b200.synth)."""
    from gncx_b200.core import BLOCK, Q4_0, Q4_K, Q6_K, Q8_0
    be, bb = BLOCK[t]
    n = out_dim * (in_dim // be)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    raw = torch.randint(0, 256, (n, bb), dtype=torch.uint8, device="cuda", generator=g)

    def scales():
        return torch.randn(n, device="cuda", generator=g).mul_(0.02).abs_().half().view(torch.uint8).view(n, 2)

    if t in (Q4_0, Q8_0, Q4_K):
        raw[:, 0:2] = scales()
    if t == Q4_K:
        raw[:, 2:4] = scales()
    if t == Q6_K:
        raw[:, 208:210] = scales()
    return raw.view(-1)


def read_traffic() -> float | None:
    """DRAM bytes per launch of the 151936x4096 Q4_K GEMV from the committed ncu summary."""
    p = ROOT / "profiles" / "gemv_q4_k_151936x4096.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def cpu_baseline(seconds: float = 8.0) -> dict:
    """The reference's CPU matvec (oracle/_ref, as-shipped flags) on the Q4_K sweep."""
    from gncx_b200 import synth
    from oracle.oracle import Oracle, RefLib, timing_reference_so
    so = timing_reference_so()
    kind = "reference" if so.exists() else "port"
    impl = RefLib(so) if kind == "reference" else Oracle()
    cores = max(2, min(os.cpu_count() or 1, 12)) if kind == "reference" else 1  # the port is one thread
    data = []
    for i, (o, n) in enumerate(SHAPES):
        data.append((synth.random_weights_fast(12, o, n, seed=10 + i), synth.random_activations(n, seed=20 + i), o))
    total_bytes, total_t, reps = 0, 0.0, 0
    t_end = time.time() + seconds
    while time.time() < t_end or reps == 0:
        for w, x, o in data:
            t0 = time.perf_counter()
            impl.matvec(w, 12, x, o)
            total_t += time.perf_counter() - t0
            total_bytes += algo_bytes(12, o, x.size)
        reps += 1
    return {"value": total_bytes / total_t / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{reps} passes over the Q4_K sweep (all four shapes), {total_t:.1f} s of CPU time",
            "host": host_info()}


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from gncx_b200 import synth
    from oracle.oracle import Oracle, RefLib, timing_reference_so
    so = timing_reference_so()
    kind = "reference" if so.exists() else "port"
    impl = RefLib(so) if kind == "reference" else Oracle()
    cores = max(2, min(os.cpu_count() or 1, 12)) if kind == "reference" else 1  # the port is one thread
    data = [(synth.random_weights_fast(12, o, n, seed=10 + i), synth.random_activations(n, seed=20 + i), o)
            for i, (o, n) in enumerate(SHAPES)]
    step_bytes = sum(algo_bytes(12, o, x.size) for _, x, o in data)
    for _ in range(args.warmup):
        for w, x, o in data:
            impl.matvec(w, 12, x, o)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for w, x, o in data:
            impl.matvec(w, 12, x, o)
    dt = time.perf_counter() - t0
    value = step_bytes * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_k weights, int8 x int8 dots, f32 accumulate",
        "data": "synthetic (seeded GGUF Q4_K blocks, x ~ N(0,1))",
        "config": {"workload": "Q4_K GEMV sweep 4096x4096, 4096x12288, 12288x4096, 151936x4096 (out x in), batch 1",
                   "l2": "inputs larger than L2 (417 MB of weights per step)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": f"{args.steps} full passes over the sweep", "host": host_info()},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def format_sweep(torch, lib, P, reps: int = 20) -> dict:
    """GB/s of every format x shape of the GEMV sweep (each timed alone, L2
    flushed between repetitions by a 256 MB write)."""
    names = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    res = {}
    stream = torch.cuda.current_stream()
    for t in SWEEP_TYPES:
        for i, (o, n) in enumerate(SHAPES):
            w = gen_weights_gpu(torch, t, o, n, seed=77 + i)
            x = torch.randn(n, device="cuda")
            y = torch.empty(o, device="cuda")
            times = []
            for r in range(reps + 2):
                flush.fill_(float(r))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                lib.gncx_xfold_universal_matvec(P(w), 0, t, P(x), None, n, o, P(y), None)
                b.record(stream)
                torch.cuda.synchronize()
                if r >= 2:
                    times.append(a.elapsed_time(b))
            ms = statistics.median(times)
            res[f"{names[t]} {o}x{n}"] = {"us": ms * 1e3, "GB/s": algo_bytes(t, o, n) / (ms / 1e3) / 1e9}
            del w
    return res


DECODE_SHAPES = [(6144, 4096), (24576, 4096), (4096, 12288), (4096, 4096)]  # 8B decode: qkv, gate/up, down, o


def gemv_kernel_sweep(torch, lib, P, shapes=DECODE_SHAPES, t: int = 12, reps: int = 5) -> dict:
    """Kernel time of the decode-sized GEMVs, no host API time: one CUDA graph
    per shape holds back-to-back drop-in matvec launches, each on its own copy
    of the weights (copies totalling >= 2x L2, so every launch streams from
    HBM), with weight prefetch across launch boundaries as in decode.  The
    graph is replayed `reps` times; time per launch = replay time / launches."""
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    peak = float(measured_peaks().get("hbm_gbs", 6650.0))
    names = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}
    res = {}
    outer = torch.cuda.current_stream()
    for i, (o, n) in enumerate(shapes):
        nbytes = algo_bytes(t, o, n)
        copies = max(4, -(-2 * l2 // nbytes))
        ws = [gen_weights_gpu(torch, t, o, n, seed=500 + 31 * i + c) for c in range(copies)]
        x = torch.randn(n, device="cuda")
        y = torch.empty(o, device="cuda")
        ptrs = [P(w) for w in ws]
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(outer)
        with torch.cuda.stream(s):
            lib.gncx_set_stream(ctypes.c_void_p(s.cuda_stream))
            lib.gncx_xfold_universal_matvec(ptrs[0], 0, t, P(x), None, n, o, P(y), None)  # configure outside capture
            s.synchronize()
            with torch.cuda.graph(g, stream=s):
                for c in range(copies):
                    lib.gncx_xfold_universal_matvec(ptrs[c], 0, t, P(x), None, n, o, P(y), None)
        lib.gncx_set_stream(ctypes.c_void_p(outer.cuda_stream))
        from gncx_b200 import core
        core.check(lib)
        g.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(outer)
            g.replay()
            b.record(outer)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) / copies)
        ms = statistics.median(times)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[f"{names[t]} {o}x{n}"] = {"us": ms * 1e3, "GB/s": gbs, "frac": gbs / peak, "launches": copies}
        del g, ws
        torch.cuda.empty_cache()
    return res


def attention_sweep(torch, lib, P, reps: int = 20) -> dict:
    """Configuration 3: one decode attention step (32 query heads, 8 KV heads,
    head_dim 128, fp32 KV cache ~ N(0,1)) through gncx_mqa_attention_step_ext
    at context 512 / 4096 / 32768 and a 4096 window; each call timed alone
    with L2 flushed.  Bytes: the K and V rows the window reads, the new K/V
    row written, q read and the output written."""
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    nh, nkv, hd = 32, 8, 128
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    peak = float(measured_peaks().get("hbm_gbs", 6650.0))
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    res = {}
    for ctx, win in ((512, 0), (4096, 0), (32768, 0), (32768, 4096)):
        kc = torch.randn(ctx * nkv * hd, device="cuda", generator=g)
        vc = torch.randn(ctx * nkv * hd, device="cuda", generator=g)
        q = torch.randn(nh * hd, device="cuda", generator=g)
        k = torch.randn(nkv * hd, device="cuda", generator=g)
        v = torch.randn(nkv * hd, device="cuda", generator=g)
        out = torch.empty(nh * hd, device="cuda")
        times = []
        for r in range(reps + 2):
            flush.fill_(float(r))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            lib.gncx_mqa_attention_step_ext(P(q), P(k), P(v), P(kc), P(vc), ctx - 1, nh, nkv, hd, scale, win, 1,
                                            P(out))
            b.record(stream)
            torch.cuda.synchronize()
            if r >= 2:
                times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        span = min(ctx, win) if win > 0 else ctx
        nbytes = 2 * span * nkv * hd * 4 + 2 * nkv * hd * 4 + 2 * nh * hd * 4
        gbs = nbytes / (ms / 1e3) / 1e9
        res[f"ctx {ctx}" + (f" window {win}" if win else "")] = {"us": ms * 1e3, "GB/s": gbs, "frac": gbs / peak}
        del kc, vc
    return res


def attention_kernel_sweep(torch, lib, P, reps: int = 5) -> dict:
    """The same attention steps without host API time: one CUDA graph per
    configuration holds back-to-back gncx_mqa_attention_step_ext calls (KV
    write, split-KV partial, merge), each on its own copy of the cache (copies
    totalling >= 2x L2, so every step streams its window from HBM), replayed
    `reps` times; time per step = replay time / steps."""
    nh, nkv, hd = 32, 8, 128
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    peak = float(measured_peaks().get("hbm_gbs", 6650.0))
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    outer = torch.cuda.current_stream()
    g0 = torch.Generator(device="cuda")
    g0.manual_seed(13)
    res = {}
    for ctx, win in ((512, 0), (4096, 0), (32768, 0), (32768, 4096)):
        span = min(ctx, win) if win > 0 else ctx
        kv_bytes = 2 * ctx * nkv * hd * 4
        copies = max(2, -(-2 * l2 // (2 * span * nkv * hd * 4)))
        copies = min(copies, max(2, (24 << 30) // kv_bytes))  # stay within a few GB of the device
        caches = [(torch.randn(ctx * nkv * hd, device="cuda", generator=g0),
                   torch.randn(ctx * nkv * hd, device="cuda", generator=g0)) for _ in range(copies)]
        q = torch.randn(nh * hd, device="cuda", generator=g0)
        k = torch.randn(nkv * hd, device="cuda", generator=g0)
        v = torch.randn(nkv * hd, device="cuda", generator=g0)
        out = torch.empty(nh * hd, device="cuda")
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(outer)
        with torch.cuda.stream(s):
            lib.gncx_set_stream(ctypes.c_void_p(s.cuda_stream))
            kc, vc = caches[0]
            lib.gncx_mqa_attention_step_ext(P(q), P(k), P(v), P(kc), P(vc), ctx - 1, nh, nkv, hd, scale, win, 1,
                                            P(out))  # workspace and attributes set up outside the capture
            s.synchronize()
            with torch.cuda.graph(g, stream=s):
                for kc, vc in caches:
                    lib.gncx_mqa_attention_step_ext(P(q), P(k), P(v), P(kc), P(vc), ctx - 1, nh, nkv, hd, scale,
                                                    win, 1, P(out))
        lib.gncx_set_stream(ctypes.c_void_p(outer.cuda_stream))
        from gncx_b200 import core
        core.check(lib)
        g.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(outer)
            g.replay()
            b.record(outer)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) / copies)
        ms = statistics.median(times)
        nbytes = 2 * span * nkv * hd * 4 + 2 * nkv * hd * 4 + 2 * nh * hd * 4
        gbs = nbytes / (ms / 1e3) / 1e9
        res[f"ctx {ctx}" + (f" window {win}" if win else "")] = {"us": ms * 1e3, "GB/s": gbs, "frac": gbs / peak,
                                                                 "steps": copies}
        del g, caches
        torch.cuda.empty_cache()
    return res


def decode_bench(args, torch) -> dict:
    """Benchmark configuration 5: random-init 8B-shaped Qwen3 decoder (Q4_K
    weights, Q6_K tied head), 2048-token seeded prompt prefilled through the
    batched prefill path, then greedy decode; device-timed."""
    import tempfile

    from gncx_b200 import gguf
    from gncx_b200.streamer import GNCXStreamer
    tmp = Path(os.environ.get("GNCX_BENCH_DIR", tempfile.gettempdir()))
    path = tmp / f"gncx_bench_{args.model}_{args.seed}.gguf"
    t0 = time.time()
    if not path.exists():
        gguf.write_random_model(path, args.model, seed=args.seed)
    write_s = time.time() - t0
    prompt = np.random.default_rng(args.seed).integers(0, 151936, args.prompt).tolist()
    res = {"model": args.model, "prompt": args.prompt, "new_tokens": args.new_tokens, "weights": "Q4_K, Q6_K head",
           "model_write_s": round(write_s, 1)}
    with GNCXStreamer(path, max_seq_len=args.prompt + args.new_tokens) as eng:
        modes = [m for m in args.decode_modes.split(",") if m]
        for mode, exact in (("split_kv", False), ("exact_softmax", True)):
            if mode not in modes:
                continue
            eng.set_exact_attention(exact)
            eng.generate_ids(prompt[:64], 8, eos_id=-1)  # warm-up (graph capture)
            ids = eng.generate_ids(prompt, args.new_tokens, eos_id=-1)
            t = eng.timing()
            res[mode] = {"decode_tok_s": t["decode_steps"] / (t["decode_ms"] / 1e3),
                         "ms_per_token": t["decode_ms"] / max(1, t["decode_steps"]),
                         "prefill_tok_s": args.prompt / (t["prefill_ms"] / 1e3), "prefill_ms": t["prefill_ms"],
                         "tokens": len(ids), "first_ids": ids[:8]}
    # reference CPU decode and prefill on the same file (bounded samples)
    if not args.no_cpu_baseline:
        res["cpu_reference"] = cpu_model_baseline(path, prompt, args.prompt + args.new_tokens)
        cpu = res["cpu_reference"]["decode_tok_s"]
        for mode in ("split_kv", "exact_softmax"):
            if mode in res:
                res[mode]["speedup_vs_cpu_decode"] = res[mode]["decode_tok_s"] / cpu
                res[mode]["speedup_vs_cpu_prefill"] = res[mode]["prefill_tok_s"] / res["cpu_reference"]["prefill_tok_s"]
    return res


def cpu_model_baseline(path, prompt, max_seq: int, n_prefill: int = 128) -> dict:
    """The reference's own kernels (oracle/_ref, its thread pool) driven by the
    restated orchestrator on the same model file: prefill tok/s over the
    first `n_prefill` prompt tokens, and decode tok/s of forward_token at the
    positions the GPU decode covers (5 steps at the start of the decode
    range and 5 at its end; a step's time does not depend on the cache's
    contents, only on its length)."""
    from oracle.oracle import OracleModel, timing_reference_so
    ref = OracleModel(path, max_seq, timing_reference_so())
    try:
        t0 = time.perf_counter()
        ref.prefill(prompt[:n_prefill])
        prefill_s = time.perf_counter() - t0
        start = len(prompt)
        positions = list(range(start, start + 5)) + list(range(max_seq - 5, max_seq))
        t0 = time.perf_counter()
        for p in positions:
            ref.forward_token(int(prompt[p % len(prompt)]), p)
        decode_s = time.perf_counter() - t0
    finally:
        ref.close()
    return {"decode_tok_s": len(positions) / decode_s, "prefill_tok_s": n_prefill / prefill_s, "kind": ref.kind,
            "host": host_info(),
            "sample": f"prefill of {n_prefill} prompt tokens; forward_token at positions {positions[0]}-"
                      f"{positions[4]} and {positions[5]}-{positions[-1]} of the {max_seq}-position cache"}


def tp_decode_bench(args, torch, dist, rank: int, world: int, local: int) -> dict:
    """Configuration 5 tensor-parallel over the `world` GPUs of this job: every
    rank loads its row share of the same random-init 8B-shaped model and the
    ranks all-gather over NVLink peer memory; device time, max over ranks."""
    import tempfile

    from gncx_b200 import gguf
    from gncx_b200.streamer import GNCXStreamer
    tmp = Path(os.environ.get("GNCX_BENCH_DIR", tempfile.gettempdir()))
    path = tmp / f"gncx_bench_{args.model}_{args.seed}.gguf"
    t0 = time.time()
    if rank == 0 and not path.exists():
        gguf.write_random_model(path, args.model, seed=args.seed)
    dist.barrier()
    write_s = time.time() - t0
    prompt = np.random.default_rng(args.seed).integers(0, 151936, args.prompt).tolist()

    def exchange(blob: bytes) -> list:
        out = [None] * world
        dist.all_gather_object(out, blob)
        return out

    eng = GNCXStreamer(path, max_seq_len=args.prompt + args.new_tokens, device=local, tp_rank=rank, tp_size=world,
                       exchange=exchange)
    try:
        eng.generate_ids(prompt[:64], 8, eos_id=-1)  # warm-up (graph capture)
        ids = eng.generate_ids(prompt, args.new_tokens, eos_id=-1)
        t = eng.timing()
    finally:
        dist.barrier()  # no rank unmaps its exchange region while another may still write into it
        eng.close()
    tt = torch.tensor([t["decode_ms"], t["prefill_ms"]], device="cuda", dtype=torch.float64)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    decode_ms, prefill_ms = tt.tolist()
    steps = max(1, t["decode_steps"])
    return {"model": args.model, "prompt": args.prompt, "new_tokens": args.new_tokens, "weights": "Q4_K, Q6_K head",
            "model_write_s": round(write_s, 1), "tensor_parallel": world,
            "split_kv": {"decode_tok_s": steps / (decode_ms / 1e3), "ms_per_token": decode_ms / steps,
                         "prefill_tok_s": args.prompt / (prefill_ms / 1e3), "prefill_ms": prefill_ms,
                         "tokens": len(ids), "first_ids": ids[:8], "timing": "device, max over ranks"}}


def run_gpu(args) -> None:
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    from gncx_b200 import core
    lib = core.load()
    stream = core.bind_torch_stream(lib)
    lib.gncx_set_synchronous(0)
    lib.gncx_set_weight_prefetch(0 if args.no_prefetch else 1)
    core.check(lib)

    def P(t):
        return ctypes.c_void_p(t.data_ptr())

    # ---- data resident in HBM
    weights = [gen_weights_gpu(torch, 12, o, n, seed=1000 * rank + i) for i, (o, n) in enumerate(SHAPES)]
    g = torch.Generator(device="cuda")
    g.manual_seed(7 + rank)
    xs = [torch.randn(n, device="cuda", generator=g) for (_, n) in SHAPES]
    ys = [torch.empty(o, device="cuda") for (o, _) in SHAPES]
    step_bytes = sum(algo_bytes(12, o, n) for (o, n) in SHAPES)
    big = len(SHAPES) - 1
    big_bytes = algo_bytes(12, *SHAPES[big])

    def launch(i):
        o, n = SHAPES[i]
        lib.gncx_xfold_universal_matvec(P(weights[i]), 0, 12, P(xs[i]), None, n, o, P(ys[i]), None)

    def barrier():
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        for i in range(len(SHAPES)):
            launch(i)
    core.check(lib)
    barrier()

    ev_big = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(local)
    time.sleep(0.05)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record(stream)
    for s in range(args.steps):
        for i in range(len(SHAPES)):
            if i == big:
                ev_big[s][0].record(stream)
                launch(i)
                ev_big[s][1].record(stream)
            else:
                launch(i)
    stop.record(stream)
    barrier()
    clocks = sampler.stop()
    core.check(lib)
    ms = start.elapsed_time(stop)
    big_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_big)
    launches = args.steps * len(SHAPES)

    # ---- end to end through the same entry point with host buffers: every
    # step copies its x vectors in from pinned host memory and its y vectors
    # back out.  The copies run on a second stream (the copy engines) into
    # double-buffered device vectors, so step s's copies overlap the GEMVs
    # of steps s-1 / s+1, as a serving loop would pipeline them.
    nx, ny = sum(n for (_, n) in SHAPES), sum(o for (o, _) in SHAPES)
    hx = torch.empty(nx, dtype=torch.float32).pin_memory()
    hy = torch.empty(ny, dtype=torch.float32).pin_memory()
    hx.copy_(torch.cat([x.cpu() for x in xs]))
    dx = [torch.empty(nx, device="cuda") for _ in range(2)]
    dy = [torch.empty(ny, device="cuda") for _ in range(2)]
    xoff = np.cumsum([0] + [n for (_, n) in SHAPES]).tolist()
    yoff = np.cumsum([0] + [o for (o, _) in SHAPES]).tolist()
    cstream = torch.cuda.Stream()
    e2e_steps = max(1, min(args.steps, 200))

    # the per-call arguments, built once (the host must keep ahead of the GPU)
    wptr = [P(wt) for wt in weights]
    xptr = [[ctypes.c_void_p(dx[k].data_ptr() + 4 * xoff[i]) for i in range(len(SHAPES))] for k in range(2)]
    yptr = [[ctypes.c_void_p(dy[k].data_ptr() + 4 * yoff[i]) for i in range(len(SHAPES))] for k in range(2)]
    matvec = lib.gncx_xfold_universal_matvec
    x_in = [torch.cuda.Event(), torch.cuda.Event()]    # dx[k] filled
    x_free = [torch.cuda.Event(), torch.cuda.Event()]  # the GEMVs that read dx[k] / wrote dy[k] are done
    y_free = [torch.cuda.Event(), torch.cuda.Event()]  # dy[k] is on the host

    def e2e_run(nsteps):
        for s in range(nsteps):
            k = s & 1
            with torch.cuda.stream(cstream):
                if s >= 2:
                    cstream.wait_event(x_free[k])
                dx[k].copy_(hx, non_blocking=True)
                x_in[k].record(cstream)
            stream.wait_event(x_in[k])
            if s >= 2:
                stream.wait_event(y_free[k])
            for i, (o, n) in enumerate(SHAPES):
                matvec(wptr[i], 0, 12, xptr[k][i], None, n, o, yptr[k][i], None)
            x_free[k].record(stream)
            with torch.cuda.stream(cstream):
                cstream.wait_event(x_free[k])
                hy.copy_(dy[k], non_blocking=True)
                y_free[k].record(cstream)
        stream.wait_event(y_free[(nsteps - 1) & 1])  # the last result is on the host before the clock stops

    e2e_run(min(3, args.warmup))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(e2e_steps)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    core.check(lib)
    if not np.array_equal(hy[yoff[-2]:yoff[-1]].numpy(), ys[-1].cpu().numpy()):
        raise RuntimeError("end-to-end result differs from the device-resident run")

    # ---- max over ranks
    t = torch.tensor([ms, e2e_ms, big_ms], device="cuda")
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms, e2e_ms, big_ms = t.tolist()
    tp_decode = None
    if pg and not args.no_decode:  # every rank takes part in the tensor-parallel decode
        del weights
        torch.cuda.empty_cache()
        try:
            tp_decode = tp_decode_bench(args, torch, pg, rank, world, local)
        except Exception as exc:  # reported in the line; the GEMV numbers stand
            tp_decode = {"error": f"{type(exc).__name__}: {exc}"[:300]}

    if rank == 0:
        peaks = measured_peaks()
        peak = float(peaks.get("hbm_gbs", 6650.0))
        peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
        value = step_bytes * args.steps * world / (ms / 1e3) / 1e9
        achieved = big_bytes / (big_ms / 1e3) / 1e9
        h2d = 4 * nx
        d2h = 4 * ny
        traffic = read_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k weights, int8 x int8 dots, f32 accumulate",
            "data": "synthetic (seeded GGUF Q4_K blocks generated on device, x ~ N(0,1))",
            "config": {"workload": "Q4_K GEMV sweep 4096x4096, 4096x12288, 12288x4096, 151936x4096 (out x in), "
                                   "batch 1, one matvec call per shape per step",
                       "l2": "inputs larger than L2 (417 MB of weights per step)",
                       "parallelism": f"replicas x{world} (rows shard with no exchange)",
                       "weight_prefetch": not args.no_prefetch,
                       "pct_of_hbm_peak": value / world / peak},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "gemv_kernel<Q4_K> 151936x4096", "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": big_bytes},
            "e2e": {"value": step_bytes * e2e_steps * world / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "gncx_xfold_universal_matvec, x from pinned host, y back to pinned host; copies on a "
                           "second stream, double-buffered, overlapping the neighbouring steps' GEMVs"},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if not args.no_sweep:
            lib.gncx_set_weight_prefetch(0)  # each sweep entry is timed alone
            line["sweep"] = format_sweep(torch, lib, P)
            lib.gncx_set_weight_prefetch(1)
            try:
                line["gemv_kernel_only"] = gemv_kernel_sweep(torch, lib, P)
            except Exception as exc:  # reported; the GEMV numbers stand
                line["gemv_kernel_only"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            lib.gncx_set_weight_prefetch(0)
            try:
                line["attention"] = attention_sweep(torch, lib, P)
            except Exception as exc:  # reported; the GEMV numbers stand
                line["attention"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            try:
                line["attention_kernel_only"] = attention_kernel_sweep(torch, lib, P)
            except Exception as exc:  # reported; the GEMV numbers stand
                line["attention_kernel_only"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        if tp_decode is not None:
            line["decode"] = tp_decode
        elif not args.no_decode:
            del weights
            torch.cuda.empty_cache()
            line["decode"] = decode_bench(args, torch)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="gncx", choices=["gncx", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-format sweep table")
    ap.add_argument("--no-decode", action="store_true", help="skip the 8B-shape decode/prefill measurement")
    ap.add_argument("--model", default="qwen3-8b", choices=["qwen3-8b", "qwen3-0.6b", "qwen3-8b-2l"],
                    help="qwen3-8b-2l: the 8B layer shape with two layers, for kernel profiling captures")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--new-tokens", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--decode-modes", default="split_kv,exact_softmax")
    ap.add_argument("--shapes", default="", help="override the timed GEMV shapes, e.g. 4096x12288,24576x4096 (out x in)")
    ap.add_argument("--no-prefetch", action="store_true",
                    help="disable weight prefetch across kernel boundaries (programmatic dependent launch)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.shapes:
        global SHAPES
        SHAPES = [tuple(int(v) for v in sh.split("x")) for sh in args.shapes.split(",")]
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
