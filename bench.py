"""Decode throughput of the Qwen3-0.6B Q8_0 token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]
                    [--config bs1_400|bs1_100|fp32|bs64|bs256]

Workload (the default): seeded synthetic Qwen3-0.6B
Q8_0 decoder (28 layers, hidden 1024, 16/8 heads of 128, FFN 3072, vocab
151936, tied embedding), prefix of 400 N(0,1) audio embeddings + 8 prompt
token ids, then fixed-length greedy decode (no end-token stop).  One bench
step = one decode token; the timed region is K consecutive decode steps
starting right after the prefill, so positions are the config's 408..408+K.

Batched configs (BASELINE configs[3] and, per GPU, configs[4]): bs64 / bs256
independent sessions with prefixes of U[50, 400] audio vectors + 8 ids,
prefilled one by one (untimed), then 128 greedy steps of every session at
once through fa_batch_generate; one bench step = one token of every session.
The default bs1 line carries both batched measurements under "batched".

Multi-GPU (torchrun): one process per GPU, each its own replica and sessions
(independent utterances, no collective on the data path): weak scaling.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (audio frames, prompt ids, decode tokens, quantized)
    "bs1_400": (400, 8, 256, True),   # BASELINE configs[1] (metric's config)
    "bs1_100": (100, 8, 128, True),   # configs[0]
    "fp32": (100, 8, 128, False),     # configs[2]
}
# name: (sessions per GPU, decode tokens per session)
BATCH_CONFIGS = {
    "bs64": (64, 128),
    "bs256": (256, 128),  # configs[4], per GPU
}
BATCH_AUDIO = (50, 400)   # prefix audio vectors ~ U[50, 400], plus 8 prompt ids
BATCH_CAPACITY = 544      # 400 + 8 + 128 decode positions, rounded up
SEED = 1234


def model_path(quantized: bool) -> Path:
    d = Path(os.environ.get("FUNASR_BENCH_DIR", "/tmp"))
    return d / f"funasrnet_b200_synth_{'q8' if quantized else 'f32'}_{SEED}.gguf"


def ensure_model(quantized: bool, rank: int, barrier, writer=None) -> Path:
    """The seeded synthetic model file.  `writer(path)` makes it; the default is
    the product library's generator, and the CPU reference arm passes the
    oracle's (which writes the same bytes), so that arm never loads the product."""
    p = model_path(quantized)
    if rank == 0 and not p.exists():
        tmp = p.with_suffix(f".tmp{os.getpid()}")
        if writer is None:
            from funasrnet_b200._lib import check, lib

            check(lib().fa_synth_write_gguf(str(tmp).encode(), SEED, 0, 0, 0, 0, 1 if quantized else 0))
        else:
            writer(tmp)
        tmp.replace(p)
    barrier()
    return p


def product_normals(seed: int, stream: int, n: int):
    from funasrnet_b200._lib import check, lib

    a = np.empty(n, np.float32)
    check(lib().fa_synth_normals(seed, stream, 0, n, a.ctypes.data))
    return a


def prefix(width: int, audio: int, ids: int, vocab: int, embed, seed: int = SEED, normals=product_normals):
    """[audio][prompt] embeddings: N(0,1) audio vectors then Embed(ids)."""
    a = normals(seed, 9001, audio * width)
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, vocab, ids).astype(np.int32)
    return np.concatenate([a, embed(toks)]), audio + ids


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def oracle_normals(seed: int, stream: int, n: int):
    from oracle import oracle as O

    return O.synth_normals(seed, stream, 0, n)


def oracle_decode(path: Path, cfg, steps: int, warmup: int, threads: int):
    """CPU restatement of the reference decoder on this host: prefill (untimed),
    `warmup` greedy steps, then `steps` timed greedy steps.  Returns
    (tokens/s, seconds, the emitted tokens: the prefill's argmax first)."""
    from oracle import oracle as O

    O.build()
    O.set_threads(threads)
    audio, ids, _, _ = cfg
    m = O.Model(path, 2048)
    s = O.Session(m)
    emb, frames = prefix(m.width, audio, ids, m.vocab, m.embed, normals=oracle_normals)
    lg = s.decode(emb, frames)
    tok = O.greedy(lg)
    toks = [tok]
    for _ in range(warmup):
        tok = O.greedy(s.decode(m.embed([tok]), 1))
        toks.append(tok)
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = O.greedy(s.decode(m.embed([tok]), 1))
        toks.append(tok)
    dt = time.perf_counter() - t0
    s.close()
    m.close()
    return steps / dt, dt, toks


def source_digest() -> str:
    """sha256 (16 hex digits) of the persistent kernel's source: the build a
    recorded DRAM traffic figure belongs to."""
    import hashlib

    return hashlib.sha256((ROOT / "funasrnet_b200" / "csrc" / "mega.cu").read_bytes()).hexdigest()[:16]


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the persistent
# kernel on the bs1_400 workload, from one `ncu` capture of the bench's first
# 3-step launch (positions 408..410): 2,042,230,528 + 4,323,328 bytes, 682.18 MB
# per step against 680.52 MB algorithmic, keyed by the digest of mega.cu it was
# captured on.  The bench reports traffic = that ratio x its own algorithmic
# bytes per step (the KV share grows with the position in proportion); when the
# source differs it reports null (not measured on this build).
MEASURED_TRAFFIC = {"bs1_400": {"traffic_over_algorithmic": 682.185e6 / 680.519e6,
                                "mega_cu_sha256_16": "d9e9182465d6a733", "captured": "2026-12-02"}}


def profile_range(on: bool):
    """cudaProfilerStart/Stop around the timed region, for `ncu --profile-from-start off`."""
    if not on:
        return contextlib.nullcontext()
    import torch

    return torch.cuda.profiler.profile()


def batch_bench(be, path, name, steps, warmup, rank, world, dist, local, barrier, sessions=None, profile=False):
    """Config 4/5: `n` ragged sessions decoded together.  Returns the result dict
    (rank 0's view; device times are max over ranks)."""
    from funasrnet_b200.decoder import BatchDecoder, CudaModel, QwenDecoder
    from funasrnet_b200.shard import max_over_ranks

    n, tokens = BATCH_CONFIGS[name]
    n = sessions or n
    steps = min(steps, tokens)
    cm = CudaModel(be, path, capacity=BATCH_CAPACITY)
    rng = np.random.default_rng(SEED + 17 * (rank + 1))
    audio = rng.integers(BATCH_AUDIO[0], BATCH_AUDIO[1] + 1, n)
    sessions = [QwenDecoder(cm) for _ in range(n)]
    prefixes = [prefix(cm.width, int(audio[i]), 8, cm.vocab, sessions[0].embed, seed=SEED + 1000 * rank + i)
                for i in range(n)]

    def prefill_all():
        for d, (emb, frames) in zip(sessions, prefixes):
            d.reset()
            d.decode(emb, frames, want_logits=False)

    b = BatchDecoder(sessions)
    try:
        prefill_all()
        b.generate(warmup)  # graph capture + warm-up (untimed)
        prefill_all()
        pos0 = np.array([d.position for d in sessions], np.float64)
        barrier()
        with ClockSampler(local) as clocks, profile_range(profile):
            toks = b.generate(steps)
        dev_ms = max_over_ranks(b.last_ms(), dist, f"cuda:{local}")
        assert toks.shape == (steps, n)
        # e2e: the public per-step call with host buffers (n token ids in, n out)
        prefill_all()
        nxt, _ = b.step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps - 1):
            nxt, _ = b.step(nxt)
        e2e_s = max_over_ranks(time.perf_counter() - t0, dist, f"cuda:{local}")
    finally:
        b.close()
        for d in sessions:
            d.close()
    # algorithmic bytes per step: every weight once + each session's K/V rows
    # [0, pos] + its embedding row
    kv_per_pos = cm.layers * 2 * cm.kv_heads * cm.head_size * 2
    mean_pos_sum = float(np.sum(pos0 + (steps - 1) / 2.0 + 1.0))
    step_bytes = cm.weight_bytes + n * 1088 + kv_per_pos * mean_pos_sum
    ms_per_step = dev_ms / steps
    peak, peak_kind = measured_peak_hbm()
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
    cm.close()
    return {
        "metric": f"decode tokens/sec (Qwen3-0.6B Q8_0 {name})",
        "value": world * n * steps / (dev_ms * 1e-3),
        "unit": "tokens/s",
        "ms_per_step": ms_per_step,
        "sessions_per_gpu": n,
        "steps": steps,
        "config": {"workload": f"qwen3-0.6b-q8_0 {n} sessions/GPU, prefix U[{BATCH_AUDIO[0]},{BATCH_AUDIO[1]}]+8, "
                               f"greedy {tokens} each",
                   "mean_prefix": float(pos0.mean()), "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: 0.63 GB of weights + per-session KV every step"},
        "e2e": {"value": world * n * (steps - 1) / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4 * n,
                "d2h_bytes_per_step": 4 * n},
        "roofline": {"bound": "hbm", "kernel": "batched decode step (CUDA graph: tcgen05 projections + attention)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "bytes_per_step": step_bytes, "peak_source": peak_kind, "traffic": None},
        "clocks": clocks.summary(),
    }


PHASES = (  # (name, (CTA set, event) at the phase's end, (CTA set, event) at its start); -1: previous layer
    ("x -> Q inputs gathered", ("g", 0), ("g", -1)),
    ("Q norm + quantise", ("g", 1), ("g", 0)),
    ("Q/K/V GEMV", ("g", 3), ("g", 1)),
    ("q/k/v hand-off", ("a", 1), ("g", 3)),
    ("score assist (GEMV CTAs)", ("g", 5), ("g", 3)),
    ("attn QK-norm, RoPE, KV write", ("a", 2), ("a", 1)),
    ("attn scores", ("a", 3), ("a", 2)),
    ("attn softmax", ("a", 4), ("a", 3)),
    ("attn V sums + publish", ("a", 5), ("a", 4)),
    ("attention -> O hand-off", ("g", 4), ("a", 5)),
    ("O GEMV + residual", ("g", 7), ("g", 4)),
    ("a -> gate/up hand-off", ("g", 8), ("g", 7)),
    ("gate/up norm + quantise", ("g", 9), ("g", 8)),
    ("gate/up GEMV + SiLU", ("g", 11), ("g", 9)),
    ("SiLU -> down hand-off", ("g", 12), ("g", 11)),
    ("down GEMV + residual", ("g", 15), ("g", 12)),
    ("layer", ("g", 15), ("g", -1)),
)


def phase_table(be, path, reps=5, steps=4):
    """Per-phase critical path of the persistent decode kernel at positions
    408.. (config 2), from `fa_session_set_trace`'s %globaltimer stamps of each
    launch's first step: for every layer after the first, the latest CTA's
    stamp at a phase's end minus the latest stamp at its start.  Prints the
    median and 90th percentile over layers and repetitions."""
    from funasrnet_b200.decoder import CudaModel, QwenDecoder

    audio, ids, _, _ = CONFIGS["bs1_400"]
    cm = CudaModel(be, path, capacity=2048)
    dec = QwenDecoder(cm)
    att_ctas = cm.heads
    emb, frames = prefix(cm.width, audio, ids, cm.vocab, dec.embed)
    rows, plain, cyc, gcyc = [], [], [], []
    for rep in range(reps + 1):
        dec.reset()
        dec.decode(emb, frames, want_logits=False)
        dec.generate(steps, end_ids=())
        plain.append(dec.last_generate_ms() / steps * 1000.0)
        dec.reset()
        dec.decode(emb, frames, want_logits=False)
        dec.trace_phases(True)
        dec.generate(steps, end_ids=())
        raw = dec.phase_trace().astype(np.uint64)
        tr = raw.astype(np.float64)
        dec.trace_phases(False)
        if rep == 0:
            continue  # warm-up
        sets = {"a": tr[:att_ctas], "g": tr[att_ctas:]}

        def latest(which, event):
            v = sets[which][:, event]
            v = v[v > 0]
            return v.max() if v.size else np.nan

        for layer in range(1, cm.layers):
            b, pb = 16 * layer, 16 * (layer - 1)
            r = {}
            for name, (ew, ee), (sw, se) in PHASES:
                start = latest(sw, pb + 15) if se == -1 else latest(sw, b + se)
                r[name] = latest(ew, b + ee) - start
            rows.append(r)
            cyc.append(sets["a"][:, b + 6:b + 10])
            g = sets["g"]
            w = g[:, [b + 2, b + 6, b + 10, b + 14]]
            span = g[:, [b + 3, b + 7, b + 11, b + 15]] - g[:, [b + 1, b + 4, b + 9, b + 12]]
            busy = (w > 0) & (span > 0)  # CTAs with rows in the phase
            gcyc.append(np.where(busy, w, np.nan))
            gcyc.append(np.where(busy, span, np.nan))
    print(f"decode_mega_kernel phase trace: Qwen3-0.6B Q8_0, prefix {audio + ids}, first step of {reps} launches; "
          f"untraced {np.median(plain[1:]):.1f} us/step")
    print(f"{'phase (per layer, layers 1..27)':34s} {'median ns':>10s} {'p90 ns':>8s}")
    for name, _, _ in PHASES:
        v = np.array([r[name] for r in rows])
        print(f"{name:34s} {np.nanmedian(v):10.0f} {np.nanpercentile(v, 90):8.0f}")
    c = np.concatenate(cyc)  # [layers x attention CTAs, 4] SM cycles
    print(f"{'attention CTA, SM cycles per layer':34s} {'median':>10s} {'p90':>8s}")
    for k, name in enumerate(("waiting for assisted scores", "waiting for V chunks", "scores gathered", "V loop")):
        print(f"{name:34s} {np.median(c[:, k]):10.0f} {np.percentile(c[:, k], 90):8.0f}")
    gw, gc = np.concatenate(gcyc[0::2]), np.concatenate(gcyc[1::2])  # [layers x GEMV CTAs, 4 phases]
    print(f"{'GEMV CTA, per layer':34s} {'median':>10s} {'p90':>8s}")
    for k, ph in enumerate(("Q/K/V", "O", "gate/up", "down")):
        print(f"{ph + ' weight wait, SM cycles':34s} {np.nanmedian(gw[:, k]):10.0f} {np.nanpercentile(gw[:, k], 90):8.0f}")
        print(f"{ph + ' phase of this CTA, ns':34s} {np.nanmedian(gc[:, k]):10.0f} {np.nanpercentile(gc[:, k], 90):8.0f}")
    dec.close()
    cm.close()


def fp32_bench(be, warmup, world, dist, local, barrier, peak, peak_kind):
    """Config 3 (FP32 weights, prefix 100+8, greedy 128) on one GPU: the CUDA
    graph step with the FP32 GEMV, timed over all 128 decode steps."""
    from funasrnet_b200.decoder import CudaModel, QwenDecoder
    from funasrnet_b200.shard import max_over_ranks

    audio, ids, tokens, _ = CONFIGS["fp32"]
    path = ensure_model(False, int(os.environ.get("RANK", "0")), barrier)
    cm = CudaModel(be, path, capacity=2048)
    dec = QwenDecoder(cm)
    emb, frames = prefix(cm.width, audio, ids, cm.vocab, dec.embed)
    try:
        dec.reset()
        dec.decode(emb, frames, want_logits=False)
        dec.generate(warmup, end_ids=())
        dec.reset()
        dec.decode(emb, frames, want_logits=False)
        barrier()
        with ClockSampler(local) as clocks:
            toks = dec.generate(tokens, end_ids=())
        assert len(toks) == tokens
        dev_ms = max_over_ranks(dec.last_generate_ms(), dist, f"cuda:{local}")
        dec.reset()
        _, tok = dec.decode(emb, frames, want_logits=False)
        barrier()
        t0 = time.perf_counter()
        for _ in range(tokens):
            tok, _ = dec.step(tok)
        e2e_s = max_over_ranks(time.perf_counter() - t0, dist, f"cuda:{local}")
        kernels = dec.kernels_per_step()
    finally:
        dec.close()
    kv_per_pos = cm.layers * 2 * cm.kv_heads * cm.head_size * 2
    step_bytes = cm.weight_bytes + cm.width * 4 + kv_per_pos * (frames + (tokens - 1) / 2.0 + 1)
    ms = dev_ms / tokens
    achieved = step_bytes / (ms * 1e-3) / 1e9
    cm.close()
    return {"metric": "decode tokens/sec (Qwen3-0.6B FP32 bs1)", "value": world * tokens / (dev_ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": tokens, "dtype": "f32",
            "workload": f"qwen3-0.6b-f32 bs1 prefix {audio}+{ids}, greedy {tokens} (BASELINE configs[2])",
            "e2e": {"value": world * tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "kernel": f"decode step (CUDA graph of {kernels} kernels, FP32 GEMV)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "bytes_per_step": step_bytes, "peak_source": peak_kind, "traffic": None},
            "gpu_launches": kernels * tokens, "clocks": clocks.summary()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--config", choices=sorted(CONFIGS) + sorted(BATCH_CONFIGS), default="bs1_400")
    ap.add_argument("--no-batched", action="store_true", help="skip the bs64/bs256 lines of the default run")
    ap.add_argument("--sessions", type=int, default=None, help="batched configs: sessions per GPU (profiling runs)")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed region with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    ap.add_argument("--cpu-baseline-steps", type=int, default=256,
                    help="greedy decode steps of the CPU restatement on all host threads (a third of them on 4); "
                         "its tokens are also compared with the GPU's")
    ap.add_argument("--no-fp32", action="store_true", help="skip the FP32 (config 3) entry of the default run")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--phase-trace", action="store_true",
                    help="print the persistent kernel's per-phase table (config 2, one GPU) instead of the JSON line")
    args = ap.parse_args()
    batched = args.config in BATCH_CONFIGS
    cfg = CONFIGS["bs1_400" if batched else args.config]
    audio, ids, tokens, quantized = cfg
    steps = min(args.steps, tokens)
    warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1 and args.impl != "reference":  # the CPU reference arm needs no process group
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist is not None:
            dist.barrier()

    config = {"workload": f"qwen3-0.6b-{'q8_0' if quantized else 'f32'} bs1 prefix {audio}+{ids}, greedy {tokens}",
              "batch_per_gpu": 1, "prefix": audio + ids, "decode_tokens": tokens,
              "timed_positions": [audio + ids, audio + ids + steps], "parallelism": f"replicas x{args.gpus}",
              "l2": "inputs larger than L2: every step streams the full 0.63 GB weight set"}
    metric = "decode tokens/sec (Qwen3-0.6B Q8_0 bs1)" if quantized else "decode tokens/sec (Qwen3-0.6B FP32 bs1)"

    if args.impl == "reference":
        # The reference is C# (.NET 10); no dotnet here, so its CPU decoder is
        # timed through the C++ restatement on all host threads (rank 0 only).
        if rank == 0:
            from oracle import oracle as O

            path = ensure_model(quantized, 0, lambda: None,
                                writer=lambda p: O.synth_write_gguf(p, SEED, quantized=quantized))
            threads = os.cpu_count() or 1
            rate, dt, _ = oracle_decode(path, cfg, steps, warmup, threads)
            line = {"metric": metric, "value": rate, "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
                    "warmup": warmup, "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "int8 x int8 -> int32, f32 accumulate", "data": "synthetic",
                    "config": config, "impl": "reference",
                    "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                                     "sample": f"{steps} decode steps after the {audio + ids}-frame prefill"},
                    "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return  # under torchrun the other ranks leave without work

    from funasrnet_b200.backend import CudaFloatBackend
    from funasrnet_b200.decoder import CudaModel, QwenDecoder
    from funasrnet_b200.shard import max_over_ranks

    path = ensure_model(quantized, rank, barrier)
    be = CudaFloatBackend(local)
    if args.phase_trace:
        phase_table(be, path)
        be.dispose()
        return
    if batched:
        r = batch_bench(be, path, args.config, args.steps, warmup, rank, world, dist, local, barrier,
                        sessions=args.sessions, profile=args.profile_range)
        line = {"metric": r["metric"], "value": r["value"], "unit": "tokens/s", "n_gpus": world,
                "steps": r["steps"], "warmup": warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 (tcgen05), f32 accumulate",
                "data": "synthetic (seeded random-init weights and prefixes)", "config": r["config"],
                "e2e": r["e2e"], "roofline": r["roofline"], "gpu_launches": None, "clocks": r["clocks"]}
        if rank == 0:
            print(json.dumps(line), flush=True)
        be.dispose()
        if dist is not None:
            dist.destroy_process_group()
        return
    cm = CudaModel(be, path, capacity=2048)
    dec = QwenDecoder(cm)
    emb, frames = prefix(cm.width, audio, ids, cm.vocab, dec.embed)

    # warm-up (untimed): prefill + W decode steps, graph capture included
    dec.reset()
    dec.decode(emb, frames, want_logits=False)
    dec.generate(warmup, end_ids=())
    # timed: fresh prefill (untimed), then K steps through the on-device loop
    dec.reset()
    _, first_tok = dec.decode(emb, frames, want_logits=False)
    barrier()
    with ClockSampler(local) as clocks, profile_range(args.profile_range):
        toks = dec.generate(steps, end_ids=())
    dev_ms = dec.last_generate_ms()
    assert len(toks) == steps
    dev_ms = max_over_ranks(dev_ms, dist, f"cuda:{local}")

    # e2e: the same K steps through the public per-token API with host buffers
    # (FunAsr.Transcribe's loop: the token id to the device, the next token id
    # back, each step), in resident serving: each call posts its token to the
    # running persistent launch through mapped pinned memory.
    dec.reset()
    _, tok = dec.decode(emb, frames, want_logits=False)
    resident = dec.set_resident(True)
    for _ in range(3):  # warm-up of the resident launch, then a fresh prefix
        tok, _ = dec.step(tok)
    dec.reset()
    _, tok = dec.decode(emb, frames, want_logits=False)
    barrier()
    t0 = time.perf_counter()
    e2e_toks = []
    for _ in range(steps):
        tok, _ = dec.step(tok)
        e2e_toks.append(tok)
    e2e_s = time.perf_counter() - t0
    dec.set_resident(False)
    e2e_s = max_over_ranks(e2e_s, dist, f"cuda:{local}")
    assert e2e_toks == list(toks[1:]) + [e2e_toks[-1]], "per-token steps differ from the on-device loop"

    # prefill, timed apart as the reference's PrefillSeconds (FunAsr.cs:24-34):
    # one Decode of the whole prefix through the public API, embeddings from
    # host memory; median of three (the warm-up above ran it once)
    pre = []
    for _ in range(3):
        dec.reset()
        t0 = time.perf_counter()
        dec.decode(emb, frames, want_logits=False)
        pre.append(time.perf_counter() - t0)
    prefill_s = max_over_ranks(sorted(pre)[1], dist, f"cuda:{local}")

    # roofline of the decode step and of its largest single launch (lm_head GEMV)
    peak, peak_kind = measured_peak_hbm()
    rec = MEASURED_TRAFFIC.get(args.config) if dec.persistent_grid() else None
    traffic = None
    kv_bytes_per_pos = cm.layers * 2 * cm.kv_heads * cm.head_size * 2
    mean_pos = frames + (steps - 1) / 2.0
    step_bytes = cm.weight_bytes + 1088 + kv_bytes_per_pos * (mean_pos + 1)
    if rec and rec["mega_cu_sha256_16"] == source_digest():
        traffic = rec["traffic_over_algorithmic"] * step_bytes
    ms_per_step = dev_ms / steps
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
    lm_ms = dec.time_lm_head(20) if quantized else None
    lm_bytes = cm.vocab * cm.width // 32 * 34 + cm.width * 4 * 2

    grid = dec.persistent_grid()
    kernel_name = (f"decode_mega_kernel (persistent, {grid} CTAs, one launch for all {steps} steps)" if grid
                   else "decode step (CUDA graph)")
    launches = 1 if grid else dec.kernels_per_step() * steps
    line = {
        "metric": metric,
        "value": world * steps / (dev_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 x int8 -> int32, f32 accumulate" if quantized else "f32",
        "data": "synthetic (seeded random-init weights and prefix; no model or audio files exist here)",
        "config": config,
        "e2e": {"value": world * steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4,
                "path": "fa_session_step per token" + (", resident serving (mapped-memory mailbox)" if resident else "")},
        "roofline": {"bound": "hbm", "kernel": kernel_name, "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "traffic_unit": "DRAM bytes per decode step: the ncu-measured traffic/algorithmic ratio of this "
                                     "source (positions 408..410) times the step's algorithmic bytes; null when "
                                     "the kernel source differs from the captured one",
                     "traffic_source": {"mega_cu_sha256_16": source_digest(),
                                        "captured_on": rec["mega_cu_sha256_16"] if rec else None,
                                        "date": rec["captured"] if rec else None},
                     "bytes_per_step": step_bytes, "peak_source": peak_kind},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    line["prefill"] = {"frames": frames, "ms": prefill_s * 1e3, "frames_per_s": frames / prefill_s,
                       "h2d_bytes": frames * cm.width * 4,
                       "path": "fa_session_decode: chunks of up to 512 frames (projections on the tcgen05 kernel, one weight pass per chunk), attention in launches of up to 512 frames"}
    if lm_ms:
        a = lm_bytes / (lm_ms * 1e-3) / 1e9
        line["gemv_lm_head"] = {"ms": lm_ms, "bytes": lm_bytes, "achieved": a, "frac": a / peak}
    dec.close()
    cm.close()
    if args.config == "bs1_400" and not args.no_batched:
        line["batched"] = {}
        for name in ("bs64", "bs256"):
            r = batch_bench(be, path, name, 128, warmup, rank, world, dist, local, barrier)
            line["batched"][name] = {k: r[k] for k in ("value", "ms_per_step", "sessions_per_gpu", "steps", "e2e",
                                                       "roofline", "clocks")}
            line["batched"][name]["workload"] = r["config"]["workload"]
    if args.config == "bs1_400" and not args.no_fp32:
        line["fp32"] = fp32_bench(be, warmup, world, dist, local, barrier, peak, peak_kind)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, dt, otoks = oracle_decode(path, cfg, args.cpu_baseline_steps, 2, threads)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{args.cpu_baseline_steps} decode steps after the {frames}-frame prefill "
                                          f"({dt:.1f} s of CPU decode)"}
        # the reference's published CPU setup runs 4 threads
        rate4, dt4, _ = oracle_decode(path, cfg, max(4, args.cpu_baseline_steps // 3), 1, 4)
        line["cpu_baseline_4_threads"] = {"value": rate4, "unit": "tokens/s", "cores": 4, "kind": "port",
                                          "sample": f"{max(4, args.cpu_baseline_steps // 3)} decode steps after the "
                                                    f"{frames}-frame prefill ({dt4:.1f} s)"}
        # the timed GPU tokens against the oracle's greedy tokens from the same prefix
        gpu = list(toks)  # generate emits the prefill's argmax first
        assert gpu[0] == first_tok
        n = min(len(gpu), len(otoks))
        line["tokens_match_oracle"] = {"compared": n, "equal": gpu[:n] == otoks[:n]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    be.dispose()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
