#!/usr/bin/env python
"""Benchmark of the per-token scoring path: tokens/s scored by the Gemma-3-270M-geometry Q8_0 model
with the two-level head (2048 classes x 128 tokens), batch 1, 512 sequential random tokens per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--numerics exact|fast]

One step scores one 512-token sequence (gem bench's loop, crates/gem/src/main.rs:270-289) through the
library's device-buffer entry point; `e2e` runs the same steps through the host-buffer entry point
(token ids copied in, log-probs and argmax copied out, every step). Under torchrun each rank scores
its own sequence on its own GPU (weak scaling, no collective on the data path); the timed region is
bracketed by barriers and the time is the max over ranks. `parity` compares rank 0's last timed
step with one untimed oracle pass of the same sequence.

Secondary legs, at every N (all ranks take part, times are the max over ranks):
  batched      256 sequences x 512 positions split over the ranks (strong scaling: fixed total)
  vocab_shard  Gemma-3-1B geometry, 1024 positions, the full head's vocabulary sharded over the ranks
               with an NCCL all-gather of per-shard statistics; checked on the box against the
               unsharded head; time in the all-gather + merge reported beside the head shard's
and at N = 1 only: the per-token schedules, the full head, the QAT layout (Q4_0 body, F16 head and
its Q8_0 requantization), the head microbenchmark and the CPU baseline.

`--impl reference` times the oracle (the CPU restatement of gem's scoring path; the reference is Rust
and no Rust toolchain exists here) on the host cores. Prints one JSON line from rank 0.
"""
from __future__ import annotations

import argparse
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
sys.path.insert(0, str(ROOT / "prefix-head_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "tokens/s scored (270M Q8_0, 2-level head) b1+batched; head GEMV HBM GB/s"
SEQ_TOKENS = 512
REF_THREADS = 8  # the pool size exact numerics reproduce (gem bench's default, main.rs:197)
BATCH_SEQS = 256
SHARD_TOKENS = 1024
CTX = 2048  # gem bench's context (main.rs:204)
CLASSES = 2048
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
# The reference's published figure for this metric and workload: gem bench, Gemma 3 270M Q8_0, two-level
# head 2048 x 128, 512 tokens, batch 1, AVX-512, 8 threads on a Ryzen 7 7700 (results/gem-bench.jsonl
# rows 26, 28, 30: 310.2, 304.5, 311.1 tokens/s).
PUBLISHED = {"value": round((310.2 + 304.5 + 311.1) / 3, 1), "unit": "tokens/s",
             "source": "results/gem-bench.jsonl:26,28,30 (gem bench, 270M Q8_0, two-level 2048 x 128, "
                       "AVX-512, 8 threads, Ryzen 7 7700; mean of 3)"}


def vs_published(value):
    return round(value / PUBLISHED["value"], 2)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--numerics", default="exact", choices=["exact", "fast"])
    p.add_argument("--no-extras", action="store_true", help="skip the full-head / head-microbench / CPU legs")
    p.add_argument("--cpu-threads", type=int, default=0, help="oracle threads for the CPU legs (0 = all cores)")
    p.add_argument("--workload", default="270m-two-level", choices=["270m-two-level", "1b-vocab-shard"],
                   help="1b-vocab-shard: Gemma-3-1B geometry, 1024 positions, full head sharded over the ranks")
    return p.parse_args()


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def hbm_peak():
    p = peaks()
    if "hbm_gbs" in p:
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """SM clock and throttle-reason samples while the timed region runs (reading only; nothing here
    changes a clock or a setting). NVML is polled every 5 ms from a thread, because the default run's
    timed region lasts ~0.1 s; where NVML cannot be opened, nvidia-smi's own loop (-lms 50) samples
    the same fields. `nvml` replaces the pynvml module (a fake in the CPU tests)."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    # NVML clocks-event reason bits (nvmlClocksEventReason*), named as nvidia-smi names the fields
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    PERIOD_S = 0.005

    def __init__(self, device: int, nvml=None):
        self.device = device
        self.nvml = nvml
        self.N = None
        self.samples = []  # NVML: (sm MHz, max sm MHz, reason bits)
        self.stop = threading.Event()
        self.t = None
        self.proc = None
        self.lines = []

    def _nvml_handle(self, N):
        try:  # the CUDA ordinal and the NVML index need not agree: match by UUID
            import torch
            u = str(torch.cuda.get_device_properties(self.device).uuid)
            return N.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:
            return N.nvmlDeviceGetHandleByIndex(self.device)

    def _poll(self, h, mx):
        N = self.N
        try:
            while not self.stop.is_set():
                self.samples.append((float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)), mx,
                                     int(N.nvmlDeviceGetCurrentClocksEventReasons(h))))
                self.stop.wait(self.PERIOD_S)
        except Exception:
            pass

    def __enter__(self):
        try:
            N = self.nvml
            if N is None:
                import pynvml as N
            N.nvmlInit()
            self.N = N
            h = self._nvml_handle(N)
            mx = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, args=(h, mx), daemon=True)
            self.t.start()
            while not self.samples and self.t.is_alive():  # the timed region starts once a sample is in
                time.sleep(0.001)
            return self
        except Exception:
            self._close_nvml()
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()  # the timed region starts once the sampler is running
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.lines.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def _close_nvml(self):
        if self.t:
            self.stop.set()
            self.t.join(timeout=5)
        if self.N:
            try:
                self.N.nvmlShutdown()
            except Exception:
                pass
            self.N = None

    def __exit__(self, *a):
        self._close_nvml()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        if self.samples:
            for mhz, mx, bits in self.samples:
                sm.append(mhz)
                reasons.update(n for n, b in self.REASON_BITS.items() if bits & b)
            source = "nvml"
        else:
            for ln in self.lines:
                f = [x.strip() for x in ln.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
            source = "nvidia-smi"
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": source}


def model_files():
    from gem_b200 import synth
    return synth.ensure("gemma3-270m", classes=CLASSES)


def bytes_per_token(info, n_pos_per_layer, extra_blocks):
    """Algorithmic HBM bytes of one scored token: every projection once (canonical GGUF sizes), the
    class table and bias, the target class's block (plus the top class's block when it differs), the
    KV rows attention reads and writes, and the small fp32 vectors (norm weights, RoPE rows)."""
    d, nl, hd, nkv, nh = info["d"], info["layers"], info["head_dim"], info["n_kv_heads"], info["n_heads"]
    k, per = info["classes"], info["per"]
    row_bytes = d + d // 32 * 2  # one Q8_0 head row with f16 scales
    kv_read = sum(n_pos_per_layer) * nkv * hd * 4 * 2
    kv_write = nl * nkv * hd * 4 * 2
    vectors = nl * (4 * d + 2 * hd + hd) * 4 + d * 4  # norm weights, q/k-norm weights, one RoPE sin/cos row
    return info["body_bytes"] + k * d * 4 + k * 4 + (1 + extra_blocks) * per * row_bytes + kv_read + kv_write + vectors


def n_pos_schedule(info, n_tokens):
    """Average number of KV positions attention reads per layer over the sequence."""
    w, nl = info["window"], info["layers"]
    tot = np.zeros(nl)
    for pos in range(n_tokens):
        for l in range(nl):
            swa = l % 6 < 5
            tot[l] += min(pos + 1, w) if swa and w > 0 else pos + 1
    return tot / n_tokens


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def gem_bench_fields(m, threads, seconds, body_s, head_s, steps):
    """The oracle's run in the fields of gem bench's JSONL record (crates/gem/src/main.rs:295-310):
    tokens/s, body and head microseconds per token, the head's share, threads, ISA; plus the CPU."""
    n = SEQ_TOKENS * steps
    return {"tok_per_s": round(n / seconds, 1), "body_us": round(body_s / n * 1e6, 1),
            "head_us": round(head_s / n * 1e6, 1), "head_share": round(head_s / max(1e-12, body_s + head_s), 3),
            "threads": threads, "isa": m.isa, "tokens": SEQ_TOKENS, "cpu": cpu_model()}


def run_reference(args):
    """Times the oracle (the CPU restatement of the reference's scoring path) on all host cores."""
    from gem_b200 import synth
    from oracle import oracle as orc
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    mf = model_files()
    threads = args.cpu_threads or os.cpu_count() or 1
    m = orc.Model(mf.gguf, ctx=CTX, threads=threads)
    m.load_twolevel(mf.twolevel)
    toks = synth.tokens(SEQ_TOKENS + 1, m.vocab, seed=1000)
    for _ in range(args.warmup):
        m.score(toks, 1)
    times, body_s, head_s = [], 0.0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _, _, tb, th = m.score(toks, 1)
        times.append(time.perf_counter() - t0)
        body_s, head_s = body_s + tb, head_s + th
    per_step = sum(times) / len(times)
    value = SEQ_TOKENS / per_step
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": vs_published(value), "published_baseline": PUBLISHED,
        "dtype": "int8 x int8 -> f32 (Q8_0)", "data": "synthetic",
        "config": {"workload": "gemma3-270m Q8_0, two-level head 2048x128, batch 1, 512 random tokens per step",
                   "geometry": "gemma3-270m (d 640, 18 layers, 4q/1kv heads, hd 256, ff 2048, vocab 262144), "
                               "random init N(0,0.02) quantized to Q8_0", "global_batch": 1, "seq_len": SEQ_TOKENS,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "isa": m.isa, "sample": f"{args.steps} x {SEQ_TOKENS}-token sequences",
                         "gem_bench": gem_bench_fields(m, threads, sum(times), body_s, head_s, args.steps)},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_vocab_shard(args):
    """--workload 1b-vocab-shard: the C5 leg (run_vocab_shard_leg) alone, as the headline line."""
    import datetime

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    with Clocks(local) as clk:
        r = run_vocab_shard_leg(torch, dist, world, rank, local, flush, args)
    if rank == 0:
        line = {
            "metric": "tokens/s scored (1B Q8_0, full head vocab-sharded across GPUs)", "value": r["value"],
            "unit": "tokens/s", "n_gpus": world, "steps": max(1, min(args.steps, 10)), "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x int8 -> f32 (Q8_0)", "data": "synthetic", "numerics": "exact",
            "config": {"workload": r["workload"], "global_batch": 1, "seq_len": SHARD_TOKENS,
                       "parallelism": f"vocab shard x{world} (body replicated)", "rows_per_rank": r["rows_per_rank"],
                       "l2": r["l2"]},
            "check_vs_unsharded": r["check_vs_unsharded"], "head_us_per_step": r["head_us_per_step"],
            "two_level_unsharded": r["two_level_unsharded"],
            "gpu_launches": int(r["gpu_launches_per_step"] * max(1, min(args.steps, 10))), "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "1b-vocab-shard":
        return run_vocab_shard(args)
    import torch
    import torch.distributed as dist
    from gem_b200 import EXACT, FAST, FULL, PARALLEL, TWO_LEVEL, Gemma, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    def barrier():
        if world > 1:
            dist.barrier()
    if rank == 0:
        mf = model_files()
    barrier()
    if rank != 0:
        mf = model_files()

    g = Gemma(mf.gguf, ctx=CTX, device=local)
    g.load_twolevel(mf.twolevel)
    g.set_numerics(EXACT if args.numerics == "exact" else FAST)
    info = g.refresh_info()
    stream = torch.cuda.ExternalStream(g.stream, device=local)
    toks_h = synth.tokens(SEQ_TOKENS + 1, g.vocab, seed=1000 + rank)
    toks_d = torch.tensor(toks_h.astype(np.int32), device="cuda")
    lp_d = torch.empty(SEQ_TOKENS, device="cuda")
    am_d = torch.empty(SEQ_TOKENS, dtype=torch.int32, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def step(head=TWO_LEVEL):
        g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, head, lp_d.data_ptr(), am_d.data_ptr())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    g.sync()

    # ---- timed region: K steps, device time with events on the model's stream, L2 flushed between ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        for a, b in evs:
            flush.zero_()
            torch.cuda.synchronize()
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize()
        g.sync()
    barrier()
    ms = sum(a.elapsed_time(b) for a, b in evs)
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = SEQ_TOKENS * args.steps * world
    value = tokens / (ms_max / 1e3)
    info = g.refresh_info()
    kind, kind_why = g.schedule_kind(TWO_LEVEL)
    launches_per_step = g.last_launches()
    am_h = am_d.cpu().numpy().astype(np.uint32)
    lp_h = lp_d.cpu().numpy()
    clocks = clk.summary()
    if kind == PARALLEL:
        roofline, sched = parallel_roofline(g, torch, step, info, ms_max / args.steps, clocks, args,
                                            token_bytes(g, info, mf, am_h, toks_h))
    else:
        roofline, sched = token_roofline(g, info, mf, am_h, toks_h, ms_max / args.steps, args, kind)
    # ---- e2e: the host-buffer entry point (H2D token ids, D2H log-probs + argmax every step) ----
    # its own untimed warm-up: a repeated call is captured once as a CUDA graph, then replayed
    for _ in range(args.warmup):
        g.score(toks_h, TWO_LEVEL)
    barrier()
    torch.cuda.synchronize()
    wall = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        g.score(toks_h, TWO_LEVEL)
        wall.append(time.perf_counter() - t0)
    barrier()
    tw = torch.tensor([sum(wall)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tw, op=dist.ReduceOp.MAX)
    e2e_value = tokens / float(tw.item())

    # ---- parity: rank 0's last timed step against one untimed oracle pass of the same sequence ----
    parity = oracle_parity(mf, toks_h, lp_h, am_h, TWO_LEVEL) if rank == 0 else None

    extras = {}
    if not args.no_extras:
        # every rank takes part: C4 split over the ranks, C5 sharded over them
        extras["batched"] = run_batched(torch, dist, world, rank, local, mf, flush, args)
        extras["vocab_shard"] = run_vocab_shard_leg(torch, dist, world, rank, local, flush, args)
        if world == 1:
            extras.update(run_extras(g, torch, stream, toks_d, lp_d, am_d, flush, args, mf))

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": vs_published(value), "published_baseline": PUBLISHED,
            "dtype": "int8 x int8 -> f32 (Q8_0)", "data": "synthetic",
            "numerics": args.numerics,
            "config": {"workload": "gemma3-270m Q8_0, two-level head 2048x128, batch 1, 512 random tokens per step",
                       "geometry": "gemma3-270m (d 640, 18 layers, 4q/1kv heads, hd 256, ff 2048, vocab 262144), "
                                "random init N(0,0.02) quantized to Q8_0",
                       "global_batch": world, "seq_len": SEQ_TOKENS, "parallelism": f"dp{world} (one sequence per GPU)",
                       "l2": "flushed (256 MiB write) before every step"},
            "schedule": sched,
            "roofline": roofline,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": (SEQ_TOKENS + 1) * 4,
                    "d2h_bytes_per_step": SEQ_TOKENS * 8},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clocks,
            "parity": parity,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    g.close()
    if world > 1:
        dist.destroy_process_group()


def body_weights(info):
    d, nl, nh, nkv, hd, ff = (info[k] for k in ("d", "layers", "n_heads", "n_kv_heads", "head_dim", "ffn"))
    return nl * ((nh + 2 * nkv) * hd * d + d * nh * hd + 2 * ff * d + d * ff)


def gemm_traffic():
    """DRAM bytes per step of the exact matrix products from the committed ncu summary, if present."""
    tf = ROOT / "profiles" / "dram_traffic.txt"
    if tf.exists():
        for ln in tf.read_text().splitlines():
            if ln.startswith("k_seq_gemm per step:"):
                return float(ln.split(":")[1].split()[0])
    return None


def token_bytes(g, info, mf, am_h, toks_h):
    """Algorithmic HBM bytes of one scored token (bytes_per_token), with the second class block counted
    for the positions whose top class is not the target's."""
    order = np.fromfile(str(mf.twolevel) + ".order", dtype="<u4")
    cls_of = np.empty(g.vocab, np.int64)
    cls_of[order] = np.arange(len(order)) // info["per"]
    extra = float(np.mean(cls_of[am_h] != cls_of[toks_h[1:]]))
    return bytes_per_token(info, n_pos_schedule(info, SEQ_TOKENS), extra)


def parallel_roofline(g, torch, step, info, ms_step, clocks, args, bpt):
    """Roofline of the dominant kernel of parallel scoring, the exact int8 matrix product (k_seq_gemm).

    A dense contraction, so its roofline is the tensor-core one (the measured bf16 GEMM peak; int8 has
    no measured figure here). The reference's rounding (one fp32 FMA per 32-block per lane,
    q8.rs:248-292) keeps it on the CUDA cores: tensor-core variants are exact only with each lane pair
    in its own accumulator column, which leaves that FMA on the CUDA cores and measured no faster. Its
    own ceiling, `cuda_core_view`, is the instruction floor at the SM clock: at least three instructions
    per int8 weight pair and position (the pair dot, its exact conversion to fp32, half a packed FMA
    plus the scale), so SMs x 128 lanes x clock / 3 pairs per second, 2 multiply-adds per pair, 2 ops
    each. `per_token_hbm_view` is the batch-1 HBM roofline of scoring (every token's bytes read once
    per token, as a token-by-token schedule must): the parallel schedule reads the weights once per
    step instead, so it can exceed it."""
    g.set_profiling(True)
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    prof = g.parallel_profile()
    g.set_profiling(False)
    gemm_us = prof["qkv"] + prof["o"] + prof["gate_up"] + prof["down"]
    ops = 2.0 * body_weights(info) * SEQ_TOKENS
    achieved = ops / (gemm_us * 1e-6) / 1e12
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    peak = sms * 128 * mhz * 1e6 / 3 * 4 / 1e12
    hbm, hbm_kind = hbm_peak()
    alg_bytes = info["body_bytes"] + info["classes"] * info["d"] * 4
    tensor_peak = peaks().get("bf16_tflops")
    tensor_kind = "measured bf16 dense (burst)"
    if not tensor_peak:
        tensor_peak, tensor_kind = 1590.0, "fallback bf16 dense"
    tok_s = SEQ_TOKENS / (ms_step * 1e-3)
    roof = {"bound": "tensor", "unit": "TFLOP/s", "achieved": round(achieved, 2), "peak": tensor_peak,
            "peak_kind": tensor_kind, "frac": round(achieved / tensor_peak, 4), "traffic": gemm_traffic(),
            "traffic_source": "the committed ncu capture's DRAM bytes per step (profiles/dram_traffic.txt: one "
                              "layer's launches with L2 as the live step leaves it, x layers), not measured "
                              "in this run",
            "kernel": "k_seq_gemm (4 launches per layer and sequence part)", "ops_per_step": ops,
            "note": "exact int8 x int8 -> fp32 products on the CUDA cores (the reference's per-block fp32 "
                    "rounding); the tensor-core peak is the dense-contraction bound, cuda_core_view this "
                    "kernel's instruction ceiling",
            "cuda_core_view": {"unit": "TOP/s", "achieved": round(achieved, 2), "peak": round(peak, 2),
                               "peak_kind": f"derived: {sms} SMs x 128 lanes x {mhz:.0f} MHz / 3 instructions "
                                            "per int8 pair x 4 ops", "frac": round(achieved / peak, 4)},
            "per_token_hbm_view": {"algorithmic_bytes_per_token": int(bpt), "tokens_s": round(tok_s, 1),
                                   "roofline_tokens_s": round(hbm * 1e9 / bpt, 1),
                                   "frac": round(tok_s * bpt / (hbm * 1e9), 4), "peak": hbm, "peak_kind": hbm_kind},
            "kernel_timing": "CUDA events around each launch group of a one-stream pass of the same step "
                             "(profiling runs the sequence as one part; the timed step runs its parts' "
                             "launches concurrently on their streams)",
            "kernel_ms_per_step": round(gemm_us / 1e3, 3),
            "share_of_step": round(gemm_us / max(1e-9, sum(prof.values())), 3),  # of the one-part profiled step
            "hbm_view": {"algorithmic_bytes_per_step": alg_bytes, "achieved_GB_s": round(alg_bytes / (ms_step * 1e-3) / 1e9, 1),
                         "peak": hbm, "peak_kind": hbm_kind},
            }
    sched = {"kind": "sequence-parallel (every position of the sequence through each layer together; the "
                     "sequence in 4 parts of 128 positions on 4 streams, each part one layer behind the one "
                     "before it; a repeated call replays them as one CUDA graph)",
             "groups_us_per_step": prof}
    return roof, sched


def token_roofline(g, info, mf, am_h, toks_h, ms_step, args, kind):
    """HBM roofline of per-token scoring: algorithmic bytes per token / time per token."""
    from gem_b200 import TWO_LEVEL
    bpt = token_bytes(g, info, mf, am_h, toks_h)
    per_token_s = ms_step / 1e3 / SEQ_TOKENS
    peak, peak_kind = hbm_peak()
    achieved = bpt / per_token_s / 1e9
    pipelined, G, GH, why = g.schedule(TWO_LEVEL)
    roof = {"bound": "hbm", "unit": "GB/s", "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "frac": round(achieved / peak, 4), "traffic": None,
            "kernel": "k_pipe_score (one launch per step)" if pipelined else "token step (a CUDA graph per token)",
            "algorithmic_bytes_per_token": int(bpt)}
    sched = ({"kind": "layer-pipelined persistent kernel", "ctas_per_layer": G, "head_ctas": GH} if pipelined
             else {"kind": "CUDA graph per token", "why": why})
    return roof, sched


def time_dev(torch, stream, fn, iters, flush):
    """Mean device time of fn() over `iters` calls, each after an L2 flush (none when `flush` is None:
    for calls whose input is larger than L2). The flush runs on the timed stream itself, so the host
    enqueues each call while the flush is still executing and the start event marks the call's first
    kernel, not the host's launch latency."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for a, b in evs:
            if flush is not None:
                flush.zero_()
            a.record(stream)
            fn()
            b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters


def oracle_parity(mf, toks_h, lp, am, head, ctx=CTX):
    """Compares scored log-probs and argmax ids with one untimed oracle pass of the same sequence (the
    oracle's AVX-512 path with the pool size exact numerics reproduce). Bar: identical argmax ids,
    |d logprob| < 1e-3 nats, the contract tolerance; exact numerics give < 2e-5."""
    from oracle import oracle as orc
    isa = "avx512" if orc.detect_isa() == "avx512" else None
    o = orc.Model(mf.gguf, ctx=ctx, threads=REF_THREADS, isa=isa)
    if mf.twolevel is not None:
        o.load_twolevel(mf.twolevel)
    lpo, amo, _, _ = o.score(np.asarray(toks_h, np.uint32), head)
    used = o.isa
    o.close()
    n = min(len(lpo), len(lp))
    err = float(np.abs(np.asarray(lp[:n], np.float32) - lpo[:n]).max()) if n else 0.0
    same = bool(np.array_equal(np.asarray(am[:n], np.uint32), amo[:n]))
    return {"against": f"oracle ({used}, {REF_THREADS}-thread pool), one untimed pass of the same sequence",
            "positions": int(n), "argmax_equal": same, "argmax_mismatches": int(np.sum(np.asarray(am[:n], np.uint32) != amo[:n])),
            "max_abs_lp": err, "tolerance": 1e-3, "pass": bool(same and err < 1e-3)}


def _max_over_ranks(torch, dist, world, v):
    t = torch.tensor([float(v)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_batched(torch, dist, world, rank, local, mf, flush, args):
    """C4: 256 independent sequences x 512 positions, two-level head, split over the ranks by
    shard.seq_range (strong scaling: the total is fixed); each rank scores its share in groups of 8
    sequences (8 KV slots). Time = max over ranks of the device time of the rank's whole share."""
    from gem_b200 import TWO_LEVEL, Gemma, shard, synth
    first, count = shard.seq_range(BATCH_SEQS, world, rank)
    gb = Gemma(mf.gguf, ctx=CTX, device=local, max_seqs=8)
    gb.load_twolevel(mf.twolevel)
    bstream = torch.cuda.ExternalStream(gb.stream, device=local)
    btoks = np.stack([synth.tokens(SEQ_TOKENS + 1, gb.vocab, seed=2000 + s) for s in range(first, first + count)])
    btd = torch.tensor(btoks.astype(np.int32), device="cuda")
    blp = torch.empty((count, SEQ_TOKENS), device="cuda")
    bam = torch.empty((count, SEQ_TOKENS), dtype=torch.int32, device="cuda")
    bcall = lambda: gb.score_batch_dev(btd.data_ptr(), count, SEQ_TOKENS, TWO_LEVEL, blp.data_ptr(), bam.data_ptr())
    bcall()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = time_dev(torch, bstream, bcall, 2, flush)
    ms = _max_over_ranks(torch, dist, world, ms)
    launches = gb.last_launches()
    parity = None
    if rank == 0:  # the rank's first sequence against the oracle
        parity = oracle_parity(mf, btoks[0], blp[0].cpu().numpy(), bam[0].cpu().numpy().astype(np.uint32), TWO_LEVEL)
        parity["sequence"] = int(first)
    gb.close()
    return {"value": round(BATCH_SEQS * SEQ_TOKENS / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3),
            "scaling": "strong", "n_gpus": world, "sequences_per_rank": count,
            "workload": f"{BATCH_SEQS} sequences x {SEQ_TOKENS} positions, two-level head, split over {world} rank(s); "
                        "one step = the whole batch; time = max over ranks",
            "gpu_launches_per_step": launches, "parity": parity}


def run_vocab_shard_leg(torch, dist, world, rank, local, flush, args):
    """C5: Gemma-3-1B geometry, one 1024-position sequence per step, the full head's vocabulary sharded
    over the ranks (one GPU each; at one rank, unsharded). The body is replicated, so the total work
    is fixed (strong scaling). Before sharding every rank scores the sequence with the unsharded head;
    the sharded results must equal it (argmax identical, log-probs within the log-sum-exp order
    difference). A profiled pass splits the head's time into this rank's rows and the all-gather +
    merge. The unsharded two-level head on the same model is timed beside it."""
    from gem_b200 import FULL, TWO_LEVEL, Gemma, shard, synth
    if rank == 0:
        mf = synth.ensure("gemma3-1b", classes=2048)
    if world > 1:
        dist.barrier()
    if rank != 0:
        mf = synth.ensure("gemma3-1b", classes=2048)
    n = SHARD_TOKENS
    g = Gemma(mf.gguf, ctx=CTX, device=local)
    g.load_twolevel(mf.twolevel)
    stream = torch.cuda.ExternalStream(g.stream, device=local)
    toks = torch.tensor(synth.tokens(n + 1, g.vocab, seed=3000).astype(np.int32), device="cuda")
    lp = torch.empty(n, device="cuda")
    am = torch.empty(n, dtype=torch.int32, device="cuda")
    call = lambda head: g.score_dev(toks.data_ptr(), n, head, lp.data_ptr(), am.data_ptr())
    call(FULL)
    g.sync()
    want_lp, want_am = lp.cpu().numpy().copy(), am.cpu().numpy().copy()
    rows = shard.row_range(g.vocab, 1, 0)
    if world > 1:
        rows = shard.init_vocab_shard(g)
    steps = max(1, min(args.steps, 10))
    for _ in range(args.warmup):
        call(FULL)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_full = _max_over_ranks(torch, dist, world, time_dev(torch, stream, lambda: call(FULL), steps, flush))
    launches = g.last_launches()
    got_lp, got_am = lp.cpu().numpy(), am.cpu().numpy()
    err = _max_over_ranks(torch, dist, world, float(np.abs(got_lp - want_lp).max()))
    bad = _max_over_ranks(torch, dist, world, float(np.sum(got_am != want_am)))
    g.set_profiling(True)
    for _ in range(2):
        call(FULL)
    g.sync()
    prof = g.parallel_profile()
    g.set_profiling(False)
    head_us = _max_over_ranks(torch, dist, world, prof["head"])
    comb_us = _max_over_ranks(torch, dist, world, prof["combine"])
    for _ in range(2):
        call(TWO_LEVEL)
    ms_two = _max_over_ranks(torch, dist, world, time_dev(torch, stream, lambda: call(TWO_LEVEL), steps, flush))
    g.close()
    return {"value": round(n / (ms_full / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms_full, 3),
            "scaling": "strong", "n_gpus": world,
            "workload": f"gemma3-1b Q8_0 (d 1152, 26 layers, ff 6912), one {n}-position sequence per step, full head "
                        f"{'sharded by vocab rows over ' + str(world) + ' ranks' if world > 1 else 'unsharded'}",
            "rows_per_rank": rows[1], "gpu_launches_per_step": launches,
            "check_vs_unsharded": {"max_abs_lp": err, "argmax_mismatches": int(bad), "pass": bool(bad == 0 and err < 2e-5)},
            "head_us_per_step": {"this_rank_rows": round(head_us, 1), "all_gather_and_merge": round(comb_us, 1),
                                 "note": "profiled pass (launched directly, events between launch groups), max over ranks"},
            "two_level_unsharded": {"value": round(n / (ms_two / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms_two, 3)},
            "l2": "flushed (256 MiB write) before every step"}


def run_qat(torch, flush, args):
    """C3: the 270M geometry in the QAT layout (Q4_0 body, F16 output matrix), full and two-level
    heads, and the same model with the head requantized to Q8_0 at load (to_q8)."""
    from gem_b200 import FULL, TWO_LEVEL, Gemma, synth
    mf = synth.ensure("gemma3-270m", body="q4_0", head="f16", classes=CLASSES)
    toks = synth.tokens(SEQ_TOKENS + 1, 262144, seed=1000)
    out = {}
    for head_bits, name in ((0, "f16_head"), (8, "q8_head")):
        g = Gemma(mf.gguf, ctx=CTX, head_bits=head_bits)
        g.load_twolevel(mf.twolevel)
        stream = torch.cuda.ExternalStream(g.stream)
        td = torch.tensor(toks.astype(np.int32), device="cuda")
        lp = torch.empty(SEQ_TOKENS, device="cuda")
        am = torch.empty(SEQ_TOKENS, dtype=torch.int32, device="cuda")
        e = {}
        for hname, head in (("two_level", TWO_LEVEL), ("full", FULL)):
            call = lambda: g.score_dev(td.data_ptr(), SEQ_TOKENS, head, lp.data_ptr(), am.data_ptr())
            for _ in range(2):
                call()
            ms = time_dev(torch, stream, call, 3, flush)
            e[hname] = {"value": round(SEQ_TOKENS / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3)}
        e["parity_two_level"] = oracle_parity_qat(mf, toks, g, td, lp, am, head_bits)
        out[name] = e
        g.close()
    out["workload"] = "gemma3-270m, Q4_0 body, F16 262144x640 output matrix (f16_head) and the same requantized " \
                      "to Q8_0 at load (q8_head); 512 random tokens per step, batch 1"
    return out


def oracle_parity_qat(mf, toks, g, td, lp, am, head_bits):
    from gem_b200 import TWO_LEVEL
    from oracle import oracle as orc
    g.score_dev(td.data_ptr(), SEQ_TOKENS, TWO_LEVEL, lp.data_ptr(), am.data_ptr())
    g.sync()
    isa = "avx512" if orc.detect_isa() == "avx512" else None
    o = orc.Model(mf.gguf, ctx=CTX, threads=REF_THREADS, isa=isa, head_bits=head_bits)
    o.load_twolevel(mf.twolevel)
    lpo, amo, _, _ = o.score(toks, TWO_LEVEL)
    o.close()
    a = am.cpu().numpy().astype(np.uint32)
    err = float(np.abs(lp.cpu().numpy() - lpo).max())
    return {"argmax_equal": bool(np.array_equal(a, amo)), "max_abs_lp": err, "positions": SEQ_TOKENS}


def run_tensor_cores(g, torch, stream, toks_d, lp_d, am_d, flush):
    """The headline step with the body products on the tensor cores (tc_gemm.cu: tcgen05 MMAs form
    each lane's exact int8 pair sums, the CUDA cores apply the reference's FMA per lane and block).
    Its log-probs and argmax ids must equal the CUDA-core products' bit for bit; the products' device
    time comes from the launch-group profile of a one-part pass, as for the headline's roofline."""
    from gem_b200 import TWO_LEVEL
    call = lambda: g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, TWO_LEVEL, lp_d.data_ptr(), am_d.data_ptr())
    call()
    g.sync()
    want_lp, want_am = lp_d.cpu().numpy().copy(), am_d.cpu().numpy().copy()
    res = {}
    for name, on in (("cuda_cores", False), ("tensor_cores", True)):
        g.set_tensor_cores(on)
        for _ in range(3):
            call()
        ms = time_dev(torch, stream, call, 5, flush)
        same = bool(np.array_equal(lp_d.cpu().numpy().view(np.uint32), want_lp.view(np.uint32)) and
                    np.array_equal(am_d.cpu().numpy(), want_am))
        g.set_profiling(True)
        for _ in range(2):
            call()
        torch.cuda.synchronize()
        prof = g.parallel_profile()
        g.set_profiling(False)
        res[name] = {"value": round(SEQ_TOKENS / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3),
                     "products_ms_per_step": round((prof["qkv"] + prof["o"] + prof["gate_up"] + prof["down"]) / 1e3, 3),
                     "bit_identical_to_cuda_cores": same}
    g.set_tensor_cores(False)
    res["note"] = ("same workload and step as the headline; products_ms_per_step from the launch-group profile of a "
                   "one-part pass; the headline runs the CUDA-core products")
    return res


def run_extras(g, torch, stream, toks_d, lp_d, am_d, flush, args, mf):
    """Secondary figures: the full head end to end, the head microbenchmark (full 262144x640 GEMV with
    fused log-sum-exp vs the two-level head, batch 1 and 64) and the CPU baseline."""
    from gem_b200 import AUTO, FULL, PIPELINED, SEQUENTIAL, TWO_LEVEL, Gemma, synth
    from oracle import oracle as orc
    out = {}
    mf_info = g.refresh_info()
    # the same workload scored token after token: as a layer-pipelined wavefront (one kernel) and with
    # each token finishing before the next starts (a CUDA graph per token)
    for name, sch, iters in (("pipelined", PIPELINED, 3), ("sequential", SEQUENTIAL, 1)):
        g.set_schedule(sch)
        g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, TWO_LEVEL, lp_d.data_ptr(), am_d.data_ptr())
        ms = time_dev(torch, stream, lambda: g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, TWO_LEVEL, lp_d.data_ptr(),
                                                         am_d.data_ptr()), iters, flush)
        am_h = am_d.cpu().numpy().astype(np.uint32)
        toks_h = toks_d.cpu().numpy().astype(np.uint32)
        roof, sched = token_roofline(g, mf_info, mf, am_h, toks_h, ms, args, sch)
        out[name] = {"value": round(SEQ_TOKENS / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3),
                     "schedule": sched, "roofline": roof}
    g.set_schedule(AUTO)
    out["tensor_cores"] = run_tensor_cores(g, torch, stream, toks_d, lp_d, am_d, flush)
    # full head, same sequence (two untimed calls: the first launches directly, the second is captured
    # as the CUDA graph the timed calls replay)
    for _ in range(2):
        g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, FULL, lp_d.data_ptr(), am_d.data_ptr())
    ms = time_dev(torch, stream, lambda: g.score_dev(toks_d.data_ptr(), SEQ_TOKENS, FULL, lp_d.data_ptr(), am_d.data_ptr()),
                  2, flush)
    out["full_head"] = {"value": round(SEQ_TOKENS / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3)}
    out["qat"] = run_qat(torch, flush, args)
    # head microbenchmark: h ~ N(0, 1)
    peak, _ = hbm_peak()
    head_bytes = g.info["head_bytes"]
    rng = np.random.default_rng(9)
    hm = {}
    for batch in (1, 64):
        H = torch.tensor(rng.standard_normal((batch, g.d)).astype(np.float32), device="cuda")
        T = torch.tensor(rng.integers(0, g.vocab, batch).astype(np.int32), device="cuda")
        lp = torch.empty(batch, device="cuda")
        am = torch.empty(batch, dtype=torch.int32, device="cuda")
        for name, fn in (("full", g.head_full_dev), ("two_level", g.head_twolevel_dev)):
            call = lambda: fn(H.data_ptr(), T.data_ptr(), batch, lp.data_ptr(), am.data_ptr(), sync=False)
            call()
            if name == "full":
                # the 178 MB output matrix is larger than L2 and streamed whole by every call, so the
                # calls run back to back, 20 between two events (one event pair per call adds the
                # timing floor below, reported beside it as us_one_call); after a 256 MiB write flush
                # the call also shares HBM with the write-back of the flush's dirty lines
                def calls20():
                    for _ in range(20):
                        call()

                us = time_dev(torch, stream, calls20, 5, None) * 1e3 / 20
                us_one = time_dev(torch, stream, call, 5, None) * 1e3
                us_wf = time_dev(torch, stream, call, 5, flush) * 1e3
                gbs = head_bytes / (us * 1e-6) / 1e9
                e = {"us": round(us, 2), "GB_s": round(gbs, 1), "frac_hbm": round(gbs / peak, 4), "bytes": head_bytes,
                     "l2": "no flush: input larger than L2", "timing": "20 calls back to back per event pair",
                     "us_one_call": round(us_one, 2), "us_after_write_flush": round(us_wf, 2)}
            else:
                us = time_dev(torch, stream, call, 5, flush) * 1e3
                e = {"us": round(us, 2), "l2": "flushed (256 MiB write) before every call"}
            hm[f"{name}_b{batch}"] = e
    # what this timing method reads for a kernel that does nothing (a one-element add on the same
    # stream after the same flush): the launch and event overhead inside every figure above
    one = torch.zeros(1, device="cuda")

    def tiny():
        with torch.cuda.stream(stream):
            one.add_(1.0)

    for _ in range(3):
        tiny()
    hm["timing_floor"] = {"us": round(time_dev(torch, stream, tiny, 10, flush) * 1e3, 2),
                          "what": "a one-element kernel timed the same way (flush, events on the same stream)"}
    out["head_microbench"] = hm
    # CPU baseline: the oracle on the host cores, one 512-token sequence, two-level head
    threads = args.cpu_threads or os.cpu_count() or 1
    m = orc.Model(mf.gguf, ctx=CTX, threads=threads)
    m.load_twolevel(mf.twolevel)
    toks = synth.tokens(SEQ_TOKENS + 1, m.vocab, seed=1000)
    t0 = time.perf_counter()
    _, _, tb, th = m.score(toks, 1)
    dt = time.perf_counter() - t0
    out["cpu_baseline"] = {"value": round(SEQ_TOKENS / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                           "isa": m.isa, "sample": f"one {SEQ_TOKENS}-token sequence, two-level head, same workload",
                           "gem_bench": gem_bench_fields(m, threads, dt, tb, th, 1)}
    m.close()
    return out


if __name__ == "__main__":
    main()
