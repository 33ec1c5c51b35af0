#!/usr/bin/env python
"""Benchmark of the arctic-embed-s int8 forward pass on B200.

Headline (BASELINE.json metric): embeddings/sec at 128 tokens, config 3 — batches of 512
sequences x 128 tokens per GPU, one batch per step, sharded over N GPUs (one process per GPU under
torchrun, no collective on the data path: weak scaling). Synthetic seeded model and token ids.

  value     device-resident throughput: token ids already in HBM, ae_forward_ragged_device per step,
            CUDA events per step on the launch stream, L2 flushed between steps (outside the events),
            total = max over ranks
  e2e       the same metric through the public host API (ae_forward_ragged): every step copies the
            ids from host memory to the GPU and the embeddings back, host wall clock, max over ranks
  latency   p50 / p99 of ae_forward_cls (batch 1, CUDA-graph replay, host buffers) at 8, 32, 128 and
            512 tokens (config 2), with latency_roofline (int8 ops / p50 against the measured int8
            peak; weight bytes / p50 against HBM)
  roofline  the dominant kernel of a step, timed with CUDA events around its launches in the step
  cpu_baseline  the CPU oracle (C++ restatement of the reference's x86 path) on a bounded sample,
            all host threads; cpu_latency: its single-threaded forward_cls at 8/32/128/512 tokens
  int8_peak the library's own tcgen05 kind::i8 loop (one CTA per SM, resident operands)
  micro     config 5: the GEMM shapes and the 64 x 12 x 512 attention (N = 1)
  ragged    config 4: 131,072 log-uniform sequences through ae_embed_batch_multi (N = 1)
  multi_api rank 0 alone drives all N GPUs through ae_embed_batch_multi (the product's multi-GPU
            entry point: planner, host threads, pipelined pinned staging, host gather); at N = 1 the
            same call on one GPU, the base of its scaling

`--impl reference` times the reference's CPU path (the oracle; the Rust crate cannot be built
here) on the same metric and prints its own JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "snowflake-arctic-embed-s-rust_b200"))
sys.path.insert(0, ROOT)

METRIC = "embeddings/sec @128 tok"
SEQ_LEN = 128
BATCH_SEQS = 512
H = 384
L2_BYTES = 126 * 1024 * 1024


def int8_ops_per_seq(L: int) -> float:
    """Algorithmic int8 ops of one sequence: 2 x (19,759,104 L + 1,474,560) MACs."""
    return 2.0 * (19759104.0 * L + 1474560.0)


def attn_flops_per_seq(L: int) -> float:
    """Algorithmic fp32 attention flop of one sequence: 2 x (8,448 L^2 + 768 L) MACs."""
    return 2.0 * (8448.0 * L * L + 768.0 * L)


# ncu summaries (committed under profiles/) with the measured DRAM bytes per launch of a kernel kind
NCU_TRAFFIC = {"attention": "k_attention_rows2_config3_ncu.md"}


def ncu_traffic(kind: str):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch from the kernel's ncu summary."""
    name = NCU_TRAFFIC.get(kind)
    if not name:
        return None, None
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for ln in f:
                if ln.startswith("| traffic_bytes_per_launch |"):
                    return int(ln.split("|")[2].strip()), "profiles/" + name
    except (OSError, ValueError):
        pass
    return None, None


def attn_bytes_per_launch(T: int) -> int:
    """Algorithmic DRAM bytes of one layer's attention: read Q, K, V (T x 1,152 fp32), write the
    context (T x 384 fp32)."""
    return T * (3 * H + H) * 4


def make_batches(n_batches: int, seed: int, seqs: int = BATCH_SEQS, L: int = SEQ_LEN):
    from arctic_embed_s_int8 import synth

    r = np.random.Generator(np.random.PCG64(seed))
    out = []
    for _ in range(n_batches):
        ids = np.concatenate([synth.token_ids(L, r) for _ in range(seqs)]).astype(np.uint16)
        cu = (np.arange(seqs + 1, dtype=np.uint32) * L).astype(np.uint32)
        out.append((ids, cu))
    return out


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms from before the warm-up on, each
    sample stamped on arrival; summary() keeps the samples inside the timed window (mark_start /
    mark_end), or the first one after its start when the window is shorter than the interval."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()
        if self.proc:  # the sample that closes the window
            deadline = self.t1 + 0.5
            while time.perf_counter() < deadline and not any(t >= self.t1 for t, _ in self.lines):
                time.sleep(0.01)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        inside = [ln for t, ln in self.lines if t0 <= t <= t1]
        if not inside:
            after = [ln for t, ln in self.lines if t >= t0]
            inside = after[:1]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in inside:
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
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "interval_ms": 50}


def cpu_baseline(seconds: float = 10.0, L: int = SEQ_LEN, threads: int | None = None):
    """Oracle embed_batch (all host threads) on a bounded sample of 128-token sequences."""
    from arctic_embed_s_int8 import synth
    from oracle import oracle as orc

    orc.build()
    threads = threads or os.cpu_count() or 1
    m = orc.OracleModel(synth.pack_path(0))
    r = np.random.Generator(np.random.PCG64(99))
    probe = [synth.token_ids(L, r) for _ in range(threads)]
    t0 = time.perf_counter()
    m.embed_batch(probe, threads)
    per_round = max(time.perf_counter() - t0, 1e-3)
    n = int(max(threads, min(8192, threads * seconds / per_round)))
    seqs = [synth.token_ids(L, r) for _ in range(n)]
    t0 = time.perf_counter()
    m.embed_batch(seqs, threads)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "embeddings/s", "cores": threads,
            "kind": "port", "sample": f"{n} sequences x {L} tokens, embed_batch over {threads} threads, {dt:.1f} s",
            "cpu": _cpu_name()}


def cpu_latency(runs: int = 100) -> dict:
    """Config 2 on the CPU: the oracle's single-threaded forward_cls (the reference's x86 path) at 8,
    32, 128 and 512 tokens, p50 / p99 over `runs` calls after 3 warm-up calls, on the same ids as
    the GPU latency (the reference's own sweep: src/bin/arctic_embed.rs:99-138)."""
    from arctic_embed_s_int8 import synth
    from oracle import oracle as orc

    orc.build()
    m = orc.OracleModel(synth.pack_path(0))
    r = np.random.Generator(np.random.PCG64(42))
    out = {"cores": 1, "kind": "port", "runs": runs, "cpu": _cpu_name(),
           "api": "oracle forward_cls, one thread (the backend SimdBackend::detect picks on this host)"}
    for L in (8, 32, 128, 512):
        ids = synth.token_ids(L, r)
        for _ in range(3):
            m.forward_cls(ids)
        ts = []
        for _ in range(runs):
            t0 = time.perf_counter()
            m.forward_cls(ids)
            ts.append((time.perf_counter() - t0) * 1e3)
        out[f"p50_ms@{L}"] = float(np.percentile(ts, 50))
        out[f"p99_ms@{L}"] = float(np.percentile(ts, 99))
    return out


def weight_bytes_per_forward() -> int:
    """Model bytes one forward pass must read: the int8 weights of layers 0-10 (QKV, attention-out,
    FFN-up, FFN-down) and of layer 11's KV / Q / attention-out / FFN, with their f32 scales and
    biases, plus the LayerNorm vectors (the embedding rows of the tokens are counted apart)."""
    H, I = 384, 1536
    lin = lambda n, k: n * k + 8 * n + 4 * k  # int8 weights + w_scale, bias + inv_smooth
    per_layer = lin(3 * H, H) + lin(H, H) + lin(I, H) + lin(H, I) + 4 * 4 * H
    last = lin(2 * H, H) + lin(H, H) + lin(H, H) + lin(I, H) + lin(H, I) + 4 * 4 * H
    return 11 * per_layer + last + 2 * 4 * H


def _cpu_name():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (oracle port) on this host's cores, rank 0 only."""
    if rank != 0:
        return 0
    from arctic_embed_s_int8 import synth
    from oracle import oracle as orc

    orc.build()
    threads = os.cpu_count() or 1
    m = orc.OracleModel(synth.pack_path(0))
    r = np.random.Generator(np.random.PCG64(7))
    per_step = max(threads, args.ref_seqs_per_step)
    for _ in range(args.warmup):
        m.embed_batch([synth.token_ids(SEQ_LEN, r) for _ in range(threads)], threads)
    times = []
    for _ in range(args.steps):
        seqs = [synth.token_ids(SEQ_LEN, r) for _ in range(per_step)]
        t0 = time.perf_counter()
        m.embed_batch(seqs, threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = per_step * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "embeddings/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 GEMM / fp32",
        "data": "synthetic (seeded .ae8 pack and token ids)",
        "config": {"workload": "config 3: 128-token sequences (a bounded sample per step on the CPU)",
                   "seq_len": SEQ_LEN, "seqs_per_step": per_step},
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} sequences x {SEQ_LEN} tokens per step, embed_batch, {threads} threads",
                         "cpu": _cpu_name()},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def step_work(T: int, n: int, L: int) -> dict:
    """Algorithmic work of one forward step per kernel kind (ops for the int8 GEMMs, flop for the
    fp32 attention, bytes for the row kernels), from the model's shapes."""
    H, I = 384, 1536
    return {
        "qkv": 2.0 * T * H * (11 * 3 * H + 2 * H),                  # int8 ops (QKV x 11 + layer-11 KV)
        "attention": 11 * n * 12 * 2.0 * 2.0 * L * L * 32,           # fp32 flop (QK^T + PV)
        "attn_out": 11 * 2.0 * T * H * H,
        "ffn_up": 11 * 2.0 * T * H * I,
        "ffn_down": 11 * 2.0 * T * I * H,
        "ctx_quant": 11 * T * (H * 4 + H + 4.0),                     # bytes read + written
        "embed": T * (2 + 2 + H + H * 4 + H + 4.0),
    }


def measure_fp32_peak() -> float:
    """Measured FP32 CUDA-core throughput (TFLOP/s): cuBLAS SGEMM 8192^3 with TF32 disabled."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    for _ in range(2):
        a @ b
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        a @ b
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * 8192 ** 3 / best / 1e9


def microbench(eng, stream, peaks: dict, i8peak: float) -> dict:
    """Config 5: the four int8 GEMM shapes x M in {512, 8192, 65536} (plain dequant epilogue, and the
    fused model epilogue where the shape has one) and the masked attention over 64 x 12 x 512 x 32
    (fp32 in the reference's order, and the reference's int8 scheme). CUDA events on the launch stream, median of 5 after warm-up, L2 flushed before each."""
    import torch

    hbm = peaks.get("hbm_gbs", 6650.0)
    g = torch.Generator(device="cpu").manual_seed(5)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def timed(fn, reps=5):
        fn()
        ts = []
        for _ in range(reps):
            with torch.cuda.stream(stream):
                flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        eng.sync()
        return float(np.median(ts))

    out = {"gemm": [], "attention": None}
    for K, N in ((384, 1152), (384, 384), (384, 1536), (1536, 384)):
        w = torch.clamp(torch.round(torch.randn(N, K, generator=g) * 40), -127, 127).to(torch.int8).cuda()
        ws = (torch.rand(N, generator=g) * 9e-3 + 1e-3).cuda()
        bias = (torch.randn(N, generator=g) * 0.02).cuda()
        for M in (512, 8192, 65536):
            a = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g).cuda()
            asc = (torch.rand(M, generator=g) * 9e-3 + 1e-3).cuda()
            o = torch.empty(M, N, device="cuda")
            ops = 2.0 * M * K * N
            ms = timed(lambda: eng.gemm_i8(0, a, asc, w, ws, bias, out=o))
            byt = M * K + K * N + 4 * N + 4 * M + 4 * M * N
            bound_ms = max(ops / (i8peak * 1e12), byt / (hbm * 1e9)) * 1e3
            row = {"K": K, "N": N, "M": M, "epilogue": "dequant f32", "ms": ms, "tops": ops / ms / 1e9,
                   "roofline_ms": bound_ms, "frac": bound_ms / ms}
            out["gemm"].append(row)
            fused = None
            if N == 384:
                res = torch.randn(M, N, device="cuda")
                gam, bet = torch.ones(384, device="cuda"), torch.zeros(384, device="cuda")
                inv = torch.ones(384, device="cuda")
                q = torch.empty(M, N, dtype=torch.int8, device="cuda")
                sc = torch.empty(M, device="cuda")
                fused = ("residual+LayerNorm+requant", lambda: eng.gemm_i8(1, a, asc, w, ws, bias, res=res, gamma=gam,
                                                                         beta=bet, inv_smooth=inv, out=res, out_q=q,
                                                                         out_scale=sc),
                         M * K + K * N + 8 * M + 2 * 4 * M * N + M * N)
            elif N == 1536:
                inv = torch.ones(1536, device="cuda")
                q = torch.empty(M, N, dtype=torch.int8, device="cuda")
                sc = torch.empty(M, device="cuda")
                fused = ("GELU+requant", lambda: eng.gemm_i8(2, a, asc, w, ws, bias, inv_smooth=inv, out_q=q,
                                                            out_scale=sc), M * K + K * N + 8 * M + M * N)
            if fused:
                ms = timed(fused[1])
                bound_ms = max(ops / (i8peak * 1e12), fused[2] / (hbm * 1e9)) * 1e3
                out["gemm"].append({"K": K, "N": N, "M": M, "epilogue": fused[0], "ms": ms, "tops": ops / ms / 1e9,
                                    "roofline_ms": bound_ms, "frac": bound_ms / ms})
    n, L = 64, 512
    qkv = torch.randn(n * L, 1152, device="cuda")
    cu = torch.arange(0, n + 1, dtype=torch.int32, device="cuda") * L
    ctx = torch.empty(n * L, 384, device="cuda")
    ms = timed(lambda: eng.attention_f32(qkv, cu, n, L, ctx))
    fl = n * 12 * 2.0 * 2.0 * L * L * 32
    out["attention"] = {"shape": "64 x 12 heads x 512 x 32, fp32, exact reference order", "ms": ms,
                        "tflops": fl / ms / 1e9}
    ms8 = timed(lambda: eng.attention_i8(qkv, cu, n, L, ctx))
    out["attention_int8"] = {"shape": "64 x 12 heads x 512 x 32, the reference's int8 scheme (dp4a Q.K, dp2a P.V)",
                             "ms": ms8, "int_tops": fl / ms8 / 1e9}
    out["basis"] = (f"roofline_ms = max(ops / int8 peak ({i8peak:.0f} TOPS, measured by ae_measure_int8_peak), "
                    f"bytes / HBM {hbm} GB/s of measured); frac = roofline_ms / ms")
    return out


def ragged_throughput(eng) -> dict:
    """Config 4: 131,072 sequences, lengths log-uniform on [8, 512], through ae_embed_batch_multi
    (host ids in, embeddings out) on this process's GPU."""
    from arctic_embed_s_int8 import embed_batch_multi, pack_sequences, synth

    r = np.random.Generator(np.random.PCG64(4))
    lens = np.exp(r.uniform(np.log(8), np.log(512), 131072)).astype(np.int64)
    seqs = [synth.token_ids(int(L), r) for L in lens]
    ids, cu = pack_sequences(seqs)
    embed_batch_multi([eng], ids=ids[: int(cu[2048])], cu=cu[:2049])  # warm-up
    t0 = time.perf_counter()
    embed_batch_multi([eng], ids=ids, cu=cu)
    dt = time.perf_counter() - t0
    # a second, profiled pass: device time per kernel kind next to the wall clock
    eng.profile(True)
    embed_batch_multi([eng], ids=ids, cu=cu)
    eng.sync()
    prof = eng.profile_read()
    eng.profile(False)
    return {"sequences": len(seqs), "tokens": int(cu[-1]), "mean_len": float(lens.mean()), "seconds": dt,
            "embeddings_per_s": len(seqs) / dt, "tokens_per_s": float(cu[-1]) / dt,
            "kernels_s": {k: round(v[0] / 1e3, 4) for k, v in prof.items()},
            "api": "ae_embed_batch_multi, host buffers (wall clock, includes packing and copies)"}


def multi_api(world: int, pack: str, steps: int) -> dict:
    """The product's multi-GPU entry point, driven by one process over all `world` GPUs:
    ae_embed_batch_multi (token-weighted shard plan, one host thread and context per GPU, pinned
    staging, host gather of the 384-d outputs; no collective) on (a) the config-3 set of this run
    (world x 512 x steps sequences of 128 tokens) and (b) config 4 (131,072 log-uniform sequences).
    Wall clock around the call (host ids in, host embeddings out), after a warm-up call; then a
    profiled pass gives each GPU's busy time (sum of its kernels' CUDA-event times)."""
    from arctic_embed_s_int8 import Engine, embed_batch_multi, pack_sequences, synth

    engines = [Engine(d).load_file(pack) for d in range(world)]
    for e in engines:  # the workspace of the largest batch (65,536 rows of 8-token sequences)
        e.reserve(65536, 8192)
    r = np.random.Generator(np.random.PCG64(2024))
    sets = {
        "config3": [synth.token_ids(SEQ_LEN, r) for _ in range(world * BATCH_SEQS * steps)],
        "config4": [synth.token_ids(int(L), r)
                    for L in np.exp(r.uniform(np.log(8), np.log(512), 131072)).astype(np.int64)],
    }
    out = {"gpus": world, "api": "ae_embed_batch_multi (one process, one context and host thread per GPU)"}
    for name, seqs in sets.items():
        ids, cu = pack_sequences(seqs)
        embed_batch_multi(engines, ids=ids, cu=cu)  # warm-up: sizes the staging buffers
        t0 = time.perf_counter()
        embed_batch_multi(engines, ids=ids, cu=cu)
        dt = time.perf_counter() - t0
        for e in engines:
            e.profile(True)
        embed_batch_multi(engines, ids=ids, cu=cu)
        busy = []
        for e in engines:
            e.sync()
            busy.append(round(sum(v[0] for v in e.profile_read().values()) / 1e3, 4))
            e.profile(False)
        out[name] = {"sequences": len(seqs), "tokens": int(cu[-1]), "seconds": dt,
                     "embeddings_per_s": len(seqs) / dt, "device_busy_s": busy,
                     "busy_over_wall": round(max(busy) / dt, 3)}
    for e in engines:
        e.close()
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--latency-runs", type=int, default=1000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seqs-per-step", type=int, default=64)
    ap.add_argument("--no-extras", action="store_true",
                    help="skip latency, kernel breakdown, CPU baselines, configs 4 and 5, multi_api")
    ap.add_argument("--cpu-latency-runs", type=int, default=100)
    ap.add_argument("--no-cpu-latency", action="store_true", help="skip the CPU latency baseline")
    ap.add_argument("--no-micro", action="store_true", help="skip the config-5 kernel microbenchmarks")
    ap.add_argument("--no-ragged", action="store_true", help="skip config 4 (131,072 ragged sequences)")
    ap.add_argument("--latency-only", type=int, default=0, metavar="L",
                    help="only replay ae_forward_cls at L tokens (--latency-runs times) and print its p50 "
                         "(a small case for profilers)")
    ap.add_argument("--micro-only", action="store_true",
                    help="only run the config-5 kernel microbenchmarks (a small case for profilers)")
    ap.add_argument("--attention", default="exact", choices=["exact", "int8"],
                    help="attention of layers 0-10: fp32 in the reference's x86 order (default) or the "
                         "reference's int8 scheme (ae_set_attention_mode)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    args.warmup = max(args.warmup, 3)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from arctic_embed_s_int8 import Engine, synth

    pack = synth.pack_path(0)
    eng = Engine(local).load_file(pack)
    if args.attention == "int8":
        from arctic_embed_s_int8 import ATTENTION_INT8

        eng.set_attention_mode(ATTENTION_INT8)
    stream = torch.cuda.Stream()
    if args.latency_only:
        # one length of config 2 alone (ae_forward_cls, CUDA-graph replay): a small case for profilers
        ids = synth.token_ids(args.latency_only, np.random.Generator(np.random.PCG64(42)))
        for _ in range(args.warmup):
            eng.forward_cls(ids)
        ts = []
        for _ in range(args.latency_runs):
            t0 = time.perf_counter()
            eng.forward_cls(ids)
            ts.append((time.perf_counter() - t0) * 1e3)
        print(json.dumps({"latency_only": args.latency_only, "runs": args.latency_runs,
                          "p50_ms": float(np.percentile(ts, 50)), "warmup": args.warmup}), flush=True)
        eng.close()
        return 0
    eng.set_stream(stream)
    if args.micro_only:
        # config 5 alone: a small case for profilers
        peaks = {}
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peaks = json.load(f)
        except OSError:
            pass
        _, i8peak = eng.measure_int8_peak(100000)
        print(json.dumps({"micro": microbench(eng, stream, peaks, i8peak), "int8_peak_tops": i8peak}), flush=True)
        eng.close()
        return 0
    n_batches = args.warmup + args.steps
    batches = make_batches(n_batches, seed=1000 + rank)
    T = BATCH_SEQS * SEQ_LEN
    eng.reserve(T, BATCH_SEQS)
    d_in = [(torch.from_numpy(ids.view(np.int16)).cuda(), torch.from_numpy(cu.view(np.int32)).cuda()) for ids, cu in batches]
    d_out = torch.empty(BATCH_SEQS, H, dtype=torch.float32, device="cuda")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    # ---- value: device-resident inputs
    launches0 = eng.kernel_launches()
    with torch.cuda.stream(stream), ClockSampler(local) as clk:
        for i in range(args.warmup):
            eng.forward_device(d_in[i][0], d_in[i][1], BATCH_SEQS, T, SEQ_LEN, d_out)
        eng.sync()
        barrier()
        launches0 = eng.kernel_launches()
        evs = []
        clk.mark_start()
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            b = d_in[args.warmup + i]
            eng.forward_device(b[0], b[1], BATCH_SEQS, T, SEQ_LEN, d_out)
            e1.record(stream)
            evs.append((e0, e1))
        stream.synchronize()
        eng.sync()
        clk.mark_end()
        barrier()
        launches = eng.kernel_launches() - launches0
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_s = max_over_ranks(sum(step_ms) / 1e3)
    value = world * BATCH_SEQS * args.steps / total_s

    # ---- e2e: host buffers through the public API
    h_batches = batches
    for i in range(args.warmup):
        eng.forward_packed(*h_batches[i])
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        out = eng.forward_packed(*h_batches[args.warmup + i])
    t_e2e = time.perf_counter() - t0
    barrier()
    t_e2e = max_over_ranks(t_e2e)
    e2e = world * BATCH_SEQS * args.steps / t_e2e
    h2d = int(batches[0][0].nbytes + batches[0][1].nbytes)
    d2h = int(out.nbytes)

    result = {
        "metric": METRIC, "value": value, "unit": "embeddings/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("int8 GEMM (int32 acc) / fp32 elementwise+attention" if args.attention == "exact" else
                  "int8 GEMM (int32 acc) / fp32 elementwise / int8 attention (the reference's SME scheme)"),
        "data": "synthetic (seeded .ae8 pack, random-init arctic-embed-s weights; token ids [CLS]+U[1000,30521]+[SEP])",
        "config": {"workload": "config 3: batches of 512 sequences x 128 tokens per GPU, one batch per step",
                   "global_batch": world * BATCH_SEQS, "seq_len": SEQ_LEN, "tokens_per_step_per_gpu": T,
                   "parallelism": f"data-parallel shards x{world}, no collective",
                   "l2": "flushed (256 MB write) between timed steps, outside the step events",
                   "attention": args.attention},
        "e2e": {"value": e2e, "unit": "embeddings/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "ae_forward_ragged (host ids in, host embeddings out; wall clock)"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    src = "of measured" if peaks else "of fallback"
    hbm = peaks.get("hbm_gbs", 6650.0)
    if not args.no_extras and rank == 0 and world == 1:
        # int8 tensor-pipe peak of this GPU: the library's own resident-operand tcgen05 kind::i8 loop
        pk_ms, i8peak = eng.measure_int8_peak(100000)
        result["int8_peak"] = {"tops": i8peak, "ms": pk_ms, "spec_dense_tops": 4500.0,
                               "api": "ae_measure_int8_peak (148 CTAs x 100,000 rounds of M128 N256 K128)"}
        # latency (config 2): p50/p99 of forward_cls, host buffers, CUDA-graph replay
        lat = {}
        r = np.random.Generator(np.random.PCG64(42))
        for L, runs in ((8, args.latency_runs), (32, args.latency_runs), (128, args.latency_runs),
                        (512, max(50, args.latency_runs // 3))):
            ids = synth.token_ids(L, r)
            for _ in range(20):
                eng.forward_cls(ids)
            ts = []
            for _ in range(runs):
                t0 = time.perf_counter()
                eng.forward_cls(ids)
                ts.append((time.perf_counter() - t0) * 1e3)
            lat[f"p50_ms@{L}"] = float(np.percentile(ts, 50))
            lat[f"p99_ms@{L}"] = float(np.percentile(ts, 99))
            lat[f"runs@{L}"] = runs
        result["latency"] = lat
        wb = weight_bytes_per_forward()
        result["latency_roofline"] = {
            f"@{L}": {"int8_tops": int8_ops_per_seq(L) / (lat[f"p50_ms@{L}"] * 1e-3) / 1e12,
                      "frac_int8_peak": int8_ops_per_seq(L) / (lat[f"p50_ms@{L}"] * 1e-3) / 1e12 / i8peak,
                      "weight_gbs": (wb + L * (H + 4) * 2) / (lat[f"p50_ms@{L}"] * 1e-3) / 1e9,
                      "frac_hbm": (wb + L * (H + 4) * 2) / (lat[f"p50_ms@{L}"] * 1e-3) / 1e9 / hbm}
            for L in (8, 32, 128, 512)}
        result["latency_roofline"]["basis"] = (
            f"int8 ops of one sequence (2 x (19,759,104 L + 1,474,560)) / p50 against the measured int8 peak "
            f"({i8peak:.0f} TOPS); model bytes one forward reads ({wb} B of weights, scales, biases and "
            f"LayerNorm vectors + the L embedding rows) / p50 against HBM {hbm} GB/s {src}")
        # model start-up (config 2's companion, the reference's ~10 ms .ae8 load): ae_model_load_file
        # of the 33.8 MB pack into a context that already exists, median of 5 after one warm-up
        lt = []
        for i in range(6):
            t0 = time.perf_counter()
            eng.load_file(pack)
            lt.append((time.perf_counter() - t0) * 1e3)
        result["model_load_ms"] = {"median": float(np.median(lt[1:])), "first": lt[0],
                                   "api": "ae_model_load_file (mmap, pinned host image, one DMA, arena reused)"}
        # per-kernel times of the forward itself: CUDA events around every launch on the launch
        # stream, over K more steps of the same workload (profiling is off in the timed region)
        eng.profile(True)
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.fill_(float(i))
                b = d_in[args.warmup + i]
                eng.forward_device(b[0], b[1], BATCH_SEQS, T, SEQ_LEN, d_out)
        eng.sync()
        prof = eng.profile_read()
        eng.profile(False)
        work = step_work(T, BATCH_SEQS, SEQ_LEN)
        per_step_ms = {k: v[0] / args.steps for k, v in prof.items() if v[1]}
        result["kernels_ms_per_step"] = {k: round(v, 4) for k, v in per_step_ms.items()}
        result["kernels_launches_per_step"] = {k: v[1] // args.steps for k, v in prof.items() if v[1]}
        dom = max(per_step_ms, key=per_step_ms.get)
        bf16 = peaks.get("bf16_tflops", 1590.0)
        launches = prof[dom][1] // args.steps
        ms_launch = per_step_ms[dom] / max(launches, 1)
        if dom in ("qkv", "attn_out", "ffn_up", "ffn_down"):
            ach = work[dom] / (per_step_ms[dom] * 1e-3) / 1e12
            result["roofline"] = {"kernel": dom, "bound": "tensor", "achieved": ach, "peak": i8peak,
                                  "unit": "TOPS (int8)", "frac": ach / i8peak, "traffic": None,
                                  "ms_per_launch": ms_launch,
                                  "peak_basis": "int8 dense, measured by ae_measure_int8_peak in this run"}
        elif dom == "attention":
            ach = work[dom] / (per_step_ms[dom] * 1e-3) / 1e12
            fp32 = measure_fp32_peak()
            traffic, tsrc = ncu_traffic(dom)
            result["roofline"] = {"kernel": dom, "bound": "fp32", "achieved": ach, "peak": fp32,
                                  "unit": "TFLOP/s (fp32 CUDA cores)", "frac": ach / fp32, "traffic": traffic,
                                  "traffic_source": tsrc, "algorithmic_bytes_per_launch": attn_bytes_per_launch(T),
                                  "ms_per_launch": ms_launch,
                                  "peak_basis": "measured here: cuBLAS SGEMM 8192^3, TF32 off (the attention keeps "
                                                "the reference's fp32 operation order, so it runs on the CUDA cores)",
                                  "fp32_issue_peak_at_max_clock": 148 * 128 * 2 * 1.965e9 / 1e12,
                                  "bf16_tensor_peak_of_measured": bf16}
        else:
            ach = work.get(dom, 0.0) / (per_step_ms[dom] * 1e-3) / 1e9
            result["roofline"] = {"kernel": dom, "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                                  "frac": ach / hbm, "traffic": None, "ms_per_launch": ms_launch,
                                  "peak_basis": f"HBM copy bandwidth {src}"}
        result["int8_tops_whole_step"] = BATCH_SEQS * int8_ops_per_seq(SEQ_LEN) / (total_s / args.steps) / 1e12
        if not args.no_micro:
            result["micro"] = microbench(eng, stream, peaks, i8peak)
        if not args.no_ragged:
            result["ragged"] = ragged_throughput(eng)
        try:
            result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        except Exception as e:  # reported, not fatal
            result["cpu_baseline"] = {"error": str(e)}
        if not args.no_cpu_latency:
            try:
                result["cpu_latency"] = cpu_latency(args.cpu_latency_runs)
            except Exception as e:  # reported, not fatal
                result["cpu_latency"] = {"error": str(e)}
        try:
            result["multi_api"] = multi_api(1, pack, args.steps)
        except Exception as e:  # reported, not fatal
            result["multi_api"] = {"error": str(e)}
    if world > 1 and not args.no_extras:
        # the product's multi-GPU entry point: rank 0 alone drives every GPU of the box while the
        # other ranks wait on a host-side (gloo) barrier, which leaves their GPUs idle
        from datetime import timedelta

        host = dist.new_group(backend="gloo", timeout=timedelta(seconds=900))
        dist.barrier(group=host)
        if rank == 0:
            try:
                result["multi_api"] = multi_api(world, pack, args.steps)
            except Exception as e:  # reported, not fatal
                result["multi_api"] = {"error": str(e)}
        dist.barrier(group=host)
    if rank == 0:
        print(json.dumps(result), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
