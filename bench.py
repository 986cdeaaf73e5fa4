#!/usr/bin/env python
"""Benchmark of the compress-zip model-plus-coder path on B200.

Workload: the shipped model v001_eng.czm at
level L5 (context 1024), batch compression of 1,024 synthetic 15,000-byte
documents (seeds 1..1024 on rank 0; rank r uses seeds r*1024+1..).  A step is
one compression of the whole batch: every chunk of every document through the
model, the CDF and the arithmetic coder (the loop of rust/src/main.rs:206-238).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``value`` is measured with the token ids already
resident in HBM (czg_compress_chunks_device); ``e2e`` is the same work through
the host-buffer C-ABI call (czg_compress_chunks), with the host->device copy of
the tokens and the device->host copy of the encoded bytes inside the timed
region.  Per-step times come from CUDA events on the stream the engine runs on;
L2 is flushed (a 256 MiB write) before every timed step, outside the timing.
The reference arm times the CPU oracle (a C restatement of the reference's Rust
path) on the host cores over a bounded sample of the same workload.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
from __graft_entry__ import load_package  # noqa: E402

load_package()
from compress_zip_b200 import czm, synth  # noqa: E402

METRIC = "compress tokens/s & MB/s at L5 ctx1024, 1/2/4/8 B200; batched decode tok/s"
MODEL = os.path.join(ROOT, "models", "v001_eng.czm")
DOC_BYTES = 15000


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--docs", type=int, default=1024)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--cpu-sample-docs", type=int, default=32)
    ap.add_argument("--decode-docs", type=int, default=4096,
                    help="config 3: documents of 4,096 B decoded at ctx 512 (0 skips)")
    ap.add_argument("--pipeline-docs", type=int, default=64,
                    help="host pipeline sample (tokenise + GPU coder + CZIPv1 + brotli); 0 skips")
    ap.add_argument("--config2-docs", type=int, default=256,
                    help="config 2: documents of 64 KiB compressed with the arch-2 model at ctx 512 (0 skips)")
    ap.add_argument("--config4-docs", type=int, default=64,
                    help="config 4 sample: documents of 64 KiB with the arch-2 model at ctx 4096 (0 skips)")
    return ap.parse_args()


def shard_seeds(rank: int, per_rank: int, first: int = 1) -> range:
    """Documents of a rank: ranks take disjoint seed ranges (weak scaling)."""
    return range(first + rank * per_rank, first + (rank + 1) * per_rank)


def reduce_over_ranks(t_max: list, n_sum: list, device) -> tuple[list, list]:
    """Max of the per-rank times and sum of the per-rank counts over all ranks."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(t_max), list(n_sum)
    a = torch.tensor(list(t_max), dtype=torch.float64, device=device)
    b = torch.tensor(list(n_sum), dtype=torch.float64, device=device)
    dist.all_reduce(a, op=dist.ReduceOp.MAX)
    dist.all_reduce(b)
    return a.tolist(), b.tolist()


def workload(mf, seeds, ctx):
    tok = mf.tokenizer()
    docs = synth.documents(seeds, DOC_BYTES)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    starts = [0]
    base = 0
    for t in ids:
        for s in range(0, len(t), ctx):
            starts.append(base + min(s + ctx, len(t)))
        base += len(t)
    tokens = np.concatenate([np.asarray(t, dtype=np.uint32) for t in ids])
    return tokens, np.asarray(starts, dtype=np.uint64), sum(len(d.encode()) for d in docs)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx.append(float(r[1]))
            except ValueError:
                continue
            for name, v in zip(names, r[3:]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), \
            "of measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "of fallback"


def per_token(name: str) -> dict:
    """A per-token figure of each kernel class from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def traffic_per_token():
    """dram bytes per token of each kernel class (read + write, one launch)."""
    return per_token("dram_bytes_per_token.json")


def algorithmic(kernel: str, info: dict, tokens_per_launch: float):
    """(bound, algorithmic amount per launch, unit) of a kernel class."""
    d, dff, V, L = info["d_model"], info["d_ff"], info["vocab_size"], info["n_layers"]
    if kernel == "attention":
        # per token and layer: K/V row (128 B) + Q row (d) read once, output (d) written once
        return "hbm", (128 + 2 * d) * tokens_per_launch, "GB/s"
    if kernel == "cdf":
        return "hbm", (4 * V + 4 + 8) * tokens_per_launch, "GB/s"
    if kernel == "encode":
        return "hbm", 8.0 * tokens_per_launch + 1.2 * tokens_per_launch, "GB/s"
    macs = {"gemm_qkv": (d + 128) * d, "gemm_o": d * d, "gemm_up_reglu": 2 * dff * d,
            "gemm_down": d * dff, "gemm_head": V * d}.get(kernel)
    if macs is not None:
        return "tensor", 2.0 * macs * tokens_per_launch, "TFLOP/s"
    return "hbm", 0.0, "GB/s"


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    mf = czm.ModelFile.load(MODEL)
    if args.impl == "reference":
        return run_reference(args, mf, rank, world)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from compress_zip_b200.engine import Engine

    seeds = shard_seeds(rank, args.docs)
    tokens, starts, nbytes = workload(mf, seeds, args.ctx)
    n_tok, n_chunks = int(len(tokens)), int(len(starts) - 1)

    eng = Engine(mf.raw, local)
    stream = torch.cuda.current_stream()
    eng.set_stream(stream.cuda_stream)
    d_tokens = torch.from_numpy(tokens.view(np.int32)).to(f"cuda:{local}")
    bound = 4 * n_tok + 8 * n_chunks
    out = np.empty(bound, dtype=np.uint8)
    lens = np.empty(n_chunks, dtype=np.uint32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")

    def step_device():
        return eng.compress_device(d_tokens.data_ptr(), starts, out, lens)

    def barrier():
        if world > 1:
            dist.barrier()

    # per-kernel CUDA events around each launch of the compress step (about 170 per
    # step, a negligible cost here) give the kernel split and the roofline duration
    eng.set_kernel_timing(True)
    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    times, launches, kern_ms, kern_n = [], 0, {}, {}
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    for _ in range(args.steps):
        flush.zero_()
        ev0.record(stream)
        nout = step_device()
        ev1.record(stream)
        torch.cuda.synchronize()
        times.append(ev0.elapsed_time(ev1))
        st = eng.last_stats()
        for k, v in st["kernels"].items():
            kern_ms[k] = kern_ms.get(k, 0.0) + v["ms"]
            kern_n[k] = kern_n.get(k, 0) + v["launches"]
            launches += v["launches"]
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    t_rank = sum(times)

    # end to end through the host-buffer ABI call (pinned host memory)
    h_tokens = torch.from_numpy(tokens.view(np.int32)).pin_memory()
    h_out = torch.empty(bound, dtype=torch.uint8).pin_memory()
    h_tok_np = h_tokens.numpy().view(np.uint32)
    h_out_np = h_out.numpy()
    import ctypes as C
    from compress_zip_b200 import engine as E

    def step_host():
        need = C.c_uint64(0)
        stt = E.lib().czg_compress_chunks(eng._h, h_tok_np.ctypes.data, starts.ctypes.data,
                                          n_chunks, h_out_np.ctypes.data, bound,
                                          lens.ctypes.data, C.byref(need))
        eng._check(stt)
        return need.value

    step_host()
    torch.cuda.synchronize()
    barrier()
    e2e_times = []
    for _ in range(args.steps):
        flush.zero_()
        ev0.record(stream)
        nout_h = step_host()
        ev1.record(stream)
        torch.cuda.synchronize()
        e2e_times.append(ev0.elapsed_time(ev1))
    barrier()
    t_e2e = sum(e2e_times)
    parity = bytes(h_out_np[:nout_h]) == bytes(out[:nout])

    dec = decode_bench(eng, mf, rank, args, stream, world) if args.decode_docs > 0 else None
    cfg2 = arch2_bench(mf, rank, args, stream, local, 2) if args.config2_docs > 0 else None
    cfg4 = arch2_bench(mf, rank, args, stream, local, 4) if args.config4_docs > 0 else None
    pipe = host_pipeline(eng, mf, args) if rank == 0 and args.pipeline_docs > 0 else None

    (t_max, t_e2e_max), (all_tok, all_bytes) = reduce_over_ranks(
        [t_rank, t_e2e], [float(n_tok), float(nbytes)], f"cuda:{local}")

    if rank == 0:
        K = args.steps
        value = all_tok * K / (t_max / 1e3)
        e2e_value = all_tok * K / (t_e2e_max / 1e3)
        hbm, bf16, bf16_sus, basis = peaks()
        dom = max(kern_ms, key=kern_ms.get)
        per_launch_ms = kern_ms[dom] / max(1, kern_n[dom])
        tok_per_launch = n_tok * K / max(1, kern_n[dom])
        if dom.startswith("gemm") or dom == "attention":
            tok_per_launch *= 1  # one launch per layer per wave
        bound, amount, unit = algorithmic(dom, eng.info, tok_per_launch)
        achieved = amount / (per_launch_ms / 1e3) / (1e9 if unit == "GB/s" else 1e12)
        peak = hbm if bound == "hbm" else 2.0 * bf16_sus
        tpt = traffic_per_token().get(dom)
        roofline = {"kernel": dom, "bound": bound, "achieved": round(achieved, 3), "peak": peak,
                    "unit": unit, "frac": round(achieved / peak, 5),
                    "traffic": None if tpt is None else round(tpt * tok_per_launch),
                    "peak_basis": (f"hbm_gbs {basis}" if bound == "hbm" else
                                   f"2 x bf16_tflops_sustained {basis} (dense int8 = 2 x bf16)")}
        ipt = per_token("inst_per_token.json").get(dom)
        if ipt is not None:
            # the issue limit: 4 warp instructions per cycle per SM at the clock seen under load
            sms = torch.cuda.get_device_properties(local).multi_processor_count
            mhz = (clk or {}).get("sm_mhz") or 1965.0
            issued = ipt * tok_per_launch / (per_launch_ms / 1e3) / 1e9
            peak_i = sms * 4 * mhz / 1e3
            roofline["issue"] = {"achieved": round(issued, 1), "peak": round(peak_i, 1),
                                 "unit": "G warp instructions/s", "frac": round(issued / peak_i, 4),
                                 "inst_per_token": ipt,
                                 "basis": "ncu smsp__inst_executed per token (profiles/inst_per_token.json) "
                                          "x tokens per launch / CUDA-event duration; peak = SMs x 4 "
                                          "schedulers x median SM clock under load"}
        cpu = cpu_baseline(mf, args) if world == 1 else None
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(t_max / K, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded Zipf lexicon text, BASELINE config 1 shapes)",
            "mb_per_s": round(all_bytes * K / (t_max / 1e3) / 1e6, 3),
            "config": {"workload": "config1: shipped v001_eng.czm, L5 ctx 1024, "
                                   f"{args.docs} docs x {DOC_BYTES} B per GPU",
                       "model": "v001_eng.czm (d384, 1 layer, 6 heads, MQA, d_ff 1024, V 1024)",
                       "ctx_len": args.ctx, "docs_per_gpu": args.docs,
                       "tokens_per_gpu": n_tok, "chunks_per_gpu": n_chunks,
                       "input_bytes_per_gpu": nbytes, "parallelism": f"dp{world} (documents)",
                       "l2": "flushed before each timed step (256 MiB write, untimed)"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * n_tok,
                    "d2h_bytes_per_step": int(nout_h + 4 * n_chunks),
                    "mb_per_s": round(all_bytes * K / (t_e2e_max / 1e3) / 1e6, 3),
                    "bytes_identical_to_device_path": parity},
            "roofline": roofline,
            "kernels_ms_per_step": {k: round(v / K, 3) for k, v in kern_ms.items()},
            "gpu_launches": int(launches),
            "clocks": clk,
            "compressed_bytes_per_gpu": int(nout),
        }
        if dec is not None:
            line["decode"] = dec
        if cfg2 is not None:
            line["config2"] = cfg2
        if cfg4 is not None:
            line["config4"] = cfg4
        if pipe is not None:
            line["host_pipeline"] = pipe
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()


def arch2_bench(mf, rank, args, stream, local, cfg):
    """BASELINE configuration 2 (cfg 2: documents of 64 KiB, seeds 3000.., at ctx 512)
    or a bounded sample of configuration 4 (cfg 4: documents of 64 KiB, seeds
    10000.., at ctx 4096; the configuration itself is a 1 GB corpus) compressed with
    the arch-2 model (d 512, 8 layers, 8 heads, 2 KV heads, d_ff 2048; synthetic
    int8 weights from seed 7, compress_zip_b200/synth.py) at that context.  Rank r
    takes seeds +r*N.  Tokens resident in HBM, L2 flushed before each timed step,
    CUDA events on the engine's stream; the per-kernel split gives the GEMMs' int8
    tensor throughput.  Each rank reports its own figure (no collective here)."""
    import torch
    from compress_zip_b200.engine import Engine

    ctx, n_docs, first = (512, args.config2_docs, 3000) if cfg == 2 else (4096, args.config4_docs, 10000)
    model = synth.arch2_model(mf, ctx)
    a = synth.ARCH2
    tok = mf.tokenizer()
    docs = synth.documents(shard_seeds(rank, n_docs, first=first), 65536)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    starts, b = [0], 0
    for t in ids:
        for s0 in range(0, len(t), ctx):
            starts.append(b + min(s0 + ctx, len(t)))
        b += len(t)
    tokens = np.concatenate([np.asarray(t, dtype=np.uint32) for t in ids])
    starts = np.asarray(starts, dtype=np.uint64)
    n_tok, n_chunks = int(len(tokens)), int(len(starts) - 1)
    eng = Engine(model, local)
    try:
        eng.set_stream(stream.cuda_stream)
        d_tokens = torch.from_numpy(tokens.view(np.int32)).to(f"cuda:{local}")
        out = np.empty(4 * n_tok + 8 * n_chunks, dtype=np.uint8)
        lens = np.empty(n_chunks, dtype=np.uint32)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
        eng.set_kernel_timing(True)
        eng.compress_device(d_tokens.data_ptr(), starts, out, lens)   # warm-up
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        steps = max(1, min(args.steps, 2))
        times, kern = [], {}
        for _ in range(steps):
            flush.zero_()
            ev0.record(stream)
            eng.compress_device(d_tokens.data_ptr(), starts, out, lens)
            ev1.record(stream)
            torch.cuda.synchronize()
            times.append(ev0.elapsed_time(ev1))
            for k, v in eng.last_stats()["kernels"].items():
                kern[k] = kern.get(k, 0.0) + v["ms"]
    finally:
        eng.close()
    t = sum(times)
    d, dff, kvd, L, V = a["d_model"], a["d_ff"], a["n_kv_heads"] * 64, a["n_layers"], a["vocab_size"]
    macs = {"gemm_qkv": (d + 2 * kvd) * d * L, "gemm_o": d * d * L, "gemm_up_reglu": 2 * dff * d * L,
            "gemm_down": d * dff * L, "head_cdf": V * d, "gemm_head": V * d}
    gemm_ms = sum(kern.get(k, 0.0) for k in macs)
    gemm_ops = sum(2.0 * m * n_tok * steps for k, m in macs.items() if kern.get(k, 0.0) > 0)
    _, _, bf16_sus, basis = peaks()
    tops = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    return {"metric": f"compress tokens/s (config {cfg}{'' if cfg == 2 else ' sample'}: arch-2 model, "
                      f"ctx {ctx}, 64 KiB docs)",
            "value": round(n_tok * steps / (t / 1e3), 1), "unit": "tokens/s", "steps": steps,
            "ms_per_step": round(t / steps, 3), "docs_per_gpu": n_docs, "tokens_per_gpu": n_tok,
            "chunks_per_gpu": n_chunks,
            "mb_per_s": round(sum(len(x.encode()) for x in docs) * steps / (t / 1e3) / 1e6, 3),
            "kernels_ms_per_step": {k: round(v / steps, 3) for k, v in kern.items() if v > 0},
            "gemm_tensor": {"achieved": round(tops, 1), "unit": "TOP/s (int8, 2 x MACs)",
                            "peak": round(2.0 * bf16_sus, 1), "frac": round(tops / (2.0 * bf16_sus), 4),
                            "peak_basis": f"2 x bf16_tflops_sustained {basis} (dense int8 = 2 x bf16)",
                            "kernels": "QKV, O, up+ReGLU, down GEMMs and the head GEMM of head_cdf, "
                                       "CUDA-event time per class"},
            "model": "arch-2 synthetic (d 512, 8 layers, 8 heads, 2 KV heads, d_ff 2048, V 1024)"}


def decode_bench(eng, mf, rank, args, stream, world):
    """decompression of 4,096 independent streams, each
    the chunks of a 4 KB document at L4 (ctx 512), seeds 2000.. (rank r: +r*4096).
    The chunks are produced by the engine itself (untimed); the timed region is
    czg_decompress_chunks from host bytes to host tokens (H2D/D2H inside), CUDA
    events on the engine's stream; the tokens must equal the originals."""
    import torch

    tok = mf.tokenizer()
    docs = synth.documents(shard_seeds(rank, args.decode_docs, first=2000), 4096)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    starts, b = [0], 0
    for t in ids:
        for s0 in range(0, len(t), 512):
            starts.append(b + min(s0 + 512, len(t)))
        b += len(t)
    tokens = np.concatenate([np.asarray(t, dtype=np.uint32) for t in ids])
    starts = np.asarray(starts, dtype=np.uint64)
    counts = np.diff(starts).astype(np.uint32)
    chunks = eng.compress_chunks(tokens, starts)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    # the timed runs go without per-kernel events (thousands of small launches: the
    # events would cost ~15%); one more run with them gives the kernel split
    eng.set_kernel_timing(False)
    got = eng.decompress_chunks(chunks, counts)   # warm-up
    exact = bool(np.array_equal(got, tokens))
    steps = max(1, min(args.steps, 3))
    times, launches = [], 0
    for _ in range(steps):
        torch.cuda.synchronize()
        ev0.record(stream)
        got = eng.decompress_chunks(chunks, counts)
        ev1.record(stream)
        torch.cuda.synchronize()
        times.append(ev0.elapsed_time(ev1))
        launches += sum(v["launches"] for v in eng.last_stats()["kernels"].values())
        exact = exact and bool(np.array_equal(got, tokens))
    (t,), (n_tok,) = reduce_over_ranks([sum(times)], [float(len(tokens))],
                                       f"cuda:{torch.cuda.current_device()}")
    eng.set_kernel_timing(True)
    exact = exact and bool(np.array_equal(eng.decompress_chunks(chunks, counts), tokens))
    kern = eng.last_stats()["kernels"]
    eng.set_kernel_timing(False)
    return {"metric": "batched decode tokens/s (config 3: 4096 x 4 KB docs, L4 ctx 512)",
            "value": round(n_tok * steps / (t / 1e3), 1), "unit": "tokens/s", "steps": steps,
            "ms_per_step": round(t / steps, 3), "streams_per_gpu": int(len(chunks)),
            "tokens_per_gpu": int(len(tokens)), "exact_roundtrip": exact,
            "gpu_launches_per_step": int(launches // steps),
            "kernels_ms_per_step": {k: round(v["ms"], 3) for k, v in kern.items() if v["launches"]},
            "kernel_split": "from one more, untimed run with per-kernel CUDA events"}


def host_pipeline(eng, mf, args):
    """The whole compress CLI path on a bounded sample, stage by stage, labelled apart
    from the hot-path figures: UTF-8 text -> token ids (the native BPE tokenizer,
    csrc/bpe_tokenizer.cpp, on up to 16 host threads) -> the
    GPU coder through the C ABI (host buffers) -> CZIPv1 container -> outer brotli
    q11 / lgwin 22 (rust/src/main.rs:186-281).  Wall clock on the host."""
    from compress_zip_b200 import container, outer_codec
    from compress_zip_b200.cli import hash_model_path

    docs = synth.documents(range(1, args.pipeline_docs + 1), DOC_BYTES)
    text_bytes = sum(len(d.encode("utf-8")) for d in docs)
    tok = mf.tokenizer()
    t0 = time.perf_counter()
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    t1 = time.perf_counter()
    streams = []
    for t in ids:   # one CZIPv1 stream per document, chunks of ctx (rust/src/main.rs:199-205)
        a = np.asarray(t, dtype=np.uint32)
        nch = (len(a) + args.ctx - 1) // args.ctx
        streams.append((a, np.array([min(i * args.ctx, len(a)) for i in range(nch + 1)], np.uint64)))
    tokens = np.concatenate([a for a, _ in streams])
    starts, base = [0], 0
    for a, st in streams:
        starts.extend(int(base + x) for x in st[1:])
        base += len(a)
    chunks = eng.compress_chunks(tokens, np.asarray(starts, np.uint64))
    t2 = time.perf_counter()
    mid = hash_model_path(MODEL)
    jobs, ci = [], 0
    for (a, st), d in zip(streams, docs):
        cf = container.CompressedFile.with_context_length(mid, 0, container.BROTLI, len(d.encode("utf-8")),
                                                          int(np.log2(args.ctx)))
        nch = len(st) - 1
        for k in range(nch):
            n = int(st[k + 1] - st[k])
            cf.add_chunk(chunks[ci], k == nch - 1, n if k == nch - 1 else args.ctx)
            ci += 1
        jobs.append(cf.to_bytes_uncompressed())

    def finish(job):   # the outer codec runs in C (ctypes releases the GIL): one file per thread
        outer, payload = job
        return len(outer) + len(outer_codec.compress(payload, container.BROTLI))

    from concurrent.futures import ThreadPoolExecutor
    nthr = min(16, os.cpu_count() or 1)
    with ThreadPoolExecutor(nthr) as ex:
        out_bytes = sum(ex.map(finish, jobs))
    t3 = time.perf_counter()
    mbs = lambda dt: round(text_bytes / dt / 1e6, 3)
    return {"sample": f"{args.pipeline_docs} docs x {DOC_BYTES} B (seeds 1..{args.pipeline_docs}), "
                      f"{len(tokens)} tokens, one CZIPv1 file per document",
            "input_bytes": text_bytes, "output_bytes": out_bytes,
            "tokenize_mb_per_s": mbs(t1 - t0),
            "tokenizer": "native" if tok.native is not None else "tiktoken",
            "gpu_coder_mb_per_s": mbs(t2 - t1),
            "container_brotli_mb_per_s": mbs(t3 - t2), "container_brotli_threads": nthr,
            "total_mb_per_s": mbs(t3 - t0),
            "clock": "host wall clock, one pass after the timed steps"}


def _oracle_sample(mf, ndocs, ctx):
    tokens, starts, nbytes = workload(mf, range(1, ndocs + 1), ctx)
    return tokens, starts, nbytes


def cpu_baseline(mf, args):
    """The C oracle (port of the reference's Rust path) on all host cores over the
    first --cpu-sample-docs documents of the workload."""
    from oracle import oracle as O

    om = O.load_model(MODEL)
    tokens, starts, nbytes = _oracle_sample(mf, args.cpu_sample_docs, args.ctx)
    cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    O.compress_chunks(om, tokens, starts, nthreads=cores, variant="avx2")
    dt = time.perf_counter() - t0
    # the same source built for the generic x86-64 target (the reference's release profile)
    g_docs = max(1, args.cpu_sample_docs // 4)
    g_end = int(np.searchsorted(starts, starts[-1] * g_docs / args.cpu_sample_docs))
    g_starts = starts[: g_end + 1]
    t1 = time.perf_counter()
    O.compress_chunks(om, tokens[: int(g_starts[-1])], g_starts, nthreads=cores, variant="generic")
    dg = time.perf_counter() - t1
    return {"value": round(len(tokens) / dt, 1), "unit": "tokens/s", "cores": cores,
            "kind": "port", "mb_per_s": round(nbytes / dt / 1e6, 4),
            "value_generic_x86_64": round(int(g_starts[-1]) / dg, 1),
            "sample": f"{args.cpu_sample_docs} docs x {DOC_BYTES} B (seeds 1..{args.cpu_sample_docs}), "
                      f"{len(tokens)} tokens, ctx {args.ctx}, {dt:.1f} s; C restatement of the "
                      "reference Rust path built for x86-64-v3 (value) and for generic x86-64 "
                      "(value_generic_x86_64, first quarter of the sample)"}


def run_reference(args, mf, rank, world):
    if rank != 0:
        return 0
    from oracle import oracle as O

    om = O.load_model(MODEL)
    ndocs = 8
    tokens, starts, nbytes = _oracle_sample(mf, ndocs, args.ctx)
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        O.compress_chunks(om, tokens, starts, nthreads=cores, variant="avx2")
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.compress_chunks(om, tokens, starts, nthreads=cores, variant="avx2")
        times.append(time.perf_counter() - t0)
    t = sum(times)
    value = len(tokens) * args.steps / t
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * t / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded Zipf lexicon text, BASELINE config 1 shapes)",
        "impl": "reference",
        "mb_per_s": round(nbytes * args.steps / t / 1e6, 4),
        "config": {"workload": "config1: shipped v001_eng.czm, L5 ctx 1024; each step a bounded "
                               f"sample of {ndocs} docs x {DOC_BYTES} B",
                   "model": "v001_eng.czm", "ctx_len": args.ctx, "tokens_per_step": int(len(tokens))},
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": cores,
                         "kind": "port",
                         "sample": f"{ndocs} docs (seeds 1..{ndocs}), {len(tokens)} tokens per step; "
                                   "C restatement of the reference Rust path built for x86-64-v3 "
                                   "(cargo is absent, the Rust crate cannot be built)"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main() or 0)
