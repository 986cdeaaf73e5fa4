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
    ap.add_argument("--parity", type=int, default=1,
                    help="1: compare GPU bytes with the CPU oracle on samples of every configuration "
                         "(outside the timed regions); a mismatch exits non-zero.  0 skips")
    ap.add_argument("--corpus-mb", type=int, default=0,
                    help="configuration 4 proper (strong scaling): this many MB of 64 KiB documents "
                         "(seeds 10000..; 1024 = the 1 GB corpus) split by document over the ranks, "
                         "compressed once per step with the arch-2 model at ctx 4096; replaces the "
                         "configuration-1 headline.  0 (default) keeps configuration 1")
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


def chunked(ids, ctx):
    """Token arrays of documents -> (tokens, chunk starts, first chunk of each document):
    each document is cut into chunks of ctx tokens, the last one shorter
    (rust/src/main.rs:199-205)."""
    starts, doc_chunk0, base = [0], [0], 0
    for t in ids:
        for s in range(0, len(t), ctx):
            starts.append(base + min(s + ctx, len(t)))
        base += len(t)
        doc_chunk0.append(len(starts) - 1)
    tokens = np.concatenate([np.asarray(t, dtype=np.uint32) for t in ids])
    return tokens, np.asarray(starts, dtype=np.uint64), doc_chunk0


def workload(mf, seeds, ctx, doc_bytes=DOC_BYTES):
    tok = mf.tokenizer()
    docs = synth.documents(seeds, doc_bytes)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    tokens, starts, doc_chunk0 = chunked(ids, ctx)
    return tokens, starts, sum(len(d.encode()) for d in docs), doc_chunk0


def doc_slice(tokens, starts, doc_chunk0, docs):
    """Tokens and chunk starts (rebased to 0) of a run of consecutive documents."""
    c0, c1 = doc_chunk0[docs[0]], doc_chunk0[docs[-1] + 1]
    st = starts[c0:c1 + 1]
    return tokens[int(st[0]):int(st[-1])], st - st[0], (c0, c1)


def gpu_chunks(out, lens, c0, c1):
    """Chunks c0..c1-1 of a packed output (chunk bytes back to back in chunk order)."""
    offs = np.concatenate([[0], np.cumsum(lens, dtype=np.uint64)]).astype(np.int64)
    raw = out[offs[c0]:offs[c1]].tobytes()
    return [raw[offs[i] - offs[c0]:offs[i + 1] - offs[c0]] for i in range(c0, c1)]


def oracle_parity(om, tokens, starts, doc_chunk0, docs, out, lens):
    """The CPU oracle's bytes for the given documents against the GPU's bytes for them."""
    from oracle import oracle as O

    toks, st, (c0, c1) = doc_slice(tokens, starts, doc_chunk0, docs)
    want = O.compress_chunks(om, toks, st, nthreads=os.cpu_count() or 1, variant="avx2")
    got = gpu_chunks(out, lens, c0, c1)
    bad = [i for i, (a, b) in enumerate(zip(got, want)) if a != b]
    return {"docs": [int(docs[0]), int(docs[-1])] if len(docs) > 1 else [int(docs[0])],
            "chunks": int(c1 - c0), "tokens": int(len(toks)),
            "identical": len(got) == len(want) and not bad,
            **({"first_bad_chunk": int(bad[0] + c0)} if bad else {})}


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


def gemm_macs(info: dict) -> dict:
    """int8 MACs per token of each GEMM class as the engine computes them (the QKV
    GEMM computes the d + 128 rows the reference reads, rust/src/attention.rs:174-194)."""
    d, dff, V, L = info["d_model"], info["d_ff"], info["vocab_size"], info["n_layers"]
    return {"gemm_qkv": (d + 128) * d * L, "gemm_o": d * d * L, "gemm_up_reglu": 2 * dff * d * L,
            "gemm_down": d * dff * L, "gemm_head": V * d, "head_cdf": V * d}


def attention_pairs_per_token(starts) -> float:
    """Mean (query, key) pairs per position and head: a chunk of n positions has
    n (n + 1) / 2 (position p attends to keys 0..p)."""
    n = np.diff(np.asarray(starts, dtype=np.int64)).astype(np.float64)
    return float((n * (n + 1) / 2).sum() / max(1.0, n.sum()))


# Algorithmic integer ALU work per token beyond the GEMMs (bench and DESIGN figures):
# ~20 integer operations per (query, key, head) pair of the exact softmax (score
# rounding, running max, exp lookup, weight) and ~20 per logit of the CDF
# (exp lookup, frequency division, prefix sums).
ALU_OPS_PER_PAIR = 20
ALU_OPS_PER_LOGIT = 20


def roofline_object(dom, info, pairs_per_tok, tok_per_launch, per_launch_ms, hbm, bf16, basis, sms, mhz) -> dict:
    """The dominant kernel against its rooflines.  For the attention the contract's
    primary ``bound`` is the int8 tensor pipe (QK^T and P.V: 2 x 64 MACs per (query,
    key, head) pair); ``hbm`` (its algorithmic bytes) and ``issue`` (warp instructions
    against 4 per cycle per SM) are given beside it."""
    d, H, L = info["d_model"], info["n_heads"], info["n_layers"]
    secs = per_launch_ms / 1e3
    tpt = traffic_per_token().get(dom)
    if dom == "attention":
        ops = 2.0 * 128 * pairs_per_tok * H * tok_per_launch   # one launch per layer and wave
        achieved = ops / secs / 1e12
        out = {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 3), "peak": round(2 * bf16, 1),
               "unit": "TOP/s", "frac": round(achieved / (2 * bf16), 5),
               "peak_basis": f"2 x bf16_tflops {basis} (dense int8 = 2 x bf16; the kernel runs at the max clock)",
               "algorithmic": "2 x 128 MACs (QK^T 64 + P.V 64) per (query, key, head) pair; "
                              f"{pairs_per_tok:.1f} pairs per position and head in this workload"}
        hb = (128 + 2 * d) * tok_per_launch
        out["hbm"] = {"achieved": round(hb / secs / 1e9, 1), "peak": hbm, "unit": "GB/s",
                      "frac": round(hb / secs / 1e9 / hbm, 5),
                      "algorithmic": "K/V row 128 B + Q row d B read, output d B written, per position"}
    else:
        macs = gemm_macs(info).get(dom)
        if macs is not None:
            ops = 2.0 * macs * tok_per_launch / (L if dom not in ("gemm_head", "head_cdf") else 1)
            achieved = ops / secs / 1e12
            out = {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 3), "peak": round(2 * bf16, 1),
                   "unit": "TOP/s", "frac": round(achieved / (2 * bf16), 5),
                   "peak_basis": f"2 x bf16_tflops {basis} (dense int8 = 2 x bf16)"}
        else:
            V = info["vocab_size"]
            by = {"cdf": 4 * V + 12, "encode": 9.2}.get(dom, 0.0) * tok_per_launch
            out = {"kernel": dom, "bound": "hbm", "achieved": round(by / secs / 1e9, 1), "peak": hbm,
                   "unit": "GB/s", "frac": round(by / secs / 1e9 / hbm, 5), "peak_basis": f"hbm_gbs {basis}"}
    out["traffic"] = None if tpt is None else round(tpt * tok_per_launch)
    out["traffic_basis"] = ("ncu dram__bytes_read.sum + dram__bytes_write.sum per token of a 24-document "
                            "capture (profiles/dram_bytes_per_token.json) x tokens per launch")
    ipt = per_token("inst_per_token.json").get(dom)
    if ipt is not None:
        issued = ipt * tok_per_launch / secs / 1e9
        peak_i = sms * 4 * mhz / 1e3
        out["issue"] = {"achieved": round(issued, 1), "peak": round(peak_i, 1),
                        "unit": "G warp instructions/s", "frac": round(issued / peak_i, 4),
                        "inst_per_token": ipt,
                        "basis": "ncu smsp__inst_executed per token (profiles/inst_per_token.json) x tokens "
                                 "per launch / CUDA-event duration; peak = SMs x 4 schedulers x median SM "
                                 "clock under load"}
    return out


def pipeline_bound(info, pairs_per_tok, value, bf16, sms, mhz, basis) -> dict:
    """Whole-pipeline bound: tokens/s against min(GEMM-bound, ALU-bound tokens/s).
    GEMM bound: int8 GEMM ops per token at 2 x the measured bf16 peak.  ALU bound:
    the algorithmic integer work of the softmax and the CDF per token at one
    operation per lane per cycle (SMs x 128 lanes x clock)."""
    gemm_ops = 2.0 * sum(v for k, v in gemm_macs(info).items() if k != "head_cdf")
    gemm_tps = 2 * bf16 * 1e12 / gemm_ops
    alu_ops = (ALU_OPS_PER_PAIR * pairs_per_tok * info["n_heads"] * info["n_layers"]
               + ALU_OPS_PER_LOGIT * info["vocab_size"])
    alu_tps = sms * 128 * mhz * 1e6 / alu_ops
    bound = min(gemm_tps, alu_tps)
    return {"gemm_bound_tokens_per_s": round(gemm_tps, 1), "alu_bound_tokens_per_s": round(alu_tps, 1),
            "frac": round(value / bound, 4), "gemm_ops_per_token": gemm_ops, "alu_ops_per_token": alu_ops,
            "basis": f"GEMM: 2 x bf16_tflops {basis}; ALU: {ALU_OPS_PER_PAIR} ops per (query, key, head) pair "
                     f"+ {ALU_OPS_PER_LOGIT} per logit at SMs x 128 lanes x median SM clock"}


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

    if args.corpus_mb > 0:
        return corpus_bench(args, mf, rank, world, local)
    seeds = shard_seeds(rank, args.docs)
    tokens, starts, nbytes, doc_chunk0 = workload(mf, seeds, args.ctx)
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
    e2e_same = bytes(h_out_np[:nout_h]) == bytes(out[:nout])

    # parity at benchmark scale (rank 0, untimed): the oracle's bytes for the first
    # documents and for the documents of the last wave against the timed run's bytes
    parity = {}
    if args.parity and rank == 0:
        from oracle import oracle as O

        om1 = O.load_model(MODEL)
        first = list(range(min(args.cpu_sample_docs, args.docs)))
        last = list(range(max(0, args.docs - 8), args.docs))
        parity["config1_first_docs"] = oracle_parity(om1, tokens, starts, doc_chunk0, first, out, lens)
        parity["config1_last_wave"] = oracle_parity(om1, tokens, starts, doc_chunk0, last, out, lens)

    dec = decode_bench(eng, mf, rank, args, stream, world, parity) if args.decode_docs > 0 else None
    cfg2 = arch2_bench(mf, rank, args, stream, local, 2, parity) if args.config2_docs > 0 else None
    cfg4 = arch2_bench(mf, rank, args, stream, local, 4, parity) if args.config4_docs > 0 else None
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
        mhz = (clk or {}).get("sm_mhz") or 1965.0
        sms = torch.cuda.get_device_properties(local).multi_processor_count
        ppt = attention_pairs_per_token(starts)
        roofline = roofline_object(dom, eng.info, ppt, tok_per_launch, per_launch_ms, hbm, bf16, basis, sms, mhz)
        roofline["pipeline"] = pipeline_bound(eng.info, ppt, value, bf16, sms, mhz, basis)
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
                    "bytes_identical_to_device_path": e2e_same},
            "roofline": roofline,
            "parity": parity if parity else None,
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
    if rank == 0 and not parity_ok(parity):
        print("parity FAILED: GPU bytes differ from the CPU oracle (see the parity object)", file=sys.stderr)
        return 1
    return 0


def parity_ok(parity) -> bool:
    return all(v.get("identical", False) for v in (parity or {}).values())


def arch2_bench(mf, rank, args, stream, local, cfg, parity):
    """BASELINE configuration 2 (cfg 2: documents of 64 KiB, seeds 3000.., at ctx 512)
    or a bounded sample of configuration 4 (cfg 4: documents of 64 KiB, seeds
    10000.., at ctx 4096; the configuration itself is a 1 GB corpus, --corpus-mb)
    compressed with the arch-2 model (d 512, 8 layers, 8 heads, 2 KV heads, d_ff
    2048; synthetic int8 weights from seed 7, compress_zip_b200/synth.py) at that
    context.  Rank r takes seeds +r*N.  Tokens resident in HBM, L2 flushed before
    each timed step, CUDA events on the engine's stream; the per-kernel split gives
    the GEMMs' int8 tensor throughput.  Each rank reports its own figure (no
    collective here).  Rank 0 then compares the first document's chunks with the
    CPU oracle's (parity[f"config{cfg}"])."""
    import torch
    from compress_zip_b200.engine import Engine

    ctx, n_docs, first = (512, args.config2_docs, 3000) if cfg == 2 else (4096, args.config4_docs, 10000)
    model = synth.arch2_model(mf, ctx)
    a = synth.ARCH2
    tok = mf.tokenizer()
    docs = synth.documents(shard_seeds(rank, n_docs, first=first), 65536)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    tokens, starts, doc_chunk0 = chunked(ids, ctx)
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
    if args.parity and rank == 0:
        import tempfile

        from oracle import oracle as O

        with tempfile.NamedTemporaryFile(suffix=".czm") as f:
            f.write(model)
            f.flush()
            om = O.load_model(f.name)
        parity[f"config{cfg}"] = oracle_parity(om, tokens, starts, doc_chunk0, [0], out, lens)
    t = sum(times)
    macs = gemm_macs(a)
    gemm_ms = sum(kern.get(k, 0.0) for k in macs)
    gemm_ops = sum(2.0 * m * n_tok * steps for k, m in macs.items() if kern.get(k, 0.0) > 0)
    _, bf16, bf16_sus, basis = peaks()
    tops = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
    return {"metric": f"compress tokens/s (config {cfg}{'' if cfg == 2 else ' sample'}: arch-2 model, "
                      f"ctx {ctx}, 64 KiB docs)",
            "value": round(n_tok * steps / (t / 1e3), 1), "unit": "tokens/s", "steps": steps,
            "ms_per_step": round(t / steps, 3), "docs_per_gpu": n_docs, "tokens_per_gpu": n_tok,
            "chunks_per_gpu": n_chunks,
            "mb_per_s": round(sum(len(x.encode()) for x in docs) * steps / (t / 1e3) / 1e6, 3),
            "kernels_ms_per_step": {k: round(v / steps, 3) for k, v in kern.items() if v > 0},
            "gemm_tensor": {"achieved": round(tops, 1), "unit": "TOP/s (int8, 2 x MACs)",
                            "peak": round(2.0 * bf16, 1), "frac": round(tops / (2.0 * bf16), 4),
                            "peak_sustained": round(2.0 * bf16_sus, 1),
                            "frac_sustained": round(tops / (2.0 * bf16_sus), 4),
                            "peak_basis": f"2 x bf16_tflops {basis} (burst; dense int8 = 2 x bf16); "
                                          "frac_sustained against 2 x bf16_tflops_sustained",
                            "kernels": "QKV (d + 128 rows computed), O, up+ReGLU, down GEMMs and the head "
                                       "GEMM of head_cdf, CUDA-event time per class"},
            "model": "arch-2 synthetic (d 512, 8 layers, 8 heads, 2 KV heads, d_ff 2048, V 1024)"}


def decode_bench(eng, mf, rank, args, stream, world, parity):
    """decompression of 4,096 independent streams, each
    the chunks of a 4 KB document at L4 (ctx 512), seeds 2000.. (rank r: +r*4096).
    The chunks are produced by the engine itself (untimed); the timed region is
    czg_decompress_chunks from host bytes to host tokens (H2D/D2H inside) into one
    reused host buffer, CUDA events on the engine's stream; the tokens must equal
    the originals.  Rank 0
    then encodes the first and last 32 documents with the CPU oracle: its bytes
    must equal the GPU's, and the GPU must decode the oracle's streams back to the
    tokens (parity["config3"])."""
    import torch

    tok = mf.tokenizer()
    docs = synth.documents(shard_seeds(rank, args.decode_docs, first=2000), 4096)
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    tokens, starts, doc_chunk0 = chunked(ids, 512)
    counts = np.diff(starts).astype(np.uint32)
    chunks = eng.compress_chunks(tokens, starts)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    # the timed runs go without per-kernel events (thousands of small launches: the
    # events would cost ~15%); one more run with them gives the kernel split
    eng.set_kernel_timing(False)
    # the decoded tokens land in one host buffer reused by every run (as a streaming
    # caller would); it is overwritten with 0xFFFFFFFF before each run, untimed, so a
    # token a run fails to write cannot pass the check
    dec_out = np.empty(max(len(tokens), 1), dtype=np.uint32)
    got = eng.decompress_chunks(chunks, counts, out=dec_out)   # warm-up
    exact = bool(np.array_equal(got, tokens))
    steps = max(1, min(args.steps, 3))
    times, launches = [], 0
    for _ in range(steps):
        dec_out.fill(0xFFFFFFFF)
        torch.cuda.synchronize()
        ev0.record(stream)
        got = eng.decompress_chunks(chunks, counts, out=dec_out)
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
    if args.parity and rank == 0:
        from oracle import oracle as O

        om = O.load_model(MODEL)
        nd = len(ids)
        sample = sorted(set(range(min(32, nd))) | set(range(max(0, nd - 32), nd)))
        ok_bytes, ok_tokens, n_ch, n_tk = True, True, 0, 0
        for run in (sample[: len(sample) // 2], sample[len(sample) // 2:]):
            toks, st, (c0, c1) = doc_slice(tokens, starts, doc_chunk0, run)
            want = O.compress_chunks(om, toks, st, nthreads=os.cpu_count() or 1, variant="avx2")
            ok_bytes = ok_bytes and want == chunks[c0:c1]
            back = eng.decompress_chunks(want, np.diff(st).astype(np.uint32))
            ok_tokens = ok_tokens and bool(np.array_equal(back, toks))
            n_ch += c1 - c0
            n_tk += len(toks)
        parity["config3"] = {"docs": [sample[0], sample[-1]], "chunks": int(n_ch), "tokens": int(n_tk),
                             "identical": ok_bytes and ok_tokens, "gpu_bytes_equal_oracle": ok_bytes,
                             "gpu_decodes_oracle_streams": ok_tokens}
    return {"metric": "batched decode tokens/s (config 3: 4096 x 4 KB docs, L4 ctx 512)",
            "value": round(n_tok * steps / (t / 1e3), 1), "unit": "tokens/s", "steps": steps,
            "ms_per_step": round(t / steps, 3), "streams_per_gpu": int(len(chunks)),
            "tokens_per_gpu": int(len(tokens)), "exact_roundtrip": exact,
            "gpu_launches_per_step": int(launches // steps),
            "kernels_ms_per_step": {k: round(v["ms"], 3) for k, v in kern.items() if v["launches"]},
            "kernel_split": "from one more, untimed run with per-kernel CUDA events"}


def _corpus_docs(bounds):
    """Documents of seeds [lo, hi) (a worker of corpus_bench's generation pool)."""
    lo, hi = bounds
    return synth.documents(range(lo, hi), 65536)


def corpus_range(rank, world, n_docs):
    """Rank `rank`'s contiguous share [lo, hi) of n_docs documents (strong scaling)."""
    return rank * n_docs // world, (rank + 1) * n_docs // world


def corpus_documents(lo, hi, workers):
    """synth.documents over seeds [lo, hi), split over a pool of spawned processes
    (untimed setup: a 1 GB corpus takes minutes in one process)."""
    if workers <= 1 or hi - lo < 256:
        return synth.documents(range(lo, hi), 65536)
    import multiprocessing as mp

    cuts = [lo + (hi - lo) * i // workers for i in range(workers + 1)]
    with mp.get_context("spawn").Pool(workers) as pool:
        parts = pool.map(_corpus_docs, [(cuts[i], cuts[i + 1]) for i in range(workers)])
    return [d for part in parts for d in part]


def corpus_bench(args, mf, rank, world, local):
    """Configuration 4 proper: a corpus of args.corpus_mb MB of 64 KiB documents
    (seeds 10000..) split by document over the ranks (strong scaling: the corpus is
    fixed, each rank compresses its contiguous share), the arch-2 model at ctx 4096.
    A step compresses the rank's whole share once (tokens resident in HBM); warm-up
    runs the first 16 documents of the share.  value = corpus tokens / max over ranks
    of the device time per step.  No collective on the data path: only the timing
    reduction."""
    import torch
    import torch.distributed as dist
    from compress_zip_b200.engine import Engine

    n_docs = args.corpus_mb * (1 << 20) // 65536
    lo, hi = corpus_range(rank, world, n_docs)
    model = synth.arch2_model(mf, 4096)
    tok = mf.tokenizer()
    docs = corpus_documents(10000 + lo, 10000 + hi, max(1, min(16, (os.cpu_count() or 1) // world)))
    ids = tok.encode_batch_arrays(docs, num_threads=min(16, os.cpu_count() or 1))
    tokens, starts, doc_chunk0 = chunked(ids, 4096)
    n_tok, n_chunks, nbytes = int(len(tokens)), int(len(starts) - 1), sum(len(d.encode()) for d in docs)
    del docs
    stream = torch.cuda.current_stream()
    eng = Engine(model, local)
    eng.set_stream(stream.cuda_stream)
    d_tokens = torch.from_numpy(tokens.view(np.int32)).to(f"cuda:{local}")
    out = np.empty(4 * n_tok + 8 * n_chunks, dtype=np.uint8)
    lens = np.empty(n_chunks, dtype=np.uint32)
    w_end = doc_chunk0[min(16, len(ids))]
    for _ in range(max(args.warmup, 1)):
        eng.compress_device(d_tokens.data_ptr(), starts[: w_end + 1], out, lens)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(args.steps):
        ev0.record(stream)
        nout = eng.compress_device(d_tokens.data_ptr(), starts, out, lens)
        ev1.record(stream)
        torch.cuda.synchronize()
        times.append(ev0.elapsed_time(ev1))
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    (t_max,), (all_tok, all_bytes, all_out) = reduce_over_ranks(
        [sum(times)], [float(n_tok), float(nbytes), float(nout)], f"cuda:{local}")
    parity = {}
    if args.parity and rank == 0:
        import tempfile

        from oracle import oracle as O

        with tempfile.NamedTemporaryFile(suffix=".czm") as f:
            f.write(model)
            f.flush()
            om = O.load_model(f.name)
        parity["config4"] = oracle_parity(om, tokens, starts, doc_chunk0, [0], out, lens)
    eng.close()
    if rank == 0:
        K = args.steps
        line = {"metric": "compress tokens/s & MB/s, config 4: 1 GB-class corpus, arch-2 model at ctx 4096",
                "value": round(all_tok * K / (t_max / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
                "steps": K, "warmup": args.warmup, "ms_per_step": round(t_max / K, 3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded Zipf lexicon text, BASELINE config 4 shapes)",
                "mb_per_s": round(all_bytes * K / (t_max / 1e3) / 1e6, 3),
                "config": {"workload": f"config4: {args.corpus_mb} MB = {n_docs} docs x 64 KiB (seeds "
                                       f"10000..{10000 + n_docs - 1}) split by document over {world} GPUs",
                           "model": "arch-2 synthetic (d 512, 8 layers, 8 heads, 2 KV heads, d_ff 2048)",
                           "ctx_len": 4096, "corpus_tokens": int(all_tok), "compressed_bytes": int(all_out),
                           "parallelism": f"dp{world} (documents)",
                           "l2": "inputs (GBs of tokens per rank) far larger than L2"},
                "clocks": clk, "parity": parity or None}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and not parity_ok(parity):
        print("parity FAILED: GPU bytes differ from the CPU oracle", file=sys.stderr)
        return 1
    return 0


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
    tokens, starts, nbytes, _ = workload(mf, range(1, ndocs + 1), ctx)
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
                         "sample": f"{ndocs} docs (seeds 1..{ndocs}), {len(tokens)} tokens in {len(starts) - 1} "
                                   f"chunks per step (one chunk per thread at a time: {cores} threads, "
                                   f"{(len(starts) - 1) / cores:.1f} chunks each); "
                                   "C restatement of the reference Rust path built for x86-64-v3 "
                                   "(cargo is absent, the Rust crate cannot be built)"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main() or 0)
