"""bench.py's reference arm on CPU: one JSON line with the driver's keys.

The reference arm times the CPU restatement of the reference path (oracle/) on a
bounded sample; this checks the line's contract, not the number."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config"):
        assert k in line, k
    assert line["impl"] == "reference" and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["value"] > 0 and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bench_parity_helpers(shipped_path, shipped_oracle, oracle_mod):
    """The bench's oracle-parity plumbing on CPU: documents -> chunk ranges -> packed
    output slices; the oracle's own packed bytes pass, a planted byte error fails."""
    import numpy as np

    sys.path.insert(0, ROOT)
    import bench
    from compress_zip_b200 import czm

    mf = czm.ModelFile.load(shipped_path)
    tokens, starts, nbytes, doc_chunk0 = bench.workload(mf, range(1, 4), 256, doc_bytes=1500)
    assert doc_chunk0[0] == 0 and doc_chunk0[-1] == len(starts) - 1
    toks, st, (c0, c1) = bench.doc_slice(tokens, starts, doc_chunk0, [1, 2])
    assert st[0] == 0 and len(toks) == int(st[-1]) and c1 - c0 == len(st) - 1
    chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
    out = np.frombuffer(b"".join(chunks), np.uint8).copy()
    lens = np.array([len(c) for c in chunks], np.uint32)
    assert bench.gpu_chunks(out, lens, c0, c1) == chunks[c0:c1]
    good = bench.oracle_parity(shipped_oracle, tokens, starts, doc_chunk0, [1, 2], out, lens)
    assert good["identical"] and good["chunks"] == c1 - c0
    off = int(lens[:c0].sum())
    out[off] ^= 1
    bad = bench.oracle_parity(shipped_oracle, tokens, starts, doc_chunk0, [1, 2], out, lens)
    assert not bad["identical"] and bad["first_bad_chunk"] == c0
    assert bench.parity_ok({"a": good}) and not bench.parity_ok({"a": good, "b": bad})
    # mean attention pairs per position: a chunk of n has n (n + 1) / 2
    assert bench.attention_pairs_per_token(np.array([0, 4, 6], np.uint64)) == (10 + 3) / 6
