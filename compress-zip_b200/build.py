"""Build libczg.so (CUDA kernels for sm_100a + the C-ABI host engine) and
libczg_tok.so (the host BPE tokenizer, plain C++) in-tree.

    python compress-zip_b200/build.py

Objects go to compress-zip_b200/_build/ (git-ignored); the shared libraries are
compress-zip_b200/libczg.so, which the Python binding (engine.py) loads, and
compress-zip_b200/libczg_tok.so (tokenizer.py).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libczg.so")
TOK_LIB = os.path.join(HERE, "libczg_tok.so")
TOK_SRC = os.path.join(CSRC, "bpe_tokenizer.cpp")
CLI_SRC = os.path.join(CSRC, "czg_cli.cpp")
CLI = os.path.join(HERE, "czg-cli")
CXX = os.environ.get("CXX", "g++")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include"),
         "-I" + CSRC]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cpp")) and os.path.join(CSRC, f) not in (TOK_SRC, CLI_SRC))


def build_tokenizer() -> str:
    """libczg_tok.so: host C++ only (no CUDA), so it also builds and runs without a GPU."""
    deps = [TOK_SRC, os.path.join(CSRC, "unicode_classes.inc"), os.path.join(ROOT, "include", "czg_tok.h")]
    if os.path.exists(TOK_LIB) and os.path.getmtime(TOK_LIB) >= max(os.path.getmtime(d) for d in deps):
        return TOK_LIB
    cmd = [CXX, "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-I" + os.path.join(ROOT, "include"),
           "-I" + CSRC, TOK_SRC, "-o", TOK_LIB]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{CXX} failed on {TOK_SRC}:\n{r.stdout}\n{r.stderr}")
    return TOK_LIB


def _headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "czg.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src, hdr_mtime):
    obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_mtime):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build_cli() -> str:
    """czg-cli: the native compress / decompress command line over both libraries."""
    deps = [CLI_SRC, os.path.join(CSRC, "czm_parse.cpp"), LIB, TOK_LIB,
            os.path.join(ROOT, "include", "czg.h"), os.path.join(ROOT, "include", "czg_tok.h")]
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= max(os.path.getmtime(d) for d in deps):
        return CLI
    cmd = [CXX, "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, CLI_SRC,
           os.path.join(CSRC, "czm_parse.cpp"), "-L" + HERE, "-l:libczg.so", "-l:libczg_tok.so", "-ldl",
           "-Wl,-rpath,$ORIGIN", "-o", CLI]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{CXX} failed on {CLI_SRC}:\n{r.stdout}\n{r.stderr}")
    return CLI


def build(verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    hm = _headers_mtime()
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, hm), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_tokenizer()
    build_cli()
    if verbose:
        print(LIB)
        print(TOK_LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
