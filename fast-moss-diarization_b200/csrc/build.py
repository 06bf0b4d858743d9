"""Build `libfmd_decoder.so` in-tree with nvcc for sm_100a.

Usage: python build.py [--force] [--verbose]
The library lands next to the package (`fast-moss-diarization_b200/libfmd_decoder.so`)
so it travels with the source tree. Without --force the library is rebuilt
unless it was built from exactly the current sources, headers and flags (a
SHA-256 of them is stored next to the objects), so a stale binary is never
reused because of file times.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
LIB = PKG / "libfmd_decoder.so"
OBJ_DIR = PKG / "_build"
SOURCES = ["fmd_kernels.cu", "fmd_gemv.cu", "fmd_gemm_tc.cu", "fmd_attn_decode.cu", "fmd_scheduler.cu", "fmd_runtime.cu",
           "fmd_noalloc.cu", "fmd_splice.cu", "fmd_attn_prefill.cu", "fmd_chain.cu", "fmd_proj_tc.cu", "fmd_lm_head_tc.cu",
           "fmd_quant.cu", "fmd_enc_gemm.cu", "fmd_enc_attn.cu", "fmd_enc_misc.cu", "fmd_audio.cu", "fmd_mel.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return cand


def _deps() -> list[Path]:
    return ([HERE / s for s in SOURCES] + sorted(HERE.glob("*.cuh")) + sorted(HERE.glob("*.h")) +
            sorted((ROOT / "include").glob("*.h")))


HASH_FILE = OBJ_DIR / "srchash"


def source_hash() -> str:
    """SHA-256 over the names and contents of every source and header plus the
    compiler flags."""
    h = hashlib.sha256()
    h.update(" ".join(ARCH + _flags()).encode())
    for p in _deps():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def needs_build() -> bool:
    if not LIB.exists() or not HASH_FILE.exists():
        return True
    return HASH_FILE.read_text().strip() != source_hash()


def _flags() -> list[str]:
    return ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
            "-I", str(ROOT / "include")]


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    OBJ_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    digest = source_hash()
    flags = ARCH + _flags()
    if verbose:
        flags += ["-Xptxas", "-v"]

    def compile_one(src: str) -> Path:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        cmd = [cc, *flags, "-c", str(HERE / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-Xcompiler", "-fPIC", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    HASH_FILE.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
