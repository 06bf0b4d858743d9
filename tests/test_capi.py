"""The C-ABI library loads on a GPU-less host and exports every symbol the
header declares; its host-side entry points work without a device."""

from __future__ import annotations

import ctypes as C
import re

import numpy as np

from conftest import PKG, ROOT


def _declared_symbols() -> list[str]:
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fmd_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = PKG.load_library()
    declared = _declared_symbols()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(PKG._lib.EXPORTS) == declared


def test_host_entry_points():
    lib = PKG.load_library()
    assert lib.fmd_version() >= 1
    assert lib.fmd_status_string(PKG._lib.FMD_EOVERFLOW).decode() == "KV cache capacity exceeded"
    cfg = PKG.TextConfig()
    # qwen3.rs:628-633: 2 x batch x heads x positions x dims x bytes, per layer
    per_layer = 2 * 4 * 8 * 1000 * 128 * 2
    assert lib.fmd_cache_bytes(C.byref(cfg.to_c()), PKG._lib.PREC_BF16, 4, 1000) == 28 * per_layer
    assert lib.fmd_cache_bytes(C.byref(cfg.to_c()), PKG._lib.PREC_F32, 4, 1000) == 28 * per_layer * 2


def test_host_quantiser_matches_the_oracle_bit_for_bit():
    from oracle import q8_0

    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0                     # an all-zero block (d = 0)
    w[4, 5] = 1e-30                     # denormal-ish tail
    w[5, :32] = np.linspace(-1, 1, 32)  # exact halves after scaling
    blocks = np.empty((64, 256 // 32, 34), dtype=np.uint8)
    lib = PKG.load_library()
    st = lib.fmd_q8_0_quantize(w.ctypes.data_as(C.POINTER(C.c_float)), 64, 256, blocks.ctypes.data)
    assert st == 0
    assert np.array_equal(blocks, q8_0.to_blocks(*q8_0.quantize(w)))


def test_headers_are_plain_c_and_cxx(tmp_path):
    """Every public header compiles as C99 (what a cgo / bindgen / ctypes user
    parses) and as C++17, on its own and together."""
    import shutil
    import subprocess

    inc = ROOT / "include"
    headers = sorted(inc.glob("*.h"))
    src = tmp_path / "all.c"
    src.write_text("".join(f'#include "{h.name}"\n' for h in headers) + "int main(void) { return 0; }\n")
    for cc, std, lang in (("gcc", "-std=c99", "c"), ("g++", "-std=c++17", "c++")):
        if shutil.which(cc) is None:
            continue
        for f in [*headers, src]:
            r = subprocess.run([cc, std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only", "-x", lang,
                                "-I", str(inc), str(f)], capture_output=True, text=True)
            assert r.returncode == 0, f"{cc} {f.name}:\n{r.stderr}"
