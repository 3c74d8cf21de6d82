"""The C ABI: the library loads, exports every declared entry point, and
rejects bad input on the host before any device work (CPU-only)."""
from __future__ import annotations

import ctypes
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT

import cases


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "aion.h").read_text()
    return re.findall(r"AION_API\s+[\w\s\*]+?\b(aion_\w+)\s*\(", text)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ("aion_load", "aion_forward", "aion_generate", "aion_free", "aion_matvec_w4a16", "aion_matvec_w4a8",
                 "aion_quantize_activations", "aion_qmatrix_upload", "aion_qmatrix_download"):
        assert must in syms


def test_library_exports_every_declared_symbol(built):
    import aion_b200 as A
    lib = A.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(A.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(aion_\w+)", out))
    for s in declared_symbols():
        assert s in exported, s
        assert getattr(lib, s) is not None


def test_header_compiles_as_c11(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "aion.h"\nint main(void){aion_opts o; aion_default_opts(&o); return o.tp_size - 1;}\n')
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-fsyntax-only", "-I", str(ROOT / "include"), str(src)],
                   check=True)


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "aion.h"

int main(int argc, char** argv) {
    /* the binding src/kernel_simd.c would use: opts, load, errors (no GPU work) */
    aion_opts o;
    aion_default_opts(&o);
    aion_ctx* ctx = NULL;
    aion_status s = aion_load(argv[1], &o, &ctx);
    const char* err = aion_last_error(NULL);
    printf("load %d %d\n", (int)s, err && err[0] ? 1 : 0);
    /* quantize_buffer's format: one group of 32 values */
    float w[32];
    for (int i = 0; i < 32; i++) w[i] = (float)(i - 16) * 0.25f;
    uint8_t packed[16];
    float scale;
    aion_quantize_buffer(w, packed, &scale, 32);
    printf("scale %.9g first %u\n", scale, (unsigned)packed[0]);
    const int32_t cfg[7] = {288, 768, 6, 6, 6, 32000, 256};
    printf("bytes %lld %lld\n", (long long)aion_checkpoint_bytes(cfg, 1), (long long)aion_checkpoint_bytes(cfg, 0));
    return ctx != NULL;
}
"""


def test_c_program_links_and_runs(built, tmp_path):
    """A C11 program binds the library the way the reference's C driver
    would (header + -laion) and runs its host-side calls."""
    import aion_b200 as A
    src = tmp_path / "bind.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "bind"
    lib_dir = A.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe),
                    "-L", str(lib_dir), "-laion", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe), str(tmp_path / "missing.int4")], capture_output=True, text=True, check=True).stdout
    lines = dict(l.split(" ", 1) for l in out.strip().splitlines())
    assert lines["load"] == "1 1"                     # AION_ERR_IO with a message
    w = (np.arange(32, dtype=np.float32) - 16) * np.float32(0.25)
    packed = np.zeros(16, np.uint8)
    scales = np.zeros(1, np.float32)
    A.lib().aion_quantize_buffer(w.ctypes.data, packed.ctypes.data, scales.ctypes.data, 32)
    assert lines["scale"] == f"{float(scales[0]):.9g} first {int(packed[0])}"
    int4, f32 = (int(v) for v in lines["bytes"].split())
    assert int4 == A.lib().aion_checkpoint_bytes((ctypes.c_int32 * 7)(*cases.TINY), 1)
    assert f32 == 28 + 4 * (cases.TINY[5] * 288 + 6 * 288 * 2 + 6 * (4 * 288 * 288 + 3 * 288 * 768) + 288 + 256 * 48)


def test_default_opts(built):
    import aion_b200 as A
    o = A.Opts()
    A.lib().aion_default_opts(ctypes.byref(o))
    assert (o.device, o.mode, o.max_batch, o.max_pos, o.tp_size, o.tp_rank, o.use_graph) == (0, 0, 1, 0, 1, 0, 1)


def _load_status(path) -> tuple[int, str]:
    import aion_b200 as A
    h = ctypes.c_void_p()
    st = A.lib().aion_load(str(path).encode(), None, ctypes.byref(h))
    return st, A.lib().aion_last_error(None).decode()


def test_load_missing_file(built, tmp_path):
    st, msg = _load_status(tmp_path / "nope.bin")
    assert st == 1 and "cannot open" in msg


def test_load_truncated_and_inconsistent(built, tmp_path, tiny_path):
    data = tiny_path.read_bytes()
    short = tmp_path / "short.bin"
    short.write_bytes(data[:20])
    assert _load_status(short)[0] == 2
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(data[:-16])
    st, msg = _load_status(trunc)
    assert st == 2 and "header implies" in msg
    longer = tmp_path / "long.bin"
    longer.write_bytes(data + b"\0" * 32)
    assert _load_status(longer)[0] == 2
    bad = tmp_path / "bad.bin"
    hdr = np.frombuffer(data[:28], np.int32).copy()
    hdr[3] = 7          # 288 % 7 != 0
    bad.write_bytes(hdr.tobytes() + data[28:])
    assert _load_status(bad)[0] == 3
    neg = tmp_path / "neg.bin"
    hdr = np.frombuffer(data[:28], np.int32).copy()
    hdr[2] = -1
    neg.write_bytes(hdr.tobytes() + data[28:])
    assert _load_status(neg)[0] == 2


def test_kernel_level_argument_errors(built):
    import aion_b200 as A
    L = A.lib()
    h = ctypes.c_void_p()
    s = np.zeros(1, np.float32)
    p = np.zeros(16, np.uint8)
    assert L.aion_qmatrix_upload(s.ctypes.data, p.ctypes.data, 1, 33, 0, ctypes.byref(h)) == 8
    assert L.aion_qmatrix_upload(s.ctypes.data, p.ctypes.data, 0, 32, 0, ctypes.byref(h)) == 8
    assert L.aion_quantize_activations(None, None, None, 32, None) == 8
    assert L.aion_matvec_w4a16(None, None, None, None) == 8
    assert L.aion_forward(None, 0, 0, None) == 8


def test_python_mirror_raises(built, tmp_path):
    import aion_b200 as A
    with pytest.raises(A.AionError) as e:
        A.Model(tmp_path / "missing.bin")
    assert e.value.code == "IO"
