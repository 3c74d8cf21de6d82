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
