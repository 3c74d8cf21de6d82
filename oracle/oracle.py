"""ctypes wrapper of the oracle -- TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (the C restatement in aion_oracle.c) and, when
present, the reference builds in oracle/_ref/ (libaionref.so from the
reference's src/kernel_simd.c, libquantref.so from its quantize.c, and the
`quantize` / `kernel_simd` binaries).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg use this module, as the checker.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBORACLE = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


# Where this build recipe reads the reference sources from: AION_REFERENCE,
# else the container's read-only checkout when it is there (the GPU box has
# none and uses the prebuilt _ref/).
REFERENCE_TREE = os.environ.get("AION_REFERENCE") or ("/root/reference" if Path("/root/reference/quantize.c").exists()
                                                      else "")


def build() -> None:
    """Builds liboracle.so (and _ref/ where the reference tree exists)."""
    cmd = ["make", "-s", "-C", str(HERE)]
    if REFERENCE_TREE:
        cmd.append(f"REF={REFERENCE_TREE}")
    subprocess.run(cmd, check=True, capture_output=True)


def _np(a) -> int:
    return a.ctypes.data


class Oracle:
    """The C restatement of the reference int4 path."""

    def __init__(self):
        if not LIBORACLE.exists():
            build()
        L = ctypes.CDLL(str(LIBORACLE))
        sig = {
            "orc_set_threads": (None, [ctypes.c_int]),
            "orc_quantize_buffer": (None, [_P, _P, _P, _I64]),
            "orc_dequant": (None, [_P, _P, _P, _I64]),
            "orc_matvec_w4a16": (None, [_P, _P, _P, _P, _I64, _I64]),
            "orc_quantize_activations": (None, [_P, _P, _P, _I64]),
            "orc_matvec_w4a8": (None, [_P, _P, _P, _P, _P, _I64, _I64]),
            "orc_rmsnorm": (None, [_P, _P, _P, _I64]),
            "orc_softmax": (None, [_P, _I64]),
            "orc_swiglu": (None, [_P, _P, _I64]),
            "orc_int4_file_size": (_I64, [_P]),
            "orc_open": (_P, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]),
            "orc_close": (None, [_P]),
            "orc_config_of": (None, [_P, _P]),
            "orc_logits": (ctypes.POINTER(ctypes.c_float), [_P]),
            "orc_reset": (None, [_P]),
            "orc_tensor": (ctypes.c_int, [_P, ctypes.c_int, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
            "orc_forward": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "orc_fp32_tensor": (_P, [_P, ctypes.c_int]),
            "orc_argmax": (ctypes.c_int, [_P, _I64, _P]),
            "orc_generate": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        self.L = L

    def set_threads(self, n: int) -> None:
        self.L.orc_set_threads(n)

    def quantize_buffer(self, w: np.ndarray):
        w = np.ascontiguousarray(w, np.float32).ravel()
        packed = np.empty(w.size // 2, np.uint8)
        scales = np.empty(w.size // 32, np.float32)
        self.L.orc_quantize_buffer(_np(w), _np(packed), _np(scales), w.size)
        return packed, scales

    def matvec_w4a16(self, x, scales, packed, n, d):
        y = np.empty(d, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self.L.orc_matvec_w4a16(_np(y), _np(x), _np(scales), _np(packed), n, d)
        return y

    def quantize_activations(self, x):
        x = np.ascontiguousarray(x, np.float32)
        qx = np.empty(x.size, np.int8)
        xs = np.empty(x.size // 32, np.float32)
        self.L.orc_quantize_activations(_np(qx), _np(xs), _np(x), x.size)
        return qx, xs

    def matvec_w4a8(self, x, scales, packed, n, d):
        qx, xs = self.quantize_activations(x)
        y = np.empty(d, np.float32)
        self.L.orc_matvec_w4a8(_np(y), _np(qx), _np(xs), _np(scales), _np(packed), n, d)
        return y

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        o = np.empty_like(x)
        self.L.orc_rmsnorm(_np(o), _np(x), _np(w), x.size)
        return o

    def dequant(self, scales, packed, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.orc_dequant(_np(out), _np(np.ascontiguousarray(scales, np.float32)),
                           _np(np.ascontiguousarray(packed, np.uint8)), n)
        return out

    def open(self, path) -> "OracleModel":
        return OracleModel(self, path)


class OracleModel:
    def __init__(self, orc: Oracle, path):
        err = ctypes.create_string_buffer(512)
        h = orc.L.orc_open(str(path).encode(), err, 512)
        if not h:
            raise RuntimeError(err.value.decode())
        self.o, self.h = orc, h
        cfg = np.zeros(7, np.int32)
        orc.L.orc_config_of(h, _np(cfg))
        self.config = tuple(int(v) for v in cfg)
        self.vocab = self.config[5]

    def close(self):
        if self.h:
            self.o.L.orc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self.o.L.orc_reset(self.h)

    def forward(self, token: int, pos: int, mode: int = 0) -> np.ndarray:
        if self.o.L.orc_forward(self.h, token, pos, mode) != 0:
            raise ValueError("bad token/pos")
        return np.ctypeslib.as_array(self.o.L.orc_logits(self.h), (self.vocab,)).copy()

    def generate(self, steps: int, bos: int = 1, mode: int = 0, dump_logits: bool = False):
        toks = np.zeros(steps, np.int32)
        gaps = np.zeros(steps, np.float32)
        logits = np.zeros((steps, self.vocab), np.float32) if dump_logits else None
        self.o.L.orc_generate(self.h, bos, steps, mode, _np(toks), _np(gaps), _np(logits) if dump_logits else None)
        return toks, gaps, logits

    def tensor(self, which: int, layer_elems: int, count: int):
        """(scales, packed) numpy views of `count` elements starting at element
        `layer_elems` of stacked tensor `which` (0 emb, 1 wq, 2 wk, 3 wv,
        4 wo, 5 w1, 6 w2, 7 w3)."""
        sp, pp = _P(), _P()
        self.o.L.orc_tensor(self.h, which, ctypes.byref(sp), ctypes.byref(pp))
        s = np.ctypeslib.as_array(ctypes.cast(sp.value + layer_elems // 32 * 4, ctypes.POINTER(ctypes.c_float)),
                                  (count // 32,))
        p = np.ctypeslib.as_array(ctypes.cast(pp.value + layer_elems // 2, ctypes.POINTER(ctypes.c_uint8)),
                                  (count // 2,))
        return s.copy(), p.copy()

    def fp32_tensor(self, which: int, count: int) -> np.ndarray:
        """Copy of the first `count` floats of fp32 tensor `which` (0 rms_att,
        1 rms_ffn, 2 rms_final, 3 freq_re, 4 freq_im)."""
        ptr = self.o.L.orc_fp32_tensor(self.h, which)
        if not ptr:
            raise ValueError("bad tensor index")
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), (count,)).copy()


class Reference:
    """The reference's own code, built from its sources into oracle/_ref/."""

    def __init__(self):
        lib = REF_DIR / "libaionref.so"
        if not lib.exists():
            raise FileNotFoundError(f"{lib} not built (needs the reference tree)")
        L = ctypes.CDLL(str(lib))
        sig = {
            "ref_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]),
            "ref_logits": (ctypes.POINTER(ctypes.c_float), []),
            "ref_config": (None, [_P]),
            "ref_reset": (None, []),
            "ref_forward": (None, [ctypes.c_int, ctypes.c_int]),
            "ref_forward_w4a8": (None, [ctypes.c_int, ctypes.c_int]),
            "ref_open_f32": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int]),
            "ref_forward_f32": (None, [ctypes.c_int, ctypes.c_int]),
            "ref_generate": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P]),
            "ref_matmul_int4_scalar": (None, [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int]),
            "ref_matmul_int4_neon": (None, [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int]),
            "ref_quantize_activations": (None, [_P, _P, _P, ctypes.c_int]),
            "ref_matmul_w4a8": (None, [_P, _P, _P, _P, _P, ctypes.c_int, ctypes.c_int]),
            "ref_rmsnorm": (None, [_P, _P, _P, ctypes.c_int]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        self.L = L
        q = REF_DIR / "libquantref.so"
        self.Q = None
        if q.exists():
            self.Q = ctypes.CDLL(str(q))
            self.Q.ref_quantize_buffer.restype = None
            self.Q.ref_quantize_buffer.argtypes = [_P, _P, _P, ctypes.c_int]

    def quantize_buffer(self, w):
        w = np.ascontiguousarray(w, np.float32).ravel()
        packed = np.empty(w.size // 2, np.uint8)
        scales = np.empty(w.size // 32, np.float32)
        self.Q.ref_quantize_buffer(_np(w), _np(packed), _np(scales), w.size)
        return packed, scales

    def matmul_int4_scalar(self, x, scales, packed, n, d):
        y = np.empty(d, np.float32)
        self.L.ref_matmul_int4_scalar(_np(y), _np(np.ascontiguousarray(x, np.float32)), _np(scales), _np(packed), n, d)
        return y

    def quantize_activations(self, x):
        x = np.ascontiguousarray(x, np.float32)
        qx = np.empty(x.size, np.int8)
        xs = np.empty(x.size // 32, np.float32)
        self.L.ref_quantize_activations(_np(qx), _np(xs), _np(x), x.size)
        return qx, xs

    def matmul_w4a8(self, x, scales, packed, n, d):
        qx, xs = self.quantize_activations(x)
        y = np.empty(d, np.float32)
        self.L.ref_matmul_w4a8(_np(y), _np(qx), _np(xs), _np(scales), _np(packed), n, d)
        return y

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32).copy()
        w = np.ascontiguousarray(w, np.float32).copy()
        o = np.empty_like(x)
        self.L.ref_rmsnorm(_np(o), _np(x), _np(w), x.size)
        return o

    def open(self, path, threads: int = 4, scalar: bool = True):
        """The reference engine is process-global: open once per process."""
        self.L.ref_open(str(path).encode(), threads, 1 if scalar else 0)
        cfg = np.zeros(7, np.int32)
        self.L.ref_config(_np(cfg))
        self.vocab = int(cfg[5])
        return self

    def open_f32(self, path, threads: int = 1):
        """The reference's fp32 path (the CLI without "int4").  With one
        thread every row takes the 4-lane fused-multiply-add block of
        matmul_block_4x4 (src/kernel_simd.c:547), which the oracle restates."""
        self.L.ref_open_f32(str(path).encode(), threads)
        cfg = np.zeros(7, np.int32)
        self.L.ref_config(_np(cfg))
        self.vocab = int(cfg[5])
        return self

    def generate(self, steps: int, bos: int = 1, w4a8: bool = False, dump_logits: bool = False):
        toks = np.zeros(steps, np.int32)
        gaps = np.zeros(steps, np.float32)
        logits = np.zeros((steps, self.vocab), np.float32) if dump_logits else None
        self.L.ref_generate(bos, steps, 1 if w4a8 else 0, _np(toks), _np(gaps), _np(logits) if dump_logits else None)
        return toks, gaps, logits


def ref_available() -> bool:
    return (REF_DIR / "libaionref.so").exists()
