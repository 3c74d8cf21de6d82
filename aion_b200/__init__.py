"""aion_b200 -- B200-native int4 Llama-2 decode (drop-in for AION's int4 path).

Python mirror of the C ABI in include/aion.h (libaion.so, loaded with
ctypes).  Names follow the reference engine (farukalpay/AION,
src/kernel_simd.c): `Model.transformer(token, pos)` is transformer() of
:1014-1169 (int4 branch) and `Model.generate(steps)` is the greedy loop of
main (:1223-1258).  Kernel-level entry points mirror matmul_int4_* (:341,
:377), quantize_activations_neon (:186) and matmul_w4a8_neon (:244).

There is no CPU fallback: if libaion.so is missing or fails to load,
importing the library raises.  Device buffers passed to the kernel-level
calls are torch CUDA tensors (used only as device memory).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "lib" / "libaion.so"

MODE_W4A16 = 0
MODE_W4A8 = 1

_STATUS = {0: "OK", 1: "IO", 2: "FORMAT", 3: "SHAPE", 4: "OOM", 5: "CUDA", 6: "NCCL", 7: "TIMEOUT", 8: "ARG",
           9: "STATE"}


class AionError(RuntimeError):
    """A libaion call returned a non-OK aion_status."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.code = _STATUS.get(status, str(status))
        super().__init__(f"AION_ERR_{self.code}: {message}")


class Sampler(ctypes.Structure):
    """aion_sampler: temperature <= 0 is greedy."""
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("seed", ctypes.c_uint64)]


class Config(ctypes.Structure):
    """The 28-byte checkpoint header (src/kernel_simd.c:40-48)."""
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len")]

    def as_tuple(self):
        return tuple(getattr(self, n) for n, _ in self._fields_)

    @property
    def head_size(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.dim * self.n_kv_heads // self.n_heads


class Opts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("mode", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("max_pos", ctypes.c_int32), ("tp_size", ctypes.c_int32), ("tp_rank", ctypes.c_int32),
                ("nccl_id", ctypes.c_void_p), ("use_graph", ctypes.c_int32), ("wait_ms", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 6)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libaion.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing; build it with `python -m aion_b200.build`")
    L = ctypes.CDLL(str(LIB_PATH))
    P, I32, I64, F, VP = ctypes.POINTER, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
    sigs = {
        "aion_default_opts": (None, [P(Opts)]),
        "aion_last_error": (ctypes.c_char_p, [VP]),
        "aion_load": (I32, [ctypes.c_char_p, P(Opts), P(VP)]),
        "aion_free": (I32, [VP]),
        "aion_get_config": (I32, [VP, P(Config)]),
        "aion_forward": (I32, [VP, I32, I32, VP]),
        "aion_logits_dev": (VP, [VP]),
        "aion_generate": (I32, [VP, I32, I32, VP, P(ctypes.c_double)]),
        "aion_reset": (I32, [VP]),
        "aion_stream": (VP, [VP]),
        "aion_decode_async": (I32, [VP, I32, I32, I32]),
        "aion_tokens": (I32, [VP, VP, I32]),
        "aion_qmatrix_upload": (I32, [VP, VP, I64, I64, I32, P(VP)]),
        "aion_qmatrix_download": (I32, [VP, VP, VP]),
        "aion_qmatrix_free": (I32, [VP]),
        "aion_matvec_w4a16": (I32, [VP, VP, VP, VP]),
        "aion_matvec_w4a8": (I32, [VP, VP, VP, VP]),
        "aion_matvec_w4a16_static": (I32, [VP, VP, VP, VP]),
        "aion_matvec_status": (I32, [VP, VP]),
        "aion_matvec_inject_timeout": (I32, [VP]),
        "aion_gemm_bf16_tn": (I32, [VP, VP, VP, I64, I64, I64, VP]),
        "aion_prefill": (I32, [VP, VP, I32, I32, VP]),
        "aion_decode_batch": (I32, [VP, I32, I32, VP, VP, VP, VP]),
        "aion_get_mode": (I32, [VP]),
        "aion_tokenizer_load": (I32, [ctypes.c_char_p, I32, VP]),
        "aion_tokenizer_free": (None, [VP]),
        "aion_encode": (I32, [VP, ctypes.c_char_p, I32, I32, VP, I32, VP]),
        "aion_decode": (ctypes.c_char_p, [VP, I32, I32]),
        "aion_set_sampler": (I32, [VP, VP]),
        "aion_read_logits": (I32, [VP, VP]),
        "aion_set_sequence": (I32, [VP, I32]),
        "aion_tp_handle": (I32, [VP, VP]),
        "aion_tp_plan": (I32, [P(Config), I32, I32, P(I64)]),
        "aion_quantize_buffer_dev": (I32, [VP, VP, VP, I64, VP]),
        "aion_tp_connect": (I32, [VP, VP]),
        "aion_quantize_activations": (I32, [VP, VP, VP, I64, VP]),
        "aion_quantize_buffer": (None, [VP, VP, VP, I64]),
        "aion_checkpoint_bytes": (I64, [P(I32), ctypes.c_int]),
        "aion_quantize_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p,
                                              ctypes.c_int]),
        "aion_synth_checkpoint": (ctypes.c_int, [ctypes.c_char_p, P(I32), ctypes.c_uint64, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_char_p, ctypes.c_int]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(status: int, ctx=None) -> None:
    if status != 0:
        msg = lib().aion_last_error(ctx)
        raise AionError(status, msg.decode() if msg else "")


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Checkpoint tools
# ---------------------------------------------------------------------------
def checkpoint_bytes(cfg, int4: bool = True) -> int:
    c = (ctypes.c_int32 * 7)(*cfg)
    return int(lib().aion_checkpoint_bytes(c, 1 if int4 else 0))


def synth_checkpoint(path, cfg, seed: int, int4: bool = True, threads: int = 0) -> None:
    """Seeded random-init checkpoint (matrices N(0, 0.02), RMSNorm 1.0, RoPE tables)."""
    c = (ctypes.c_int32 * 7)(*cfg)
    err = ctypes.create_string_buffer(512)
    rc = lib().aion_synth_checkpoint(str(path).encode(), c, seed, 1 if int4 else 0, threads, err, 512)
    if rc != 0:
        raise AionError(rc, err.value.decode())


def quantize_file(src, dst, threads: int = 0) -> None:
    """fp32 llama2.c file -> int4 file in the quantize.c format (quantize.c:119-238)."""
    err = ctypes.create_string_buffer(512)
    rc = lib().aion_quantize_file(str(src).encode(), str(dst).encode(), threads, err, 512)
    if rc != 0:
        raise AionError(rc, err.value.decode())


def quantize_buffer(w: np.ndarray):
    """quantize_buffer (quantize.c:59-109): returns (packed uint8[n/2], scales fp32[n/32])."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    if w.size % 32:
        raise ValueError("size must be a multiple of 32")
    packed = np.empty(w.size // 2, np.uint8)
    scales = np.empty(w.size // 32, np.float32)
    lib().aion_quantize_buffer(_ptr(w), _ptr(packed), _ptr(scales), w.size)
    return packed, scales


# ---------------------------------------------------------------------------
# Model level
# ---------------------------------------------------------------------------
class Tokenizer:
    """llama2.c tokenizer.bin: encode text to token ids, decode ids to text
    (aion_tokenizer_load / aion_encode / aion_decode)."""

    def __init__(self, path, vocab_size: int):
        h = ctypes.c_void_p()
        _check(lib().aion_tokenizer_load(str(path).encode(), vocab_size, ctypes.byref(h)))
        self._h = h

    def encode(self, text: str, bos: bool = True, eos: bool = False) -> list[int]:
        raw = text.encode("utf-8")
        out = np.empty(len(raw) + 3, np.int32)
        n = ctypes.c_int32()
        _check(lib().aion_encode(self._h, raw, 1 if bos else 0, 1 if eos else 0, _ptr(out), out.size, ctypes.byref(n)))
        return out[:n.value].tolist()

    def decode_bytes(self, prev: int, token: int) -> bytes:
        p = lib().aion_decode(self._h, prev, token)
        if p is None:
            raise ValueError(f"token {token} out of range")
        return p

    def decode(self, tokens) -> str:
        """Concatenated text of a token stream (BOS and EOS contribute nothing)."""
        out, prev = b"", -1
        for t in tokens:
            if t not in (1, 2):
                out += self.decode_bytes(prev, t)
            prev = t
        return out.decode("utf-8", errors="replace")

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().aion_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_plan(cfg7, tp_size: int, tp_rank: int) -> dict:
    """Rows and columns that rank tp_rank of tp_size holds (aion_tp_plan)."""
    c = Config(*cfg7)
    out = (ctypes.c_int64 * 9)()
    _check(lib().aion_tp_plan(ctypes.byref(c), tp_size, tp_rank, out))
    keys = ["q0", "q", "kv0", "kv", "hid0", "hid", "vocab0", "vocab", "heads"]
    return dict(zip(keys, list(out)))


class Model:
    """A device-resident int4 model: load_checkpoint_int4 + RunState of the
    reference (src/kernel_simd.c:941-1008), on one B200."""

    def __init__(self, path, device: int = 0, mode: str = "int4", max_pos: int = 0, use_graph: bool = True,
                 max_batch: int = 1, tp_size: int = 1, tp_rank: int = 0, wait_ms: int = 0):
        L = lib()
        o = Opts()
        L.aion_default_opts(ctypes.byref(o))
        o.device = device
        o.mode = {"int4": MODE_W4A16, "w4a16": MODE_W4A16, "w4a8": MODE_W4A8}[mode]
        o.max_pos = max_pos
        o.use_graph = 1 if use_graph else 0
        o.max_batch = max_batch
        o.tp_size = tp_size
        o.tp_rank = tp_rank
        o.wait_ms = wait_ms
        h = ctypes.c_void_p()
        _check(L.aion_load(str(path).encode(), ctypes.byref(o), ctypes.byref(h)))
        self._h = h
        cfg = Config()
        _check(L.aion_get_config(self._h, ctypes.byref(cfg)), self._h)
        self.config = cfg
        self.mode = {MODE_W4A16: "int4", MODE_W4A8: "w4a8", 2: "f32"}[L.aion_get_mode(self._h)]
        self.tp_size = tp_size

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().aion_free(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def transformer(self, token: int, pos: int) -> np.ndarray:
        """Logits of (token, pos); writes the KV cache at pos (src/kernel_simd.c:1014)."""
        out = np.empty(self.config.vocab_size, np.float32)
        _check(lib().aion_forward(self._h, token, pos, _ptr(out)), self._h)
        return out

    forward = transformer

    def prefill(self, tokens) -> np.ndarray:
        """Runs tokens[n_seq][n_tok] through the model at positions 0..n_tok-1
        of sequences 0..n_seq-1 (their KV caches) on the tensor cores;
        returns the logits of each sequence's last position."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.ndim == 1:
            t = t[None, :]
        out = np.empty((t.shape[0], self.config.vocab_size), np.float32)
        _check(lib().aion_prefill(self._h, _ptr(t), t.shape[0], t.shape[1], _ptr(out)), self._h)
        return out

    def decode_batch(self, first_tokens, pos0, steps: int, want_logits: bool = False):
        """Lock-step greedy decode of sequences 0..n-1 from first_tokens[b] at
        positions pos0[b]; returns (tokens[steps + 1][n], logits[n][vocab] of
        the last step or None).  Row i of tokens holds step i's inputs, the
        last row the picks after the last step."""
        f = np.ascontiguousarray(first_tokens, dtype=np.int32).ravel()
        p = np.ascontiguousarray(pos0, dtype=np.int32).ravel()
        if f.size != p.size:
            raise ValueError("first_tokens and pos0 differ in length")
        toks = np.empty((steps + 1, f.size), np.int32)
        lg = np.empty((f.size, self.config.vocab_size // self.tp_size), np.float32) if want_logits else None
        _check(lib().aion_decode_batch(self._h, f.size, steps, _ptr(f), _ptr(p), _ptr(toks),
                                       _ptr(lg) if lg is not None else None), self._h)
        return toks, lg

    def set_sampler(self, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, seed: int = 0) -> None:
        """Next-token rule of the decode calls: greedy when temperature <= 0,
        else a seeded draw with temperature, top-k and top-p (aion_set_sampler)."""
        sp = Sampler(temperature, top_p, top_k, 0, seed)
        _check(lib().aion_set_sampler(self._h, ctypes.byref(sp)), self._h)

    def read_logits(self) -> np.ndarray:
        """Logits of the last step run by decode_async / generate."""
        out = np.empty(self.config.vocab_size // self.tp_size, np.float32)
        _check(lib().aion_read_logits(self._h, _ptr(out)), self._h)
        return out

    def tp_handle(self) -> bytes:
        """This rank's exchange-region handle, for every rank's tp_connect."""
        buf = ctypes.create_string_buffer(64)
        _check(lib().aion_tp_handle(self._h, buf), self._h)
        return buf.raw

    def tp_connect(self, handles) -> None:
        """Maps the other ranks' exchange regions (handles in rank order)."""
        blob = b"".join(handles)
        _check(lib().aion_tp_connect(self._h, ctypes.create_string_buffer(blob, len(blob))), self._h)

    def set_sequence(self, seq: int) -> None:
        """Selects the sequence (KV cache) that forward / decode calls use."""
        _check(lib().aion_set_sequence(self._h, seq), self._h)

    def generate(self, steps: int, bos: int = 1):
        """Greedy decode from `bos`; returns (input token of each step, seconds)."""
        toks = np.zeros(max(steps, 1), np.int32)
        secs = ctypes.c_double()
        _check(lib().aion_generate(self._h, bos, steps, _ptr(toks), ctypes.byref(secs)), self._h)
        return toks[:steps].tolist(), secs.value

    def reset(self) -> None:
        _check(lib().aion_reset(self._h), self._h)

    def decode_async(self, steps: int, token: int = -1, pos: int = -1) -> None:
        """Enqueues `steps` greedy steps without waiting (token/pos < 0: continue)."""
        _check(lib().aion_decode_async(self._h, token, pos, steps), self._h)

    def stream_ptr(self) -> int:
        """The context's cudaStream_t, for events recorded by the caller."""
        return int(lib().aion_stream(self._h) or 0)

    def tokens(self, n: int) -> list[int]:
        """Input tokens of positions [0, n) as recorded on the device."""
        out = np.zeros(max(n, 1), np.int32)
        _check(lib().aion_tokens(self._h, _ptr(out), n), self._h)
        return out[:n].tolist()

    def logits_dev_ptr(self) -> int:
        return int(lib().aion_logits_dev(self._h))


# ---------------------------------------------------------------------------
# Kernel level
# ---------------------------------------------------------------------------
def _dev_ptr(t, dtype_name: str, numel: int) -> int:
    if not (t.is_cuda and t.is_contiguous()):
        raise ValueError("expected a contiguous CUDA tensor")
    if str(t.dtype) != dtype_name or t.numel() < numel:
        raise ValueError(f"expected {dtype_name} with >= {numel} elements, got {t.dtype} x {t.numel()}")
    return t.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


class QMatrix:
    """One int4 matrix [rows][cols] resident on a device, re-tiled (the QWeight
    view of src/kernel_simd.c:113-116, uploaded)."""

    def __init__(self, scales: np.ndarray, packed: np.ndarray, rows: int, cols: int, device: int = 0):
        scales = np.ascontiguousarray(scales, np.float32)
        packed = np.ascontiguousarray(packed, np.uint8)
        if scales.size != rows * cols // 32 or packed.size != rows * cols // 2:
            raise ValueError("scales / packed sizes do not match rows x cols")
        h = ctypes.c_void_p()
        _check(lib().aion_qmatrix_upload(_ptr(scales), _ptr(packed), rows, cols, device, ctypes.byref(h)))
        self._h, self.rows, self.cols, self.device = h, rows, cols, device

    def download(self):
        scales = np.empty(self.rows * self.cols // 32, np.float32)
        packed = np.empty(self.rows * self.cols // 2, np.uint8)
        _check(lib().aion_qmatrix_download(self._h, _ptr(scales), _ptr(packed)))
        return scales, packed

    def matvec_w4a16(self, x, y, stream=None) -> None:
        """y = W x (matmul_int4_*, src/kernel_simd.c:341/377, all rows)."""
        _check(lib().aion_matvec_w4a16(self._h, _dev_ptr(x, "torch.float32", self.cols),
                                       _dev_ptr(y, "torch.float32", self.rows), _stream_ptr(stream)))

    def matvec_w4a8(self, x, y, stream=None) -> None:
        """y = W x with per-32 int8 activations (quantize_activations_neon + matmul_w4a8_neon)."""
        _check(lib().aion_matvec_w4a8(self._h, _dev_ptr(x, "torch.float32", self.cols),
                                      _dev_ptr(y, "torch.float32", self.rows), _stream_ptr(stream)))

    def status(self, stream=None) -> None:
        """Waits for the stream; raises AionError (AION_ERR_TIMEOUT) if a matvec
        on this matrix gave up a bounded wait since the last check."""
        _check(lib().aion_matvec_status(self._h, _stream_ptr(stream)))

    def free(self) -> None:
        if getattr(self, "_h", None):
            lib().aion_qmatrix_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def quantize_activations(x, qx, xs, stream=None) -> None:
    """Per-32 int8 quantization (quantize_activations_neon, src/kernel_simd.c:186)."""
    n = x.numel()
    _check(lib().aion_quantize_activations(_dev_ptr(x, "torch.float32", n), _dev_ptr(qx, "torch.int8", n),
                                           _dev_ptr(xs, "torch.float32", n // 32), n, _stream_ptr(stream)))


__all__ = ["AionError", "Config", "Model", "QMatrix", "checkpoint_bytes", "lib", "quantize_activations",
           "quantize_buffer", "quantize_file", "synth_checkpoint", "MODE_W4A16", "MODE_W4A8"]
