"""Shared fixtures.  Tests marked `gpu` need a CUDA device (a B200); the
rest run on a CPU-only host.  The oracle (oracle/) is the checker."""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
TESTS = ROOT / "tests"
GOLDEN = TESTS / "golden"
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

import cases  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def built():
    """Builds libaion.so and the oracle (no-ops when up to date)."""
    from aion_b200.build import build
    from oracle import oracle as orc
    build()
    orc.build()
    return True


@pytest.fixture(scope="session")
def oracle(built):
    from oracle.oracle import Oracle
    o = Oracle()
    o.set_threads(min(16, os.cpu_count() or 1))
    return o


@pytest.fixture(scope="session")
def golden_tiny():
    return json.loads((GOLDEN / "tiny.json").read_text())


@pytest.fixture(scope="session")
def golden_kat():
    return json.loads((GOLDEN / "kat.json").read_text())


@pytest.fixture(scope="session")
def golden_7b():
    p = GOLDEN / "7b.json"
    if not p.exists():
        pytest.skip("7b fixture not generated")
    return json.loads(p.read_text())


@pytest.fixture(scope="session")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("aion")


@pytest.fixture(scope="session")
def tiny_path(built, workdir, golden_tiny):
    """The tiny int4 checkpoint, written by the product's synthesizer and
    checked against the hash of the reference quantize.c output."""
    import aion_b200 as A
    p = workdir / "tiny_int4.bin"
    A.synth_checkpoint(p, cases.TINY, cases.SEEDS["tiny"], int4=True)
    assert hashlib.sha256(p.read_bytes()).hexdigest() == golden_tiny["int4_sha"]
    return p


@pytest.fixture(scope="session")
def tiny_f32_path(built, workdir, golden_tiny):
    """The tiny model as an fp32 llama2.c file (the input of quantize.c),
    checked against the hash recorded with the reference's fixtures."""
    import aion_b200 as A
    p = workdir / "tiny_f32.bin"
    A.synth_checkpoint(p, cases.TINY, cases.SEEDS["tiny"], int4=False)
    assert hashlib.sha256(p.read_bytes()).hexdigest() == golden_tiny["fp32_sha"]
    return p


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda(built):
    if not cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    torch.cuda.init()
    return torch


def _sha(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


@pytest.fixture(scope="session")
def ckpt7b(cuda, golden_7b):
    import aion_b200 as A
    d = Path(os.environ.get("AION_CKPT_DIR", Path(tempfile.gettempdir()) / "aion_ckpt"))
    d.mkdir(parents=True, exist_ok=True)
    path = d / "llama2_7b_seed1.int4"
    done = path.with_suffix(".done")
    if not done.exists():
        tmp = path.with_suffix(".tmp")
        A.synth_checkpoint(tmp, cases.LLAMA7B, cases.SEEDS["7b"], int4=True)
        tmp.rename(path)
        done.write_text("ok")
    assert path.stat().st_size == golden_7b["int4_bytes"]
    assert _sha(path) == golden_7b["int4_sha"]
    return path
