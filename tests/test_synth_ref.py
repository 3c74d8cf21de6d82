"""The reference arm's checkpoint writer (oracle/_ref/synth_ckpt: the seeded
generator feeding the reference's own quantize_buffer from quantize.c)
writes the same bytes as the library's aion_synth_checkpoint, so both bench
arms and the golden fixtures see one model.  CPU only."""
from __future__ import annotations

import hashlib
import subprocess

import pytest

from oracle.oracle import REF_DIR

SYNTH = REF_DIR / "synth_ckpt"

CONFIGS = [
    ((288, 768, 6, 6, 6, 32000, 256), 0),      # the tiny workload model
    ((256, 512, 3, 8, 4, 1000, 64), 7),         # grouped-query attention, odd seed
    ((512, 1376, 2, 4, 4, 4000, 128), 1),       # 7B-like hidden ratio
]


def _sha(p) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


@pytest.mark.parametrize("cfg,seed", CONFIGS)
def test_reference_writer_matches_library(built, tmp_path, cfg, seed):
    if not SYNTH.exists():
        pytest.skip("oracle/_ref/synth_ckpt not built (no reference tree)")
    import aion_b200 as A
    a, b = tmp_path / "aion.int4", tmp_path / "ref.int4"
    A.synth_checkpoint(a, cfg, seed, int4=True)
    subprocess.run([str(SYNTH), str(b), *map(str, cfg), str(seed), "2"], check=True)
    assert a.stat().st_size == b.stat().st_size
    assert _sha(a) == _sha(b)


def test_reference_writer_rejects_bad_config(tmp_path):
    if not SYNTH.exists():
        pytest.skip("oracle/_ref/synth_ckpt not built (no reference tree)")
    r = subprocess.run([str(SYNTH), str(tmp_path / "x"), "100", "256", "1", "3", "3", "10", "8", "0"],
                       capture_output=True, text=True)
    assert r.returncode != 0 and "invalid config" in r.stderr
