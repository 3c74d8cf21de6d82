"""Failure detection without a GPU fault: a bounded wait that runs out.

The reference has one failure mode, exit(1) on a bad file
(src/kernel_simd.c:908-916); its matmuls spin in their barrier
(:93-106) forever if a worker never arrives.  Here every wait inside the
decode kernels is bounded, and a wait that runs out makes the call return
AION_ERR_TIMEOUT with the context still usable.

The case: a two-rank tensor-parallel context on one GPU whose second rank
(a child process) connects its exchange region but never decodes.  Only
rank 0 launches a kernel; its wait for rank 1's partial rows (a flag that
nothing sets) gives up after opts.wait_ms, the call reports the timeout,
aion_reset clears it, the next call times out the same way (bounded, not a
hang), and afterwards an ordinary context on the same GPU decodes the
reference's stream.  No trap, no bad address, no endless loop; the child
leaves between calls with nothing in flight.
"""
from __future__ import annotations

import multiprocessing as mp
import time

import pytest

pytestmark = pytest.mark.gpu

AION_ERR_TIMEOUT = 7
CFG = (256, 512, 2, 4, 4, 1024, 64)    # shards over 2 ranks: 64-column slices, 32-row vocab tiles
WAIT_MS = 200


def _silent_rank(path: str, conn) -> None:
    """Rank 1: loads its shards, swaps exchange handles, then only waits."""
    import aion_b200 as A
    m = A.Model(path, tp_size=2, tp_rank=1, wait_ms=WAIT_MS)
    conn.send(m.tp_handle())
    h0 = conn.recv()
    m.tp_connect([h0, m.tp_handle()])
    conn.send("connected")
    conn.recv()                          # "exit": rank 0 is done
    m.close()
    conn.send("closed")


def test_tp_wait_runs_out_and_context_recovers(cuda, workdir, tiny_path, golden_tiny):
    import aion_b200 as A
    path = workdir / "tp_fail.int4"
    A.synth_checkpoint(path, CFG, 5, int4=True)
    ctx = mp.get_context("spawn")
    here, there = ctx.Pipe()
    child = ctx.Process(target=_silent_rank, args=(str(path), there), daemon=True)
    child.start()
    try:
        m = A.Model(path, tp_size=2, tp_rank=0, wait_ms=WAIT_MS)
        assert here.poll(120), "rank 1 did not start"
        h1 = here.recv()
        here.send(m.tp_handle())
        m.tp_connect([m.tp_handle(), h1])
        assert here.poll(60) and here.recv() == "connected"
        for _ in range(2):
            t0 = time.monotonic()
            with pytest.raises(A.AionError) as err:
                m.generate(2)
            assert err.value.status == AION_ERR_TIMEOUT
            assert time.monotonic() - t0 < 10.0   # bounded by wait_ms, not a hang
            m.reset()
        m.close()
    finally:
        here.send("exit")
        if here.poll(60):
            here.recv()
        child.join(60)
    assert child.exitcode == 0
    # The GPU and the process stay healthy: an ordinary context decodes the
    # reference's tiny stream.
    with A.Model(tiny_path) as m2:
        toks, _ = m2.generate(16)
    assert toks == golden_tiny["w4a16_tokens"][:16]
