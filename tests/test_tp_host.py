"""Tensor parallelism on the host: the shard plan (aion_tp_plan, used by the
loader) and the rank data flow of the decode kernel's exchange, run as gloo
ranks on the CPU.

Each rank takes its rows of wq/wk/wv/w1/w3 and of the classifier and its
columns of wo/w2 from the plan, computes its heads' attention and its slice
of the hidden layer with the oracle's int4 matvec (src/kernel_simd.c:341
restated), and sums the ranks' partial rows in rank order after an
all_gather, as the decode kernel does over peer memory; the next token is
the first maximum across ranks (strict '>' in rank order, the argmax of
src/kernel_simd.c:1236-1243).  The result must match the oracle's
single-process forward (src/kernel_simd.c:1014-1169): logits within 1e-4
relative of the largest logit (only the summation order of the partials
and of numpy's dot products differs) and the same greedy tokens.
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest

# dim, hidden, layers, heads, kv_heads (grouped: 2 query heads per K/V head), vocab, seq_len
CFG = (256, 768, 2, 8, 4, 512, 64)
SEED = 11
STEPS = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _first_max(v: np.ndarray):
    best, idx = np.float32(-1e9), 0
    i = int(np.argmax(v))
    if v[i] > best:
        best, idx = v[i], i
    return float(best), idx


def _tp_rank(rank: int, world: int, port: int, path: str, res) -> None:
    try:
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        import aion_b200 as A
        from oracle.oracle import Oracle

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=120))
        o = Oracle()
        om = o.open(path)
        dim, hid, L, nh, nkv, vocab, seq = om.config
        hs, kvd = dim // nh, dim * nkv // nh
        kv_mul = nh // nkv
        p = A.tp_plan(om.config, world, rank)

        def rows(which, layer, n_rows, n_cols, r0, nr):
            s, q = om.tensor(which, (layer * n_rows + r0) * n_cols, nr * n_cols)
            return s, q, n_cols, nr

        def cols(which, layer, n_rows, n_cols, c0, nc):
            s, q = om.tensor(which, layer * n_rows * n_cols, n_rows * n_cols)
            s = s.reshape(n_rows, n_cols // 32)[:, c0 // 32:(c0 + nc) // 32]
            q = q.reshape(n_rows, n_cols // 2)[:, c0 // 2:(c0 + nc) // 2]
            return np.ascontiguousarray(s).ravel(), np.ascontiguousarray(q).ravel(), nc, n_rows

        def mv(x, w):
            return o.matvec_w4a16(x, w[0], w[1], w[2], w[3])

        def reduce_in_rank_order(part):
            got = [torch.empty(part.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(got, torch.from_numpy(part))
            total = np.zeros_like(part)
            for g in got:
                total += g.numpy()
            return total

        W = [dict(wq=rows(1, l, dim, dim, p["q0"], p["q"]), wk=rows(2, l, kvd, dim, p["kv0"], p["kv"]),
                  wv=rows(3, l, kvd, dim, p["kv0"], p["kv"]), wo=cols(4, l, dim, dim, p["q0"], p["q"]),
                  w1=rows(5, l, hid, dim, p["hid0"], p["hid"]), w3=rows(7, l, hid, dim, p["hid0"], p["hid"]),
                  w2=cols(6, l, dim, hid, p["hid0"], p["hid"])) for l in range(L)]
        cls = rows(0, 0, vocab, dim, p["vocab0"], p["vocab"])
        rms_att = om.fp32_tensor(0, L * dim).reshape(L, dim)
        rms_ffn = om.fp32_tensor(1, L * dim).reshape(L, dim)
        rms_final = om.fp32_tensor(2, dim)
        fre = om.fp32_tensor(3, seq * hs // 2).reshape(seq, hs // 2)
        fim = om.fp32_tensor(4, seq * hs // 2).reshape(seq, hs // 2)
        kc = np.zeros((L, seq, p["kv"]), np.float32)
        vc = np.zeros((L, seq, p["kv"]), np.float32)

        def rope(v, pos):
            a, b = v[0::2].copy(), v[1::2].copy()
            fr = np.tile(fre[pos], v.size // hs)
            fi = np.tile(fim[pos], v.size // hs)
            v[0::2] = a * fr - b * fi
            v[1::2] = a * fi + b * fr

        tokens, slices, tok = [], [], 1
        for pos in range(STEPS):
            tokens.append(tok)
            s, q = om.tensor(0, tok * dim, dim)
            x = o.dequant(s, q, dim)
            for l in range(L):
                xb = o.rmsnorm(x, rms_att[l])
                qv, kv, vv = mv(xb, W[l]["wq"]), mv(xb, W[l]["wk"]), mv(xb, W[l]["wv"])
                rope(qv, pos)
                rope(kv, pos)
                kc[l, pos], vc[l, pos] = kv, vv
                att = np.empty(p["q"], np.float32)
                for h in range(p["heads"]):
                    g = h // kv_mul
                    qh = qv[h * hs:(h + 1) * hs]
                    sc = (kc[l, :pos + 1, g * hs:(g + 1) * hs] @ qh) / np.float32(np.sqrt(hs))
                    e = np.exp(sc - sc.max())
                    att[h * hs:(h + 1) * hs] = (e / e.sum()) @ vc[l, :pos + 1, g * hs:(g + 1) * hs]
                x = x + reduce_in_rank_order(mv(att, W[l]["wo"]))
                xb = o.rmsnorm(x, rms_ffn[l])
                h1, h3 = mv(xb, W[l]["w1"]), mv(xb, W[l]["w3"])
                x = x + reduce_in_rank_order(mv((h1 / (1 + np.exp(-h1)) * h3).astype(np.float32), W[l]["w2"]))
            logits = mv(o.rmsnorm(x, rms_final), cls)
            slices.append(logits)
            best, i = _first_max(logits)
            cand = [None] * world
            dist.all_gather_object(cand, (best, p["vocab0"] + i))
            win = (np.float32(-1e9), 0)
            for b, gi in cand:          # strict '>' in rank order: the first maximum wins
                if b > win[0]:
                    win = (b, gi)
            tok = win[1]
        om.close()
        dist.barrier()
        dist.destroy_process_group()
        res.put((rank, p, tokens, np.stack(slices)))
    except Exception as e:  # reported to the parent
        import traceback
        res.put((rank, "error", traceback.format_exc(), repr(e)))


@pytest.fixture(scope="module")
def tp_model(built, workdir):
    import aion_b200 as A
    path = workdir / "tp_host.int4"
    if not path.exists():
        A.synth_checkpoint(path, CFG, SEED, int4=True)
    return path


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ranks_match_oracle(oracle, tp_model, world):
    om = oracle.open(tp_model)
    want, tok = [], 1
    want_tokens = []
    for pos in range(STEPS):
        want_tokens.append(tok)
        lg = om.forward(tok, pos)
        want.append(lg)
        tok = int(np.argmax(lg))
    om.close()
    want = np.stack(want)

    ctx = mp.get_context("spawn")
    res = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, port, str(tp_model), res)) for r in range(world)]
    for pr in procs:
        pr.start()
    try:
        out = [res.get(timeout=300) for _ in range(world)]
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.terminate()
    out = {o[0]: o for o in out}
    for r in range(world):
        assert out[r][1] != "error", out[r][2]
    v0 = 0
    for r in range(world):
        _, plan, toks, slices = out[r]
        assert plan["vocab0"] == v0
        v0 += plan["vocab"]
        assert toks == want_tokens
        ref = want[:, plan["vocab0"]:plan["vocab0"] + plan["vocab"]]
        assert np.abs(slices - ref).max() <= 1e-4 * np.abs(want).max()
    assert v0 == CFG[5]


SHAPES = {
    "llama2-7b": (4096, 11008, 32, 32, 32, 32000, 2048),
    "llama2-13b": (5120, 13824, 40, 40, 40, 32000, 2048),
    "small-gqa": CFG,
}


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_plan_partitions(built, name, world):
    """The ranks' ranges tile every sharded dimension exactly once, in rank order."""
    import aion_b200 as A
    cfg = SHAPES[name]
    dim, hid, _, nh, nkv, vocab, _ = cfg
    if nh % world or nkv % world:
        with pytest.raises(A.AionError):
            A.tp_plan(cfg, world, 0)
        return
    full = {"q": dim, "kv": dim * nkv // nh, "hid": hid, "vocab": vocab}
    nxt = dict.fromkeys(full, 0)
    for r in range(world):
        p = A.tp_plan(cfg, world, r)
        assert p["heads"] * world == nh
        assert p["q"] == p["heads"] * (dim // nh)
        for k in full:
            assert p[k + "0"] == nxt[k] and p[k] > 0
            nxt[k] += p[k]
    assert nxt == full


@pytest.mark.parametrize("cfg,world,rank", [
    ((288, 768, 6, 6, 6, 32000, 256), 2, 0),     # 144-column slice of wo: not whole 32-element groups
    ((288, 768, 6, 6, 6, 32000, 256), 4, 1),     # 6 heads over 4 ranks
    ((256, 768, 2, 8, 4, 520, 64), 2, 0),        # vocab not a multiple of 2 x 16-row tiles
    (CFG, 2, 2),                                 # rank out of range
    (CFG, 0, 0),                                 # no ranks
])
def test_tp_plan_rejects(built, cfg, world, rank):
    import aion_b200 as A
    with pytest.raises(A.AionError):
        A.tp_plan(cfg, world, rank)
