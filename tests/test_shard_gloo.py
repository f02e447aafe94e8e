"""Multi-rank chunk sharding on CPU (gloo, world sizes 2 and 3).

Each rank takes its contiguous chunk range from the library's shard planner
(mbr_plan_shard, host-only), holds only the track window its chunks read
(mbr_plan_shard_window), runs a stand-in per-chunk model, overlap-adds its
chunks with the reference fade windows (src/inference_app.cpp:186-218),
exchanges boundaries with both neighbours at once (its tail to rank + 1, the
previous rank's tail into its head: one batched isend / irecv), and normalises
its disjoint output range — the protocol bench.py runs with NCCL.
The assembled result must equal a single-process restatement of
process_chunked (src/inference_app.cpp:72-232) with the same stand-in model.
"""
import os
import socket

import numpy as np
import pytest

CHUNK, OVERLAP, DEFAULT = 44100, 4.0, 2
N = 7 * 44100 + 321
S, C = 2, 2


def _stand_in_model(x: np.ndarray) -> np.ndarray:
    """[C][chunk] -> [S][C][chunk]; any deterministic per-chunk function."""
    return np.stack([np.tanh(0.7 * x), 0.25 * x + 0.01 * np.roll(x, 1, axis=-1)]).astype(np.float32)


def _reflect(p, n):
    while p < 0 or p >= n:
        if p < 0:
            p = -p
        if p >= n:
            p = 2 * (n - 1) - p
    return p


def _fade(chunk: int):
    fade = chunk // 10
    w = np.ones(chunk, np.float32)
    if fade == 1:
        w[0] = w[-1] = 0
    elif fade > 1:
        a = np.arange(fade, dtype=np.float32) / np.float32(fade - 1)
        w[:fade] = a
        w[chunk - fade:] = np.float32(1) - a
    return w, fade


def _read_index(total, border, padded, st, q, Ntr):
    """Track sample chunk position q of the chunk at padded start st reads (or None)."""
    al = min(CHUNK, total - st)
    if q < al:
        pp = st + q
    elif al > CHUNK // 2:
        pp = st + _reflect(q, al)
    else:
        return None
    return _reflect(pp - border, Ntr) if padded else pp


def _chunk_input(track, total, border, padded, st, tr_lo=0, Ntr=None):
    """Chunk input from `track`, which holds track samples [tr_lo, tr_lo + width)."""
    Ntr = track.shape[1] if Ntr is None else Ntr
    al = min(CHUNK, total - st)
    out = np.zeros((C, CHUNK), np.float32)
    for q in range(CHUNK):
        t = _read_index(total, border, padded, st, q, Ntr)
        if t is not None:
            assert tr_lo <= t < tr_lo + track.shape[1], "chunk reads outside the track window"
            out[:, q] = track[:, t - tr_lo]
    return out, al


def _window(st, al, total, fade, fw):
    w = fw.copy()
    last = st + al >= total
    if fade > 0 and (st == 0 or last):
        if st == 0:
            w[:fade] = 1
        if last:
            w[CHUNK - fade:] = 1
    return w[:al]


def _accumulate(track, plan, c0, c1, lo, hi, tr_lo=0, Ntr=None):
    step, border, total = plan["step"], plan["border"], plan["total"]
    fw, fade = _fade(CHUNK)
    acc = np.zeros((S * C, hi - lo), np.float32)
    ws = np.zeros(hi - lo, np.float32)
    for c in range(c0, c1):
        st = c * step
        x, al = _chunk_input(track, total, border, border > 0, st, tr_lo, Ntr)
        y = _stand_in_model(x).reshape(S * C, CHUNK)[:, :al]
        w = _window(st, al, total, fade, fw)
        acc[:, st - lo:st - lo + al] += y * w
        ws[st - lo:st - lo + al] += w
    return acc, ws


def _single_process(track):
    import cudasep

    plan = cudasep.plan_shard(N, CHUNK, OVERLAP, DEFAULT, 0, 1)
    acc, ws = _accumulate(track, plan, 0, plan["n_chunks"], 0, plan["total"])
    b = plan["border"]
    a, w = acc[:, b:b + N], ws[b:b + N]
    return np.where(w > 1e-8, a / np.where(w > 1e-8, w, 1), a)


def _rank_main(rank, world, port, track, result_path):
    import torch
    import torch.distributed as dist

    import cudasep

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    p = cudasep.plan_shard(N, CHUNK, OVERLAP, DEFAULT, rank, world)
    w_lo, w_hi = cudasep.plan_shard_window(N, CHUNK, OVERLAP, DEFAULT, rank, world)
    window = np.ascontiguousarray(track[:, w_lo:w_hi])  # all the rank receives of the track
    acc, ws = _accumulate(window, p, p["c0"], p["c1"], p["lo"], p["hi"], w_lo, N)
    # the tail sent on is disjoint from the head received, so both go at once
    ops = []
    rlen = 0
    if rank > 0:
        prev = cudasep.plan_shard(N, CHUNK, OVERLAP, DEFAULT, rank - 1, world)
        rlen = prev["hi"] - prev["send_lo"]
        assert rank == world - 1 or prev["hi"] <= p["send_lo"]
        racc = torch.empty((S * C, rlen))
        rws = torch.empty((rlen,))
        ops += [dist.P2POp(dist.irecv, racc, rank - 1), dist.P2POp(dist.irecv, rws, rank - 1)]
    if rank < world - 1:
        off = p["send_lo"] - p["lo"]
        ops += [dist.P2POp(dist.isend, torch.from_numpy(np.ascontiguousarray(acc[:, off:])), rank + 1),
                dist.P2POp(dist.isend, torch.from_numpy(np.ascontiguousarray(ws[off:])), rank + 1)]
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    if rank > 0:
        acc[:, :rlen] += racc.numpy()
        ws[:rlen] += rws.numpy()
    # own range: padded samples [max(lo, border), min(own_hi, border + N))
    own_hi = p["send_lo"] if rank < world - 1 else p["total"]
    b = p["border"]
    p0, p1 = max(p["lo"], b), min(own_hi, b + N)
    a, w = acc[:, p0 - p["lo"]:p1 - p["lo"]], ws[p0 - p["lo"]:p1 - p["lo"]]
    mine = np.where(w > 1e-8, a / np.where(w > 1e-8, w, 1), a).astype(np.float32)
    assert p0 - b == p["out_lo"] and p1 - b == p["out_hi"]
    np.save(f"{result_path}.{rank}.npy", mine)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_overlap_add_matches_single_process(tmp_path, world):
    import torch.multiprocessing as mp

    track = np.random.default_rng(world).uniform(-0.5, 0.5, (C, N)).astype(np.float32)
    ref = _single_process(track)
    res = str(tmp_path / "part")
    mp.start_processes(_rank_main, args=(world, _free_port(), track, res), nprocs=world, start_method="spawn",
                       join=True)
    import cudasep

    out = np.zeros_like(ref)
    covered = np.zeros(N, bool)
    for r in range(world):
        p = cudasep.plan_shard(N, CHUNK, OVERLAP, DEFAULT, r, world)
        part = np.load(f"{res}.{r}.npy")
        out[:, p["out_lo"]:p["out_hi"]] = part
        assert not covered[p["out_lo"]:p["out_hi"]].any()
        covered[p["out_lo"]:p["out_hi"]] = True
    assert covered.all()
    assert np.abs(out - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


def test_shard_plan_partitions_chunks():
    import cudasep

    for world in (1, 2, 4, 8):
        Nn = 30 * 44100 * world
        plans = [cudasep.plan_shard(Nn, 352800, 4.0, 4, r, world) for r in range(world)]
        assert plans[0]["c0"] == 0 and plans[-1]["c1"] == plans[0]["n_chunks"]
        for a, b in zip(plans, plans[1:]):
            assert a["c1"] == b["c0"] and a["send_lo"] == b["lo"] and a["out_hi"] == b["out_lo"]
            assert a["hi"] - a["send_lo"] == 352800 - plans[0]["step"]  # the exchanged boundary
        assert plans[0]["out_lo"] == 0 and plans[-1]["out_hi"] == Nn


@pytest.mark.parametrize("n_sec,world,overlap", [(7.3, 1, 4.0), (7.3, 3, 4.0), (9.0, 4, 2.0), (2.6, 2, 0.5)])
def test_shard_window_covers_reads(n_sec, world, overlap):
    """mbr_plan_shard_window is exactly the span of track samples the shard's
    chunks read (through the reflect padding and the last chunk's fold)."""
    import cudasep

    Nn = int(n_sec * 44100)
    for r in range(world):
        p = cudasep.plan_shard(Nn, CHUNK, overlap, DEFAULT, r, world)
        lo, hi = cudasep.plan_shard_window(Nn, CHUNK, overlap, DEFAULT, r, world)
        reads = [t for c in range(p["c0"], p["c1"]) for q in range(CHUNK)
                 if (t := _read_index(p["total"], p["border"], p["border"] > 0, c * p["step"], q, Nn)) is not None]
        assert (lo, hi) == (min(reads), max(reads) + 1), (r, lo, hi, min(reads), max(reads) + 1)
