"""Expert-parallel exchange on CPU ranks (gloo): the protocol of
dsb_ep_dispatch / dsb_ep_combine, restated in oracle/ep.py, run by separate
processes that exchange counts, token rows and expert outputs.

Checks: the result equals a single-process moe_step over the same tokens bit
for bit (float64, linear experts), every expert sees its rows in the order of
the single-GPU permutation (the oracle's orc_moe_permute over all ranks'
picks in rank order), ranks with no tokens take part, and a rank that fails
before the count exchange makes the others' exchange end with an error
instead of hanging.  The GPU kernels reach the same layout in two steps
(fixed staging slots per source and local expert, then the owner's
compaction); a host restatement of those steps is checked against the
direct placement.
"""

import datetime
import os
import socket

import numpy as np
import pytest

E, K, D, NS = 16, 4, 32, 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s=60):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _problem(t_per_rank):
    rng = np.random.default_rng(100)  # identical on every rank: experts and every rank's tokens
    W = rng.standard_normal((E, D, D))
    Ws = rng.standard_normal((NS, D, D))
    xs = [rng.standard_normal((T, D)) for T in t_per_rank]
    ids = [np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32) if T
           else np.zeros((0, K), np.int32) for T in t_per_rank]
    wts = [rng.random((T, K)) for T in t_per_rank]
    return W, Ws, xs, ids, wts


def _worker(rank, world, port, t_per_rank):
    import torch

    import oracle as O
    import oracle.ep as EP

    dist = _setup(rank, world, port)
    W, Ws, xs, ids, wts = _problem(t_per_rank)
    x, my_ids, w = xs[rank], ids[rank], wts[rank]
    T, EL = len(x), E // world
    # 1. counts: every rank's [world][E_local] row to every rank
    c = torch.from_numpy(EP.counts(my_ids, E, world))
    rows_all = [torch.zeros_like(c) for _ in range(world)]
    dist.all_gather(rows_all, c)
    cm = torch.stack(rows_all).numpy()  # [src][dst][el]
    # 2. rows to their owners, at the placements of the model
    dst, row = EP.placements(my_ids, cm, rank, E)
    picks = np.arange(T * K)
    sent = [None] * world
    dist.all_gather_object(sent, {p: (row[dst == p], picks[dst == p], x[picks[dst == p] // K]) for p in range(world)})
    cap = world * max(t_per_rank) * K
    recv = np.zeros((cap, D))
    meta = np.full((cap, 2), -1)
    for src in range(world):
        r, pk, data = sent[src][rank]
        recv[r] = data
        meta[r] = np.stack([np.full(len(pk), src), pk], 1)
    ro = EP.recv_offsets(cm, rank)
    # every expert's rows in the single-GPU permutation order of all picks
    flat = np.concatenate([i.ravel() for i in ids]).astype(np.int32)
    base = np.concatenate([[0], np.cumsum([len(i.ravel()) for i in ids])])
    n = len(flat)
    cnt, off = np.zeros(E, np.int32), np.zeros(E + 1, np.int32)
    dest, src_pair = np.zeros(max(n, 1), np.int32), np.zeros(max(n, 1), np.int32)
    if n:
        O.oracle().orc_moe_permute(O.p(flat, O.i32p), n, 1, E, O.p(cnt, O.i32p), O.p(off, O.i32p),
                                   O.p(dest, O.i32p), O.p(src_pair, O.i32p))
    for el in range(EL):
        e = rank * EL + el
        got = [tuple(m) for m in meta[ro[el]:ro[el + 1]]]
        want = [(int(np.searchsorted(base, g, side="right") - 1), int(g - base[np.searchsorted(base, g, side="right") - 1]))
                for g in src_pair[off[e]:off[e + 1]]]
        assert got == want, (rank, el, got, want)
    # 3. the experts (linear here) on the received rows
    y = np.zeros((cap, D))
    for el in range(EL):
        for r in range(ro[el], ro[el + 1]):
            y[r] = W[rank * EL + el] @ recv[r]
    # 4. outputs back to their picks' home ranks
    back = [None] * world
    dist.all_gather_object(back, {p: (meta[(meta[:, 0] == p), 1], y[meta[:, 0] == p]) for p in range(world)})
    inbox = np.zeros((T * K, D))
    for src in range(world):
        pk, data = back[src][rank]
        inbox[pk] = data
    # 5. combine in moe_step order, then compare with the single-process layer
    h = np.zeros((T, D))
    ref = np.zeros((T, D))
    for t in range(T):
        acc = np.zeros(D)
        racc = np.zeros(D)
        for j in range(K):
            acc = acc + w[t, j] * inbox[t * K + j]
            racc = racc + w[t, j] * (W[my_ids[t, j]] @ x[t])
        for s in range(NS):
            acc = acc + Ws[s] @ x[t]
            racc = racc + Ws[s] @ x[t]
        h[t], ref[t] = acc, racc
    assert np.array_equal(h, ref), rank
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("t_per_rank", [(7, 5), (6, 0), (3, 9, 1, 4)])
def test_ep_exchange_equals_single_process_moe(t_per_rank):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(len(t_per_rank), _port(), t_per_rank), nprocs=len(t_per_rank), join=True)


def _failing_worker(rank, world, port, flag_dir):
    import torch

    dist = _setup(rank, world, port, timeout_s=10)
    if rank == 1:
        os._exit(3)  # dies before the count exchange
    c = torch.zeros(4, dtype=torch.int64)
    rows = [torch.zeros_like(c) for _ in range(world)]
    try:
        dist.all_gather(rows, c)
    except Exception:  # noqa: BLE001 - the exchange must end with an error, not hang
        open(os.path.join(flag_dir, "rank0_saw_error"), "w").close()


def test_ep_exchange_fails_when_a_rank_dies(tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.start_processes(_failing_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(60)
    assert all(not p.is_alive() for p in ctx.processes)
    assert (tmp_path / "rank0_saw_error").exists()


def test_staged_layout_equals_direct_placement():
    """The two-step exchange (fixed staging slots per source and local expert,
    then the owner's compaction) gives every owner the same rows in the same
    order, and the same receive offsets, as placing each pick directly at
    its final row from the full count matrix; ranks with no tokens included."""
    import oracle.ep as OE

    rng = np.random.default_rng(4)
    for world, t_per_rank in [(2, [5, 0]), (4, [3, 7, 0, 1]), (8, [2] * 8), (2, [16, 16])]:
        Ek = 8 * world
        ids = [np.stack([rng.choice(Ek, K, replace=False) for _ in range(t)]) if t else np.zeros((0, K), np.int64)
               for t in t_per_rank]
        T_max = max(max(t_per_rank), 1)
        cm = np.stack([OE.counts(i, Ek, world) if len(i) else np.zeros((world, Ek // world), np.int64) for i in ids])
        staged = OE.staged_layout(ids, Ek, world, T_max)
        for d in range(world):
            direct = {}
            for s in range(world):
                if len(ids[s]) == 0:
                    continue
                dst, row = OE.placements(ids[s], cm, s, Ek)
                for i in range(len(dst)):
                    if dst[i] == d:
                        direct[int(row[i])] = (s, i)
            rows, offs = staged[d]
            assert rows == [direct[r] for r in range(len(direct))]
            assert np.array_equal(offs, OE.recv_offsets(cm, d))
