"""Host model of the expert-parallel exchange (TEST INFRASTRUCTURE ONLY; see
oracle/__init__.py for who may import it).

The reference runs one GPU with B = 1 and has no expert parallelism; this is
the permutation the GPU exchange (dsb_ep_dispatch / dsb_ep_combine) follows,
restated in numpy so the protocol can be checked on CPU ranks:

  * expert e lives on rank e // (E // world);
  * a rank's picks (flattened [T, k], pick i = t*k + j) go to the owners, each
    owner's receive buffer grouped by local expert, sources in rank order,
    one source's picks of an expert in pick order;
  * every output returns to its pick's slot at home, and home sums
    w[t,j] * out[t,j] over j, then its shared experts (moe_step,
    src/models/deepseek/ops.cpp:133-145).
"""

from __future__ import annotations

import numpy as np


def owner(e, E: int, world: int):
    return np.asarray(e) // (E // world)


def counts(ids: np.ndarray, E: int, world: int) -> np.ndarray:
    """This rank's [world][E_local] pick counts (ids: int [T, k] global experts)."""
    return np.bincount(np.asarray(ids).ravel(), minlength=E).reshape(world, E // world).astype(np.int64)


def slots(ids: np.ndarray) -> np.ndarray:
    """Stable slot of every pick among this rank's picks of the same expert."""
    flat = np.asarray(ids).ravel()
    out = np.zeros(len(flat), np.int64)
    seen: dict[int, int] = {}
    for i, e in enumerate(flat):
        out[i] = seen.get(int(e), 0)
        seen[int(e)] = out[i] + 1
    return out


def send_offsets(cm: np.ndarray, rank: int) -> np.ndarray:
    """[dst][el]: first row of `rank`'s picks of local expert el in dst's
    receive buffer.  cm: count matrix [src][dst][el] of every rank."""
    world, _, EL = cm.shape
    off = np.zeros((world, EL), np.int64)
    for dst in range(world):
        for el in range(EL):
            off[dst, el] = cm[:, dst, :el].sum() + cm[:rank, dst, el].sum()
    return off


def recv_offsets(cm: np.ndarray, rank: int) -> np.ndarray:
    """[E_local + 1]: row range of each local expert in `rank`'s buffer."""
    per = cm[:, rank, :].sum(0)
    return np.concatenate([[0], np.cumsum(per)]).astype(np.int64)


def placements(ids: np.ndarray, cm: np.ndarray, rank: int, E: int):
    """For every pick of `rank`: (destination rank, row in its buffer)."""
    world, _, EL = cm.shape
    flat = np.asarray(ids).ravel()
    off = send_offsets(cm, rank)
    sl = slots(ids)
    dst = flat // EL
    row = off[dst, flat % EL] + sl
    return dst, row


def staged_layout(ids_per_rank, E: int, world: int, T_max: int):
    """Owner-side layout of the exchange as the kernels run it in two steps:
    every source s puts its pick of local expert el of owner d into the
    staging slot [s][el][slot] of d (slot = the pick's rank among s's picks
    of that expert, so slot < T <= T_max), with s's per-expert counts; the
    owner then lays the staged rows out expert by expert, sources in rank
    order, slots in order.  Returns, per owner, the (source, pick) of every
    received row in row order and the owner's receive offsets [E_local + 1].
    This must equal the direct placement (placements / recv_offsets)."""
    EL = E // world
    staged = [[[None] * T_max for _ in range(EL)] for _ in range(world * world)]  # [(s, d)][el][slot]
    counts = np.zeros((world, world, EL), np.int64)
    for s, ids in enumerate(ids_per_rank):
        flat = np.asarray(ids).ravel()
        sl = slots(ids) if flat.size else np.zeros(0, np.int64)
        for i, e in enumerate(flat):
            d, el = int(e) // EL, int(e) % EL
            assert sl[i] < T_max
            staged[s * world + d][el][sl[i]] = (s, i)
            counts[s, d, el] += 1
    out = []
    for d in range(world):
        rows = []
        offs = [0]
        for el in range(EL):
            for s in range(world):
                rows.extend(staged[s * world + d][el][: counts[s, d, el]])
            offs.append(len(rows))
        out.append((rows, np.asarray(offs, np.int64)))
    return out
