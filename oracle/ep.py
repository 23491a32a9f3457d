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
