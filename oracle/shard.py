"""NumPy restatement of the bank-sharded forward's integer steps -- TEST INFRASTRUCTURE ONLY.

The reference has no sharded path (it runs the layer on one device,
implementation/bdm/model.py:88-140), so these functions restate the partition
and filtering rules that bdm_b200's bank-sharded forward defines, as the
checker for its kernels:

* ``oracle_bank_histogram``  events per bank over write and read routes
* ``oracle_bank_owners``     contiguous or load-balanced partition of the bank table
* ``oracle_dispatch_owned``  pack_bank_events ordering (gdn2_banks.py:174-185) restricted
                             to one rank's banks, sequences renumbered (batch, local bank)
* ``oracle_combine_partial`` scatter_bank_outputs' ascending-bank FP32 sum
                             (gdn2_banks.py:265-283) over one rank's banks only

Nothing in the product imports this module.
"""
from __future__ import annotations

import numpy as np


GREEDY_GROUPS = 128  # groups of the balanced partition dealt greedily


def oracle_bank_histogram(wi, ri, bank_count: int) -> np.ndarray:
    banks = np.concatenate([np.asarray(wi, np.int64).ravel(), np.asarray(ri, np.int64).ravel()])
    banks = np.clip(banks, 0, bank_count - 1)
    return np.bincount(banks, minlength=bank_count).astype(np.int32)


def oracle_bank_owners(counts, bank_count: int, world: int, mode: str = 'balanced'):
    """-> (owner [J], slot [J], members [world, J/world]) int32.

    contiguous: owner = bank // (J/world).  balanced: banks in (count desc, index
    asc) order are dealt out in groups of ``world``.  In the first GREEDY_GROUPS
    groups the p-th heaviest bank of a group goes to the rank with the p-th
    smallest load so far (ties to the lower rank); the remaining groups go in a
    serpentine (forward on even groups, backward on odd ones, counted from the
    first tail group) over the ranks ordered by their load after those groups.
    Slots number each rank's banks in ascending bank order.
    """
    if bank_count % world:
        raise ValueError('bank count must divide over the ranks')
    per = bank_count // world
    if mode == 'contiguous':
        owner = np.arange(bank_count) // per
    elif mode == 'balanced':
        c = np.maximum(np.asarray(counts, np.int64), 0)
        order = sorted(range(bank_count), key=lambda j: (-c[j], j))
        load = [0] * world
        owner = np.empty(bank_count, np.int64)
        head = min(per, GREEDY_GROUPS)
        for g in range(head):
            ranks = sorted(range(world), key=lambda r: (load[r], r))
            for p, r in enumerate(ranks):
                j = order[g * world + p]
                owner[j] = r
                load[r] += int(c[j])
        ranks = sorted(range(world), key=lambda r: (load[r], r))
        for g in range(head, per):
            k = g - head
            for p in range(world):
                owner[order[g * world + p]] = ranks[world - 1 - p] if k % 2 else ranks[p]
    else:
        raise ValueError(mode)
    slot = np.empty(bank_count, np.int64)
    members = np.empty((world, per), np.int64)
    for r in range(world):
        mine = np.nonzero(owner == r)[0]
        slot[mine] = np.arange(len(mine))
        members[r] = mine
    return owner.astype(np.int32), slot.astype(np.int32), members.astype(np.int32)


def oracle_dispatch_owned(wi, ri, bank_count: int, owner, slot, rank: int, local_banks: int):
    """Owned events sorted by (batch*local_banks + slot, event order); then the rest in id order.

    Event ids follow bdm_dispatch: write (token, j) -> token*KW + j, read -> NT*KW + token*KR + j.
    Returns (order [E], cu_seqlens [B*local_banks + 1]).
    """
    wi, ri = np.asarray(wi, np.int64), np.asarray(ri, np.int64)
    batch, time, kw = wi.shape
    kr = ri.shape[-1]
    nt = batch * time
    sentinel = batch * local_banks
    ids, seqs = [], []
    for tok in range(nt):
        b = tok // time
        for role, idx, k in ((0, wi, kw), (1, ri, kr)):
            for j in range(k):
                bank = int(np.clip(idx.reshape(nt, k)[tok, j], 0, bank_count - 1))
                eid = tok * kw + j if role == 0 else nt * kw + tok * kr + j
                seq = b * local_banks + int(slot[bank]) if int(owner[bank]) == rank else sentinel
                ids.append(eid)
                seqs.append(seq)
    ids, seqs = np.asarray(ids, np.int64), np.asarray(seqs, np.int64)
    perm = np.argsort(seqs, kind='stable')
    order = ids[perm]
    cu = np.searchsorted(seqs[perm], np.arange(sentinel + 1), side='left').astype(np.int64)
    return order, cu


def oracle_combine_partial(reads, ri, owner, rank: int) -> np.ndarray:
    """reads [NT, KR, V], ri [NT, KR] -> FP32 [NT, V]: ascending-bank sum over this rank's banks."""
    reads = np.asarray(reads, np.float32)
    ri = np.asarray(ri, np.int64)
    nt, kr, width = reads.shape
    out = np.zeros((nt, width), np.float32)
    bank_count = len(owner)
    for t in range(nt):
        banks = np.clip(ri[t], 0, bank_count - 1)
        for j in np.argsort(banks, kind='stable'):
            if int(owner[banks[j]]) == rank:
                out[t] += reads[t, j]
    return out
