"""GPU: attention over a paged K/V cache (attn_flash_paged_stream).

Each sequence's keys live in pages of a shared pool, in the order its block table lists them
(the pages are shuffled across the pool, the tail of a last page holds unrelated data). The
oracle gathers every sequence's pages into contiguous K and V and runs the fp32 reference
(flash.c:262-314 restated) per sequence; the GPU result must pass the same bounds as the
contiguous entry point. Covers page sizes below, at and above the 128-key tile, decode
(Sq=1) and causal multi-token steps, a one-key and an empty sequence, D=64, and a page id
outside the pool (the kernel stops and reports it; the library stays usable).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import scratch_for, to_dev

pytestmark = pytest.mark.gpu


def build_cache(lens, Hkv, D, P, rng, spare=3):
    """Pools [num_pages][Hkv][P][D] holding each sequence's K/V rows, a shuffled block table and
    the contiguous per-sequence K/V the oracle uses."""
    need = [(L + P - 1) // P for L in lens]
    max_pages = max(1, max(need))
    num_pages = sum(need) + spare
    order = rng.permutation(num_pages)
    st = np.random.default_rng(7)
    junk = lambda n: (st.standard_normal(n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731
    Kp = junk(num_pages * Hkv * P * D).reshape(num_pages, Hkv, P, D)
    Vp = junk(num_pages * Hkv * P * D).reshape(num_pages, Hkv, P, D)
    table = np.full((len(lens), max_pages), -1, np.int32)
    seqs, nxt = [], 0
    for b, L in enumerate(lens):
        Kb, Vb = (junk(Hkv * max(L, 1) * D).reshape(Hkv, max(L, 1), D) for _ in range(2))
        for j in range(need[b]):
            pid = int(order[nxt]); nxt += 1
            table[b, j] = pid
            rows = slice(j * P, min(L, (j + 1) * P))
            n = rows.stop - rows.start
            Kp[pid, :, :n] = Kb[:, rows]
            Vp[pid, :, :n] = Vb[:, rows]
        table[b, need[b]:] = int(order[0])  # entries past the sequence's pages are never read
        seqs.append((Kb[:, :L].copy(), Vb[:, :L].copy()))
    return Kp, Vp, table, max_pages, num_pages, seqs


def run_paged(Q, Kp, Vp, table, lens, B, Hq, Hkv, Sq, D, causal, P, num_pages, max_pages, dev):
    q, kp, vp = to_dev(Q, dev), to_dev(Kp.reshape(-1), dev), to_dev(Vp.reshape(-1), dev)
    bt = torch.from_numpy(table.reshape(-1)).to(dev)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    o = torch.full((B * Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
    scr = scratch_for(D, 128, dev)
    rc = ts.attn_flash_paged_stream(q, kp, vp, bt, sl, o, B, Hq, Hkv, Sq, D, causal, P, num_pages, max_pages, scr)
    assert rc == ts.ATTN_OK, ts.strerror(rc)
    return o, scr


CASES = [
    # (name, lens, Hq, Hkv, Sq, D, causal, page_size)
    ("decode p16", [1000, 1, 4096, 777], 32, 8, 1, 128, 0, 16),
    ("decode p64", [5000, 300, 64, 2049], 32, 8, 1, 128, 0, 64),
    ("decode p128", [129, 3000, 128, 4000], 16, 2, 1, 128, 0, 128),
    ("decode p256 mqa", [2500, 1, 513], 16, 1, 1, 128, 0, 256),
    ("causal 4 new tokens p32", [700, 4, 1500], 32, 8, 4, 128, 1, 32),
    ("head dim 64 p8", [300, 90], 8, 2, 3, 64, 1, 8),
    ("empty sequence", [0, 400], 8, 2, 1, 128, 0, 16),
]


@pytest.mark.parametrize("name,lens,Hq,Hkv,Sq,D,causal,P", CASES, ids=[c[0] for c in CASES])
def test_paged_matches_reference(cuda_dev, name, lens, Hq, Hkv, Sq, D, causal, P):
    rng = np.random.default_rng(sum(lens) + P)
    B = len(lens)
    Kp, Vp, table, max_pages, num_pages, seqs = build_cache(lens, Hkv, D, P, rng)
    Q, _, _ = oracle.seeded_inputs(B * Hq, 1, Sq, 1, D, seed=21)
    o, _ = run_paged(Q, Kp, Vp, table, lens, B, Hq, Hkv, Sq, D, causal, P, num_pages, max_pages, cuda_dev)
    out = o.cpu().numpy().reshape(B, Hq * Sq * D)
    rows = np.arange(Sq, dtype=np.int32)
    for b, L in enumerate(lens):
        Qb = Q.reshape(B, -1)[b].copy()
        if L == 0:
            assert np.all(out[b] == 0.0), f"{name}: empty sequence {b} must give zero rows"
            continue
        Kb, Vb = seqs[b]
        ref = oracle.attn_ref(Qb, Kb.reshape(-1), Vb.reshape(-1), Hq, Hkv, Sq, L, D, causal, rows)
        c = oracle.cmp_rows(ref, out[b], Hq, Sq, D, rows)
        assert oracle.passes(c), f"{name} sequence {b} (len {L}): {c}"


def test_bad_page_id_is_reported_and_library_recovers(cuda_dev):
    lens, Hq, Hkv, Sq, D, P = [600, 300], 8, 2, 1, 128, 64
    rng = np.random.default_rng(5)
    Kp, Vp, table, max_pages, num_pages, seqs = build_cache(lens, Hkv, D, P, rng)
    Q, _, _ = oracle.seeded_inputs(2 * Hq, 1, Sq, 1, D, seed=22)
    bad = table.copy()
    bad[0, 3] = num_pages + 5  # inside sequence 0's 600 keys (page 3 covers keys 192..255)
    o, scr = run_paged(Q, Kp, Vp, bad, lens, 2, Hq, Hkv, Sq, D, 0, P, num_pages, max_pages, cuda_dev)
    rc, code = ts.attn_flash_status(scr)
    assert rc == ts.ATTN_ERR_DEVICE and code & (1 << 5), (rc, code)
    o, scr = run_paged(Q, Kp, Vp, table, lens, 2, Hq, Hkv, Sq, D, 0, P, num_pages, max_pages, cuda_dev)
    rc, code = ts.attn_flash_status(scr)
    assert rc == ts.ATTN_OK, (rc, code)
    out = o.cpu().numpy().reshape(2, -1)
    rows = np.arange(Sq, dtype=np.int32)
    Kb, Vb = seqs[1]
    ref = oracle.attn_ref(Q.reshape(2, -1)[1].copy(), Kb.reshape(-1), Vb.reshape(-1), Hq, Hkv, Sq, lens[1], D, 0, rows)
    assert oracle.passes(oracle.cmp_rows(ref, out[1], Hq, Sq, D, rows))
