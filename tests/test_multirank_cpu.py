"""CPU, world_size 2 over `gloo`: the multi-GPU decomposition's host logic.

The key-axis split of long-context decode (transfer_station_b200.multigpu): each rank computes
the (m, l, acc) partials of its key shard (here with a numpy stand-in for the partial kernel,
using the kernel's conventions: m in base-2 units of the scaled score, l and acc unnormalised),
the partials are all-gathered with torch.distributed, and the merge (the same formula the
combine kernel applies, restated in oracle/) must equal one-shot attention over all keys.
Also the prefill unit split and the key-shard boundaries."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from transfer_station_b200 import multigpu


def np_partial(Q, K, V, Hq, Hkv, Sq, Sk_total, k_begin, Sk_local, D, causal):
    """(m, l, acc) of keys [k_begin, k_begin + Sk_local) for every row of [Hq*Sq]."""
    q = oracle.bf16_to_f32(Q).reshape(Hq, Sq, D).astype(np.float64)
    k = oracle.bf16_to_f32(K).reshape(Hkv, Sk_local, D).astype(np.float64)
    v = oracle.bf16_to_f32(V).reshape(Hkv, Sk_local, D).astype(np.float64)
    g = Hq // Hkv
    c = (1.0 / np.sqrt(D)) * np.log2(np.e)
    m = np.full(Hq * Sq, -np.inf, np.float32)
    l = np.zeros(Hq * Sq, np.float32)
    acc = np.zeros((Hq * Sq, D), np.float32)
    keys = k_begin + np.arange(Sk_local)
    for h in range(Hq):
        s = (q[h] @ k[h // g].T) * c  # [Sq, Sk_local]
        if causal:
            lim = Sk_total - Sq + np.arange(Sq)
            s = np.where(keys[None, :] <= lim[:, None], s, -np.inf)
        mx = s.max(axis=1)
        live = np.isfinite(mx)
        p = np.where(live[:, None], np.exp2(s - np.where(live, mx, 0)[:, None]), 0.0)
        r = slice(h * Sq, (h + 1) * Sq)
        m[r] = mx
        l[r] = p.sum(1)
        acc[r] = p @ v[h // g]
    return m, l, acc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Hq, Hkv, Sq, Sk, D, causal = case
        Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
        k0, kl = multigpu.key_shard(Sk, world, rank, align=64)
        Ks = np.ascontiguousarray(K.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
        Vs = np.ascontiguousarray(V.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
        m, l, acc = np_partial(Q, Ks, Vs, Hq, Hkv, Sq, Sk, k0, kl, D, causal)
        rows = Hq * Sq
        buf = torch.zeros(multigpu.packed_floats(rows, D), dtype=torch.float32)
        pm, pl, pacc = multigpu.packed_views(buf, rows, D)
        pm.copy_(torch.from_numpy(m))
        pl.copy_(torch.from_numpy(l))
        pacc.copy_(torch.from_numpy(acc))
        parts = multigpu.gather_packed(buf).view(world, -1)  # one collective for all three
        views = [multigpu.packed_views(parts[r], rows, D) for r in range(world)]
        all_m = np.stack([v[0].numpy() for v in views])
        all_l = np.stack([v[1].numpy() for v in views])
        all_acc = np.stack([v[2].numpy() for v in views])
        O = oracle.combine(all_m, all_l, all_acc, world, rows, D)
        if rank == 0:
            np.save(out_path, O)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(8, 2, 1, 1000, 64, 0), (4, 2, 40, 300, 32, 1)])
def test_key_sharded_merge_two_ranks(tmp_path, case):
    world = 2
    out = tmp_path / "o.npy"
    mp.spawn(_worker, args=(world, _free_port(), case, str(out)), nprocs=world, join=True)
    Hq, Hkv, Sq, Sk, D, causal = case
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    c = oracle.cmp_rows(ref, np.load(out), Hq, Sq, D, rows)
    assert c["nbad"] == 0 and c["mad"] < 1e-5, c  # no bf16 P here: exact up to fp32 sums


def test_unit_and_key_shards_partition():
    for n, world in [(8, 8), (32, 8), (7, 4), (3, 8), (1024, 3)]:
        spans = [multigpu.unit_shard(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    for Sk, world in [(131072, 8), (131072, 3), (1000, 4), (100, 8)]:
        sh = [multigpu.key_shard(Sk, world, r) for r in range(world)]
        assert sum(k for _, k in sh) == Sk
        assert all(b % 128 == 0 or b == Sk for b, _ in sh)
        assert all(sh[r][0] + sh[r][1] == sh[r + 1][0] for r in range(world - 1))


def _prefill_worker(rank, world, port, case, out_dir):
    """A rank of the (batch x kv-head group) sharded prefill, with a CPU stand-in for
    attn_flash_stream (oracle.attn_ref on the numpy views the library would receive), so the
    real multigpu.sharded_prefill code chooses the units, offsets and sizes."""
    import transfer_station_b200 as ts

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, Hq, Hkv, Sq, Sk, D, causal = case
        Q, K, V = oracle.lcg_inputs(B * Hq, B * Hkv, Sq, Sk, D)
        q = torch.from_numpy(Q.view(np.int16))
        k = torch.from_numpy(K.view(np.int16))
        v = torch.from_numpy(V.view(np.int16))
        O = torch.full((B * Hq * Sq * D,), float("nan"), dtype=torch.float32)

        def stand_in(qv, kv_, vv, ov, hq, hkv, sq, sk, d, c, bk, scratch, vp, stream):
            ref = oracle.attn_ref(qv.numpy().view(np.uint16), kv_.numpy().view(np.uint16),
                                  vv.numpy().view(np.uint16), hq, hkv, sq, sk, d, c)
            ov.copy_(torch.from_numpy(ref))
            return ts.ATTN_OK

        ts.attn_flash_stream = stand_in  # this process only
        s = multigpu.sharded_prefill(q, k, v, O, B, Hq, Hkv, Sq, Sk, D, causal, scratch=None)
        np.save(os.path.join(out_dir, f"o{rank}.npy"), O.numpy())
        np.save(os.path.join(out_dir, f"s{rank}.npy"), np.array(s, np.int64))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(2, 8, 2, 40, 56, 32, 1), (3, 4, 4, 16, 16, 16, 0), (1, 6, 3, 24, 30, 8, 0)])
def test_sharded_prefill_two_ranks(tmp_path, case):
    """Each rank writes exactly its units' rows of O (the others stay untouched), the ranks'
    units partition the problem, and together they give the full attention."""
    world = 2
    mp.spawn(_prefill_worker, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, join=True)
    B, Hq, Hkv, Sq, Sk, D, causal = case
    Q, K, V = oracle.lcg_inputs(B * Hq, B * Hkv, Sq, Sk, D)
    want = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, Sq, Sk, D, causal)
    full = np.full_like(want, np.nan)
    spans = []
    for r in range(world):
        o = np.load(tmp_path / f"o{r}.npy")
        s = multigpu.PrefillSlice(*np.load(tmp_path / f"s{r}.npy").tolist())
        spans.append((s.u0, s.u1))
        mine = np.zeros(o.size, bool)
        mine[s.q_off:s.q_off + s.hq * Sq * D] = True
        assert np.all(np.isnan(o[~mine])), f"rank {r} wrote outside its units"
        full[mine] = o[mine]
    assert spans[0][0] == 0 and spans[-1][1] == B * Hkv and spans[0][1] == spans[1][0]
    assert np.array_equal(full, want)
