"""GPU, 2 ranks over NCCL: key-sharded long-context decode (BASELINE config 5 decode shape at
batch 1, Sk = 65536 split over 2 GPUs) through transfer_station_b200.multigpu.sharded_decode,
and the (batch x kv-head group) sharded prefill through multigpu.sharded_prefill, each checked
against the fp32 oracle. Skipped on a box with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path):
    from datetime import timedelta

    import transfer_station_b200 as ts
    from transfer_station_b200 import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        Hq, Hkv, Sq, Sk, D = 64, 8, 1, 65536, 128
        Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=4, a=0.0, b=0.5)
        k0, kl = multigpu.key_shard(Sk, world, rank)
        Ks = np.ascontiguousarray(K.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
        Vs = np.ascontiguousarray(V.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
        q = torch.from_numpy(Q.view(np.int16)).to(dev)
        ks = torch.from_numpy(Ks.view(np.int16)).to(dev)
        vs = torch.from_numpy(Vs.view(np.int16)).to(dev)
        o = torch.empty(Hq * Sq * D, dtype=torch.float32, device=dev)
        scratch = torch.empty(ts.attn_flash_scratch_bytes(D, 128), dtype=torch.uint8, device=dev)
        multigpu.sharded_decode(q, ks, vs, o, Hq, Hkv, Sq, Sk, k0, D, 0, scratch)
        torch.cuda.synchronize()
        rc, code = ts.attn_flash_status(scratch)
        assert rc == ts.ATTN_OK, code
        if rank == 0:
            np.save(out_path, o.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_key_sharded_decode(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "o.npy"
    mp.spawn(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    Hq, Hkv, Sq, Sk, D = 64, 8, 1, 65536, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=4, a=0.0, b=0.5)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    c = oracle.cmp_rows(ref, np.load(out), Hq, Sq, D, rows)
    assert oracle.passes(c), c


def _prefill_worker(rank, world, port, out_path):
    from datetime import timedelta

    import transfer_station_b200 as ts
    from transfer_station_b200 import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        B, Hq, Hkv, S, D = 2, 64, 8, 4096, 128
        Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, S, S, D, seed=4, a=0.0, b=0.5)
        q = torch.from_numpy(Q.view(np.int16)).to(dev)
        k = torch.from_numpy(K.view(np.int16)).to(dev)
        v = torch.from_numpy(V.view(np.int16)).to(dev)
        o = torch.full((B * Hq * S * D,), float("nan"), dtype=torch.float32, device=dev)
        scratch = torch.empty(ts.attn_flash_scratch_bytes(D, 128), dtype=torch.uint8, device=dev)
        s = multigpu.sharded_prefill(q, k, v, o, B, Hq, Hkv, S, S, D, 0, scratch)
        torch.cuda.synchronize()
        rc, code = ts.attn_flash_status(scratch)
        assert rc == ts.ATTN_OK, code
        np.save(out_path + f".{rank}.npy", o.cpu().numpy()[s.q_off:s.q_off + s.hq * S * D])
        np.save(out_path + f".{rank}.off.npy", np.array([s.q_off], np.int64))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_prefill(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "o")
    mp.spawn(_prefill_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    B, Hq, Hkv, S, D = 2, 64, 8, 4096, 128
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, S, S, D, seed=4, a=0.0, b=0.5)
    full = np.full(B * Hq * S * D, np.nan, np.float32)
    for r in range(2):
        part = np.load(out + f".{r}.npy")
        off = int(np.load(out + f".{r}.off.npy")[0])
        full[off:off + part.size] = part
    assert not np.isnan(full).any()
    rows = oracle.rowset(S, 6)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, rows)
    c = oracle.cmp_rows(ref, full, B * Hq, S, D, rows)
    assert oracle.passes(c), c


def _peer_worker(rank, world, port, out_path):
    from datetime import timedelta

    import transfer_station_b200 as ts
    from transfer_station_b200 import multigpu

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    merge = None
    try:
        Hq, Hkv, Sq, Sk, D = 64, 8, 1, 65536, 128
        merge = multigpu.PeerMerge(Hq * Sq, D, device=dev)
        scratch = torch.empty(ts.attn_flash_scratch_bytes(D, 128), dtype=torch.uint8, device=dev)
        outs = []
        for step in range(3):  # epochs 1..3: both buffers, new data every step
            Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=40 + step, a=0.0, b=0.5)
            k0, kl = multigpu.key_shard(Sk, world, rank)
            Ks = np.ascontiguousarray(K.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
            Vs = np.ascontiguousarray(V.reshape(Hkv, Sk, D)[:, k0:k0 + kl]).reshape(-1)
            q = torch.from_numpy(Q.view(np.int16)).to(dev)
            ks = torch.from_numpy(Ks.view(np.int16)).to(dev)
            vs = torch.from_numpy(Vs.view(np.int16)).to(dev)
            o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
            multigpu.sharded_decode_peers(q, ks, vs, o, Hq, Hkv, Sq, Sk, k0, D, 0, scratch, merge)
            torch.cuda.synchronize()
            rc, code = ts.attn_flash_status(scratch)
            assert rc == ts.ATTN_OK, code
            outs.append(o.cpu().numpy())
        np.save(out_path + f".{rank}.npy", np.stack(outs))
    finally:
        if merge is not None:
            merge.close()
        dist.destroy_process_group()


def test_two_gpu_decode_merged_by_peer_stores(tmp_path):
    """The merge kernel's real exchange over NVLink: 2 ranks, 3 steps; every rank ends with the
    full output, equal on both ranks and within tolerance of the fp32 reference."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "o")
    mp.spawn(_peer_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    Hq, Hkv, Sq, Sk, D = 64, 8, 1, 65536, 128
    o0, o1 = np.load(out + ".0.npy"), np.load(out + ".1.npy")
    assert np.array_equal(o0, o1)
    rows = np.arange(Sq, dtype=np.int32)
    for step in range(3):
        Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=40 + step, a=0.0, b=0.5)
        ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
        c = oracle.cmp_rows(ref, o0[step], Hq, Sq, D, rows)
        assert oracle.passes(c), (step, c)
