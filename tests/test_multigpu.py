"""GPU, 2 ranks over NCCL: key-sharded long-context decode (BASELINE config 5 decode shape at
batch 1, Sk = 65536 split over 2 GPUs) through transfer_station_b200.multigpu.sharded_decode,
checked against the fp32 oracle. Skipped on a box with fewer than 2 GPUs."""
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
