"""GPU: re-entrancy. flash.c's attn_flash is re-entrant given one scratch block per calling
thread (flash.c:588-592); the C ABI keeps that contract with device scratch and one stream per
thread. Host threads call the entry points at the same time, each on its own stream and scratch,
over different shapes (prefill, decode with split keys, causal, the QKV producer); every result
must be bit-identical to the same call made alone (the kernels are deterministic)."""
from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from oracle import qkv_rope as orq
from tests.gpu_util import scratch_for, to_dev

pytestmark = pytest.mark.gpu

CASES = [  # Hq, Hkv, Sq, Sk, D, causal
    (32, 8, 512, 512, 128, 0),
    (32, 8, 1, 8192, 128, 0),
    (8, 2, 300, 700, 64, 1),
    (16, 16, 130, 130, 128, 1),
]


def _attn_job(dev, case, seed):
    Hq, Hkv, Sq, Sk, D, causal = case
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=seed)
    q, k, v = to_dev(Q, dev), to_dev(K, dev), to_dev(V, dev)
    o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
    scratch = scratch_for(D, 128, dev)

    def run(stream):
        with torch.cuda.stream(stream):
            rc = ts.attn_flash_stream(q, k, v, o, Hq, Hkv, Sq, Sk, D, causal, 128, scratch, 0, stream)
            assert rc == ts.ATTN_OK, ts.strerror(rc)
            assert ts.attn_flash_status(scratch, stream) == (ts.ATTN_OK, 0)
        return o.cpu().numpy().copy()

    return run


def _producer_job(dev, seed):
    B, S, Hq, Hkv, D = 2, 64, 8, 2, 128
    rng = np.random.default_rng(seed)
    qkv = to_dev(oracle.f32_to_bf16(rng.normal(size=(B * S, (Hq + 2 * Hkv) * D)).astype(np.float32)), dev)
    pos = to_dev(np.tile(np.arange(S, dtype=np.int32), B), dev)
    cs = to_dev(orq.rope_table(S, D, 1e6), dev)
    w = to_dev(oracle.f32_to_bf16(rng.uniform(0.5, 1.5, D).astype(np.float32)), dev)
    q = torch.empty(B * Hq * S * D, dtype=torch.int16, device=dev)
    k = torch.empty(B * Hkv * S * D, dtype=torch.int16, device=dev)
    v = torch.empty_like(k)
    scratch = scratch_for(D, 128, dev)

    def run(stream):
        with torch.cuda.stream(stream):
            rc = ts.attn_qkv_rope_stream(qkv, pos, cs, S, w, w, 1e-6, B, S, Hq, Hkv, D, D, ts.ATTN_ROPE_NEOX, q, k, v,
                                         S, scratch, stream)
            assert rc == ts.ATTN_OK
            assert ts.attn_flash_status(scratch, stream) == (ts.ATTN_OK, 0)
        return np.concatenate([t.cpu().numpy().view(np.uint16) for t in (q, k, v)])

    return run


def test_concurrent_host_threads(cuda_dev):
    jobs = [_attn_job(cuda_dev, c, seed=20 + i) for i, c in enumerate(CASES)] + [_producer_job(cuda_dev, 31)]
    alone = [job(torch.cuda.Stream(cuda_dev)) for job in jobs]
    streams = [torch.cuda.Stream(cuda_dev) for _ in jobs]
    results: list = [None] * len(jobs)
    errors: list = []
    start = threading.Barrier(len(jobs))

    def worker(i):
        try:
            torch.cuda.set_device(cuda_dev)
            start.wait()
            out = None
            for _ in range(3):  # overlapping repeats on every stream
                out = jobs[i](streams[i])
            results[i] = out
        except Exception as e:  # reported below, in the main thread
            errors.append((i, repr(e)))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(jobs))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads), "a worker thread did not finish"
    assert not errors, errors
    for i, (a, b) in enumerate(zip(alone, results)):
        assert np.array_equal(a.view(np.uint32) if a.dtype == np.float32 else a,
                              b.view(np.uint32) if b.dtype == np.float32 else b), f"job {i} differs"
