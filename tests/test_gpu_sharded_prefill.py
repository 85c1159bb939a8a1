"""GPU: the (batch x kv-head group) sharded prefill (transfer_station_b200.multigpu.sharded_prefill)
through the C ABI, every rank's share run in turn on one GPU, checked against the fp32
reference. The split is flash.c's head loop (flash.c:779-782, kv = h / group) partitioned by
kv head; on N GPUs each rank runs exactly the call made here for its rank (tests/test_multigpu.py
runs it on 2 GPUs)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import scratch_for, to_dev
from transfer_station_b200 import multigpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 2, 3, 8, 40])
def test_sharded_prefill_all_ranks_on_one_gpu(cuda_dev, world):
    """Config 5's head layout (64/8 heads per sequence) at batch 4 and S=2048: 32 units over
    `world` ranks, including uneven shares (3) and more ranks than units (40: idle ranks). Every
    rank writes only its own rows (O starts NaN), and the assembled O matches the reference."""
    B, Hq, Hkv, S, D = 4, 64, 8, 2048, 128
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, S, S, D, seed=4, a=0.0, b=0.5)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    O = torch.full((B * Hq * S * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    covered = 0
    for rank in range(world):
        s = multigpu.sharded_prefill(q, k, v, O, B, Hq, Hkv, S, S, D, 0, scratch, rank=rank, world=world)
        torch.cuda.synchronize()
        assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)
        assert s.u0 == covered
        covered = s.u1
        # nothing past this rank's units has been written yet
        assert torch.isnan(O[s.q_off + s.hq * S * D:]).all()
    assert covered == B * Hkv
    out = O.cpu().numpy()
    rows = oracle.rowset(S, 6)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, rows)
    c = oracle.cmp_rows(ref, out, B * Hq, S, D, rows)
    assert oracle.passes(c), c


def test_sharded_prefill_causal_uneven(cuda_dev):
    """Causal, GQA 6/2 heads per sequence, batch 3, Sq=300, Sk=420: 6 units over 4 ranks."""
    B, Hq, Hkv, Sq, Sk, D = 3, 6, 2, 300, 420, 64
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, Sq, Sk, D, seed=9)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    O = torch.full((B * Hq * Sq * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    for rank in range(4):
        multigpu.sharded_prefill(q, k, v, O, B, Hq, Hkv, Sq, Sk, D, 1, scratch, rank=rank, world=4)
    torch.cuda.synchronize()
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, Sq, Sk, D, 1, rows)
    c = oracle.cmp_rows(ref, O.cpu().numpy(), B * Hq, Sq, D, rows)
    assert oracle.passes(c), c
