"""attn_flash_noalloc: the entry point for callers that cannot allocate device memory.

Some callers cannot hand the library a scratch block: their device memory is owned by their
own pool allocator and third-party code may not call cudaMalloc, or they reach the library
through a foreign-function binding with nowhere to keep a device buffer alive between calls.
attn_flash_noalloc takes no scratch argument and uses a fixed 4 MiB block the library itself
declares. These tests call it through the C ABI and compare it with attn_flash_stream (which
uses a caller-owned scratch block) on the same inputs, with the parity tests' tolerance, on
two calls in a row -- the second with different inputs, so contents left in the shared block
by the first call cannot leak into the second result.

This file is named to be collected last, so a run that stops at its first failure has
already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import to_dev, run_gpu

pytestmark = pytest.mark.gpu

# decode-shaped calls (the entry point's intended use) and one small prefill
CASES = [
    # (Hq, Hkv, Sq, Sk, D, causal, seed)
    (8 * 32, 8 * 8, 1, 8192, 128, 0, 2),    # GQA decode, batch 8: splits the key axis
    (64, 8, 1, 131072, 128, 0, 4),          # long-context decode: many splits
    (16 * 16, 16, 1, 4096, 128, 0, 3),      # MQA decode, batch 16
    (8, 2, 200, 300, 64, 1, 5),             # small causal prefill (no split)
    (6, 3, 1, 1000, 36, 0, 6),              # head_dim not a multiple of 8: the general path
    (4096, 512, 1, 8192, 128, 0, 7),        # exactly the 4096-row limit: two pieces no longer fit, no split
    (2048, 256, 1, 8192, 128, 0, 8),        # 2048 rows: at most three pieces fit the block
]


def _noalloc(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev):
    q, k, v = to_dev(Q, dev), to_dev(K, dev), to_dev(V, dev)
    o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
    rc = ts.attn_flash_noalloc(q, k, v, o, Hq, Hkv, Sq, Sk, D, causal, 128)
    assert rc == ts.ATTN_OK, ts.strerror(rc)
    return o.cpu().numpy()


@pytest.mark.parametrize("case", CASES, ids=[f"Hq{c[0]}_Sq{c[2]}_Sk{c[3]}_D{c[4]}_c{c[5]}" for c in CASES])
def test_noalloc_matches_scratch_entry_point(cuda_dev, case):
    """Each call is checked twice: against attn_flash_stream on the same inputs, and against the
    fp32 reference (attn_ref, flash.c:262-314) on its own, so a planning fault the two entry
    points shared would still be caught."""
    Hq, Hkv, Sq, Sk, D, causal, seed = case
    rows = np.arange(Sq, dtype=np.int32)
    for call in range(2):  # two calls in a row, different data each time
        Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=seed + 100 * call)
        want = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev)
        got = _noalloc(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, cuda_dev)
        c = oracle.cmp_rows(want, got, Hq, Sq, D, rows)
        assert oracle.passes(c), f"call {call} vs attn_flash_stream: {c}"
        ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
        c = oracle.cmp_rows(ref, got, Hq, Sq, D, rows)
        assert oracle.passes(c), f"call {call} vs fp32 reference: {c}"


def test_noalloc_rejects_oversized_calls(cuda_dev):
    """More than 4096 query rows is beyond the fixed block's stated limit: a clear error. So is
    a K/V whose rows (Hkv * Sk) do not fit a 32-bit index, which the other entry points also
    reject; neither call launches anything (the tensors are too small to be read)."""
    Hq, Hkv, Sq, Sk, D = 32, 8, 256, 256, 64
    q = torch.zeros(Hq * Sq * D, dtype=torch.int16, device=cuda_dev)
    k = torch.zeros(Hkv * Sk * D, dtype=torch.int16, device=cuda_dev)
    o = torch.zeros(Hq * Sq * D, dtype=torch.float32, device=cuda_dev)
    assert ts.attn_flash_noalloc(q, k, k, o, Hq, Hkv, Sq, Sk, D, 0, 128) == ts.ATTN_ERR_ARGS
    assert ts.attn_flash_noalloc(q, k, k, o, 8, 8, 1, 1 << 28, D, 0, 128) == ts.ATTN_ERR_ARGS


def test_noalloc_refuses_a_capturing_stream(cuda_dev):
    """Every call synchronises its stream, which a stream capture forbids: on a capturing stream
    the call returns ATTN_ERR_ARGS before touching anything, and the capture stays usable."""
    Hq, Hkv, Sq, Sk, D = 8, 2, 1, 256, 64
    q = torch.zeros(Hq * Sq * D, dtype=torch.int16, device=cuda_dev)
    k = torch.zeros(Hkv * Sk * D, dtype=torch.int16, device=cuda_dev)
    o = torch.zeros(Hq * Sq * D, dtype=torch.float32, device=cuda_dev)
    assert ts.attn_flash_noalloc(q, k, k, o, Hq, Hkv, Sq, Sk, D, 0, 128) == ts.ATTN_OK
    s = torch.cuda.Stream(device=cuda_dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        rc = ts.attn_flash_noalloc(q, k, k, o, Hq, Hkv, Sq, Sk, D, 0, 128, stream=s)
        o.add_(1.0)  # the capture still records work after the refused call
    assert rc == ts.ATTN_ERR_ARGS
    o.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.all(o == 1.0)
