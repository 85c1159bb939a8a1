"""GPU: attn_flash_stream_out -- the same attention with O written as bf16 bits.

The fp32 and bf16 calls run the same kernels up to the final store, so every bf16 element must
equal the reference's own rounding (flash.c:78-92: round to nearest even, NaN/Inf passed
through) of the fp32 call's element, bit for bit -- on every path that stores O: the tensor-core
epilogue, the combine kernel that merges key pieces (the last wave of a prefill, decode), and
the general CUDA-core path. One case also checks the bf16 output against the fp32 reference.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import scratch_for, to_dev

pytestmark = pytest.mark.gpu

CASES = [
    # (name, Hq, Hkv, Sq, Sk, D, causal)
    ("prefill", 8, 2, 300, 520, 128, 0),
    ("causal", 8, 2, 300, 300, 128, 1),
    ("last wave split", 32, 8, 1200, 1200, 128, 0),
    ("decode pieces", 64, 8, 1, 8192, 128, 0),
    ("head dim 64", 8, 4, 200, 333, 64, 1),
    ("general path", 6, 3, 130, 300, 40, 0),
]


def rne_bf16(x: np.ndarray) -> np.ndarray:
    """flash.c:78-92 on an fp32 array: bf16 bits as uint16."""
    u = x.astype(np.float32).view(np.uint32)
    special = ((u >> 23) & 0xFF) == 0xFF
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (u >> 16).astype(np.uint16), r)


def _run(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev, out_dtype):
    q, k, v = to_dev(Q, dev), to_dev(K, dev), to_dev(V, dev)
    if out_dtype == ts.ATTN_OUT_BF16:
        o = torch.full((Hq * Sq * D,), -1, dtype=torch.int16, device=dev)
    else:
        o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
    scr = scratch_for(D, 128, dev)
    rc = ts.attn_flash_stream_out(q, k, v, o, out_dtype, Hq, Hkv, Sq, Sk, D, causal, 128, scr)
    assert rc == ts.ATTN_OK, ts.strerror(rc)
    rc, code = ts.attn_flash_status(scr)
    assert rc == ts.ATTN_OK, (ts.strerror(rc), code)
    return o.cpu().numpy()


@pytest.mark.parametrize("name,Hq,Hkv,Sq,Sk,D,causal", CASES, ids=[c[0] for c in CASES])
def test_bf16_output_is_the_rounded_fp32_output(cuda_dev, name, Hq, Hkv, Sq, Sk, D, causal):
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=11)
    o32 = _run(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, cuda_dev, ts.ATTN_OUT_F32)
    o16 = _run(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, cuda_dev, ts.ATTN_OUT_BF16).view(np.uint16)
    assert not np.isnan(o32).any()
    want = rne_bf16(o32)
    bad = np.nonzero(o16 != want)[0]
    assert bad.size == 0, f"{name}: {bad.size} elements differ, first at {bad[:5]}"


def test_f32_output_type_matches_attn_flash_stream(cuda_dev):
    Hq, Hkv, Sq, Sk, D = 8, 2, 200, 400, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=12)
    a = _run(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, cuda_dev, ts.ATTN_OUT_F32)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    o = torch.empty(Hq * Sq * D, dtype=torch.float32, device=cuda_dev)
    ts.attn_flash_checked(q, k, v, o, Hq, Hkv, Sq, Sk, D, 1, 128, scratch_for(D, 128, cuda_dev))
    assert np.array_equal(a.view(np.uint32), o.cpu().numpy().view(np.uint32))


def test_bf16_output_parity_with_fp32_reference(cuda_dev):
    Hq, Hkv, Sq, Sk, D = 32, 8, 1024, 1024, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=1)
    rows = oracle.rowset(Sq, 24)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    o16 = _run(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, cuda_dev, ts.ATTN_OUT_BF16).view(np.uint16)
    out = (o16.astype(np.uint32) << 16).view(np.float32)
    c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
    assert oracle.passes(c), c
