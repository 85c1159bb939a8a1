"""GPU: repeated calls give bit-identical results, whatever ran before them.

Tensor memory (TMEM) and the caller's scratch block keep their contents from one launch to the
next, so a kernel that read TMEM or scratch before writing it in the same launch would return
results that depend on the previous call. Each case here runs once, then an unrelated problem
(other shapes and data, leaving different TMEM and scratch contents behind), then again: both
runs must match the fp32 oracle and each other bit for bit. The cases cover every work plan of
the tensor-core path: whole units, key pieces merged by the combine kernel, the split of only
the last wave's units, causal ordering, and decode.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.gpu_util import run_gpu, scratch_for

pytestmark = pytest.mark.gpu

CASES = [
    # (name, Hq, Hkv, Sq, Sk, D, causal)
    ("key pieces", 8, 2, 150, 1000, 128, 0),
    ("key pieces causal", 8, 2, 150, 1000, 128, 1),
    ("last wave split", 32, 8, 1200, 1200, 128, 0),
    ("causal longest first", 32, 8, 1200, 1200, 128, 1),
    ("decode", 64, 8, 1, 4096, 128, 0),
    ("head dim 64", 16, 4, 600, 900, 64, 0),
]


def _other_problem(dev):
    """Different shapes and data: leaves other TMEM and scratch contents behind."""
    Q, K, V = oracle.seeded_inputs(16, 2, 700, 1500, 128, seed=99, dist="uniform", a=-3.0, b=3.0)
    run_gpu(Q, K, V, 16, 2, 700, 1500, 128, 1, dev=dev)


@pytest.mark.parametrize("name,Hq,Hkv,Sq,Sk,D,causal", CASES, ids=[c[0] for c in CASES])
def test_repeat_is_bit_identical(cuda_dev, name, Hq, Hkv, Sq, Sk, D, causal):
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=7)
    rows = oracle.rowset(Sq, 24 if Sq > 24 else 0)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    scratch = scratch_for(D, 128, cuda_dev)
    first = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev, scratch=scratch)
    _other_problem(cuda_dev)
    scratch.fill_(0xFF)  # NaN in every partial slot: an unwritten slot cannot pass
    second = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev, scratch=scratch)
    torch.cuda.synchronize()
    for out, which in ((first, "first"), (second, "second")):
        c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
        assert oracle.passes(c), f"{name} ({which} call): {c}"
    assert np.array_equal(first.view(np.uint32), second.view(np.uint32)), f"{name}: repeated call differs"
