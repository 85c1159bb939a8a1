"""GPU parity at the BASELINE configs' full sizes, against both of the reference's checks.

The benchmark times configs 2-5 at their full batch sizes, and the work plan (units, key
pieces, last-wave split, persistent items) depends on those sizes, so the exact shapes that
are timed are checked here, as the reference's harness checks every case before timing it
(flash.c:1095-1100, ahead of the timed loop at flash.c:1113-1123):

* against the fp32 reference attn_ref (flash.c:262-314, restated bit-exactly in oracle/) on
  spread query rows of every head, the last row always included (ref_rowset, flash.c:889-931);
* against the reference KERNEL itself -- flash.c's own attn_flash (flash.c:727-864) compiled
  from the reference sources into oracle/_ref -- on head x row-slice sub-problems. A slice of
  rows [r0, r0+n) of head h is the same computation as the full problem for those rows when
  its kv head's first Sk - Sq + r0 + n keys are passed (that keeps bottom-right causal
  alignment; non-causal slices take every key).

Bounds are the parity tests' (oracle.passes): mad <= 8e-3 * maxref with nbad == 0, max abs
<= 2e-2 and relative L2 <= 1e-2.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle
from tests.gpu_util import run_gpu

pytestmark = pytest.mark.gpu


def _check(ref, out, Hq, Sq, D, rows, what):
    c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
    assert oracle.passes(c), f"{what}: {c}"
    return c


def _slices(Hq, Sq, nslices, nrows, seed):
    """(head, first row, rows) slices spread over heads, the last one ending at row Sq-1."""
    rng = np.random.default_rng(seed)
    n = min(nrows, Sq)
    out = []
    for s in range(nslices):
        h = int(rng.integers(Hq)) if s else Hq - 1
        r0 = Sq - n if s == 0 else int(rng.integers(0, Sq - n + 1))
        out.append((h, r0, n))
    return out


def check_against_reference_kernel(Q, K, V, out, Hq, Hkv, Sq, Sk, D, causal, nslices=8, nrows=16, what=""):
    """Compares `out` (the GPU's [Hq][Sq][D] fp32 result) with flash.c's own attn_flash run on
    head x row-slice sub-problems (one host thread per slice)."""
    if not oracle.ref_available(128):
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built")
    group = Hq // Hkv
    Q3, K3, V3 = Q.reshape(Hq, Sq, D), K.reshape(Hkv, Sk, D), V.reshape(Hkv, Sk, D)
    O3 = out.reshape(Hq, Sq, D)

    def one(sl):
        h, r0, n = sl
        kv = h // group
        sk = Sk - Sq + r0 + n if causal else Sk
        sk = min(sk, Sk)
        if sk < 1:  # every row of the slice attends no key: the output rows are exact zeros
            assert np.all(O3[h, r0:r0 + n] == 0.0)
            return None
        q = np.ascontiguousarray(Q3[h, r0:r0 + n])
        k = np.ascontiguousarray(K3[kv, :sk])
        v = np.ascontiguousarray(V3[kv, :sk])
        ref = oracle.ref_attn_flash(q, k, v, 1, 1, n, sk, D, causal, bk=128, bq=128)
        got = np.ascontiguousarray(O3[h, r0:r0 + n]).reshape(-1)
        return sl, oracle.cmp_rows(ref, got, 1, n, D, np.arange(n, dtype=np.int32))

    with ThreadPoolExecutor(max_workers=nslices) as ex:
        for res in ex.map(one, _slices(Hq, Sq, nslices, nrows, seed=Sq + Sk + Hq)):
            if res is not None:
                sl, c = res
                assert oracle.passes(c), f"{what} vs reference kernel, slice {sl}: {c}"


def _run_case(Hq, Hkv, Sq, Sk, D, causal, seed, dist, a, b, cap, what, nrows=16):
    import torch

    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=seed, dist=dist, a=a, b=b)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=torch.device("cuda:0"))
    rows = oracle.rowset(Sq, cap) if Sq > 1 else np.arange(1, dtype=np.int32)
    assert rows[-1] == Sq - 1
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    _check(ref, out, Hq, Sq, D, rows, what + " vs fp32 reference")
    check_against_reference_kernel(Q, K, V, out, Hq, Hkv, Sq, Sk, D, causal, nrows=nrows, what=what)


@pytest.mark.parametrize("S,causal", [(1024, 0), (2048, 0), (4096, 0), (1024, 1), (2048, 1), (4096, 1)])
def test_config2_prefill_full(cuda_dev, S, causal):
    """Config 2: Qwen3-8B-shaped GQA prefill, batch 1, 32/8 heads, D=128, N(0,1) seed 1."""
    _run_case(32, 8, S, S, 128, causal, 1, "normal", 0.0, 1.0, 16, f"config2 S={S} causal={causal}")


def test_config3_decode_b64(cuda_dev):
    """Config 3 at its full batch: decode B=64, 32/8 heads, Sk=8192, N(0,1) seed 2 (2 GiB of K/V)."""
    B = 64
    _run_case(B * 32, B * 8, 1, 8192, 128, 0, 2, "normal", 0.0, 1.0, 1, "config3 decode B=64", nrows=1)


def test_config4_prefill_b8(cuda_dev):
    """Config 4 prefill at its full batch: MQA 16/1 heads, B=8, Sq=Sk=2048, U(-2,2) seed 3."""
    B = 8
    _run_case(B * 16, B * 1, 2048, 2048, 128, 0, 3, "uniform", -2.0, 2.0, 8, "config4 prefill B=8")


def test_config4_decode_b128(cuda_dev):
    """Config 4 decode at its full batch: MQA 16/1 heads, B=128, Sk=4096, U(-2,2) seed 3."""
    B = 128
    _run_case(B * 16, B * 1, 1, 4096, 128, 0, 3, "uniform", -2.0, 2.0, 1, "config4 decode B=128", nrows=1)


def test_config5_prefill_b4(cuda_dev):
    """Config 5 prefill at its full batch on one GPU: B=4, 64/8 heads, Sq=Sk=16384, N(0,0.5)
    seed 4 (256 query heads x 16384 rows; 2 GiB of fp32 output)."""
    B = 4
    _run_case(B * 64, B * 8, 16384, 16384, 128, 0, 4, "normal", 0.0, 0.5, 3, "config5 prefill B=4", nrows=8)


def test_config5_decode_b4(cuda_dev):
    """Config 5 decode at its full batch on one GPU: B=4, 64/8 heads, Sk=131072, N(0,0.5) seed 4."""
    B = 4
    _run_case(B * 64, B * 8, 1, 131072, 128, 0, 4, "normal", 0.0, 0.5, 1, "config5 decode B=4", nrows=1)
