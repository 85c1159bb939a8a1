"""GPU: the key-sharded partial-attention API used by multi-GPU long-context decode
(attn_flash_partial_stream + attn_flash_combine_stream). Key shards are emulated on one GPU:
each shard's K/V slice goes through the partial entry with its global key offset, the partials
are stacked as an all-gather would stack them, and the combine must reproduce the one-shot
attention (fp32 oracle, flash.c:262-314) within the parity tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import scratch_for, to_dev

pytestmark = pytest.mark.gpu


def _sharded(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, bounds, dev):
    rows = Hq * Sq
    world = len(bounds) - 1
    m = torch.empty(world, rows, dtype=torch.float32, device=dev)
    l = torch.empty(world, rows, dtype=torch.float32, device=dev)
    acc = torch.empty(world, rows, D, dtype=torch.float32, device=dev)
    K3 = K.reshape(Hkv, Sk, D)
    V3 = V.reshape(Hkv, Sk, D)
    q = to_dev(Q, dev)
    scratch = scratch_for(D, 128, dev)
    for r in range(world):
        k0, k1 = bounds[r], bounds[r + 1]
        ks = to_dev(np.ascontiguousarray(K3[:, k0:k1]).reshape(-1), dev)
        vs = to_dev(np.ascontiguousarray(V3[:, k0:k1]).reshape(-1), dev)
        rc = ts.attn_flash_partial_stream(q, ks, vs, m[r], l[r], acc[r], Hq, Hkv, Sq, k1 - k0, Sk, k0, D, causal,
                                          128, scratch)
        assert rc == ts.ATTN_OK, ts.strerror(rc)
        rc, code = ts.attn_flash_status(scratch)
        assert rc == ts.ATTN_OK, code
    o = torch.empty(rows * D, dtype=torch.float32, device=dev)
    assert ts.attn_flash_combine_stream(m, l, acc, world, rows, D, o) == ts.ATTN_OK
    torch.cuda.synchronize()
    return o.cpu().numpy(), m.cpu().numpy()


@pytest.mark.parametrize("world", [2, 4])
def test_key_sharded_decode_matches_full(cuda_dev, world):
    """BASELINE config 5 decode shape at batch 1 with Sk=32768 split over `world` shards."""
    Hq, Hkv, Sq, Sk, D = 64, 8, 1, 32768, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=4, a=0.0, b=0.5)
    bounds = [Sk * r // world for r in range(world + 1)]
    out, _ = _sharded(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, bounds, cuda_dev)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
    assert oracle.passes(c), c


def test_key_sharded_causal_uneven(cuda_dev):
    """Causal masking uses global key positions: a multi-row query block against uneven key
    shards. Row i attends keys <= Sk - Sq + i = 604 + i, so the last shard [650, 700) holds
    only future keys for rows i < 46 and must report m = -inf (no key seen) exactly there."""
    Hq, Hkv, Sq, Sk, D = 8, 2, 96, 700, 64
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    bounds = [0, 130, 650, 700]
    out, m = _sharded(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, bounds, cuda_dev)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, rows)
    c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
    assert oracle.passes(c), c
    last = m.reshape(3, Hq, Sq)[2]
    assert np.all(np.isneginf(last[:, :46])) and np.all(np.isfinite(last[:, 46:]))


def test_partial_of_whole_range_equals_attention(cuda_dev):
    """One shard holding every key: combine of a single partial is the attention itself."""
    Hq, Hkv, Sq, Sk, D = 32, 8, 4, 4096, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=9)
    out, _ = _sharded(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, [0, Sk], cuda_dev)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    assert oracle.passes(oracle.cmp_rows(ref, out, Hq, Sq, D, rows))


@pytest.mark.parametrize("nparts", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("rows,D", [(9, 64), (17, 70), (512, 128)])
def test_packed_combine_equals_separate(cuda_dev, nparts, rows, D):
    """attn_flash_combine_packed_stream over back-to-back packed blocks (what one all-gather of
    the ranks' blocks yields) gives the same bits as attn_flash_combine_stream over separate
    m, l, acc arrays: odd row counts exercise the padding before acc, D=70 the unvectorised
    kernel, and a part with m = -inf (an empty key shard) must contribute nothing."""
    g = torch.Generator().manual_seed(rows * 31 + nparts)
    m = torch.randn(nparts, rows, generator=g) * 4
    l = torch.rand(nparts, rows, generator=g) * 50 + 1
    acc = torch.randn(nparts, rows, D, generator=g)
    if nparts > 1:
        m[-1, ::3] = float("-inf")
        l[-1, ::3] = 0
        acc[-1, ::3] = 0
    stride = ts.attn_flash_packed_floats(rows, D)
    off = -(-2 * rows // 4) * 4
    assert stride == off + rows * D
    packed = torch.zeros(nparts, stride)
    packed[:, :rows] = m
    packed[:, rows:2 * rows] = l
    packed[:, off:] = acc.reshape(nparts, -1)
    md, ld, ad, pd = (t.contiguous().to(cuda_dev) for t in (m, l, acc, packed))
    o1 = torch.empty(rows * D, dtype=torch.float32, device=cuda_dev)
    o2 = torch.empty_like(o1)
    assert ts.attn_flash_combine_stream(md, ld, ad, nparts, rows, D, o1) == ts.ATTN_OK
    assert ts.attn_flash_combine_packed_stream(pd, nparts, rows, D, o2) == ts.ATTN_OK
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int32), o2.view(torch.int32))
    ref = oracle.combine(m.numpy(), l.numpy(), acc.numpy(), nparts, rows, D)  # m in the log2 domain
    assert np.allclose(o2.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)
