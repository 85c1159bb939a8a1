"""GPU: the QKV producer (attn_qkv_rope.h) against the oracle (oracle/qkv_rope.py), which is
pinned to transformers' Qwen3 / GPT-J functions by the golden vectors.

Without an RMSNorm the producer's fp32 arithmetic is specified exactly, so Q, K and V must be
bit-identical to the oracle; with the norm (rsqrt is not correctly rounded) every q/k element
must lie within one bf16 ulp of the float64 value. Covers both pairings, partial rotary
dimensions, D = 64/128/256, the contiguous and the paged cache (rows not written keep their
bytes), decode appends at late positions, the rope table, a producer -> attention round trip,
and positions / page ids outside the cache (skipped and reported, the rest still written).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from oracle import qkv_rope as orq
from tests.gpu_util import scratch_for, to_dev

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
SENTINEL = 0x7F11  # a bf16 NaN pattern no producer output can take by rounding


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def _inputs(B, S, Hq, Hkv, D, seed, norm):
    rng = np.random.default_rng(seed)
    qkv = oracle.f32_to_bf16(rng.normal(0.0, 1.0, (B * S, (Hq + 2 * Hkv) * D)).astype(np.float32))
    qw = oracle.f32_to_bf16(rng.uniform(0.5, 1.5, D).astype(np.float32)) if norm else None
    kw = oracle.f32_to_bf16(rng.uniform(0.5, 1.5, D).astype(np.float32)) if norm else None
    return qkv, qw, kw


def _run_contig(dev, qkv, pos, table, qw, kw, eps, B, S, Hq, Hkv, D, rot, style, cache_len, K0=None, V0=None):
    q = torch.full((B * Hq * S * D,), SENTINEL, dtype=torch.int16, device=dev)
    k = to_dev(K0, dev) if K0 is not None else torch.full((B * Hkv * cache_len * D,), SENTINEL, dtype=torch.int16,
                                                          device=dev)
    v = to_dev(V0, dev) if V0 is not None else torch.full_like(k, SENTINEL)
    scratch = scratch_for(D, 128, dev)
    cs = to_dev(table, dev) if table is not None else None
    rc = ts.attn_qkv_rope_stream(to_dev(qkv, dev), to_dev(pos, dev), cs, 0 if table is None else table.shape[0],
                                 None if qw is None else to_dev(qw, dev), None if kw is None else to_dev(kw, dev), eps,
                                 B, S, Hq, Hkv, D, rot, style, q, k, v, cache_len, scratch)
    assert rc == ts.ATTN_OK, ts.strerror(rc)
    st = ts.attn_flash_status(scratch)
    return (_bits(q).reshape(B * Hq, S, D), _bits(k).reshape(B, Hkv, cache_len, D),
            _bits(v).reshape(B, Hkv, cache_len, D), st)


def _check_qk(got_bits, ref, exact):
    if exact:
        assert np.array_equal(got_bits, ref)
    else:
        ok = orq.within_one_ulp(got_bits, ref, atol=2e-6 * float(np.abs(ref).max()))
        assert ok.all(), f"{(~ok).sum()} of {ok.size} elements off by more than one bf16 ulp"


@pytest.mark.parametrize("D,rot,style,norm", [
    (128, 128, orq.NEOX, False), (128, 128, orq.NEOX, True), (128, 64, orq.NEOX, False),
    (64, 64, orq.GPTJ, False), (64, 32, orq.NEOX, True), (256, 64, orq.GPTJ, False),
    (256, 256, orq.NEOX, True), (128, 0, orq.NEOX, True), (128, 128, orq.GPTJ, True),
])
def test_contiguous_prompt(cuda_dev, D, rot, style, norm):
    """A prompt of S tokens per sequence at positions 0..S-1 into a cache of exactly S rows: the
    result is attn_flash's Q, K, V for that prompt."""
    B, S, Hq, Hkv = 2, 37, 8, 2
    qkv, qw, kw = _inputs(B, S, Hq, Hkv, D, 100 + D + rot, norm)
    pos = np.tile(np.arange(S, dtype=np.int32), B)
    table = orq.rope_table(S, rot, 1e6) if rot else None
    Q, K, V, st = _run_contig(cuda_dev, qkv, pos, table, qw, kw, 1e-6, B, S, Hq, Hkv, D, rot, style, S)
    assert st == (ts.ATTN_OK, 0)
    rQ, rK, rV = orq.produce(qkv, pos, table, qw, kw, 1e-6, B, S, Hq, Hkv, D, rot, style)
    _check_qk(Q, rQ, not norm)
    _check_qk(K, rK.transpose(0, 2, 1, 3), not norm)
    assert np.array_equal(V, rV.transpose(0, 2, 1, 3))


def test_decode_append_late_positions(cuda_dev):
    """One new token per sequence at its own late position (up to 131071) into a long cache:
    exactly row positions[b] of each (sequence, kv head) changes; every other row keeps its
    previous bytes."""
    B, S, Hq, Hkv, D, rot, L = 4, 1, 8, 2, 128, 128, 131072
    qkv, qw, kw = _inputs(B, S, Hq, Hkv, D, 7, True)
    pos = np.array([0, 5, 70000, L - 1], np.int32)
    table = orq.rope_table(L, rot, 1e6)
    rng = np.random.default_rng(3)
    K0 = rng.integers(0, 0x7F00, B * Hkv * L * D, dtype=np.uint16)
    V0 = rng.integers(0, 0x7F00, B * Hkv * L * D, dtype=np.uint16)
    Q, K, V, st = _run_contig(cuda_dev, qkv, pos, table, qw, kw, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX, L, K0, V0)
    assert st == (ts.ATTN_OK, 0)
    rQ, rK, rV = orq.produce(qkv, pos, table, qw, kw, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX)
    _check_qk(Q, rQ, False)
    K0 = K0.reshape(B, Hkv, L, D).copy()
    V0 = V0.reshape(B, Hkv, L, D).copy()
    for b in range(B):
        _check_qk(K[b, :, pos[b]], rK[b, 0], False)
        assert np.array_equal(V[b, :, pos[b]], rV[b, 0])
        K0[b, :, pos[b]] = K[b, :, pos[b]]
        V0[b, :, pos[b]] = V[b, :, pos[b]]
    assert np.array_equal(K, K0) and np.array_equal(V, V0)


@pytest.mark.parametrize("page_size", [16, 64, 128])
def test_paged_cache(cuda_dev, page_size):
    """Tokens of a multi-token step at positions ragged per sequence land in shuffled pages of
    the pool; unwritten page rows (and spare pages) keep their bytes."""
    B, S, Hq, Hkv, D, rot = 3, 20, 8, 2, 128, 128
    start = [0, 45, 300]
    max_pages = (max(start) + S + page_size - 1) // page_size
    num_pages = B * max_pages + 2
    rng = np.random.default_rng(page_size)
    perm = rng.permutation(num_pages)[:B * max_pages].astype(np.int32)
    table_b = perm.reshape(B, max_pages)
    pos = np.concatenate([np.arange(s0, s0 + S, dtype=np.int32) for s0 in start])
    qkv, qw, kw = _inputs(B, S, Hq, Hkv, D, 21, False)
    cs = orq.rope_table(512, rot, 1e6)
    pool0 = rng.integers(0, 0x7F00, num_pages * Hkv * page_size * D, dtype=np.uint16)
    dev = cuda_dev
    q = torch.full((B * Hq * S * D,), SENTINEL, dtype=torch.int16, device=dev)
    kp, vp = to_dev(pool0, dev), to_dev(pool0[::-1].copy(), dev)
    scratch = scratch_for(D, 128, dev)
    rc = ts.attn_qkv_rope_paged_stream(to_dev(qkv, dev), to_dev(pos, dev), to_dev(cs, dev), cs.shape[0], None, None,
                                       1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX, q, kp, vp, to_dev(table_b, dev),
                                       page_size, num_pages, max_pages, scratch)
    assert rc == ts.ATTN_OK
    assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)
    rQ, rK, rV = orq.produce(qkv, pos, cs, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX)
    assert np.array_equal(_bits(q).reshape(B * Hq, S, D), rQ)
    K = _bits(kp).reshape(num_pages, Hkv, page_size, D)
    V = _bits(vp).reshape(num_pages, Hkv, page_size, D)
    Kx = pool0.reshape(num_pages, Hkv, page_size, D).copy()
    Vx = pool0[::-1].copy().reshape(num_pages, Hkv, page_size, D)
    for b in range(B):
        for s in range(S):
            p = int(pos[b * S + s])
            pg, r = int(table_b[b, p // page_size]), p % page_size
            Kx[pg, :, r] = rK[b, s]
            Vx[pg, :, r] = rV[b, s]
    assert np.array_equal(K, Kx) and np.array_equal(V, Vx)


@pytest.mark.parametrize("name", ["rope_qwen3_norm", "rope_neox_plain_longpos", "rope_gptj_partial"])
def test_golden_vectors(cuda_dev, name):
    """The producer on the fixture inputs against transformers' fp32 outputs rounded to bf16:
    exact without a norm, within one bf16 ulp with Qwen3's q/k RMSNorm."""
    c = json.loads((GOLDEN / "rope_manifest.json").read_text())[name]
    z = np.load(GOLDEN / f"{name}.npz")
    B, S, Hq, Hkv, D, rot = c["B"], c["S"], c["Hq"], c["Hkv"], c["D"], c["rot"]
    table = orq.rope_table(c["max_pos"], rot, c["theta"])
    pos = z["positions"]
    qw = z["q_norm"] if c["norm"] else None
    kw = z["k_norm"] if c["norm"] else None
    Q, K, V, st = _run_contig(cuda_dev, z["qkv"], np.tile(np.arange(S, dtype=np.int32), B), None, None, None, 0.0,
                              B, S, Hq, Hkv, D, 0, c["style"], S)  # rot=0 first: a pure layout pass
    x = z["qkv"].reshape(B, S, Hq + 2 * Hkv, D)
    assert np.array_equal(Q, x[:, :, :Hq].transpose(0, 2, 1, 3).reshape(B * Hq, S, D))
    # Now the real call, each token at its fixture position, into a cache as long as the table.
    L = c["max_pos"]
    Q, K, V, st = _run_contig(cuda_dev, z["qkv"], pos, table, qw, kw, c["eps"], B, S, Hq, Hkv, D, rot, c["style"], L)
    assert st == (ts.ATTN_OK, 0)
    ref_q = z["q_out"].transpose(0, 2, 1, 3).reshape(B * Hq, S, D)
    ref_k = z["k_out"]  # [B][S][Hkv][D]
    got_k = np.stack([K[b, :, pos[b * S + s]] for b in range(B) for s in range(S)]).reshape(B, S, Hkv, D)
    if c["norm"]:
        _check_qk(Q, ref_q.astype(np.float64), False)
        _check_qk(got_k, ref_k.astype(np.float64), False)
    else:
        assert np.array_equal(Q, oracle.f32_to_bf16(ref_q))
        assert np.array_equal(got_k, oracle.f32_to_bf16(ref_k))


def test_rope_table(cuda_dev):
    """attn_rope_table_stream against the float64 definition rounded to fp32: within one fp32
    ulp everywhere, equal almost everywhere."""
    for max_pos, rot, theta in [(131072, 128, 1e6), (4096, 64, 1e4), (100, 256, 5e5)]:
        t = torch.empty(max_pos * rot, dtype=torch.float32, device=cuda_dev)
        assert ts.attn_rope_table_stream(t, max_pos, rot, theta) == ts.ATTN_OK
        got = t.cpu().numpy().reshape(max_pos, rot)
        ref = orq.rope_table(max_pos, rot, theta)
        diff = np.abs(got.astype(np.float64) - ref)
        assert diff.max() <= 1.2e-7, diff.max()
        assert (got == ref).mean() > 0.999


def test_producer_then_attention(cuda_dev):
    """Producer output fed straight to attn_flash_stream: the attention of the oracle-produced
    Q/K/V (same bits), checked against the fp32 attention oracle."""
    B, S, Hq, Hkv, D, rot = 1, 256, 8, 2, 128, 128
    qkv, qw, kw = _inputs(B, S, Hq, Hkv, D, 5, False)
    pos = np.arange(S, dtype=np.int32)
    table = orq.rope_table(S, rot, 1e6)
    Q, K, V, st = _run_contig(cuda_dev, qkv, pos, table, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX, S)
    assert st == (ts.ATTN_OK, 0)
    rQ, rK, rV = orq.produce(qkv, pos, table, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX)
    Qh, Kh, Vh = rQ.reshape(-1), rK.transpose(0, 2, 1, 3).reshape(-1), rV.transpose(0, 2, 1, 3).reshape(-1)
    q, k, v = to_dev(Q.reshape(-1), cuda_dev), to_dev(K.reshape(-1), cuda_dev), to_dev(V.reshape(-1), cuda_dev)
    o = torch.empty(Hq * S * D, dtype=torch.float32, device=cuda_dev)
    ts.attn_flash_checked(q, k, v, o, Hq, Hkv, S, S, D, 1, 128, scratch_for(D, 128, cuda_dev))
    rows = np.arange(S, dtype=np.int32)
    ref = oracle.attn_ref(Qh, Kh, Vh, Hq, Hkv, S, S, D, 1, rows)
    assert oracle.passes(oracle.cmp_rows(ref, o.cpu().numpy(), Hq, S, D, rows))


def test_bad_positions_are_skipped_and_reported(cuda_dev):
    """Positions past the table or the cache, and a negative one, skip those tokens whole and
    set the status; the valid tokens are still written; the next clean call reports OK."""
    B, S, Hq, Hkv, D, rot, L = 1, 6, 4, 2, 64, 64, 32
    qkv, _, _ = _inputs(B, S, Hq, Hkv, D, 9, False)
    pos = np.array([0, 31, 32, -1, 40, 3], np.int32)
    table = orq.rope_table(36, rot, 1e4)  # 32 <= p < 36 is inside the table but past the cache
    Q, K, V, st = _run_contig(cuda_dev, qkv, pos, table, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX, L)
    assert st[0] == ts.ATTN_ERR_DEVICE and st[1] == 1 << 6
    good = [0, 1, 5]
    rQ, rK, _ = orq.produce(qkv, np.where(pos < 0, 0, np.minimum(pos, 35)), table, None, None, 1e-6, B, S, Hq, Hkv, D,
                            rot, orq.NEOX)
    assert np.array_equal(Q[:, good], rQ[:, good])
    assert np.all(Q[:, [2, 3, 4]] == SENTINEL)
    for s in good:
        assert np.array_equal(K[0, :, pos[s]], rK[0, s])
    written = {int(pos[s]) for s in good}
    assert all(np.all(K[0, :, r] == SENTINEL) for r in range(L) if r not in written)
    Q, K, V, st = _run_contig(cuda_dev, qkv, np.arange(S, dtype=np.int32), table, None, None, 1e-6, B, S, Hq, Hkv, D,
                              rot, orq.NEOX, L)
    assert st == (ts.ATTN_OK, 0)


def test_bad_page_is_reported(cuda_dev):
    B, S, Hq, Hkv, D, rot, P = 2, 2, 4, 1, 64, 64, 16
    qkv, _, _ = _inputs(B, S, Hq, Hkv, D, 10, False)
    table_b = np.array([[0, 1], [2, 9]], np.int32)  # page 9 is outside a pool of 4
    pos = np.array([0, 1, 15, 16], np.int32)  # sequence 1's second token falls in page 9
    dev = cuda_dev
    cs = to_dev(orq.rope_table(64, rot, 1e4), dev)
    q = torch.full((B * Hq * S * D,), SENTINEL, dtype=torch.int16, device=dev)
    kp = torch.full((4 * Hkv * P * D,), SENTINEL, dtype=torch.int16, device=dev)
    vp = torch.full_like(kp, SENTINEL)
    scratch = scratch_for(D, 128, dev)
    rc = ts.attn_qkv_rope_paged_stream(to_dev(qkv, dev), to_dev(pos, dev), cs, 64, None, None, 1e-6, B, S, Hq, Hkv, D,
                                       rot, orq.NEOX, q, kp, vp, to_dev(table_b, dev), P, 4, 2, scratch)
    assert rc == ts.ATTN_OK
    assert ts.attn_flash_status(scratch) == (ts.ATTN_ERR_DEVICE, 1 << 5)
    Qb = _bits(q).reshape(B * Hq, S, D)
    assert np.all(Qb[Hq:, 1] == SENTINEL) and not np.any(Qb[:Hq] == SENTINEL)


def test_empty_batch_is_a_no_op(cuda_dev):
    """B*S = 0 tokens: the call succeeds, launches nothing that writes, and reports a clean status."""
    D = 128
    q = torch.full((64,), SENTINEL, dtype=torch.int16, device=cuda_dev)
    k = torch.full((64,), SENTINEL, dtype=torch.int16, device=cuda_dev)
    v = torch.full_like(k, SENTINEL)
    qkv = torch.zeros(8, dtype=torch.int16, device=cuda_dev)
    pos = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    cs = to_dev(orq.rope_table(4, D, 1e4), cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    for B, S in ((0, 5), (3, 0)):
        rc = ts.attn_qkv_rope_stream(qkv, pos, cs, 4, None, None, 1e-6, B, S, 4, 2, D, D, orq.NEOX, q, k, v, 4,
                                     scratch)
        assert rc == ts.ATTN_OK
        assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)
    assert np.all(_bits(q) == SENTINEL) and np.all(_bits(k) == SENTINEL) and np.all(_bits(v) == SENTINEL)


@pytest.mark.parametrize("Hq,Hkv", [(6, 6), (5, 3), (1, 1)])
def test_head_layouts(cuda_dev, Hq, Hkv):
    """MHA (Hq = Hkv), a head count that is not a multiple of Hkv (the producer does not need
    one), and a single head: every head lands where the oracle puts it, bit for bit."""
    B, S, D, rot = 2, 11, 64, 64
    qkv, _, _ = _inputs(B, S, Hq, Hkv, D, 50 + Hq + Hkv, False)
    pos = np.tile(np.arange(S, dtype=np.int32), B)
    table = orq.rope_table(S, rot, 1e4)
    Q, K, V, st = _run_contig(cuda_dev, qkv, pos, table, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX, S)
    assert st == (ts.ATTN_OK, 0)
    rQ, rK, rV = orq.produce(qkv, pos, table, None, None, 1e-6, B, S, Hq, Hkv, D, rot, orq.NEOX)
    assert np.array_equal(Q, rQ)
    assert np.array_equal(K, rK.transpose(0, 2, 1, 3)) and np.array_equal(V, rV.transpose(0, 2, 1, 3))
