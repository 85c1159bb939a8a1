"""CPU: the work plan of the tensor-core path (attn_diag_plan: the planner's host arithmetic,
no device touched).

`model_plan` restates transfer_station_b200/csrc/attn_flash.c's ts_plan_core: first the split
plan, the number of key pieces s minimising ceil(units*s / SMs) * (blocks/s + 1) with every
piece >= 2 key blocks and the partials fitting ATTN_PARTIAL_ROWS; otherwise, without causal
masking, the tail split: a last wave of L <= SMs/2 units runs as floor(SMs/L) key pieces each.
"""
from __future__ import annotations

import random

import pytest

import transfer_station_b200 as ts

SMS = 148  # B200
PARTIAL_ROWS = 65536  # ATTN_PARTIAL_ROWS


def units_of(Hq, Hkv, Sq):
    rows = (Hq // Hkv) * Sq
    unit_rows = 256 if rows > 128 else 128
    return -(-rows // unit_rows) * Hkv, unit_rows


def model_plan(Hq, Hkv, Sq, Sk, causal, sms):
    rows = Hq * Sq
    nblk = -(-Sk // 128)
    ctas, unit_rows = units_of(Hq, Hkv, Sq)
    cap = PARTIAL_ROWS // rows
    smax = min(nblk // 2, cap, 256)
    best, best_t = 1, float("inf")
    for s in range(1, max(smax, 1) + 1):
        bps = -(-nblk // s)
        if -(-nblk // bps) != s:
            continue
        t = -(-(ctas * s) // sms) * (bps + 1.0)
        if t < best_t * 0.999:
            best, best_t = s, t
    bps = -(-nblk // best)
    plan = [best, bps * 128, 0, 0, ctas]
    if best > 1 or causal or ctas <= sms:
        return plan
    L = ctas % sms
    if L == 0 or 2 * L > sms:
        return plan
    tiles = ctas // Hkv
    u0 = ctas - L
    row_base = (u0 // tiles) * (Hq // Hkv) * Sq + (u0 % tiles) * unit_rows
    s = min(sms // L, nblk // 2)
    while s >= 2 and (rows - row_base) * s > PARTIAL_ROWS:
        s -= 1
    if s < 2:
        return plan
    bps = -(-nblk // s)
    return [-(-nblk // bps), bps * 128, u0, row_base, ctas]


def test_bench_shapes(built_lib):
    # config 2 at S=4096: 512 units = 3 waves + 68 -> the 68 run as 2 key pieces each
    p = ts.attn_diag_plan(32, 8, 4096, 4096, 128, 0, SMS)
    assert (p.nsplit, p.n_direct, p.units) == (2, 444, 512), p
    assert p.row_base == (444 // 64) * 4 * 4096 + (444 % 64) * 256
    # S=1024 and S=2048: whole units (one wave; a 73%-full second wave)
    for S, units in ((1024, 128), (2048, 256)):
        p = ts.attn_diag_plan(32, 8, S, S, 128, 0, SMS)
        assert (p.nsplit, p.n_direct, p.units) == (1, 0, units), p
    # config 3 decode: 512 one-tile units, every unit split in 2 pieces, merged by the combine
    p = ts.attn_diag_plan(2048, 512, 1, 8192, 128, 0, SMS)
    assert (p.nsplit, p.keys_per_split, p.n_direct, p.units) == (2, 4096, 0, 512), p
    # causal: no tail split (the longest-first walk evens the CTAs instead)
    p = ts.attn_diag_plan(32, 8, 4096, 4096, 128, 1, SMS)
    assert (p.nsplit, p.n_direct) == (1, 0), p


def test_planner_matches_its_model_sweep(built_lib):
    rng = random.Random(5)
    for _ in range(800):
        hkv = rng.choice([1, 2, 4, 8, 16, 64])
        hq = hkv * rng.choice([1, 2, 4, 8, 16])
        sq = rng.choice([1, 1, rng.randint(2, 9000), 1024, 2048, 4096])
        sk = rng.choice([sq, rng.randint(1, 40000)])
        causal = rng.choice([0, 1])
        sms = rng.choice([148, 132, 114, 16, 7, 1])
        got = list(ts.attn_diag_plan(hq, hkv, sq, sk, 128, causal, sms))
        assert got == model_plan(hq, hkv, sq, sk, causal, sms), (hq, hkv, sq, sk, causal, sms)
        nsplit, _, n_direct, row_base, _ = got
        assert nsplit == 1 or (hq * sq - row_base) * nsplit <= PARTIAL_ROWS  # the partials fit


def test_plan_rejects_bad_arguments(built_lib):
    with pytest.raises(ts.AttnError):
        ts.attn_diag_plan(6, 4, 10, 10, 64, 0, 148)  # Hq not a multiple of Hkv
    with pytest.raises(ts.AttnError):
        ts.attn_diag_plan(8, 2, 10, 10, 64, 0, 0)
    with pytest.raises(ts.AttnError):
        ts.attn_diag_plan(8, 2, 10, 0, 64, 0, 148)
