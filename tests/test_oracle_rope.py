"""CPU: the QKV-producer oracle (oracle/qkv_rope.py) against golden vectors made with
transformers' Qwen3 and GPT-J rotary/RMSNorm functions (tests/golden/make_rope_golden.py),
and its cos/sin table against the float64 definition."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import qkv_rope as orq

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "rope_manifest.json").read_text())


def _load(name):
    return MANIFEST[name], np.load(GOLDEN / f"{name}.npz")


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_matches_transformers(name):
    """Without a norm the oracle's fp32 arithmetic reproduces transformers' fp32 result bit for
    bit (x*cos + rotate(x)*sin rounds exactly like x*cos - y*sin); with Qwen3's q/k RMSNorm the
    float64 oracle agrees to fp32 rounding."""
    c, z = _load(name)
    B, S, Hq, Hkv, D = c["B"], c["S"], c["Hq"], c["Hkv"], c["D"]
    T = B * S
    x = oracle.bf16_to_f32(z["qkv"]).reshape(T, Hq + 2 * Hkv, D)
    rows = z["rows"][:, None, :]
    ref_q = z["q_out"].reshape(T, Hq, D)
    ref_k = z["k_out"].reshape(T, Hkv, D)
    if not c["norm"]:
        got_q = orq.rope_f32(x[:, :Hq], rows, c["rot"], c["style"])
        got_k = orq.rope_f32(x[:, Hq:Hq + Hkv], rows, c["rot"], c["style"])
        assert np.array_equal(got_q.view(np.uint32), ref_q.view(np.uint32))
        assert np.array_equal(got_k.view(np.uint32), ref_k.view(np.uint32))
    else:
        qn = orq.rms_norm_f64(x[:, :Hq], oracle.bf16_to_f32(z["q_norm"]), c["eps"])
        kn = orq.rms_norm_f64(x[:, Hq:Hq + Hkv], oracle.bf16_to_f32(z["k_norm"]), c["eps"])
        got_q = orq.rope_f64(qn, rows, c["rot"], c["style"])
        got_k = orq.rope_f64(kn, rows, c["rot"], c["style"])
        for got, ref in ((got_q, ref_q), (got_k, ref_k)):
            scale = np.abs(ref).max(axis=-1, keepdims=True)
            assert np.all(np.abs(got - ref) <= 4e-6 * scale)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_fixture_rows_are_the_table(name):
    c, z = _load(name)
    table = orq.rope_table(c["max_pos"], c["rot"], c["theta"])
    assert np.array_equal(table[z["positions"]], z["rows"])


def test_table_definition():
    """cos/sin of p * theta^(-2i/rot) evaluated one scalar at a time in double precision."""
    rot, theta = 32, 1e6
    t = orq.rope_table(70000, rot, theta)
    for p in (0, 1, 17, 4095, 69999):
        for i in range(rot // 2):
            a = p * theta ** (-2.0 * i / rot)
            assert t[p, i] == np.float32(math.cos(a)) and t[p, rot // 2 + i] == np.float32(math.sin(a))


def test_produce_layouts():
    """produce() returns Q in attn_flash's [B*Hq][S][D] order and K/V in token order, with v
    heads untouched and rot=0 an identity on q/k."""
    B, S, Hq, Hkv, D = 2, 3, 4, 2, 64
    rng = np.random.default_rng(0)
    qkv = oracle.f32_to_bf16(rng.normal(size=(B * S, (Hq + 2 * Hkv) * D)).astype(np.float32))
    pos = np.arange(B * S, dtype=np.int32) % S
    Q, K, V = orq.produce(qkv, pos, None, None, None, 1e-6, B, S, Hq, Hkv, D, 0, orq.NEOX)
    x = qkv.reshape(B, S, Hq + 2 * Hkv, D)
    assert np.array_equal(Q, x[:, :, :Hq].transpose(0, 2, 1, 3).reshape(B * Hq, S, D))
    assert np.array_equal(K, x[:, :, Hq:Hq + Hkv]) and np.array_equal(V, x[:, :, Hq + Hkv:])


def test_one_ulp_check():
    ref = np.array([1.0, 1.0, -3.0, 1e-3], np.float64)
    one_up = oracle.f32_to_bf16(np.array([1.0078125, 1.015625, -3.015625, 1e-3], np.float32))
    assert orq.within_one_ulp(one_up, ref).tolist() == [True, False, True, True]
