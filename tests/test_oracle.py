"""CPU: the oracle restatement pinned against the reference's own outputs (tests/golden/,
generated from flash.c itself by tests/golden/make_golden.py), plus the reference's known
answers and the tolerance machinery (flash.c:900-980, README.md:359-436, EXEC_LOG F9-F17)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())


def _load(name):
    m = MANIFEST[name]
    z = np.load(GOLDEN / f"{name}.npz")
    return m, z


def _full(z, m, key):
    """Scatter the stored rows of an output back into a zero [Hq][Sq][D] array."""
    O = np.zeros((m["Hq"], m["Sq"], m["D"]), np.float32)
    O[:, z["rows"], :] = z[key]
    return O.reshape(-1)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_inputs_reproduce(name):
    """The oracle's generators reproduce the fixture inputs bit for bit (the LCG of
    flash.c:867-871 in Q, K, V order; the seeded N(0,1) of BASELINE config 1)."""
    m, z = _load(name)
    if m["data"] == "lcg":
        Q, K, V = oracle.lcg_inputs(m["Hq"], m["Hkv"], m["Sq"], m["Sk"], m["D"])
    else:
        Q, K, V = oracle.seeded_inputs(m["Hq"], m["Hkv"], m["Sq"], m["Sk"], m["D"], seed=0)
    assert np.array_equal(Q, z["Q"]) and np.array_equal(K, z["K"]) and np.array_equal(V, z["V"])


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_attn_ref_bit_exact(name):
    """orc_attn_ref == the reference's attn_ref (flash.c:262-314), bit for bit."""
    m, z = _load(name)
    got = oracle.attn_ref(z["Q"], z["K"], z["V"], m["Hq"], m["Hkv"], m["Sq"], m["Sk"], m["D"], m["causal"],
                          z["rows"])
    want = _full(z, m, "o_attn_ref")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_blocked_matches_reference_kernel(name):
    """orc_attn_blocked (flash.c:727-864 restated) against the reference's attn_flash: the same
    blocking, the same bf16 P; only exp (expf vs fast_exp) and the summation order differ."""
    m, z = _load(name)
    Vin = z["Vin"] if m["v_prepacked"] else z["V"]
    got = oracle.attn_blocked(z["Q"], z["K"], Vin, m["Hq"], m["Hkv"], m["Sq"], m["Sk"], m["D"], m["causal"],
                              bk=m["bk"], bq=m["bq"], v_prepacked=m["v_prepacked"])
    want = _full(z, m, "o_attn_flash")
    c = oracle.cmp_rows(want, got, m["Hq"], m["Sq"], m["D"], z["rows"])
    assert oracle.passes(c) and c["err_scale"] < 1e-3, c
    # and the restatement passes the reference's own check against the fp32 oracle
    ref = _full(z, m, "o_attn_ref")
    c2 = oracle.cmp_rows(ref, got, m["Hq"], m["Sq"], m["D"], z["rows"])
    assert oracle.passes(c2), c2
    assert abs(c2["err_scale"] - m["ref_err_scale"]) < 1.5e-3


def test_shipped_suite_err_scale_matches_log():
    """flash_long.log:12-20 prints the shipped suite's err/scale; the reference kernel's
    fixtures reproduce those printed values (2 significant digits)."""
    logged = {"mha_prefill": 1.4e-3, "mha_prefill_causal": 9.4e-4, "gqa_prefill": 1.5e-3,
              "gqa_prefill_causal": 1.3e-3, "mqa_prefill": 1.6e-3, "odd_multiblock": 1.3e-3,
              "gqa_big_head_dim": 1.5e-3, "mha_decode": 1.1e-3, "gqa_decode": 1.7e-3}
    for k, v in logged.items():
        assert float(f"{MANIFEST[k]['ref_err_scale']:.1e}") == pytest.approx(v), k


def test_sk1_gives_v0_exactly():
    """EXEC_LOG F17: Sk=1 -> the one-element softmax is exactly 1, O = V[0] bit for bit."""
    m, z = _load("sk1")
    O = oracle.attn_blocked(z["Q"], z["K"], z["V"], m["Hq"], m["Hkv"], m["Sq"], 1, m["D"], 0).reshape(
        m["Hq"], m["Sq"], m["D"])
    Vf = oracle.bf16_to_f32(z["V"]).reshape(m["Hkv"], m["D"])
    g = m["Hq"] // m["Hkv"]
    for h in range(m["Hq"]):
        assert np.array_equal(O[h], np.broadcast_to(Vf[h // g], O[h].shape))


def test_fully_masked_rows_are_zero():
    """EXEC_LOG F15: causal rows with Sk - Sq + i < 0 attend no key -> exact zero rows in both
    the fp32 reference and the kernel restatement."""
    m, z = _load("masked_rows")
    nm = m["Sq"] - m["Sk"]
    ref = _full(z, m, "o_attn_ref").reshape(m["Hq"], m["Sq"], m["D"])
    blk = oracle.attn_blocked(z["Q"], z["K"], z["V"], m["Hq"], m["Hkv"], m["Sq"], m["Sk"], m["D"], 1).reshape(
        m["Hq"], m["Sq"], m["D"])
    assert np.all(ref[:, :nm] == 0) and np.all(blk[:, :nm] == 0)
    assert np.any(ref[:, nm:] != 0)


def test_dropped_key_block_fails():
    """README.md:601-621: a kernel that drops one key block must FAIL the pooled bound (the
    mistake is planted in the oracle's input, on the CPU)."""
    Hq, Hkv, Sq, Sk, D = 4, 2, 32, 512, 64
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    Kb = K.reshape(Hkv, Sk, D).copy()
    Kb[:, 128:256, :] = 0xFF80  # -inf keys: that block gets zero weight
    bad = oracle.attn_blocked(Q, Kb.reshape(-1), V, Hq, Hkv, Sq, Sk, D, 0, bk=128)
    assert not oracle.passes(oracle.cmp_rows(ref, bad, Hq, Sq, D, rows))


def test_nan_is_counted_out_of_band():
    """flash.c:946-957 / EXEC_LOG F16: a NaN in the kernel output fails the case even though
    mad/maxref (over the finite rest) look fine."""
    m, z = _load("gqa_prefill")
    ref = _full(z, m, "o_attn_ref")
    dut = ref.copy()
    dut[5] = np.nan
    c = oracle.cmp_rows(ref, dut, m["Hq"], m["Sq"], m["D"], z["rows"])
    assert c["nbad"] == 1 and not oracle.passes(c) and c["mad"] == 0.0


def test_uniform_scale_error_detected():
    """EXEC_LOG:252-262: a uniform x1.01 output error fails the pooled bound."""
    m, z = _load("config1_mha_s256_d64")
    ref = _full(z, m, "o_attn_ref")
    c = oracle.cmp_rows(ref, ref * 1.01, m["Hq"], m["Sq"], m["D"], z["rows"])
    assert not oracle.passes(c)


def test_rowset_spread():
    """flash.c:900-913: spread rows always include 0 and Sq-1; cap 1 -> only Sq-1."""
    r = oracle.rowset(4096, 8)
    assert r[0] == 0 and r[-1] == 4095 and len(r) == 8 and np.all(np.diff(r) > 0)
    assert list(oracle.rowset(100, 1)) == [99]
    assert list(oracle.rowset(5, 0)) == [0, 1, 2, 3, 4]


def test_pick_bk_model_readme_table():
    """README.md:420-426 (at the README's BQ=64): the analytical model's documented picks."""
    MiB = 1 << 20
    assert [oracle.pick_bk_model(128, l2, 64) for l2 in (MiB, 2 * MiB, 4 * MiB, 8 * MiB)] == [256, 512, 1024, 2048]
    assert [oracle.pick_bk_model(d, MiB, 64) for d in (64, 128, 256, 512)] == [512, 256, 128, 64]
    assert oracle.pick_bk_model(128, 0, 64) == 16
    assert oracle.pick_bk_model(0, 1 << 62, 64) == 4096
    assert oracle.pick_bk_model(2**31 - 1, 2 * 10**12, 64) == 16  # EXEC_LOG F35's overflow case


def test_reference_scratch_bytes():
    """The reference's scratch size, as its own runs printed it (198656 B at D=128, bk=128 with
    the shipped BQ=128; flash_long.log:11 printed 115968 B from the BQ=64 build)."""
    assert oracle.ref_scratch_bytes(128, 128, 128) == 198656
    assert oracle.ref_scratch_bytes(128, 128, 64) == 115968


def test_attn_pairs():
    """flash.c:874-887: causal Sq=Sk=n has n(n+1)/2 pairs; Sk<Sq drops the masked rows."""
    assert oracle.attn_pairs(1024, 1024, 0) == 1024 * 1024
    assert oracle.attn_pairs(1024, 1024, 1) == 1024 * 1025 / 2
    assert oracle.attn_pairs(130, 70, 1) == sum(max(0, min(70, 70 - 130 + i + 1)) for i in range(130))


def test_combine_of_key_splits_equals_full():
    """The split-KV merge (used by the decode path and the multi-GPU key split): partials over
    disjoint key ranges, merged in base-2 units, equal the one-shot softmax."""
    rng = np.random.default_rng(0)
    rows, Sk, D, parts = 6, 300, 16, 4
    s = rng.normal(size=(rows, Sk)).astype(np.float64)
    v = rng.normal(size=(Sk, D)).astype(np.float64)
    bounds = np.linspace(0, Sk, parts + 1).astype(int)
    m = np.zeros((parts, rows), np.float32)
    l = np.zeros((parts, rows), np.float32)
    acc = np.zeros((parts, rows, D), np.float32)
    for p in range(parts):
        blk = s[:, bounds[p]:bounds[p + 1]] * np.log2(np.e)
        mx = blk.max(axis=1)
        e = np.exp2(blk - mx[:, None])
        m[p], l[p], acc[p] = mx, e.sum(1), e @ v[bounds[p]:bounds[p + 1]]
    m[1, 2] = -np.inf  # a partial that saw no key
    l[1, 2] = 0
    acc[1, 2] = 0
    O = oracle.combine(m, l, acc, parts, rows, D).reshape(rows, D)
    keep = np.ones((rows, Sk), bool)
    keep[2, bounds[1]:bounds[2]] = False
    w = np.where(keep, np.exp(s - s.max(1, keepdims=True)), 0)
    want = (w / w.sum(1, keepdims=True)) @ v
    assert np.allclose(O, want, atol=1e-5)


def _splitmix_seq(state: int, ndraws: int):
    """splitmix64 (Steele, Lea, Flood 2014) as one sequential stream of uniform doubles."""
    M = (1 << 64) - 1
    out = []
    for _ in range(ndraws):
        state = (state + 0x9E3779B97F4A7C15) & M
        z = state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        z ^= z >> 31
        out.append(((z >> 11) + 0.5) / 9007199254740992.0)
    return state, out


@pytest.mark.parametrize("n", [1, 2, 7, 64, 1001])
def test_seeded_generators_match_a_sequential_stream(n):
    """The parallel fill (each element's draw computed from the state arithmetic) equals one
    sequential splitmix64 pass, for even and odd counts, and leaves the state where that pass
    would: Box-Muller pairs for the normal fill, one draw per element for the uniform fill."""
    import ctypes

    st = ctypes.c_uint64(12345)
    got_n = oracle.normal_bf16(n, st, 0.5, 2.0)
    got_u = oracle.uniform_bf16(n, st, -2.0, 2.0)
    s, u = _splitmix_seq(12345, 2 * ((n + 1) // 2))
    want_n = []
    for p in range(0, len(u), 2):
        r = np.sqrt(-2.0 * np.log(u[p]))
        want_n += [0.5 + 2.0 * r * np.cos(2 * np.pi * u[p + 1]), 0.5 + 2.0 * r * np.sin(2 * np.pi * u[p + 1])]
    s, u2 = _splitmix_seq(s, n)
    want_u = [-2.0 + 4.0 * x for x in u2]
    assert np.array_equal(got_n, oracle.f32_to_bf16(np.array(want_n[:n], np.float32)))
    assert np.array_equal(got_u, oracle.f32_to_bf16(np.array(want_u, np.float32)))
    assert st.value == s
