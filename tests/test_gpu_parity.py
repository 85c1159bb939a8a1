"""GPU parity: the C-ABI attention path on a B200 against the CPU oracle.

Every case checks the GPU output against the fp32 reference (attn_ref, flash.c:262-314,
restated bit-exactly in oracle/) with the reference's pooled bound (mad <= 8e-3 * maxref,
nbad == 0, flash.c:935-980) plus the task's bounds (max abs <= 2e-2, rel L2 <= 1e-2), and
where it is cheap also against the blocked-kernel restatement (flash.c:727-864) to the same
bounds. Cases: the reference's shipped suite (flash.c:1287-1299, LCG data), the benchmark
configs at test-sized or full shapes, and the edge cases the reference's log probes.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.gpu_util import run_gpu

pytestmark = pytest.mark.gpu


def check(Oref, Odut, Hq, Sq, D, rows, what=""):
    c = oracle.cmp_rows(Oref, Odut, Hq, Sq, D, rows)
    assert oracle.passes(c), f"{what}: {c}"
    return c


# flash.c:1287-1299 -- the shipped default suite, every row checked (ref_cap = 0).
SHIPPED = [
    ("MHA prefill", 4, 4, 8, 8, 64, 0),
    ("MHA prefil.causal", 4, 4, 8, 8, 64, 1),
    ("GQA prefill", 8, 2, 8, 8, 64, 0),
    ("GQA prefil.causal", 8, 2, 8, 8, 64, 1),
    ("MQA prefill", 8, 1, 8, 8, 64, 0),
    ("odd + multiblock", 6, 3, 130, 70, 40, 1),
    ("GQA big head_dim", 8, 2, 4, 12, 128, 0),
    # the two decode cases of flash_long.log:16-17
    ("MHA decode(Sq=1)", 4, 4, 1, 16, 64, 0),
    ("GQA decode(Sq=1)", 8, 2, 1, 16, 64, 0),
]


@pytest.mark.parametrize("name,Hq,Hkv,Sq,Sk,D,causal", SHIPPED, ids=[s[0] for s in SHIPPED])
def test_shipped_suite(cuda_dev, name, Hq, Hkv, Sq, Sk, D, causal):
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    blk = oracle.attn_blocked(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, bk=128, bq=128)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev)
    check(ref, out, Hq, Sq, D, rows, name + " vs fp32 ref")
    check(blk, out, Hq, Sq, D, rows, name + " vs blocked kernel")


def test_config1_mha_small(cuda_dev):
    """MHA 4/4, Sq=Sk=256, D=64, N(0,1) seed 0, full check."""
    Hq, Hkv, S, D = 4, 4, 256, 64
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, S, S, D, seed=0)
    rows = np.arange(S, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, S, S, D, 0, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, S, S, D, 0, dev=cuda_dev)
    check(ref, out, Hq, S, D, rows, "config1")
    blk = oracle.attn_blocked(Q, K, V, Hq, Hkv, S, S, D, 0, bk=128, bq=64)
    check(blk, out, Hq, S, D, rows, "config1 vs blocked (BQ=64)")


@pytest.mark.parametrize("S,causal", [(1024, 0), (2048, 0), (4096, 0), (1024, 1), (2048, 1)])
def test_config2_gqa_prefill(cuda_dev, S, causal):
    """BASELINE config 2 (Qwen3-8B-shaped GQA 32/8, D=128), spread rows incl. Sq-1. At S=4096
    the 512 CTAs leave a last wave of 68 on 148 SMs, whose units run as key pieces and are
    merged afterwards: the spread rows of heads 27-31 come from that path."""
    Hq, Hkv, D = 32, 8, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, S, S, D, seed=1)
    rows = oracle.rowset(S, 24)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, S, S, D, causal, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, S, S, D, causal, dev=cuda_dev)
    check(ref, out, Hq, S, D, rows, f"config2 S={S} causal={causal}")


def test_config3_gqa_decode(cuda_dev):
    """BASELINE config 3 shape at batch 8 (the bench runs batch 64): Sq=1, 32/8, Sk=8192."""
    B, Hq, Hkv, Sk, D = 8, 32, 8, 8192, 128
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, 1, Sk, D, seed=2)
    rows = np.arange(1, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, rows)
    out = run_gpu(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, dev=cuda_dev)
    check(ref, out, B * Hq, 1, D, rows, "config3 decode")


def test_config4_mqa(cuda_dev):
    """MQA 16/1, U(-2,2) seed 3. Prefill at batch 2 (bench: 8), decode at
    batch 128 / Sk 4096 (full size)."""
    Hq, Hkv, D = 16, 1, 128
    B, S = 2, 2048
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, S, S, D, seed=3, dist="uniform", a=-2.0, b=2.0)
    rows = oracle.rowset(S, 16)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, rows)
    out = run_gpu(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, dev=cuda_dev)
    check(ref, out, B * Hq, S, D, rows, "config4 prefill")
    B, Sk = 128, 4096
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, 1, Sk, D, seed=3, dist="uniform", a=-2.0, b=2.0)
    rows = np.arange(1, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, rows)
    out = run_gpu(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, dev=cuda_dev)
    check(ref, out, B * Hq, 1, D, rows, "config4 decode")


def test_config5_long_decode_single_gpu(cuda_dev):
    """BASELINE config 5 decode at batch 1 (bench: batch 4), Sk=131072, N(0,0.5) seed 4."""
    B, Hq, Hkv, Sk, D = 1, 64, 8, 131072, 128
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, 1, Sk, D, seed=4, a=0.0, b=0.5)
    rows = np.arange(1, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, rows)
    out = run_gpu(Q, K, V, B * Hq, B * Hkv, 1, Sk, D, 0, dev=cuda_dev)
    check(ref, out, B * Hq, 1, D, rows, "config5 decode")


def test_config5_long_prefill_single_gpu(cuda_dev):
    """BASELINE config 5 prefill at batch 1 (bench: batch 4), Sq=Sk=16384, 64/8 heads, N(0,0.5)
    seed 4: 128 key blocks per unit, spread rows checked against the fp32 reference."""
    B, Hq, Hkv, S, D = 1, 64, 8, 16384, 128
    Q, K, V = oracle.seeded_inputs(B * Hq, B * Hkv, S, S, D, seed=4, a=0.0, b=0.5)
    rows = oracle.rowset(S, 6)
    ref = oracle.attn_ref(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, rows)
    out = run_gpu(Q, K, V, B * Hq, B * Hkv, S, S, D, 0, dev=cuda_dev)
    check(ref, out, B * Hq, S, D, rows, "config5 prefill")


# --------------------------------------------------------------------- edge cases
def test_sk1_is_v0_exactly(cuda_dev):
    """Sk=1: the one-element softmax is exactly 1, so O = V[0] bit for bit (EXEC_LOG F17)."""
    Hq, Hkv, Sq, Sk, D = 4, 2, 64, 1, 64
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, dev=cuda_dev).reshape(Hq, Sq, D)
    Vf = oracle.bf16_to_f32(V).reshape(Hkv, D)
    for h in range(Hq):
        assert np.array_equal(out[h], np.broadcast_to(Vf[h // 2], (Sq, D)))


@pytest.mark.parametrize("Sq,Sk", [(200, 33), (129, 1), (64, 1), (300, 64)])
def test_causal_fully_masked_rows_are_zero(cuda_dev, Sq, Sk):
    """Causal with Sk < Sq: rows i < Sq-Sk attend no key and must be exact zeros
    (flash.c:851-860 / attn_ref's zero row), the rest within tolerance."""
    Hq, Hkv, D = 4, 4, 64
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, dev=cuda_dev)
    o3 = out.reshape(Hq, Sq, D)
    assert np.all(o3[:, : Sq - Sk, :] == 0.0)
    check(ref, out, Hq, Sq, D, rows, f"masked {Sq}x{Sk}")


@pytest.mark.parametrize("Sk", [1, 63, 127, 128, 129, 256, 257, 70, 1000])
@pytest.mark.parametrize("causal", [0, 1])
def test_key_tails(cuda_dev, Sk, causal):
    """Key-block tail probe set (EXEC_LOG:1110-1124): Sk around the 128-key tile edges."""
    Hq, Hkv, Sq, D = 8, 2, 150, 128
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev)
    check(ref, out, Hq, Sq, D, rows, f"Sk={Sk} causal={causal}")


@pytest.mark.parametrize("D", [1, 2, 7, 8, 16, 24, 33, 40, 64, 72, 96, 120, 128, 160, 256])
def test_head_dims(cuda_dev, D):
    """Head dims 1..256: D % 8 == 0 and D <= 128 run on the tensor core, others on the
    general CUDA-core path."""
    Hq, Hkv, Sq, Sk = 6, 3, 130, 300
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    for causal in (0, 1):
        ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
        out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, dev=cuda_dev)
        check(ref, out, Hq, Sq, D, rows, f"D={D} causal={causal}")


@pytest.mark.parametrize("Sk", [256, 1000, 4096])
def test_v_prepacked(cuda_dev, Sk):
    """v_prepacked=1: V given as V^T [Hkv][D][Sk] (pack_v_full, flash.c:714-718)."""
    Hq, Hkv, Sq, D = 8, 2, 200, 128
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    Vp = oracle.pack_v_full(V, Hkv, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    for causal in (0, 1):
        ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
        out = run_gpu(Q, K, Vp, Hq, Hkv, Sq, Sk, D, causal, v_prepacked=1, dev=cuda_dev)
        check(ref, out, Hq, Sq, D, rows, f"prepacked Sk={Sk} causal={causal}")


@pytest.mark.parametrize("bk", [16, 32, 64, 128, 256, 1024, 4096])
def test_bk_invariance(cuda_dev, bk):
    """Every legal bk gives a result within tolerance (multi-key-block shape, README:540-558)."""
    Hq, Hkv, Sq, Sk, D = 4, 2, 128, 1024, 128
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, bk=bk, dev=cuda_dev)
    check(ref, out, Hq, Sq, D, rows, f"bk={bk}")


def test_qwen3_long_causal(cuda_dev):
    """flash.c:1312-1314 (--long): Qwen3 16/8 D128 causal 4k, 8 spread rows."""
    Hq, Hkv, S, D = 16, 8, 4096, 128
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, S, S, D)
    rows = oracle.rowset(S, 8)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, S, S, D, 1, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, S, S, D, 1, dev=cuda_dev)
    c = check(ref, out, Hq, S, D, rows, "qwen3 4k")
    assert c["err_scale"] < 2.76e-3  # the reference's measured noise floor (README.md:566-571)


def test_dropped_block_negative_control(cuda_dev):
    """The check has teeth: perturbing one key block of the GPU output's input must FAIL
    (README.md:601-621). The mistake is planted on the CPU side: the oracle sees V with one
    128-key block zeroed, the GPU the real V."""
    Hq, Hkv, Sq, Sk, D = 4, 2, 64, 1024, 128
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, dev=cuda_dev)
    Vbad = V.reshape(Hkv, Sk, D).copy()
    Vbad[:, 256:384, :] = 0
    rows = np.arange(Sq, dtype=np.int32)
    bad = oracle.attn_ref(Q, K, Vbad.reshape(-1), Hq, Hkv, Sq, Sk, D, 0, rows)
    c = oracle.cmp_rows(bad, out, Hq, Sq, D, rows)
    assert not oracle.passes(c)


def test_blocking_call_leaves_phase_totals(cuda_dev):
    """The blocking attn_flash(.., tm) (flash.c:727-729): the reference adds each phase's seconds
    into *tm (flash.c:822-849) and its harness accumulates over calls; with the phases fused in
    one kernel nothing is added, so a caller's running totals come back unchanged. The output is
    the attention itself (tm = NULL and tm given alike)."""
    import ctypes

    import torch

    import transfer_station_b200 as ts
    from tests.gpu_util import scratch_for, to_dev

    class AttnTimes(ctypes.Structure):
        _fields_ = [("packv", ctypes.c_double), ("qxk", ctypes.c_double), ("softmax", ctypes.c_double),
                    ("sxv", ctypes.c_double)]

    Hq, Hkv, Sq, Sk, D = 8, 2, 64, 300, 64
    Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 1, rows)
    tm = AttnTimes(1.5, 2.5, 3.5, 4.5)
    L = ts.load_library()
    for tmp in (ctypes.cast(ctypes.pointer(tm), ctypes.c_void_p), None):
        o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
        L.attn_flash(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), Hq, Hkv, Sq, Sk, D, 1, 128,
                     scratch.data_ptr(), 0, tmp)
        check(ref, o.cpu().numpy(), Hq, Sq, D, rows, "blocking attn_flash")
    assert (tm.packv, tm.qxk, tm.softmax, tm.sxv) == (1.5, 2.5, 3.5, 4.5)


def test_rows_beyond_partial_capacity(cuda_dev):
    """A decode step with more query rows (Hq*Sq = 70016) than the scratch block holds key-piece
    partials for (ATTN_PARTIAL_ROWS = 65536): the plan must run every unit over its whole key
    range (no split), 8752 work items on a persistent grid, and still match the fp32 reference."""
    Hq, Hkv, Sk, D = 70016, 8752, 300, 64
    import transfer_station_b200 as ts

    assert Hq > ts.ATTN_PARTIAL_ROWS
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, 1, Sk, D, seed=6)
    rows = np.arange(1, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, 1, Sk, D, 0, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, 1, Sk, D, 0, dev=cuda_dev)
    check(ref, out, Hq, 1, D, rows, "rows beyond the partial capacity")
