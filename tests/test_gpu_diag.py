"""GPU: what the attention entry points alone cannot show, through the diagnostic C ABI
(include/attn_flash_diag.h).

* Tensor-memory history. Every read of TMEM in the attention kernel follows a write made earlier
  in the same call: the score tile S_t of key block j is written whole by that block's Q K^T MMA
  (accumulate off on its first K step) before the softmax's s_full wait lets it be read; P is
  stored into S_t's first 64 columns by every softmax path (including the all-masked one, which
  stores zeros) before the p_full arrive that lets the P V MMA read it; O_t is written whole by
  the item's first P V MMA (accumulate off on its first key step) before the softmax's rescale
  (only at j > 0, after s_full(j) proves P V(j-1) finished) or the epilogue (after o_full) reads
  it. So no result may depend on what an earlier kernel left there: each plan runs after every
  SM's TMEM was filled with NaN, with -inf and with zeros, and the three results must be
  bit-identical (and within tolerance of the fp32 reference).
* The exponentials: the FMA-pipe polynomial's relative error over [-125, 0], its clamp, exact
  powers of two; the MUFU ex2.approx against exp2.
* A bounded wait that runs out: the kernel build that never loads Q must end with the timeout
  reported in the status word and the context still usable (no hang, no trap).
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import run_gpu, scratch_for, to_dev

pytestmark = pytest.mark.gpu

NAN_BITS, NEG_INF_BITS = 0x7FC00000, 0xFF800000

# Work plans of the tensor-core kernel: plain prefill (two tiles per CTA, persistent walk with a
# split last wave), causal (longest-first snake, masked and all-masked blocks), decode (one tile,
# split keys + combine), head_dim 64, a caller's V^T, MQA decode.
PLANS = [
    ("prefill_s4096", 32, 8, 4096, 4096, 128, 0, 0),
    ("prefill_s2048_causal", 32, 8, 2048, 2048, 128, 1, 0),
    ("decode_b8", 256, 64, 1, 8192, 128, 0, 0),
    ("d64_causal_tails", 8, 2, 300, 1000, 64, 1, 0),
    ("vt_prefill", 8, 2, 200, 1000, 128, 0, 1),
    ("mqa_decode_b32", 512, 32, 1, 4096, 128, 0, 0),
]


@pytest.mark.parametrize("plan", PLANS, ids=[p[0] for p in PLANS])
def test_result_does_not_depend_on_tmem_history(cuda_dev, plan):
    name, Hq, Hkv, Sq, Sk, D, causal, vt = plan
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=11)
    Vin = oracle.pack_v_full(V, Hkv, Sk, D) if vt else V
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(Vin, cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    outs = []
    for bits in (NAN_BITS, NEG_INF_BITS, 0):
        assert ts.attn_diag_fill_tmem(bits) == ts.ATTN_OK
        o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
        ts.attn_flash_checked(q, k, v, o, Hq, Hkv, Sq, Sk, D, causal, 128, scratch, vt)
        torch.cuda.synchronize()
        outs.append(o)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2]), name
    rows = oracle.rowset(Sq, 8) if Sq > 1 else np.arange(1, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
    c = oracle.cmp_rows(ref, outs[0].cpu().numpy(), Hq, Sq, D, rows)
    assert oracle.passes(c), (name, c)


def _exp2_dev(x: np.ndarray, method: int, dev) -> np.ndarray:
    xd = torch.from_numpy(x.astype(np.float32)).to(dev)
    yd = torch.full_like(xd, float("nan"))
    assert ts.attn_diag_exp2(xd, yd, xd.numel(), method) == ts.ATTN_OK
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def _exp2_inputs() -> np.ndarray:
    rng = np.random.default_rng(5)
    ints = np.arange(-125, 1, dtype=np.float32)
    return np.concatenate([
        rng.uniform(-125.0, 0.0, 4_000_000).astype(np.float32),
        rng.uniform(-20.0, 0.0, 1_000_000).astype(np.float32),   # the softmax's usual range
        ints, ints + 0.5, ints - 0.5, np.nextafter(ints, 0), np.nextafter(ints, -200),
        np.linspace(-125.0, -124.0, 100_001, dtype=np.float32),  # the exponent-add's lowest range
        np.float32([0.0, -0.0, -1e-30, -124.5, -124.50001, -125.0]),
    ]).astype(np.float32)


def test_exp2_polynomial_accuracy(cuda_dev):
    """The FMA-pipe 2^x (round-to-nearest range reduction, degree-3 polynomial, exponent added
    to the bits): relative error <= 1.02e-4 over [-125, 0] (the fitted polynomial's own bound;
    bf16 rounding of P, next, is 2^-9 relative), exactly 2^n at every integer n, and no denormal or
    zero result anywhere in that range."""
    x = _exp2_inputs()
    x = x[(x >= -125.0) & (x <= 0.0)]
    y = _exp2_dev(x, ts.ATTN_DIAG_EXP2_POLY, cuda_dev).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(y / want - 1.0)
    assert rel.max() <= 1.02e-4, (rel.max(), x[rel.argmax()])
    ints = np.arange(-125, 1, dtype=np.float32)
    assert np.array_equal(_exp2_dev(ints, ts.ATTN_DIAG_EXP2_POLY, cuda_dev), np.exp2(ints))
    assert y.min() >= 2.0 ** -125 * (1 - 1.02e-4)


def test_exp2_polynomial_clamp(cuda_dev):
    """Below -125 the input is clamped, so the result is exactly 2^-125 (a normal float), never
    a denormal or zero; the softmax only sends it finite arguments of full blocks."""
    x = np.float32([-125.0, -125.25, -126.0, -130.5, -149.0, -1e4, -3.0e38])
    y = _exp2_dev(x, ts.ATTN_DIAG_EXP2_POLY, cuda_dev)
    assert np.all(y == np.float32(2.0 ** -125)), y


def test_exp2_mufu_accuracy(cuda_dev):
    """The hardware ex2.approx.ftz.f32 against exp2 over [-125, 0]: relative error below 2^-21,
    and 2^-inf = +0 (the masked path relies on it)."""
    x = _exp2_inputs()
    x = x[(x >= -125.0) & (x <= 0.0)]
    y = _exp2_dev(x, ts.ATTN_DIAG_EXP2_MUFU, cuda_dev).astype(np.float64)
    rel = np.abs(y / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 2.0 ** -21, (rel.max(), x[rel.argmax()])
    assert _exp2_dev(np.float32([-np.inf, -np.inf]), ts.ATTN_DIAG_EXP2_MUFU, cuda_dev).tolist() == [0.0, 0.0]


def test_bounded_wait_runs_out_and_is_reported(cuda_dev):
    """The kernel build whose producer never loads Q: the MMA issuer's wait for Q runs out after
    its ~2 s limit, every role unwinds (in-flight K/V copies drained, TMEM freed), the call ends
    with a timeout in the status word, O is untouched, and the next ordinary call on the same
    context is correct. The producer's wait for a free K/V slot starts at the same moment and
    runs out just as long after, so whichever of the two expires first is the one reported (the
    other role sees the abort flag and returns without a report)."""
    Hq, Hkv, Sq, Sk, D = 8, 4, 32, 1024, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=12)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    t0 = time.perf_counter()
    assert ts.attn_diag_wait_timeout(q, k, v, o, Hq, Hkv, Sq, Sk, scratch) == ts.ATTN_OK
    rc, code = ts.attn_flash_status(scratch)
    dt = time.perf_counter() - t0
    assert rc == ts.ATTN_ERR_DEVICE and code & (ts.ATTN_DEV_TIMEOUT_Q | ts.ATTN_DEV_TIMEOUT_KV), (rc, code)
    assert not code & (ts.ATTN_DEV_BAD_PAGE | ts.ATTN_DEV_BAD_POS | ts.ATTN_DEV_TIMEOUT_PEER), code
    assert 1.0 < dt < 30.0, dt  # the wait's ~2 s limit, not a hang
    assert torch.isnan(o).all()
    assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)  # read-and-clear
    rows = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, rows)
    out = run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, dev=cuda_dev, scratch=scratch)
    c = oracle.cmp_rows(ref, out, Hq, Sq, D, rows)
    assert oracle.passes(c), c
