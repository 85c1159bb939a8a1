"""oracle -- TEST INFRASTRUCTURE ONLY: the CPU checker for the B200 attention path.

ctypes bindings for
  * ``liboracle.so``: the C restatement of the reference algorithm (attn_oracle.c), and
  * ``_ref/libflashref*.so``: the reference's own flash.c compiled natively through the SVE
    shim (built only where the reference sources exist; the .so travels with the repo).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this package,
and only as the checker / the timed CPU reference -- never as the product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libflashref.so"
REF_LIB_BQ64 = HERE / "_ref" / "libflashref_bq64.so"
# The reference checkout: TS_REFERENCE_DIR, else a `reference` directory beside the repository.
REF_DIR = Path(os.environ.get("TS_REFERENCE_DIR") or (HERE.parent.parent / "reference")).resolve()

_lib = None
_ref = {}

_P = ctypes.c_void_p
_I = ctypes.c_int


def build(ref: bool = True) -> None:
    """make -C oracle (the restatement always; the reference build when its sources exist)."""
    targets = ["oracle"]
    if ref and (REF_DIR / "flash.c").exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_DIR={REF_DIR}", *targets], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build(ref=False)
        L = ctypes.CDLL(str(LIB))
        L.orc_fill_lcg.argtypes = [_P, ctypes.c_size_t, _P, ctypes.c_size_t, _P, ctypes.c_size_t, ctypes.c_uint32]
        L.orc_fill_normal.argtypes = [_P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_float,
                                      ctypes.c_float]
        L.orc_fill_uniform.argtypes = [_P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_float,
                                       ctypes.c_float]
        L.orc_attn_ref.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I]
        L.orc_attn_blocked.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I]
        L.orc_attn_blocked_rows.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I]
        L.orc_pack_v_full.argtypes = [_P, _P, _I, _I, _I]
        L.orc_ref_rowset.argtypes = [_I, _I, _P]
        L.orc_ref_rowset.restype = _I
        L.orc_cmp_rows.argtypes = [_P, _P, _I, _I, _I, _P, _I, _P]
        L.orc_cmp_rows.restype = ctypes.c_long
        L.orc_attn_pairs.argtypes = [_I, _I, _I]
        L.orc_attn_pairs.restype = ctypes.c_double
        L.orc_ref_scratch_bytes.argtypes = [_I, _I, _I]
        L.orc_ref_scratch_bytes.restype = ctypes.c_size_t
        L.orc_pick_bk_model.argtypes = [_I, ctypes.c_size_t, _I]
        L.orc_pick_bk_model.restype = _I
        L.orc_combine.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.orc_f32_to_bf16_array.argtypes = [_P, _P, ctypes.c_size_t]
        L.orc_bf16_to_f32_array.argtypes = [_P, _P, ctypes.c_size_t]
        _lib = L
    return _lib


def ref_available(bq: int = 128) -> bool:
    return (REF_LIB if bq == 128 else REF_LIB_BQ64).exists()


def ref_lib(bq: int = 128) -> ctypes.CDLL:
    """The reference's own flash.c (BQ=128 as shipped, or the -DBQ=64 build)."""
    if bq not in _ref:
        path = REF_LIB if bq == 128 else REF_LIB_BQ64
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (needs the reference sources)")
        L = ctypes.CDLL(str(path))
        L.ref_attn_flash.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I]
        L.ref_attn_ref.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I]
        L.ref_scratch_bytes.argtypes = [_I, _I]
        L.ref_scratch_bytes.restype = ctypes.c_size_t
        L.ref_pack_v_full.argtypes = [_P, _P, _I, _I, _I]
        L.ref_bq.restype = _I
        _ref[bq] = L
    return _ref[bq]


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ----------------------------------------------------------------- data
def lcg_inputs(Hq, Hkv, Sq, Sk, D, seed=0x12345678):
    """flash.c:1030,1055-1060: the reference harness's Q, K, V (one LCG stream)."""
    Q = np.empty(Hq * Sq * D, np.uint16)
    K = np.empty(Hkv * Sk * D, np.uint16)
    V = np.empty(Hkv * Sk * D, np.uint16)
    lib().orc_fill_lcg(_p(Q), Q.size, _p(K), K.size, _p(V), V.size, seed)
    return Q, K, V


def normal_bf16(n: int, state: ctypes.c_uint64, mean=0.0, sigma=1.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_fill_normal(_p(out), n, ctypes.byref(state), mean, sigma)
    return out


def uniform_bf16(n: int, state: ctypes.c_uint64, lo=-2.0, hi=2.0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_fill_uniform(_p(out), n, ctypes.byref(state), lo, hi)
    return out


def seeded_inputs(Hq, Hkv, Sq, Sk, D, seed, dist="normal", a=0.0, b=1.0):
    """Seeded bf16 Q, K, V in that order: dist 'normal' (mean a, sigma b) or 'uniform' [a, b)."""
    st = ctypes.c_uint64(seed)
    gen = normal_bf16 if dist == "normal" else uniform_bf16
    Q = gen(Hq * Sq * D, st, a, b)
    K = gen(Hkv * Sk * D, st, a, b)
    V = gen(Hkv * Sk * D, st, a, b)
    return Q, K, V


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    return (x.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.size, np.uint16)
    lib().orc_f32_to_bf16_array(_p(x), _p(out), x.size)
    return out.reshape(x.shape)


# ----------------------------------------------------------------- algorithms
def rowset(Sq: int, ref_cap: int) -> np.ndarray:
    rows = np.empty(max(Sq, 1), np.int32)
    n = lib().orc_ref_rowset(Sq, ref_cap, _p(rows))
    return rows[:n].copy()


def attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows=None) -> np.ndarray:
    """flash.c:262-314 restated; only `rows` are written (others stay 0)."""
    if rows is None:
        rows = np.arange(Sq, dtype=np.int32)
    rows = np.ascontiguousarray(rows, np.int32)
    O = np.zeros(Hq * Sq * D, np.float32)
    lib().orc_attn_ref(_p(Q), _p(K), _p(V), _p(O), Hq, Hkv, Sq, Sk, D, int(causal), _p(rows), rows.size)
    return O


def attn_blocked(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, bk=128, bq=128, v_prepacked=0, nthreads=0) -> np.ndarray:
    """flash.c:727-864 restated (blocked online softmax, bf16 P)."""
    O = np.zeros(Hq * Sq * D, np.float32)
    lib().orc_attn_blocked(_p(Q), _p(K), _p(V), _p(O), Hq, Hkv, Sq, Sk, D, int(causal), bk, bq, int(v_prepacked),
                           nthreads)
    return O


def attn_blocked_rows(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, row_lo, row_hi, bk=128, bq=128, nthreads=0):
    lib().orc_attn_blocked_rows(_p(Q), _p(K), _p(V), _p(O), Hq, Hkv, Sq, Sk, D, int(causal), bk, bq, 0, row_lo,
                                row_hi, nthreads)


def pack_v_full(V, Hkv, Sk, D) -> np.ndarray:
    Vp = np.empty_like(V)
    lib().orc_pack_v_full(_p(V), _p(Vp), Hkv, Sk, D)
    return Vp


def cmp_rows(Oref, Odut, Hq, Sq, D, rows):
    """Returns dict(mad, maxref, rel_l2, nbad, err_scale) over the checked rows."""
    rows = np.ascontiguousarray(rows, np.int32)
    res = np.zeros(3, np.float64)
    nbad = lib().orc_cmp_rows(_p(np.ascontiguousarray(Oref, np.float32)),
                              _p(np.ascontiguousarray(Odut, np.float32)), Hq, Sq, D, _p(rows), rows.size, _p(res))
    mad, maxref, rel = float(res[0]), float(res[1]), float(res[2])
    return dict(mad=mad, maxref=maxref, rel_l2=rel, nbad=int(nbad), err_scale=(mad / maxref) if maxref > 0 else 0.0)


# Tolerances: the reference's pooled bound (flash.c:935-937, 977) and the task's two bounds.
TOL_SCALE = 8e-3
TOL_ABS = 2e-2
TOL_REL_L2 = 1e-2


def passes(c: dict) -> bool:
    ok_scale = c["mad"] <= TOL_SCALE * c["maxref"]
    return c["nbad"] == 0 and ok_scale and c["mad"] <= TOL_ABS and c["rel_l2"] <= TOL_REL_L2


def attn_pairs(Sq, Sk, causal) -> float:
    return float(lib().orc_attn_pairs(Sq, Sk, int(causal)))


def ref_scratch_bytes(D, bk, bq=128) -> int:
    return int(lib().orc_ref_scratch_bytes(D, bk, bq))


def pick_bk_model(D, l2, bq) -> int:
    return int(lib().orc_pick_bk_model(D, l2, bq))


def combine(m, l, acc, nparts, rows, D) -> np.ndarray:
    O = np.zeros(rows * D, np.float32)
    lib().orc_combine(_p(np.ascontiguousarray(m, np.float32)), _p(np.ascontiguousarray(l, np.float32)),
                      _p(np.ascontiguousarray(acc, np.float32)), nparts, rows, D, _p(O))
    return O


# ----------------------------------------------------------------- the reference itself
def ref_attn_flash(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, bk=128, bq=128, v_prepacked=0) -> np.ndarray:
    L = ref_lib(bq)
    O = np.zeros(Hq * Sq * D, np.float32)
    scratch = np.zeros(L.ref_scratch_bytes(D, bk) + 64, np.uint8)
    base = scratch.ctypes.data
    aligned = (base + 63) & ~63
    L.ref_attn_flash(_p(Q), _p(K), _p(V), _p(O), Hq, Hkv, Sq, Sk, D, int(causal), bk, aligned, int(v_prepacked))
    return O


def ref_attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows=None) -> np.ndarray:
    L = ref_lib(128)
    if rows is None:
        rows = np.arange(Sq, dtype=np.int32)
    rows = np.ascontiguousarray(rows, np.int32)
    O = np.zeros(Hq * Sq * D, np.float32)
    L.ref_attn_ref(_p(Q), _p(K), _p(V), _p(O), Hq, Hkv, Sq, Sk, D, int(causal), _p(rows), rows.size)
    return O
