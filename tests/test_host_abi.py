"""CPU: the C-ABI library's host side -- it loads, exports every symbol the header declares,
keeps the reference's bk contract (abort at both doors, flash.c:641-647), sizes scratch
independently of Sq/Sk (flash.c:679-682), picks bk with the reference's model
(README.md:359-436), and validates arguments before touching the GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest

import oracle
import transfer_station_b200 as ts

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / "include").glob("*.h"))


def _header_text() -> str:
    return re.sub(r"/\*.*?\*/", "", "\n".join(h.read_text() for h in HEADERS), flags=re.S)


def declared_functions() -> set[str]:
    return set(re.findall(r"\b(attn_\w+)\s*\(", _header_text()))


def test_library_exports_every_declared_symbol(built_lib):
    names = declared_functions()
    assert {"attn_flash", "attn_flash_scratch_bytes", "attn_flash_pick_bk"} <= names
    for n in names:
        assert hasattr(built_lib, n), n
    assert names == set(ts.EXPORTS), "the Python mirror binds exactly the declared symbols"


def declared_arity() -> dict[str, int]:
    """Parameter count of every function prototype in the header."""
    out = {}
    for name, params in re.findall(r"\b(attn_\w+)\s*\(([^)]*)\)\s*;", _header_text()):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_python_bindings_match_header_arity():
    """Every ctypes signature in the Python mirror takes exactly the header's parameters."""
    arity = declared_arity()
    assert set(arity) == set(ts.EXPORTS)
    for name, (_, args) in ts.EXPORTS.items():
        assert len(args) == arity[name], (name, len(args), arity[name])


def test_library_has_sm100a_code(built_lib):
    """The .so carries sm_100a device code (cuobjdump --list-elf only names the embedded images)."""
    res = subprocess.run(["cuobjdump", "--list-elf", str(ts.LIB_PATH)], capture_output=True, text=True)
    assert res.returncode == 0 and "sm_100a" in res.stdout


def _abort_run(code: str) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=REPO)


@pytest.mark.parametrize("bk", [0, -16, 8, 100, 8192, 48])
def test_bad_bk_aborts_scratch_bytes(built_lib, bk):
    r = _abort_run(f"import transfer_station_b200 as t; t.attn_flash_scratch_bytes(128, {bk})")
    assert r.returncode < 0  # SIGABRT
    assert f"attn_flash_scratch_bytes: bk={bk} is invalid" in r.stderr and "POWER OF TWO in [16, 4096]" in r.stderr


def test_bad_bk_aborts_attn_flash(built_lib):
    """The second door: the attention entry itself re-checks bk before anything else."""
    r = _abort_run("import transfer_station_b200 as t; t.load_library().attn_flash_stream("
                   "None, None, None, None, 4, 4, 8, 8, 64, 0, 100, None, 0, None)")
    assert r.returncode < 0 and "attn_flash: bk=100 is invalid" in r.stderr


@pytest.mark.parametrize("bk", [16, 32, 64, 128, 256, 512, 1024, 2048, 4096])
def test_scratch_bytes_contract(built_lib, bk):
    s128 = ts.attn_flash_scratch_bytes(128, bk)
    assert s128 % ts.ATTN_SCRATCH_ALIGN == 0
    assert s128 >= 256 + ts.ATTN_PARTIAL_ROWS * (128 + 2) * 4
    assert ts.attn_flash_scratch_bytes(64, bk) < s128 < ts.attn_flash_scratch_bytes(256, bk)


def test_pick_bk_is_reference_model_capped_at_gpu_tile(built_lib):
    MiB = 1 << 20
    for D in (1, 8, 40, 64, 128, 256, 512, 2**31 - 1):
        for l2 in (0, 1, 4096, MiB, 8 * MiB, 126 * MiB, 2**63):
            want = min(oracle.pick_bk_model(D, l2, 128), ts.ATTN_GPU_KEY_TILE)
            got = ts.attn_flash_pick_bk(D, l2)
            assert got == want, (D, l2)
            assert got & (got - 1) == 0 and ts.ATTN_BK_MIN <= got <= ts.ATTN_GPU_KEY_TILE
    assert ts.attn_flash_pick_bk(-5, MiB) == ts.attn_flash_pick_bk(1, MiB)  # D < 1 clamped


def _lib_call(**kw):
    a = dict(Q=1 << 20, K=1 << 20, V=1 << 20, O=1 << 20, Hq=8, Hkv=2, Sq=16, Sk=16, D=64, causal=0, bk=128,
             scratch=1 << 20, vp=0)
    a.update(kw)
    return ts.load_library().attn_flash_stream(a["Q"], a["K"], a["V"], a["O"], a["Hq"], a["Hkv"], a["Sq"], a["Sk"],
                                               a["D"], a["causal"], a["bk"], a["scratch"], a["vp"], None)


@pytest.mark.parametrize("bad", [dict(Q=0), dict(O=0), dict(scratch=0), dict(Hq=6, Hkv=4), dict(Hkv=0),
                                 dict(Sq=0), dict(Sk=0), dict(D=0), dict(D=257)])
def test_argument_validation_before_any_gpu_work(built_lib, bad):
    assert _lib_call(**bad) == ts.ATTN_ERR_ARGS


@pytest.mark.parametrize("out_dtype", [-1, 2, 7])
def test_bad_output_type_is_rejected(built_lib, out_dtype):
    L = ts.load_library()
    rc = L.attn_flash_stream_out(1 << 20, 1 << 20, 1 << 20, 1 << 20, out_dtype, 8, 2, 16, 16, 64, 0, 128, 1 << 20, 0,
                                 None)
    assert rc == ts.ATTN_ERR_ARGS


@pytest.mark.parametrize("bad", [dict(ps=24), dict(ps=0), dict(ps=200), dict(D=72 + 64), dict(D=36), dict(B=0),
                                 dict(Hq=6, Hkv=4), dict(npages=0), dict(maxp=0)])
def test_paged_argument_validation(built_lib, bad):
    a = dict(ps=16, D=128, B=2, Hq=8, Hkv=2, npages=4, maxp=2)
    a.update(bad)
    L = ts.load_library()
    rc = L.attn_flash_paged_stream(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, a["B"], a["Hq"], a["Hkv"], 1,
                                   a["D"], 0, a["ps"], a["npages"], a["maxp"], 1 << 20, None)
    assert rc == ts.ATTN_ERR_ARGS


def test_misaligned_scratch(built_lib):
    assert _lib_call(scratch=(1 << 20) + 4) == ts.ATTN_ERR_ALIGN


def test_no_b200_is_reported_not_faked(built_lib):
    """Without a compute-capability-10 device the call returns a status -- there is no CPU
    fallback path."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _lib_call() == ts.ATTN_ERR_NOT_SM100


def test_strerror(built_lib):
    for code in (ts.ATTN_OK, ts.ATTN_ERR_ARGS, ts.ATTN_ERR_ALIGN, ts.ATTN_ERR_CUDA, ts.ATTN_ERR_DEVICE,
                 ts.ATTN_ERR_NOT_SM100):
        assert ts.strerror(code) and ts.strerror(code) != "unknown status"
    assert ts.strerror(12345) == "unknown status"


def test_missing_library_raises_no_fallback(tmp_path):
    with pytest.raises(FileNotFoundError):
        ts.load_library(tmp_path / "nope.so")


def test_kernel_launch_counter_starts_at_zero(built_lib):
    assert isinstance(ts.attn_flash_kernel_launches(), int)


def _rope_call(paged=False, **kw):
    a = dict(qkv=1 << 20, pos=1 << 20, cs=1 << 20, max_pos=64, qw=None, kw=None, eps=1e-6, B=2, S=4, Hq=8, Hkv=2,
             D=128, rot=128, style=ts.ATTN_ROPE_NEOX, Q=1 << 20, K=1 << 20, V=1 << 20, cache_len=64, bt=1 << 20,
             ps=16, npages=4, maxp=4, scratch=1 << 20)
    a.update(kw)
    L = ts.load_library()
    head = (a["qkv"], a["pos"], a["cs"], a["max_pos"], a["qw"], a["kw"], a["eps"], a["B"], a["S"], a["Hq"],
            a["Hkv"], a["D"], a["rot"], a["style"], a["Q"], a["K"], a["V"])
    if paged:
        return L.attn_qkv_rope_paged_stream(*head, a["bt"], a["ps"], a["npages"], a["maxp"], a["scratch"], None)
    return L.attn_qkv_rope_stream(*head, a["cache_len"], a["scratch"], None)


@pytest.mark.parametrize("bad", [dict(D=96), dict(D=32), dict(rot=8), dict(rot=256), dict(rot=-16), dict(style=2),
                                 dict(qkv=None), dict(Q=None), dict(pos=None), dict(scratch=None), dict(cs=None),
                                 dict(max_pos=0), dict(cache_len=0), dict(Hq=0), dict(Hkv=0), dict(B=-1),
                                 dict(qw=1 << 20, eps=-1.0), dict(kw=1 << 20, eps=float("nan"))])
def test_rope_argument_validation(built_lib, bad):
    assert _rope_call(**bad) == ts.ATTN_ERR_ARGS


@pytest.mark.parametrize("bad", [dict(bt=None), dict(ps=0), dict(npages=0), dict(maxp=0), dict(D=80)])
def test_rope_paged_argument_validation(built_lib, bad):
    assert _rope_call(paged=True, **bad) == ts.ATTN_ERR_ARGS


@pytest.mark.parametrize("bad", [dict(qkv=(1 << 20) + 8), dict(K=(1 << 20) + 2), dict(cs=(1 << 20) + 4),
                                 dict(qw=(1 << 20) + 8), dict(scratch=(1 << 20) + 16)])
def test_rope_alignment(built_lib, bad):
    assert _rope_call(**bad) == ts.ATTN_ERR_ALIGN


def test_rope_needs_no_table_without_rotation(built_lib):
    """rot = 0 (norm / layout only) takes no table; the call then fails only for want of a B200."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _rope_call(rot=0, cs=None, max_pos=0) == ts.ATTN_ERR_NOT_SM100
    L = ts.load_library()
    assert L.attn_rope_table_stream(1 << 20, 0, 128, 1e4, None) == ts.ATTN_ERR_ARGS
    assert L.attn_rope_table_stream(1 << 20, 8, 24, 1e4, None) == ts.ATTN_ERR_ARGS
    assert L.attn_rope_table_stream(1 << 20, 8, 64, 1.0, None) == ts.ATTN_ERR_ARGS
    assert L.attn_rope_table_stream(1 << 20, 8, 64, 1e4, None) == ts.ATTN_ERR_NOT_SM100
