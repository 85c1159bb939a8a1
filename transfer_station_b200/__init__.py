"""transfer_station_b200 -- B200 (sm_100a) bf16 flash-attention forward behind flash.c's C API.

The product is the in-tree shared library ``lib/libattn_flash_b200.so`` (C host layer +
tcgen05/TMA/TMEM CUDA kernels) whose entry points are declared in ``include/attn_flash.h``
(the attention path) and ``include/attn_qkv_rope.h`` (the QKV producer before it).
This module is the thin Python mirror of that C ABI (ctypes), used by the tests and the
benchmark: same names, same argument meaning, same error behaviour. It never computes
anything itself -- if the library is missing it raises, there is no fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import NamedTuple

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libattn_flash_b200.so"

ATTN_BK_MIN = 16
ATTN_BK_MAX = 4096
ATTN_BK_DEFAULT = 128
ATTN_SCRATCH_ALIGN = 256
ATTN_GPU_KEY_TILE = 128
ATTN_D_MAX = 256
ATTN_PARTIAL_ROWS = 65536

ATTN_PEERS_MAX = 8
ATTN_PEER_HANDLE_BYTES = 128

ATTN_OUT_F32 = 0
ATTN_OUT_BF16 = 1

ATTN_ROPE_GPTJ = 0
ATTN_ROPE_NEOX = 1

ATTN_DEV_TIMEOUT_Q = 1
ATTN_DEV_TIMEOUT_KV = 2
ATTN_DEV_TIMEOUT_S = 4
ATTN_DEV_TIMEOUT_P = 8
ATTN_DEV_TIMEOUT_DRAIN = 16
ATTN_DEV_BAD_PAGE = 32
ATTN_DEV_BAD_POS = 64
ATTN_DEV_TIMEOUT_PEER = 128
ATTN_DIAG_EXP2_POLY = 0
ATTN_DIAG_EXP2_MUFU = 1

ATTN_OK = 0
ATTN_ERR_ARGS = -1
ATTN_ERR_ALIGN = -2
ATTN_ERR_CUDA = -3
ATTN_ERR_DEVICE = -4
ATTN_ERR_NOT_SM100 = -5

# Every symbol include/*.h declares, with its ctypes signature.
_u16p = ctypes.c_void_p
_f32p = ctypes.c_void_p
EXPORTS = {
    "attn_flash_scratch_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    "attn_flash_pick_bk": (ctypes.c_int, [ctypes.c_int, ctypes.c_size_t]),
    "attn_flash": (None, [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 7 + [ctypes.c_void_p, ctypes.c_int,
                                                                                 ctypes.c_void_p]),
    "attn_flash_stream": (ctypes.c_int, [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 7 + [ctypes.c_void_p,
                                                                                          ctypes.c_int,
                                                                                          ctypes.c_void_p]),
    "attn_flash_stream_out": (ctypes.c_int, [_u16p, _u16p, _u16p, ctypes.c_void_p, ctypes.c_int] + [ctypes.c_int] * 7 +
                              [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "attn_flash_paged_stream": (ctypes.c_int, [_u16p, _u16p, _u16p, ctypes.c_void_p, ctypes.c_void_p, _f32p] +
                                [ctypes.c_int] * 9 + [ctypes.c_void_p, ctypes.c_void_p]),
    "attn_flash_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "attn_flash_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "attn_flash_kernel_launches": (ctypes.c_ulonglong, []),
    "attn_flash_partial_stream": (ctypes.c_int, [_u16p, _u16p, _u16p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 9 +
                                  [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "attn_flash_combine_stream": (ctypes.c_int, [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 _f32p, ctypes.c_void_p]),
    "attn_flash_packed_floats": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    "attn_flash_combine_packed_stream": (ctypes.c_int, [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                                        ctypes.c_void_p]),
    "attn_flash_noalloc": (ctypes.c_int, [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 8 + [ctypes.c_void_p]),
    "attn_flash_peer_block_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "attn_peer_export": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "attn_peer_import": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "attn_peer_close": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "attn_flash_decode_peers_stream": (ctypes.c_int, [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 9 +
                                       [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint,
                                        ctypes.c_void_p]),
    # include/attn_flash_diag.h
    "attn_diag_fill_tmem": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_void_p]),
    "attn_diag_exp2": (ctypes.c_int, [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "attn_diag_plan": (ctypes.c_int, [ctypes.c_int] * 7 + [ctypes.POINTER(ctypes.c_int)]),
    "attn_diag_wait_timeout": (ctypes.c_int, [_u16p, _u16p, _u16p, _f32p] + [ctypes.c_int] * 4 +
                               [ctypes.c_void_p, ctypes.c_void_p]),
    # include/attn_qkv_rope.h
    "attn_rope_table_stream": (ctypes.c_int, [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_void_p]),
    "attn_qkv_rope_stream": (ctypes.c_int, [_u16p, ctypes.c_void_p, _f32p, ctypes.c_int, _u16p, _u16p, ctypes.c_float]
                             + [ctypes.c_int] * 7 + [_u16p, _u16p, _u16p, ctypes.c_int, ctypes.c_void_p,
                                                     ctypes.c_void_p]),
    "attn_qkv_rope_paged_stream": (ctypes.c_int, [_u16p, ctypes.c_void_p, _f32p, ctypes.c_int, _u16p, _u16p,
                                                  ctypes.c_float] + [ctypes.c_int] * 7
                                   + [_u16p, _u16p, _u16p, ctypes.c_void_p] + [ctypes.c_int] * 3
                                   + [ctypes.c_void_p, ctypes.c_void_p]),
}

_lib = None


class AttnError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: status {status} ({strerror(status)})" if what else strerror(status))


def load_library(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Loads the in-tree library (raises FileNotFoundError when it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: run `python -m transfer_station_b200.build` (no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def strerror(status: int) -> str:
    return load_library().attn_flash_strerror(status).decode()


def attn_flash_kernel_launches() -> int:
    return int(load_library().attn_flash_kernel_launches())


def attn_flash_scratch_bytes(D: int, bk: int) -> int:
    """flash.c:679-682. Aborts the process on an illegal bk, exactly like the reference."""
    return int(load_library().attn_flash_scratch_bytes(D, bk))


def attn_flash_pick_bk(D: int, l2_bytes: int) -> int:
    return int(load_library().attn_flash_pick_bk(D, l2_bytes))


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream_handle(stream) -> int:
    if stream is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream)
    return int(getattr(stream, "cuda_stream", stream))


def attn_flash_stream(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked=0, stream=None) -> int:
    """Asynchronous attention on a torch stream (default: the current stream). Tensors are
    CUDA torch tensors: Q/K/V int16 or uint16 bf16 bit patterns (or torch.bfloat16), O float32,
    scratch a uint8 tensor of attn_flash_scratch_bytes(D, bk) bytes. Returns the status."""
    return int(load_library().attn_flash_stream(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), Hq, Hkv, Sq, Sk, D,
                                                 int(causal), bk, _ptr(scratch), int(v_prepacked),
                                                 _stream_handle(stream)))


def attn_flash_stream_out(Q, K, V, O, out_dtype, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked=0,
                          stream=None) -> int:
    """attn_flash_stream with a choice of output type: ATTN_OUT_F32 (O float32) or ATTN_OUT_BF16
    (O int16/uint16 holding bf16 bits, rounded to nearest even). Returns the status."""
    return int(load_library().attn_flash_stream_out(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), int(out_dtype), Hq, Hkv,
                                                     Sq, Sk, D, int(causal), bk, _ptr(scratch), int(v_prepacked),
                                                     _stream_handle(stream)))


def attn_flash_paged_stream(Q, K_pages, V_pages, block_table, seq_lens, O, B, Hq, Hkv, Sq, D, causal, page_size,
                            num_pages, max_pages, scratch, stream=None) -> int:
    """Attention over a paged K/V cache: pools [num_pages][Hkv][page_size][D] (bf16 bits),
    block_table int32 [B][max_pages], seq_lens int32 [B], all CUDA tensors. Returns the status."""
    return int(load_library().attn_flash_paged_stream(
        _ptr(Q), _ptr(K_pages), _ptr(V_pages), _ptr(block_table), _ptr(seq_lens), _ptr(O), B, Hq, Hkv, Sq, D,
        int(causal), page_size, num_pages, max_pages, _ptr(scratch), _stream_handle(stream)))


def attn_rope_table_stream(cos_sin, max_pos, rot, theta, stream=None) -> int:
    """Fill cos_sin fp32 [max_pos][rot] (cos in columns [0, rot/2), sin after) for frequencies
    theta^(-2i/rot). Returns the status."""
    return int(load_library().attn_rope_table_stream(_ptr(cos_sin), max_pos, rot, float(theta),
                                                      _stream_handle(stream)))


def attn_qkv_rope_stream(qkv, positions, cos_sin, max_pos, q_norm_w, k_norm_w, eps, B, S, Hq, Hkv, D, rot, style,
                         Q, K_cache, V_cache, cache_len, scratch, stream=None) -> int:
    """Split a fused QKV projection [B*S][(Hq+2Hkv)*D] (bf16 bits), RMSNorm (optional weights)
    and rotate q/k heads, write Q [B*Hq][S][D] and K/V rows positions[t] of the contiguous cache
    [B*Hkv][cache_len][D]. Returns the status."""
    return int(load_library().attn_qkv_rope_stream(
        _ptr(qkv), _ptr(positions), _ptr(cos_sin), max_pos, _ptr(q_norm_w), _ptr(k_norm_w), float(eps), B, S, Hq,
        Hkv, D, rot, style, _ptr(Q), _ptr(K_cache), _ptr(V_cache), cache_len, _ptr(scratch),
        _stream_handle(stream)))


def attn_qkv_rope_paged_stream(qkv, positions, cos_sin, max_pos, q_norm_w, k_norm_w, eps, B, S, Hq, Hkv, D, rot,
                               style, Q, K_pages, V_pages, block_table, page_size, num_pages, max_pages, scratch,
                               stream=None) -> int:
    """attn_qkv_rope_stream writing K/V into page pools [num_pages][Hkv][page_size][D] through
    block_table int32 [B][max_pages] (attn_flash_paged_stream's cache). Returns the status."""
    return int(load_library().attn_qkv_rope_paged_stream(
        _ptr(qkv), _ptr(positions), _ptr(cos_sin), max_pos, _ptr(q_norm_w), _ptr(k_norm_w), float(eps), B, S, Hq,
        Hkv, D, rot, style, _ptr(Q), _ptr(K_pages), _ptr(V_pages), _ptr(block_table), page_size, num_pages,
        max_pages, _ptr(scratch), _stream_handle(stream)))


def attn_flash_packed_floats(rows: int, D: int) -> int:
    """Floats of one packed partial block (m, l, padding, acc)."""
    return int(load_library().attn_flash_packed_floats(rows, D))


def attn_flash_combine_packed_stream(parts, nparts, rows, D, O, stream=None) -> int:
    """Merge nparts packed partial blocks laid out back to back into O [rows][D] fp32."""
    return int(load_library().attn_flash_combine_packed_stream(_ptr(parts), nparts, rows, D, _ptr(O),
                                                                _stream_handle(stream)))


def attn_flash(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked=0) -> None:
    """The blocking, void entry (flash.c:727): runs on the legacy default stream, aborts the
    process on error like the C function. Prefer attn_flash_checked in tests."""
    load_library().attn_flash(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), Hq, Hkv, Sq, Sk, D, int(causal), bk,
                              _ptr(scratch), int(v_prepacked), None)


def attn_flash_status(scratch, stream=None) -> tuple[int, int]:
    code = ctypes.c_int(0)
    rc = load_library().attn_flash_status(_ptr(scratch), _stream_handle(stream), ctypes.byref(code))
    return int(rc), int(code.value)


def attn_flash_checked(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked=0, stream=None) -> None:
    """attn_flash_stream + attn_flash_status, raising AttnError instead of aborting."""
    rc = attn_flash_stream(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked, stream)
    if rc != ATTN_OK:
        raise AttnError(rc, "attn_flash_stream")
    rc, code = attn_flash_status(scratch, stream)
    if rc != ATTN_OK:
        raise AttnError(rc, f"attn_flash_status (device code {code})")


def attn_flash_partial_stream(Q, K, V, m, l, acc, Hq, Hkv, Sq, Sk_local, Sk_total, k_begin, D, causal, bk, scratch,
                              v_prepacked=0, stream=None) -> int:
    return int(load_library().attn_flash_partial_stream(_ptr(Q), _ptr(K), _ptr(V), _ptr(m), _ptr(l), _ptr(acc), Hq,
                                                        Hkv, Sq, Sk_local, Sk_total, k_begin, D, int(causal), bk,
                                                        _ptr(scratch), int(v_prepacked), _stream_handle(stream)))


def attn_flash_noalloc(Q, K, V, O, Hq, Hkv, Sq, Sk, D, causal, bk, v_prepacked=0, stream=None) -> int:
    """attn_flash for callers that cannot allocate: no scratch argument (the library's own
    fixed 4 MiB device block is used), at most 4096 query rows, blocking. Returns the status."""
    return int(load_library().attn_flash_noalloc(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), Hq, Hkv, Sq, Sk, D, int(causal),
                                                 bk, int(v_prepacked), _stream_handle(stream)))


def attn_flash_peer_block_bytes(world: int, rows: int, D: int) -> int:
    return int(load_library().attn_flash_peer_block_bytes(world, rows, D))


def attn_peer_export(block) -> bytes:
    """The ATTN_PEER_HANDLE_BYTES handle of a device block (for peers to import)."""
    buf = ctypes.create_string_buffer(ATTN_PEER_HANDLE_BYTES)
    rc = load_library().attn_peer_export(_ptr(block), buf)
    if rc != ATTN_OK:
        raise AttnError(rc, "attn_peer_export")
    return buf.raw


def attn_peer_import(handle: bytes) -> int:
    """Maps a peer's exported block into this process; returns its device address here."""
    out = ctypes.c_void_p(0)
    rc = load_library().attn_peer_import(ctypes.create_string_buffer(handle, ATTN_PEER_HANDLE_BYTES),
                                         ctypes.byref(out))
    if rc != ATTN_OK:
        raise AttnError(rc, "attn_peer_import")
    return int(out.value)


def attn_peer_close(addr: int, handle: bytes) -> int:
    return int(load_library().attn_peer_close(addr, ctypes.create_string_buffer(handle, ATTN_PEER_HANDLE_BYTES)))


def attn_flash_decode_peers_stream(Q, K, V, O, Hq, Hkv, Sq, Sk_local, Sk_total, k_begin, D, causal, bk, scratch,
                                   blocks, world, rank, epoch, stream=None) -> int:
    """`blocks`: every rank's exchange block as device addresses in this process (ints)."""
    arr = (ctypes.c_void_p * len(blocks))(*blocks)
    return int(load_library().attn_flash_decode_peers_stream(
        _ptr(Q), _ptr(K), _ptr(V), _ptr(O), Hq, Hkv, Sq, Sk_local, Sk_total, k_begin, D, int(causal), bk,
        _ptr(scratch), arr, world, rank, epoch, _stream_handle(stream)))


def attn_diag_fill_tmem(bits: int, stream=None) -> int:
    """Diagnostic: write the 32-bit pattern `bits` into all tensor memory of every SM."""
    return int(load_library().attn_diag_fill_tmem(bits & 0xFFFFFFFF, _stream_handle(stream)))


def attn_diag_exp2(x, y, n, method, stream=None) -> int:
    """Diagnostic: y = 2^x by the attention kernel's polynomial (method 0) or MUFU (method 1)."""
    return int(load_library().attn_diag_exp2(_ptr(x), _ptr(y), n, method, _stream_handle(stream)))


class Plan(NamedTuple):
    """The work plan of attn_flash_stream for one problem (attn_diag_plan)."""
    nsplit: int          # key pieces per split unit
    keys_per_split: int
    n_direct: int        # units run whole before a split last wave
    row_base: int        # first query row of the split units
    units: int           # query-row tiles x kv heads


def attn_diag_plan(Hq, Hkv, Sq, Sk, D, causal, sms) -> Plan:
    """Diagnostic: the tensor-core work plan for a GPU with `sms` SMs (host arithmetic only)."""
    out = (ctypes.c_int * 5)()
    rc = int(load_library().attn_diag_plan(Hq, Hkv, Sq, Sk, D, int(causal), sms, out))
    if rc != ATTN_OK:
        raise AttnError(rc, "attn_diag_plan")
    return Plan(*[int(v) for v in out])


def attn_diag_wait_timeout(Q, K, V, O, Hq, Hkv, Sq, Sk, scratch, stream=None) -> int:
    """Diagnostic: the attention kernel with its Q load left out, so a bounded wait runs out."""
    return int(load_library().attn_diag_wait_timeout(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), Hq, Hkv, Sq, Sk,
                                                     _ptr(scratch), _stream_handle(stream)))


def attn_flash_combine_stream(m, l, acc, nparts, rows, D, O, stream=None) -> int:
    return int(load_library().attn_flash_combine_stream(_ptr(m), _ptr(l), _ptr(acc), nparts, rows, D, _ptr(O),
                                                        _stream_handle(stream)))


__all__ = [n for n in dir() if n.startswith("attn_") or n.startswith("ATTN_")] + [
    "AttnError", "load_library", "strerror", "LIB_PATH", "EXPORTS"]
