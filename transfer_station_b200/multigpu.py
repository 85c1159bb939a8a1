"""Multi-GPU partitioning of the attention path (one process per GPU, torch.distributed).

Two decompositions, as the work shards (none of them exists in flash.c, which is one call on one
core):

* Prefill shards by (batch x kv-head group): the units are independent -- every query head of
  a group reads only its kv head's K/V -- so each rank runs attn_flash on whole kv groups and
  writes its own slice of O (sharded_prefill). No collective.

* Long-context decode with few kv heads shards the KEY axis: rank r holds keys
  [k_begin, k_begin + Sk_local) of every kv head, runs attn_flash_partial_stream on them
  (masking by global key position) straight into one packed block of per-row partials
  (m, l, acc) -- a few hundred KB -- which one NCCL all-gather collects over NVLink, and every
  rank merges them with attn_flash_combine_packed_stream into the full output. This is the key
  loop of flash.c:798 split across GPUs, with the online-softmax merge of flash.c:535-576
  applied across shards.

  Two ways to merge: `sharded_decode` (the partial kernel into a packed block, one NCCL
  all-gather, the combine kernel) and `sharded_decode_peers` with a `PeerMerge` (the partial
  kernel, then ONE merge kernel that stores each rank's partials straight into every peer's
  exchange block over NVLink, signals with flags, and merges: no collective per step).

The NCCL path uses only torch.distributed collectives, so the same code runs with the `gloo`
backend on CPU tensors (the tests do that with a CPU stand-in for the partial kernel).
"""
from __future__ import annotations

from typing import NamedTuple

import torch
import torch.distributed as dist

import transfer_station_b200 as ts


def unit_shard(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [start, end) of n_units independent units for `rank` (the first
    n_units % world ranks take one more)."""
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class PrefillSlice(NamedTuple):
    """One rank's share of a prefill sharded by (batch x kv-head group) units: units [u0, u1) of
    the B*Hkv units, as an attn_flash problem of hq query heads and hkv kv heads whose Q / O
    start `q_off` elements into [B*Hq][Sq][D] and whose K / V start `kv_off` elements into
    [B*Hkv][Sk][D]. Unit u is kv head u of that layout, and its query heads u*group ..
    u*group + group - 1 (b*Hq + kv*group == (b*Hkv + kv)*group), so a rank's share is one
    contiguous range of each tensor: no gather, no copy."""

    u0: int
    u1: int
    hq: int
    hkv: int
    q_off: int
    kv_off: int


def prefill_slice(B: int, Hq: int, Hkv: int, Sq: int, Sk: int, D: int, world: int, rank: int) -> PrefillSlice:
    """The (batch x kv-head group) units of a B-sequence prefill that `rank` of `world` runs:
    flash.c's head loop (flash.c:779-782, kv = h / group) partitioned by kv head, every query
    head of a group staying with the kv head it reads."""
    if Hq % Hkv:
        raise ValueError("Hq must be a multiple of Hkv")
    group = Hq // Hkv
    u0, u1 = unit_shard(B * Hkv, world, rank)
    return PrefillSlice(u0, u1, (u1 - u0) * group, u1 - u0, u0 * group * Sq * D, u0 * Sk * D)


def _rank_world(group, rank, world):
    if rank is not None and world is not None:
        return rank, world
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def sharded_prefill(q, k, v, O, B: int, Hq: int, Hkv: int, Sq: int, Sk: int, D: int, causal: int, scratch,
                    bk: int = ts.ATTN_BK_DEFAULT, group=None, stream=None, rank: int | None = None,
                    world: int | None = None) -> PrefillSlice:
    """Prefill of B sequences ([B*Hq][Sq][D] queries, [B*Hkv][Sk][D] keys and values, O
    [B*Hq][Sq][D] fp32) sharded over the ranks of `group` by (batch x kv-head group) units.
    The tensors have the full problem's layout on every rank, but a rank reads only its units'
    Q, K and V and writes only its units' rows of O, through one attn_flash_stream call on
    those contiguous ranges; no collective is issued (each rank's O rows are final where they
    are). `rank` / `world` override the process group's (one process may then run every
    rank's share in turn). Returns the rank's PrefillSlice; raises AttnError on a library error."""
    rank, world = _rank_world(group, rank, world)
    s = prefill_slice(B, Hq, Hkv, Sq, Sk, D, world, rank)
    if s.hkv == 0:  # more ranks than units: nothing to do here
        return s
    nq, nkv = s.hq * Sq * D, s.hkv * Sk * D
    qv = q.view(-1)[s.q_off:s.q_off + nq]
    kv_ = k.view(-1)[s.kv_off:s.kv_off + nkv]
    vv = v.view(-1)[s.kv_off:s.kv_off + nkv]
    ov = O.view(-1)[s.q_off:s.q_off + nq]
    rc = ts.attn_flash_stream(qv, kv_, vv, ov, s.hq, s.hkv, Sq, Sk, D, causal, bk, scratch, 0, stream)
    if rc != ts.ATTN_OK:
        raise ts.AttnError(rc, "attn_flash_stream (sharded prefill)")
    return s


def key_shard(Sk: int, world: int, rank: int, align: int = ts.ATTN_GPU_KEY_TILE) -> tuple[int, int]:
    """Key range (k_begin, k_len) of `rank` when Sk keys are split over `world` ranks. Shard
    boundaries fall on multiples of `align` (the kernel's key tile) so no tile straddles two
    ranks; the last rank takes the remainder. A rank may get an empty range when Sk is small."""
    blocks = -(-Sk // align)
    b0, b1 = unit_shard(blocks, world, rank)
    k0 = min(Sk, b0 * align)
    k1 = min(Sk, b1 * align)
    return k0, k1 - k0


def packed_floats(rows: int, D: int) -> int:
    """Floats of one rank's packed partial block: m [rows], l [rows], padding to a multiple of 4,
    acc [rows][D] (attn_flash_packed_floats, restated so the CPU tests need no library)."""
    return -(-2 * rows // 4) * 4 + rows * D


def packed_views(buf: torch.Tensor, rows: int, D: int):
    """(m, l, acc) views into one packed block (acc 16-byte aligned when buf is)."""
    off = -(-2 * rows // 4) * 4
    return buf[:rows], buf[rows:2 * rows], buf[off:off + rows * D].view(rows, D)


def gather_packed(buf: torch.Tensor, group=None) -> torch.Tensor:
    """One all-gather of every rank's packed block: [world * packed_floats] (the rank's own
    block alone when there is no process group or a single rank)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return buf
    world = dist.get_world_size(group)
    out = torch.empty(world * buf.numel(), dtype=buf.dtype, device=buf.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    return out


def sharded_decode(q, k_shard, v_shard, O, Hq: int, Hkv: int, Sq: int, Sk_total: int, k_begin: int, D: int,
                   causal: int, scratch, bk: int = ts.ATTN_BK_DEFAULT, group=None, stream=None):
    """Attention over a key axis split across the ranks of `group`. Every rank passes its own
    K/V shard ([Hkv][Sk_local][D], keys k_begin.. of the global axis) and the full Q; every rank
    receives the full O [Hq*Sq*D] (fp32). The partial kernel writes (m, l, acc) straight into one
    packed block, one NCCL all-gather collects every rank's block and the combine merges them
    from the gathered buffer. Raises AttnError on a library error."""
    rows = Hq * Sq
    Sk_local = k_shard.numel() // (Hkv * D)
    buf = torch.empty(packed_floats(rows, D), dtype=torch.float32, device=q.device)
    m, l, acc = packed_views(buf, rows, D)
    if Sk_local > 0:
        rc = ts.attn_flash_partial_stream(q, k_shard, v_shard, m, l, acc, Hq, Hkv, Sq, Sk_local, Sk_total, k_begin,
                                          D, causal, bk, scratch, 0, stream)
        if rc != ts.ATTN_OK:
            raise ts.AttnError(rc, "attn_flash_partial_stream")
    else:  # an empty shard contributes nothing: m = -inf, l = 0
        m.fill_(float("-inf"))
        l.zero_()
        acc.zero_()
    parts = gather_packed(buf, group)
    nparts = parts.numel() // buf.numel()
    rc = ts.attn_flash_combine_packed_stream(parts, nparts, rows, D, O, stream)
    if rc != ts.ATTN_OK:
        raise ts.AttnError(rc, "attn_flash_combine_packed_stream")
    return O


class PeerMerge:
    """The exchange blocks of a key-split decode merged by peer stores (one per rank, CUDA IPC).

    Created collectively by every rank of `group` (the process group carries the handles once, at
    set-up; the steps use none). Each rank allocates its block (attn_flash_peer_block_bytes,
    zeroed), exports it, imports every peer's, and keeps the epoch counter the kernel's flags
    use. `close()` (collective) unmaps the peers' blocks."""

    def __init__(self, rows: int, D: int, group=None, device=None):
        self.rank, self.world = _rank_world(group, None, None)
        if self.world > ts.ATTN_PEERS_MAX:
            raise ValueError(f"at most {ts.ATTN_PEERS_MAX} ranks")
        self.group = group
        self.rows, self.D = rows, D
        nbytes = ts.attn_flash_peer_block_bytes(self.world, rows, D)
        if nbytes == 0:
            raise ValueError("bad exchange block shape")
        self.block = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(self.block.device)
        handle = ts.attn_peer_export(self.block) if self.world > 1 else b""
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle, group=group)
        self.handles = handles
        self.addrs = [self.block.data_ptr() if r == self.rank else ts.attn_peer_import(handles[r])
                      for r in range(self.world)]
        self.epoch = 0
        if self.world > 1:
            dist.barrier(group=group)  # every block mapped everywhere before the first store

    def close(self):
        if self.world > 1:
            dist.barrier(group=self.group)  # nobody stores into a block being unmapped
        for r, a in enumerate(self.addrs):
            if r != self.rank and a:
                ts.attn_peer_close(a, self.handles[r])
        self.addrs = []


def sharded_decode_peers(q, k_shard, v_shard, O, Hq: int, Hkv: int, Sq: int, Sk_total: int, k_begin: int, D: int,
                         causal: int, scratch, merge: PeerMerge, bk: int = ts.ATTN_BK_DEFAULT, stream=None):
    """sharded_decode with the merge done by one kernel over NVLink instead of the NCCL
    all-gather and the combine: the partial kernel on this rank's key shard, then the peer
    merge kernel, which leaves the full O [Hq*Sq*D] fp32 on every rank. Every rank makes every
    call, in the same order. Raises AttnError on a library error."""
    Sk_local = k_shard.numel() // (Hkv * D) if k_shard is not None else 0
    merge.epoch += 1
    rc = ts.attn_flash_decode_peers_stream(q, k_shard if Sk_local else None, v_shard if Sk_local else None, O, Hq,
                                           Hkv, Sq, Sk_local, Sk_total, k_begin, D, causal, bk, scratch, merge.addrs,
                                           merge.world, merge.rank, merge.epoch, stream)
    if rc != ts.ATTN_OK:
        raise ts.AttnError(rc, "attn_flash_decode_peers_stream")
    return O
