"""GPU, one device: the key-split decode's merge kernel (attn_flash_decode_peers_stream) through
the C ABI -- the online-softmax merge of flash.c:535-576 done across ranks by peer stores.

On one GPU a merge kernel may only wait for flags that are already raised or that nothing
raises (two ranks' kernels never run as separate launches on one GPU, since nothing makes them
run at the same time). So the other rank of a two-rank merge is emulated from the host: its
partials (from attn_flash_partial_stream on its key shard) and its raised flags are written into
this rank's exchange block before the launch, where rank 1's own kernel would have stored them.
The two-GPU test in tests/test_multigpu.py runs the real exchange."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import transfer_station_b200 as ts
from tests.gpu_util import scratch_for, to_dev
from transfer_station_b200 import multigpu

pytestmark = pytest.mark.gpu

FLAG_BYTES = ts.ATTN_PEERS_MAX * 128 * 4


def _slot_floats(rows, D):
    return (ts.attn_flash_packed_floats(rows, D) * 4 + 255) // 256 * 64


@pytest.mark.parametrize("case", [(64, 8, 1, 65536, 128, 0), (256, 32, 1, 8192, 128, 0), (24, 6, 3, 5000, 64, 1),
                                  (6, 3, 1, 700, 40, 0)])
def test_single_rank_merge_matches_reference(cuda_dev, case):
    """world = 1: the partial kernel's key pieces merged by the merge kernel, over several calls
    (epochs 1..3, both buffers) with new data each time, against the fp32 reference."""
    Hq, Hkv, Sq, Sk, D, causal = case
    merge = multigpu.PeerMerge(Hq * Sq, D, device=cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    rows = np.arange(Sq, dtype=np.int32)
    for call in range(3):
        Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=20 + call, a=0.0, b=0.5)
        q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
        o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
        multigpu.sharded_decode_peers(q, k, v, o, Hq, Hkv, Sq, Sk, 0, D, causal, scratch, merge)
        torch.cuda.synchronize()
        assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)
        ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
        c = oracle.cmp_rows(ref, o.cpu().numpy(), Hq, Sq, D, rows)
        assert oracle.passes(c), (call, c)
    assert merge.epoch == 3
    merge.close()


def test_two_rank_merge_with_emulated_peer(cuda_dev):
    """Rank 0 of a two-rank merge; rank 1's partials and flags placed in rank 0's block from the
    host beforehand (its kernel would have stored them over NVLink). The kernel also stores rank
    0's partials and flags into rank 1's block (here a second local buffer): both are checked."""
    Hq, Hkv, Sq, Sk, D = 64, 8, 1, 20000, 128
    rows = Hq * Sq
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=30, a=0.0, b=0.5)
    k0, kl0 = multigpu.key_shard(Sk, 2, 0)
    k1, kl1 = multigpu.key_shard(Sk, 2, 1)
    K3, V3 = K.reshape(Hkv, Sk, D), V.reshape(Hkv, Sk, D)
    shard = lambda a, b, n: to_dev(np.ascontiguousarray(a[:, b:b + n]).reshape(-1), cuda_dev)  # noqa: E731
    q = to_dev(Q, cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    # rank 1's partial of its shard (what its own merge kernel would store)
    pf = ts.attn_flash_packed_floats(rows, D)
    part1 = torch.zeros(pf, dtype=torch.float32, device=cuda_dev)
    m1, l1, acc1 = multigpu.packed_views(part1, rows, D)
    assert ts.attn_flash_partial_stream(q, shard(K3, k1, kl1), shard(V3, k1, kl1), m1, l1, acc1, Hq, Hkv, Sq, kl1, Sk,
                                        k1, D, 0, 128, scratch, 0) == ts.ATTN_OK
    nbytes = ts.attn_flash_peer_block_bytes(2, rows, D)
    blocks = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda_dev) for _ in range(2)]
    epoch = 1
    sf = _slot_floats(rows, D)
    fb = FLAG_BYTES // 4
    own = blocks[0].view(torch.float32)
    buf = epoch & 1
    own[fb + (buf * 2 + 1) * sf: fb + (buf * 2 + 1) * sf + pf] = part1
    blocks[0].view(torch.int32)[1 * 128: 1 * 128 + 128] = epoch  # rank 1's flags, every CTA
    o = torch.full((rows * D,), float("nan"), dtype=torch.float32, device=cuda_dev)
    rc = ts.attn_flash_decode_peers_stream(q, shard(K3, k0, kl0), shard(V3, k0, kl0), o, Hq, Hkv, Sq, kl0, Sk, k0, D,
                                           0, 128, scratch, [b.data_ptr() for b in blocks], 2, 0, epoch)
    assert rc == ts.ATTN_OK
    torch.cuda.synchronize()
    assert ts.attn_flash_status(scratch) == (ts.ATTN_OK, 0)
    r = np.arange(Sq, dtype=np.int32)
    ref = oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, r)
    c = oracle.cmp_rows(ref, o.cpu().numpy(), Hq, Sq, D, r)
    assert oracle.passes(c), c
    # rank 0's stores into the peer's block: its slot holds rank 0's partial, its flags the epoch
    peer = blocks[1].view(torch.float32)
    slot0 = peer[fb + (buf * 2 + 0) * sf: fb + (buf * 2 + 0) * sf + pf]
    pm, pl, pacc = multigpu.packed_views(slot0, rows, D)
    ctas = min(rows, 128)
    assert torch.all(blocks[1].view(torch.int32)[:ctas] == epoch)
    assert torch.all(torch.isfinite(pm)) and torch.all(pl > 0)
    # merged with rank 1's partial it gives the same output
    both = torch.stack([slot0, part1])
    o2 = torch.empty_like(o)
    assert ts.attn_flash_combine_packed_stream(both.view(-1), 2, rows, D, o2) == ts.ATTN_OK
    torch.cuda.synchronize()
    assert torch.allclose(o, o2, rtol=1e-6, atol=1e-7)


def test_peer_that_never_arrives_is_reported(cuda_dev):
    """A two-rank merge whose other rank never stores its partials (its flags stay 0: nothing
    raises them): the bounded wait runs out after ~2 s, the call reports ATTN_DEV_TIMEOUT_PEER
    through the status word instead of hanging, and the context stays usable."""
    Hq, Hkv, Sq, Sk, D = 8, 2, 1, 1024, 128
    Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=31)
    q, k, v = to_dev(Q, cuda_dev), to_dev(K, cuda_dev), to_dev(V, cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    nbytes = ts.attn_flash_peer_block_bytes(2, Hq * Sq, D)
    blocks = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda_dev) for _ in range(2)]
    o = torch.zeros(Hq * Sq * D, dtype=torch.float32, device=cuda_dev)
    rc = ts.attn_flash_decode_peers_stream(q, k, v, o, Hq, Hkv, Sq, Sk, Sk, 0, D, 0, 128, scratch,
                                           [b.data_ptr() for b in blocks], 2, 0, 1)
    assert rc == ts.ATTN_OK
    rc, code = ts.attn_flash_status(scratch)
    assert rc == ts.ATTN_ERR_DEVICE and code & ts.ATTN_DEV_TIMEOUT_PEER, (rc, code)
    # still usable: an ordinary single-rank merge afterwards is correct
    merge = multigpu.PeerMerge(Hq * Sq, D, device=cuda_dev)
    multigpu.sharded_decode_peers(q, k, v, o, Hq, Hkv, Sq, Sk, 0, D, 0, scratch, merge)
    torch.cuda.synchronize()
    r = np.arange(Sq, dtype=np.int32)
    c = oracle.cmp_rows(oracle.attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, 0, r), o.cpu().numpy(), Hq, Sq, D, r)
    assert oracle.passes(c), c


def test_bad_arguments_are_rejected(cuda_dev):
    """epoch 0, too many ranks, rank out of range, a misaligned block: ATTN_ERR_* without a launch."""
    Hq, Hkv, Sq, Sk, D = 8, 2, 1, 256, 128
    q = torch.zeros(Hq * Sq * D, dtype=torch.int16, device=cuda_dev)
    k = torch.zeros(Hkv * Sk * D, dtype=torch.int16, device=cuda_dev)
    o = torch.zeros(Hq * Sq * D, dtype=torch.float32, device=cuda_dev)
    scratch = scratch_for(D, 128, cuda_dev)
    blk = torch.zeros(ts.attn_flash_peer_block_bytes(1, Hq * Sq, D) + 256, dtype=torch.uint8, device=cuda_dev)
    p = blk.data_ptr()
    call = lambda blocks, world, rank, epoch: ts.attn_flash_decode_peers_stream(  # noqa: E731
        q, k, k, o, Hq, Hkv, Sq, Sk, Sk, 0, D, 0, 128, scratch, blocks, world, rank, epoch)
    assert call([p], 1, 0, 0) == ts.ATTN_ERR_ARGS
    assert call([p] * 9, 9, 0, 1) == ts.ATTN_ERR_ARGS
    assert call([p], 1, 1, 1) == ts.ATTN_ERR_ARGS
    assert call([p + 16], 1, 0, 1) == ts.ATTN_ERR_ALIGN
    assert ts.attn_flash_peer_block_bytes(9, 8, 128) == 0
