"""Helpers for the GPU parity tests: move oracle-generated bf16 inputs to the device, run the
C-ABI entry point, bring the output back."""
from __future__ import annotations

import numpy as np
import torch

import transfer_station_b200 as ts


def to_dev(a: np.ndarray, dev) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def scratch_for(D: int, bk: int, dev) -> torch.Tensor:
    return torch.empty(ts.attn_flash_scratch_bytes(D, bk), dtype=torch.uint8, device=dev)


def run_gpu(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, bk=128, v_prepacked=0, dev="cuda:0", scratch=None) -> np.ndarray:
    """Runs attn_flash_stream + attn_flash_status on device copies of host bf16 arrays."""
    q, k, v = to_dev(Q, dev), to_dev(K, dev), to_dev(V, dev)
    o = torch.full((Hq * Sq * D,), float("nan"), dtype=torch.float32, device=dev)
    if scratch is None:
        scratch = scratch_for(D, bk, dev)
    ts.attn_flash_checked(q, k, v, o, Hq, Hkv, Sq, Sk, D, causal, bk, scratch, v_prepacked)
    torch.cuda.synchronize()
    return o.cpu().numpy()
