"""Generates tests/golden/rope_*.npz: golden vectors for the QKV producer (attn_qkv_rope.h).

The reference has no producer (its projections never reach the attention kernel,
flash.c:1301-1304), so the vectors come from a widely used implementation of the same
formulas: transformers' own Qwen3 functions (Qwen3RMSNorm, apply_rotary_pos_emb with
rotate_half) and GPT-J's apply_rotary_pos_emb (rotate_every_two, partial rotary slice as
GPT-J's attention applies it). Run in a container that has transformers:

    python tests/golden/make_rope_golden.py

Inputs are bf16 values (seeded), evaluated in fp32 by transformers, with each token's cos/sin
taken from the oracle's table rows (also stored) so the fixture pins the rotation and the norm;
the table itself is pinned to its float64 definition separately. Each file holds the inputs,
the table rows and transformers' fp32 outputs for the q and k heads.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from oracle import qkv_rope as orq  # noqa: E402

# name, B, S, Hq, Hkv, D, rot, style, norm, max_pos, theta, seed
CASES = [
    ("rope_qwen3_norm", 2, 3, 4, 2, 128, 128, orq.NEOX, True, 40960, 1e6, 11),
    ("rope_neox_plain_longpos", 1, 5, 2, 1, 64, 64, orq.NEOX, False, 131072, 1e6, 12),
    ("rope_gptj_partial", 2, 2, 2, 2, 256, 64, orq.GPTJ, False, 2048, 1e4, 13),
]


def bf16_bits(a: np.ndarray) -> np.ndarray:
    return oracle.f32_to_bf16(a.astype(np.float32))


def hf_qwen3(q, k, c, s, qw, kw, eps, norm):
    """q [B,Hq,S,D], k [B,Hkv,S,D] fp32; c, s [B,S,rot/2] fp32 (rot = D for Qwen3)."""
    from transformers.models.qwen3 import modeling_qwen3 as m

    if norm:
        qn = m.Qwen3RMSNorm(q.shape[-1], eps=eps)
        kn = m.Qwen3RMSNorm(k.shape[-1], eps=eps)
        with torch.no_grad():
            qn.weight.copy_(qw)
            kn.weight.copy_(kw)
            q, k = qn(q), kn(k)
    cos = torch.cat([c, c], dim=-1)
    sin = torch.cat([s, s], dim=-1)
    with torch.no_grad():
        return m.apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1)


def hf_gptj(x, c, s, rot):
    """x [B,S,H,D] fp32 (GPT-J's head layout); c, s [B,S,rot/2]. Rotates x[..., :rot] and passes
    the rest through, as GPT-J's attention does."""
    from transformers.models.gptj import modeling_gptj as g

    with torch.no_grad():
        xr = g.apply_rotary_pos_emb(x[..., :rot], s, c)
    return torch.cat([xr, x[..., rot:]], dim=-1)


def main() -> None:
    oracle.build(ref=False)
    manifest = {}
    for name, B, S, Hq, Hkv, D, rot, style, norm, max_pos, theta, seed in CASES:
        rng = np.random.default_rng(seed)
        T, H = B * S, Hq + 2 * Hkv
        qkv = bf16_bits(rng.normal(0.0, 1.0, (T, H * D)))
        pos = rng.integers(0, max_pos, T).astype(np.int32)
        pos[0] = max_pos - 1
        qw = bf16_bits(rng.uniform(0.6, 1.4, D))
        kw = bf16_bits(rng.uniform(0.6, 1.4, D))
        eps = 1e-6
        table = orq.rope_table(max_pos, rot, theta)
        rows = table[pos]
        half = rot // 2
        x = oracle.bf16_to_f32(qkv).reshape(B, S, H, D)
        c = torch.from_numpy(rows[:, :half].reshape(B, S, half).copy())
        s = torch.from_numpy(rows[:, half:].reshape(B, S, half).copy())
        if style == orq.NEOX:
            q = torch.from_numpy(x[:, :, :Hq].transpose(0, 2, 1, 3).copy())
            k = torch.from_numpy(x[:, :, Hq:Hq + Hkv].transpose(0, 2, 1, 3).copy())
            qo, ko = hf_qwen3(q, k, c, s, torch.from_numpy(oracle.bf16_to_f32(qw)),
                              torch.from_numpy(oracle.bf16_to_f32(kw)), eps, norm)
            q_out = qo.numpy().transpose(0, 2, 1, 3)  # back to [B,S,H,D]
            k_out = ko.numpy().transpose(0, 2, 1, 3)
        else:
            assert not norm
            q_out = hf_gptj(torch.from_numpy(x[:, :, :Hq].copy()), c, s, rot).numpy()
            k_out = hf_gptj(torch.from_numpy(x[:, :, Hq:Hq + Hkv].copy()), c, s, rot).numpy()
        np.savez_compressed(HERE / f"{name}.npz", qkv=qkv, positions=pos, rows=rows, q_norm=qw, k_norm=kw,
                            q_out=q_out.astype(np.float32), k_out=k_out.astype(np.float32))
        manifest[name] = dict(B=B, S=S, Hq=Hq, Hkv=Hkv, D=D, rot=rot, style=style, norm=norm, max_pos=max_pos,
                              theta=theta, eps=eps, seed=seed,
                              source="transformers " + __import__("transformers").__version__)
        print(name, "written")
    (HERE / "rope_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")


if __name__ == "__main__":
    main()
