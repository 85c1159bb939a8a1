"""Generates tests/golden/*.npz from the REFERENCE's own flash.c.

Run in a container that has the reference sources (TS_REFERENCE_DIR, or a `reference`
directory beside the repository):

    python tests/golden/make_golden.py

It builds oracle/_ref (flash.c compiled unmodified through oracle/sve_shim), then for each
case below records the inputs and the outputs of the reference's `attn_ref` (its fp32
oracle, flash.c:262-314) and its `attn_flash` (the SVE kernel, flash.c:727-864; at BQ=128 as
shipped, or the -DBQ=64 build where the case says so). Inputs come from the reference's LCG
(flash.c:867-871, seed 0x12345678 as its harness uses) or from the seeded generators of the
benchmark configs (oracle/attn_oracle.c). The fixtures are what the CPU tests pin the oracle
restatement against; the GPU box never needs the reference sources.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402

# name, Hq, Hkv, Sq, Sk, D, causal, bk, bq, data, v_prepacked
CASES = [
    # flash.c:1287-1299, the shipped suite, plus the two decode cases of flash_long.log:16-17
    ("mha_prefill", 4, 4, 8, 8, 64, 0, 128, 128, "lcg", 0),
    ("mha_prefill_causal", 4, 4, 8, 8, 64, 1, 128, 128, "lcg", 0),
    ("gqa_prefill", 8, 2, 8, 8, 64, 0, 128, 128, "lcg", 0),
    ("gqa_prefill_causal", 8, 2, 8, 8, 64, 1, 128, 128, "lcg", 0),
    ("mqa_prefill", 8, 1, 8, 8, 64, 0, 128, 128, "lcg", 0),
    ("odd_multiblock", 6, 3, 130, 70, 40, 1, 128, 128, "lcg", 0),
    ("gqa_big_head_dim", 8, 2, 4, 12, 128, 0, 128, 128, "lcg", 0),
    ("mha_decode", 4, 4, 1, 16, 64, 0, 128, 128, "lcg", 0),
    ("gqa_decode", 8, 2, 1, 16, 64, 0, 128, 128, "lcg", 0),
    # multi-key-block online softmax (several rescales), bk below and above the tile
    ("multiblock_causal_bk32", 4, 2, 96, 300, 64, 1, 32, 128, "lcg", 0),
    ("multiblock_full_bk64", 4, 2, 64, 600, 64, 0, 64, 128, "lcg", 0),
    # pre-transposed V (pack_v_full, flash.c:714-718)
    ("prepacked_v", 4, 2, 64, 200, 64, 1, 64, 128, "lcg", 1),
    # tails: Sk=1 (O = V[0]) and Sk < Sq causal (fully masked rows)
    ("sk1", 4, 2, 16, 1, 64, 0, 128, 128, "lcg", 0),
    ("masked_rows", 4, 4, 200, 33, 32, 1, 128, 128, "lcg", 0),
    # BASELINE config 1 (N(0,1) seed 0, BQ=64, bk=128)
    ("config1_mha_s256_d64", 4, 4, 256, 256, 64, 0, 128, 64, "normal0", 0),
]


def main() -> None:
    oracle.build(ref=True)
    manifest = {}
    for name, Hq, Hkv, Sq, Sk, D, causal, bk, bq, data, vp in CASES:
        if data == "lcg":
            Q, K, V = oracle.lcg_inputs(Hq, Hkv, Sq, Sk, D)
        else:
            Q, K, V = oracle.seeded_inputs(Hq, Hkv, Sq, Sk, D, seed=0)
        # every row for small cases; 32 spread rows (flash.c:900-913) for config 1
        rows = oracle.rowset(Sq, 32 if Sq > 128 and data != "lcg" else 0)
        o_ref = oracle.ref_attn_ref(Q, K, V, Hq, Hkv, Sq, Sk, D, causal, rows)
        Vin = V
        if vp:
            L = oracle.ref_lib(128)
            Vin = np.empty_like(V)
            L.ref_pack_v_full(V.ctypes.data, Vin.ctypes.data, Hkv, Sk, D)
        o_flash = oracle.ref_attn_flash(Q, K, Vin, Hq, Hkv, Sq, Sk, D, causal, bk=bk, bq=bq, v_prepacked=vp)
        c = oracle.cmp_rows(o_ref, o_flash, Hq, Sq, D, rows)
        sel = lambda O: O.reshape(Hq, Sq, D)[:, rows, :].copy()  # noqa: E731
        extra = {"Vin": Vin} if vp else {}
        np.savez_compressed(HERE / f"{name}.npz", Q=Q, K=K, V=V, rows=rows, o_attn_ref=sel(o_ref),
                            o_attn_flash=sel(o_flash), **extra)
        manifest[name] = dict(Hq=Hq, Hkv=Hkv, Sq=Sq, Sk=Sk, D=D, causal=causal, bk=bk, bq=bq, data=data,
                              v_prepacked=vp, ref_err_scale=c["err_scale"], ref_nbad=c["nbad"])
        print(f"{name:26s} err/scale(ref kernel vs ref fp32) = {c['err_scale']:.2e}")
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")


if __name__ == "__main__":
    main()
