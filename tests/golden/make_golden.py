"""Writes the golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

1. quant_kat.json -- the known-answer tests of the reference's block code,
   crates/jevons-formats/src/quant.rs:199-237 (zojeda/jevons-rs), restated as data:
     * q4k_scale_min on 12 fixed scale bytes -> pairs 0, 4, 7 = (1,5), (50,33), (8,23)   (:200-208)
     * Q8_0 block with d = 0.5, q[0] = -4, q[31] = 7 -> out[0] = -2.0, out[31] = 3.5    (:211-218)
     * Q5_0 block with d = 1.0, qh = 1 | 1<<16, qs[0] = 0x3f -> out[0,16,1] = 15, 3, -16 (:220-225)
     * pack(Q8_0) of d = 0.5, q[0..4] = 1,2,3,4 -> 8 q words, d = [0.5], q[0] = LE(1,2,3,4);
       pack of 33 bytes fails                                                           (:229-237)
   The reference is Rust and cannot be built in this container (no cargo/rustc), so these
   values are copied from its test source rather than produced by running it.

2. oracle_vectors.npz -- seeded blocks of every supported type with the oracle's dequantized
   f32 output, as a regression guard for the oracle itself (the oracle is pinned by (1) and by
   agreement with a second, word-level restatement, see tests/test_oracle.py).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "jevons-rs_b200"))


def f16_le(v):
    return list(np.array([v], np.float16).view(np.uint8))


def kat():
    q8 = [0] * 34
    q8[0:2] = f16_le(0.5)
    q8[2] = (-4) & 0xFF
    q8[33] = 7
    q5 = [0] * 22
    q5[0:2] = f16_le(1.0)
    q5[2:6] = list(np.array([1 | (1 << 16)], "<u4").view(np.uint8))
    q5[6] = 0x3F
    pk = [0] * 34
    pk[0:2] = f16_le(0.5)
    pk[2:6] = [1, 2, 3, 4]
    return {
        "source": "crates/jevons-formats/src/quant.rs:199-237",
        "q4k_scale_min": {
            "scales": [0xC1, 0x82, 0x43, 0x04, 0x85, 0xC6, 0x07, 0x48, 0x12, 0x34, 0x56, 0x78],
            "expect": {"0": [1, 5], "4": [50, 33], "7": [8, 23]},
        },
        "q8_0": {"type": 8, "bytes": [int(b) for b in q8], "expect": {"0": -2.0, "31": 3.5}},
        "q5_0": {"type": 6, "bytes": [int(b) for b in q5], "expect": {"0": 15.0, "16": 3.0, "1": -16.0}},
        "pack_q8_0": {"type": 8, "bytes": [int(b) for b in pk], "q_len": 8, "d": [0.5],
                      "q0": int(np.array([1, 2, 3, 4], np.uint8).view("<u4")[0]), "bad_len": 33},
    }


def vectors():
    from oracle import oracle
    from jevons_kernels import synth
    rng = np.random.default_rng(20261201)
    out = {}
    for name, kind, k in (("q4k", 12, 512), ("q6k", 14, 512), ("q8_0", 8, 128), ("q5_0", 6, 128)):
        raw = synth.weights(kind, rng, 2, k)
        out[f"{name}_raw"] = raw
        out[f"{name}_f32"] = oracle.dequantize(kind, raw)
    return out


if __name__ == "__main__":
    with open(os.path.join(HERE, "quant_kat.json"), "w") as f:
        json.dump(kat(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_vectors.npz"), **vectors())
    print("wrote quant_kat.json, oracle_vectors.npz")
