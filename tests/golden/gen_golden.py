"""Generates tests/golden/*.npz from the CPU oracle.

The reference (GPULlama3.java) has no attention tests or golden vectors and
cannot run here, so these fixtures are produced by the oracle's restatement
of InferenceCore.java:105-144 and pin it against regressions; kernels are
checked against them too.  Inputs come from tests/inputs.py (numpy PCG64,
~N(0,1)); large inputs are stored only as a SHA-256 of their bytes and
regenerated from the seed.

Run: python tests/golden/gen_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "tests"), os.path.join(REPO, "oracle")]

import inputs  # noqa: E402
import oracle  # noqa: E402

# name: (seed, n_heads, n_kv_heads, head_dim, n_pos, f16_cache, store_inputs)
DECODE_CASES = {
    "gqa4_hd64_pos39": (1, 8, 2, 64, 40, False, True),
    "gqa7_hd128_pos32": (2, 14, 2, 128, 33, False, True),
    "mha_hd96_pos16": (3, 4, 4, 96, 17, False, True),
    "gqa4_hd64_pos0": (4, 4, 1, 64, 1, False, True),
    "gqa4_hd128_pos49_f16": (5, 8, 2, 128, 50, True, True),
    # Llama-3.2-1B shape, seed 0, position 511
    "c1_llama32_1b_pos511": (0, 32, 8, 64, 512, False, False),
}

ROPE_CASES = {
    # name: (seed, n_heads, n_kv_heads, head_dim, position, theta, style)
    "rope_llama3_theta5e5_pos123": (10, 24, 8, 128, 123, 500000.0, "interleaved"),
    "rope_neox_theta1e6_pos77": (11, 28, 4, 128, 77, 1000000.0, "neox"),
}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    oracle.build()
    out = {}
    for name, (seed, nh, nkv, hd, npos, f16, store) in DECODE_CASES.items():
        q, k, v = inputs.decode_case(seed, nh, nkv, hd, npos)
        if f16:
            k16, v16 = inputs.to_f16_bits(k), inputs.to_f16_bits(v)
            xb = oracle.decode_f16(q, k16, v16, nh, nkv, hd, npos, n_threads=1)
            kin, vin = k16, v16
        else:
            xb = oracle.decode_f32(q, k, v, nh, nkv, hd, npos, n_threads=1)
            kin, vin = k, v
        out[f"{name}/meta"] = np.array([seed, nh, nkv, hd, npos, int(f16)], dtype=np.int64)
        out[f"{name}/xb"] = xb
        out[f"{name}/sha256"] = np.array(sha(q, kin, vin))
        if store:
            out[f"{name}/q"] = q
            out[f"{name}/k"] = kin
            out[f"{name}/v"] = vin
    for name, (seed, nh, nkv, hd, pos, theta, style) in ROPE_CASES.items():
        rng = np.random.Generator(np.random.PCG64(seed))
        q = rng.standard_normal(nh * hd, dtype=np.float32)
        k = rng.standard_normal(nkv * hd, dtype=np.float32)
        cr, ci = oracle.rope_freqs(pos + 1, hd, theta)
        q2, k2 = q.copy(), k.copy()
        if style == "interleaved":
            oracle.rope_interleaved(q2, k2, hd, pos, cr, ci)
        else:
            oracle.rope_neox(q2, k2, nh, nkv, hd, pos, cr, ci)
        out[f"{name}/meta"] = np.array([seed, nh, nkv, hd, pos, 0 if style == "interleaved" else 1],
                                       dtype=np.int64)
        out[f"{name}/theta"] = np.array(theta)
        out[f"{name}/q_in"] = q
        out[f"{name}/k_in"] = k
        out[f"{name}/q_out"] = q2
        out[f"{name}/k_out"] = k2
    path = os.path.join(HERE, "attention_golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
