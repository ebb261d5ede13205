"""Regenerate tests/golden/qkv_golden.npz from the CPU oracle.

The reference (nathansutton/chad) ships no stored vectors for this path and MLX cannot run
here, so these fixtures pin the oracle's restatement against itself over time (and give
the GPU tests byte-exact expectations): small seeded inputs, their 4-/8-bit codes, scales,
biases, dequantized values and the fp32 attention outputs.

    python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import qkv_oracle as orc  # noqa: E402


def build():
    rng = np.random.default_rng(20261201)
    out = {}
    q = orc.round_to(rng.standard_normal((1, 8, 2, 128), dtype=np.float32), "bf16")
    k = orc.make_kv(rng, (1, 2, 96, 128), outliers=True)
    v = orc.make_kv(rng, (1, 2, 96, 128), outliers=False)
    out["q"], out["k"], out["v"] = q, k, v
    for bits in (4, 8):
        kq = orc.affine_quantize(k, bits, 64, "bf16")
        vq = orc.affine_quantize(v, bits, 64, "bf16")
        for name, t in zip(("w", "s", "b"), kq):
            out[f"k{bits}_{name}"] = t
        for name, t in zip(("w", "s", "b"), vq):
            out[f"v{bits}_{name}"] = t
        out[f"kdq{bits}"] = orc.dequantize(*kq, bits, 64, "bf16")
        out[f"kdq{bits}_per_op"] = orc.dequantize(*kq, bits, 64, "bf16", "per_op")
        out[f"attn{bits}"] = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 90, bits)
        out[f"attn{bits}_causal"] = orc.attention_quantized_fp32(q, kq, vq, 128 ** -0.5, 90,
                                                                 bits, mask="causal")
    return out


if __name__ == "__main__":
    np.savez_compressed(os.path.join(HERE, "qkv_golden.npz"), **build())
    print("wrote", os.path.join(HERE, "qkv_golden.npz"))
