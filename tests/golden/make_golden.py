"""Generates tests/golden/formats.npz: golden vectors for the GGML block formats.

Run in a container where the `gguf` Python package (gguf-py 0.19.0, the llama.cpp project's
published reader/writer of GGML quant formats) is importable:

    python tests/golden/make_golden.py

The fixtures pin the oracle's format code against an implementation it shares nothing with:
  * q8_inputs / q8_bytes: gguf.quants.quantize(..., Q8_0) of seeded N(0, 0.02) and sin-pattern
    data (the sin pattern of the reference's own fixtures, src/moe/tests.rs:190-200);
  * q4k_bytes / q4k_dequant: Q4_K super-blocks (bytes from the oracle's quantiser) and
    gguf.quants.dequantize of those bytes.
The tests never import gguf; they only read the committed .npz.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

import gguf  # noqa: E402
import gguf.quants as gq  # noqa: E402

from oracle import oracle  # noqa: E402


def main():
    rng = np.random.Generator(np.random.Philox(20261201))
    gauss = rng.normal(0.0, 0.02, size=(8, 256)).astype(np.float32)
    i = np.arange(4 * 64, dtype=np.float32)
    sinpat = (np.sin(i * np.float32(0.37) + np.float32(0.7)) * np.float32(0.5)).astype(np.float32).reshape(4, 64)
    q8_inputs = np.concatenate([gauss.reshape(-1), sinpat.reshape(-1)]).astype(np.float32)
    q8_bytes = gq.quantize(q8_inputs.reshape(-1, 32), gguf.GGMLQuantizationType.Q8_0).reshape(-1)

    w = rng.normal(0.0, 0.02, size=(6, 256)).astype(np.float32)
    w[3] += 0.05  # a super-block with all-positive mins
    w[5] *= 40.0  # large range
    q4k_bytes, _ = oracle.quantize(oracle.DT_Q4_K, w)
    q4k_dequant = gq.dequantize(q4k_bytes.reshape(6, 144), gguf.GGMLQuantizationType.Q4_K).reshape(-1)

    np.savez_compressed(
        os.path.join(HERE, "formats.npz"),
        q8_inputs=q8_inputs,
        q8_bytes=np.asarray(q8_bytes, dtype=np.uint8),
        q4k_inputs=w.reshape(-1),
        q4k_bytes=q4k_bytes,
        q4k_dequant=np.asarray(q4k_dequant, dtype=np.float32),
        gguf_version=np.array(["gguf-py 0.19.0"]),
    )
    print("wrote formats.npz", q8_bytes.shape, q4k_bytes.shape)


if __name__ == "__main__":
    main()
