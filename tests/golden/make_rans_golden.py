"""Generate tests/golden/rans.npz: seeded byte inputs and their VQ2A streams as written by the C
oracle (oracle/rans_oracle.c). The fixture pins the stream format: the product host encoder must
reproduce these bytes and the GPU decoder must expand them back to the inputs.

The VQ2A format is this repository's own (the reference's ANS coder, the third-party
`constriction` package used in vq2/export.py:26-36, is not installed and no reference test pins
its streams), so these vectors come from the oracle, not from the reference.

Usage: python tests/golden/make_rans_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import rans as R  # noqa: E402


def inputs():
    rng = np.random.default_rng(20261201)
    skew = np.minimum(np.abs(rng.normal(0, 3000, 12000)), 65535).astype(np.uint16).view(np.uint8)
    return {
        "empty": np.zeros(0, np.uint8),
        "one": np.array([201], np.uint8),
        "const": np.full(9000, 17, np.uint8),
        "two_symbols": rng.choice(np.array([0, 255], np.uint8), 700, p=[0.9, 0.1]).astype(np.uint8),
        "uniform_8191": rng.integers(0, 256, 8191).astype(np.uint8),
        "geom_8192": np.minimum(rng.geometric(0.08, 8192), 255).astype(np.uint8),
        "nib_8193": rng.integers(0, 16, 8193).astype(np.uint8),
        "skew_u16": skew,
    }


def main():
    out = {}
    for k, v in inputs().items():
        out[f"in_{k}"] = v
        out[f"enc_{k}"] = R.encode(v)
    counts = np.random.default_rng(3).integers(0, 1000, 256).astype(np.uint64)
    counts[::7] = 0
    out["q_counts"] = counts
    out["q_freq"] = R.quantize(counts)
    np.savez_compressed(os.path.join(HERE, "rans.npz"), **out)
    print({k: v.size for k, v in out.items()})


if __name__ == "__main__":
    main()
