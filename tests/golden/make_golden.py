"""Generate tests/golden/golden.npz: small seeded GEMV fixtures for every format.

For each format: seeded packed weights (Q4_K from the reference quantizer restated in the
oracle; Q6_K/Q8_0 from the project quantizers; the IQ and the other block formats as random
valid blocks), a seeded
N(0,1) input, and two outputs:
  * ``_y``     -- the oracle's f32 output (regression pin of the restatement), and
  * ``_y64``   -- an independent float64 product of the weights decoded by gguf-py 0.19.0
                  (a third-party GGUF decoder; the reference itself cannot run here).
Run from the repo root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from tests.helpers import quantized  # noqa: E402


def main() -> None:
    import gguf
    from gguf.quants import dequantize

    Q = gguf.GGMLQuantizationType
    fmts = {"q4_k": (oracle.Q4_K, Q.Q4_K), "q6_k": (oracle.Q6_K, Q.Q6_K), "q8_0": (oracle.Q8_0, Q.Q8_0),
            "iq2_xxs": (oracle.IQ2_XXS, Q.IQ2_XXS), "iq2_xs": (oracle.IQ2_XS, Q.IQ2_XS),
            "iq2_s": (oracle.IQ2_S, Q.IQ2_S), "iq3_xxs": (oracle.IQ3_XXS, Q.IQ3_XXS),
            "iq3_s": (oracle.IQ3_S, Q.IQ3_S), "q4_0": (oracle.Q4_0, Q.Q4_0), "q4_1": (oracle.Q4_1, Q.Q4_1),
            "q5_0": (oracle.Q5_0, Q.Q5_0), "q5_1": (oracle.Q5_1, Q.Q5_1), "q2_k": (oracle.Q2_K, Q.Q2_K),
            "q3_k": (oracle.Q3_K, Q.Q3_K), "q5_k": (oracle.Q5_K, Q.Q5_K), "iq4_nl": (oracle.IQ4_NL, Q.IQ4_NL),
            "iq4_xs": (oracle.IQ4_XS, Q.IQ4_XS)}
    out = {}
    m, n = 16, 512
    for i, (name, (t, qt)) in enumerate(fmts.items()):
        w = quantized(t, m, n, seed=9000 + i)
        x = oracle.normal(9100 + i, n)
        bs = oracle.BLOCK[t][1]
        dense = dequantize(w.reshape(-1, bs), qt).reshape(m, n).astype(np.float64)
        out[name + "_meta"] = np.array([t, m, n], np.int64)
        out[name + "_w"] = w
        out[name + "_x"] = x
        out[name + "_y"] = oracle.gemv(t, m, n, w, x)
        out[name + "_y64"] = dense @ x.astype(np.float64)
    path = os.path.join(ROOT, "tests", "golden", "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
