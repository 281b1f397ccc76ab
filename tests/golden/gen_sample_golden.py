#!/usr/bin/env python3
"""Generate tests/golden/sample.npz from the reference's own sampler
(c/sample.h apus_sample_logits_u and the splitmix64 stream, compiled into
oracle/_ref/libapus_ref.so by oracle/Makefile from the reference sources):

    make -C oracle && python tests/golden/gen_sample_golden.py

For every case of sample_cases.cases() it records the token the reference
draws from the widened BF16 row with u = u53 * 2^-53, and for three seeds
the first 8 outputs of apus_rng_next."""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from sample_cases import cases  # noqa: E402


def main():
    assert O.REF is not None, "oracle/_ref/libapus_ref.so is not built (needs the reference sources)"
    names, tokens = [], []
    for name, row, temp, top_p, u53 in cases():
        names.append(name)
        tokens.append(O.ref_sample_logits_u(row, temp, top_p, u53 * 2.0 ** -53))
    O.REF.apus_rng_next.restype = C.c_uint64
    O.REF.apus_rng_next.argtypes = [C.POINTER(C.c_uint64)]
    seeds = np.array([0, 12345, (1 << 64) - 1], np.uint64)
    draws = np.zeros((3, 8), np.uint64)
    for i, s in enumerate(seeds):
        st = C.c_uint64(int(s))
        for j in range(8):
            draws[i, j] = O.REF.apus_rng_next(C.byref(st))
    np.savez_compressed(os.path.join(HERE, "sample.npz"), names=np.array(names), tokens=np.array(tokens, np.int32),
                        rng_seeds=seeds, rng_draws=draws)
    print(f"{len(names)} cases")


if __name__ == "__main__":
    main()
