#!/usr/bin/env python3
"""Generate the golden fixtures of tests/golden/ from the reference's own
numpy oracle (apus tools/oracle.py), imported from a checkout of the
reference.  Run in a container that has the reference:

    python tests/golden/gen_golden.py /path/to/apus-reference

The fixtures pin the CPU restatement in oracle/ (the checker of the CUDA
path) to the reference semantics:
  * linear.npz — FP8 128x128 block dequant (oracle.fp8_dequant + bf16_round,
    one f32 multiply per element, ceil-shaped edge blocks as in
    tests/m3g/gen_golden.py:87-102), BF16 GEMM with the oracle's sequential
    fp32 _mm, and the fp8_linear composition; all bitwise.
  * codec.npz — all 256 E4M3 codes decoded, and a sweep of f32 values
    through the bf16 RNE rounding.
Every case is drawn from a fixed seed, so regeneration is reproducible.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_oracle(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import oracle  # the reference numpy oracle
    return oracle


def codes_of(oracle, x):
    return (oracle.bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def f32_of(c):
    return (c.astype(np.uint32) << np.uint32(16)).view(np.float32)


def fp8_codes(rng, shape):
    c = rng.integers(0, 256, size=shape, dtype=np.uint8)
    c[c == 0x7F] = 0x7E          # NaN codes are refused by the converter
    c[c == 0xFF] = 0xFE
    return c


def scales_for(rng, shape):
    s = np.exp2(rng.uniform(-18.0, 18.0, size=shape)).astype(np.float32)
    flat = s.reshape(-1)
    corners = [1.0, 0.0, 2.0 ** -126, 2.0 ** -127, 2.0 ** 40, 0.5]
    for i, c in enumerate(corners[:flat.size]):
        flat[i] = np.float32(c)
    return s


def dequant(oracle, codes, scales):
    O, K = codes.shape
    w = oracle.E4M3_TABLE[codes].astype(np.float32)
    s = scales[(np.arange(O) // 128)][:, (np.arange(K) // 128)]
    return codes_of(oracle, w * s)


def mm_codes(oracle, x_codes, w_codes):
    y = oracle._mm(f32_of(x_codes), f32_of(w_codes).T)
    return codes_of(oracle, y)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    oracle = load_oracle(ref_root)
    rng = np.random.default_rng(0x5EED)
    out = {}
    deq_shapes = [(128, 128), (256, 384), (200, 136), (1, 128), (5, 129),
                  (128, 127), (300, 264), (64, 4096 // 8)]
    for i, (O, K) in enumerate(deq_shapes):
        c = fp8_codes(rng, (O, K))
        c.reshape(-1)[:12] = [0x00, 0x80, 0x01, 0x07, 0x08, 0x38, 0x7E, 0xFE,
                              0xC0, 0x81, 0x77, 0x6F][:min(12, c.size)]
        s = scales_for(rng, ((O + 127) // 128, (K + 127) // 128))
        out[f"deq{i}_codes"] = c
        out[f"deq{i}_scales"] = s
        out[f"deq{i}_out"] = dequant(oracle, c, s)
    gem_shapes = [(1, 1, 1), (1, 3, 5), (2, 8, 32), (4, 16, 128), (5, 17, 129),
                  (8, 64, 256), (3, 13, 200), (1, 128, 384), (4, 40, 512)]
    for i, (M, O, K) in enumerate(gem_shapes):
        w = codes_of(oracle, rng.uniform(-2, 2, size=(O, K)).astype(np.float32))
        x = codes_of(oracle, rng.uniform(-2, 2, size=(M, K)).astype(np.float32))
        w.reshape(-1)[0] = 0x0000
        if w.size > 1:
            w.reshape(-1)[1] = 0x8000
        out[f"gem{i}_w"] = w
        out[f"gem{i}_x"] = x
        out[f"gem{i}_y"] = mm_codes(oracle, x, w)
    lin_shapes = [(1, 128, 128), (4, 256, 256), (3, 128, 384), (4, 256, 512)]
    for i, (M, O, K) in enumerate(lin_shapes):
        c = fp8_codes(rng, (O, K))
        s = np.exp2(rng.uniform(-10, -4, size=((O + 127) // 128, (K + 127) // 128))).astype(np.float32)
        x = codes_of(oracle, rng.standard_normal((M, K)).astype(np.float32))
        wd = dequant(oracle, c, s)
        out[f"lin{i}_codes"] = c
        out[f"lin{i}_scales"] = s
        out[f"lin{i}_x"] = x
        out[f"lin{i}_y"] = mm_codes(oracle, x, wd)
    np.savez_compressed(os.path.join(HERE, "linear.npz"), **out)

    codec = {"e4m3_table": oracle.E4M3_TABLE.astype(np.float32)}
    vals = np.concatenate([
        rng.standard_normal(4096).astype(np.float32) * np.float32(100.0),
        np.array([0.0, -0.0, 1.0, -1.0, 3.3895314e38, 1e-40, -1e-40,
                  1.00390625, 1.01171875, 65504.0], np.float32)]).astype(np.float32)
    codec["bf16_in"] = vals
    codec["bf16_out"] = codes_of(oracle, vals)
    q = np.clip(rng.standard_normal(4096).astype(np.float32) * np.float32(64.0), -448, 448)
    codec["e4m3_in"] = q.astype(np.float32)
    codec["e4m3_out"] = oracle.e4m3_quant_rne(q.astype(np.float32))
    np.savez_compressed(os.path.join(HERE, "codec.npz"), **codec)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
