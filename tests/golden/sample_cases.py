"""Seeded sampling cases (test helper): logits rows as BF16 codes with the
temperature, top_p and 53-bit uniform each case draws with.  The rows are
rebuilt from their seeds wherever a test needs them; sample.npz holds only
the recipe's outputs (the reference's tokens)."""
import numpy as np

M53 = (1 << 53) - 1


def bf16_codes(x):
    """float32 -> BF16 codes, round to nearest even (c/num.h:153-160)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def _row(seed, V, sigma, kind):
    rng = np.random.default_rng(seed)
    v = rng.standard_normal(V).astype(np.float32) * np.float32(sigma)
    if kind == "flat":                     # every logit equal: ties over the whole row
        v[:] = np.float32(0.25)
    elif kind == "two":                    # two values: two large tie groups
        v = np.where(v > 0, np.float32(1.0), np.float32(-1.0)).astype(np.float32)
    elif kind == "zeros":                  # max value 0 held by -0 (first) and +0
        v = -np.abs(v) - np.float32(0.5)
        v[3], v[7], v[11] = np.float32(-0.0), np.float32(0.0), np.float32(-0.0)
    elif kind == "peak":                   # one dominant logit
        v[V // 3] = np.float32(30.0)
    u53 = int(rng.integers(0, 1 << 53))
    return bf16_codes(v), u53


def cases():
    """List of (name, logits codes, temp, top_p, u53)."""
    out = []
    k = 0
    for V in (384, 4096, 154880):
        for sigma in (0.5, 2.0, 6.0):
            for temp, top_p in ((0.8, 0.95), (1.0, 1.0), (0.5, 0.5), (1.3, 0.9), (2.0, 0.3)):
                row, u53 = _row(1000 + k, V, sigma, "normal")
                out.append((f"V{V}_s{sigma}_t{temp}_p{top_p}", row, temp, top_p, u53))
                k += 1
    for kind in ("flat", "two", "zeros", "peak"):
        for temp, top_p in ((0.8, 0.95), (1.0, 1.0), (0.0, 1.0)):
            row, u53 = _row(2000 + k, 4096, 1.0, kind)
            out.append((f"{kind}_t{temp}_p{top_p}", row, temp, top_p, u53))
            k += 1
    row, _ = _row(3000, 4096, 3.0, "normal")
    for top_p in (0.0, -1.0, 2.0, 5.0, float("nan"), 1e-9):
        out.append((f"top_p_{top_p}", row, 0.9, top_p, 123456789))
    for u53 in (0, M53, 1 << 52):
        out.append((f"u53_{u53}", row, 0.9, 0.95, u53))
    row, u53 = _row(3001, 154880, 60.0, "normal")       # most probabilities underflow to 0
    out.append(("underflow", row, 0.3, 0.99, u53))
    row, u53 = _row(3002, 154880, 0.02, "normal")       # the config's N(0, 0.02)-scale logits
    for temp, top_p in ((0.8, 0.95), (1.0, 1.0)):
        out.append((f"small_t{temp}", row, temp, top_p, u53))
    return out
