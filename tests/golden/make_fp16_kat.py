"""Writes fp16_kat.json: the reference's f32 -> f16 known-answer test, as data.

Source: crates/vxg-tensor/src/fp16.rs:89-108 (`f16_subnormal_rounding_boundaries_both_signs`).
Each case below is that test's (value, expected f16 bits) pair, evaluated here in float32
exactly as the Rust expressions do; the test asserts both `f32_to_f16(v) == e` and
`f32_to_f16(-v) == 0x8000 | e`.  Run: python tests/golden/make_fp16_kat.py
"""
import json
import os

import numpy as np


def f32_bits(x):
    return int(np.float32(x).view(np.uint32))


def from_bits(b):
    return np.uint32(b).view(np.float32)


midpoint = np.float32(2.0) ** np.float32(-25)
# f16_to_f32(0x03ff): largest f16 subnormal, 1023 * 2^-24 (exact in f32)
f16_max_sub = np.float32(1023) * np.float32(2.0) ** np.float32(-24)
cases = [
    (np.float32(0.0), 0x0000),
    (from_bits(1), 0x0000),
    (from_bits(f32_bits(midpoint) - 1), 0x0000),
    (midpoint, 0x0000),
    (from_bits(f32_bits(midpoint) + 1), 0x0001),
    (np.float32(0.75) * np.float32(2.0) ** np.float32(-24), 0x0001),
    (np.float32(2.0) ** np.float32(-24), 0x0001),
    (np.float32(3.0) * midpoint, 0x0002),
    (np.float32(5.0) * midpoint, 0x0002),
    (np.float32(f16_max_sub + midpoint), 0x0400),
]
rows = []
for v, e in cases:
    rows.append({"f32_bits": f32_bits(v), "f16_bits": e})
    rows.append({"f32_bits": f32_bits(-v), "f16_bits": 0x8000 | e})
out = {
    "source": "crates/vxg-tensor/src/fp16.rs:89-108",
    "note": "f32_to_f16 round-to-nearest-even at the subnormal and half-ULP boundaries, both signs",
    "cases": rows,
}
path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fp16_kat.json")
with open(path, "w") as f:
    json.dump(out, f, indent=1)
print(path, len(rows), "cases")
