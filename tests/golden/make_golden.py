"""Writes the golden fixtures the oracle is pinned against.

The reference (cublas-rs) ships no unit tests; its correctness checks are the
example binaries' all-ones known answers.  They cannot be run here (no Rust
toolchain, and cuda-oxide is an un-vendored git dependency), so this script
records them as data, each with the file:line it comes from, together with
  * the published PCG32 known-answer sequence (pcg32_srandom(42, 54), the
    pcg-c-basic demo), which pins the input generator, and
  * bit-level vectors of the reference's own f16 conversions
    (crates/cublas-l3/src/hgemm.rs:20-51), derived by evaluating that code's
    branches by hand for chosen inputs (flush, truncation, saturation, nan).

Run:  python tests/golden/make_golden.py   (rewrites the .json files here)
"""
import json
import math
import os

HERE = os.path.dirname(os.path.abspath(__file__))

KNOWN_ANSWERS = {
    "about": "Known answers from the cublas-rs example binaries.  GEMM/SGEMV cases are all-ones "
             "(A = B = 1, x = 1), so every output equals the inner dimension; the HGEMV case is the "
             "example's ramp, checked against an f32 sum of the same f16 values; the reductions use "
             "x = [0, 1, ..., n-1], whose sums have closed forms.",
    "cases": [
        {"op": "sgemm", "variants": ["naive", "tiled", "vectorized", "double_buf"], "m": 512, "n": 512, "k": 512,
         "alpha": 1.0, "beta": 0.0, "expect": 512.0, "tol_abs": 1e-3,
         "ref": "examples/sgemm/src/main.rs:12-14,17-23,32-43,178-206 (tolerance :192)"},
        {"op": "dgemm", "variants": ["naive", "tiled"], "m": 512, "n": 512, "k": 512, "alpha": 1.0, "beta": 0.0,
         "expect": 512.0, "tol_abs": 1e-3, "ref": "examples/sgemm/src/main.rs:45-63,208-234 (tolerance :220)"},
        {"op": "strided_batched_sgemm", "batch": 8, "m": 64, "n": 64, "k": 64, "alpha": 1.0, "beta": 0.0,
         "stride_a": 4096, "stride_b": 4096, "stride_c": 4096, "expect": 64.0, "tol_abs": 1e-3,
         "ref": "examples/sgemm/src/main.rs:65-111"},
        {"op": "batched_sgemm", "batch": 8, "m": 64, "n": 64, "k": 64, "alpha": 1.0, "beta": 0.0, "expect": 64.0,
         "tol_abs": 1e-3, "ref": "examples/sgemm/src/main.rs:113-134"},
        {"op": "hgemm", "m": 128, "n": 128, "k": 128, "alpha": 1.0, "beta": 0.0, "expect": 128.0,
         "tol_rel": 5e-3, "ref": "examples/sgemm/src/main.rs:136-175 (tolerance :162)"},
        {"op": "sgemm", "variants": ["naive", "tiled", "vectorized", "double_buf"], "m": 256, "n": 256,
         "k": 256, "alpha": 1.0, "beta": 0.0, "expect": 256.0, "tol_abs": 1e-3,
         "ref": "examples/gemm_bench/src/main.rs:23-26,147-153"},
        {"op": "sgemm", "variants": ["naive", "tiled", "vectorized", "double_buf"], "m": 1024, "n": 1024,
         "k": 1024, "alpha": 1.0, "beta": 0.0, "expect": 1024.0, "tol_abs": 1e-3,
         "ref": "examples/gemm_bench/src/main.rs:23-26,147-153"},
        {"op": "dgemm", "variants": ["naive", "tiled", "vectorized", "double_buf"], "m": 256, "n": 256,
         "k": 256, "alpha": 1.0, "beta": 0.0, "expect": 256.0, "tol_abs": 1e-3,
         "ref": "examples/gemm_bench/src/main.rs:23-26,147-153 (dgemm section)"},
        {"op": "sgemv", "trans": "N", "m": 16, "n": 24, "alpha": 1.0, "beta": 0.0, "expect": 24.0, "tol_abs": 1e-3,
         "ref": "examples/saxpy/src/main.rs:88-106"},
        {"op": "sgemv", "trans": "T", "m": 16, "n": 24, "alpha": 1.0, "beta": 0.0, "expect": 16.0, "tol_abs": 1e-3,
         "ref": "examples/saxpy/src/main.rs:108-124"},
        {"op": "hgemv", "trans": "N", "m": 16, "n": 24, "alpha": 1.0, "beta": 0.0,
         "a": "f16 round-to-nearest of 0.01*i, i the flat index", "x": "f16 round-to-nearest of 0.1*j",
         "expect": "f32 sum over j of f32(a[i,j]) * f32(x[j]) in j order", "tol_rel": 5e-3,
         "ref": "examples/saxpy/src/main.rs:132-172 (tolerance :160)"},
        {"op": "sdot", "n": 1024, "x": "i", "y": "i", "expect": 357389824.0, "tol_rel": 1e-3,
         "ref": "examples/saxpy/src/main.rs:12-14,39,44,48-56 (sum of i^2 = (n-1)n(2n-1)/6)"},
        {"op": "snrm2", "n": 1024, "x": "i", "expect": math.sqrt(357389824.0),
         "tol_rel": 1e-3, "ref": "examples/saxpy/src/main.rs:40,45,57"},
        {"op": "sasum", "n": 1024, "x": "i", "expect": 523776.0, "tol_rel": 1e-3,
         "ref": "examples/saxpy/src/main.rs:41,46,58 (sum of i = n(n-1)/2)"},
        {"op": "isamax", "n": 1024, "x": "i", "expect": 1023, "ref": "examples/saxpy/src/main.rs:42,59-63"},
    ],
}

PCG32_KAT = {
    "about": "pcg32 (XSH-RR 64->32), pcg32_srandom(initstate=42, initseq=54): first six outputs, "
             "as printed by the pcg-c-basic demo program.",
    "seed": 42, "stream": 54,
    "outputs": [0xa15c02b7, 0x7b47f409, 0xba1d3330, 0x83d2f293, 0xbfa4784b, 0xcbed606e],
}

# crates/cublas-l3/src/hgemm.rs:34-51 (f32_to_f16, truncating) evaluated by hand.
F32_TO_F16_REF = [
    (1.0, 0x3C00, "exp 127 -> 15, mantissa 0"),
    (-2.0, 0xC000, "sign kept"),
    (65504.0, 0x7BFF, "largest f16"),
    (65520.0, 0x7BFF, "truncation: no rounding up to inf (RNE would give 0x7C00)"),
    (65536.0, 0x7C00, "new_exp >= 31 saturates to inf"),
    (1.000732421875, 0x3C00, "1 + 3*2^-12 truncates (RNE gives 0x3C01)"),
    (0.333251953125, 0x3555, "exact f16 value"),
    (6.103515625e-05, 0x0400, "smallest normal f16"),
    (3.0517578125e-05, 0x0000, "below normal range flushes to +0 (RNE gives subnormal 0x0200)"),
    (-3.0517578125e-05, 0x8000, "flushes to -0"),
    (float("inf"), 0x7C00, "inf"),
    (float("-inf"), 0xFC00, "-inf"),
    (float("nan"), 0x7C01, "nan -> exponent all ones, mantissa 1"),
]

# crates/cublas-l3/src/hgemm.rs:20-32 (f16_to_f32) evaluated by hand.
F16_TO_F32_REF = [
    (0x3C00, 1.0, "one"),
    (0xC000, -2.0, "minus two"),
    (0x7BFF, 65504.0, "largest"),
    (0x0400, 6.103515625e-05, "smallest normal"),
    (0x0001, 0.0, "subnormal flushes to +0"),
    (0x83FF, -0.0, "negative subnormal flushes to -0"),
    (0x7C00, float("inf"), "inf"),
    (0x3555, 0.333251953125, "exact"),
]


def _enc(x):
    if x != x:
        return "nan"
    if x in (float("inf"), float("-inf")):
        return "inf" if x > 0 else "-inf"
    return x


def main():
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(KNOWN_ANSWERS, f, indent=1)
    with open(os.path.join(HERE, "pcg32_kat.json"), "w") as f:
        json.dump(PCG32_KAT, f, indent=1)
    conv = {
        "about": "cublas-rs's software f16 conversions (crates/cublas-l3/src/hgemm.rs:20-51), one row per branch.",
        "f32_to_f16": [{"x": _enc(x), "bits": b, "why": w} for x, b, w in F32_TO_F16_REF],
        "f16_to_f32": [{"bits": b, "x": _enc(x), "negzero": (x == 0.0 and str(x).startswith("-")), "why": w}
                       for b, x, w in F16_TO_F32_REF],
    }
    with open(os.path.join(HERE, "f16_conversions.json"), "w") as f:
        json.dump(conv, f, indent=1)


if __name__ == "__main__":
    main()
