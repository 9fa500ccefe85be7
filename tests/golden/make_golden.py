"""Copy the reference's known-answer vectors for the quantized dot path.

The reference checks its dequantizers against C ground truth with these files
(src/quant_dequant.zig:1126-1205, tolerance 1e-3): for each type, 96 packed
256-element rows (`{TYPE}.bin`), the activation `A_x.f32` (256 f32) and the
expected dot(dequant(row), A_x) per row (`{TYPE}_expected.f32`).  They live in
the reference tree at testdata/udtest/; the GPU box has no reference tree, so
the subset on this project's hot path is committed here.

Usage: python tests/golden/make_golden.py [reference-root]
"""
import os
import shutil
import sys

TYPES = ["Q4_K", "Q5_K", "Q6_K", "IQ4_NL", "Q4_0", "Q4_1", "IQ4_XS", "F16"]


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    src = os.path.join(root, "testdata", "udtest")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "udtest")
    os.makedirs(dst, exist_ok=True)
    names = ["A_x.f32"] + [f"{t}{s}" for t in TYPES for s in (".bin", "_expected.f32")]
    for n in names:
        shutil.copyfile(os.path.join(src, n), os.path.join(dst, n))
        os.chmod(os.path.join(dst, n), 0o644)
    print(f"copied {len(names)} files to {dst}")


if __name__ == "__main__":
    main()
