"""Writes tests/golden/blake3_vectors.json: BLAKE3 (plain hash, 32 bytes) of the input
pattern byte(i) = i mod 251 at lengths that cross every block, chunk and tree-level
boundary up to 100 KiB, computed with the `blake3` Python package (the BLAKE3 team's
binding of the reference implementation; the reference's pvlc-pack uses the blake3 crate,
Cargo.lock 1.8.5).  Run from the repository root: python tests/golden/make_blake3_vectors.py"""
import json
import os

import blake3

LENGTHS = [0, 1, 2, 63, 64, 65, 127, 128, 129, 1023, 1024, 1025, 2048, 2049, 3072, 3073,
           4096, 4097, 5120, 5121, 6144, 6145, 7168, 7169, 8192, 8193, 16384, 31744,
           102400]


def main():
    out = {"pattern": "i mod 251", "digests": {}}
    for n in LENGTHS:
        data = bytes(i % 251 for i in range(n))
        out["digests"][str(n)] = blake3.blake3(data).hexdigest()
    path = os.path.join(os.path.dirname(__file__), "blake3_vectors.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
