"""Regenerates tests/golden/rng.json: the first draws of the oracle's mulberry32(42)
(src/math/random.ts:8-17 restated).  Run from the repository root:
    python tests/golden/make_golden.py
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import Oracle  # noqa: E402


def main():
    o = Oracle()
    st = o.rng(42)
    vals = [o.rng_next(st) for _ in range(8)]
    out = {"src": "src/math/random.ts:8-17", "seed": 42, "values": vals}
    with open(os.path.join(ROOT, "tests", "golden", "rng.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
