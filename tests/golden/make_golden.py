"""Extract the reference's checked-in golden bit patterns into a JSON fixture.

The reference pins its CPU trainer with literal IEEE-754 bit patterns in
``tests/test_golden_bits.mojo`` (seven fixtures; the fixture definitions are at
``tests/test_golden_bits.mojo:7920-8120`` of ajhendel/mojoboost).  This script
reads that file as text (it runs only where the reference checkout is present)
and writes ``golden_bits.json`` beside itself.  The large fixture's per-row raw
scores and predictions (12,000 rows each) are stored as a SHA-256 digest of the
little-endian uint64 bit array plus the first 64 entries, to keep the fixture
small; every other array is stored in full.

Usage:  python tests/golden/make_golden.py <path to reference checkout>
"""
import hashlib
import json
import os
import re
import struct
import sys


def _blocks(text):
    out = {}
    for m in re.finditer(r'comptime (_[A-Z0-9_]+) = """\n(.*?)"""', text, re.S):
        out[m.group(1)] = m.group(2).split()
    return out


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOJOTREES_REFERENCE", "")
    src = os.path.join(ref, "tests", "test_golden_bits.mojo")
    text = open(src).read()
    blocks = _blocks(text)
    fixtures = {}
    for name in ("L2", "LOGIT", "MULTI", "BAG", "FFRAC", "MISSCAT", "LARGE"):
        ints = [int(v) for v in blocks[f"_{name}_INTS"]]
        vals = blocks[f"_{name}_VALS"]
        raw = blocks[f"_{name}_RAW"]
        pred = blocks[f"_{name}_PRED"]
        fx = {"ints": ints, "vals": vals}
        for key, arr in (("raw", raw), ("pred", pred)):
            if name == "LARGE":
                packed = b"".join(struct.pack("<Q", int(h, 16)) for h in arr)
                fx[key + "_sha256"] = hashlib.sha256(packed).hexdigest()
                fx[key + "_len"] = len(arr)
                fx[key + "_head"] = arr[:64]
            else:
                fx[key] = arr
        fixtures[name.lower()] = fx
    doc = {
        "source": "tests/test_golden_bits.mojo (ajhendel/mojoboost), GOLDEN BEGIN..END block",
        "platform_of_record": "arm64-apple-darwin, Mojo 1.0.0",
        "fixtures": fixtures,
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_bits.json")
    with open(dst, "w") as f:
        json.dump(doc, f, separators=(",", ":"))
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main()
