"""Regenerates the golden fixtures in this folder from the reference checkout (run in the build container only;
the GPU box has no reference tree).  The fixtures are the reference's own test data, re-serialised:

* ``frac_tiles.json`` -- the 70 real exllamav3 tiles of plugins/turboexl3_ds41/src/frac_tiles.json (stored words and
  the expected row-major f16 decode), checked by plugins/turboexl3_ds41/src/frac_test.zig:23-57.
* ``manifest_golden.json`` -- the ``golden`` block of plugins/turboexl3_ds41/src/exl3/kernels/exl3/manifest.json: the
  mul1 table digest and the four splitmix64 planes (seed, K, projection, code/W_hat/one-hot digests), checked by
  plugins/turboexl3_ds41/src/exl3/selfcheck.zig:861-930.

Usage: python tests/golden/make_golden.py REFERENCE_ROOT   (or set EXL3_REFERENCE_ROOT)
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    src = os.path.join(ref_root, "plugins/turboexl3_ds41/src/frac_tiles.json")
    with open(src) as f:
        frac = json.load(f)
    tiles = [{"src": t["src"], "n": t["n"], "words": t["words"], "expect": t["expect"]} for t in frac["tiles"]]
    with open(os.path.join(HERE, "frac_tiles.json"), "w") as f:
        json.dump({"from": "plugins/turboexl3_ds41/src/frac_tiles.json", "what": frac.get("what", ""), "tiles": tiles},
                  f, separators=(",", ":"))
    man = os.path.join(ref_root, "plugins/turboexl3_ds41/src/exl3/kernels/exl3/manifest.json")
    with open(man) as f:
        golden = json.load(f)["golden"]
    with open(os.path.join(HERE, "manifest_golden.json"), "w") as f:
        json.dump({"from": "plugins/turboexl3_ds41/src/exl3/kernels/exl3/manifest.json#golden", "golden": golden}, f,
                  indent=1, sort_keys=True)
    print(f"wrote {len(tiles)} frac tiles and {len(golden['planes'])} golden planes")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("EXL3_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the reference checkout), or set EXL3_REFERENCE_ROOT")
    main(root)
