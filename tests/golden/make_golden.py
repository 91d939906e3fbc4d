"""Writes tests/golden/luts.json from the reference's public/*_lut.bin (Git LFS
pointer files: the sha256 object id and byte size of each table) and
public/luts_meta.json.  Run where the reference tree is present, naming its root:

    python tests/golden/make_golden.py PATH_TO_REFERENCE

The tests read only the JSON this writes (the reference is not needed to run them).
"""
import json
import os
import sys


def lfs_pointer(path):
    fields = dict(line.split(" ", 1) for line in open(path).read().splitlines() if " " in line)
    algo, oid = fields["oid"].split(":", 1)
    assert algo == "sha256", path
    return dict(oid=oid, size=int(fields["size"]))


def main(ref):
    pub = os.path.join(ref, "public")
    out = {name: lfs_pointer(os.path.join(pub, f"{name}_lut.bin")) for name in ("mul", "requant", "relu")}
    out["meta"] = json.load(open(os.path.join(pub, "luts_meta.json")))
    out["source"] = "public/{mul,requant,relu}_lut.bin (Git LFS pointers) and public/luts_meta.json"
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "luts.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py PATH_TO_REFERENCE (the reference project's root directory)")
    main(sys.argv[1])
