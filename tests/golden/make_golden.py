"""Regenerates tests/golden/emitter.json from the reference's committed emitter
output (reports/generated-native/ in the reference tree: 19 cases of
`jade-runtime emit-suite`, src/bin/jade-runtime.rs:218-244).

Only digests (of the .cu, .metal and .json files) and the small launch/binding records are stored, not the emitted
source text: the tests compare sha256 of this repository's emitter output with
the reference's, byte for byte.

Usage: python tests/golden/make_golden.py [/path/to/reference]
"""
import hashlib
import json
import os
import sys

REF = (sys.argv[1] if len(sys.argv) > 1 else os.environ.get("JADE_REFERENCE_ROOT")
       or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
SRC = os.path.join(REF, "reports", "generated-native")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "emitter.json")


def sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def main():
    with open(os.path.join(SRC, "manifest.json")) as f:
        manifest = json.load(f)
    cases = []
    for c in manifest["cases"]:
        name = c["case"]
        cases.append({
            "case": name,
            "cu_sha256": sha(os.path.join(SRC, name + ".cu")),
            "metal_sha256": sha(os.path.join(SRC, name + ".metal")),
            "spec_json_sha256": sha(os.path.join(SRC, name + ".json")),
            "launch": c["launch"],
            "bindings": c["bindings"],
        })
    doc = {"source": "reports/generated-native (reference emit-suite output)",
           "manifest_sha256": sha(os.path.join(SRC, "manifest.json")), "cases": cases}
    with open(OUT, "w") as f:
        json.dump(doc, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {OUT}: {len(cases)} cases")


if __name__ == "__main__":
    main()
