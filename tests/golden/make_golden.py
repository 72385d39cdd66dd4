#!/usr/bin/env python3
"""Copy the reference's own kernel golden vectors into tests/golden/.

The files are data written by the reference's llama.cpp-based fixture
generator (fixtures/inference/kernels/provenance.json in sulewicz/promptboot)
and its analytic expf edge table (fixtures/analytic/expf-edge.u32le).  They
are copied byte for byte and each copy is checked against the SHA-256 that the
reference's provenance file records, so the parity tests can run on machines
that do not hold the reference tree.

Usage:  python tests/golden/make_golden.py REFERENCE_ROOT

REFERENCE_ROOT is the root of a sulewicz/promptboot checkout.
"""
from __future__ import annotations

import hashlib
import json
import pathlib
import shutil
import sys

HERE = pathlib.Path(__file__).resolve().parent

KERNEL_FILES = [
    "q8.bin", "dots.bin", "rms.bin", "swiglu.bin", "rope.bin",
    "attention-256.bin", "attention-512.bin", "scores-256.bin", "scores-512.bin",
]


def main() -> int:
    if len(sys.argv) != 2:
        print("usage: make_golden.py REFERENCE_ROOT (a sulewicz/promptboot checkout)", file=sys.stderr)
        return 2
    root = pathlib.Path(sys.argv[1])
    kernels = root / "fixtures" / "inference" / "kernels"
    provenance = json.loads((kernels / "provenance.json").read_text())
    manifest = {}
    for name in KERNEL_FILES:
        data = (kernels / name).read_bytes()
        digest = hashlib.sha256(data).hexdigest()
        expected = provenance["outputs"][name]["sha256"]
        if digest != expected or len(data) != provenance["outputs"][name]["bytes"]:
            print(f"golden mismatch for {name}: {digest} != {expected}", file=sys.stderr)
            return 1
        shutil.copyfile(kernels / name, HERE / name)
        manifest[name] = {"bytes": len(data), "sha256": digest,
                          "source": f"fixtures/inference/kernels/{name}"}
    edge = root / "fixtures" / "analytic" / "expf-edge.u32le"
    data = edge.read_bytes()
    shutil.copyfile(edge, HERE / "expf-edge.u32le")
    manifest["expf-edge.u32le"] = {"bytes": len(data),
                                   "sha256": hashlib.sha256(data).hexdigest(),
                                   "source": "fixtures/analytic/expf-edge.u32le"}
    rope = json.loads((root / "fixtures" / "inference" / "rope-table.provenance.json").read_text())
    manifest["rope-table"] = {"bytes": rope["bytes"], "sha256": rope["sha256"],
                              "selected_bits": rope["selected_bits"],
                              "source": "fixtures/inference/rope-table.provenance.json"}
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"copied {len(manifest) - 1} golden files into {HERE}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
