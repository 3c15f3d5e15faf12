"""SHA-256 of the GGUF files the reference's own builder writes for the tiny goldens.

For each of llama_tiny, moe_tiny and c1_small (the seeded synthetic
checkpoints whose greedy decodes the reference executor recorded), build the
checkpoint with the reference's GGUFFileBuilder (tests/gguf_builder.py in the
reference, the writer its own tests use) from pyrite_b200.synthetic's tensors
and metadata, and record the file's size and SHA-256 in gguf_digests.json.
tests/test_gguf.py writes the same checkpoints with tests/gguf_writer.py and
must reproduce these digests byte for byte; the loader is then tested on
those files.  Runs where the reference tree is present:

    python tests/golden/make_gguf_digests.py [--ref PATH]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

CASES = {"llama_tiny": "llama_tiny.json", "moe_tiny": "moe_tiny.json", "c1_small": "c1_small.json"}


def spec_and_tensors(golden: dict):
    from dataclasses import fields

    from pyrite_b200.synthetic import DenseSpec, MoESpec, dense_tensors, metadata, moe_metadata, moe_tensors
    s = golden["spec"]
    if s["architecture"] == "qwen3moe":
        spec = MoESpec(**{k: v for k, v in s.items() if k in {f.name for f in fields(MoESpec)}})
        return spec, moe_metadata(spec), list(moe_tensors(spec))
    spec = DenseSpec(**{k: v for k, v in s.items() if k in {f.name for f in fields(DenseSpec)}})
    return spec, metadata(spec), list(dense_tensors(spec))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=str(ROOT.parent / "reference"))
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from tests.gguf_builder import GGUFFileBuilder  # the reference's builder

    out = {}
    for case, golden_name in CASES.items():
        golden = json.loads((ROOT / "tests" / "golden" / golden_name).read_text())
        spec, meta, tensors = spec_and_tensors(golden)
        b = GGUFFileBuilder(spec.architecture)
        for k, v in meta.items():
            b.add(k, v)
        for name, dims, t, payload in tensors:
            b.add_tensor(name, dims, t, payload)
        data = b.to_bytes()
        out[case] = {"golden": golden_name, "bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()}
        print(case, out[case], flush=True)
    out["generator"] = "tests/golden/make_gguf_digests.py (the reference's tests/gguf_builder.GGUFFileBuilder)"
    (ROOT / "tests" / "golden" / "gguf_digests.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
