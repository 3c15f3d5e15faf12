"""Golden greedy decode of configs[0] (Qwen3-0.6B-shaped, Q8_0) by the reference executor.

Writes the seeded synthetic checkpoint (pyrite_b200.synthetic) as a real GGUF
file with the reference's own writer (tests/gguf_builder.py), opens it with
the reference's ``open_executor`` (a ``DenseExecutor``, native C kernels on),
and records the greedy decode of the seeded prompt plus the top logits of
every forward pass:

    python tests/golden/make_c1_golden.py [--spec c1|c3] [--layers N] [--vocab V] [--out NAME]

Defaults are configs[0] in full (28 layers, vocab 151936, 16-token prompt,
8 new tokens, KV limit 512); ``--spec c3`` is the Llama-3-8B-shaped Q4_K_M
model of configs[2] (use --layers to keep the reference run short), ``c3tiny``
the same architecture and mix at toy width.  Needs the reference tree (``PYRITE_REF_ROOT``,
default: a ``reference`` directory beside the repository); the committed JSON is what the tests read.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from dataclasses import replace
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
REF = Path(os.environ.get("PYRITE_REF_ROOT", ROOT.parent / "reference"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--spec", choices=("c1", "c3", "c3tiny"), default="c1")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--vocab", type=int, default=None)
    ap.add_argument("--new", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--out", default="c1_decode.json")
    args = ap.parse_args()

    from pyrite_b200.synthetic import DenseSpec, dense_tensors, metadata, prompt_ids

    spec = DenseSpec.c1() if args.spec == "c1" else DenseSpec.c3()
    if args.spec == "c3tiny":  # the configs[2] architecture and mix at toy width
        spec = replace(spec, hidden_size=512, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       intermediate_size=1024, vocab_size=2048)
    if args.layers is not None:
        spec = replace(spec, num_hidden_layers=args.layers)
    if args.vocab is not None:
        spec = replace(spec, vocab_size=args.vocab)

    sys.path.insert(0, str(REF))
    from pyrite.config import RuntimeConfig  # noqa: E402
    from pyrite.executor import open_executor  # noqa: E402
    from tests.gguf_builder import GGUFFileBuilder  # noqa: E402

    t0 = time.time()
    builder = GGUFFileBuilder(spec.architecture)
    for key, value in metadata(spec).items():
        builder.add(key, value)
    for name, dims, ggml_type, payload in dense_tensors(spec):
        builder.add_tensor(name, dims, ggml_type, payload)
    path = Path(tempfile.gettempdir()) / f"pyrite_b200_c1_{spec.num_hidden_layers}_{spec.vocab_size}.gguf"
    builder.write(path)
    print(f"wrote {path} ({path.stat().st_size} bytes) in {time.time() - t0:.1f}s", flush=True)

    ids = prompt_ids(spec, n=args.prompt)
    cfg = RuntimeConfig(ram_budget_mb=32768, max_context_tokens=512, max_kv_tokens=512)
    top: list[list[list[float]]] = []
    with open_executor(path, config=cfg, sampler_seed=0) as ex:
        original = ex.logits

        def recording(token_id: int, position: int) -> list[float]:
            out = original(token_id, position)
            order = sorted(range(len(out)), key=lambda i: -out[i])[:16]
            top.append([[i, out[i]] for i in order])
            return out

        ex.logits = recording
        t1 = time.time()
        generated = ex.generate(ids, args.new, temperature=0.0)
        seconds = time.time() - t1
        stats = ex.stats.to_dict()
    result = {
        "spec": {k: getattr(spec, k) for k in spec.__dataclass_fields__},
        "prompt": ids,
        "generated": generated[len(ids):],
        "top_logits": top,
        "reference_seconds": seconds,
        "reference_tokens_per_second": len(generated) / seconds,
        "native_kernel_calls": stats["native_kernel_calls"],
        "generator": "tests/golden/make_c1_golden.py (reference pyrite.executor.open_executor, DenseExecutor)",
    }
    (ROOT / "tests" / "golden" / args.out).write_text(json.dumps(result, indent=1))
    print(json.dumps({k: result[k] for k in ("prompt", "generated", "reference_seconds")}))
    path.unlink()


if __name__ == "__main__":
    main()
