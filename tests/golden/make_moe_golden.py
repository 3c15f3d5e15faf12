"""Golden greedy decode of a synthetic Qwen3-MoE checkpoint by the reference.

Writes the seeded checkpoint (pyrite_b200.synthetic.moe_tensors: the Q4_K_M
mix of configs[3]) as a real GGUF file with the reference's own
writer (tests/gguf_builder.py), opens it with the reference's
``open_executor`` (a ``Qwen3MoEExecutor``, native C kernels on) and records
the greedy decode of a seeded prompt, the top logits of every forward pass
and the experts routed at every layer of every pass:

    python tests/golden/make_moe_golden.py --spec tiny --out moe_tiny.json
    python tests/golden/make_moe_golden.py --spec c4 --layers 2 --out moe_c4_2l.json
    python tests/golden/make_moe_golden.py --spec c5 --layers 2 --out moe_c5_2l.json

Needs the reference tree (``PYRITE_REF_ROOT``, default: a ``reference`` directory beside the repository); the
committed JSON is what the tests read.
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
    ap.add_argument("--spec", choices=("tiny", "c4", "c5"), default="tiny")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--vocab", type=int, default=None)
    ap.add_argument("--prompt", type=int, default=8)
    ap.add_argument("--new", type=int, default=8)
    ap.add_argument("--out", default="moe_tiny.json")
    args = ap.parse_args()

    from pyrite_b200.synthetic import MoESpec, moe_metadata, moe_tensors, prompt_ids

    spec = {"tiny": MoESpec.tiny, "c4": MoESpec.c4, "c5": MoESpec.c5}[args.spec]()
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
    for key, value in moe_metadata(spec).items():
        builder.add(key, value)
    for name, dims, ggml_type, payload in moe_tensors(spec):
        builder.add_tensor(name, dims, ggml_type, payload)
    path = Path(tempfile.gettempdir()) / f"pyrite_b200_moe_{args.spec}_{spec.num_hidden_layers}_{spec.vocab_size}.gguf"
    builder.write(path)
    print(f"wrote {path} ({path.stat().st_size} bytes) in {time.time() - t0:.1f}s", flush=True)

    ids = prompt_ids(spec, n=args.prompt)
    cfg = RuntimeConfig(ram_budget_mb=32768, max_context_tokens=512, max_kv_tokens=512)
    top: list[list[list[float]]] = []
    experts: list[list[list[int]]] = []
    # per pass and layer: the router logits' gap between the last chosen expert
    # and the first one left out (softmax is monotone, so this is the routing
    # decision's margin), and that runner-up expert
    margins: list[list[float]] = []
    order_margins: list[list[float]] = []  # smallest gap between consecutive chosen experts
    runner_up: list[list[int]] = []
    routers: dict[int, list[float]] = {}
    k = spec.num_experts_per_tok
    with open_executor(path, config=cfg, sampler_seed=0) as ex:
        original = ex.logits
        original_matvec = ex._tensor_matvec

        def router_matvec(name, rows, cols, vector):
            out = original_matvec(name, rows, cols, vector)
            if name.endswith(".ffn_gate_inp.weight"):
                routers[int(name.split(".")[1])] = list(out)
            return out

        def recording(token_id: int, position: int) -> list[float]:
            out = original(token_id, position)
            order = sorted(range(len(out)), key=lambda i: -out[i])[:16]
            top.append([[i, out[i]] for i in order])
            experts.append([list(ex._last_experts.get(layer, ())) for layer in range(spec.num_hidden_layers)])
            gaps, inner, nexts = [], [], []
            for layer in range(spec.num_hidden_layers):
                r = routers[layer]
                ranked = sorted(range(len(r)), key=lambda e: (-r[e], e))
                gaps.append(r[ranked[k - 1]] - r[ranked[k]])
                inner.append(min(r[ranked[i]] - r[ranked[i + 1]] for i in range(k - 1)))
                nexts.append(ranked[k])
            margins.append(gaps)
            order_margins.append(inner)
            runner_up.append(nexts)
            return out

        ex._tensor_matvec = router_matvec
        ex.logits = recording
        t1 = time.time()
        generated = ex.generate(ids, args.new, temperature=0.0)
        seconds = time.time() - t1
    result = {
        "spec": {k: getattr(spec, k) for k in spec.__dataclass_fields__},
        "prompt": ids,
        "generated": generated[len(ids):],
        "top_logits": top,
        "experts": experts,
        "router_margin": margins,
        "router_order_margin": order_margins,
        "runner_up": runner_up,
        "reference_seconds": seconds,
        "reference_tokens_per_second": len(generated) / seconds,
        "generator": "tests/golden/make_moe_golden.py (reference pyrite.executor.open_executor, Qwen3MoEExecutor)",
    }
    (ROOT / "tests" / "golden" / args.out).write_text(json.dumps(result, indent=1))
    print(json.dumps({k: result[k] for k in ("prompt", "generated", "reference_seconds")}))
    path.unlink()


if __name__ == "__main__":
    main()
