"""Multi-sequence decode (pyrite_b200.batch.BatchDecoder) against independent runs (B200).

The reference serves several prompts with one ``generate`` each
(pyrite/executor.py:878-939).  The oracle here is therefore one
single-sequence greedy decode per prompt (MixedDecoder.generate, itself
checked against the reference executor's greedy ids in test_gpu_decode.py /
test_gpu_moe.py); sequence 0 carries the golden's own prompt, so it is also
compared with the ids the reference executor produced.  Covered: a tiny
Qwen3-MoE (routed experts, 16 experts top-4), the configs[3]-shaped MoE at
full width with two layers (128 experts top-8, batch 16), and a tiny dense
llama.
"""
from __future__ import annotations

import json
from dataclasses import fields
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _spec(g):
    from pyrite_b200.synthetic import DenseSpec, MoESpec
    cls = MoESpec if g["spec"]["architecture"] == "qwen3moe" else DenseSpec
    return cls(**{k: v for k, v in g["spec"].items() if k in {f.name for f in fields(cls)}})


@pytest.mark.parametrize("golden,batch", [("moe_tiny.json", 16), ("moe_c4_2l.json", 16), ("llama_tiny.json", 4)])
def test_batch_decode_equals_independent_runs(cuda_device, golden, batch):
    from pyrite_b200.batch import BatchDecoder
    from pyrite_b200.kernels import cuda as K
    g = json.loads((GOLDEN / golden).read_text())
    spec = _spec(g)
    dec = BatchDecoder.synthetic(spec, device=cuda_device, max_ctx=64, batch=batch)
    prompt, new = g["prompt"], len(g["generated"])
    rng = np.random.default_rng(len(prompt) + batch)
    prompts = [prompt] + [list(map(int, rng.integers(0, spec.vocab_size, len(prompt)))) for _ in range(batch - 1)]
    got = dec.bgenerate(prompts, new)
    assert K.status() == 0
    assert got[0][len(prompt):] == g["generated"], "sequence 0 differs from the reference executor"
    for b, p in enumerate(prompts):
        want = dec.generate(p, new)
        assert got[b] == want, f"sequence {b} differs from its own single-sequence decode"


def test_batch_decode_rejects_unequal_prompts(cuda_device):
    from pyrite_b200.batch import BatchDecoder
    g = json.loads((GOLDEN / "moe_tiny.json").read_text())
    dec = BatchDecoder.synthetic(_spec(g), device=cuda_device, max_ctx=32, batch=2)
    with pytest.raises(ValueError):
        dec.breset([[1, 2, 3], [1, 2]])
    with pytest.raises(ValueError):
        dec.breset([[1, 2, 3]])
