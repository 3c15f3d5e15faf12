"""One rank of a tensor-parallel decode (run under torchrun by tests/test_gpu_sharded.py).

    python -m torch.distributed.run --nproc-per-node N tests/sharded_worker.py GOLDEN.json

Rebuilds the golden file's synthetic checkpoint, decodes its prompt greedily on
N GPUs (pyrite_b200.sharded.ShardedDecoder: heads / rows / experts sharded,
NCCL allreduce after the output and down projections, allgather of the
logits) and checks the generated ids (and, for MoE, the routed experts) against
the reference's; rank 0 prints one JSON line.
"""
from __future__ import annotations

import datetime
import json
import os
import sys
from dataclasses import fields
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main() -> int:
    import torch
    import torch.distributed as dist

    from pyrite_b200.sharded import ShardedDecoder
    from pyrite_b200.synthetic import DenseSpec, MoESpec

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    g = json.loads(Path(sys.argv[1]).read_text())
    cls = MoESpec if g["spec"].get("architecture") == "qwen3moe" else DenseSpec
    names = {f.name for f in fields(cls)}
    spec = cls(**{k: v for k, v in g["spec"].items() if k in names})
    dec = ShardedDecoder.synthetic(spec, rank, world, device=dev, max_ctx=128)
    prompt, want = g["prompt"], g["generated"]
    got = dec.generate(prompt, len(want))[len(prompt):]
    ok = got == want
    routed_ok = None
    if dec.moe:
        dec.reset(prompt)
        routed_ok = True
        for step in range(len(prompt) + len(want) - 1):
            dec.run_steps(1)
            torch.cuda.synchronize(dev)
            routed_ok &= dec.route_log.cpu().tolist() == g["experts"][step]
    from pyrite_b200.kernels import cuda as K
    status = K.status()
    if rank == 0:
        print(json.dumps({"world": world, "ids_match": ok, "got": got, "want": want, "routed_match": routed_ok,
                          "status": status}), flush=True)
    dec.graph = None
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok and routed_ok in (None, True) and status == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
