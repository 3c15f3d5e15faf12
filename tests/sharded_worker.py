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
    if sys.argv[1] == "allreduce":
        return allreduce_check(rank, world, dev)
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
    dec.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok and routed_ok in (None, True) and status == 0 else 1


def allreduce_check(rank: int, world: int, dev) -> int:
    """pyrite_cuda_allreduce_sum against NCCL's allreduce on seeded partials:
    within fp32 summation-order rounding of it, bit-identical on every rank,
    over many calls in a row (alternating slots, growing flags) and inside a
    replayed CUDA graph."""
    import ctypes

    import torch
    import torch.distributed as dist

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    from pyrite_b200.kernels.cuda import _check
    lib = _lib.require()
    n = 4096
    ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
    size = int(lib.pyrite_cuda_allreduce_buffer_size(n))
    _check(lib.pyrite_cuda_ipc_buffer_create(size, ctypes.byref(ptr), handle), "c")
    handles = [None] * world
    dist.all_gather_object(handles, bytes(handle))
    ptrs, opened = [], []
    for r, hb in enumerate(handles):
        if r == rank:
            ptrs.append(ptr.value)
        else:
            p = ctypes.c_void_p()
            _check(lib.pyrite_cuda_ipc_buffer_open(hb, ctypes.byref(p)), "open")
            opened.append(p.value)
            ptrs.append(p.value)
    peers = torch.tensor(ptrs, dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    dist.barrier()
    ok, worst = True, 0.0
    s = torch.cuda.current_stream(dev)
    for it in range(20):
        g = torch.Generator(device=dev).manual_seed(1000 * it + rank)
        part = torch.randn(n, device=dev, generator=g)
        base = torch.full((n,), float(it), device=dev)
        out = base.clone()
        assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), n, peers.data_ptr(), size, world, rank,
                                             epoch.data_ptr(), s.cuda_stream) == 0
        ref = part.clone()
        dist.all_reduce(ref)
        torch.cuda.synchronize(dev)
        worst = max(worst, float((out - (base + ref)).abs().max()))
        everyone = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(everyone, out)
        ok &= all(torch.equal(everyone[0], o) for o in everyone)
    # the same call replayed from a CUDA graph
    part = torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(7 + rank))
    out = torch.zeros(n, device=dev)
    side = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(side):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), n, peers.data_ptr(), size, world, rank,
                                                 epoch.data_ptr(), side.cuda_stream) == 0
    torch.cuda.synchronize(dev)
    dist.barrier()
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize(dev)
    ref = part.clone()
    dist.all_reduce(ref)
    torch.cuda.synchronize(dev)
    worst = max(worst, float((out - 5 * ref).abs().max()) / 5)
    # time per call: 100 calls in one graph, ours against NCCL's
    timing = {}
    for name in ("nvlink", "nccl"):
        with torch.cuda.stream(side):
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=side):
                for _ in range(100):
                    if name == "nvlink":
                        assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), n, peers.data_ptr(),
                                                             size, world, rank, epoch.data_ptr(), side.cuda_stream) == 0
                    else:
                        dist.all_reduce(part)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            g2.replay()
            e0.record(side)
            g2.replay()
            e1.record(side)
        torch.cuda.synchronize(dev)
        timing[name + "_us_per_call"] = round(e0.elapsed_time(e1) * 10.0, 2)
        del g2
        torch.cuda.synchronize(dev)
        dist.barrier()
    status = K.status()
    del graph
    dist.barrier()
    for p in opened:
        lib.pyrite_cuda_ipc_buffer_close(p, 0)
    dist.barrier()
    lib.pyrite_cuda_ipc_buffer_close(ptr.value, 1)
    good = ok and worst <= 1e-5 and status == 0
    if rank == 0:
        print(json.dumps({"world": world, "identical_on_ranks": ok, "max_abs_diff_vs_nccl": worst, "status": status,
                          "allreduce_ok": good, **timing}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if good else 1


if __name__ == "__main__":
    sys.exit(main())
