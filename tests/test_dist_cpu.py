"""The multi-GPU partitions on CPU ranks (gloo, world size 2 or 4): each rank runs
the oracle on its tensor-parallel slice (intermediate split), its expert-parallel
window, or both (bench.py's TP x EP2 map for config 4), the partial outputs meet
in an all-reduce, and the sum equals the unpartitioned layer. This checks the partition arithmetic the GPU path uses
(megamoe.shard, forward(partial=True) + all_reduce + finalize_partial) with no
GPU involved."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, queue):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "sgl-nvidia-mega_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from megamoe import shard
        from oracle import oracle as O

        H, I, E, K, T = 512, 256, 8, 2, 5
        layer = O.make_layer(H, I, E, shared=True, seed=3)
        x, _, _ = O.make_inputs(T, H, E, seed=3, router=False)
        g = torch.Generator().manual_seed(3)
        ids = np.stack([torch.randperm(E, generator=g)[:K].numpy() for _ in range(T)]).astype(np.int32)
        w = torch.rand((T, K), generator=g).numpy()
        full, _, _ = O.moe_layer(x, ids, w, layer)
        if mode == "tpxep":  # bench.partition for 4 ranks: TP2 x EP2 (config 4's 2-D split)
            import bench

            tp, ep = bench.partition(world, "nvfp4")
            assert (tp, ep) == (2, 2)
            ep_rank, tp_rank = rank // tp, rank % tp
            offset, local = shard.ep_window(E, ep_rank, ep)
            win = [t[offset:offset + local] for t in (layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"])]
            part = dict(layer)
            part["w13"], part["w13_scale"], part["w2"], part["w2_scale"] = shard.tp_slice(*win, tp_rank, tp)
            # the shared expert lives in EP group 0, TP-split across its ranks
            part["shared"] = shard.tp_slice(*layer["shared"], tp_rank, tp) if ep_rank == 0 else None
            out, _, _ = O.moe_layer(x, ids, w, part, expert_offset=offset, local_experts=local)
        elif mode == "tp":
            part = dict(layer)
            part["w13"], part["w13_scale"], part["w2"], part["w2_scale"] = shard.tp_slice(
                layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"], rank, world)
            part["shared"] = shard.tp_slice(*layer["shared"], rank, world)
            out, _, _ = O.moe_layer(x, ids, w, part)
        else:
            offset, local = shard.ep_window(E, rank, world)
            part = dict(layer)
            part["w13"], part["w13_scale"], part["w2"], part["w2_scale"] = shard.ep_slice(
                [layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"]], rank, world)
            if rank != 0:
                part["shared"] = None  # the shared expert counted once
            out, _, _ = O.moe_layer(x, ids, w, part, expert_offset=offset, local_experts=local)
        dist.all_reduce(out)
        if rank == 0:
            err = float((out - full).abs().max() / full.abs().max())
            queue.put(err)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,world", [("tp", 2), ("ep", 2), ("tpxep", 4)])
def test_partitions_sum_to_the_full_layer(mode, world):
    from oracle import oracle as O

    O.build()  # compile the C oracle once, before the ranks import it
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = queue.get(timeout=5)
    assert err < 1e-5, err
