"""Two-GPU parity: the layer split tensor-parallel on the intermediate, or
expert-parallel by expert windows, over two ranks; each rank runs the chain on its
part. Two combines: (1) forward(partial=True), the fp32 partial sums meet in an
NCCL all-reduce and finalize_partial rounds them; (2) forward(comm=PeerAllReduce),
the combine fused with the all-reduce over NVLink peer memory, which must equal
bit for bit the oracle's rank-order sum of every rank's combine of its own rows.
Both must match the fp32 oracle of the whole layer within BASELINE's bar.
Skipped with fewer than two GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, peer, queue):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "sgl-nvidia-mega_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import megamoe
        from megamoe import shard
        from oracle import oracle as O

        H, I, E, K, T = 1024, 512, 32, 8, 8
        layer = O.make_layer(H, I, E, shared=True, seed=9)
        x, wr, bias = O.make_inputs(T, H, E, seed=9)
        if mode == "tp":
            w = shard.tp_slice(layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"], rank, world)
            sh = shard.tp_slice(*layer["shared"], rank, world)
            moe = megamoe.RoutedMoE(*(t.to(dev) for t in w), K, 16, shared=[t.to(dev) for t in sh])
        else:
            offset, local = shard.ep_window(E, rank, world)
            w = shard.ep_slice([layer["w13"], layer["w13_scale"], layer["w2"], layer["w2_scale"]], rank, world)
            sh = [t.to(dev) for t in layer["shared"]] if rank == 0 else None
            moe = megamoe.RoutedMoE(*(t.to(dev) for t in w), K, 16, router_experts=E, expert_offset=offset,
                                    shared=sh)
        bufs = {}
        xg, wg, bg = x.to(dev), wr.to(dev), bias.to(dev)
        exact = True
        if not peer:
            part = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, partial=True, buffers=bufs)
            dist.all_reduce(part)
            out = megamoe.finalize_partial(part)
        else:
            comm = megamoe.PeerAllReduce(16, H)
            for _ in range(3):
                out = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs, comm=comm)
            torch.cuda.synchronize()
            shared = moe.shared_rows(bufs["rows"], T)
            mine = (O.bf16_bits(bufs["rows"].cpu()), bufs["weights"].cpu().numpy(), bufs["permuted"].cpu().numpy(),
                    None if shared is None else O.bf16_bits(shared.cpu()))
            every = [None] * world
            dist.all_gather_object(every, mine)
            want = O.allreduce_ranks([O.finalize(*r) for r in every])
            exact = bool(np.array_equal(O.bf16_bits(out.cpu()), want))
            # the decoder hop: residual + RMSNorm of the group sum, same launch
            gr = torch.Generator().manual_seed(31)
            res = torch.randn((T, H), generator=gr).to(torch.bfloat16)
            gamma = (1 + 0.1 * torch.randn(H, generator=gr)).to(torch.bfloat16)
            want_r, want_n = O.allreduce_norm([O.finalize(*r) for r in every], O.bf16_bits(res),
                                              O.bf16_bits(gamma), comm.eps)
            norm, r_out = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs,
                                      comm=comm, residual=res.to(dev), gamma=gamma.to(dev))
            exact = exact and bool(np.array_equal(O.bf16_bits(r_out.cpu()), want_r))
            exact = exact and bool(np.array_equal(O.bf16_bits(norm.cpu()), want_n))
            out = moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs, comm=comm)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                moe.forward(xg, router_weight=wg, bias=bg, routed_scaling_factor=2.5, buffers=bufs, comm=comm)
            first = out.clone()
            for _ in range(3):
                bufs["out"].zero_()
                graph.replay()
                torch.cuda.synchronize()
                exact = exact and torch.equal(bufs["out"], first)
            comm.check()
            del graph
            dist.barrier()
            comm.close()
        torch.cuda.synchronize()
        moe.check()
        if rank == 0:
            logits = O.router_gemv(O.bf16_bits(x), O.bf16_bits(wr))
            ow, oids = O.gate_topk(logits, bias.numpy(), K, scale=2.5)
            same_ids = bool(np.array_equal(bufs["ids"].cpu().numpy(), oids))
            ref, _, _ = O.moe_layer(x, oids, ow, layer)
            queue.put((same_ids, exact, O.max_abs_rel(out.float().cpu().numpy(), ref.numpy())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("peer", [False, True], ids=["nccl", "peer"])
@pytest.mark.parametrize("mode", ["tp", "ep"])
def test_two_gpu_partitions_match_the_oracle(mode, peer):
    from oracle import oracle as O

    O.build()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, peer, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same_ids, exact, err = queue.get(timeout=5)
    assert same_ids
    assert exact
    assert err <= 2e-2, err


def _stack_worker(rank, world, port, queue):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "sgl-nvidia-mega_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import megamoe
        from megamoe import shard
        from oracle import oracle as O

        n, H, I, E, K, T = 3, 1024, 256, 32, 8, 8
        g = torch.Generator().manual_seed(50)
        offset, local = shard.ep_window(E, rank, world)
        moes, routers, biases, gammas = [], [], [], []
        for i in range(n):
            L = O.make_layer(H, I, E, shared=False, seed=51 + i)
            w = shard.ep_slice([L["w13"], L["w13_scale"], L["w2"], L["w2_scale"]], rank, world)
            moes.append(megamoe.RoutedMoE(*(t.to(dev) for t in w), K, 16, router_experts=E, expert_offset=offset))
            routers.append(((torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16)).to(dev))
            biases.append(((torch.randn((E,), generator=g) * 0.01).float()).to(dev))
            gammas.append(((1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)).to(dev))
        x = torch.randn((T, H), generator=g).to(torch.bfloat16).to(dev)
        res0 = torch.randn((T, H), generator=g).to(torch.bfloat16).to(dev)
        comm = megamoe.PeerAllReduce(16, H)
        stack = megamoe.MoEStack(moes, routers, gammas, comm, biases=biases, routed_scaling_factor=2.5)
        r = res0.clone()
        out = stack.forward(x, r).clone()
        cur, rl = x, res0.clone()
        for i, m in enumerate(moes):
            cur, rl = m.forward(cur, router_weight=routers[i], bias=biases[i], routed_scaling_factor=2.5,
                                buffers={}, comm=comm, residual=rl, gamma=gammas[i])
            cur, rl = cur.clone(), rl.clone()
        torch.cuda.synchronize()
        stack.check()
        same_loop = bool(torch.equal(out, cur) and torch.equal(r, rl))
        every = [None] * world
        dist.all_gather_object(every, (O.bf16_bits(out.cpu()), O.bf16_bits(r.cpu())))
        same_ranks = all(np.array_equal(e[0], every[0][0]) and np.array_equal(e[1], every[0][1]) for e in every)
        finite = bool(torch.isfinite(out.float()).all())
        if rank == 0:
            queue.put((same_loop, same_ranks, finite))
        dist.barrier()
        comm.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_expert_parallel_stack():
    """Three MoE layers, EP2, chained through the fused hop: every rank's output
    and residual equal its own per-layer loop and are identical across ranks."""
    from oracle import oracle as O

    O.build()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stack_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same_loop, same_ranks, finite = queue.get(timeout=5)
    assert same_loop and same_ranks and finite
