"""Bounded device waits that run out: the launch ends, the error word reports a
timeout, later waits of the launch give up at once, and the objects work again.

The reference's remote waits carry deadlines too (common/sync.py:157-185,
all_reduce_mhc.py:917-924) but trap the GPU when one expires; here an expired
wait sets the layer's (or comm's) error word and the launch returns. Each test
makes a wait run out on a flag that nothing sets, with a short budget; nothing
is injected on the device and no kernel is left waiting without a bound:

  * the expert kernel's gate_up -> down mailboxes re-armed out of reach
    (``block_downs``): the down units' activation loads wait, time out, and the
    launch drains its copies and MMAs and frees its TMEM before it ends;
  * a combine + all-reduce of a group of two ranks of which only one calls:
    its poll of the absent rank's partial times out."""

import time

import numpy as np
import pytest
import torch

import oracle.oracle as O

pytestmark = pytest.mark.gpu

BUDGET_US = 5000  # 5 ms


def _layer_and_step(H=1024, I=256, E=32, K=8, T=8, seed=3):
    import megamoe

    layer = O.make_layer(H, I, E, shared=True, seed=seed)
    x, wr, bias = O.make_inputs(T, H, E, seed=seed)
    dev = torch.device("cuda", 0)
    moe = megamoe.RoutedMoE(*(layer[k].to(dev) for k in ("w13", "w13_scale", "w2", "w2_scale")), K, 16,
                            shared=[t.to(dev) for t in layer["shared"]])
    return moe, x.to(dev), wr.to(dev), bias.to(dev)


def test_expert_kernel_wait_runs_out_and_the_layer_recovers():
    from megamoe import _lib

    moe, x, wr, bias = _layer_and_step()
    bufs = {}
    want = moe.forward(x, router_weight=wr, bias=bias, routed_scaling_factor=2.5, buffers=bufs).clone()
    moe.check()
    T = x.size(0)
    moe.set_wait_budget(BUDGET_US)
    for attempt in range(2):  # the layer times out again after a timeout
        moe.block_downs()
        t0 = time.perf_counter()
        moe.rerun_experts(T, bufs["record"], bufs["rows"], rearm=False)
        with pytest.raises(_lib.DeviceTimeoutError):
            moe.check()
        elapsed = time.perf_counter() - t0
        # the budget (5 ms) plus the teardown drains (20 ms at most per stage):
        # far below the default 1.5 s budget
        assert elapsed < 1.0, (attempt, elapsed)
    moe.check()  # the word was cleared by the check that reported it
    # the next front pass re-arms the tables: the layer computes the same output
    moe.set_wait_budget(1_500_000)
    got = moe.forward(x, router_weight=wr, bias=bias, routed_scaling_factor=2.5, buffers=bufs)
    moe.check()
    assert torch.equal(got, want)
    # and the relaunch hook works again after a normal re-arm
    moe.rerun_experts(T, bufs["record"], bufs["rows"])
    moe.check()


def test_wait_budget_bounds():
    moe, _, _, _ = _layer_and_step()
    for bad in (0, -5, 60_000_001):
        with pytest.raises(ValueError):
            moe.set_wait_budget(bad)
    moe.set_wait_budget(1)
    moe.set_wait_budget(60_000_000)


def test_peer_poll_runs_out_when_a_rank_never_arrives():
    """Two ranks of one group on one GPU (a local group: each reaches the
    other's mailbox directly); only rank 0 calls. Its partial goes into rank
    1's mailbox, its poll of rank 1's partial runs out, and check() reports
    the timeout. A rebuilt group (of one) then gives the oracle's combine."""
    import megamoe
    from megamoe import _lib

    H, K, P, T = 1024, 8, 64, 4
    g = torch.Generator().manual_seed(1)
    rows = torch.randn((P, H), generator=g).to(torch.bfloat16).cuda()
    w = torch.rand((T, K), generator=g).cuda()
    perm = torch.randint(-1, P, (T, K), generator=g).int().cuda()
    shared = torch.randn((T, H), generator=g).to(torch.bfloat16).cuda()
    pair = megamoe.PeerAllReduce.local_group(8, H, ["cuda:0", "cuda:0"])
    pair[0].set_wait_budget(BUDGET_US)
    t0 = time.perf_counter()
    pair[0].finalize(rows, w, perm, shared)
    with pytest.raises(_lib.DeviceTimeoutError):
        pair[0].check()
    assert time.perf_counter() - t0 < 1.0
    res = torch.randn((T, H), generator=g).to(torch.bfloat16).cuda()
    gamma = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    pair[0].moe_finalize_all_reduce_rms_norm(routed_output=rows, expert_weights=w, permuted_indices=perm,
                                             gated_shared_output=shared, residual=res, gamma=gamma)
    with pytest.raises(_lib.DeviceTimeoutError):  # the hop's poll (clusters of CTAs) ends the same way
        pair[0].check()
    pair[1].check()  # rank 1 never launched: nothing to report
    for m in pair:
        m.close()
    solo = megamoe.PeerAllReduce(8, H)
    out = solo.finalize(rows, w, perm, shared)
    solo.check()
    want = O.allreduce_ranks([O.finalize(O.bf16_bits(rows.cpu()), w.cpu().numpy(), perm.cpu().numpy(),
                                         O.bf16_bits(shared.cpu()))])
    assert np.array_equal(O.bf16_bits(out.cpu()), want)
    solo.close()
