"""Expert-parallel exchange on CPU ranks (gloo, world size 2 and 4).

The product's EPExchange (dispatch all-gather, combine all-to-all) moves
real tensors between processes; the expert math in between is the CPU
oracle restricted to each rank's experts, and the owner-select + weighted sum
is what ep_combine computes.  The expert-parallel result of every token must
equal the single-process MoE block bit for bit.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tests.helpers import alpha_bf, bf, randn_bf, tern_packed

B, H, E, TOPK, INTER = 8, 128, 8, 2, 64


def _problem():
    rs = np.random.RandomState(0)
    x = randn_bf(rs, B, H)
    ids = np.stack([rs.permutation(E)[:TOPK] for _ in range(B)]).astype(np.int32)
    w = rs.random_sample((B, TOPK)).astype(np.float32)
    res = randn_bf(rs, B, H)
    up = tern_packed(rs, E, 2 * INTER, H)
    up_a = bf(alpha_bf(rs, E, 2 * INTER) * 20)
    down = tern_packed(rs, E, H, INTER)
    down_a = alpha_bf(rs, E, H)
    return x, ids, w, res, up, up_a, down, down_a


def _single():
    x, ids, w, res, up, up_a, down, down_a = _problem()
    h = oracle.expert_swiglu(x, up, up_a, ids)
    y = oracle.expert_gemv(h.reshape(-1, INTER), down, down_a, ids, x_rows_per_token=1)
    return oracle.moe_reduce_add(y.reshape(B, TOPK, H), w, res)


def _worker(rank, world, port, out):
    from maple_flash_dgx_spark_b200.expert_parallel import EPExchange, expert_range, token_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, ids, w, res, up, up_a, down, down_a = _problem()
        ex = EPExchange(None, rank, world, E)
        t0, T = token_range(B, rank, world)
        x_all, ids_all = ex.dispatch(torch.from_numpy(x[t0:t0 + T]), torch.from_numpy(ids[t0:t0 + T]))
        assert torch.equal(x_all.contiguous(), torch.from_numpy(x)) and torch.equal(ids_all, torch.from_numpy(ids))
        # this rank's experts only; other ranks' slots hold NaN and must never be read
        e0, nl = expert_range(E, rank, world)
        ia = ids_all.numpy()
        local = (ia >= e0) & (ia < e0 + nl)
        h = oracle.expert_swiglu(x_all.contiguous().numpy(), up, up_a, ia)
        y = oracle.expert_gemv(h.reshape(-1, INTER), down, down_a, ia, x_rows_per_token=1)
        y[~local.reshape(-1)] = np.nan
        recv = ex.combine_exchange(torch.from_numpy(y)).numpy()  # [W, T*k, H]
        mine = ids[t0:t0 + T]
        owner = mine // (E // world)
        sel = np.stack([recv[owner[t, j], t * TOPK + j] for t in range(T) for j in range(TOPK)])
        o = oracle.moe_reduce_add(sel.reshape(T, TOPK, H), w[t0:t0 + T], res[t0:t0 + T])
        out[rank] = o
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_equals_single_process(world):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
        got = np.concatenate([out[r] for r in range(world)])
    np.testing.assert_array_equal(got, _single())


def test_shard_and_ranges():
    from maple_flash_dgx_spark_b200.expert_parallel import expert_range, shard_expert_weights, token_range

    assert expert_range(64, 3, 8) == (24, 8)
    assert token_range(64, 7, 8) == (56, 8)
    with pytest.raises(ValueError):
        expert_range(64, 0, 3)
    cfg = {"num_experts": 4}
    wts = {"model.layers.0.mlp.switch_mlp.up_proj.weight": torch.arange(4 * 3).reshape(4, 3),
           "model.layers.0.mlp.switch_mlp.down_proj.row_alpha": torch.arange(4 * 2).reshape(4, 2),
           "model.layers.0.mlp.gate.weight": torch.zeros(4, 5)}
    s = shard_expert_weights(wts, cfg, 1, 2)
    assert torch.equal(s["model.layers.0.mlp.switch_mlp.up_proj.weight"], wts[
        "model.layers.0.mlp.switch_mlp.up_proj.weight"][2:4])
    assert s["model.layers.0.mlp.gate.weight"].shape == (4, 5)
