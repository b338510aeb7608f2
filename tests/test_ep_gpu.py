"""Expert-parallel batched decode on 2 GPUs (NCCL) vs single-GPU batched
decode: identical greedy ids for every row (GPU; needs 2 GPUs)."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

B, CTX, STEPS, SEED = 8, 40, 6, 3


def _cfg():
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    return synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2, inter=128,
                            vocab=1024)


def _reference_ids(dev):
    """Single-GPU batched greedy decode of all B rows."""
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import fill_kv_cache, synthetic_tokens, synthetic_weights

    cfg = _cfg()
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, SEED, dev), device=dev)
    cache = model.make_cache(max_len=CTX + STEPS + 2, batch=B)
    fill_kv_cache(cache, SEED, CTX)
    tok = synthetic_tokens(SEED, B, cfg["vocab_size"], dev).reshape(B, 1)
    out = []
    with torch.inference_mode():
        for _ in range(STEPS):
            tok = model.forward(tok, cache=cache)[:, -1].argmax(-1).reshape(B, 1)
            out.append(tok.reshape(-1).cpu())
    return torch.stack(out, 1)


def _worker(rank, world, port, q, transport):
    import datetime

    import torch.distributed as dist

    from maple_flash_dgx_spark_b200.expert_parallel import (EPDecodeGraph, EPDecoder, EPExchange, EPExchangeP2P,
                                                            shard_expert_weights, token_range)
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import fill_kv_cache, synthetic_tokens, synthetic_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = _cfg()
        t0, T = token_range(B, rank, world)
        if transport == "p2p":
            ex = EPExchangeP2P(None, rank, world, cfg["num_experts"], tokens=T, hidden=cfg["hidden_size"],
                               topk=cfg["num_experts_per_tok"], device=dev)
        else:
            ex = EPExchange(None, rank, world, cfg["num_experts"])
        w = shard_expert_weights(synthetic_weights(cfg, SEED, dev), cfg, rank, world)
        model = MapleForCausalLM.from_weight_dict(cfg, w, device=dev)
        cache = model.make_cache(max_len=CTX + STEPS + 2, batch=T)
        fill_kv_cache(cache, SEED, CTX, row0=t0, total_rows=B)
        tok = synthetic_tokens(SEED, B, cfg["vocab_size"], dev)[t0:t0 + T].reshape(T, 1)
        dec = EPDecoder(model, ex)
        ids = []
        with torch.inference_mode():
            for _ in range(STEPS // 2):
                tok = dec.step(tok, cache).reshape(T, 1)
                ids.append(tok.reshape(-1).cpu())
            g = EPDecodeGraph(dec, cache, T)
            for _ in range(STEPS - STEPS // 2):
                tok = g.replay(tok).reshape(T, 1).clone()
                cache.advance_host(1, T)
                ids.append(tok.reshape(-1).cpu())
            del g
        from maple_flash_dgx_spark_b200 import _lib

        assert int(_lib.error_word(dev).item()) == 0, "a bounded peer wait gave up"
        if transport == "p2p":
            ex.close()
        q.put((rank, torch.stack(ids, 1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_ep_decode_equals_single_gpu(cuda, transport):
    """NCCL collectives, and the NVLink peer-store exchange kernels."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ref = _reference_ids(cuda)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, transport)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.testing.assert_close(torch.cat([got[0], got[1]]), ref, rtol=0, atol=0)
