"""Expert-parallel batched decode on 2 GPUs vs single-GPU batched decode:
identical greedy ids for every row, and one MoE block's output rows equal bit
for bit, over NCCL and over the NVLink peer-memory exchange (GPU; needs 2
GPUs)."""

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


def _moe_inputs(cfg, dev):
    g = torch.Generator(device="cpu").manual_seed(SEED + 11)
    x = (torch.randn(B, cfg["hidden_size"], generator=g) * 0.5).to(torch.bfloat16).to(dev)
    res = torch.randn(B, cfg["hidden_size"], generator=g).to(torch.bfloat16).to(dev)
    return x, res


def _reference_moe(dev):
    """Layer 0's MoE block (+ residual) over all B rows on one GPU."""
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_weights

    cfg = _cfg()
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, SEED, dev), device=dev)
    x, res = _moe_inputs(cfg, dev)
    with torch.inference_mode():
        return model.layers[0].mlp(x, residual=res).cpu()


def _worker(rank, world, port, q, transport, mode="decode"):
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
        if mode == "moe":
            x, res = _moe_inputs(cfg, dev)
            with torch.inference_mode():
                out = model.layers[0].mlp(x[t0:t0 + T].contiguous(), residual=res[t0:t0 + T].contiguous())
            torch.cuda.synchronize(dev)
            if transport == "p2p":
                ex.close()
            q.put((rank, out.cpu()))
            return
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


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_ep_moe_block_bit_exact(cuda, transport):
    """One expert-parallel MoE block (dispatch, local experts, combine with the
    residual) gives the single-GPU block's rows bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ref = _reference_moe(cuda)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, transport, "moe")) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out = torch.cat([got[0], got[1]])
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
