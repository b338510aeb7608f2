"""Decode driver: prefill, a CUDA-graph decode step, and the token loop.

Reference: generate.py:91-120 (sample_next), :168-373 (decode graph capture and
the replay == eager gate), :703-816 (bucketed batch graphs), :842-1028
(batched_generate), :1107-1281 (run_generate).  Text-side pieces (chat
templates, think/tool parsing, detokenisation) are outside this engine: the
loop takes and returns token ids.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from dataclasses import dataclass, field

import torch

from maple_flash_dgx_spark_b200.kernels import (
    MAX_TOP_K,
    argmax,
    batched_sampler_workspace,
    fused_sample,
    fused_sample_batched,
)

DEFAULT_TEMPERATURE = 1.0
DEFAULT_TOP_P = 0.95
DEFAULT_TOP_K = 20
_GRAPH_WARMUP = 3
_GRAPH_CHECK_TOKENS = 8
_DECODE_BUCKETS = (1, 2, 4, 8, 16, 32)


def _log_print(msg: str) -> None:
    print(msg, flush=True)


def is_greedy(temperature: float, top_k: int) -> bool:
    """Reference generate.py:66-68."""
    return temperature <= 0.0 or top_k == 1


def can_fuse_sampler(temperature: float, top_p: float, top_k: int) -> bool:
    """Reference generate.py:71-77."""
    return not is_greedy(temperature, top_k) and 0 < top_k <= MAX_TOP_K and 0.0 < top_p <= 1.0


def sample_next(logits: torch.Tensor, *, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0,
                generator: torch.Generator | None = None) -> torch.Tensor:
    """Next token from 1-D logits (reference generate.py:91-120): argmax when
    greedy, else top-k / temperature / nucleus with one uniform from
    ``generator``.  Runs on the fused sampler (top_k 1..64)."""
    if is_greedy(temperature, top_k):
        return argmax(logits)
    if not can_fuse_sampler(temperature, top_p, top_k):
        raise ValueError(f"sampling needs 0 < top_k <= {MAX_TOP_K} and 0 < top_p <= 1.")
    u = torch.rand((), device=logits.device, generator=generator)
    return fused_sample(logits, u, temperature=temperature, top_p=top_p, top_k=top_k)


@dataclass
class GenerateResult:
    token_ids: list[int]
    prompt_len: int
    n_new: int
    prefill_s: float
    decode_s: float
    finish_reason: str = "length"
    used_graph: bool = False

    @property
    def decode_tok_s(self) -> float:
        return self.n_new / self.decode_s if self.decode_s > 0 else 0.0

    @property
    def prefill_tok_s(self) -> float:
        return self.prompt_len / self.prefill_s if self.prefill_s > 0 else 0.0


def _length_snapshot(cache):
    return cache.seqlen.clone(), list(cache.seen)


def _length_restore(cache, snap):
    cache.seqlen.copy_(snap[0])
    cache.seen = list(snap[1])


class DecodeGraph:
    """``forward(tokens)`` plus next-token selection for a fixed batch width,
    captured in one CUDA graph (reference generate.py:168-227, 703-816).

    Only lengths are snapshotted around warm-up and capture: the steps write
    K/V at positions >= each row's length, which attention never reads before
    the real tokens overwrite them, so the (possibly huge) cache is not
    copied."""

    def __init__(self, model, cache, *, width: int = 1, sample: tuple | None = None):
        dev = model.device
        self.width = width
        self.sample = sample
        self.token_ids = torch.zeros(width, 1, dtype=torch.long, device=dev)
        self.uniform = torch.zeros(width, dtype=torch.float32, device=dev)
        snap = _length_snapshot(cache)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            for _ in range(_GRAPH_WARMUP):
                self._step(model, cache)
                _length_restore(cache, snap)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self.logits, self.next_id = self._step(model, cache)
        torch.cuda.current_stream(dev).wait_stream(stream)
        torch.cuda.synchronize(dev)
        _length_restore(cache, snap)

    def _step(self, model, cache):
        logits = model.forward(self.token_ids, cache=cache, logits_to_keep=1)
        last = logits[:, -1, :]
        if self.sample is None:
            nxt = argmax(last)
        else:
            ws, temperature, top_p, top_k = self.sample
            nxt = fused_sample_batched(last, self.uniform, temperature=temperature, top_p=top_p, top_k=top_k,
                                       workspace=ws)
        return logits, nxt

    def replay(self, tokens: torch.Tensor | None = None, uniform: torch.Tensor | None = None) -> torch.Tensor:
        if tokens is not None:
            self.token_ids[: tokens.numel()].copy_(tokens.reshape(-1, 1), non_blocking=True)
        if uniform is not None:
            self.uniform[: uniform.numel()].copy_(uniform.reshape(-1), non_blocking=True)
        self.graph.replay()
        return self.next_id


@torch.inference_mode()
def run_generate(model, input_ids: torch.Tensor, *, max_tokens: int = 128, temperature: float = DEFAULT_TEMPERATURE,
                 top_p: float = DEFAULT_TOP_P, top_k: int = DEFAULT_TOP_K, seed: int | None = None,
                 use_graph: bool = True, stop_ids: set[int] | None = None,
                 log: Callable[[str], None] | None = _log_print) -> GenerateResult:
    """Prefill ``input_ids`` then decode up to ``max_tokens`` (reference generate.py:1107-1281).

    Each step copies the new id to pinned host memory and waits on an event,
    as the reference loop does (the host needs every id for stop checks)."""
    dev = model.device
    if input_ids.dim() == 1:
        input_ids = input_ids.unsqueeze(0)
    input_ids = input_ids.to(dev).long()
    prompt_len = int(input_ids.shape[-1])
    greedy = is_greedy(temperature, top_k)
    if not greedy and not can_fuse_sampler(temperature, top_p, top_k):
        raise ValueError(f"sampling needs 0 < top_k <= {MAX_TOP_K} and 0 < top_p <= 1.")
    gen = None
    if seed is not None and not greedy:
        gen = torch.Generator(device=dev)
        gen.manual_seed(int(seed))
    stop_ids = stop_ids or set()
    cache = model.make_cache(max_len=prompt_len + max(max_tokens, 1))
    sample = None if greedy else (batched_sampler_workspace(model.vocab_size, top_k, 1, dev)[0], temperature, top_p,
                                  top_k)

    def pick(logits):
        last = logits[:, -1, :]
        if greedy:
            return argmax(last)
        u = torch.rand(1, device=dev, generator=gen)
        return fused_sample_batched(last, u, temperature=temperature, top_p=top_p, top_k=top_k, workspace=sample[0])

    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    logits = model.forward(input_ids, cache=cache, logits_to_keep=1)
    next_t = pick(logits)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    graph = DecodeGraph(model, cache, width=1, sample=sample) if (use_graph and max_tokens > 1) else None
    pinned = torch.empty(1, dtype=torch.long, pin_memory=True)
    ready = torch.cuda.Event()
    torch.cuda.synchronize(dev)
    t2 = time.perf_counter()
    out: list[int] = []
    reason = "length"
    for i in range(max_tokens):
        pinned.copy_(next_t.reshape(1), non_blocking=True)
        ready.record()
        if i + 1 < max_tokens:
            if graph is not None:
                u = None if greedy else torch.rand(1, device=dev, generator=gen)
                next_t = graph.replay(next_t, u)
            else:
                next_t = pick(model.forward(next_t.reshape(1, 1), cache=cache, logits_to_keep=1))
        ready.synchronize()
        tok = int(pinned[0])
        out.append(tok)
        if tok in stop_ids:
            reason = "stop"
            break
    torch.cuda.synchronize(dev)
    t3 = time.perf_counter()
    res = GenerateResult(out, prompt_len, len(out), t1 - t0, t3 - t2, reason, graph is not None)
    if log is not None:
        log(f"Prefill: {prompt_len} tok in {res.prefill_s:.3f}s; decode: {res.n_new} tok in {res.decode_s:.3f}s "
            f"({res.decode_tok_s:.1f} tok/s, graph={graph is not None})")
    return res


def decode_buckets(max_batch: int, buckets=_DECODE_BUCKETS) -> tuple[int, ...]:
    """Graph widths for a cache of ``max_batch`` rows (reference generate.py:687-700)."""
    widths = [w for w in buckets if w < max_batch]
    widths.append(int(max_batch))
    return tuple(sorted(set(widths)))
