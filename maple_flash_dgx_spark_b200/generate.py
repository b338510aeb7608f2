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


def resolve_max_tokens(max_tokens: int, prompt_len: int, max_context: int) -> int:
    """A request's token cap within the context left after its prompt; -1
    means no cap of its own (reference generate.py:31-38)."""
    remaining = max(int(max_context) - int(prompt_len), 0)
    if max_tokens == -1:
        return remaining
    if max_tokens < 0:
        raise ValueError("max_tokens must be >= 0 or -1")
    return min(int(max_tokens), remaining)


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


def stop_token_ids(model, tokenizer=None) -> set[int]:
    """Token ids that end a response (reference generate.py:427-433)."""
    ids: set[int] = set()
    for src in (getattr(model, "eos_token_id", None),
                getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None,
                getattr(tokenizer, "pad_token_id", None) if tokenizer is not None else None):
        if src is None:
            continue
        ids |= {int(t) for t in (src if isinstance(src, (list, tuple, set)) else [src])}
    return ids


class BucketedDecodeGraphs:
    """One decode graph per batch width, replayed at the narrowest width that
    fits the live rows (reference generate.py:703-816).  All widths share the
    token / uniform buffers.  Rows past the live count are padding: they run
    against the cache rows above the live ones, so the caller keeps live
    sequences in the low slots (``KVCache.swap_slots``); the graphs read the
    slot -> cache-row map, so compaction needs no re-capture."""

    def __init__(self, model, cache, *, widths: tuple[int, ...], sample: tuple | None = None,
                 log: Callable[[str], None] | None = _log_print):
        if not cache.remap:
            raise ValueError("BucketedDecodeGraphs needs cache.remap enabled.")
        dev = model.device
        self.widths = tuple(sorted(set(int(w) for w in widths)))
        self.max_width = self.widths[-1]
        if self.max_width > cache.batch:
            raise ValueError(f"widest graph {self.max_width} exceeds the cache batch {cache.batch}.")
        self.sample = sample
        self.token_ids = torch.zeros(self.max_width, 1, dtype=torch.long, device=dev)
        self.uniform = torch.zeros(self.max_width, dtype=torch.float32, device=dev)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.next_id: dict[int, torch.Tensor] = {}
        self.logits: dict[int, torch.Tensor] = {}
        snap = _length_snapshot(cache)
        stream = torch.cuda.Stream(dev)
        try:
            for w in self.widths:
                stream.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(stream):
                    for _ in range(_GRAPH_WARMUP):
                        self._step(model, cache, w)
                        _length_restore(cache, snap)
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=stream):
                        self.logits[w], self.next_id[w] = self._step(model, cache, w)
                torch.cuda.current_stream(dev).wait_stream(stream)
                torch.cuda.synchronize(dev)
                _length_restore(cache, snap)
                self.graphs[w] = graph
        finally:
            _length_restore(cache, snap)
        if log is not None:
            log(f"Bucketed decode graphs: widths {list(self.widths)}"
                + (" with fused sampler" if sample is not None else " greedy"))

    def _step(self, model, cache, w: int):
        logits = model.forward(self.token_ids[:w], cache=cache, logits_to_keep=1)
        last = logits[:, -1, :]
        if self.sample is None:
            nxt = argmax(last)
        else:
            ws, temperature, top_p, top_k = self.sample
            nxt = fused_sample_batched(last, self.uniform[:w], temperature=temperature, top_p=top_p, top_k=top_k,
                                       workspace=ws)
        return logits, nxt

    def width_for(self, live: int) -> int:
        for w in self.widths:
            if w >= live:
                return w
        raise ValueError(f"live batch {live} exceeds widest graph {self.max_width}.")

    def _load(self, tokens, uniform):
        live = int(tokens.shape[0])
        w = self.width_for(live)
        self.token_ids[:live].copy_(tokens.reshape(live, 1))
        if live < w:
            self.token_ids[live:w].zero_()
        if uniform is not None:
            self.uniform[:live].copy_(uniform.reshape(-1)[:live])
        return live, w

    def replay(self, tokens: torch.Tensor, uniform: torch.Tensor | None = None) -> torch.Tensor:
        """Step ``tokens`` ``[live, 1]``; returns the next ids ``[live]``."""
        live, w = self._load(tokens, uniform)
        self.graphs[w].replay()
        return self.next_id[w][:live]

    def replay_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Step ``tokens``; returns last-token logits ``[live, vocab]``."""
        live, w = self._load(tokens, None)
        self.graphs[w].replay()
        return self.logits[w][:live].reshape(live, -1)


@dataclass
class BatchedResult:
    """Per-row token ids plus timings (reference generate.py:819-840)."""

    token_ids: list[list[int]]
    prompt_lens: list[int]
    finish_reasons: list[str]
    prefill_s: float
    decode_s: float
    steps: int
    widths: list[int] = field(default_factory=list)

    @property
    def n_new(self) -> int:
        return sum(len(t) for t in self.token_ids)

    @property
    def decode_tok_s(self) -> float:
        return self.n_new / self.decode_s if self.decode_s > 0 else 0.0


def _first_id(logits, greedy, temperature, top_p, top_k, gen):
    last = logits[0, -1]
    if greedy:
        return argmax(last)
    return fused_sample(last, torch.rand((), device=last.device, generator=gen), temperature=temperature,
                        top_p=top_p, top_k=top_k)


def _try_batched_decode_graphs(model, cache, pending: list[int], *, sample, buckets=None,
                               log: Callable[[str], None] | None = _log_print):
    """Capture the bucketed graphs; keep them only if one replay at the full
    width gives the eager step's ids (reference generate.py:1045-1104)."""
    widths = tuple(buckets) if buckets else decode_buckets(cache.batch)
    try:
        runner = BucketedDecodeGraphs(model, cache, widths=widths, sample=sample, log=log)
    except Exception as exc:  # capture is an optimisation; eager decode stays correct
        if log is not None:
            log(f"CUDA graph capture failed ({exc}); using eager decode")
        return None
    live = len(pending)
    tokens = torch.tensor(pending, device=model.device, dtype=torch.long).view(live, 1)
    u = torch.rand(live, device=model.device) if sample is not None else None
    snap = _length_snapshot(cache)
    last = model.forward(tokens, cache=cache, logits_to_keep=1)[:, -1, :]
    if sample is None:
        eager = argmax(last)
    else:
        ws, temperature, top_p, top_k = sample
        eager = fused_sample_batched(last, u, temperature=temperature, top_p=top_p, top_k=top_k, workspace=ws)
    eager = eager.tolist()
    _length_restore(cache, snap)
    graph = runner.replay(tokens, u).tolist()
    _length_restore(cache, snap)
    if eager != graph:
        if log is not None:
            log(f"CUDA graph replay diverged (eager {eager[:8]} vs graph {graph[:8]}); using eager decode")
        return None
    return runner


@torch.inference_mode()
def batched_generate(model, prompts, *, max_tokens: int = 128, max_new: list[int] | None = None,
                     temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, seed: int | None = None,
                     stop_ids: set[int] | None = None, cache=None, graphs: bool = False,
                     buckets: tuple[int, ...] | None = None, runner: BucketedDecodeGraphs | None = None,
                     log: Callable[[str], None] | None = _log_print) -> BatchedResult:
    """Decode several sequences in one batch (reference generate.py:842-1028).

    Each prompt is prefilled into its own cache slot; decode goes wide, so the
    batched GEMMs read every weight once per step for all rows.  Finished
    rows are swapped out of the low slots; with ``graphs`` each step replays
    the narrowest captured width that holds the live rows."""
    dev = model.device
    rows = [torch.as_tensor(p, device=dev, dtype=torch.long).reshape(-1) for p in prompts]
    if not rows:
        raise ValueError("batched_generate needs at least one prompt.")
    bsz = len(rows)
    prompt_lens = [int(t.numel()) for t in rows]
    if max_new is None:
        caps = [int(max_tokens)] * bsz
    else:
        if len(max_new) != bsz:
            raise ValueError(f"max_new length {len(max_new)} != {bsz} prompts.")
        caps = [int(c) for c in max_new]
        if any(c < 1 for c in caps):
            raise ValueError("each max_new row must be >= 1")
    horizon = max(caps)
    if stop_ids is None:
        stop_ids = stop_token_ids(model)
    need = max(prompt_lens) + max(horizon, 1)
    if cache is None:
        cache = model.make_cache(max_len=need, batch=bsz)
    elif cache.batch < bsz:
        raise ValueError(f"cache batch {cache.batch} < {bsz} prompts.")
    elif cache.max_len < need:
        raise ValueError(f"cache max_len {cache.max_len} < longest prompt {max(prompt_lens)} + {horizon} tokens.")
    else:
        cache.reset_identity()
    greedy = is_greedy(temperature, top_k)
    if not greedy and not can_fuse_sampler(temperature, top_p, top_k):
        raise ValueError(f"batched decode needs 0 < top_k <= {MAX_TOP_K} and 0 < top_p <= 1.")
    gen = None
    if seed is not None:
        gen = torch.Generator(device=dev)
        gen.manual_seed(int(seed))

    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    pending = [0] * bsz
    for b, row in enumerate(rows):
        with cache.prefill_slot(b):
            logits = model.forward(row.view(1, -1), cache=cache, logits_to_keep=1)
        pending[b] = int(_first_id(logits, greedy, temperature, top_p, top_k, gen))
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0

    cache.remap = True
    sample_ws = None
    if not greedy:
        sample_ws = batched_sampler_workspace(model.vocab_size, int(top_k), cache.batch, dev)
    if graphs and runner is None:
        runner = _try_batched_decode_graphs(model, cache, pending,
                                            sample=None if greedy else (sample_ws, temperature, top_p, top_k),
                                            buckets=buckets, log=log)

    def step(tokens):
        live = int(tokens.shape[0])
        u = None if greedy else torch.rand(live, device=dev, generator=gen)
        if runner is not None:
            return runner.replay(tokens, u)
        last = model.forward(tokens, cache=cache, logits_to_keep=1)[:, -1, :]
        if greedy:
            return argmax(last)
        return fused_sample_batched(last, u, temperature=temperature, top_p=top_p, top_k=top_k, workspace=sample_ws)

    out: list[list[int]] = [[] for _ in range(bsz)]
    reasons = ["length"] * bsz
    owner = list(range(bsz))  # slot -> output row
    live, steps = bsz, 0
    widths: list[int] = []
    t0 = time.perf_counter()
    for i in range(int(horizon)):
        finished = []
        for slot in range(live):
            b = owner[slot]
            out[b].append(pending[slot])
            if pending[slot] in stop_ids:
                reasons[b] = "stop"
                finished.append(slot)
            elif len(out[b]) >= caps[b]:
                reasons[b] = "length"
                finished.append(slot)
        if i + 1 >= int(horizon):
            break
        for slot in reversed(finished):  # descending: a slot pulled down was never retired here
            last_slot = live - 1
            if slot != last_slot:
                cache.swap_slots(slot, last_slot)
                owner[slot], owner[last_slot] = owner[last_slot], owner[slot]
                pending[slot], pending[last_slot] = pending[last_slot], pending[slot]
            live -= 1
        if live == 0:
            break
        tokens = torch.tensor(pending[:live], device=dev, dtype=torch.long).view(live, 1)
        nxt = step(tokens)
        pending[:live] = [int(x) for x in nxt.tolist()]
        steps += 1
        if runner is not None:
            width = runner.width_for(live)
            widths.append(width)
            cache.advance_host(1, width)
    torch.cuda.synchronize(dev)
    decode_s = time.perf_counter() - t0
    return BatchedResult(out, prompt_lens, reasons, prefill_s, decode_s, steps, widths)
