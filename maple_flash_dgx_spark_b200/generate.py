"""Decode driver: prefill, a CUDA-graph decode step, and the token loop.

Reference: generate.py:91-120 (sample_next), :168-373 (decode graph capture and
the replay == eager gate), :703-816 (bucketed batch graphs), :842-1028
(batched_generate), :1107-1281 (run_generate): same entry points, arguments
and results; the batched driver and graph ladder are this engine's own
(per-row records, two-cursor slot compaction, a logits-level replay gate).  Text-side pieces (chat
templates, think/tool parsing, detokenisation) are outside this engine: the
loop takes and returns token ids.
"""

from __future__ import annotations

import bisect
import time
from collections.abc import Callable
from dataclasses import dataclass, field

import torch

from maple_flash_dgx_spark_b200._lib import raise_device_errors
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
    captured in one CUDA graph (reference generate.py:168-227).

    ``tokens`` / ``uniform`` may be buffers shared with graphs of other widths
    (the first ``width`` entries are this graph's inputs).  Only lengths are
    snapshotted around warm-up and capture: the steps write K/V at positions
    >= each row's length, which attention never reads before the real tokens
    overwrite them, so the (possibly huge) cache is not copied.  ``keep_graph``
    keeps the captured graph inspectable (``graph.raw_cuda_graph()``)."""

    def __init__(self, model, cache, *, width: int = 1, sample: tuple | None = None,
                 tokens: torch.Tensor | None = None, uniform: torch.Tensor | None = None, keep_graph: bool = False):
        dev = model.device
        self.width = width
        self.sample = sample
        self.token_ids = tokens if tokens is not None else torch.zeros(width, 1, dtype=torch.long, device=dev)
        self.uniform = uniform if uniform is not None else torch.zeros(width, dtype=torch.float32, device=dev)
        snap = _length_snapshot(cache)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        try:
            with torch.cuda.stream(stream):
                for _ in range(_GRAPH_WARMUP):
                    self._step(model, cache)
                    _length_restore(cache, snap)
                self.graph = torch.cuda.CUDAGraph(keep_graph=keep_graph)
                with torch.cuda.graph(self.graph, stream=stream):
                    self.logits, self.next_id = self._step(model, cache)
            torch.cuda.current_stream(dev).wait_stream(stream)
            torch.cuda.synchronize(dev)
        finally:
            _length_restore(cache, snap)

    def _step(self, model, cache):
        w = self.width
        logits = model.forward(self.token_ids[:w], cache=cache, logits_to_keep=1)
        last = logits[:, -1, :]
        if self.sample is None:
            nxt = argmax(last)
        else:
            ws, temperature, top_p, top_k = self.sample
            nxt = fused_sample_batched(last, self.uniform[:w], temperature=temperature, top_p=top_p, top_k=top_k,
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
    raise_device_errors(dev, "run_generate")
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
    """Decode graphs for a ladder of batch widths over one cache (the
    reference's bucketed graphs, generate.py:703-816, same observable
    behaviour): a step replays the narrowest rung that holds the live rows.

    Every rung is a :class:`DecodeGraph` reading the same token / uniform
    buffers, so loading a step's inputs is one copy whatever the rung.  Rows
    between the live count and the rung width are padding that runs on the
    cache rows above the live ones: callers keep live sequences packed into
    the low slots (:func:`compact_slots`).  The graphs read the slot ->
    cache-row map at replay time, so slot moves need no re-capture."""

    def __init__(self, model, cache, *, widths: tuple[int, ...], sample: tuple | None = None,
                 log: Callable[[str], None] | None = _log_print):
        if not cache.remap:
            raise ValueError("BucketedDecodeGraphs needs cache.remap enabled.")
        self.widths = tuple(sorted({int(w) for w in widths}))
        if not self.widths or self.widths[0] < 1:
            raise ValueError(f"graph widths must be >= 1, got {widths}.")
        self.max_width = self.widths[-1]
        if self.max_width > cache.batch:
            raise ValueError(f"widest graph {self.max_width} exceeds the cache batch {cache.batch}.")
        dev = model.device
        self.sample = sample
        self.token_ids = torch.zeros(self.max_width, 1, dtype=torch.long, device=dev)
        self.uniform = torch.zeros(self.max_width, dtype=torch.float32, device=dev)
        self._rungs = {w: DecodeGraph(model, cache, width=w, sample=sample, tokens=self.token_ids,
                                      uniform=self.uniform) for w in self.widths}
        if log is not None:
            log(f"decode graphs at widths {list(self.widths)} ({'sampled' if sample is not None else 'greedy'})")

    def width_for(self, live: int) -> int:
        i = bisect.bisect_left(self.widths, int(live))
        if i == len(self.widths):
            raise ValueError(f"live batch {live} exceeds widest graph {self.max_width}.")
        return self.widths[i]

    def _run(self, tokens: torch.Tensor, uniform: torch.Tensor | None) -> tuple[int, DecodeGraph]:
        live = int(tokens.shape[0])
        rung = self._rungs[self.width_for(live)]
        self.token_ids[:live].copy_(tokens.reshape(live, 1))
        self.token_ids[live:rung.width].zero_()
        if uniform is not None:
            self.uniform[:live].copy_(uniform.reshape(-1)[:live])
        rung.graph.replay()
        return live, rung

    def replay(self, tokens: torch.Tensor, uniform: torch.Tensor | None = None) -> torch.Tensor:
        """Step ``tokens`` ``[live, 1]``; returns the next ids ``[live]``."""
        live, rung = self._run(tokens, uniform)
        return rung.next_id[:live]

    def replay_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Step ``tokens``; returns last-token logits ``[live, vocab]``."""
        live, rung = self._run(tokens, None)
        return rung.logits[:live].reshape(live, -1)


def checked_decode_graphs(model, cache, probe: list[int], *, sample=None, widths=None,
                          log: Callable[[str], None] | None = _log_print) -> BucketedDecodeGraphs | None:
    """Capture the decode graphs and keep them only if a replay reproduces
    the eager step (reference generate.py:1045-1104, the replay == eager
    gate).  The probe step feeds ``probe`` (one id per live slot) from the
    cache's current lengths, once eagerly and once through the graph of its
    width, and compares the last-token logits bit for bit (a stronger check
    than the sampled ids, and independent of the sampler's uniforms).  The
    cache lengths are left as they were."""
    try:
        graphs = BucketedDecodeGraphs(model, cache, widths=tuple(widths or decode_buckets(cache.batch)),
                                      sample=sample, log=log)
    except Exception as exc:  # capture is an optimisation; eager decode stays correct
        if log is not None:
            log(f"CUDA graph capture failed ({exc}); decoding eagerly")
        return None
    tokens = torch.tensor(probe, device=model.device, dtype=torch.long).view(-1, 1)
    snap = _length_snapshot(cache)
    try:
        eager = model.forward(tokens, cache=cache, logits_to_keep=1)[:, -1, :].clone()
        _length_restore(cache, snap)
        replayed = graphs.replay_logits(tokens).clone()
    finally:
        _length_restore(cache, snap)
    if not torch.equal(eager, replayed):
        if log is not None:
            log("CUDA graph replay differs from the eager step; decoding eagerly")
        return None
    return graphs


def compact_slots(cache, entries: list, keep: list[bool]) -> int:
    """Pack the kept slots among the first ``len(keep)`` (the live ones) into
    the low slots and return how many there are.  Two cursors walk inwards:
    the lowest dropped slot takes the highest kept one (a cache row-map swap,
    no K/V moves) until they meet, so the fewest swaps fill every hole below
    the new live count.  ``entries`` (one per slot) and ``keep`` are permuted
    alongside; entries past the live ones are left alone."""
    lo, hi = 0, len(keep) - 1
    while True:
        while lo <= hi and keep[lo]:
            lo += 1
        while hi > lo and not keep[hi]:
            hi -= 1
        if lo >= hi:
            break
        cache.swap_slots(lo, hi)
        entries[lo], entries[hi] = entries[hi], entries[lo]
        keep[lo], keep[hi] = keep[hi], keep[lo]
        lo += 1
        hi -= 1
    return sum(keep)


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


@dataclass
class _Row:
    """One sequence of a batched decode: its output row, cap and the id it
    will emit next."""

    index: int
    cap: int
    nxt: int
    out: list[int] = field(default_factory=list)
    reason: str = "length"

    def emit(self, stop_ids: set[int]) -> bool:
        """Append the pending id; True while the row wants another step."""
        self.out.append(self.nxt)
        if self.nxt in stop_ids:
            self.reason = "stop"
            return False
        return len(self.out) < self.cap


class _Picker:
    """Next-id selection shared by prefill and decode steps: argmax, or the
    fused sampler with one uniform per row from the caller's generator."""

    def __init__(self, model, rows: int, *, temperature, top_p, top_k, seed):
        self.dev = model.device
        self.greedy = is_greedy(temperature, top_k)
        if not self.greedy and not can_fuse_sampler(temperature, top_p, top_k):
            raise ValueError(f"sampled decode needs 0 < top_k <= {MAX_TOP_K} and 0 < top_p <= 1.")
        self.params = (float(temperature), float(top_p), int(top_k))
        self.gen = None
        if seed is not None and not self.greedy:
            self.gen = torch.Generator(device=self.dev)
            self.gen.manual_seed(int(seed))
        self.ws = None if self.greedy else batched_sampler_workspace(model.vocab_size, int(top_k), rows, self.dev)

    @property
    def graph_sample(self):
        return None if self.greedy else (self.ws, *self.params)

    def uniforms(self, n: int) -> torch.Tensor | None:
        return None if self.greedy else torch.rand(n, device=self.dev, generator=self.gen)

    def pick(self, last: torch.Tensor, u: torch.Tensor | None) -> torch.Tensor:
        if self.greedy:
            return argmax(last)
        t, p, k = self.params
        return fused_sample_batched(last, u, temperature=t, top_p=p, top_k=k, workspace=self.ws)


@torch.inference_mode()
def batched_generate(model, prompts, *, max_tokens: int = 128, max_new: list[int] | None = None,
                     temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, seed: int | None = None,
                     stop_ids: set[int] | None = None, cache=None, graphs: bool = False,
                     buckets: tuple[int, ...] | None = None, runner: BucketedDecodeGraphs | None = None,
                     log: Callable[[str], None] | None = _log_print) -> BatchedResult:
    """Decode several sequences as one batch (reference generate.py:842-1028,
    same arguments and result).

    Each prompt is prefilled into cache slot i; decode then runs all live
    rows per step, so the batched GEMMs read every weight once per step.  A
    row leaves the batch when it emits a stop id or reaches its cap (its own
    ``max_new`` entry, else ``max_tokens``); the survivors are packed into
    the low slots, and with ``graphs`` each step replays the narrowest
    captured width holding them."""
    dev = model.device
    seqs = [torch.as_tensor(p, device=dev, dtype=torch.long).reshape(-1) for p in prompts]
    n = len(seqs)
    if n == 0:
        raise ValueError("batched_generate needs at least one prompt.")
    caps = [int(max_tokens)] * n if max_new is None else [int(c) for c in max_new]
    if len(caps) != n:
        raise ValueError(f"max_new has {len(caps)} entries for {n} prompts.")
    if min(caps) < 1:
        raise ValueError("every row needs a cap of at least one token.")
    prompt_lens = [int(t.numel()) for t in seqs]
    need = max(prompt_lens) + max(caps)
    if cache is None:
        cache = model.make_cache(max_len=need, batch=n)
    elif cache.batch < n or cache.max_len < need:
        raise ValueError(f"cache ({cache.batch} rows x {cache.max_len}) cannot hold {n} rows of {need} positions.")
    else:
        cache.reset_identity()
    stops = stop_token_ids(model) if stop_ids is None else set(stop_ids)
    picker = _Picker(model, cache.batch, temperature=temperature, top_p=top_p, top_k=top_k, seed=seed)

    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    rows: list[_Row] = []
    for i, ids in enumerate(seqs):
        with cache.prefill_slot(i):
            last = model.forward(ids.view(1, -1), cache=cache, logits_to_keep=1)[:, -1, :]
        rows.append(_Row(index=i, cap=caps[i], nxt=int(picker.pick(last, picker.uniforms(1))[0])))
    torch.cuda.synchronize(dev)
    prefill_s = time.perf_counter() - t0

    cache.remap = True
    if graphs and runner is None:
        runner = checked_decode_graphs(model, cache, [r.nxt for r in rows], sample=picker.graph_sample,
                                       widths=buckets, log=log)
    widths: list[int] = []
    steps = 0
    t0 = time.perf_counter()
    live = n
    while live:
        keep = [r.emit(stops) for r in rows[:live]]
        live = compact_slots(cache, rows, keep)
        if not live:
            break
        tokens = torch.tensor([r.nxt for r in rows[:live]], device=dev, dtype=torch.long).view(live, 1)
        u = picker.uniforms(live)
        if runner is not None:
            nxt = runner.replay(tokens, u)
            widths.append(runner.width_for(live))
            cache.advance_host(1, widths[-1])
        else:
            nxt = picker.pick(model.forward(tokens, cache=cache, logits_to_keep=1)[:, -1, :], u)
        for r, tok in zip(rows, nxt.tolist()):
            r.nxt = int(tok)
        steps += 1
    torch.cuda.synchronize(dev)
    decode_s = time.perf_counter() - t0
    raise_device_errors(dev, "batched_generate")
    by_index = sorted(rows, key=lambda r: r.index)
    return BatchedResult([r.out for r in by_index], prompt_lens, [r.reason for r in by_index], prefill_s, decode_s,
                         steps, widths)
