"""Continuous-batching decode worker over persistent KV-cache slots.

Reference: server.py:352-795 (``PackedEngine``): same client API
(``run`` / ``wait_ready`` / ``close``, ``ServerDefaults``, ``Sampling``,
``RequestError``) and the same observable scheduling -- a request joins a
free cache slot as soon as one is free, every live slot decodes in the same
step, each row samples with its own parameters and generator, and a request
ends at a stop id, at its cap, or when its slot's cache is full.

The worker here is this engine's own design.  One thread owns the model and
a KV cache of ``max_batch`` rows and repeats a round: take queued requests
into the free slots (prefill + first id), run one decode step for all live
slots (the narrowest captured graph that holds them), deliver each produced
id at once, then pack the surviving slots into the low rows with the
two-cursor :func:`compact_slots` and reset the rows that were freed.  Token
ids go in and come out: the HTTP / OpenAI protocol, chat templates and
detokenisation are outside this engine.
"""

from __future__ import annotations

import itertools
import queue
import threading
import time
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any

import torch

from maple_flash_dgx_spark_b200._lib import raise_device_errors
from maple_flash_dgx_spark_b200.generate import (
    DEFAULT_TEMPERATURE,
    DEFAULT_TOP_K,
    DEFAULT_TOP_P,
    GenerateResult,
    can_fuse_sampler,
    checked_decode_graphs,
    compact_slots,
    is_greedy,
    resolve_max_tokens,
    stop_token_ids,
)
from maple_flash_dgx_spark_b200.kernels import (
    MAX_TOP_K,
    argmax,
    batched_sampler_workspace,
    fused_sample_batched,
)

DEFAULT_MAX_BATCH = 8
DEFAULT_MAX_LEN = 4096


class RequestError(ValueError):
    """A request the engine refuses (reference server.py RequestError)."""


@dataclass
class ServerDefaults:
    """Engine-wide defaults (reference server.py:67-76)."""

    temperature: float = DEFAULT_TEMPERATURE
    top_p: float = DEFAULT_TOP_P
    top_k: int = DEFAULT_TOP_K
    max_tokens: int = 128
    seed: int | None = None
    flash_head: bool = False
    model_id: str = "maple-2bit"
    max_batch: int = DEFAULT_MAX_BATCH
    max_len: int = DEFAULT_MAX_LEN


@dataclass(frozen=True)
class Sampling:
    """One request's sampling parameters (reference server.py:79-87)."""

    temperature: float
    top_p: float
    top_k: int
    max_tokens: int
    seed: int | None
    stream: bool = False
    model: str = ""


@dataclass
class _Request:
    """A queued request and the handle its caller waits on."""

    input_ids: Any
    sampling: Sampling
    stop_ids: set[int] | None = None
    on_token: Callable[[int], None] | None = None
    done: threading.Event = field(default_factory=threading.Event)
    result: GenerateResult | None = None
    error: BaseException | None = None

    def fail(self, exc: BaseException) -> None:
        if self.error is None and self.result is None:
            self.error = exc
        self.done.set()


@dataclass
class _Active:
    """A request decoding in a cache slot: what it has emitted and the id it
    feeds to the next step."""

    request: _Request
    cap: int
    prompt_len: int
    prefill_s: float
    started: float
    stops: set[int]
    generator: torch.Generator | None
    nxt: int = 0
    out: list[int] = field(default_factory=list)
    reason: str = "length"

    @property
    def sample_key(self):
        s = self.request.sampling
        return None if is_greedy(s.temperature, s.top_k) else (s.temperature, s.top_p, s.top_k)


_CLOSE = object()


def _log(msg: str) -> None:
    print(msg, flush=True)


class PackedEngine:
    """Load once; a worker thread admits requests into persistent cache slots
    and decodes them together (reference server.py:352-795)."""

    def __init__(self, model, tokenizer=None, defaults: ServerDefaults | None = None,
                 log: Callable[[str], None] | None = _log):
        self.model = model
        self.tokenizer = tokenizer
        self.defaults = defaults if defaults is not None else ServerDefaults()
        self.max_batch = int(self.defaults.max_batch)
        self.max_len = int(self.defaults.max_len)
        if self.max_batch < 1 or self.max_len < 2:
            raise ValueError("PackedEngine needs max_batch >= 1 and max_len >= 2.")
        self._log = log
        self._inbox: queue.Queue = queue.Queue()
        self._ready = threading.Event()
        self._closing = threading.Event()
        self._start_error: BaseException | None = None
        self._slots: list[_Active] = []   # slot i holds _slots[i]; live slots are always the low ones
        self._cache = None
        self._graphs = None
        self._sample_ws = None
        self._worker = threading.Thread(target=self._worker_main, name="maple-batch", daemon=True)
        self._worker.start()

    # ---------------------------------------------------------------- client
    @property
    def live(self) -> int:
        """Requests decoding right now (one per occupied cache slot)."""
        return len(self._slots)

    @property
    def cache(self):
        return self._cache

    def wait_ready(self) -> None:
        self._ready.wait()
        if self._start_error is not None:
            raise self._start_error

    def close(self) -> None:
        self._closing.set()
        self._inbox.put(_CLOSE)
        self._worker.join(timeout=30)

    def run(self, input_ids, *, max_tokens: int = 128, temperature: float = 0.0, top_p: float = 1.0,
            top_k: int = 1, seed: int | None = None, stop_ids: set[int] | None = None,
            on_token: Callable[[int], None] | None = None) -> GenerateResult:
        """Decode ``input_ids`` on the worker and wait for the result (the
        reference's token-id entry point).  ``on_token`` is called on the
        worker thread with each emitted id."""
        sampling = Sampling(temperature=float(temperature), top_p=float(top_p), top_k=int(top_k),
                            max_tokens=int(max_tokens), seed=seed, stream=on_token is not None,
                            model=self.defaults.model_id)
        return self._submit(input_ids, sampling, stop_ids=stop_ids, on_token=on_token)

    def _submit(self, input_ids, sampling: Sampling, *, stop_ids=None, on_token=None) -> GenerateResult:
        self.wait_ready()
        if not is_greedy(sampling.temperature, sampling.top_k) and not can_fuse_sampler(
                sampling.temperature, sampling.top_p, sampling.top_k):
            raise RequestError(f"sampling needs 0 < top_k <= {MAX_TOP_K} and 0 < top_p <= 1.")
        req = _Request(input_ids=input_ids, sampling=sampling, stop_ids=stop_ids, on_token=on_token)
        self._inbox.put(req)
        req.done.wait()
        if req.error is not None:
            raise req.error
        assert req.result is not None
        return req.result

    # ---------------------------------------------------------------- worker
    def _worker_main(self) -> None:
        try:
            self._prepare()
        except Exception as exc:  # reported to every caller through wait_ready
            self._start_error = exc
            self._ready.set()
            return
        self._ready.set()
        with torch.inference_mode():
            try:
                while self._round():
                    pass
            except Exception as exc:
                for a in self._slots:
                    a.request.fail(exc)
                self._slots = []
            self._shut()

    def _prepare(self) -> None:
        """Cache of ``max_batch`` slots and the checked decode graphs (greedy
        logits graphs; sampling runs after the replay, per row group)."""
        model = self.model
        dev = model.device
        torch.cuda.set_device(dev)
        if getattr(model, "lm_head_flash", None) is not None:
            model.lm_head_flash = None  # FlashHead is a batch-1 head; batched rows use the exact head
            if self._log is not None:
                self._log("continuous batch uses the exact lm_head (FlashHead is B=1 only)")
        with torch.inference_mode():
            cache = model.make_cache(max_len=self.max_len, batch=self.max_batch)
            # one position in every slot, so the capture and its probe step attend to real rows
            one = torch.zeros(1, 1, dtype=torch.long, device=dev)
            for slot in range(self.max_batch):
                with cache.prefill_slot(slot):
                    model.forward(one, cache=cache, logits_to_keep=1)
            cache.remap = True
            self._graphs = checked_decode_graphs(model, cache, [0] * self.max_batch, log=self._log)
            for slot in range(self.max_batch):
                cache.reset_slot(slot)
            self._cache = cache
        self._sample_ws = batched_sampler_workspace(int(model.config["vocab_size"]), MAX_TOP_K, self.max_batch, dev)

    def _round(self) -> bool:
        """Take queued requests into free slots, then one decode step for
        the live slots.  False once the engine is closing."""
        while len(self._slots) < self.max_batch:
            if self._closing.is_set():
                return False
            try:
                item = self._inbox.get(block=not self._slots)
            except queue.Empty:
                break
            if item is _CLOSE:
                return False
            self._admit(item)
        if self._slots:
            self._step()
        return True

    def _shut(self) -> None:
        """Fail what is queued or decoding once the engine closes."""
        stopped = RuntimeError("engine stopped")
        for a in self._slots:
            a.request.fail(stopped)
        self._slots = []
        while True:
            try:
                item = self._inbox.get_nowait()
            except queue.Empty:
                return
            if item is not _CLOSE:
                item.fail(stopped)

    def _admit(self, req: _Request) -> None:
        model, dev = self.model, self.model.device
        ids = torch.as_tensor(req.input_ids, device=dev, dtype=torch.long).reshape(-1)
        plen = int(ids.numel())
        if not 0 < plen < self.max_len:
            req.fail(RequestError(f"prompt length {plen} must be in [1, max_len {self.max_len})."))
            return
        try:
            cap = resolve_max_tokens(req.sampling.max_tokens, plen, self.max_len)
        except ValueError as exc:
            req.fail(RequestError(str(exc)))
            return
        if cap <= 0:
            req.result = GenerateResult([], plen, 0, 0.0, 0.0, "length", self._graphs is not None)
            req.done.set()
            return
        s = req.sampling
        gen = None
        if s.seed is not None and not is_greedy(s.temperature, s.top_k):
            gen = torch.Generator(device=dev)
            gen.manual_seed(int(s.seed))
        stops = req.stop_ids if req.stop_ids is not None else stop_token_ids(model, self.tokenizer)
        slot = len(self._slots)
        self._cache.reset_slot(slot)
        t0 = time.perf_counter()
        with self._cache.prefill_slot(slot):
            last = model.forward(ids.view(1, -1), cache=self._cache, logits_to_keep=1)[:, -1, :]
        entry = _Active(request=req, cap=cap, prompt_len=plen, prefill_s=0.0, started=0.0, stops=set(stops),
                        generator=gen)
        first = self._choose(last, [entry])[0]
        entry.prefill_s = time.perf_counter() - t0
        entry.started = time.perf_counter()
        self._slots.append(entry)
        if not self._deliver(slot, first):
            self._retire([False if i == slot else True for i in range(len(self._slots))])

    def _deliver(self, slot: int, tok: int) -> bool:
        """Emit ``tok`` for the request in ``slot``; True while it continues."""
        a = self._slots[slot]
        a.out.append(tok)
        a.nxt = tok
        if a.request.on_token is not None:
            try:
                a.request.on_token(tok)
            except Exception as exc:  # a failing callback ends its own request only
                a.request.error = exc
                return False
        if tok in a.stops:
            a.reason = "stop"
            return False
        # the cap, or the slot's last cache position used: no room for another step
        return len(a.out) < a.cap and self._cache.seen[slot] < self.max_len

    def _retire(self, keep: list[bool]) -> None:
        """Pack the continuing slots low; free and reset the rest before
        their callers are told they are done."""
        n = compact_slots(self._cache, self._slots, keep)
        gone, self._slots = self._slots[n:], self._slots[:n]
        for slot, a in enumerate(gone, start=n):
            self._cache.reset_slot(slot)
            if a.request.result is None and a.request.error is None:
                a.request.result = GenerateResult(list(a.out), a.prompt_len, len(a.out), a.prefill_s,
                                                  max(time.perf_counter() - a.started, 0.0), a.reason,
                                                  self._graphs is not None)
            a.request.done.set()

    def _step(self) -> None:
        """One decode step of every live slot."""
        n = len(self._slots)
        dev = self.model.device
        tokens = torch.tensor([a.nxt for a in self._slots], device=dev, dtype=torch.long).view(n, 1)
        if self._graphs is not None:
            logits = self._graphs.replay_logits(tokens)
            width = self._graphs.width_for(n)
            self._cache.advance_host(1, n)
            for slot in range(n, width):  # padding rows of a wider graph ran on free slots
                self._cache.reset_slot(slot)
        else:
            logits = self.model.forward(tokens, cache=self._cache, logits_to_keep=1)[:, -1, :]
        produced = self._choose(logits, self._slots)
        raise_device_errors(dev, "PackedEngine decode step")
        keep = [self._deliver(slot, tok) for slot, tok in enumerate(produced)]
        if not all(keep):
            self._retire(keep)

    def _choose(self, logits: torch.Tensor, entries: list[_Active]) -> list[int]:
        """Next id per row: one argmax over all rows, then each group of
        sampled rows with equal (temperature, top_p, top_k) through one
        batched fused-sampler launch, every row drawing its uniform from its
        own generator."""
        dev = logits.device
        nxt = argmax(logits)
        sampled = sorted((i for i, a in enumerate(entries) if a.sample_key is not None),
                         key=lambda i: entries[i].sample_key)
        for key, grp in itertools.groupby(sampled, key=lambda i: entries[i].sample_key):
            rows = list(grp)
            idx = torch.tensor(rows, device=dev, dtype=torch.long)
            u = torch.stack([torch.rand((), device=dev, generator=entries[i].generator) for i in rows])
            temperature, top_p, top_k = key
            nxt[idx] = fused_sample_batched(logits[idx], u, temperature=temperature, top_p=top_p, top_k=top_k,
                                            workspace=self._sample_ws)
        return [int(x) for x in nxt.tolist()]
