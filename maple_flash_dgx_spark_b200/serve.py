"""Continuous-batching decode worker over persistent KV-cache slots.

Reference: server.py:352-795 (``PackedEngine``).  One worker thread owns the
model and a KV cache of ``max_batch`` rows.  Requests queue up; the worker
prefills each admitted request into a free cache slot, decodes all live slots
together (one bucketed decode graph per width, the narrowest that holds the
live rows), samples every row with its own sampling parameters, and retires
finished rows by swapping them above the live ones, so the live rows stay
dense in the low slots.  Requests carry and return token ids: the HTTP /
OpenAI protocol, chat templates and detokenisation are outside this engine.
"""

from __future__ import annotations

import queue
import threading
import time
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any

import torch

from maple_flash_dgx_spark_b200.generate import (
    DEFAULT_TEMPERATURE,
    DEFAULT_TOP_K,
    DEFAULT_TOP_P,
    GenerateResult,
    _try_batched_decode_graphs,
    can_fuse_sampler,
    is_greedy,
    resolve_max_tokens,
    stop_token_ids,
)
from maple_flash_dgx_spark_b200.kernels import (
    MAX_TOP_K,
    argmax,
    batched_sampler_workspace,
    fused_sample,
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
class _Job:
    input_ids: Any
    sampling: Sampling
    stop_ids: set[int] | None = None
    on_token: Callable[[int], None] | None = None
    done: threading.Event = field(default_factory=threading.Event)
    result: GenerateResult | None = None
    error: BaseException | None = None


@dataclass
class _Slot:
    job: _Job
    pending: int                 # sampled, not yet emitted nor fed back
    max_tokens: int
    prompt_len: int
    prefill_s: float
    decode_t0: float
    stop_ids: set[int]
    generator: torch.Generator | None
    token_ids: list[int] = field(default_factory=list)
    finish_reason: str = "length"


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
        self._queue: queue.Queue[_Job | None] = queue.Queue()
        self._ready = threading.Event()
        self._stop = threading.Event()
        self._start_error: BaseException | None = None
        self._live = 0
        self._slots: list[_Slot | None] = [None] * self.max_batch
        self._cache = None
        self._runner = None
        self._sample_ws = None
        self._worker = threading.Thread(target=self._run, name="maple-batch", daemon=True)
        self._worker.start()

    # ---------------------------------------------------------------- client
    def wait_ready(self) -> None:
        self._ready.wait()
        if self._start_error is not None:
            raise self._start_error

    def close(self) -> None:
        self._stop.set()
        self._queue.put(None)
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
        job = _Job(input_ids=input_ids, sampling=sampling, stop_ids=stop_ids, on_token=on_token)
        self._queue.put(job)
        job.done.wait()
        if job.error is not None:
            raise job.error
        assert job.result is not None
        return job.result

    # ---------------------------------------------------------------- worker
    def _run(self) -> None:
        try:
            self._setup()
        except Exception as exc:  # reported to every waiter through wait_ready
            self._start_error = exc
            self._ready.set()
            return
        self._ready.set()
        try:
            with torch.inference_mode():
                while True:
                    if not self._admit():
                        break
                    if self._live == 0:
                        continue
                    self._emit_and_retire()
                    if self._live == 0:
                        continue
                    if self._stop.is_set():
                        self._drain_stop()
                        break
                    self._decode_step()
        except Exception as exc:
            self._fail_all(exc)

    def _setup(self) -> None:
        model = self.model
        dev = model.device
        torch.cuda.set_device(dev)
        if getattr(model, "lm_head_flash", None) is not None:
            # FlashHead is a batch-1 head; batched rows use the exact head
            model.lm_head_flash = None
            if self._log is not None:
                self._log("continuous batch uses the exact lm_head (FlashHead is B=1 only)")
        with torch.inference_mode():
            self._cache = model.make_cache(max_len=self.max_len, batch=self.max_batch)
            dummy = torch.zeros(1, 1, dtype=torch.long, device=dev)
            pending: list[int] = []
            for b in range(self.max_batch):
                with self._cache.prefill_slot(b):
                    logits = model.forward(dummy, cache=self._cache, logits_to_keep=1)
                pending.append(int(argmax(logits[0, -1])))
            self._cache.remap = True
            self._runner = _try_batched_decode_graphs(model, self._cache, pending, sample=None, log=self._log)
            for b in range(self.max_batch):
                self._cache.reset_slot(b)
        self._sample_ws = batched_sampler_workspace(int(model.config["vocab_size"]), MAX_TOP_K, self.max_batch, dev)

    def _admit(self) -> bool:
        """Fill free slots from the queue; False when the worker should exit."""
        while self._live < self.max_batch:
            if self._stop.is_set():
                self._drain_stop()
                return False
            if self._live == 0:
                job = self._queue.get()
            else:
                try:
                    job = self._queue.get_nowait()
                except queue.Empty:
                    return True
            if job is None:
                self._drain_stop()
                return False
            self._admit_job(job)
        return True

    def _drain_stop(self) -> None:
        while True:
            try:
                left = self._queue.get_nowait()
            except queue.Empty:
                break
            if left is not None:
                left.error = RuntimeError("engine stopped")
                left.done.set()
        for slot in range(self._live):
            self._finish_slot(slot, error=RuntimeError("engine stopped"))
        self._live = 0

    def _admit_job(self, job: _Job) -> None:
        dev = self.model.device
        ids = torch.as_tensor(job.input_ids, device=dev, dtype=torch.long).reshape(-1)
        prompt_len = int(ids.numel())
        if prompt_len == 0 or prompt_len >= self.max_len:
            job.error = RequestError(f"prompt length {prompt_len} must be in [1, max_len {self.max_len}).")
            job.done.set()
            return
        try:
            cap = resolve_max_tokens(job.sampling.max_tokens, prompt_len, self.max_len)
        except ValueError as exc:
            job.error = RequestError(str(exc))
            job.done.set()
            return
        if cap <= 0:
            job.result = GenerateResult([], prompt_len, 0, 0.0, 0.0, "length", self._runner is not None)
            job.done.set()
            return
        slot = self._live
        self._cache.reset_slot(slot)
        t0 = time.perf_counter()
        with self._cache.prefill_slot(slot):
            logits = self.model.forward(ids.view(1, -1), cache=self._cache, logits_to_keep=1)
        s = job.sampling
        gen = None
        if s.seed is not None and not is_greedy(s.temperature, s.top_k):
            gen = torch.Generator(device=dev)
            gen.manual_seed(int(s.seed))
        pending = int(self._first_id(logits, s, gen))
        prefill_s = time.perf_counter() - t0
        stop = job.stop_ids if job.stop_ids is not None else stop_token_ids(self.model, self.tokenizer)
        self._slots[slot] = _Slot(job=job, pending=pending, max_tokens=cap, prompt_len=prompt_len,
                                  prefill_s=prefill_s, decode_t0=time.perf_counter(), stop_ids=set(stop),
                                  generator=gen)
        self._live += 1

    @staticmethod
    def _first_id(logits, s: Sampling, gen):
        last = logits[0, -1]
        if is_greedy(s.temperature, s.top_k):
            return argmax(last)
        u = torch.rand((), device=last.device, generator=gen)
        return fused_sample(last, u, temperature=s.temperature, top_p=s.top_p, top_k=s.top_k)

    def _emit_and_retire(self) -> None:
        """Emit every live slot's pending id; retire the slots that stop."""
        done: list[int] = []
        for slot in range(self._live):
            row = self._slots[slot]
            tok = row.pending
            row.token_ids.append(tok)
            if row.job.on_token is not None:
                try:
                    row.job.on_token(tok)
                except Exception as exc:  # a failing callback ends its own request only
                    row.job.error = exc
                    done.append(slot)
                    continue
            if tok in row.stop_ids:
                row.finish_reason = "stop"
                done.append(slot)
            elif len(row.token_ids) >= row.max_tokens:
                row.finish_reason = "length"
                done.append(slot)
            elif self._cache.seen[slot] >= self.max_len:
                # the slot's last cache position is used: no room for the next step
                row.finish_reason = "length"
                done.append(slot)
        for slot in reversed(done):
            last = self._live - 1
            if slot != last:
                self._cache.swap_slots(slot, last)
                self._slots[slot], self._slots[last] = self._slots[last], self._slots[slot]
            row = self._slots[last]
            # the slot is free and empty before its request is told it is done
            self._cache.reset_slot(last)
            self._slots[last] = None
            self._live -= 1
            self._finish_row(row)

    def _finish_slot(self, slot: int, error: BaseException | None = None) -> None:
        self._finish_row(self._slots[slot], error)

    def _finish_row(self, row: _Slot | None, error: BaseException | None = None) -> None:
        if row is None:
            return
        job = row.job
        if error is not None and job.error is None:
            job.error = error
        if job.result is None and job.error is None:
            job.result = GenerateResult(list(row.token_ids), row.prompt_len, len(row.token_ids), row.prefill_s,
                                        max(time.perf_counter() - row.decode_t0, 0.0), row.finish_reason,
                                        self._runner is not None)
        job.done.set()

    def _decode_step(self) -> None:
        live = self._live
        dev = self.model.device
        tokens = torch.tensor([self._slots[s].pending for s in range(live)], device=dev,
                              dtype=torch.long).view(live, 1)
        if self._runner is not None:
            logits = self._runner.replay_logits(tokens)
            width = self._runner.width_for(live)
            self._cache.advance_host(1, live)
            # padding rows of a wider graph ran on free slots: put them back to empty
            for s in range(live, width):
                self._cache.reset_slot(s)
        else:
            logits = self.model.forward(tokens, cache=self._cache, logits_to_keep=1)[:, -1, :]
        for s, tok in enumerate(self._sample_rows(logits)):
            self._slots[s].pending = int(tok)

    def _sample_rows(self, logits) -> list[int]:
        """Greedy rows by argmax; the others grouped by (temperature, top_p,
        top_k) through the batched fused sampler, each row drawing its
        uniform from its own generator."""
        live = logits.shape[0]
        dev = logits.device
        nxt = torch.empty(live, dtype=torch.long, device=dev)
        greedy: list[int] = []
        groups: dict[tuple[float, float, int], list[int]] = {}
        for s in range(live):
            sp = self._slots[s].job.sampling
            if is_greedy(sp.temperature, sp.top_k):
                greedy.append(s)
            else:
                groups.setdefault((sp.temperature, sp.top_p, sp.top_k), []).append(s)
        if greedy:
            idx = torch.tensor(greedy, device=dev, dtype=torch.long)
            nxt[idx] = argmax(logits[idx])
        for (temperature, top_p, top_k), rows in groups.items():
            idx = torch.tensor(rows, device=dev, dtype=torch.long)
            u = torch.empty(len(rows), device=dev)
            for n, s in enumerate(rows):
                u[n] = torch.rand((), device=dev, generator=self._slots[s].generator)
            nxt[idx] = fused_sample_batched(logits[idx], u, temperature=temperature, top_p=top_p, top_k=top_k,
                                            workspace=self._sample_ws)
        return [int(x) for x in nxt.tolist()]

    def _fail_all(self, exc: BaseException) -> None:
        for slot in range(self._live):
            self._finish_slot(slot, error=exc)
        self._live = 0
