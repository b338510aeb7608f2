"""Expert-parallel batched decode over the GPUs of one node.

One process per GPU (``torch.distributed``, NCCL).  For a batch of B
sequences on W ranks:

* attention is data-parallel: rank r holds B/W sequences, their KV cache and
  a replica of the attention, router and norm weights;
* experts are partitioned: rank r holds experts [r*E/W, (r+1)*E/W);
* per MoE layer, an all-gather carries every rank's routed rows and top-k ids
  to every rank (dispatch), each rank runs its experts over the slots routed
  to them (grouped GEMMs, weights read once), and an all-to-all returns to
  each token's rank the rows computed for its slots (combine), summed in the
  single-GPU order by ``ep_combine``;
* the RTN-4 lm_head is vocabulary-sharded: each rank scores its V/W rows for
  all B tokens, takes its local argmax, and an all-gather of (value, index)
  candidates picks the global first maximum.

Every per-row result equals single-GPU batched decode bit for bit: routing,
expert rows, the combine order and the argmax tie rule are the same.

Reference: model.py:448-474 (MoE block), generate.py:842-1028 (batched
decode); the reference itself runs on one GPU.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from maple_flash_dgx_spark_b200 import _lib
from maple_flash_dgx_spark_b200._lib import check, dtype_code, lib, ptr, stream_ptr

from maple_flash_dgx_spark_b200.kernels import (
    add_rms_norm,
    argmax,
    ep_combine,
    moe_plan,
    rtn4_gemv,
    router_topk,
    ternary_expert_gemv,
    ternary_expert_swiglu,
)

PHASES = ("qkv", "attention", "o_norm", "router", "dispatch", "experts", "combine", "head")


class PhaseMarks:
    """Timing events at the phase boundaries of one decode step, recorded as
    event nodes when the step is captured in a CUDA graph (``external``
    events), so a replay can be split into its phases: qkv (input norm + QKV
    projection), attention (QK-norm, RoPE, K/V store, attention), o_norm (O
    projection, residual add + norm), router, dispatch, experts (SwiGLU +
    down), combine, and the sharded head (final norm, row gather, head GEMV,
    candidate gather).  Phase times are summed over the layers."""

    def __init__(self):
        self.events: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str) -> None:
        # only the captured step counts: warm-up steps run eagerly before it
        if not torch.cuda.is_current_stream_capturing():
            return
        ev = torch.cuda.Event(enable_timing=True, external=True)
        ev.record()
        self.events.append((name, ev))

    def phase_ms(self) -> dict[str, float]:
        """Milliseconds per phase of the last replay (events must be complete)."""
        out = {p: 0.0 for p in PHASES}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] += a.elapsed_time(b)
        return out

_EXPERT_KEYS = ("up_proj", "gate_proj", "down_proj")


def expert_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """(first expert, experts held) of ``rank``."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks.")
    per = n_experts // world
    return rank * per, per


def token_range(batch: int, rank: int, world: int) -> tuple[int, int]:
    """(first row, rows) of the batch held by ``rank``."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks.")
    per = batch // world
    return rank * per, per


def shard_expert_weights(weights: dict, config: dict, rank: int, world: int) -> dict:
    """Keep only this rank's experts of every layer (packed-ternary-v1 names)."""
    e0, n = expert_range(int(config["num_experts"]), rank, world)
    out = {}
    for k, v in weights.items():
        if ".mlp.switch_mlp." in k and any(f".{e}." in k for e in _EXPERT_KEYS):
            out[k] = v[e0:e0 + n].contiguous()
        else:
            out[k] = v
    return out


class EPExchange:
    """The collectives of one expert-parallel MoE layer.  Layout only (no
    compute), so the same code runs over NCCL on GPUs and over gloo in the
    CPU tests."""

    def __init__(self, group, rank: int, world: int, n_experts: int):
        self.group = group
        self.rank = rank
        self.world = world
        self.n_experts = n_experts
        self.e_first, self.n_local = expert_range(n_experts, rank, world)

    def dispatch(self, hidden: torch.Tensor, idx: torch.Tensor):
        """All-gather ``hidden [T, H]`` and ``idx [T, k]`` (int32) from every
        rank as one packed byte buffer; returns ``x_all [W*T, H]`` (rows in
        rank order, a strided view) and ``ids_all [W*T, k]``."""
        T, H = hidden.shape
        k = idx.shape[1]
        hb = H * hidden.element_size()
        send = torch.empty(T, hb + 4 * k, dtype=torch.uint8, device=hidden.device)
        send[:, :hb].copy_(hidden.contiguous().view(torch.uint8).reshape(T, hb))
        send[:, hb:].copy_(idx.to(torch.int32).contiguous().view(torch.uint8).reshape(T, 4 * k))
        recv = torch.empty(self.world * T, hb + 4 * k, dtype=torch.uint8, device=hidden.device)
        dist.all_gather_into_tensor(recv, send, group=self.group)
        x_all = recv[:, :hb].view(hidden.dtype)
        ids_all = recv[:, hb:].contiguous().view(torch.int32)
        return x_all, ids_all

    def combine_exchange(self, y_all: torch.Tensor) -> torch.Tensor:
        """``y_all [W*T*k, N]`` (rows by slot of the gathered tokens) ->
        ``[W, T*k, N]``: from every rank, its rows for this rank's slots."""
        rows, n = y_all.shape
        recv = torch.empty_like(y_all)
        dist.all_to_all_single(recv, y_all.contiguous(), group=self.group)
        return recv.view(self.world, rows // self.world, n)

    def gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty(self.world * x.shape[0], *x.shape[1:], dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out


class _DeviceMem:
    """__cuda_array_interface__ view of raw device memory (zero-copy)."""

    def __init__(self, addr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False), "version": 3,
                                         "strides": None}


class SymmetricBuffer:
    """One device buffer of the same size on every rank, mapped into the other
    ranks through CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle), zeroed.
    ``bases`` is the ctypes array of every rank's address as seen here."""

    def __init__(self, nbytes: int, group, rank: int, world: int, device: torch.device):
        from cuda.bindings import runtime as rt

        self.rt, self.rank, self.world, self.group = rt, rank, world, group
        self.nbytes = int(nbytes)
        with torch.cuda.device(device):
            err, base = rt.cudaMalloc(self.nbytes)
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaMalloc of the symmetric buffer failed: {err}")
            rt.cudaMemset(base, 0, self.nbytes)
            rt.cudaDeviceSynchronize()
            err, handle = rt.cudaIpcGetMemHandle(base)
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaIpcGetMemHandle failed: {err}")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.reserved), group=group)
        self.own = int(base)
        self.opened = []
        addrs = []
        with torch.cuda.device(device):
            for r in range(world):
                if r == rank:
                    addrs.append(self.own)
                    continue
                h = rt.cudaIpcMemHandle_t()
                h.reserved = handles[r]
                err, peer = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                if err != rt.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaIpcOpenMemHandle of rank {r} failed: {err}")
                self.opened.append(peer)
                addrs.append(int(peer))
        dist.barrier(group=group)
        self.bases = (ctypes.c_void_p * world)(*addrs)
        self.device = device

    def view(self, offset: int, nbytes: int) -> torch.Tensor:
        return torch.as_tensor(_DeviceMem(self.own + offset, nbytes), device=self.device)

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's."""
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            self.rt.cudaIpcCloseMemHandle(p)
        dist.barrier(group=self.group)
        self.rt.cudaFree(self.own)
        self.own = None


def _round256(n: int) -> int:
    return (n + 255) // 256 * 256


class EPExchangeP2P(EPExchange):
    """EPExchange over NVLink peer memory (``maple_p2p_*``): ``dispatch``
    sends this rank's routed rows and top-k ids to every rank as tagged words
    and gathers every rank's into dense local buffers; ``combine`` sends each
    row its experts computed to the token's owner and sums the slots in the
    same kernel.  Buffers are sized for ``tokens`` rows per rank, fixed for
    the object's life."""

    def __init__(self, group, rank: int, world: int, n_experts: int, *, tokens: int, hidden: int, topk: int,
                 device: torch.device, dtype=torch.bfloat16):
        super().__init__(group, rank, world, n_experts)
        self.tokens, self.hidden, self.topk, self.dtype = tokens, hidden, topk, dtype
        code = _lib._DTYPE[dtype]
        L = lib()
        self.off_dispatch = 0
        self.off_combine = _round256(L.maple_p2p_dispatch_bytes(world, tokens, hidden, code, topk))
        total = self.off_combine + _round256(L.maple_p2p_combine_bytes(tokens, topk, hidden, code))
        self.buf = SymmetricBuffer(total, group, rank, world, device)
        self.rows_all = torch.empty(world * tokens, hidden, dtype=dtype, device=device)
        self.ids_all = torch.empty(world * tokens, topk, dtype=torch.int32, device=device)
        self.state = torch.zeros(4, dtype=torch.int32, device=device)  # seq/ticket of dispatch, then of combine
        self.err = _lib.error_word(device)
        self.device = device

    def _state(self, i):
        return self.state.data_ptr() + 4 * i

    def dispatch(self, hidden: torch.Tensor, idx: torch.Tensor):
        T, H = hidden.shape
        k = idx.shape[1]
        if T != self.tokens or H != self.hidden or k != self.topk or hidden.dtype != self.dtype:
            raise ValueError(f"EPExchangeP2P sized for {self.tokens}x{self.hidden} {self.dtype} top-{self.topk}, got "
                             f"{T}x{H} {hidden.dtype} top-{k}.")
        x = hidden if hidden.stride(1) == 1 else hidden.contiguous()
        ids = idx.to(torch.int32).contiguous()
        check(lib().maple_p2p_dispatch(self.buf.bases, self.world, self.rank, self.off_dispatch, ptr(x),
                                       dtype_code(x, "p2p_dispatch"), x.stride(0), T, H, ptr(ids), k,
                                       ptr(self.rows_all), ptr(self.ids_all), self._state(0), self._state(1),
                                       ptr(self.err), stream_ptr(self.device)), "p2p_dispatch")
        return self.rows_all, self.ids_all

    def combine(self, y_all: torch.Tensor, plan, wt: torch.Tensor, residual=None) -> torch.Tensor:
        """``y_all``: rows by slot of the gathered tokens (this rank's experts'
        slots filled, as listed by ``plan``); returns this rank's MoE output
        rows (+ ``residual``)."""
        y = y_all.reshape(-1, self.hidden)
        if not y.is_contiguous():
            y = y.contiguous()
        out = torch.empty(self.tokens, self.hidden, dtype=y.dtype, device=y.device)
        w = wt.float().contiguous()
        res = residual.reshape(self.tokens, self.hidden).contiguous() if residual is not None else None
        check(lib().maple_p2p_combine(self.buf.bases, self.world, self.rank, self.off_combine, ptr(y),
                                      dtype_code(y, "p2p_combine"), ptr(plan.offsets), ptr(plan.slots),
                                      plan.n_experts, self.tokens, self.topk, self.hidden, ptr(w), ptr(res), ptr(out),
                                      self._state(2), self._state(3), ptr(self.err), stream_ptr(self.device)),
              "p2p_combine")
        return out

    def close(self) -> None:
        self.buf.close()


class EPMoeBlock:
    """Drop-in for ``MapleSparseMoeBlock`` holding this rank's experts only."""

    def __init__(self, block, exchange: EPExchange):
        self.block = block
        self.ex = exchange
        self.marks: PhaseMarks | None = None

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            self.marks.mark(name)

    def __call__(self, hidden_states, residual=None):
        b = self.block
        idx, wt = router_topk(hidden_states, b.gate_weight, b.top_k)
        self._mark("router")
        x_all, ids_all = self.ex.dispatch(hidden_states, idx)
        self._mark("dispatch")
        plan = moe_plan(ids_all, self.ex.n_experts, e_first=self.ex.e_first, n_local=self.ex.n_local)
        h = ternary_expert_swiglu(x_all, b.up_gate.packed_weight, b.up_gate.row_alpha, ids_all, plan=plan)
        y = ternary_expert_gemv(h, b.down.packed_weight, b.down.row_alpha, ids_all, plan=plan)
        self._mark("experts")
        if isinstance(self.ex, EPExchangeP2P):
            out = self.ex.combine(y, plan, wt, residual)
        else:
            recv = self.ex.combine_exchange(y.reshape(-1, y.shape[-1]))
            out = ep_combine(recv, idx, wt, self.ex.n_experts, residual)
        self._mark("combine")
        return out


class EPHead:
    """Vocabulary-sharded RTN-4 lm_head with the greedy pick: rank r scores
    rows [r*V/W, (r+1)*V/W) for every gathered token, and the candidates'
    (value, index) pairs meet in an all-gather."""

    def __init__(self, lm_head, exchange: EPExchange):
        V = lm_head.packed_weight.shape[0]
        w = exchange.world
        if V % w:
            raise ValueError(f"vocab {V} does not split over {w} ranks.")
        self.shard = V // w
        r0 = exchange.rank * self.shard
        self.codes = lm_head.packed_weight[r0:r0 + self.shard].contiguous()
        self.scales = lm_head.scales[r0:r0 + self.shard].contiguous()
        self.biases = None if lm_head.biases is None else lm_head.biases[r0:r0 + self.shard].contiguous()
        self.group_size = lm_head.group_size
        self.ex = exchange

    def next_ids(self, normed: torch.Tensor) -> torch.Tensor:
        T = normed.shape[0]
        h_all = self.ex.gather_rows(normed)
        logits = rtn4_gemv(h_all, self.codes, self.scales, self.biases, group_size=self.group_size)
        li = argmax(logits)
        lv = logits.gather(1, li.reshape(-1, 1)).float()
        cand = torch.cat([lv.view(torch.int32), li.to(torch.int32).reshape(-1, 1)], 1)  # [W*T, 2] int32
        allc = self.ex.gather_rows(cand).view(self.ex.world, -1, 2)  # [W, W*T, 2]
        vals = allc[:, :, 0].contiguous().view(torch.float32).t().contiguous()  # [W*T, W]
        r = argmax(vals)  # ties and NaN: lowest rank = lowest vocabulary index
        rows = torch.arange(vals.shape[0], device=normed.device)
        ids = allc[r, rows, 1].long() + r * self.shard
        return ids[self.ex.rank * T:(self.ex.rank + 1) * T]


class EPDecoder:
    """One greedy decode step of this rank's rows: embedding, the layers
    (data-parallel attention, expert-parallel MoE), final norm, sharded head."""

    def __init__(self, model, exchange: EPExchange):
        self.model = model
        self.ex = exchange
        for layer in model.layers:
            if not isinstance(layer.mlp, EPMoeBlock):
                layer.mlp = EPMoeBlock(layer.mlp, exchange)
        self.head = EPHead(model.lm_head, exchange)
        self.marks: PhaseMarks | None = None

    def set_marks(self, marks: PhaseMarks | None) -> None:
        """Record phase boundaries into ``marks`` during the next steps
        (``None`` stops recording)."""
        self.marks = marks
        for layer in self.model.layers:
            layer.mlp.marks = marks
            layer.self_attn.marks = marks

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            self.marks.mark(name)

    def step(self, tokens: torch.Tensor, cache) -> torch.Tensor:
        """One decode step; the layer body is MapleDecoderLayer's (attention
        with the input norm fused into QKV, residual add + post-attention
        norm, MoE with the residual) written out so phases can be marked."""
        m = self.model
        rows = tokens.shape[0]
        seqlen = cache.seqlen[:rows]
        row_map = cache.row_map[:rows] if cache.remap else None
        m.rotary.ensure_length(cache.max_len)
        hidden = m.embed(tokens.reshape(rows))
        self._mark("head")  # the step's start; embedding time counts with the head
        for layer in m.layers:
            attn = layer.self_attn(hidden, seqlen, row_map, m.rotary, cache,
                                   rms_weight=layer.input_layernorm.weight, rms_eps=layer.input_layernorm.eps,
                                   kv_final=True)
            post = layer.post_attention_layernorm
            hidden, mlp_in = add_rms_norm(hidden, attn, post.weight, post.eps)
            self._mark("o_norm")
            hidden = layer.mlp(mlp_in, residual=hidden)
        cache.advance(1, rows)
        ids = self.head.next_ids(m.norm(hidden))
        self._mark("head")
        return ids


class EPDecodeGraph:
    """``EPDecoder.step`` captured in a CUDA graph (collectives included)."""

    def __init__(self, decoder: EPDecoder, cache, rows: int, warmup: int = 3, keep_graph: bool = False):
        dev = decoder.model.device
        self.token_ids = torch.zeros(rows, 1, dtype=torch.long, device=dev)
        snap = (cache.seqlen.clone(), list(cache.seen))
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            for _ in range(warmup):
                decoder.step(self.token_ids, cache)
                cache.seqlen.copy_(snap[0])
                cache.seen = list(snap[1])
            self.graph = torch.cuda.CUDAGraph(keep_graph=keep_graph)
            with torch.cuda.graph(self.graph, stream=st):
                self.next_id = decoder.step(self.token_ids, cache)
        torch.cuda.current_stream(dev).wait_stream(st)
        torch.cuda.synchronize(dev)
        cache.seqlen.copy_(snap[0])
        cache.seen = list(snap[1])

    def replay(self, tokens: torch.Tensor | None = None) -> torch.Tensor:
        if tokens is not None:
            self.token_ids.copy_(tokens.reshape(-1, 1))
        self.graph.replay()
        return self.next_id


def check_step_errors(device: torch.device) -> None:
    """Raise if a kernel of the expert-parallel steps run since the last
    check flagged an error (a peer flag wait that gave up leaves the ranks'
    exchange counters out of step: the exchange must be rebuilt)."""
    _lib.raise_device_errors(device, "expert-parallel decode step")
