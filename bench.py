"""Benchmark of the sm_100a decode engine on the synthetic 48-layer packed
ternary MoE model (BASELINE.json configs[2] architecture).  Prints one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

Workloads (``--workload``, default ``auto``):

* ``bs1`` (configs[2]; the default of a plain ``python bench.py``): a step is
  one greedy decode token (48 layers + RTN-4 head + argmax) at batch 1 after a
  512-token prompt; the context grows 512 -> 512+W+K.  About 1.06 GB of
  weights and K/V are streamed from HBM every step (> L2).
* ``bs64`` (configs[3]; the default under torchrun, any world size): 64
  sequences with 8192 cached positions each, one token per row per step.
  One GPU: batched decode.  N GPUs: expert parallelism (64/N experts and 64/N
  sequences per rank, NVLink peer-memory dispatch/combine, vocabulary-sharded
  head), with a per-phase breakdown of the step.
* ``long``: long-context sampling.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PROMPT_LEN = 512
SEED = 2
SYNTH_DATA = ("synthetic: seeded random-init weights of the configs' architecture from a counter-hash generator; "
              "ternary P(0)=0.4, P(+-1)=0.3 exact; 'normal' draws are Irwin-Hall sums of four 16-bit uniforms "
              "(variance-matched, bounded at 3.46 sigma) standing in for N(0, s)")


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bs64", action="store_true",
                    help="bs1 on one GPU: skip the batch-64 point measured after the batch-1 line")
    ap.add_argument("--breakdown", action="store_true",
                    help="also time each operator of the decode step in its own CUDA graph (48 layers)")
    ap.add_argument("--workload", choices=["auto", "bs1", "bs64", "long", "attn", "prefill", "kmeans"],
                    default="auto",
                    help="auto: bs64 under torchrun (expert-parallel scaling), else bs1; bs1: configs[2] batch-1 "
                         "decode; bs64: configs[3] batch-64 decode at 8192 cached positions per row; long: "
                         "configs[4] long-context sampling (FlashHead at batch 1); attn: the decode-attention "
                         "kernels alone (--batch rows x --context positions); prefill: the configs[2] 512-token "
                         "prompt with and without the tcgen05 expert GEMM, and that GEMM alone; kmeans: the FlashHead "
                         "balanced spherical k-means of --rows head rows")
    ap.add_argument("--context", type=int, default=None,
                    help="cached positions per row (bs64: 8192, long: 65536)")
    ap.add_argument("--batch", type=int, default=1, help="long: rows (1, 16 or 256)")
    ap.add_argument("--rows", type=int, default=151936, help="kmeans: head rows (a multiple of 32)")
    return ap.parse_args()


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled DURING the timed
    region: NVML read every ~2 ms from a thread (reading only; no setting of
    the GPU is changed), so even a 40 ms region gets a few dozen samples."""

    # NVML clocks-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.index = device_index
        self.period = period_s
        self.sm: list[float] = []
        self.bits = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._nvml = None

    def _handle(self, nv):
        try:
            import torch

            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{getattr(pr, 'pci_domain_id', 0):08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            self._nvml = nv
            self._h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        except Exception:
            self._nvml = None
        return self

    def _poll(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)))
                self.bits |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        if self._nvml is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted(name for bit, name in self.REASONS.items() if self.bits & bit)
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.sm), "source": "nvml, ~2 ms polling"}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(cfg, n_tokens: int = 3):
    """The CPU oracle (restatement of the reference's decode) on the host cores:
    build the 48-layer model, feed a few context tokens, time ``n_tokens``
    decode steps.  Returns (tok/s, cores, sample description)."""
    import oracle.model as om

    t0 = time.time()
    m = om.OracleModel(cfg, SEED, max_len=PROMPT_LEN + 64, split_len=32)
    m.fill_cache(SEED, PROMPT_LEN)
    build_s = time.time() - t0
    tok = 1
    m.step(tok)  # warm
    t0 = time.time()
    for _ in range(n_tokens):
        tok = m.step(tok)
    dt = time.time() - t0
    cores = os.cpu_count()
    return n_tokens / dt, cores, (f"{n_tokens} decode tokens of the 48-layer model at context {PROMPT_LEN} on "
                                  f"{cores} OpenMP threads (model build {build_s:.0f}s untimed)")


def run_reference(args):
    """--impl reference: the reference's decode restated on the CPU (the
    oracle port: the reference has no CPU kernels, its Triton kernels need a
    GPU), timed on the host cores; rank 0 only, on the workload our arm runs
    with the same arguments (bs1 by default, bs64 under torchrun).  bs1: a
    step is one decode token of the 48-layer model over a random-filled
    512-position cache (no prompt prefill: a CPU prefill of 512 tokens takes
    minutes).  bs64: a step is one row's decode token at 8192 random cached
    positions (the 64 rows are independent; the CPU port decodes row by row),
    so the value is rows decoded per second.  Each run is capped at about
    90 s of decode."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    workload = args.workload
    if workload == "auto":
        workload = "bs64" if "WORLD_SIZE" in os.environ else "bs1"
    cfg = synthetic_config(num_layers=args.layers)
    import oracle.model as om

    if workload == "bs64":
        ctx = int(args.context or 8192)
        metric, config = "decode tok/s (bs64, configs[3])", bs64_config(cfg, world, ctx, args.warmup, args.steps)
        scaling = "strong"
    else:
        ctx = PROMPT_LEN
        metric, config = "decode tok/s (bs1, configs[2])", bs1_config(cfg, world)
        scaling = "weak"
    t_build = time.time()
    m = om.OracleModel(cfg, SEED, max_len=ctx + args.warmup + args.steps + 8, split_len=32 if ctx <= 512 else 256)
    m.fill_cache(SEED, ctx)
    build_s = time.time() - t_build
    tok = 1
    for _ in range(max(1, min(args.warmup, 2))):
        tok = m.step(tok)
    budget_s, n = 90.0, 0
    t0 = time.time()
    while n < args.steps:
        tok = m.step(tok)
        n += 1
        if time.time() - t0 > budget_s:
            break
    dt = time.time() - t0
    v = n / dt
    cores = os.cpu_count()
    what = (f"{n} row decode tokens at {ctx} random cached positions (rows of the batch are independent)"
            if workload == "bs64" else f"{n} decode tokens over a random-filled {ctx}-position cache")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": v, "unit": "tok/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": 1000 * dt / n, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": SYNTH_DATA,
        "config": config,
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{what} of the {cfg['num_hidden_layers']}-layer model: the CPU oracle port on "
                                   f"{cores} OpenMP threads, attention split {m.P}, cap {budget_s:.0f} s "
                                   f"(model build and cache fill {build_s:.0f} s untimed)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = _args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "auto":
        args.workload = "bs64" if "WORLD_SIZE" in os.environ else "bs1"
    if args.workload == "bs64":
        run_bs64(args)
        return
    if args.workload == "long":
        run_long(args)
        return
    if args.workload == "attn":
        run_attn(args)
        return
    if args.workload == "prefill":
        run_prefill(args)
        return
    if args.workload == "kmeans":
        run_kmeans(args)
        return
    line = run_bs1(args)
    world, rank, _ = _dist()
    if line is None:
        return
    if world == 1 and not args.no_bs64:
        # the batch-64 point of the same single-GPU run (configs[3] on one GPU),
        # so a 1..N scaling series has its one-GPU batch-64 number
        import gc

        import torch

        gc.collect()
        torch.cuda.empty_cache()
        sub = argparse.Namespace(**vars(args))
        sub.steps, sub.warmup, sub.context = min(args.steps, 64), max(3, min(args.warmup, 5)), None
        b64 = run_bs64(sub, emit=False)
        line["bs64"] = {k: b64.get(k) for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup",
                                                 "scaling", "config", "e2e", "roofline", "hbm_roofline_step",
                                                 "gpu_launches", "clocks", "device_errors", "phases_ms_per_step")}
    print(json.dumps(line), flush=True)


def run_bs1(args):
    """batch-1 greedy decode after a 512-token prompt.  Returns
    the JSON line on rank 0 (None elsewhere)."""
    import torch

    from maple_flash_dgx_spark_b200 import _lib
    from maple_flash_dgx_spark_b200 import kernels as K
    from maple_flash_dgx_spark_b200.generate import DecodeGraph
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM, kv_bytes_per_token, packed_decode_bytes
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_tokens, synthetic_weights

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    cfg = synthetic_config(num_layers=args.layers)
    W, Kst = args.warmup, args.steps
    max_len = PROMPT_LEN + W + Kst + 2
    torch.manual_seed(0)
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, SEED + rank, dev), device=dev)
    prompt = synthetic_tokens(SEED, PROMPT_LEN, cfg["vocab_size"], dev)
    cache = model.make_cache(max_len=max_len)
    with torch.inference_mode():
        # time to first token: the 512-token prompt prefilled in one forward
        model.forward(prompt.reshape(1, -1), cache=model.make_cache(max_len=PROMPT_LEN + 1))  # warm
        torch.cuda.synchronize(dev)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        logits = model.forward(prompt.reshape(1, -1), cache=cache)
        first = K.argmax(logits[:, -1, :])
        p1.record()
        torch.cuda.synchronize(dev)
        ttft_ms = p0.elapsed_time(p1)
        graph = DecodeGraph(model, cache, width=1, keep_graph=True)
        launches_per_step = graph_kernel_launches(graph.graph)
        # ---- device-resident timing: next id feeds back on the device ----
        graph.token_ids.copy_(first.reshape(1, 1))
        nxt = graph.next_id
        for _ in range(W):
            graph.graph.replay()
            graph.token_ids.copy_(nxt.reshape(1, 1))
        cache.advance_host(W, 1)  # the replays advanced the device lengths
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx0 = int(cache.seen[0])
        with ClockSampler(local) as clocks:
            torch.cuda.nvtx.range_push("maple_decode")
            start.record()
            for _ in range(Kst):
                graph.graph.replay()
                graph.token_ids.copy_(nxt.reshape(1, 1))
            end.record()
            torch.cuda.synchronize(dev)
            torch.cuda.nvtx.range_pop()
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        cache.advance_host(Kst, 1)  # keep host lengths in step with the replays
        tok_s = world * Kst / (ms / 1000.0)

        # ---- end to end through the public decode-graph API: the token goes
        # host -> device from pinned memory and the id comes back every step ----
        e2e_cache = model.make_cache(max_len=PROMPT_LEN + Kst + 2)
        logits = model.forward(prompt.reshape(1, -1), cache=e2e_cache)
        g2 = DecodeGraph(model, e2e_cache, width=1)
        pin_in = torch.empty(1, 1, dtype=torch.long, pin_memory=True)
        pin_out = torch.empty(1, dtype=torch.long, pin_memory=True)
        pin_in[0, 0] = int(K.argmax(logits[:, -1, :]).item())
        ev = torch.cuda.Event()
        ne2e = min(Kst, 256)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(ne2e):
            g2.token_ids.copy_(pin_in, non_blocking=True)
            g2.graph.replay()
            pin_out.copy_(g2.next_id.reshape(1), non_blocking=True)
            ev.record()
            ev.synchronize()
            pin_in[0, 0] = pin_out[0]
        e2e_s = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = world * ne2e / e2e_s

        # ---- dominant kernel: expert SwiGLU, one launch per layer at batch 1 ----
        launch_us, swiglu_bytes = swiglu_roofline(model, prompt, dev)
        device_errors = _lib.take_device_errors(dev)

    peak, peak_kind = _peaks()
    traffic = _profiled_traffic("expert_swiglu")
    weights_bytes = packed_decode_bytes(cfg)["packed_weight_bytes"]
    ctx_mid = ctx0 + Kst // 2
    step_bytes = weights_bytes + kv_bytes_per_token(cfg, ctx_mid)
    line = {
        "metric": "decode tok/s (bs1, configs[2])",
        "value": tok_s,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": Kst,
        "warmup": W,
        "ms_per_step": ms / Kst,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": SYNTH_DATA + "; 512 random prompt ids",
        "config": bs1_config(cfg, world),
        "context": [ctx0, ctx0 + Kst],
        "hbm_roofline_step": {"bytes_per_token": step_bytes, "achieved_gbs": step_bytes * (Kst / (ms / 1000.0)) / 1e9,
                              "peak_gbs": peak, "frac": step_bytes * (Kst / (ms / 1000.0)) / 1e9 / peak},
        "roofline": {"kernel": "tgemv2_kernel<swiglu> (expert up|gate + SwiGLU, bs1)", "bound": "hbm",
                     "achieved": swiglu_bytes / (launch_us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": swiglu_bytes / (launch_us * 1e-6) / 1e9 / peak, "traffic": traffic,
                     "algorithmic_bytes": swiglu_bytes, "launch_us": launch_us, "peak_kind": f"{peak_kind} hbm_gbs"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "gpu_launches": Kst * (launches_per_step or _step_launches(cfg["num_hidden_layers"])),
        "gpu_launches_source": ("kernel nodes of this library in the captured decode graph x steps"
                                if launches_per_step else "estimate"),
        "clocks": clocks.summary(),
        "device_errors": device_errors,
        "prefill": {"prompt_tokens": PROMPT_LEN, "ttft_ms": ttft_ms, "prompt_tok_s": PROMPT_LEN / (ttft_ms / 1000.0),
                    "note": "one eager forward of the prompt (expert GEMMs on tcgen05 where experts average >= 16 "
                            "routed slots) plus the first argmax, CUDA events"},
    }
    if device_errors:
        raise SystemExit(f"device error word {device_errors:#x} set during the run: the numbers are not valid")
    if args.breakdown:
        line["breakdown_us_per_launch"] = op_breakdown(model, cache, dev)
    if rank == 0 and not args.no_cpu_baseline:
        v, cores, sample = cpu_baseline(cfg)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}
    if world > 1:
        del graph, g2
        dist.destroy_process_group()
    return line if rank == 0 else None


def bs1_config(cfg, world: int) -> dict:
    """The bs1 workload description (both arms): configs[2] at context 512."""
    from maple_flash_dgx_spark_b200.model import kv_bytes_per_token, packed_decode_bytes

    step = packed_decode_bytes(cfg)["packed_weight_bytes"] + kv_bytes_per_token(cfg, PROMPT_LEN)
    return {"workload": f"configs[2]: {cfg['num_hidden_layers']}-layer ternary MoE, bs1 greedy decode after a "
                        f"{PROMPT_LEN}-token prompt",
            "global_batch": world, "seq_len": PROMPT_LEN,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": f"{step / 1e9:.2f} GB of weights and K/V streamed per step (> 126 MB L2), no flush needed"}


BS64_ROWS = 64


def bs64_step_bytes(cfg, world: int, ctx: int) -> int:
    """HBM bytes one GPU streams per configs[3] step at ``ctx`` cached
    positions: replicated attention / router / norm weights, 1/world of the
    experts and of the head, the K/V of its 64/world rows."""
    from maple_flash_dgx_spark_b200.model import packed_decode_bytes

    wb = packed_decode_bytes(cfg)
    experts_all = cfg["num_hidden_layers"] * cfg["num_experts"] * (
        (2 * cfg["moe_intermediate_size"] * cfg["hidden_size"] + cfg["hidden_size"] * cfg["moe_intermediate_size"])
        // 4 + (2 * cfg["moe_intermediate_size"] + cfg["hidden_size"]) * 2)
    rep = wb["packed_weight_bytes"] - wb["expert_bytes"] - wb["head_bytes"]
    weights_gpu = rep + (experts_all + wb["head_bytes"]) // world
    kv_gpu = (BS64_ROWS // world) * cfg["num_hidden_layers"] * cfg["num_key_value_heads"] * cfg["head_dim"] * 4 * ctx
    return int(weights_gpu + kv_gpu)


def bs64_config(cfg, world: int, ctx: int, warmup: int, steps: int) -> dict:
    """The bs64 workload description (both arms)."""
    step = bs64_step_bytes(cfg, world, ctx + warmup + steps // 2)
    return {"workload": f"configs[3]: bs{BS64_ROWS} greedy decode, {ctx} cached positions per row",
            "global_batch": BS64_ROWS, "seq_len": ctx,
            "parallelism": f"ep{world}+dp-attention{world}" if world > 1 else "single",
            "l2": f"{step / 1e9:.1f} GB streamed per GPU per step (> 126 MB L2), no flush needed"}


def graph_kernel_launches(graph):
    """Kernel nodes of a captured CUDA graph (``keep_graph=True``) whose
    function belongs to this package's library (C++ namespace ``mb``, mangled
    ``_ZN2mb``): this library's launches per replay, torch's and NCCL's
    kernels excluded.  None when the graph cannot be inspected."""
    try:
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt

        g = rt.cudaGraph_t(init_value=int(graph.raw_cuda_graph()))
        err, _, n = rt.cudaGraphGetNodes(g, 0)
        if err != rt.cudaError_t.cudaSuccess:
            return None
        err, nodes, n = rt.cudaGraphGetNodes(g, n)
        if err != rt.cudaError_t.cudaSuccess:
            return None
        count = 0
        for nd in nodes[:n]:
            err, kind = rt.cudaGraphNodeGetType(nd)
            if err != rt.cudaError_t.cudaSuccess or kind != rt.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                continue
            err, prm = drv.cuGraphKernelNodeGetParams(drv.CUgraphNode(init_value=int(nd)))
            if err != drv.CUresult.CUDA_SUCCESS:
                return None
            err, name = drv.cuFuncGetName(prm.func)
            if err != drv.CUresult.CUDA_SUCCESS:
                return None
            if bytes(name).startswith(b"_ZN2mb"):
                count += 1
        return count or None
    except Exception:
        return None


def _time_graph(fns, dev, reps=5):
    """Capture ``fns`` in one CUDA graph, replay it ``reps`` times, return ms per replay."""
    import torch

    for f in fns:
        f()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for f in fns:
                f()
    torch.cuda.current_stream(dev).wait_stream(st)
    g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def run_bs64(args, emit: bool = True):
    """64 independent sequences, each with ``--context`` random
    cached positions (bf16 N(0,1) K/V written directly), one new token per row
    per step, greedy.  One GPU: batched decode.  N GPUs (torchrun): expert
    parallelism -- each rank holds 64/N sequences (data-parallel attention),
    64/N experts and 1/N of the vocabulary; NCCL all-gather (dispatch) and
    all-to-all (combine) per MoE layer, candidate all-gather for the head.
    Returns the JSON line (printed on rank 0 when ``emit``)."""
    import datetime

    import torch
    import torch.distributed as dist

    from maple_flash_dgx_spark_b200 import _lib
    from maple_flash_dgx_spark_b200 import kernels as K
    from maple_flash_dgx_spark_b200.generate import DecodeGraph
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM, packed_decode_bytes
    from maple_flash_dgx_spark_b200.synth import fill_kv_cache, synthetic_config, synthetic_tokens, synthetic_weights

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # a process group at every world size (a single-rank one without torchrun):
    # the per-phase pass runs the expert-parallel step even on one GPU
    if "WORLD_SIZE" in os.environ:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    else:
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=300), device_id=dev)
    B, ctx = BS64_ROWS, int(args.context or 8192)
    cfg = synthetic_config(num_layers=args.layers)
    W, Kst = args.warmup, args.steps
    weights = synthetic_weights(cfg, SEED, dev)
    T, t0 = B, 0
    from maple_flash_dgx_spark_b200.expert_parallel import (PHASES, EPDecodeGraph, EPDecoder, EPExchange,
                                                            EPExchangeP2P, PhaseMarks, check_step_errors,
                                                            shard_expert_weights, token_range)

    if world > 1:
        weights = shard_expert_weights(weights, cfg, rank, world)
        t0, T = token_range(B, rank, world)
    model = MapleForCausalLM.from_weight_dict(cfg, weights, device=dev)
    del weights
    torch.cuda.empty_cache()
    cache = model.make_cache(max_len=ctx + W + 2 * Kst + 8, batch=T)
    fill_kv_cache(cache, SEED, ctx, row0=t0, total_rows=B)
    tokens = synthetic_tokens(SEED, B, cfg["vocab_size"], dev)[t0:t0 + T].reshape(T, 1)
    graph_kind = "cuda graph"
    with torch.inference_mode():
        # MAPLE_EP_TRANSPORT=nccl selects the NCCL collectives; default: NVLink peer-store kernels
        transport = os.environ.get("MAPLE_EP_TRANSPORT", "p2p")

        def make_decoder():
            if transport == "nccl":
                exch = EPExchange(None, rank, world, cfg["num_experts"])
            else:
                exch = EPExchangeP2P(None, rank, world, cfg["num_experts"], tokens=T, hidden=cfg["hidden_size"],
                                     topk=cfg["num_experts_per_tok"], device=dev)
            return exch, EPDecoder(model, exch)

        holder = {}  # the only references to captured graphs (freed before the group is destroyed)
        ex = None
        launches_per_step = None
        if world > 1:
            ex, dec = make_decoder()
            try:
                holder["g"] = EPDecodeGraph(dec, cache, T, keep_graph=True)
                launches_per_step = graph_kernel_launches(holder["g"].graph)
                ids_buf = holder["g"].token_ids

                def step(tok=None):
                    return holder["g"].replay()

                nxt_of = lambda: holder["g"].next_id  # noqa: E731
            except Exception as exc:  # NCCL capture unsupported: eager steps (same collectives)
                graph_kind = f"eager ({type(exc).__name__})"
                ids_buf = torch.zeros(T, 1, dtype=torch.long, device=dev)
                state = {}

                def step(tok=None):
                    state["n"] = dec.step(ids_buf, cache)
                    return state["n"]

                nxt_of = lambda: state["n"]  # noqa: E731
        else:
            g = DecodeGraph(model, cache, width=T, keep_graph=True)
            launches_per_step = graph_kernel_launches(g.graph)
            ids_buf = g.token_ids
            nxt_of = lambda: g.next_id  # noqa: E731

            def step(tok=None):
                g.graph.replay()
                return g.next_id
        ids_buf.copy_(tokens)
        for _ in range(W):
            step()
            ids_buf.copy_(nxt_of().reshape(T, 1))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx0 = ctx + W
        with ClockSampler(local) as clocks:
            torch.cuda.nvtx.range_push("maple_decode")
            start.record()
            for _ in range(Kst):
                step()
                ids_buf.copy_(nxt_of().reshape(T, 1))
            end.record()
            torch.cuda.synchronize(dev)
            torch.cuda.nvtx.range_pop()
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        if graph_kind == "cuda graph":
            cache.advance_host(W + Kst, T)
        tok_s = B * Kst / (ms / 1000.0)
        # ---- end to end: this rank's ids host -> device and back every step ----
        pin_in = torch.empty(T, 1, dtype=torch.long, pin_memory=True)
        pin_out = torch.empty(T, dtype=torch.long, pin_memory=True)
        pin_in.copy_(tokens.cpu())
        ev = torch.cuda.Event()
        ne2e = max(1, min(Kst, 32))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t_0 = time.perf_counter()
        for _ in range(ne2e):
            ids_buf.copy_(pin_in, non_blocking=True)
            step()
            pin_out.copy_(nxt_of().reshape(T), non_blocking=True)
            ev.record()
            ev.synchronize()
            pin_in[:, 0] = pin_out
        e2e_s = time.perf_counter() - t_0
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e = B * ne2e / e2e_s
        if world > 1:
            check_step_errors(dev)
        device_errors = _lib.take_device_errors(dev)
        # ---- per-phase breakdown: the expert-parallel step (also at one GPU)
        # captured once more with timing events at its phase boundaries ----
        if ex is None:
            ex, dec = make_decoder()
        phases = None
        try:
            marks = PhaseMarks()
            dec.set_marks(marks)
            holder["phases"] = EPDecodeGraph(dec, cache, T)
            dec.set_marks(None)
            reps, acc = 3, {p: 0.0 for p in PHASES}
            dist.barrier()
            for _ in range(reps):
                holder["phases"].replay()
                torch.cuda.synchronize(dev)
                for k, v in marks.phase_ms().items():
                    acc[k] += v / reps
            cache.advance_host(reps, T)
            vec = torch.tensor([acc[p] for p in PHASES], device=dev)
            dist.all_reduce(vec, op=dist.ReduceOp.MAX)
            phases = {p: round(float(v), 4) for p, v in zip(PHASES, vec.tolist())}
            phases["sum"] = round(sum(phases[p] for p in PHASES), 4)
            check_step_errors(dev)
        except Exception as exc:  # the breakdown is diagnostic; the timed number stands without it
            phases = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
        # ---- dominant kernel: decode attention over this rank's rows ----
        att = model.layers[0].self_attn
        q = torch.randn(T, model.num_heads, 1, model.head_dim, device=dev).to(torch.bfloat16)
        pos = torch.full((T,), ctx0, dtype=torch.int64, device=dev)
        fns = [lambda i=i: K.decode_gqa_attn(q, cache.k[i], cache.v[i], pos, scale=att.scale, window=None,
                                             split_len=cache.split_len, kv_final=True, tensor_cores=cache.attn_tc)
               for i in range(len(model.layers))]
        att_us = _time_graph(fns, dev) * 1000.0 / len(fns)
        kv_per_launch = T * model.num_kv_heads * model.head_dim * 2 * 2 * (ctx0 + 1)
    peak, peak_kind = _peaks()
    step_bytes = bs64_step_bytes(cfg, world, ctx0 + Kst // 2)
    sec = ms / Kst / 1000.0
    line = {
        "metric": "decode tok/s (bs64, configs[3])", "value": tok_s, "unit": "tok/s", "n_gpus": world,
        "steps": Kst, "warmup": W, "ms_per_step": ms / Kst, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": SYNTH_DATA + "; cached K/V bf16 from the same generator (N(0,1) stand-in)",
        "config": bs64_config(cfg, world, ctx, W, Kst),
        "context": [ctx0, ctx0 + Kst], "step": graph_kind,
        "ep_transport": os.environ.get("MAPLE_EP_TRANSPORT", "p2p") if world > 1 else None,
        "hbm_roofline_step": {"bytes_per_gpu_step": step_bytes, "achieved_gbs": step_bytes / sec / 1e9,
                              "peak_gbs": peak, "frac": step_bytes / sec / 1e9 / peak},
        "roofline": {"kernel": _attn_kernel_name(cache, T, ctx), "bound": "hbm",
                     "achieved": kv_per_launch / (att_us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": kv_per_launch / (att_us * 1e-6) / 1e9 / peak, "traffic": None,
                     "algorithmic_bytes": kv_per_launch, "launch_us": att_us, "peak_kind": f"{peak_kind} hbm_gbs"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * T, "d2h_bytes_per_step": 8 * T},
        "gpu_launches": Kst * (launches_per_step or (12 + _attn_launches(cache)) * cfg["num_hidden_layers"] + 4),
        "gpu_launches_source": ("kernel nodes of this library in the captured step graph x steps"
                                if launches_per_step else "estimate"),
        "clocks": clocks.summary(),
        "device_errors": device_errors,
        "phases_ms_per_step": phases,
        "phases_note": "expert-parallel step captured with timing events at phase boundaries (max over ranks, "
                       "summed over 48 layers; at one GPU the same step with a one-rank exchange)",
    }
    if rank == 0 and emit:
        print(json.dumps(line), flush=True)
    # a CUDA graph holding NCCL calls must be released before the group goes
    import gc

    holder.clear()
    del step, nxt_of
    gc.collect()
    torch.cuda.synchronize(dev)
    if hasattr(ex, "close"):
        ex.close()
    dist.barrier()
    dist.destroy_process_group()
    if device_errors:
        raise SystemExit(f"device error word {device_errors:#x} set during the run: the numbers are not valid")
    return line


def run_long(args):
    """``--batch`` rows (1, 16 or 256) with ``--context`` (65536)
    random cached positions each; every step samples with the fused sampler
    (T=1.0, top_p 0.95, top_k 20) from per-sequence counter-based uniforms.
    Batch 1 scores through FlashHead (4748 clusters x 32, 512 probes) with the
    dense RTN-4 head run alongside off the clock for the top-20 check; batch
    16/256 use the dense batched head.  Batch 256 does not fit (1.65 TB of
    K/V): its rows alias 16 physical cache rows through the row map -- every
    row's K/V is read as issued, the rows sharing a physical row write the
    same new position (last writer wins), so it is a throughput stress only."""
    import torch

    from maple_flash_dgx_spark_b200 import kernels as K
    from maple_flash_dgx_spark_b200.flash_head import attach_flash_head
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM, packed_decode_bytes
    from maple_flash_dgx_spark_b200.synth import fill_kv_cache, synthetic_config, synthetic_tokens, synthetic_weights

    world, rank, local = _dist()
    if world > 1:
        raise SystemExit("--workload long runs one GPU per process")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, ctx = int(args.batch), int(args.context or 65536)
    phys = min(B, 16)
    cfg = synthetic_config(num_layers=args.layers)
    W, Kst = args.warmup, args.steps
    weights = synthetic_weights(cfg, SEED, dev)
    use_flash = B == 1
    t_cluster = 0.0
    if use_flash:
        t0 = time.perf_counter()
        attach_flash_head(cfg, weights, n_clusters=4748, n_probes=512)
        torch.cuda.synchronize(dev)
        t_cluster = time.perf_counter() - t0
    model = MapleForCausalLM.from_weight_dict(cfg, weights, device=dev, use_flash_head=use_flash)
    del weights
    torch.cuda.empty_cache()
    cache = model.make_cache(max_len=ctx + W + Kst + 8, batch=phys)
    fill_kv_cache(cache, SEED, ctx)
    if B > phys:  # aliased rows (throughput stress)
        cache.batch = B
        cache.seqlen = torch.full((B,), ctx, dtype=torch.int64, device=dev)
        cache.seen = [ctx] * B
        cache.row_of = list(range(B))
        cache.row_map = (torch.arange(B, device=dev) % phys).to(torch.int32)
        cache.remap = True
    ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
    ids.copy_(synthetic_tokens(SEED, B, cfg["vocab_size"], dev).reshape(B, 1))
    rng = K.RowUniform(range(1000, 1000 + B), dev)
    ws = K.batched_sampler_workspace(cfg["vocab_size"], 20, B, dev)

    def step():
        logits = model.forward(ids, cache=cache, logits_to_keep=1)
        return K.fused_sample_batched(logits[:, -1, :], rng(), temperature=1.0, top_p=0.95, top_k=20, workspace=ws)

    with torch.inference_mode():
        snap = (cache.seqlen.clone(), list(cache.seen))
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            for _ in range(3):
                step()
                cache.seqlen.copy_(snap[0])
                cache.seen = list(snap[1])
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                nxt = step()
        torch.cuda.current_stream(dev).wait_stream(st)
        torch.cuda.synchronize(dev)
        cache.seqlen.copy_(snap[0])
        cache.seen = list(snap[1])
        for _ in range(W):
            graph.replay()
            ids.copy_(nxt.reshape(B, 1))
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            torch.cuda.nvtx.range_push("maple_decode")
            start.record()
            for _ in range(Kst):
                graph.replay()
                ids.copy_(nxt.reshape(B, 1))
            end.record()
            torch.cuda.synchronize(dev)
            torch.cuda.nvtx.range_pop()
        ms = start.elapsed_time(end)
        cache.advance_host(W + Kst, B)
        tok_s = B * Kst / (ms / 1000.0)
        pin_in = torch.empty(B, 1, dtype=torch.long, pin_memory=True)
        pin_out = torch.empty(B, dtype=torch.long, pin_memory=True)
        pin_in.copy_(ids.cpu())
        ev = torch.cuda.Event()
        ne2e = max(1, min(Kst, 16))
        torch.cuda.synchronize(dev)
        t_0 = time.perf_counter()
        for _ in range(ne2e):
            ids.copy_(pin_in, non_blocking=True)
            graph.replay()
            pin_out.copy_(nxt.reshape(B), non_blocking=True)
            ev.record()
            ev.synchronize()
            pin_in[:, 0] = pin_out
        e2e = B * ne2e / (time.perf_counter() - t_0)
        cache.advance_host(ne2e, B)
        flash = None
        if use_flash:
            # FlashHead vs the dense head on random decode-like hidden states: top-20 recall at 512 probes
            hs = torch.randn(8, 1, 1, cfg["hidden_size"], device=dev).to(torch.bfloat16)
            rec = []
            for h in hs:
                fl = model.lm_head_flash(h).reshape(-1).float()
                de = model.lm_head(h.reshape(1, -1)).reshape(-1).float()
                a = set(torch.topk(fl, 20).indices.tolist())
                b_ = set(torch.topk(de, 20).indices.tolist())
                rec.append(len(a & b_) / 20.0)
            flash = {"n_clusters": 4748, "n_probes": 512, "recall_at_20": sum(rec) / len(rec),
                     "head_bytes": model.lm_head_flash.head_bytes(), "clustering_s": round(t_cluster, 1)}
        att = model.layers[0].self_attn
        q = torch.randn(phys, model.num_heads, 1, model.head_dim, device=dev).to(torch.bfloat16)
        pos = torch.full((phys,), ctx, dtype=torch.int64, device=dev)
        fns = [lambda i=i: K.decode_gqa_attn(q, cache.k[i], cache.v[i], pos, scale=att.scale, window=None,
                                             split_len=cache.split_len, kv_final=True, tensor_cores=cache.attn_tc)
               for i in range(len(model.layers))]
        att_us = _time_graph(fns, dev) * 1000.0 / len(fns)
        kv_per_launch = phys * model.num_kv_heads * model.head_dim * 2 * 2 * (ctx + 1)
    peak, peak_kind = _peaks()
    wb = packed_decode_bytes(cfg)
    head = flash["head_bytes"] if flash else wb["head_bytes"]
    kv_step = B * cfg["num_hidden_layers"] * cfg["num_key_value_heads"] * cfg["head_dim"] * 2 * 2 * (ctx + W + Kst // 2)
    expert_rows = min(B * cfg["num_experts_per_tok"], cfg["num_experts"])
    weights_step = wb["packed_weight_bytes"] - wb["head_bytes"] + head + wb["expert_bytes"] * (expert_rows /
                                                                                             cfg["num_experts_per_tok"] - 1)
    step_bytes = int(weights_step + kv_step)
    sec = ms / Kst / 1000.0
    line = {
        "metric": f"decode tok/s (long context {ctx}, bs{B}, configs[4])", "value": tok_s, "unit": "tok/s",
        "n_gpus": 1, "steps": Kst, "warmup": W, "ms_per_step": ms / Kst, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": SYNTH_DATA + "; cached K/V bf16 from the same generator (N(0,1) stand-in)",
        "config": {"workload": f"configs[4]: bs{B}, {ctx} cached positions, sampled T=1.0 top_p=0.95 top_k=20, "
                               f"per-sequence counter RNG, {'FlashHead 4748x32 / 512 probes' if use_flash else 'dense RTN-4 head'}",
                   "global_batch": B, "seq_len": ctx, "physical_cache_rows": phys,
                   "parallelism": "single", "l2": f"{step_bytes / 1e9:.1f} GB streamed per step (> 126 MB L2)"},
        "hbm_roofline_step": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes / sec / 1e9, "peak_gbs": peak,
                              "frac": step_bytes / sec / 1e9 / peak},
        "roofline": {"kernel": _attn_kernel_name(cache, phys, ctx), "bound": "hbm",
                     "achieved": kv_per_launch / (att_us * 1e-6) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": kv_per_launch / (att_us * 1e-6) / 1e9 / peak, "traffic": None,
                     "algorithmic_bytes": kv_per_launch, "launch_us": att_us, "peak_kind": f"{peak_kind} hbm_gbs"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 8 * B},
        "gpu_launches": Kst * ((5 + _attn_launches(cache)) * cfg["num_hidden_layers"] + 8),
        "clocks": clocks.summary(),
    }
    if flash:
        line["flash_head"] = flash
    print(json.dumps(line), flush=True)


def _event_ms(fn, reps: int) -> float:
    """Mean CUDA-event time of ``fn`` over ``reps`` calls after one warm call."""
    import torch

    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_attn(args):
    """The decode-attention kernels alone: ``--batch`` rows x ``--context``
    positions of one layer's bf16 cache (seeded random q / K / V, 32 query and
    4 KV heads of 128 dims), the tensor-core kernel (+ its merge launch) and
    the canonical CUDA-core kernel, eager launches timed with CUDA events."""
    import torch

    from maple_flash_dgx_spark_b200 import kernels as K

    dev = torch.device("cuda", 0)
    rows, ctx, reps = int(args.batch), int(args.context or 8192), max(int(args.steps), 1)
    Hq, Hkv, D = 32, 4, 128
    T = ctx + 16
    g = torch.Generator(device=dev).manual_seed(0)
    kc = torch.randn(rows, Hkv, T, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(rows, Hkv, T, D, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(rows, Hq, 1, D, device=dev, generator=g).to(torch.bfloat16)
    sl = torch.full((rows,), ctx - 1, device=dev, dtype=torch.int64)
    nbytes = rows * Hkv * ctx * D * 2 * 2
    peak, peak_kind = _peaks()
    out = {"workload": f"decode attention alone, {rows} rows x {ctx} positions, bf16 cache", "algorithmic_bytes": nbytes}
    for tc in (True, False):
        us = _event_ms(lambda: K.decode_gqa_attn(q, kc, vc, sl, scale=D ** -0.5, window=None, split_len=128,
                                                 tensor_cores=tc), reps) * 1000.0
        out["tensor_cores" if tc else "cuda_cores"] = {"us_per_launch": us, "gbs": nbytes / us / 1e3,
                                                       "frac": nbytes / us / 1e3 / peak}
    out["peak_gbs"] = peak
    out["peak_kind"] = f"{peak_kind} hbm_gbs"
    print(json.dumps(out), flush=True)


def run_kmeans(args):
    """FlashHead clustering of the configs[4] head: the balanced spherical
    k-means (CUDA) of ``--rows`` unit rows of the head's 2048 columns into
    rows/32 clusters, ``--steps`` iterations from the reference's initial draw.
    Reports the wall time per iteration (host bookkeeping included), the
    assignment launch alone (CUDA events) against fp32 CUDA-core FMA
    throughput, and the balance of the result."""
    import torch

    from maple_flash_dgx_spark_b200 import _lib
    from maple_flash_dgx_spark_b200.flash_head import balanced_spherical_kmeans

    dev = torch.device("cuda", 0)
    n, d = int(args.rows), 2048
    k = n // 32
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(n, d, device=dev, generator=g)
    w = (w / (w.norm(dim=1, keepdim=True) + 1e-8)).contiguous()
    iters = max(int(args.steps), 1)
    balanced_spherical_kmeans(w, k, n_iter=1)  # warm
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    cent, labels = balanced_spherical_kmeans(w, k, n_iter=iters)
    torch.cuda.synchronize(dev)
    wall = (time.perf_counter() - t0) / iters
    L = _lib.lib()
    lab = torch.empty(n, dtype=torch.int32, device=dev)
    best = torch.empty(n, dtype=torch.float32, device=dev)
    ws = torch.empty(L.maple_km_assign_workspace_bytes(n, k), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    def assign():
        _lib.check(L.maple_km_assign(w.data_ptr(), n, d, cent.data_ptr(), k, lab.data_ptr(), best.data_ptr(),
                                     ws.data_ptr(), ws.numel(), st), "km_assign")

    ms = _event_ms(assign, 5)
    flops = 2.0 * n * k * d
    counts = torch.bincount(labels.long(), minlength=k)
    fp32_nominal = 148 * 128 * 2 * 1.965e9 / 1e12  # TFLOP/s: 148 SMs x 128 FP32 lanes x FMA x 1965 MHz
    print(json.dumps({
        "workload": f"FlashHead balanced spherical k-means, {n} x {d} unit rows into {k} clusters of 32",
        "iterations": iters, "s_per_iteration": wall,
        "assign_ms": ms, "assign_tflops": flops / (ms * 1e-3) / 1e12,
        "assign_frac_of_fp32_nominal": flops / (ms * 1e-3) / 1e12 / fp32_nominal,
        "fp32_nominal_tflops": fp32_nominal,
        "balanced": bool((counts == 32).all()), "device_errors": _lib.take_device_errors(dev)}), flush=True)


def run_prefill(args):
    """Prompt prefill of the configs[2] model (``--layers`` layers, 512-token
    prompt) with the tcgen05 grouped expert GEMM and with the mma.sync one
    (time to first token, CUDA events), plus the grouped expert SwiGLU GEMM
    alone at prefill routing (512 tokens x top-8 over 64 experts, seeded
    random codes)."""
    import torch

    from maple_flash_dgx_spark_b200 import kernels as K
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_tokens, synthetic_weights

    dev = torch.device("cuda", 0)
    reps = max(int(args.steps), 1)
    g = torch.Generator(device=dev).manual_seed(0)
    T, E, k, H, I = PROMPT_LEN, 64, 8, 2048, 1024
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    ug = (torch.randint(0, 2 ** 31, (E, 2 * I, H // 16), device=dev, generator=g, dtype=torch.int64)
          .to(torch.int32) & 0x55555555).view(torch.uint32)  # codes 0/1 (every 2-bit field < 3)
    ua = (torch.rand(E, 2 * I, device=dev, generator=g) * 0.02 + 1e-3).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device=dev, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    plan = K.moe_plan(ids, E)
    out = {"workload": f"configs[2] {PROMPT_LEN}-token prefill, {args.layers} layers; grouped SwiGLU at "
                       f"{T} tokens x top-{k} over {E} experts"}
    default = K.TC_GEMM_MIN_SLOTS
    try:
        for tc in (True, False):
            K.TC_GEMM_MIN_SLOTS = 0 if tc else 10 ** 9
            out[f"grouped_swiglu_us_{'tcgen05' if tc else 'mma_sync'}"] = _event_ms(
                lambda: K.ternary_expert_swiglu(x, ug, ua, ids, plan=plan), reps) * 1000.0
        if args.layers > 0:
            cfg = synthetic_config(num_layers=args.layers)
            model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, SEED, dev), device=dev)
            prompt = synthetic_tokens(SEED, PROMPT_LEN, cfg["vocab_size"], dev).reshape(1, -1)
            for tc in (True, False):
                K.TC_GEMM_MIN_SLOTS = 0 if tc else 10 ** 9
                ms = _event_ms(lambda: model.forward(prompt, cache=model.make_cache(max_len=PROMPT_LEN + 8)), reps)
                out[f"ttft_ms_{'tcgen05' if tc else 'mma_sync'}"] = ms
    finally:
        K.TC_GEMM_MIN_SLOTS = default
    print(json.dumps(out), flush=True)


def swiglu_roofline(model, prompt, dev):
    """Average duration of one batch-1 expert SwiGLU launch over the 48
    layers' weights (cold: 403 MB > L2), captured in a graph and timed with
    CUDA events; returns (us per launch, algorithmic bytes per launch)."""
    import torch

    from maple_flash_dgx_spark_b200 import kernels as K

    H = model.hidden_size
    x = model.embed(prompt[:1])
    ids = [K.router_topk(x, lay.mlp.gate_weight, model.top_k)[0] for lay in model.layers]
    for lay, idx in zip(model.layers, ids):
        lay.mlp.up_gate.swiglu(x, idx)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for lay, idx in zip(model.layers, ids):
                lay.mlp.up_gate.swiglu(x, idx)
    torch.cuda.current_stream(dev).wait_stream(s)
    g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    us = a.elapsed_time(b) * 1000.0 / (reps * len(model.layers))
    k, inter = model.top_k, model.moe_intermediate
    nbytes = k * (2 * inter * H // 4 + 2 * inter * 2) + H * 2 + k * inter * 2
    return us, nbytes


def _step_launches(n_layers: int) -> int:
    """This engine's kernel launches in one batch-1 decode step: per layer QKV,
    attention with QK-norm / RoPE / K-V store, O, add-norm + router, SwiGLU,
    down (seven with the QK-norm as its own launch); plus embedding, final
    norm, head and argmax."""
    return _attn_launches() * n_layers + 4 * n_layers + 4


def _attn_kernel_name(cache, rows: int, ctx: int) -> str:
    """The decode-attention kernel the model runs for this cache, as the ncu
    launch list names it, plus its merge launch."""
    if cache.attn_tc:
        return f"gqa_tc_kernel + gqa_merge_kernel (tensor-core decode attention, {rows} rows x {ctx} positions)"
    return f"gqa_decode_kernel (CUDA-core decode attention, {rows} rows x {ctx} positions, split-K)"


def _attn_launches(cache=None) -> int:
    """Launches of the attention block of a decode layer besides O: QKV + the
    fused attention, or QKV + QK-norm + attention (the model fuses only where
    a row's attention splits fit one cluster)."""
    from maple_flash_dgx_spark_b200.model import _QK_FUSED_MAX_SPLITS, _fused_qk_attention

    splits = 1 if cache is None else -(-int(cache.max_len) // int(cache.split_len))
    return 2 if _fused_qk_attention() and splits <= _QK_FUSED_MAX_SPLITS else 3


def op_breakdown(model, cache, dev):
    """Warm in-graph time of each operator of the batch-1 decode step: run one
    step layer by layer keeping every intermediate, then replay each operator
    over the 48 layers in its own CUDA graph (launched like the decode step,
    with PDL).  The attention replays re-store the same K/V row."""
    import torch

    from maple_flash_dgx_spark_b200 import kernels as K

    pos = torch.full((1,), int(cache.seen[0]) - 1, dtype=torch.int64, device=dev)
    rot = model.rotary
    steps = {name: [] for name in ("qkv_gemv", "attention_qk", "o_gemv", "add_norm_router", "expert_swiglu",
                                   "expert_down_reduce")}
    h = model.embed(torch.ones(1, dtype=torch.long, device=dev))
    with torch.inference_mode():
        for i, lay in enumerate(model.layers):
            at, mlp = lay.self_attn, lay.mlp
            kc, vc = cache.k[i][:1], cache.v[i][:1]
            pl = lay.post_attention_layernorm.weight

            def attn_qk(at=at, kc=kc, vc=vc, qkv=None):
                return K.decode_gqa_attn_qk(qkv, at.q_norm.weight, at.k_norm.weight, rot.cos_table, rot.sin_table,
                                            kc, vc, pos, num_heads=at.num_heads, num_kv_heads=at.num_kv_heads,
                                            head_dim=at.head_dim, rotary_dim=rot.rotary_dim, use_rope=at.use_rope,
                                            eps=model.rms_eps, scale=at.scale, window=None,
                                            split_len=cache.split_len)

            qkv = at.qkv_proj(h, rms_weight=lay.input_layernorm.weight, rms_eps=model.rms_eps)
            attn = attn_qk(qkv=qkv)
            o = at.o_proj(attn.reshape(1, -1))
            res, normed, idx, wt = K.add_rms_norm_router_topk(h, o, pl, model.rms_eps, mlp.gate_weight, mlp.top_k)
            hs = mlp.up_gate.swiglu(normed, idx)
            h2 = mlp.down.down_reduce(hs, idx, wt, residual=res)
            steps["qkv_gemv"].append(lambda at=at, h=h, lay=lay: at.qkv_proj(
                h, rms_weight=lay.input_layernorm.weight, rms_eps=model.rms_eps))
            steps["attention_qk"].append(lambda f=attn_qk, qkv=qkv: f(qkv=qkv))
            steps["o_gemv"].append(lambda at=at, attn=attn: at.o_proj(attn.reshape(1, -1)))
            steps["add_norm_router"].append(lambda h=h, o=o, pl=pl, mlp=mlp: K.add_rms_norm_router_topk(
                h, o, pl, model.rms_eps, mlp.gate_weight, mlp.top_k))
            steps["expert_swiglu"].append(lambda mlp=mlp, normed=normed, idx=idx: mlp.up_gate.swiglu(normed, idx))
            steps["expert_down_reduce"].append(lambda mlp=mlp, hs=hs, idx=idx, wt=wt, res=res: mlp.down.down_reduce(
                hs, idx, wt, residual=res))
            h = h2
        out = {}
        for name, fns in steps.items():
            for f in fns:
                f()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream(dev)
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    for f in fns:
                        f()
            torch.cuda.current_stream(dev).wait_stream(st)
            g.replay()
            torch.cuda.synchronize(dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(10):
                g.replay()
            b.record()
            torch.cuda.synchronize(dev)
            out[name] = round(a.elapsed_time(b) * 1000.0 / (10 * len(fns)), 2)
    return out


def _profiled_traffic(name: str):
    """DRAM bytes per launch of ``name`` from the committed ncu summary, if any."""
    p = REPO / "profiles" / f"{name}.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


if __name__ == "__main__":
    main()
