"""Packed-ternary-v1 checkpoint writer (the reader is
``MapleForCausalLM.from_packed``).

Reference: convert.py:257-303 (config and shard layout) and the shard set
``model.py:664-706`` reads: ``config.json`` with ``maple_run.format =
"packed-ternary-v1"``, ``model.safetensors.index.json`` mapping every tensor
to a shard, ``model-0000i-of-0000n.safetensors`` shards, and FlashHead data in
``model-flashhead.safetensors`` (loaded only on request).  Tensor names and
dtypes are the reference's: ternary codes uint32 ``[N, K/16]`` (experts
``[E, N, K/16]``) with ``row_alpha``, RTN-4 codes uint32 ``[N, K/8]`` with
``scales`` (and ``biases`` unless symmetric).
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

FLASHHEAD_SHARD = "model-flashhead.safetensors"
PACKED_FORMAT = "packed-ternary-v1"


def _tensor_bytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def save_packed(model_dir, config: dict, weights: dict[str, torch.Tensor], *,
                max_shard_bytes: int = 4 << 30) -> dict:
    """Write ``weights`` (device or host tensors) and ``config`` as a
    packed-ternary-v1 directory; returns the index.  Tensors are copied to the
    host shard by shard."""
    from safetensors.torch import save_file

    fmt = (config.get("maple_run") or {}).get("format")
    if fmt != PACKED_FORMAT:
        raise ValueError(f"config maple_run.format must be {PACKED_FORMAT!r}, got {fmt!r}.")
    out = Path(model_dir).expanduser()
    out.mkdir(parents=True, exist_ok=True)
    body = sorted(k for k in weights if not k.startswith("lm_head_flash."))
    flash = sorted(k for k in weights if k.startswith("lm_head_flash."))
    shards: list[list[str]] = [[]]
    size = 0
    for k in body:
        b = _tensor_bytes(weights[k])
        if shards[-1] and size + b > max_shard_bytes:
            shards.append([])
            size = 0
        shards[-1].append(k)
        size += b
    n = len(shards)
    weight_map: dict[str, str] = {}
    total = 0
    for i, keys in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file({k: weights[k].detach().contiguous().cpu() for k in keys}, str(out / name),
                  metadata={"format": "pt"})
        for k in keys:
            weight_map[k] = name
            total += _tensor_bytes(weights[k])
    if flash:
        save_file({k: weights[k].detach().contiguous().cpu() for k in flash}, str(out / FLASHHEAD_SHARD),
                  metadata={"format": "pt"})
        for k in flash:
            weight_map[k] = FLASHHEAD_SHARD
            total += _tensor_bytes(weights[k])
    index = {"metadata": {"total_size": total}, "weight_map": weight_map}
    (out / "model.safetensors.index.json").write_text(json.dumps(index, indent=2, sort_keys=True))
    (out / "config.json").write_text(json.dumps(config, indent=2, sort_keys=True))
    return index


def load_packed_weights(model_dir, *, device="cpu", flash_head: bool = False) -> tuple[dict, dict]:
    """``(config, weights)`` of a packed-ternary-v1 directory without building a
    model (host or device tensors)."""
    from safetensors.torch import load_file

    d = Path(model_dir).expanduser()
    config = json.loads((d / "config.json").read_text())
    index = json.loads((d / "model.safetensors.index.json").read_text())
    weights: dict[str, torch.Tensor] = {}
    for name in sorted(set(index["weight_map"].values())):
        if name == FLASHHEAD_SHARD and not flash_head:
            continue
        weights.update(load_file(str(d / name), device=str(device)))
    return config, weights
