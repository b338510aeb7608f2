"""Greedy-decode golden ids of the full configs[2] model from the CPU oracle.

    python tests/golden/make_cfg2_greedy.py

Builds the 48-layer synthetic model (seed 2) on the host with the oracle's own
generator, feeds the 512-token synthetic prompt token by token through the
oracle's restatement of the reference decode step, and records in
tests/golden/cfg2_greedy.json (about 10 minutes on 8 cores):

* the first 64 greedy ids;
* for each of those 64 steps, the SHA-1 of the step's bf16 logits (the 151936
  bf16 bit patterns, little-endian) -- a bit-exact fingerprint of the whole
  step, routing of all 48 layers included, that the greedy ids alone (random
  weights drive the output towards a few tokens) cannot give;
* each step's top-1/top-2 logit margin.
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import hashlib  # noqa: E402

import numpy as np  # noqa: E402

import oracle  # noqa: E402
from maple_flash_dgx_spark_b200.synth import synthetic_config  # noqa: E402  (config dict only)
from oracle.model import OracleModel, synth_tokens  # noqa: E402


def logits_sha1(logits) -> str:
    """SHA-1 of a logits row's bf16 bit patterns."""
    bits = oracle.bf16_bits(np.asarray(logits, np.float32)).astype("<u2")
    return hashlib.sha1(bits.tobytes()).hexdigest()


SEED, PROMPT, N_NEW, SPLIT = 2, 512, 64, 64


def main():
    cfg = synthetic_config()
    t0 = time.time()
    m = OracleModel(cfg, SEED, max_len=PROMPT + N_NEW, split_len=SPLIT)
    prompt = synth_tokens(SEED, PROMPT, cfg["vocab_size"])
    for i, tok in enumerate(prompt[:-1]):
        m.step(int(tok))
        if (i + 1) % 64 == 0:
            print(f"  prefill {i + 1}/{PROMPT} ({time.time() - t0:.0f}s)", flush=True)
    ids, shas, margins = [], [], []
    tok = int(prompt[-1])
    for _ in range(N_NEW):
        tok, logits = m.step(tok, want_logits=True)
        top2 = np.sort(logits)[-2:]
        ids.append(tok)
        shas.append(logits_sha1(logits))
        margins.append(float(top2[1] - top2[0]))
    out = {"seed": SEED, "prompt_len": PROMPT, "n_new": N_NEW, "split_len": SPLIT, "max_len": PROMPT + N_NEW,
           "ids": ids, "logits_sha1": shas, "top2_margin": margins, "oracle_seconds": round(time.time() - t0, 1)}
    (HERE / "cfg2_greedy.json").write_text(json.dumps(out, indent=1))
    print(out)


if __name__ == "__main__":
    main()
