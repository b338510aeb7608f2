"""Greedy-decode golden ids of the full configs[2] model from the CPU oracle.

    python tests/golden/make_cfg2_greedy.py

Builds the 48-layer synthetic model (seed 2) on the host with the oracle's own
generator, feeds the 512-token synthetic prompt token by token through the
oracle's restatement of the reference decode step, and records the first 64
greedy ids in tests/golden/cfg2_greedy.json (about 10 minutes on 8 cores).
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from maple_flash_dgx_spark_b200.synth import synthetic_config  # noqa: E402  (config dict only)
from oracle.model import OracleModel, synth_tokens  # noqa: E402

SEED, PROMPT, N_NEW, SPLIT = 2, 512, 64, 64


def main():
    cfg = synthetic_config()
    t0 = time.time()
    m = OracleModel(cfg, SEED, max_len=PROMPT + N_NEW, split_len=SPLIT)
    prompt = synth_tokens(SEED, PROMPT, cfg["vocab_size"])
    ids = m.greedy(prompt, N_NEW, log_every=64)
    out = {"seed": SEED, "prompt_len": PROMPT, "n_new": N_NEW, "split_len": SPLIT, "max_len": PROMPT + N_NEW,
           "ids": ids, "oracle_seconds": round(time.time() - t0, 1)}
    (HERE / "cfg2_greedy.json").write_text(json.dumps(out, indent=1))
    print(out)


if __name__ == "__main__":
    main()
