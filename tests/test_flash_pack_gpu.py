"""GPU packing kernels and the FlashHead driver vs the reference's pack.py
golden vectors and the CPU oracle: bit-exact (GPU).

Reference coverage: tests/test_pack.py (known words, ternarize, alpha, zero
rows) and tests/test_flash_head.py:89-112 (all probes == exact head).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from tests.golden.make_pack_golden import RTN, TERNARIZE, rtn_input, ternarize_input
from tests.helpers import bf, randn_bf, rng, to_dev, to_np

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).parent / "golden" / "reference_pack.npz")


@pytest.fixture(scope="module")
def P():
    from maple_flash_dgx_spark_b200 import pack

    return pack


@pytest.mark.parametrize("seed,n,k", TERNARIZE)
def test_ternarize_equals_reference(cuda, P, seed, n, k):
    w = ternarize_input(seed, n, k)
    packed, alpha = P.ternarize(to_dev(w, cuda))
    np.testing.assert_array_equal(to_np(packed.view(torch.int32)).view(np.uint32), GOLD[f"tern_{seed}_packed"])
    np.testing.assert_array_equal(to_np(alpha), GOLD[f"tern_{seed}_alpha"])


def test_ternarize_bf16_weights(cuda, P):
    w = randn_bf(rng(8), 5, 2048, scale=0.02)
    packed, alpha = P.ternarize(to_dev(w, cuda, torch.bfloat16))
    p_o, a_o = oracle.ternarize(w)
    np.testing.assert_array_equal(to_np(packed.view(torch.int32)).view(np.uint32), p_o)
    np.testing.assert_array_equal(to_np(alpha), bf(a_o))
    assert alpha.dtype == torch.bfloat16


@pytest.mark.parametrize("seed,n,k,g", RTN)
def test_rtn_equals_reference(cuda, P, seed, n, k, g):
    packed, scales, biases = P.quantize_rtn(to_dev(rtn_input(seed, n, k), cuda), group_size=g)
    np.testing.assert_array_equal(to_np(packed.view(torch.int32)).view(np.uint32), GOLD[f"rtn_{seed}_packed"])
    np.testing.assert_array_equal(to_np(scales), GOLD[f"rtn_{seed}_scales"])
    np.testing.assert_array_equal(to_np(biases), GOLD[f"rtn_{seed}_biases"])
    deq = P.dequantize_rtn(packed, scales, biases, group_size=g)
    np.testing.assert_array_equal(to_np(deq), oracle.dequantize_rtn(GOLD[f"rtn_{seed}_packed"],
                                                                    GOLD[f"rtn_{seed}_scales"],
                                                                    GOLD[f"rtn_{seed}_biases"], g))


def test_pack_unpack_round_trip_and_overflow(cuda, P):
    rs = rng(2)
    c2 = rs.randint(0, 3, size=(7, 2048)).astype(np.uint8)
    c4 = rs.randint(0, 16, size=(3, 512)).astype(np.uint8)
    p2 = P.pack_2bit(to_dev(c2, cuda))
    p4 = P.pack_4bit(to_dev(c4, cuda))
    np.testing.assert_array_equal(to_np(p2.view(torch.int32)).view(np.uint32), oracle.pack_2bit(c2))
    np.testing.assert_array_equal(to_np(p4.view(torch.int32)).view(np.uint32), oracle.pack_4bit(c4))
    np.testing.assert_array_equal(to_np(P.unpack_2bit(p2)), c2)
    np.testing.assert_array_equal(to_np(P.unpack_4bit(p4)), c4)
    ov = P.pack_2bit(to_dev(GOLD["pack_overflow_codes"].astype(np.uint8), cuda))
    np.testing.assert_array_equal(to_np(ov.view(torch.int32)).view(np.uint32), GOLD["pack_overflow_words"])


@pytest.mark.parametrize("n,k,dt", [(4748, 512, torch.bfloat16), (4748, 512, torch.float32), (151936, 64, torch.float32),
                                    (100, 100, torch.float32), (33, 1, torch.bfloat16)])
def test_topk_select(cuda, n, k, dt):
    from maple_flash_dgx_spark_b200.flash_head import topk_select

    rs = rng(n + k)
    x = np.round(rs.standard_normal(n) * 6).astype(np.float32) / 4  # ties
    x[rs.randint(0, n)] = np.nan
    x[rs.randint(0, n)] = -np.inf
    x = bf(x) if dt == torch.bfloat16 else x
    sel = topk_select(to_dev(x, cuda, dt), k)
    np.testing.assert_array_equal(to_np(sel), oracle.topk_select(x, k))


def _tiny_flash(cuda, n_probes, force=(0, 7, 4095)):
    from maple_flash_dgx_spark_b200.flash_head import attach_flash_head, build_flash_head
    from maple_flash_dgx_spark_b200.linear import PackedRTN4Linear
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_weights

    cfg = synthetic_config(num_layers=1, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2, inter=128,
                           vocab=4096)
    weights = synthetic_weights(cfg, 5, cuda)
    attach_flash_head(cfg, weights, n_clusters=128, n_probes=n_probes, force_tokens=force)
    head = PackedRTN4Linear(weights["lm_head.weight"], weights["lm_head.scales"].to(torch.bfloat16),
                            weights.get("lm_head.biases"), group_size=cfg["maple_run"]["rtn_4bit"]["group_size"])
    w = dict(weights)
    w["lm_head_flash.centroids.scales"] = w["lm_head_flash.centroids.scales"].to(torch.bfloat16)
    w["lm_head_flash.centroids.biases"] = w["lm_head_flash.centroids.biases"].to(torch.bfloat16)
    fh = build_flash_head(config=cfg, lm_head=head, weights=w, device=cuda, dtype=torch.bfloat16)
    return cfg, head, fh


def _u32np(t):
    return to_np(t.contiguous().view(torch.int32)).view(np.uint32)


def _sf(t):
    return None if t is None else to_np(t.float())


@pytest.mark.parametrize("n_probes", [16, 128])
def test_flash_head_equals_oracle(cuda, n_probes):
    cfg, head, fh = _tiny_flash(cuda, n_probes)
    hidden = to_dev(randn_bf(rng(12), 1, 1, 256), cuda, torch.bfloat16)
    full = to_np(fh(hidden)).reshape(-1)
    want, cids = oracle.flash_head(
        to_np(hidden), centroids_weight=_u32np(fh.centroids_weight), centroids_scales=_sf(fh.centroids_scales),
        centroids_biases=_sf(fh.centroids_biases), centroid_group=fh.centroid_group_size,
        token_map=to_np(fh.token_map), head_weight=_u32np(fh.head_weight), head_scales=_sf(fh.head_scales),
        head_biases=_sf(fh.head_biases), group_size=fh.group_size, force_ids=to_np(fh.force_ids),
        force_weight=_u32np(fh.force_weight), force_scales=_sf(fh.force_scales), force_biases=_sf(fh.force_biases),
        n_probes=n_probes, vocab_size=cfg["vocab_size"])
    np.testing.assert_array_equal(to_np(fh._cluster_ids), cids)
    np.testing.assert_array_equal(full, want)
    if n_probes == fh.n_clusters:
        # every cluster probed: the exact head, bit for bit (reference test_flash_head.py:89-112)
        np.testing.assert_array_equal(full, to_np(head(hidden.reshape(1, -1))).reshape(-1))
    else:
        assert np.isinf(full).sum() == cfg["vocab_size"] - len(np.unique(np.concatenate(
            [to_np(fh.token_map)[cids].reshape(-1), to_np(fh.force_ids)])))


def test_model_decode_with_flash_head(cuda):
    """Greedy decode through FlashHead with every cluster probed equals the
    dense-head decode; the FlashHead step is captured in the decode graph."""
    from maple_flash_dgx_spark_b200.flash_head import attach_flash_head
    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_tokens, synthetic_weights

    cfg = synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2, inter=128,
                           vocab=4096)
    weights = synthetic_weights(cfg, 6, cuda)
    dense = MapleForCausalLM.from_weight_dict(cfg, dict(weights), device=cuda)
    attach_flash_head(cfg, weights, n_clusters=64, n_probes=64)
    flash = MapleForCausalLM.from_weight_dict(cfg, weights, device=cuda, use_flash_head=True)
    prompt = synthetic_tokens(6, 9, cfg["vocab_size"], cuda).cpu()
    a = run_generate(dense, prompt, max_tokens=12, temperature=0.0, log=None)
    b = run_generate(flash, prompt, max_tokens=12, temperature=0.0, log=None)
    assert a.token_ids == b.token_ids
    assert b.used_graph


def test_flash_head_full_vocab_all_probes_exact(cuda):
    """configs[4]'s head (151936 x 2048, RTN-4 group 128) in 4748 clusters of
    32: with every cluster probed FlashHead returns the dense head's logits
    bit for bit (reference tests/test_flash_head.py:89-112); at the default
    512 probes the probed clusters' rows and the forced tokens equal the
    dense logits, every other entry is -inf, and the top-20 recall is
    printed."""
    from maple_flash_dgx_spark_b200.flash_head import attach_flash_head
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_weights

    cfg = synthetic_config(num_layers=1)
    assert cfg["vocab_size"] == 151936 and cfg["hidden_size"] == 2048
    weights = synthetic_weights(cfg, 7, cuda)
    force = [151643, 151645]
    attach_flash_head(cfg, weights, n_clusters=4748, n_probes=4748, force_tokens=force)
    full = MapleForCausalLM.from_weight_dict(cfg, dict(weights), device=cuda, use_flash_head=True)
    cfg512 = dict(cfg)
    cfg512["flash_head"] = dict(cfg["flash_head"], n_probes=512)
    part = MapleForCausalLM.from_weight_dict(cfg512, dict(weights), device=cuda, use_flash_head=True)
    g = torch.Generator(device="cpu").manual_seed(29)
    recall = []
    for _ in range(4):
        h = torch.randn(1, 1, cfg["hidden_size"], generator=g).to(torch.bfloat16).to(cuda)
        dense = full.lm_head(h.reshape(1, -1)).reshape(-1)
        got = full.lm_head_flash(h).reshape(-1)
        assert torch.equal(got.view(torch.int16), dense.view(torch.int16))
        sub = part.lm_head_flash(h).reshape(-1)
        fh = part.lm_head_flash
        probed = fh.token_map[fh._cluster_ids.long()].reshape(-1).long()
        keep = torch.zeros_like(sub, dtype=torch.bool)
        keep[probed] = True
        keep[torch.tensor(force, device=cuda)] = True
        assert torch.equal(sub[keep].view(torch.int16), dense[keep].view(torch.int16))
        assert bool(torch.isneginf(sub[~keep]).all())
        top_d = set(torch.topk(dense.float(), 20).indices.tolist())
        top_f = set(torch.topk(sub.float(), 20).indices.tolist())
        recall.append(len(top_d & top_f) / 20)
    print(f"FlashHead 4748x32, 512 probes: top-20 recall {sum(recall) / len(recall):.3f} on random hidden states")
