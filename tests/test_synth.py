"""The synthetic Zipf(1.1) workload of the prefill configs, on CPU: the
per-expert targets, and the routing that the calibrated router bias produces
for the benchmark's own seeds through the oracle's router, with the
butterquant router's centring (which must keep the skew)."""
import numpy as np
import torch

import synth
from oracle import oracle as O

H, E, TOPK = O.H, O.E, O.TOPK


def test_zipf_targets():
    T = 4096
    t = synth.zipf_targets(T)
    assert abs(t.sum() - 8 * T) < 1e-6 * 8 * T
    assert t.max() <= T + 1e-9
    assert (np.diff(t) <= 1e-9).all()             # non-increasing in expert rank
    assert t[0] == T                              # 22.6 % share capped at one route per token
    w = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    assert np.allclose(t[-40:] / t[-41], w[-40:] / w[-41])   # uncapped tail keeps the power law


def test_zipf_routing_tracks_targets_through_centred_router():
    """The benchmark's layer seed and first token batch (bench.py: make_layer
    seed 0x6E6D6F45, zipf_tokens seed 1000): the head experts' route counts
    through the oracle router, bf16 router and centred (butterquant) router
    alike, track the Zipf targets."""
    g = torch.Generator()
    g.manual_seed(0x6E6D6F45)
    # make_layer draws router_proj first from this generator
    router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    raw = {"router_proj": router, "router_scale": torch.ones(H, dtype=torch.bfloat16)}
    z = synth.apply_zipf(raw)
    wr = synth.to_numpy(z["router_proj"])
    T = 4096
    x = synth.to_numpy(synth.zipf_tokens(T, seed=1000))
    rs = O.bake_router_scale(synth.to_numpy(raw["router_scale"]))
    pes = O.f32_to_bf16(np.ones(E, np.float32))
    tgt = synth.zipf_targets(T)
    counts = []
    for w in (wr, O.router_center(wr)):
        idx, _, _ = O.router(x, w, rs, pes)
        cnt = np.bincount(idx.reshape(-1), minlength=E)
        assert cnt.sum() == 8 * T
        assert (np.abs(cnt[:8] - tgt[:8]) <= 0.05 * tgt[:8]).all(), (cnt[:8], tgt[:8])
        assert cnt[:16].sum() > 0.6 * 8 * T       # uniform routing would give 12.5 %
        counts.append(cnt)
    # centring shifts every logit of a token alike: same selection up to margins
    assert np.abs(counts[0] - counts[1]).max() <= 0.02 * T


def test_balanced_placement_of_the_zipf_load():
    """gmoe.balanced_placement (the ep-prefill-16k workload's expert
    placement): 128/G experts per rank, and the Zipf(1.1) target load of
    16384 tokens spread within 1 % of even at G = 2 and 4; at G = 8 the hottest
    expert alone is a full rank's share, which bounds the spread (1.17 against
    5.1 for contiguous blocks)."""
    import gmoe
    t = synth.zipf_targets(16384)
    for G, bound in ((2, 1.01), (4, 1.01), (8, 1.17)):
        rank_of = np.asarray(gmoe.balanced_placement(t, G))
        assert (np.bincount(rank_of, minlength=G) == E // G).all()
        load = np.bincount(rank_of, weights=t, minlength=G)
        contiguous = np.bincount(np.arange(E) // (E // G), weights=t, minlength=G)
        assert load.max() / load.mean() <= bound
        assert contiguous.max() / contiguous.mean() > 1.7
