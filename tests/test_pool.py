"""Expert residency: the cache policy pinned against the reference's own
FrequencyWeightedCache trace (tests/golden/cache_trace.npz, made by
tests/golden/make_golden.py), and the HBM slot pool against the resident
layer forward."""
import os

import numpy as np
import pytest

from conftest import REPO

GOLDEN = os.path.join(REPO, "tests", "golden", "cache_trace.npz")


@pytest.fixture(scope="module")
def P():
    from expertflow_b200 import build

    build.build()
    from expertflow_b200 import pool

    return pool


def test_policy_replays_reference_cache_trace(P):
    """Every hit/miss, every per-token eviction count and every resident set of
    the reference run (budget 96 over 4 layers x 128 experts, decay 0.95)."""
    z = np.load(GOLDEN)
    pol = P.CachePolicy(int(z["budget"]), float(z["decay"]))
    tok = 0
    for key, hit in zip(z["accesses"].tolist(), z["hits"].tolist()):
        if key == -1:
            continue
        if key == -2:  # end of token: trim
            ev = pol.trim()
            assert len(ev) == int(z["evicted"][tok]), tok
            res = z["resident"][tok]
            assert pol.keys() == sorted(int(r) for r in res if r >= 0), tok
            tok += 1
            continue
        h = pol.get(key)
        assert int(h) == hit, (tok, key)
        if not h:
            pol.put(key)
    assert tok == len(z["evicted"])
    pol.close()


def test_policy_tie_breaks_to_first_inserted_and_decays(P):
    pol = P.CachePolicy(2, 0.5)
    for k in (7, 3, 9):
        assert not pol.get(k)
        pol.put(k)
    assert pol.trim() == [7]          # equal scores: the first inserted goes
    assert pol.keys() == [3, 9]
    assert pol.score(3) == 0.5        # 1.0 decayed once
    assert pol.get(9) and pol.score(9) == 1.5
    pol.put(1)                        # scores: 3 -> 0.5, 9 -> 1.5, 1 -> 1.0
    assert pol.trim() == [3] and pol.keys() == [1, 9]
    pol.close()


def test_policy_lru(P):
    pol = P.CachePolicy(2, kind="lru")
    for k in (1, 2, 3):
        pol.put(k)
    pol.get(1)
    assert pol.trim() == [2]
    assert pol.keys() == [1, 3]
    pol.close()


def test_zipf_bias_rows_are_shuffled_log_probabilities(P):
    b = P.zipf_layer_bias(4, 128, 1.1, seed=42)
    assert b.shape == (4, 128) and b.dtype == np.float32
    np.testing.assert_allclose(np.exp(b.astype(np.float64)).sum(1), 1.0, rtol=1e-5)
    # the same multiset of probabilities, in a different order per layer
    np.testing.assert_allclose(np.sort(b[0]), np.sort(b[1]), rtol=1e-6)
    assert not np.array_equal(b[0], b[1])
    z = np.load(GOLDEN)  # the reference's layer probabilities for the same recipe and seed
    np.testing.assert_allclose(np.exp(b.astype(np.float64)), z["layer_probs"], rtol=1e-6)


# ---------------------------------------------------------------- GPU
def _small_spec():
    from expertflow_b200.spec import MoESpec

    return MoESpec(hidden=1024, n_experts=32, top_k=4, inter=256, bits=4, router="softmax", norm_topk=True,
                   act_dtype="bfloat16")


@pytest.mark.gpu
def test_pool_forward_matches_resident_layers_and_policy(P):
    import torch
    from expertflow_b200 import moe, synthetic

    spec = _small_spec()
    n_layers, budget, steps = 4, 6, 12
    dev = torch.device("cuda")
    host = P.make_host_layers(spec, n_layers, seed=100)
    bias = torch.from_numpy(P.zipf_layer_bias(n_layers, spec.n_experts, 1.1, seed=3)).to(dev)
    gates, resident = [], []
    for layer in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(500 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * 0.02).to(torch.float16)
        gates.append(moe.MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
        d = {"gate_w": gw, "e_bias": None, "shared": None}
        for k in ("gate", "up", "down"):
            d[k] = tuple(a.to(dev) for a in host[layer][k])
        m = moe.MoELayer.from_arrays(spec, d)
        m.gate = gates[layer]
        resident.append(m)
    pool = P.ExpertSlotPool(spec, host, budget=budget, headroom=spec.top_k)
    pool.record_routing(True)
    ref_pol = [P.CachePolicy(budget, 0.95) for _ in range(n_layers)]
    acc = hits = 0
    trace = []  # the reference's routing_trace: per token, (layer, expert) per routed entry
    for t in range(steps):
        x = synthetic.make_x_torch(spec, 1, seed=900 + t)
        trace.append([])
        for layer in range(n_layers):
            inds = torch.empty((1, spec.top_k), dtype=torch.int32, device=dev)
            nxt = gates[layer + 1] if layer + 1 < n_layers else None
            y = pool.forward(layer, x, gates[layer], nxt, inds_out=inds, out_dtype=torch.float32)
            y_ref = resident[layer](x, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(y, y_ref), (t, layer)
            trace[-1].extend((layer, int(e)) for e in inds.flatten().tolist())
            for e in sorted(set(inds.flatten().tolist())):
                acc += 1
                if ref_pol[layer].get(e):
                    hits += 1
                else:
                    ref_pol[layer].put(e)
            x = (x.float() + y).to(x.dtype)
        pool.end_token()
        for layer in range(n_layers):
            ref_pol[layer].trim()
            assert pool.resident(layer) == ref_pol[layer].keys(), (t, layer)
    st = pool.stats()
    assert st["accesses"] == acc and st["hits"] == hits and st["misses"] == acc - hits
    assert st["copies_sync"] + st["prefetch_used"] == st["misses"]
    eb = spec.expert_bytes()
    assert st["h2d_bytes"] == (st["copies_sync"] + st["copies_prefetch"]) * eb
    assert st["tokens"] == steps and st["copies_prefetch"] > 0 and st["copy_ms"] > 0
    assert pool.routing_trace == trace
    pool.record_routing(False)
    from expertflow_b200.moe import device_error
    assert device_error() == 0
    pool.close()


@pytest.mark.gpu
def test_pool_rejects_device_arrays(P):
    import torch

    spec = _small_spec()
    host = P.make_host_layers(spec, 1, seed=1)
    host[0]["gate"] = tuple(a.cuda() for a in host[0]["gate"])
    with pytest.raises(ValueError):
        P.ExpertSlotPool(spec, host, budget=4)


@pytest.mark.gpu
def test_pool_decode_step_independent_of_residency(P):
    """The in-library multi-layer decode step: pools with 6 of 32 experts per
    layer in HBM (one- and two-layer lookahead) and one holding every expert
    produce bit-identical residual streams (residency changes where weights
    come from, never the result)."""
    import torch
    from expertflow_b200 import moe, synthetic

    spec = _small_spec()
    n_layers, steps = 4, 6
    dev = torch.device("cuda")
    host = P.make_host_layers(spec, n_layers, seed=200)
    bias = torch.from_numpy(P.zipf_layer_bias(n_layers, spec.n_experts, 1.1, seed=9)).to(dev)
    gates = []
    for layer in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(700 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * 0.02).to(torch.float16)
        gates.append(moe.MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
    out = []
    for budget, la in ((6, 1), (6, 2), (spec.n_experts, 0)):
        pl = P.ExpertSlotPool(spec, host, budget=budget, headroom=spec.top_k)
        rs = []
        for t in range(steps):
            r = synthetic.make_x_torch(spec, 2, seed=40 + t).float().contiguous()
            pl.decode_step(r, gates, lookahead=la)
            rs.append(r.clone())
        torch.cuda.synchronize()
        out.append((torch.stack(rs), pl.stats()))
        pl.close()
    (ra, sa), (r2, s2), (rb, sb) = out
    assert torch.isfinite(ra).all() and torch.equal(ra, rb) and torch.equal(r2, rb)
    assert sa["tokens"] == steps and sa["copies_prefetch"] > 0
    assert s2["copies_prefetch"] > 0
    assert sb["copies_sync"] <= spec.n_experts * n_layers
    pl = P.ExpertSlotPool(spec, host, budget=6, headroom=spec.top_k)
    with pytest.raises(ValueError):
        pl.decode_step(synthetic.make_x_torch(spec, 1, seed=1).float().contiguous(), gates, lookahead=3)
    pl.close()
    assert moe.device_error() == 0


# ---------------------------------------------------------------- learned eviction
BELADY = os.path.join(REPO, "tests", "golden", "belady_trace.npz")
_NETK = ("w1", "b1", "w2", "b2", "w3", "b3")


def _trace_tokens():
    c = np.load(GOLDEN)
    toks, cur = [], []
    for a in c["accesses"].tolist():
        if a == -2:
            toks.append(cur)
            cur = []
        elif a >= 0:
            cur.append(a)
    return toks


def _net(z, name):
    return {k: z[f"{name}_{k}"] for k in _NETK} | {"trained": True}


@pytest.mark.parametrize("name", ["untrained", "seed0", "seed4x4", "trained"])
def test_belady_policy_replays_reference(P, name):
    """BeladyExpertCache (ef_engine.py:163-279) driven by the reference's Zipf
    trace with its own predictors: every hit/miss, eviction count and resident
    set.  (seed1 / seed1x4 are left to the score test below: their rankings
    hold exact ties that the reference breaks by fp32 BLAS rounding noise.)"""
    z = np.load(BELADY)
    pol = P.CachePolicy(int(z["budget"]), float(z["decay"]), kind="belady",
                        predictor=None if name == "untrained" else _net(z, name))
    hits, ev = [], []
    for t, tok in enumerate(_trace_tokens()):
        for key in tok:
            h = pol.get(key)
            if not h:
                pol.put(key)
            hits.append(int(h))
        ev.append(len(pol.trim()))
        pol.end_token()
        assert pol.keys() == sorted(int(r) for r in z[f"{name}_resident"][t] if r >= 0), (name, t)
    np.testing.assert_array_equal(np.asarray(hits, np.int8), z[f"{name}_hits"])
    np.testing.assert_array_equal(np.asarray(ev), z[f"{name}_evicted"])
    pol.close()


def test_belady_scores_match_reference(P):
    """The predictor's score of every resident key just before the reference's
    first eviction (seed1), within fp32 rounding of the reference's numpy."""
    z = np.load(BELADY)
    pol = P.CachePolicy(int(z["budget"]), float(z["decay"]), kind="belady", predictor=_net(z, "seed1"))
    toks = _trace_tokens()
    T = int(z["snapshot_token"])
    for t in range(T + 1):
        for key in toks[t]:
            if not pol.get(key):
                pol.put(key)
        if t < T:
            assert pol.trim() == []
            pol.end_token()
    ours = np.array([pol.score(int(k)) for k in z["snapshot_keys"]])
    np.testing.assert_allclose(ours, z["snapshot_scores"].astype(np.float64), rtol=2e-6, atol=1e-9)
    pol.close()


def test_belady_untrained_is_frequency_fallback(P):
    """Untrained: evict the lowest count * decay^recency, the first inserted
    among equals; counts are truncated by decay after each trim."""
    pol = P.CachePolicy(2, 0.5, kind="belady")
    for k in (5, 6, 7):
        pol.put(k)
    assert pol.trim() == [5] and pol.keys() == [6, 7]   # equal scores: first inserted goes
    pol.end_token()
    assert pol.get(7)                                     # count(7): 1 -> floor(0.5) = 0, +1 = 1
    assert pol.score(6) == 0.0                            # count(6): floor(1 * 0.5) = 0
    pol.put(8)
    assert pol.trim() == [6]
    pol.close()


def test_predictor_file_format(P, tmp_path):
    """A predictor saved the way the reference saves one (BeladyPredictor.save)."""
    z = np.load(BELADY)
    w = _net(z, "trained")
    f = tmp_path / "belady.npz"
    np.savez(f, **{k: w[k] for k in _NETK}, trained=np.array([True]), input_dim=np.array([3]),
             hidden_dim=np.array([64]))
    loaded = P.load_predictor(str(f))
    assert loaded["trained"] and loaded["w3"].shape == (64,)
    with pytest.raises(ValueError):
        P.load_predictor({**w, "w2": w["w2"][:10]})


@pytest.mark.gpu
def test_pool_belady_policy_matches_host_replay(P):
    """A pool with the learned policy: outputs bit-identical to resident layers,
    and each layer's residency equal to a host-side BeladyExpertCache replay of
    the routed experts (trim, then end_token, per token)."""
    import torch
    from expertflow_b200 import moe, synthetic

    spec = _small_spec()
    n_layers, budget, steps = 3, 6, 10
    dev = torch.device("cuda")
    z = np.load(BELADY)
    net = _net(z, "trained")
    host = P.make_host_layers(spec, n_layers, seed=300)
    bias = torch.from_numpy(P.zipf_layer_bias(n_layers, spec.n_experts, 1.1, seed=5)).to(dev)
    gates, resident = [], []
    for layer in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(800 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * 0.02).to(torch.float16)
        gates.append(moe.MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
        d = {"gate_w": gw, "e_bias": None, "shared": None}
        for k in ("gate", "up", "down"):
            d[k] = tuple(a.to(dev) for a in host[layer][k])
        m = moe.MoELayer.from_arrays(spec, d)
        m.gate = gates[layer]
        resident.append(m)
    pool = P.ExpertSlotPool(spec, host, budget=budget, headroom=spec.top_k, policy="belady")
    pool.set_predictor(net)
    ref = [P.CachePolicy(budget, 0.95, kind="belady", predictor=net) for _ in range(n_layers)]
    for t in range(steps):
        x = synthetic.make_x_torch(spec, 1, seed=950 + t)
        for layer in range(n_layers):
            inds = torch.empty((1, spec.top_k), dtype=torch.int32, device=dev)
            y = pool.forward(layer, x, gates[layer], None, inds_out=inds, out_dtype=torch.float32)
            y_ref = resident[layer](x, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(y, y_ref), (t, layer)
            for e in sorted(set(inds.flatten().tolist())):
                if not ref[layer].get(e):
                    ref[layer].put(e)
            x = (x.float() + y).to(x.dtype)
        pool.end_token()
        for layer in range(n_layers):
            ref[layer].trim()
            ref[layer].end_token()
            assert pool.resident(layer) == ref[layer].keys(), (t, layer)
    assert moe.device_error() == 0
    pool.close()
