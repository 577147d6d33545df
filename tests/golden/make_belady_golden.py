"""Generate tests/golden/belady_trace.npz by executing the REFERENCE's own
``BeladyExpertCache`` (ef_engine.py:163-279; read from a reference checkout
given by --reference or the EF_REFERENCE environment variable, through
``mlx_shim`` because ef_engine imports MLX).

The access trace is the one in ``cache_trace.npz`` (the reference's
SimulatedMoERouter Zipf trace, 4 layers x 128 experts, 160 tokens).  Per token
the cache sees ``get`` (``put`` on a miss) for each routed (layer, expert),
then ``trim()`` and ``end_token()``, the order of the reference's decode loop
(ef_engine.py:866-869).  Three predictors:

* ``untrained`` -- the frequency fallback (count * decay^recency);
* ``seed0``, ``seed1``, ``seed1x4``, ``seed4x4`` -- ``BeladyPredictor()`` after
  ``np.random.seed(s)``, marked trained (``x4``: every weight times 4 and a
  random first-layer bias): four predictors that rank the cached experts
  differently on this trace;
* ``trained``   -- ``train_belady_predictor`` (ef_engine.py:358-451) on the
  ``compute_belady_labels`` samples (ef_engine.py:282-355) of the first 40
  tokens, 3 epochs, after ``np.random.seed(0)``.

Recorded: per access hit/miss, per token the eviction count and the resident
set, and the predictor weights.

Run:  python tests/golden/make_belady_golden.py --reference <reference checkout>
"""
from __future__ import annotations

import argparse
import io
import os
import sys
from contextlib import redirect_stdout

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

BUDGET, DECAY = 96, 0.95


def tokens_of(z):
    """Per token, the (layer, expert) accesses in order."""
    n_exp = int(z["n_experts"])
    out, cur = [], []
    for a in z["accesses"].tolist():
        if a == -2:
            out.append(cur)
            cur = []
        elif a >= 0:
            cur.append((a // n_exp, a % n_exp))
    return out


def replay(ef_engine, toks, predictor):
    cache = ef_engine.BeladyExpertCache(budget=BUDGET, decay=DECAY)
    if predictor is not None:
        cache.predictor = predictor
    hits, evicted, resident = [], [], []
    n_exp = 128
    for tok in toks:
        for key in tok:
            if cache.get(key) is None:
                cache.put(key, 1)
                hits.append(0)
            else:
                hits.append(1)
        evicted.append(cache.trim())
        cache.end_token()
        resident.append(sorted(l * n_exp + e for (l, e) in cache.cache.keys()))
    res = np.full((len(toks), BUDGET), -1, np.int32)
    for i, r in enumerate(resident):
        res[i, :len(r)] = r
    return np.asarray(hits, np.int8), np.asarray(evicted, np.int32), res


def weights(p):
    return {k: getattr(p, k).astype(np.float32) for k in ("w1", "b1", "w2", "b2", "w3", "b3")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EF_REFERENCE"),
                    required="EF_REFERENCE" not in os.environ,
                    help="reference checkout to import (default: $EF_REFERENCE)")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    import mlx_shim

    mlx_shim.install()
    sys.path.insert(0, args.reference)
    import ef_engine  # noqa: E402  (reference module, imported read-only)

    z = np.load(os.path.join(HERE, "cache_trace.npz"))
    toks = tokens_of(z)
    out = {"budget": BUDGET, "decay": DECAY}
    # untrained: frequency fallback
    h, e, r = replay(ef_engine, toks, None)
    out.update(untrained_hits=h, untrained_evicted=e, untrained_resident=r)
    # seeded random weights marked trained (seed, scale of every weight, random first-layer bias):
    # four predictors whose rankings differ from each other on this trace
    names = []
    for seed, scale, bias in ((0, 1.0, False), (1, 1.0, False), (1, 4.0, True), (4, 4.0, True)):
        np.random.seed(seed)
        p = ef_engine.BeladyPredictor()
        p.trained = True
        for k in ("w1", "b1", "w2", "b2", "w3", "b3"):
            setattr(p, k, (getattr(p, k) * scale).astype(np.float32))
        if bias:
            p.b1 = (np.random.RandomState(seed).randn(p.hidden_dim) * 0.5).astype(np.float32)
        name = f"seed{seed}" + ("x4" if scale != 1.0 else "")
        h, e, r = replay(ef_engine, toks, p)
        out.update({f"{name}_hits": h, f"{name}_evicted": e, f"{name}_resident": r},
                   **{f"{name}_{k}": v for k, v in weights(p).items()})
        names.append(name)
    # seed1: the reference's scores of every resident key just before its first
    # eviction (its argmax among keys with identical features follows fp32 BLAS
    # rounding, which differs by row position, so later trims are not pinned)
    np.random.seed(1)
    p = ef_engine.BeladyPredictor()
    p.trained = True
    cache = ef_engine.BeladyExpertCache(budget=BUDGET, decay=DECAY)
    cache.predictor = p
    for t, tok in enumerate(toks):
        for key in tok:
            if cache.get(key) is None:
                cache.put(key, 1)
        if len(cache.cache) > BUDGET:
            keys = list(cache.cache.keys())
            out["snapshot_token"] = t
            out["snapshot_keys"] = np.asarray([l * 128 + e for (l, e) in keys], np.int32)
            out["snapshot_scores"] = p.predict(cache._build_features(keys)).astype(np.float32)
            break
        cache.trim()
        cache.end_token()
    # trained on Belady labels of the first 40 tokens
    samples = ef_engine.compute_belady_labels(toks[:40], BUDGET)
    np.random.seed(0)
    with redirect_stdout(io.StringIO()):
        p = ef_engine.train_belady_predictor(samples, epochs=3, lr=3e-3)
    h, e, r = replay(ef_engine, toks, p)
    out.update(trained_hits=h, trained_evicted=e, trained_resident=r, n_label_samples=len(samples),
               **{f"trained_{k}": v for k, v in weights(p).items()})
    names.append("trained")
    out["predictors"] = np.array(names)
    # a few labelled samples (features, Belady victim) for the label restatement
    out["label_victims"] = np.asarray([s[1] for s in samples], np.int32)
    out["label_sizes"] = np.asarray([s[0].shape[0] for s in samples], np.int32)
    out["label_features"] = np.concatenate([s[0] for s in samples[:20]]).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "belady_trace.npz"), **out)
    print(f"belady_trace: {len(toks)} tokens, {len(samples)} label samples; hit rates " +
          ", ".join(f"{n} {out[n + '_hits'].mean():.3f}" for n in ["untrained"] + names))


if __name__ == "__main__":
    main()
