"""Generates tests/golden/golden.npz: outputs of the engine's own sampler and verifier logic
(oracle/_ref/libsixiref.so, built from the engine's sources by oracle/Makefile) on seeded inputs.

The inputs are not stored: tests/test_oracle.py regenerates them from the same seeds with
`cases()` below and checks the C restatement (oracle/liboracle.so) against the stored outputs, so
the restatement stays pinned to the engine where the engine's sources are absent (the GPU box).
Run: python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "sixi-asi_b200"))

import sixi_smp as S  # noqa: E402  (parameter records only; the library is not loaded)
from sixi_smp import workloads as W  # noqa: E402

OUT = HERE / "golden.npz"
MAX_CANDS = 64


def engine_test_logits(v: int = 5000) -> np.ndarray:
    """The logits of the engine's sampler unit test (tests/test_routing_and_numerics.cpp:488-492),
    evaluated in fp32 like the test (sinf of a float argument)."""
    i = np.arange(v, dtype=np.float32)
    x = np.sin((i * np.float32(0.37)).astype(np.float32)).astype(np.float32) * np.float32(3.0)
    return (x + np.where(np.arange(v) % 97 == 0, np.float32(2.5), np.float32(0.0))).astype(np.float32)


def cases() -> list[dict]:
    """Seeded single-row sampler cases: logits, params, history, mask, uniform."""
    out = []
    rng = np.random.default_rng(20261201)
    x = engine_test_logits()
    for tk, tp, t in [(20, 1.0, 1.0), (20, 0.5, 1.0), (0, 0.9, 0.8), (5, 0.95, 0.5), (0, 1.0, 0.0)]:
        p = S.make_params(1, temperature=t, top_k=tk, top_p=tp, mode=S.STRICT_REPLAY)
        out.append(dict(logits=x, params=p, hist=None, mask=None, u=float(rng.random())))
    for v in (33, 4097, 151_936):
        for j in range(6):
            logits = rng.normal(0.0, 2.5, size=v).astype(np.float32)
            if j % 3 == 1:
                logits = np.round(logits).astype(np.float32)  # ties
            t = float(rng.choice([0.0, 0.3, 0.7, 1.1]))
            tk = int(rng.choice([0, 1, 20, 40, 100, 300]))
            tp = float(rng.choice([1.0, 0.7, 0.85, 0.99]))
            rep = float(rng.choice([1.0, 1.1, 1.3]))
            pres = float(rng.choice([0.0, 0.0, 0.4]))
            p = S.make_params(1, temperature=t, top_k=tk, top_p=tp, repetition_penalty=rep,
                              presence_penalty=pres, mode=S.ADAPTIVE)
            hist = rng.integers(-1, v + 1, size=int(rng.integers(0, 300)), dtype=np.int32)
            mask = None
            if j % 2 == 1:
                mask = W.pack_mask(W.run_mask(rng, v, float(rng.choice([0.01, 0.2, 0.6])), mean_run=8.0)[None])[0]
                p["flags"] = S.ROW_MASKED
            bf = j == 5
            row = W.f32_to_bf16_bits(logits) if bf else logits
            out.append(dict(logits=row, params=p, hist=hist, mask=mask, u=float(rng.random())))
    return out


def verify_cases() -> list[dict]:
    out = []
    for seed, stochastic, dense in [(7, False, True), (8, True, True), (9, True, False), (10, True, True)]:
        d = W.config4(streams=6, k=4, vocab=2000, seed=seed, stochastic=stochastic, masked=(seed % 2 == 0))
        d["dense"] = dense
        out.append(d)
    return out


def main() -> int:
    from oracle import binding

    ref = binding.reference()
    if ref is None:
        print("reference build missing: run `make -C oracle` where the engine's sources are present")
        return 1
    res: dict[str, np.ndarray] = {}
    for i, c in enumerate(cases()):
        st, ids, probs, n = ref.candidates(c["logits"], c["params"], c["hist"], c["mask"])
        st2, tok = ref.sample(c["logits"], c["params"], c["hist"], c["mask"], c["u"])
        k = min(n, MAX_CANDS)
        res[f"c{i}_status"] = np.array([st, st2], dtype=np.int32)
        res[f"c{i}_n"] = np.array([n], dtype=np.int64)
        res[f"c{i}_ids"] = ids[:k]
        res[f"c{i}_probs"] = probs[:k]
        res[f"c{i}_token"] = np.array([tok], dtype=np.int32)
    for i, d in enumerate(verify_cases()):
        o = ref.verify(d["target_bits"], d["drafts"], d["params"], q=d["q"] if d["dense"] else None,
                       masks=d["masks"], hist=d["hist"], hist_off=d["hist_off"], uniforms=d["uniforms"])
        for k2, v in o.items():
            res[f"v{i}_{k2}"] = v
    # the engine's greedy tie-break vector (tests/test_determinism_and_speculative.cpp:56-61)
    res["tie_argmax"] = np.array([ref.greedy_argmax(np.array([-1.0, 5.5, 3.2, 5.5, 5.5, 0.0], np.float32))])
    np.savez_compressed(OUT, **res)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(res)} arrays)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
