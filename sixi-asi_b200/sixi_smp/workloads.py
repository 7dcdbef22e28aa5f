"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

No dataset is involved: every configuration is synthetic by definition (logits ~ N(0, sigma^2),
parameter mixes drawn from a seed). Arrays are plain numpy on the host; callers move them to the
device. Configurations:
  1  single row, V=151,936, N(0, 2.5^2) with 16 tokens boosted by +8, 64-token history,
     rep 1.1, T 0.7, top-k 20, top-p 0.8 (plus a greedy run)
  2  B rows, N(0, 2.5^2), per-row T ~ U[0.3, 1.2] with 25% greedy, top-k in {0, 20, 40, 100},
     top-p ~ U[0.7, 1.0], rep ~ U[1.0, 1.3], histories of U[256, 8192] ids uniform over V
  3  config 2 plus a packed allowed-token bitmask per row, allowed fraction log-uniform in
     [1e-4, 0.6], laid out as contiguous id runs
  4  S streams x k drafts: bf16 target logits N(0, 3^2) [S, k+1, V], draft logits target + N(0, 1)
     [S, k, V] and their dense probabilities softmax(draft logits), drafts sampled from them,
     20%-density masks on half the streams
"""

from __future__ import annotations

import numpy as np

from . import ADAPTIVE, PARAMS_DTYPE, ROW_MASKED, make_params

QWEN_VOCAB = 151_936


def mask_words(vocab: int) -> int:
    return (vocab + 31) // 32


def pack_mask(allowed: np.ndarray) -> np.ndarray:
    """bool [rows, V] -> uint32 [rows, ceil(V/32)], bit (i % 32) of word (i // 32)."""
    rows, v = allowed.shape
    w = mask_words(v)
    pad = np.zeros((rows, w * 32), dtype=bool)
    pad[:, :v] = allowed
    b = np.packbits(pad.reshape(rows, w, 32), axis=2, bitorder="little")
    return b.reshape(rows, w * 4).view("<u4").reshape(rows, w).copy()


def unpack_mask(words: np.ndarray, vocab: int) -> np.ndarray:
    rows = words.shape[0]
    b = np.unpackbits(words.view(np.uint8).reshape(rows, -1), axis=1, bitorder="little")
    return b[:, :vocab].astype(bool)


def run_mask(rng: np.random.Generator, vocab: int, frac: float, mean_run: float = 48.0) -> np.ndarray:
    """Allowed ids in contiguous runs (geometric run and gap lengths), about `frac` allowed."""
    frac = float(min(max(frac, 1e-6), 1.0))
    allowed = np.zeros(vocab, dtype=bool)
    mean_gap = mean_run * (1.0 - frac) / frac
    pos = int(rng.integers(0, max(1, int(mean_gap) + 1)))
    while pos < vocab:
        run = int(rng.geometric(1.0 / mean_run))
        allowed[pos:pos + run] = True
        pos += run + int(rng.geometric(1.0 / (mean_gap + 1.0)))
    if not allowed.any():
        allowed[int(rng.integers(0, vocab))] = True
    return allowed


def config1(vocab: int = QWEN_VOCAB, seed: int = 1, greedy: bool = False) -> dict:
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, 2.5, size=(1, vocab)).astype(np.float32)
    boost = rng.choice(vocab, size=min(16, vocab), replace=False)
    logits[0, boost] += np.float32(8.0)
    hist = rng.integers(0, vocab, size=64, dtype=np.int32)
    params = make_params(1, temperature=0.0 if greedy else 0.7, top_k=20, top_p=0.8,
                         repetition_penalty=1.1, mode=ADAPTIVE, seed=seed)
    return dict(logits=logits, params=params, hist=hist, hist_off=np.array([0, 64], dtype=np.int64),
                masks=None)


def config2(rows: int = 32, vocab: int = QWEN_VOCAB, seed: int = 2, hist_lo: int = 256,
            hist_hi: int = 8192) -> dict:
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, 2.5, size=(rows, vocab)).astype(np.float32)
    t = rng.uniform(0.3, 1.2, size=rows).astype(np.float32)
    t[rng.random(rows) < 0.25] = 0.0
    params = make_params(
        rows,
        temperature=t,
        top_k=rng.choice(np.array([0, 20, 40, 100], dtype=np.int32), size=rows),
        top_p=rng.uniform(0.7, 1.0, size=rows).astype(np.float32),
        repetition_penalty=rng.uniform(1.0, 1.3, size=rows).astype(np.float32),
        mode=ADAPTIVE,
        seed=rng.integers(0, 2**63, size=rows, dtype=np.uint64),
    )
    lens = rng.integers(hist_lo, hist_hi + 1, size=rows)
    off = np.zeros(rows + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
    boost_rows(np.random.default_rng(seed + 0xB005), logits)
    return dict(logits=logits, params=params, hist=hist, hist_off=off, masks=None)


def config2_mix(rows: int, vocab: int = QWEN_VOCAB, seed: int = 5, hist_lo: int = 256,
                hist_hi: int = 8192) -> dict:
    """The config-2 parameter mix and histories for `rows` rows, without logits (config 5 draws
    its 8,192 rows of logits on the device: 4.98 GB do not belong in host memory)."""
    rng = np.random.default_rng(seed)
    t = rng.uniform(0.3, 1.2, size=rows).astype(np.float32)
    t[rng.random(rows) < 0.25] = 0.0
    params = make_params(
        rows,
        temperature=t,
        top_k=rng.choice(np.array([0, 20, 40, 100], dtype=np.int32), size=rows),
        top_p=rng.uniform(0.7, 1.0, size=rows).astype(np.float32),
        repetition_penalty=rng.uniform(1.0, 1.3, size=rows).astype(np.float32),
        mode=ADAPTIVE,
        seed=rng.integers(0, 2**63, size=rows, dtype=np.uint64),
    )
    lens = rng.integers(hist_lo, hist_hi + 1, size=rows)
    off = np.zeros(rows + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
    return dict(params=params, hist=hist, hist_off=off, masks=None)


def config2_logits_device(rows: int, vocab: int, seed: int, device):
    """Config-2 logits drawn on the device: N(0, 2.5^2) with 16 distinct ids per row boosted by +8
    (ids base + j * stride mod V with stride < V / 16, so the 16 are distinct)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((rows, vocab), generator=g, device=device, dtype=torch.float32).mul_(2.5)
    base = torch.randint(0, vocab, (rows, 1), generator=g, device=device)
    stride = torch.randint(1, max(2, vocab // 16), (rows, 1), generator=g, device=device)
    ids = (base + stride * torch.arange(16, device=device)) % vocab
    x.scatter_add_(1, ids, torch.full(ids.shape, 8.0, device=device))
    return x


def boost_rows(rng: np.random.Generator, logits: np.ndarray, n: int = 16, by: float = 8.0) -> np.ndarray:
    """Adds `by` to `n` distinct random ids of every row (the boosted tokens of configs 1 and 2)."""
    vocab = logits.shape[1]
    for r in range(logits.shape[0]):
        logits[r, rng.choice(vocab, size=min(n, vocab), replace=False)] += np.float32(by)
    return logits


def config2_logits(rng: np.random.Generator, rows: int = 32, vocab: int = QWEN_VOCAB) -> np.ndarray:
    """Fresh config-2 logits: N(0, 2.5^2) with 16 ids per row boosted by +8."""
    return boost_rows(rng, rng.normal(0.0, 2.5, size=(rows, vocab)).astype(np.float32))


def config3(rows: int = 32, vocab: int = QWEN_VOCAB, seed: int = 3, **kw) -> dict:
    d = config2(rows, vocab, seed, **kw)
    rng = np.random.default_rng(seed + 1000)
    fr = np.exp(rng.uniform(np.log(1e-4), np.log(0.6), size=rows))
    allowed = np.stack([run_mask(rng, vocab, f) for f in fr])
    d["masks"] = pack_mask(allowed)
    d["params"]["flags"] |= ROW_MASKED
    d["allowed_fraction"] = allowed.mean(axis=1)
    return d


def softmax_rows(x: np.ndarray) -> np.ndarray:
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float64))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = x.astype(np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def config4(streams: int = 32, k: int = 8, vocab: int = QWEN_VOCAB, seed: int = 4,
            stochastic: bool = True, masked: bool = True, param_mix: bool = True) -> dict:
    rng = np.random.default_rng(seed)
    tgt = rng.normal(0.0, 3.0, size=(streams, k + 1, vocab)).astype(np.float32)
    target_bits = f32_to_bf16_bits(tgt)
    target = bf16_bits_to_f32(target_bits)
    noisy = target[:, :k, :] + rng.normal(0.0, 1.0, size=(streams, k, vocab)).astype(np.float32)
    q = softmax_rows(noisy)
    # drafts sampled from q (inverse CDF with seeded uniforms)
    cdf = np.cumsum(q.astype(np.float64), axis=-1)
    u = rng.random(size=(streams, k))
    drafts = np.empty((streams, k), dtype=np.int32)
    for s in range(streams):
        for i in range(k):
            drafts[s, i] = min(int(np.searchsorted(cdf[s, i], u[s, i] * cdf[s, i, -1], side="right")),
                               vocab - 1)
    if param_mix:
        p2 = config2(streams, 8, seed + 7)["params"]  # parameter mix of config 2
        params = p2
    else:
        params = make_params(streams, temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.1)
    if not stochastic:
        params["temperature"] = 0.0
    else:
        params["temperature"] = np.where(params["temperature"] <= 0, 0.7, params["temperature"])
    masks = None
    if masked:
        allowed = np.ones((streams, k + 1, vocab), dtype=bool)
        for s in range(0, streams, 2):
            for i in range(k + 1):
                a = run_mask(rng, vocab, 0.2)
                if i < k:
                    a[drafts[s, i]] = True  # the automaton accepts the drafted token
                allowed[s, i] = a
            params["flags"][s] |= ROW_MASKED
        masks = pack_mask(allowed.reshape(streams * (k + 1), vocab))
    lens = rng.integers(64, 512, size=streams)
    off = np.zeros(streams + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
    uniforms = rng.random(size=(streams, k + 1))
    return dict(target_bits=target_bits.reshape(streams * (k + 1), vocab), q=q.reshape(streams * k, vocab),
                draft_logits=noisy.reshape(streams * k, vocab), drafts=drafts, params=params, masks=masks, hist=hist,
                hist_off=off, uniforms=uniforms, k=k, streams=streams)


def uniforms_for(params: np.ndarray, step: int = 0, slots: int = 1) -> np.ndarray:
    """The Philox uniforms the library draws when none are supplied (host restatement)."""
    from . import philox_uniform

    out = np.empty((len(params), slots))
    for r, p in enumerate(params):
        for s in range(slots):
            out[r, s] = philox_uniform(int(p["seed"]), int(p["counter"]) + step, s)
    return out


__all__ = ["config1", "config2", "config3", "config4", "pack_mask", "unpack_mask", "run_mask",
           "mask_words", "f32_to_bf16_bits", "bf16_bits_to_f32", "softmax_rows", "uniforms_for",
           "PARAMS_DTYPE", "QWEN_VOCAB"]


# A response_format json_schema of the kind an extraction request sends: nested objects, an array
# of objects without an item bound (so that answers run long), integer bounds, enums, a pattern and
# a format. Used by the json_schema bench line.
RESPONSE_SCHEMA = {
    "type": "object",
    "properties": {
        "order_id": {"type": "string", "pattern": "^[A-Z]{2}-[0-9]{6}$"},
        "placed": {"type": "string", "format": "date"},
        "status": {"enum": ["open", "shipped", "delivered", "cancelled"]},
        "customer": {"type": "object",
                     "properties": {"name": {"type": "string", "maxLength": 40},
                                    "email": {"type": "string"},
                                    "vip": {"type": "boolean"}},
                     "required": ["name"], "additionalProperties": False},
        "lines": {"type": "array",
                  "items": {"type": "object",
                            "properties": {"sku": {"type": "string"},
                                           "qty": {"type": "integer", "minimum": 1, "maximum": 999},
                                           "price": {"type": "number"},
                                           "note": {"anyOf": [{"type": "string"}, {"type": "null"}]}},
                            "required": ["sku", "qty"], "additionalProperties": False}},
        "total": {"type": "number"},
    },
    "required": ["order_id", "status", "lines"],
    "additionalProperties": False,
}
