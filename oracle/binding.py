"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (parity checker).

Loads either implementation of oracle/sixi_oracle.h:
  port()       liboracle.so        - plain-C restatement of the engine's sampler and verifier
  reference()  _ref/libsixiref.so  - the engine's own DeterministicSampler built from its sources
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the product
library never calls it.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libsixiref.so"
UNSUPPORTED = -2

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64

_SIGS = {
    "orc_full_distribution": (None, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float,
                                     ctypes.c_void_p]),
    "orc_kind": (_I32, []),
    "orc_philox_uniform": (ctypes.c_double, [_U64, _U64, _U32]),
    "orc_greedy_argmax": (_I32, [_P, _U64]),
    "orc_greedy_row": (_I32, [_P, _U32, _U64, _P, _P]),
    "orc_candidates": (_I32, [_P, _U32, _U64, _P, _P, _U64, _P, _U64, _P, _P, _P]),
    "orc_sample": (_I32, [_P, _U32, _U64, _P, _P, _U64, _P, ctypes.c_double, _P]),
    "orc_sample_batch": (_I32, [_P, _U32, _U32, _U64, _U64, _P, _P, _P, _P, _P, _U64, _P, _P, _I32]),
    "orc_numeric_policy": (_I32, [_P, ctypes.c_int64, _U32, ctypes.c_float, _P]),
    "orc_suffix_draft": (_I32, [_P, _U64, _U32, _U32, _I32, _I32, _U32, _P]),
    "orc_verify": (_I32, [_P, _U32, _U64, _U64, _P, _P, _P, _U32, _U32, _P, _P, _P, _P, _P, _U64,
                          _P, _P, _P, _P, _P, _P, _I32]),
    # the engine's own SpeculativeDecoder::step and DeterministicRng (reference build only)
    "orc_ref_rng_uniform": (ctypes.c_double, [_P]),
    "orc_ref_rng_seed": (None, [_U64, _U64, _P]),
    "orc_ref_spec_step": (_I32, [_I32, _P, _P, _U64, _P, _P, _U32, _P, _P, _U64, _P, _P, _P, _P, _P]),
    "orc_ref_spec_step_batch": (_I32, [_P, _U32, _U64, _P, _P, _U32, _U32, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _I32]),
    # JSON-object grammar automaton (sixi_json_oracle.c)
    "orc_json_feed": (_I32, [_P, _P, _U64]),
    "orc_json_fill_masks": (None, [_P, _P, _P, _U32, _I32, _P, _U32, _P, _U64, _I32]),
    "orc_json_advance": (None, [_P, _P, _P, _U32, _I32, _P, _U32, _P, _U64, _P, _P]),
    "orc_json_expand": (None, [_P, _P, _P, _U32, _I32, _P, _U32, _P, _U32, _P, _P]),
}


NUMERIC_REPORT = np.dtype([("healthy", "u1"), ("request_corrupted", "u1"), ("state_invalidated", "u1"),
                           ("emergency_clamped", "u1"), ("status", "<i4"), ("nan_count", "<u8"),
                           ("inf_count", "<u8"), ("first_bad_index", "<i8")])  # sixi_smp_numeric_report


def build() -> None:
    """Builds liboracle.so and, when the reference sources are present, _ref/libsixiref.so."""
    subprocess.run(["make", "-s", "-C", str(HERE), "-j8"], check=True)


def _p(a) -> int:
    return 0 if a is None else a.ctypes.data


def _dtype_of(a: np.ndarray) -> int:
    return 1 if a.dtype == np.uint16 else 0


class Oracle:
    def __init__(self, path: Path):
        self.path = Path(path)
        self.lib = ctypes.CDLL(str(self.path))
        for name, (res, args) in _SIGS.items():
            if name.startswith("orc_json_") and not hasattr(self.lib, name):
                continue  # the grammar automaton exists only in the port (the engine's is binary-only)
            if name.startswith("orc_ref_") and not hasattr(self.lib, name):
                continue  # the engine's decoder and RNG exist only in the reference build
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args
        self.kind = "reference" if self.lib.orc_kind() == 1 else "port"

    def numeric_policy(self, data: np.ndarray, policy: int, clamp_abs_max: float) -> tuple[int, np.void]:
        """inspect_and_apply_numeric_policy on one fp32 row, in place: (status, report record)."""
        assert data.dtype == np.float32 and data.flags.c_contiguous
        rep = np.zeros(1, dtype=NUMERIC_REPORT)
        st = self.lib.orc_numeric_policy(_p(data), data.size, policy, clamp_abs_max, _p(rep))
        return int(st), rep[0]

    def suffix_draft(self, hist: np.ndarray, min_match_len: int, max_window_tokens: int, k: int,
                     anchor: int | None = None) -> tuple[int, np.ndarray]:
        """SuffixDrafter(min_match_len, max_window_tokens).propose(hist, k) (or propose_anchored with
        `anchor`): (match_len, 0 without a proposal; drafts int32 [k], -1 without one)."""
        h = np.ascontiguousarray(hist, dtype=np.int32)
        out = np.zeros(max(k, 1), dtype=np.int32)
        m = self.lib.orc_suffix_draft(_p(h), h.size, min_match_len, max_window_tokens, 0 if anchor is None else 1,
                                      0 if anchor is None else int(anchor), k, _p(out))
        return int(m), out[:k]

    # -- the engine's SpeculativeDecoder::step (reference build) ------------------------------------
    def rng_seed(self, seed: int, seq: int = 54) -> np.ndarray:
        """(state, inc) of the engine's DeterministicRng(seed, seq)."""
        st = np.zeros(2, dtype=np.uint64)
        self.lib.orc_ref_rng_seed(seed, seq, _p(st))
        return st

    def rng_uniforms(self, state: np.ndarray, n: int) -> np.ndarray:
        """n uniforms of the engine's RNG from `state` (advanced in place)."""
        return np.array([self.lib.orc_ref_rng_uniform(_p(state)) for _ in range(n)])

    def spec_step(self, rows: np.ndarray, drafts: np.ndarray, params: np.ndarray, hist=None, draft_probs=None,
                  rng_state=None, fast: bool = False, anchor_row=None) -> dict:
        """One SpeculativeDecoder::step of the engine (slow path; fast path with `fast`, see
        orc_ref_spec_step) on fp32 rows [k+1, V]. `rng_state` (state, inc) is advanced in place."""
        rows = np.ascontiguousarray(rows, dtype=np.float32)
        d = np.ascontiguousarray(drafts, dtype=np.int32)
        k, v = d.size, rows.shape[1]
        q = None if draft_probs is None else np.ascontiguousarray(draft_probs, dtype=np.float32)
        h = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
        a = None if anchor_row is None else np.ascontiguousarray(anchor_row, dtype=np.float32)
        st = self.rng_seed(1) if rng_state is None else rng_state
        toks = np.full(k + 2, -1, dtype=np.int32)
        n, acc, fr = (np.zeros(1, dtype=np.int32) for _ in range(3))
        rc = self.lib.orc_ref_spec_step(1 if fast else 0, _p(a), _p(rows), v, _p(q), _p(d), k, _p(params), _p(h),
                                        0 if h is None else h.size, _p(st), _p(toks), _p(n), _p(acc), _p(fr))
        return dict(status=int(rc), tokens=toks[:int(n[0])].copy(), accepted=int(acc[0]), first_reject=int(fr[0]),
                    rng=st.copy())

    def spec_step_batch(self, rows: np.ndarray, drafts: np.ndarray, params: np.ndarray, hist, hist_off,
                        draft_probs, rng_states: np.ndarray, n_threads: int = 0) -> dict:
        """The slow-path step for S streams: rows [S*(k+1), V] (fp32 or bf16 bits), drafts [S, k],
        draft_probs [S*k, V]; rng_states [S, 2] advanced in place."""
        rows = np.ascontiguousarray(rows)
        S, k = drafts.shape
        v = rows.shape[1]
        toks = np.full((S, k + 2), -1, dtype=np.int32)
        n, acc, fr, sts = (np.zeros(S, dtype=np.int32) for _ in range(4))
        self.lib.orc_ref_spec_step_batch(_p(rows), _dtype_of(rows), v, _p(draft_probs),
                                         _p(np.ascontiguousarray(drafts, dtype=np.int32)), S, k, _p(params),
                                         _p(hist), _p(hist_off), _p(rng_states), _p(toks), _p(n), _p(acc), _p(fr),
                                         _p(sts), n_threads)
        return dict(tokens=toks, n_tokens=n, accepted=acc, first_reject=fr, status=sts)

    def philox_uniform(self, seed: int, counter: int, slot: int) -> float:
        return float(self.lib.orc_philox_uniform(seed, counter, slot))

    def greedy_argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return int(self.lib.orc_greedy_argmax(_p(x), x.size))

    def greedy_row(self, row: np.ndarray, mask=None) -> tuple[int, int]:
        row = np.ascontiguousarray(row)
        tok = np.zeros(1, dtype=np.int32)
        st = self.lib.orc_greedy_row(_p(row), _dtype_of(row), row.size, _p(mask), _p(tok))
        return int(st), int(tok[0])

    def candidates(self, row: np.ndarray, params: np.ndarray, hist=None, mask=None, cap=None):
        """Returns (status, ids, probs) with the full sorted candidate list (up to cap)."""
        row = np.ascontiguousarray(row)
        v = row.size
        cap = v if cap is None else cap
        ids = np.zeros(cap, dtype=np.int32)
        probs = np.zeros(cap, dtype=np.float64)
        n = np.zeros(1, dtype=np.uint64)
        h = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
        st = self.lib.orc_candidates(_p(row), _dtype_of(row), v, _p(params), _p(h), 0 if h is None else h.size,
                                     _p(mask), cap, _p(ids), _p(probs), _p(n))
        k = int(min(int(n[0]), cap))
        return int(st), ids[:k].copy(), probs[:k].copy(), int(n[0])

    def sample(self, row: np.ndarray, params: np.ndarray, hist=None, mask=None, u: float = 0.5):
        row = np.ascontiguousarray(row)
        tok = np.zeros(1, dtype=np.int32)
        h = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
        st = self.lib.orc_sample(_p(row), _dtype_of(row), row.size, _p(params), _p(h),
                                 0 if h is None else h.size, _p(mask), float(u), _p(tok))
        return int(st), int(tok[0])

    def sample_batch(self, logits: np.ndarray, params: np.ndarray, masks=None, hist=None, hist_off=None,
                     uniforms=None, step: int = 0, n_threads: int = 0, vocab: int | None = None):
        logits = np.ascontiguousarray(logits)
        n, stride = logits.shape
        vocab = stride if vocab is None else vocab
        tok = np.zeros(n, dtype=np.int32)
        sts = np.zeros(n, dtype=np.int32)
        self.lib.orc_sample_batch(_p(logits), _dtype_of(logits), n, stride, vocab, _p(params), _p(masks),
                                  _p(hist), _p(hist_off), _p(uniforms), step, _p(tok), _p(sts), n_threads)
        return tok, sts

    def full_distribution(self, row: np.ndarray, temperature: float) -> np.ndarray:
        row = np.ascontiguousarray(row)
        out = np.zeros(row.size, dtype=np.float32)
        self.lib.orc_full_distribution(_p(row), _dtype_of(row), row.size, ctypes.c_float(temperature), _p(out))
        return out

    def verify(self, target: np.ndarray, drafts: np.ndarray, params: np.ndarray, q=None, n_drafts=None,
               masks=None, hist=None, hist_off=None, uniforms=None, step: int = 0, n_threads: int = 0,
               vocab: int | None = None):
        target = np.ascontiguousarray(target)
        S, k = drafts.shape
        stride = target.shape[-1]
        vocab = stride if vocab is None else vocab
        out = dict(accepted=np.zeros(S, np.int32), tokens=np.zeros((S, k + 1), np.int32),
                   n_tokens=np.zeros(S, np.int32), first_reject=np.zeros(S, np.int32),
                   uniforms_used=np.zeros(S, np.int32), status=np.zeros(S, np.int32))
        self.lib.orc_verify(_p(target), _dtype_of(target), stride, vocab, _p(q), _p(drafts), _p(n_drafts), S, k,
                            _p(params), _p(masks), _p(hist), _p(hist_off), _p(uniforms), step,
                            _p(out["accepted"]), _p(out["tokens"]), _p(out["n_tokens"]),
                            _p(out["first_reject"]), _p(out["uniforms_used"]), _p(out["status"]), n_threads)
        return out


class JsonVocab:
    """A vocabulary for the JSON-grammar oracle (token texts as CSR bytes)."""

    def __init__(self, tokens: list[bytes], flags=None, eos_id: int = -1):
        self.off = np.zeros(len(tokens) + 1, dtype=np.uint64)
        self.off[1:] = np.cumsum([len(t) for t in tokens])
        self.data = np.frombuffer(b"".join(tokens) or b"\0", dtype=np.uint8).copy()
        self.flags = None if flags is None else np.ascontiguousarray(flags, dtype=np.uint8)
        self.vocab = len(tokens)
        self.eos = eos_id


def json_feed(o: Oracle, state: np.ndarray, text: bytes) -> bool:
    """Feeds bytes to a 32-byte state in place; False (state unchanged) when refused."""
    buf = np.frombuffer(text or b"\0", dtype=np.uint8)
    return bool(o.lib.orc_json_feed(state.ctypes.data, buf.ctypes.data, len(text)))


def json_fill_masks(o: Oracle, v: JsonVocab, states: np.ndarray, n_threads: int = 0) -> np.ndarray:
    states = np.ascontiguousarray(states, dtype=np.uint8).reshape(-1, 32)
    w = (v.vocab + 31) // 32
    out = np.zeros((states.shape[0], w), dtype=np.uint32)
    o.lib.orc_json_fill_masks(v.data.ctypes.data, v.off.ctypes.data, _p(v.flags), v.vocab, v.eos,
                              states.ctypes.data, states.shape[0], out.ctypes.data, w, n_threads)
    return out


def json_advance(o: Oracle, v: JsonVocab, states: np.ndarray, tokens: np.ndarray, n_tokens=None) -> np.ndarray:
    """Advances uint8 [n, 32] states in place by tokens ([n] or [n, m] with n_tokens); statuses."""
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    n = states.shape[0]
    stride = tokens.shape[1] if tokens.ndim == 2 else 1
    nt = None if n_tokens is None else np.ascontiguousarray(n_tokens, dtype=np.int32)
    st = np.zeros(n, dtype=np.int32)
    o.lib.orc_json_advance(v.data.ctypes.data, v.off.ctypes.data, _p(v.flags), v.vocab, v.eos, states.ctypes.data,
                           n, tokens.ctypes.data, stride, _p(nt), st.ctypes.data)
    return st


def json_expand(o: Oracle, v: JsonVocab, states: np.ndarray, drafts: np.ndarray, n_drafts=None) -> np.ndarray:
    drafts = np.ascontiguousarray(drafts, dtype=np.int32)
    s, k = drafts.shape
    nd = None if n_drafts is None else np.ascontiguousarray(n_drafts, dtype=np.int32)
    out = np.zeros((s * (k + 1), 32), dtype=np.uint8)
    o.lib.orc_json_expand(v.data.ctypes.data, v.off.ctypes.data, _p(v.flags), v.vocab, v.eos, states.ctypes.data,
                          s, drafts.ctypes.data, k, _p(nd), out.ctypes.data)
    return out


_cache: dict[str, Oracle] = {}


def port() -> Oracle:
    if "port" not in _cache:
        if not PORT_PATH.exists():
            build()
        _cache["port"] = Oracle(PORT_PATH)
    return _cache["port"]


def reference() -> Oracle | None:
    """The engine's own sampler, or None when it was not built (reference sources absent)."""
    if "ref" not in _cache:
        if not REF_PATH.exists():
            return None
        _cache["ref"] = Oracle(REF_PATH)
    return _cache["ref"]
