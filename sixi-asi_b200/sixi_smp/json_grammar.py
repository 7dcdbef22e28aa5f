"""Device-side grammar-mask producer for JSON-object answers (include/sixi_json.h).

The engine decodes `response_format: {"type": "json_object"}` answers under a grammar whose
automaton ships only in binary form (docs/API.md:45-76 in the engine). `JsonGrammar` keeps one
automaton state per row on the device; a constrained decoding step is

    grammar.fill_masks(states, masks)                  # allowed-token bitmask per row
    sampler.sample(logits, params | ROW_MASKED, masks)  # the sampler applies it (-inf)
    grammar.advance(states, tokens)                     # the sampled tokens extend the text

with no host round trip. Synthetic vocabularies and documents for tests and the benchmark are in
`json_vocab` / `json_documents` (no tokenizer or dataset is available offline).
"""

from __future__ import annotations

import ctypes
import json

import numpy as np

from . import INVALID_ARGUMENT, OK, SixiError, _check, _lib, _ptr  # noqa: F401

STATE_BYTES = 32
TOKEN_SPECIAL = 1
MAX_DEPTH = 128
# automaton modes (sixi_json_state.mode)
START, OBJ_FIRST, OBJ_KEY, COLON, VALUE, ARR_FIRST, AFTER, DONE, STRING = range(9)


def _stream(stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def csr(tokens: list[bytes]) -> tuple[np.ndarray, np.ndarray]:
    """Token texts -> (bytes uint8, offsets uint64 [V + 1])."""
    off = np.zeros(len(tokens) + 1, dtype=np.uint64)
    off[1:] = np.cumsum([len(t) for t in tokens])
    data = np.frombuffer(b"".join(tokens), dtype=np.uint8).copy() if off[-1] else np.zeros(1, np.uint8)
    return data, off


class JsonGrammar:
    """A vocabulary uploaded to one device (sixi_json_vocab_create)."""

    def __init__(self, device: int, tokens: list[bytes], flags: np.ndarray | None = None, eos_id: int = -1):
        data, off = csr(tokens)
        fl = None if flags is None else np.ascontiguousarray(flags, dtype=np.uint8)
        h = ctypes.c_void_p()
        _check("sixi_json_vocab_create", _lib().sixi_json_vocab_create(
            device, data.ctypes.data, off.ctypes.data, len(tokens), 0 if fl is None else fl.ctypes.data,
            eos_id, ctypes.byref(h)))
        self.h = h
        self.device = device
        self.vocab = len(tokens)
        self.mask_words = (self.vocab + 31) // 32
        self.eos_id = eos_id

    def close(self) -> None:
        if self.h:
            _lib().sixi_json_vocab_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_states(self, n: int):
        """n start states on the device (uint8 [n, 32])."""
        import torch

        return torch.zeros((n, STATE_BYTES), dtype=torch.uint8, device=torch.device("cuda", self.device))

    def reset(self, states, stream=None) -> None:
        _check("sixi_json_reset", _lib().sixi_json_reset(self.h, _ptr(states), states.shape[0], _stream(stream)))

    def fill_masks(self, states, out=None, stream=None):
        """int32 [n, ceil(V/32)] mask words (bit i % 32 of word i / 32: token i allowed)."""
        import torch

        n = states.shape[0]
        if out is None:
            out = torch.empty((n, self.mask_words), dtype=torch.int32, device=states.device)
        _check("sixi_json_fill_masks", _lib().sixi_json_fill_masks(self.h, _ptr(states), n, _ptr(out),
                                                                     out.stride(0), _stream(stream)))
        return out

    def advance(self, states, tokens, n_tokens=None, out_status=None, stream=None):
        """Applies tokens ([n] or [n, m] with n_tokens [n]) to the states; returns int32 statuses."""
        import torch

        n = states.shape[0]
        if out_status is None:
            out_status = torch.empty(n, dtype=torch.int32, device=states.device)
        stride = tokens.stride(0) if tokens.dim() == 2 else 1
        _check("sixi_json_advance", _lib().sixi_json_advance(self.h, _ptr(states), n, _ptr(tokens), stride,
                                                               _ptr(n_tokens), _ptr(out_status), _stream(stream)))
        return out_status

    def expand_drafts(self, states, drafts, n_drafts=None, out=None, stream=None):
        """[S * (k + 1), 32] states: row j of stream s after its first j drafts."""
        import torch

        s, k = drafts.shape
        if out is None:
            out = torch.empty((s * (k + 1), STATE_BYTES), dtype=torch.uint8, device=states.device)
        _check("sixi_json_expand_drafts", _lib().sixi_json_expand_drafts(
            self.h, _ptr(states), s, _ptr(drafts), k, _ptr(n_drafts), _ptr(out), _stream(stream)))
        return out


# ---------------------------------------------------------------------------------------------
# synthetic vocabularies and documents

_STRUCTURAL = [
    b"{", b"}", b"[", b"]", b":", b",", b'"', b'{"', b'":', b'": "', b'",', b'", "', b'"}', b'"},', b"},",
    b"}}", b"],", b"]}", b"[{", b"{}", b"[]", b", ", b": ", b",\n", b"\n", b"\n  ", b"\n    ", b"  ", b"    ",
    b" ", b"\t", b"\r\n", b"true", b"false", b"null", b" true", b" false", b" null", b"true,", b"null}",
    b'\\n', b'\\"', b"\\\\", b"\\/", b"\\t", b"\\u00", b"\\u", b".0", b".5", b"e+", b"e-", b"E", b"-1", b"-0",
    b"0.", b'"]', b'["', b'":[', b'":{', b'": [', b'": {', b'" :', b" }", b" ]", b"{ ", b"[ ",
]
_UNICODE = ["é", "ü", "ß", "ñ", "日本", "中文", "語", "Ж", "λ", "😀", "🙂", "€", "–", "“", "”", "…"]


def json_vocab(vocab: int = 151_936, seed: int = 5) -> tuple[list[bytes], np.ndarray, int]:
    """A seeded tokenizer-like vocabulary: every single byte, JSON punctuation runs, literals,
    digit runs, escapes, UTF-8 pieces (whole and split), words with and without quotes and
    leading spaces, a few long tokens (> 16 bytes) and control tokens. Returns (tokens, flags,
    eos_id)."""
    rng = np.random.default_rng(seed)
    toks: list[bytes] = [bytes([b]) for b in range(256)]
    seen = set(toks)

    def add(t: bytes) -> None:
        if t and t not in seen and len(toks) < vocab - 3:
            seen.add(t)
            toks.append(t)

    for t in _STRUCTURAL:
        add(t)
    for u in _UNICODE:
        b = u.encode()
        add(b)
        add(b" " + b)
        if len(b) > 1:
            add(b[:-1])  # a split sequence: only valid when the rest follows
    for n in range(100):
        add(str(n).encode())
    for n in range(100, 1000, 7):
        add(str(n).encode())
    for n in (16, 20, 24, 32):
        add(b" " * n)  # long whitespace runs
    letters = np.frombuffer(b"abcdefghijklmnopqrstuvwxyz", dtype=np.uint8)
    punct = [b"()", b"();", b"->", b"==", b"!=", b"/*", b"*/", b"//", b"::", b"=>", b"...", b"--", b"**", b"<=", b">=",
             b"();\n", b"){", b"});", b"':", b"',", b"('", b"')", b"=\"", b"\">", b"</", b"/>", b"#", b"@", b"$", b"%"]
    # form probabilities of a byte-level BPE vocabulary: words with and without a leading space
    # dominate, then capitalised words, CJK and accented pieces (some split mid-character),
    # code punctuation, and a few percent of pieces that carry a double quote
    forms = np.array([0.30, 0.38, 0.07, 0.07, 0.10, 0.01, 0.02, 0.03, 0.02])
    while len(toks) < vocab - 3:
        ln = int(rng.choice([2, 3, 4, 5, 6, 7, 8, 9, 10, 12, 14, 18, 24], p=[.06, .12, .16, .16, .14, .11, .08,
                                                                             .06, .04, .03, .02, .015, .005]))
        w = bytes(letters[rng.integers(0, 26, size=ln)])
        form = int(rng.choice(len(forms), p=forms / forms.sum()))
        if form == 1:
            w = b" " + w
        elif form == 2:
            w = w.capitalize()
        elif form == 3:
            w = b" " + w.capitalize()
        elif form in (4, 5):
            cps = rng.integers(0x4E00, 0xA000, size=int(rng.integers(1, 3))) if rng.random() < 0.7 else \
                rng.integers(0xC0, 0x250, size=int(rng.integers(1, 4)))
            w = "".join(chr(int(c)) for c in cps).encode()
            if form == 5:  # a piece split inside a UTF-8 sequence
                cut = int(rng.integers(1, len(w)))
                w = w[:cut] if rng.random() < 0.5 else w[cut:]
            elif rng.random() < 0.3:
                w = b" " + w
        elif form == 6:
            w = punct[int(rng.integers(0, len(punct)))] + (w[:2] if rng.random() < 0.5 else b"")
        elif form == 7:
            w = [b'"' + w, w + b'"', b'"' + w + b'":', b' "' + w + b'": "', b' "' + w, w + b'",'][int(rng.integers(0, 6))]
        elif form == 8:
            w = str(int(rng.integers(0, 10 ** int(rng.integers(1, 6))))).encode()
        add(w)
    specials = [b"<|im_start|>", b"<|im_end|>", b"<|endoftext|>"]
    flags = np.zeros(len(toks) + len(specials), dtype=np.uint8)
    flags[len(toks):] = TOKEN_SPECIAL
    toks += specials
    eos = len(toks) - 1
    flags[eos] = 0  # end-of-sequence: allowed exactly at the end of the document
    return toks, flags, eos


def _random_value(rng: np.random.Generator, depth: int):
    kind = int(rng.integers(0, 10 if depth < 4 else 7))
    if kind <= 2:
        words = ["alpha", "beta", "name", "value", "x", "日本", "é", "line\nbreak", 'quo"te', "back\\slash", "tab\t",
                 "😀", "", "id", "count"]
        return " ".join(str(rng.choice(words)) for _ in range(int(rng.integers(0, 4))))
    if kind == 3:
        return int(rng.integers(-10**6, 10**6))
    if kind == 4:
        return float(rng.normal() * 10 ** int(rng.integers(-5, 6)))
    if kind == 5:
        return [True, False, None][int(rng.integers(0, 3))]
    if kind == 6:
        return int(rng.integers(0, 10))
    if kind <= 8:
        return {f"k{int(rng.integers(0, 100))}": _random_value(rng, depth + 1) for _ in range(int(rng.integers(0, 5)))}
    return [_random_value(rng, depth + 1) for _ in range(int(rng.integers(0, 5)))]


def json_documents(n: int, seed: int = 6) -> list[bytes]:
    """n seeded JSON-object documents with mixed formatting (compact, spaced, indented; ASCII or
    raw UTF-8)."""
    rng = np.random.default_rng(seed)
    docs = []
    for _ in range(n):
        obj = {f"key{i}": _random_value(rng, 1) for i in range(int(rng.integers(1, 6)))}
        style = int(rng.integers(0, 3))
        kw = dict(ensure_ascii=bool(rng.integers(0, 2)))
        if style == 0:
            s = json.dumps(obj, separators=(",", ":"), **kw)
        elif style == 1:
            s = json.dumps(obj, **kw)
        else:
            s = json.dumps(obj, indent=int(rng.integers(1, 5)), **kw)
        docs.append(s.encode())
    return docs


class Tokenizer:
    """Greedy longest-match tokenizer over a vocabulary (every single byte is a token)."""

    def __init__(self, tokens: list[bytes], flags: np.ndarray | None = None):
        self.ids = {}
        for i, t in enumerate(tokens):
            if t and (flags is None or not flags[i] & TOKEN_SPECIAL) and t not in self.ids:
                self.ids[t] = i
        self.maxlen = max(len(t) for t in self.ids)

    def encode(self, text: bytes) -> list[int]:
        out, i = [], 0
        while i < len(text):
            for ln in range(min(self.maxlen, len(text) - i), 0, -1):
                t = self.ids.get(text[i:i + ln])
                if t is not None:
                    out.append(t)
                    i += ln
                    break
        return out


def prefix_states_tokens(docs: list[bytes], tok: Tokenizer, rows: int, seed: int = 7,
                         max_len: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Token prefixes of random documents (one per row, cut at a random token boundary), padded:
    (tokens int32 [rows, L], lengths int32 [rows]). Applying them to start states gives states
    spread over the automaton's modes the way decoding visits them."""
    rng = np.random.default_rng(seed)
    seqs = []
    for r in range(rows):
        ids = tok.encode(docs[int(rng.integers(0, len(docs)))])
        cut = int(rng.integers(0, len(ids) + 1))
        seqs.append(ids[:cut])
    L = max(max_len, max((len(s) for s in seqs), default=0), 1)
    out = np.zeros((rows, L), dtype=np.int32)
    lens = np.zeros(rows, dtype=np.int32)
    for r, s in enumerate(seqs):
        out[r, :len(s)] = s
        lens[r] = len(s)
    return out, lens
