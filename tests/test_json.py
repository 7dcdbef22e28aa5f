"""CPU tests of the JSON-object grammar automaton behind the mask producer (include/sixi_json.h).

The engine's automaton is binary-only, so the oracle (oracle/sixi_json_oracle.c) is pinned to an
independent RFC 8259 parser, Python's json module: every prefix of a valid document is accepted,
and on mutated documents "the oracle reaches the end of a complete object" and "json.loads returns
a dict" agree. The synthetic vocabulary and tokenizer used by the device tests and the benchmark
are checked here too, and the library's JSON entry points reject bad arguments without a GPU."""

from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest

from oracle import binding as B


def _reject_constant(name):
    raise ValueError(f"non-RFC constant {name}")


def loads_object(text: bytes):
    """The dict json.loads reads from `text` under RFC 8259 (strict UTF-8, no NaN/Infinity), or
    None when it is not exactly one JSON object followed by nothing."""
    try:
        s = text.decode("utf-8")
        v = json.loads(s, parse_constant=_reject_constant)
    except (UnicodeDecodeError, ValueError, RecursionError):
        return None
    if not isinstance(v, dict) or s != s.rstrip(" \t\n\r"):
        return None
    return v


def walk(o, text: bytes):
    """(all bytes accepted, final state)."""
    st = np.zeros(32, np.uint8)
    for i in range(len(text)):
        if not B.json_feed(o, st, text[i:i + 1]):
            return False, st
    return True, st


def test_every_prefix_of_a_valid_document_is_accepted(port):
    from sixi_smp.json_grammar import DONE, json_documents

    docs = json_documents(150, seed=11)
    docs += [b"{}", b' \n{"a":{}}', b'{"a":[[],[[]],{}]}', '{"日本":"é😀","x":-0.5e+10}'.encode(),
             b'{"s":"\\u00e9\\n\\"\\\\\\/\\b\\f\\r\\t"}', b'{"n":[0,-0,1e5,1E-5,2.25,-12.5e3,true,false,null]}']
    for d in docs:
        assert loads_object(d) is not None, d
        ok, st = walk(port, d)
        assert ok, d
        assert st[0] == DONE, d


def test_rejections(port):
    bad = [b"[1]", b'"x"', b"1", b"{", b'{"a" 1}', b'{"a": 01}', b'{"a": 1.}', b'{"a": .5}', b'{"a": +1}',
           b'{"a": 1e}', b'{"a": tru}', b'{"a": nul}', b'{"a": "\x01"}', b'{"a": "\\x"}', b'{"a": "\\u12g4"}',
           b'{"a": 1,}', b'{,}', b'{"a":1} ', b"{} {}", b'{"a": NaN}', b'{"a": Infinity}', b"{'a': 1}",
           b'{"a": "\xc0\x80"}', b'{"a": "\xed\xa0\x80"}', b'{"a": "\xf4\x90\x80\x80"}', b'{"a": "\xe0\x80\x80"}',
           b'{"a": "\xff"}', b'\xef\xbb\xbf{}', b'{"a":]', b'{"a":[}']
    for t in bad:
        ok, st = walk(port, t)
        complete = ok and st[0] == 7
        assert not complete, t
        assert loads_object(t) is None, t


def test_mutations_agree_with_pythons_json(port):
    from sixi_smp.json_grammar import DONE, json_documents

    rng = np.random.default_rng(12)
    docs = json_documents(120, seed=13)
    alphabet = list(b'{}[]:,"\\ 0123456789.eE+-tfnrul\t\n\x01') + [0xC3, 0xA9, 0xE6, 0x97, 0xA5, 0xF0, 0x9F, 0xED,
                                                                   0xA0, 0x80, 0xFF]
    agree = complete = 0
    for d in docs:
        for _ in range(40):
            b = bytearray(d)
            for _ in range(int(rng.integers(1, 4))):
                op = int(rng.integers(0, 3))
                i = int(rng.integers(0, len(b) + 1))
                c = int(alphabet[int(rng.integers(0, len(alphabet)))])
                if op == 0:
                    b.insert(i, c)
                elif op == 1 and i < len(b):
                    del b[i]
                elif i < len(b):
                    b[i] = c
            text = bytes(b)
            ok, st = walk(port, text)
            mine = ok and st[0] == DONE
            theirs = loads_object(text) is not None
            assert mine == theirs, text
            agree += 1
            complete += mine
    assert agree == 120 * 40 and complete > 100


def test_depth_limit(port):
    deep_ok = b'{"a":' + b"[" * 127 + b"]" * 127 + b"}"
    ok, st = walk(port, deep_ok)
    assert ok and st[0] == 7
    too_deep = b'{"a":' + b"[" * 128
    ok, _ = walk(port, too_deep)
    assert not ok


def test_masks_advance_and_expand_are_consistent(port):
    """fill_masks, advance and expand agree with feeding token texts one by one."""
    from sixi_smp.json_grammar import Tokenizer, json_documents, json_vocab, prefix_states_tokens

    toks, flags, eos = json_vocab(4096, seed=3)
    v = B.JsonVocab(toks, flags, eos)
    tk = Tokenizer(toks, flags)
    docs = json_documents(40, seed=4)
    for d in docs:
        assert b"".join(toks[i] for i in tk.encode(d)) == d
    pre, lens = prefix_states_tokens(docs, tk, 24, seed=5)
    states = np.zeros((24, 32), np.uint8)
    st = B.json_advance(port, v, states, pre, lens)
    assert (st == 0).all()
    masks = B.json_fill_masks(port, v, states, n_threads=4)
    rng = np.random.default_rng(6)
    for r in range(24):
        for i in rng.integers(0, len(toks), size=200).tolist() + [eos]:
            s = states[r].copy()
            if i == eos:
                want = s[0] == 7
            elif flags[i]:
                want = False
            else:
                want = B.json_feed(port, s, toks[i])
            assert bool((masks[r, i // 32] >> (i % 32)) & 1) == want
    # a refused token freezes the row and reports INVALID_ARGUMENT
    frozen = states.copy()
    bad = np.array([toks.index(b"]") if s[0] == 0 else eos if s[0] != 7 else 0 for s in frozen], np.int32)
    st2 = B.json_advance(port, v, frozen, bad)
    assert ((st2 == 1) == (frozen[:, 6] == 1)).all()
    drafts = rng.integers(0, len(toks), size=(24, 4)).astype(np.int32)
    ex = B.json_expand(port, v, states, drafts)
    assert (ex[0::5] == states).all()


def test_library_entry_points_reject_bad_arguments_without_gpu():
    import sixi_smp

    lib = sixi_smp.load()
    h = ctypes.c_void_p()
    off = np.zeros(2, np.uint64)
    assert lib.sixi_json_vocab_create(0, None, off.ctypes.data, 0, None, -1, ctypes.byref(h)) == 1
    assert lib.sixi_json_vocab_create(0, None, off.ctypes.data, 1, None, 5, ctypes.byref(h)) == 1
    assert lib.sixi_json_fill_masks(None, None, 0, None, 0, None) == 1
    assert lib.sixi_json_advance(None, None, 0, None, 0, None, None, None) == 1
    assert lib.sixi_json_vocab_size(None) == 0


@pytest.mark.parametrize("n", [1, 7])
def test_state_layout(n):
    from sixi_smp.json_grammar import STATE_BYTES

    assert STATE_BYTES == 32
    assert np.zeros((n, STATE_BYTES), np.uint8).nbytes == 32 * n
