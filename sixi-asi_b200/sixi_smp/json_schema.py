"""Grammar masks for `response_format: json_schema` answers (include/sixi_schema.h).

`SchemaGrammar(device, schema, tokens, flags, eos_id)` compiles a JSON schema against a tokenizer
vocabulary (in the library, on the host) and uploads both; one automaton state per row lives on
the device. A constrained decoding step is

    grammar.fill_masks(states, masks)                   # allowed-token bitmask per row
    sampler.sample(logits, params | ROW_MASKED, masks)   # the sampler applies it (-inf)
    grammar.advance(states, tokens)                      # the sampled tokens extend the text

Schema errors raise `SchemaError` with the library's message, which names the place in the schema
("JSON schema: #/properties/a: keyword 'uniqueItems' is not supported"). `device=-1` compiles for
host checks only (`check_text`), which needs no GPU.
"""

from __future__ import annotations

import ctypes
import json

import numpy as np

from . import INVALID_ARGUMENT, _check, _lib, _ptr  # noqa: F401
from .json_grammar import csr

STATE_BYTES = 800  # SIXI_SCHEMA_STATE_BYTES
MAX_DEPTH = 32
NOT_PREFIX, PREFIX, COMPLETE = 0, 1, 2


class SchemaError(ValueError):
    pass


def _stream(stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


class SchemaGrammar:
    def __init__(self, device: int, schema, tokens: list[bytes] | None = None, flags=None, eos_id: int = -1):
        text = schema if isinstance(schema, (str, bytes)) else json.dumps(schema)
        raw = text.encode() if isinstance(text, str) else text
        tokens = tokens or []
        data, off = csr(tokens)
        fl = None if flags is None else np.ascontiguousarray(flags, dtype=np.uint8)
        err = ctypes.create_string_buffer(512)
        h = ctypes.c_void_p()
        st = _lib().sixi_schema_compile(device, raw, len(raw), data.ctypes.data, off.ctypes.data, len(tokens),
                                        0 if fl is None else fl.ctypes.data, eos_id, err, len(err), ctypes.byref(h))
        if st != 0:
            msg = err.value.decode(errors="replace")
            if st == INVALID_ARGUMENT and msg:
                raise SchemaError(msg)
            _check("sixi_schema_compile", st)
        self.h = h
        self.device = device
        self.vocab = len(tokens)
        self.mask_words = (self.vocab + 31) // 32
        self.eos_id = eos_id

    def close(self) -> None:
        if self.h:
            _lib().sixi_schema_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check_text(self, text: bytes) -> int:
        """NOT_PREFIX, PREFIX or COMPLETE for a text under the schema (host automaton)."""
        buf = np.frombuffer(text or b"\0", dtype=np.uint8)
        return int(_lib().sixi_schema_check_text(self.h, buf.ctypes.data, len(text)))

    def new_states(self, n: int):
        """n start states on the device (uint8 [n, STATE_BYTES])."""
        import torch

        st = torch.zeros((n, STATE_BYTES), dtype=torch.uint8, device=torch.device("cuda", self.device))
        self.reset(st)
        return st

    def reset(self, states, stream=None) -> None:
        _check("sixi_schema_reset", _lib().sixi_schema_reset(self.h, _ptr(states), states.shape[0], _stream(stream)))

    def fill_masks(self, states, out=None, stream=None):
        import torch

        n = states.shape[0]
        if out is None:
            out = torch.empty((n, self.mask_words), dtype=torch.int32, device=states.device)
        _check("sixi_schema_fill_masks", _lib().sixi_schema_fill_masks(self.h, _ptr(states), n, _ptr(out),
                                                                       out.stride(0), _stream(stream)))
        return out

    def advance(self, states, tokens, n_tokens=None, out_status=None, stream=None):
        import torch

        n = states.shape[0]
        if out_status is None:
            out_status = torch.empty(n, dtype=torch.int32, device=states.device)
        stride = tokens.stride(0) if tokens.dim() == 2 else 1
        _check("sixi_schema_advance", _lib().sixi_schema_advance(self.h, _ptr(states), n, _ptr(tokens), stride,
                                                                 _ptr(n_tokens), _ptr(out_status), _stream(stream)))
        return out_status
