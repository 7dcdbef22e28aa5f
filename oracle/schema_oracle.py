"""TEST INFRASTRUCTURE ONLY: an independent validator of complete documents against a JSON schema,
the checker of the json_schema grammar (include/sixi_schema.h). Nothing in the product imports it.

It parses the document text with its own recursive-descent JSON parser (keeping every value's
raw text) and validates the schema's semantics directly: allOf as "every branch holds" and anyOf
as "some branch holds" (the library merges and dispatches instead), $ref by lookup, formats and
patterns with Python's `re` (expressions written here, not taken from the library). On top of
JSON Schema it checks the textual conventions the grammar documents, so that "the automaton
accepts the text as a complete document" can be compared with "this validator accepts it":
  - nothing may follow the top-level value (whitespace before it is fine);
  - a declared property's key is written literally (its JSON escaping, minimal escapes);
  - enum / const values are written in compact JSON;
  - integers are written without fraction or exponent;
  - strings under a pattern or format hold printable ASCII without escapes;
  - a declared key is not repeated (undeclared keys are not tracked), and an undeclared key is
    written without escapes;
  - string lengths count code points, each escape sequence as one.
The engine's own automaton is binary-only, so parity with the engine is unpinned; this validator
pins the grammar to the schema's meaning instead (tests/test_json_schema.py).
"""

from __future__ import annotations

import json
import re

_WS = b" \t\n\r"


class _Bad(Exception):
    pass


class _V:
    __slots__ = ("kind", "val", "raw", "items", "keys")

    def __init__(self, kind, val, raw, items=None, keys=None):
        self.kind, self.val, self.raw, self.items, self.keys = kind, val, raw, items, keys


class _P:
    def __init__(self, t: bytes):
        self.t, self.i = t, 0

    def ws(self):
        while self.i < len(self.t) and self.t[self.i] in _WS:
            self.i += 1

    def value(self, depth=0):
        if depth > 64:
            raise _Bad("deep")
        self.ws()
        if self.i >= len(self.t):
            raise _Bad("end")
        c = self.t[self.i]
        s0 = self.i
        if c == ord("{"):
            self.i += 1
            keys, items = [], []
            self.ws()
            if self.i < len(self.t) and self.t[self.i] == ord("}"):
                self.i += 1
                return _V("object", None, self.t[s0:self.i], items, keys)
            while True:
                self.ws()
                k = self.string()
                self.ws()
                if self.i >= len(self.t) or self.t[self.i] != ord(":"):
                    raise _Bad(":")
                self.i += 1
                v = self.value(depth + 1)
                keys.append(k)
                items.append(v)
                self.ws()
                if self.i < len(self.t) and self.t[self.i] == ord(","):
                    self.i += 1
                    continue
                if self.i < len(self.t) and self.t[self.i] == ord("}"):
                    self.i += 1
                    return _V("object", None, self.t[s0:self.i], items, keys)
                raise _Bad("}")
        if c == ord("["):
            self.i += 1
            items = []
            self.ws()
            if self.i < len(self.t) and self.t[self.i] == ord("]"):
                self.i += 1
                return _V("array", None, self.t[s0:self.i], items)
            while True:
                items.append(self.value(depth + 1))
                self.ws()
                if self.i < len(self.t) and self.t[self.i] == ord(","):
                    self.i += 1
                    continue
                if self.i < len(self.t) and self.t[self.i] == ord("]"):
                    self.i += 1
                    return _V("array", None, self.t[s0:self.i], items)
                raise _Bad("]")
        if c == ord('"'):
            return self.string()
        for lit, val in ((b"true", True), (b"false", False), (b"null", None)):
            if self.t.startswith(lit, self.i):
                self.i += len(lit)
                return _V("literal", val, lit)
        m = re.compile(rb"-?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][+-]?[0-9]+)?").match(self.t, self.i)
        if not m or m.end() == self.i:
            raise _Bad("value")
        self.i = m.end()
        return _V("number", float(m.group(0)), m.group(0))

    def string(self):
        if self.i >= len(self.t) or self.t[self.i] != ord('"'):
            raise _Bad('"')
        j = self.i + 1
        while True:
            if j >= len(self.t):
                raise _Bad("unterminated")
            c = self.t[j]
            if c == ord('"'):
                break
            if c == ord("\\"):
                j += 2
                continue
            j += 1
        raw = self.t[self.i:j + 1]
        self.i = j + 1
        try:
            val = json.loads(raw.decode("utf-8"))  # escapes, UTF-8 and control characters checked
        except Exception as e:
            raise _Bad("string") from e
        return _V("string", val, raw)


def _escape(s: str) -> bytes:
    out = []
    for ch in s:
        o = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif ch in "\n\r\t\b\f":
            out.append({"\n": "\\n", "\r": "\\r", "\t": "\\t", "\b": "\\b", "\f": "\\f"}[ch])
        elif o < 0x20:
            out.append("\\u%04x" % o)
        else:
            out.append(ch)
    return "".join(out).encode("utf-8")


def _compact(v) -> bytes:
    if isinstance(v, str):
        return b'"' + _escape(v) + b'"'
    if isinstance(v, bool) or v is None:
        return {True: b"true", False: b"false", None: b"null"}[v]
    if isinstance(v, list):
        return b"[" + b",".join(_compact(x) for x in v) + b"]"
    if isinstance(v, dict):
        return b"{" + b",".join(b'"' + _escape(k) + b'":' + _compact(x) for k, x in v.items()) + b"}"
    return json.dumps(v).encode()


def _units(raw: bytes) -> int:
    """Characters of a string's raw text (quotes included): each escape sequence counts as one,
    each UTF-8 encoded code point as one."""
    body = raw[1:-1]
    n, i = 0, 0
    while i < len(body):
        c = body[i]
        if c == 0x5C:  # backslash
            i += 6 if body[i + 1] == ord("u") else 2
        elif c < 0x80:
            i += 1
        elif c < 0xE0:
            i += 2
        elif c < 0xF0:
            i += 3
        else:
            i += 4
        n += 1
    return n


_FORMATS = {
    "date": r"\d{4}-(0[1-9]|1[012])-(0[1-9]|[12]\d|3[01])",
    "time": r"([01]\d|2[0-3]):[0-5]\d:([0-5]\d|60)(\.\d+)?([Zz]|[+-]([01]\d|2[0-3]):[0-5]\d)",
    "uuid": r"[0-9a-fA-F]{8}(-[0-9a-fA-F]{4}){3}-[0-9a-fA-F]{12}",
}
_FORMATS["date-time"] = _FORMATS["date"] + "[Tt]" + _FORMATS["time"]


class Validator:
    def __init__(self, schema, raw_enum_texts: dict | None = None):
        self.root = schema
        self.raw_enums = raw_enum_texts or {}

    def _ref(self, ref):
        if ref == "#":
            return self.root
        for sect in ("$defs", "definitions"):
            pre = "#/" + sect + "/"
            if ref.startswith(pre):
                return self.root[sect][ref[len(pre):]]
        raise KeyError(ref)

    @staticmethod
    def _type_of(v: _V) -> set:
        if v.kind == "object":
            return {"object"}
        if v.kind == "array":
            return {"array"}
        if v.kind == "string":
            return {"string"}
        if v.kind == "literal":
            return {"null"} if v.val is None else {"boolean"}
        if re.fullmatch(rb"-?(0|[1-9][0-9]*)", v.raw):  # integers written as integers
            return {"integer", "number"}
        return {"number"}

    def ok(self, v: _V, s, depth=0) -> bool:
        if depth > 200:
            return False
        if s is True:
            return True
        if s is False:
            return False
        if "$ref" in s and not self.ok(v, self._ref(s["$ref"]), depth + 1):
            return False
        if "allOf" in s and not all(self.ok(v, x, depth + 1) for x in s["allOf"]):
            return False
        if "anyOf" in s and not any(self.ok(v, x, depth + 1) for x in s["anyOf"]):
            return False
        t = s.get("type")
        if t is None:
            # without a type, the keywords of one kind imply that kind (the grammar's rule)
            if any(k in s for k in ("properties", "required", "additionalProperties")):
                t = "object"
            elif any(k in s for k in ("items", "prefixItems", "minItems", "maxItems")):
                t = "array"
            elif any(k in s for k in ("minLength", "maxLength", "pattern", "format")):
                t = "string"
            elif any(k in s for k in ("minimum", "maximum", "exclusiveMinimum", "exclusiveMaximum")):
                t = "integer"
        types = [t] if isinstance(t, str) else (t or [])
        vt = self._type_of(v)
        if types and not any(x in vt for x in types):
            return False
        if "const" in s or "enum" in s:
            allowed = [s["const"]] if "const" in s else list(s["enum"])
            if "const" in s and "enum" in s and _compact(s["const"]) not in [_compact(x) for x in s["enum"]]:
                return False
            if v.raw not in [_compact(x) for x in allowed]:
                return False
        if v.kind == "number" and "integer" in vt and "integer" in types:
            x = int(v.raw)
            if "minimum" in s and x < s["minimum"]:
                return False
            if "maximum" in s and x > s["maximum"]:
                return False
            if "exclusiveMinimum" in s and x <= s["exclusiveMinimum"]:
                return False
            if "exclusiveMaximum" in s and x >= s["exclusiveMaximum"]:
                return False
        if v.kind == "string":
            n = _units(v.raw)  # code points, an escape sequence counting as one
            if n < s.get("minLength", 0) or n > s.get("maxLength", 1 << 62):
                return False
            pat = s.get("pattern")
            fmt = s.get("format")
            if pat is not None or fmt is not None:
                body = v.raw[1:-1]
                if b"\\" in body or any(c < 0x20 or c > 0x7E for c in body):
                    return False
                if pat is not None and not re.fullmatch(pat[1:-1], v.val):
                    return False
                if fmt is not None and not re.fullmatch(_FORMATS[fmt], v.val):
                    return False
        if v.kind == "array":
            pre = s.get("prefixItems", [])
            items = s.get("items", True)
            if len(v.items) < s.get("minItems", 0) or len(v.items) > s.get("maxItems", 1 << 62):
                return False
            for i, x in enumerate(v.items):
                sub = pre[i] if i < len(pre) else items
                if not self.ok(x, sub, depth + 1):
                    return False
        if v.kind == "object":
            props = s.get("properties", {})
            addl = s.get("additionalProperties", True)
            seen = set()
            for k, x in zip(v.keys, v.items):
                if k.val in props:
                    if k.val in seen:  # a declared key may not repeat
                        return False
                    if k.raw != b'"' + _escape(k.val) + b'"':
                        return False
                    if not self.ok(x, props[k.val], depth + 1):
                        return False
                else:
                    if b"\\" in k.raw:  # an undeclared key is written without escapes
                        return False
                    if not self.ok(x, addl, depth + 1):
                        return False
                seen.add(k.val)
            if any(r not in seen for r in s.get("required", [])):
                return False
        return True

    def accepts(self, text: bytes) -> bool:
        """The text is one complete document matching the schema (the grammar's conventions)."""
        p = _P(text)
        try:
            v = p.value()
        except _Bad:
            return False
        if p.i != len(text):
            return False
        return self.ok(v, self.root)
