"""The json_schema grammar (include/sixi_schema.h) on the host: the library's compiler and automaton
(sixi_schema_check_text, no GPU) against an independent validator of complete documents
(oracle/schema_oracle.py, recursive-descent over the text, allOf / anyOf by their meaning).

  refusals        unsupported keywords and constructs are refused with the place in the schema
  documents       seeded valid documents of each schema (random whitespace, optional properties,
                  additional properties, enum values, formats): every prefix is a prefix for the
                  automaton, the whole is complete, and the validator accepts it
  mutations       random byte edits of those documents: the automaton reports "complete" exactly
                  when the validator accepts the edited text
  random walks    texts grown one allowed byte at a time (the automaton's own choices): no prefix
                  is a dead end (some byte is allowed, or the document is complete), and every
                  completed text is accepted by the validator
"""

from __future__ import annotations

import json
import random

import pytest

from oracle.schema_oracle import Validator
from sixi_smp.json_schema import COMPLETE, NOT_PREFIX, PREFIX, SchemaError, SchemaGrammar

PERSON = {
    "type": "object",
    "properties": {
        "name": {"type": "string", "minLength": 1, "maxLength": 12},
        "age": {"type": "integer", "minimum": 0, "maximum": 150},
        "tags": {"type": "array", "items": {"enum": ["red", "green", "blue"]}, "maxItems": 4},
        "address": {"type": "object", "properties": {"street": {"type": "string"},
                                                      "zip": {"type": "string", "pattern": "^[0-9]{5}$"}},
                    "required": ["street"], "additionalProperties": False},
        "active": {"type": "boolean"},
        "nick": {"anyOf": [{"type": "string", "maxLength": 6}, {"type": "null"}]},
    },
    "required": ["name", "age"],
    "additionalProperties": False,
}
TREE = {
    "$defs": {"node": {"type": "object", "properties": {"v": {"type": "integer", "minimum": -99, "maximum": 99},
                                                        "kids": {"type": "array", "items": {"$ref": "#/$defs/node"},
                                                                 "maxItems": 3}},
                       "required": ["v"], "additionalProperties": False}},
    "$ref": "#/$defs/node",
}
TUPLE = {"type": "array", "prefixItems": [{"type": "integer"}, {"type": "string", "maxLength": 4}],
         "items": {"type": "boolean"}, "minItems": 2, "maxItems": 5}
ALLOF = {"allOf": [{"type": "object", "properties": {"a": {"type": "integer", "minimum": 1}}, "required": ["a"]},
                   {"properties": {"b": {"type": "string", "enum": ["x", "y"]}, "a": {"maximum": 9}},
                    "required": ["b"]}]}
ENUM = {"enum": [1, "a", None, True, {"k": [1, 2]}, [3, "b"]]}
FORMATS = {"type": "object", "properties": {"d": {"type": "string", "format": "date"},
                                            "t": {"type": "string", "format": "time"},
                                            "dt": {"type": "string", "format": "date-time"},
                                            "u": {"type": "string", "format": "uuid"}},
           "required": ["d", "u"], "additionalProperties": False}
BOUNDED = {"type": "integer", "exclusiveMinimum": -5, "exclusiveMaximum": 1000}
OPEN = {"type": "object", "properties": {"n": {"type": "string"}},
        "additionalProperties": {"type": "integer", "maximum": 50}, "required": ["n"]}
NUMBER = {"type": ["number", "null"]}
SHORT = {"type": "string", "minLength": 2, "maxLength": 5}
SCHEMAS = {"person": PERSON, "tree": TREE, "tuple": TUPLE, "allof": ALLOF, "enum": ENUM, "formats": FORMATS,
           "bounded": BOUNDED, "open": OPEN, "number": NUMBER, "short": SHORT}


# ---------------------------------------------------------------------------------------- generator
class Gen:
    """Random valid documents of the test schemas, written with random whitespace between tokens
    (none inside enum values or after the top-level value)."""

    def __init__(self, schema, seed):
        self.root = schema
        self.r = random.Random(seed)

    def ws(self):
        return self.r.choice(["", "", "", " ", "\n  ", "\t"])

    def ref(self, s):
        while isinstance(s, dict) and "$ref" in s:
            ref = s["$ref"]
            s = self.root if ref == "#" else self.root["$defs"][ref.split("/")[-1]]
        return s

    def merged(self, s):
        s = self.ref(s)
        if not isinstance(s, dict) or "allOf" not in s:
            return s
        m = {k: v for k, v in s.items() if k != "allOf"}
        for b in s["allOf"]:
            b = self.merged(b)
            for k, v in b.items():
                if k == "properties":
                    props = dict(m.get("properties", {}))
                    for pk, pv in v.items():
                        props[pk] = {"allOf": [props[pk], pv]} if pk in props else pv
                    m["properties"] = props
                elif k == "required":
                    m["required"] = list(dict.fromkeys(m.get("required", []) + v))
                elif k == "maximum":
                    m[k] = min(m.get(k, v), v)
                elif k == "minimum":
                    m[k] = max(m.get(k, v), v)
                else:
                    m[k] = v
        return m

    def value(self, s, depth=0) -> str:
        s = self.merged(s)
        if s is True or s == {}:
            s = {"type": self.r.choice(["integer", "string", "boolean", "null"])}
        if "anyOf" in s:
            return self.value(self.r.choice(s["anyOf"]), depth)
        if "enum" in s or "const" in s:
            vals = [s["const"]] if "const" in s else s["enum"]
            return json.dumps(self.r.choice(vals), separators=(",", ":"), ensure_ascii=False)
        t = s.get("type")
        if isinstance(t, list):
            t = self.r.choice(t)
        if t is None:
            t = "object" if "properties" in s else "array" if "prefixItems" in s or "items" in s else "string"
        if t == "null":
            return "null"
        if t == "boolean":
            return self.r.choice(["true", "false"])
        if t == "integer":
            lo = s.get("minimum", s.get("exclusiveMinimum", -1000) + 1 if "exclusiveMinimum" in s else -1000)
            hi = s.get("maximum", s.get("exclusiveMaximum", 100000) - 1 if "exclusiveMaximum" in s else 100000)
            return str(self.r.randint(int(lo), int(hi)))
        if t == "number":
            return self.r.choice([str(self.r.randint(-50, 50)), repr(round(self.r.uniform(-1e3, 1e3), 3)),
                                  "%de%d" % (self.r.randint(1, 9), self.r.randint(-3, 3))])
        if t == "string":
            return '"' + self.string(s) + '"'
        if t == "array":
            pre = s.get("prefixItems", [])
            items = s.get("items", True)
            lo = s.get("minItems", 0)
            hi = s.get("maxItems", lo + 3)
            n = self.r.randint(lo, min(hi, lo + 3)) if items is not False else min(len(pre), hi)
            n = max(n, lo)
            if depth > 3:
                n = lo
            out = []
            for i in range(n):
                sub = pre[i] if i < len(pre) else items
                out.append(self.ws() + self.value(sub, depth + 1) + self.ws())
            return "[" + ",".join(out) + "]" if out else "[" + self.ws() + "]"
        # object
        props = s.get("properties", {})
        req = s.get("required", [])
        keys = [k for k in props if k in req or (depth < 3 and self.r.random() < 0.5)]
        addl = s.get("additionalProperties", True)
        extra = []
        if addl is not False and self.r.random() < 0.4:
            extra = ["x%d" % self.r.randint(0, 99)]
            extra = [k for k in extra if k not in props]
        self.r.shuffle(keys)
        parts = []
        for k in keys + extra:
            sub = props[k] if k in props else addl
            parts.append(self.ws() + json.dumps(k) + self.ws() + ":" + self.ws() + self.value(sub, depth + 1) + self.ws())
        return "{" + ",".join(parts) + "}" if parts else "{" + self.ws() + "}"

    def string(self, s):
        fmt = s.get("format")
        r = self.r
        if fmt == "date":
            return "%04d-%02d-%02d" % (r.randint(1900, 2100), r.randint(1, 12), r.randint(1, 28))
        if fmt == "time":
            return "%02d:%02d:%02d%s" % (r.randint(0, 23), r.randint(0, 59), r.randint(0, 59), r.choice(["Z", "+05:30"]))
        if fmt == "date-time":
            return self.string({"format": "date"}) + "T" + self.string({"format": "time"})
        if fmt == "uuid":
            h = "".join(r.choice("0123456789abcdef") for _ in range(32))
            return "-".join([h[:8], h[8:12], h[12:16], h[16:20], h[20:]])
        if s.get("pattern") == "^[0-9]{5}$":
            return "".join(r.choice("0123456789") for _ in range(5))
        lo = s.get("minLength", 0)
        hi = min(s.get("maxLength", lo + 8), lo + 8)
        n = r.randint(lo, hi)
        pieces = ["a", "Z", "é", "中", "\\n", "\\\"", "\\u00e9", " ", "7"]
        return "".join(r.choice(pieces) for _ in range(n))


def docs(name, n, seed):
    g = Gen(SCHEMAS[name], seed)
    return [(g.ws().strip("\t") + g.value(SCHEMAS[name])).encode() for _ in range(n)]


@pytest.fixture(scope="module")
def grammars():
    out = {k: SchemaGrammar(-1, v) for k, v in SCHEMAS.items()}
    yield out
    for g in out.values():
        g.close()


@pytest.mark.parametrize("name", sorted(SCHEMAS))
def test_valid_documents_and_their_prefixes(grammars, name):
    g, v = grammars[name], Validator(SCHEMAS[name])
    for d in docs(name, 40, seed=hash(name) % 1000):
        assert v.accepts(d), d
        assert g.check_text(d) == COMPLETE, d
        for i in range(len(d)):
            assert g.check_text(d[:i]) != NOT_PREFIX, (d, i)


@pytest.mark.parametrize("name", sorted(SCHEMAS))
def test_mutations_agree_with_the_validator(grammars, name):
    g, v = grammars[name], Validator(SCHEMAS[name])
    r = random.Random(7 + len(name))
    alphabet = b'{}[]",:01-9aeflnrstux \\.E+' + bytes([0xC3, 0xA9])
    n_acc = 0
    for d in docs(name, 60, seed=31 + len(name)):
        for _ in range(15):
            t = bytearray(d)
            op = r.randrange(3)
            i = r.randrange(len(t) + (op == 0))
            if op == 0:
                t.insert(i, r.choice(alphabet))
            elif op == 1 and len(t) > 1:
                del t[i]
            else:
                t[i % len(t)] = r.choice(alphabet)
            t = bytes(t)
            want = v.accepts(t)
            got = g.check_text(t) == COMPLETE
            assert got == want, (t, got, want)
            n_acc += want
    assert n_acc > 0


@pytest.mark.parametrize("name", sorted(SCHEMAS))
def test_random_walks_never_dead_end(grammars, name):
    g, v = grammars[name], Validator(SCHEMAS[name])
    r = random.Random(1000 + len(name))
    closing = set(b'"}]')
    # the schema's own characters (property names, enum texts, literals, JSON punctuation): the
    # walk prefers them, so that required keys and enum values get written
    hint = set(b'{}[],:" -0123456789truefalsn')

    def collect(x):
        if isinstance(x, dict):
            for k, v in x.items():
                hint.update(k.encode())
                collect(v)
        elif isinstance(x, list):
            for v in x:
                collect(v)
        elif isinstance(x, str):
            hint.update(x.encode())

    collect(SCHEMAS[name])
    completed = 0
    for _ in range(12):
        text = b""
        while True:
            st = g.check_text(text)
            assert st != NOT_PREFIX
            if st == COMPLETE and (r.random() < 0.35 or len(text) > 120):
                assert v.accepts(text), text
                completed += 1
                break
            allowed = [b for b in range(256) if g.check_text(text + bytes([b])) != NOT_PREFIX]
            assert allowed or st == COMPLETE, ("dead end", text)
            if not allowed:
                assert v.accepts(text), text
                completed += 1
                break
            ascii_ok = [b for b in allowed if b < 0x80] or allowed
            hinted = [b for b in ascii_ok if b in hint]
            if hinted and r.random() < 0.85:
                ascii_ok = hinted
            if len(text) > 60:  # steer toward the end of the document: closings, then short values
                pref = ascii_ok
                for group in (closing, set(b":"), set(b"0123456789"), set(b"tfn"), set(b"-."),
                              set(range(0x20, 0x7F)) - set(b"{[,")):
                    cand = [b for b in ascii_ok if b in group]
                    if cand:
                        pref = cand
                        break
                b = r.choice(pref)
            else:
                b = r.choice(ascii_ok)
            text += bytes([b])
            if len(text) > 400:
                break
    WALKS_COMPLETED[name] = completed


WALKS_COMPLETED: dict[str, int] = {}


def test_random_walks_complete_documents():
    """Across the schemas, the walks end in many completed documents (each checked above)."""
    if len(WALKS_COMPLETED) < len(SCHEMAS):
        pytest.skip("the walks did not all run in this session")
    assert sum(WALKS_COMPLETED.values()) >= 40, WALKS_COMPLETED


REFUSED = [
    ({"type": "array", "uniqueItems": True}, "#: keyword 'uniqueItems' is not supported"),
    ({"type": "object", "properties": {"a": {"not": {}}}}, "#/properties/a: keyword 'not' is not supported"),
    ({"oneOf": [{"type": "string"}]}, "keyword 'oneOf' is not supported"),
    ({"type": "number", "minimum": 0}, "bounds on non-integers are not supported"),
    ({"type": "string", "format": "email"}, "format 'email' is not supported"),
    ({"type": "string", "pattern": "[a-z]+"}, "anchored"),
    ({"anyOf": [{"type": "object"}, {"type": "object", "required": []}]}, "begin with the same character"),
    ({"$ref": "#/$defs/missing"}, "does not resolve"),
    ({"type": "integer", "minimum": 5, "maximum": 4}, "admit no value"),
    ({"type": "object", "required": ["z"], "additionalProperties": False}, "is not allowed by additionalProperties"),
    ({"allOf": [{"properties": {"a": {}}, "additionalProperties": False}, {"properties": {"b": {}}}]},
     "does not declare 'b'"),
]


@pytest.mark.parametrize("schema,msg", REFUSED)
def test_unsupported_schemas_are_refused_with_the_place(schema, msg):
    with pytest.raises(SchemaError) as ei:
        SchemaGrammar(-1, schema)
    assert msg in str(ei.value), str(ei.value)
    assert str(ei.value).startswith("JSON schema: ")


def test_annotations_have_no_effect():
    a = SchemaGrammar(-1, {"type": "integer", "title": "t", "description": "d", "default": 3, "examples": [1]})
    b = SchemaGrammar(-1, {"type": "integer"})
    for t in [b"1", b"-3", b"1.5", b'"x"', b"12"]:
        assert a.check_text(t) == b.check_text(t)


def test_unions_reached_through_refs_stay_flat():
    # a $ref to an anyOf, itself an alternative of an anyOf, and a recursive array of a union: the
    # automaton walks them without nested unions (its device form is not recursive)
    schema = {"$defs": {"opt": {"anyOf": [{"type": "string", "maxLength": 3}, {"type": "null"}]},
                        "v": {"anyOf": [{"type": "integer", "minimum": 0}, {"type": "array", "items": {"$ref": "#/$defs/v"},
                                                                             "maxItems": 2}]}},
              "type": "object",
              "properties": {"a": {"anyOf": [{"$ref": "#/$defs/opt"}, {"type": "boolean"}]}, "b": {"$ref": "#/$defs/v"}},
              "additionalProperties": False}
    g = SchemaGrammar(-1, schema)
    v = Validator(schema)
    for text in [b'{"a":"xy"}', b'{"a":null}', b'{"a":true}', b'{"a":"long"}', b'{"a":3}', b'{"b":[1,[2,[]]]}',
                 b'{"b":[1,2,3]}', b'{"b":-1}', b'{"a":false,"b":7}', b'{"b":[[[[0]]]]}']:
        assert (g.check_text(text) == COMPLETE) == v.accepts(text), text
    assert g.check_text(b'{"a":n') == PREFIX and g.check_text(b'{"a":1') == NOT_PREFIX


def test_integers_near_the_64_bit_limits_end_cleanly():
    # magnitudes whose next power of ten passes 2^64: a digit is allowed only while the value can
    # still end inside the bounds, so no prefix is a dead end
    for schema in [{"type": "integer"}, {"type": "integer", "minimum": -5, "maximum": 4_000_000_000_000_000_000},
                   {"type": "array", "items": {"type": "integer"}}]:
        g = SchemaGrammar(-1, schema)
        v = Validator(schema)
        pre = b"[" if schema.get("type") == "array" else b""
        for digits in [b"409562218754484177", b"1152921504606846976", b"230584300921369395", b"9223372036854775807"]:
            for sign in [b"", b"-"]:
                text = pre + sign
                for c in digits:
                    nxt = text + bytes([c])
                    if g.check_text(nxt) == NOT_PREFIX:
                        break
                    text = nxt
                # what was accepted is no dead end: some byte follows, or the document is complete
                assert g.check_text(text) == COMPLETE or any(
                    g.check_text(text + bytes([b])) != NOT_PREFIX for b in range(256)), text
                ends = [text + b"]"] if pre else [text]
                for t in ends:
                    assert (g.check_text(t) == COMPLETE) == v.accepts(t), t
