#pragma once
// smp_schema_auto.cuh - the json_schema automaton: the compiled schema program and the byte-level
// transition function, shared by the device kernels (masks, advance) and the host check of
// smp_schema.cu.
//
// A row's state is a stack of frames. The bottom frame is the document root; every open value
// (object, array, string, number, literal, object key) has a frame on top of its container's.
// step() applies one byte: it either moves the top frame, opens a value (push), completes one
// (pop, and the container moves on), or refuses the byte. Every transition it accepts keeps the
// text a prefix of some matching document (the compiler trims patterns to live states, integer
// digits are checked against their bounds, and containers admit a ',' or a close only when the
// rest of the value can still be completed), so a mask built from step() never leads the model
// into a dead end. Numbers and literals end at the first byte that cannot extend them: that byte
// completes the value and is applied again to the container.
#include <stdint.h>

namespace sixi_b200 {
namespace schema {

constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr int kMaxDepth = 32;  // SIXI_SCHEMA_MAX_DEPTH

// node kinds
enum : uint8_t { N_ANY = 0, N_OBJECT, N_ARRAY, N_STRING, N_INTEGER, N_NUMBER, N_ENUM, N_UNION };

struct Node {           // 48 bytes
    uint8_t kind;
    uint8_t flags;      // unused for now
    uint16_t n;         // properties / prefix items / literals / alternatives
    uint32_t first;     // first index into props / ids / lits / ids
    uint32_t extra;     // OBJECT: additional-properties node; ARRAY: items node; STRING: dfa (kNone: none)
    uint32_t pad;
    uint64_t required;  // OBJECT: required property bits
    int64_t lo, hi;     // INTEGER: bounds; ARRAY: items; STRING: length (code points)
};
static_assert(sizeof(Node) == 40 || sizeof(Node) == 48, "node layout");

struct Prop {  // a declared property: its key text as written in JSON (escaped, no quotes)
    uint32_t name_off, name_len, node, pad;
};
struct Lit {  // an enum / const value in compact JSON
    uint32_t off, len;
};
struct Dfa {  // a pattern or format: next[state * 128 + ascii] (-1: dead), accept and distance tables
    uint32_t next_off, info_off, n_states, start;
};
struct DfaInfo {       // per state
    uint16_t accept;   // 1 when the state accepts
    uint16_t min_left; // fewest characters to an accepting state
    uint16_t max_left; // most characters to an accepting state (0xFFFF: unbounded)
    uint16_t pad;
};

struct Prog {  // device or host pointers
    const Node* nodes;
    const Prop* props;
    const uint32_t* ids;    // prefix items and union alternatives
    const Lit* lits;
    const uint8_t* bytes;   // property names and literal texts
    const Dfa* dfas;
    const int16_t* next;
    const DfaInfo* info;
    uint32_t root;
    uint32_t any_object, any_array, any_string, any_number, any_literal;  // nodes of generic values
    uint32_t n_nodes, n_dfas;  // table sizes the row-state check tests frames against
    const uint8_t* base;       // device: the one allocation holding every table (nullptr on the host)
    uint32_t base_bytes;       // its size
};

// The same program with every table pointer moved from `P.base` to `to` (a copy of the
// allocation, e.g. in shared memory).
__host__ __device__ inline Prog rebase(const Prog& P, const uint8_t* to) {
    Prog Q = P;
    auto mv = [&](const void* p) { return to + (static_cast<const uint8_t*>(p) - P.base); };
    Q.nodes = reinterpret_cast<const Node*>(mv(P.nodes));
    Q.props = reinterpret_cast<const Prop*>(mv(P.props));
    Q.ids = reinterpret_cast<const uint32_t*>(mv(P.ids));
    Q.lits = reinterpret_cast<const Lit*>(mv(P.lits));
    Q.bytes = mv(P.bytes);
    Q.dfas = reinterpret_cast<const Dfa*>(mv(P.dfas));
    Q.next = reinterpret_cast<const int16_t*>(mv(P.next));
    Q.info = reinterpret_cast<const DfaInfo*>(mv(P.info));
    Q.base = to;
    return Q;
}

// frame kinds
enum : uint8_t { F_ROOT = 0, F_OBJ, F_KEY, F_ARR, F_STR, F_NUM, F_LIT };
// ROOT phases
enum : uint8_t { R_START = 0, R_DONE };
// OBJ phases
enum : uint8_t { O_FIRST = 0, O_KEY, O_COLON, O_VALUE, O_AFTER };
// ARR phases
enum : uint8_t { A_FIRST = 0, A_VALUE, A_AFTER };
// NUM phases
enum : uint8_t { U_NEG = 0, U_ZERO, U_INT, U_DOT, U_FRAC, U_EXP, U_ESIGN, U_EDIG };

struct Frame {      // 24 bytes
    uint32_t node;
    uint8_t kind;
    uint8_t phase;
    uint16_t pos;   // KEY / LIT: byte position; STR: escape state (0 none, 1 after '\', 2-5 hex left+1)
    uint32_t a;     // OBJ: selected property (0xFF: an additional one); ARR: items so far; STR: code
                    // points; KEY: generic string escape state; NUM: 1 when negative
    uint32_t b;     // STR / KEY: UTF-8 continuation bytes due (bits 0-1) and range (bits 2-4); STR: DFA
                    // state (bits 8-23, 0xFFFF: none); KEY: 1 << 31 while the text can still be an
                    // undeclared key (one is allowed and no escape was typed)
    uint64_t m;     // OBJ: properties seen; KEY / LIT: candidates; NUM: magnitude (saturating)
};
static_assert(sizeof(Frame) == 24, "frame layout");

struct State {                  // the row state of sixi_schema_state (800 bytes)
    uint32_t depth;             // frames in use
    uint32_t failed;
    uint32_t pad[6];
    Frame f[kMaxDepth];
};
static_assert(sizeof(State) == 800, "state size: SIXI_SCHEMA_STATE_BYTES");

__host__ __device__ inline bool is_ws(uint32_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
__host__ __device__ inline bool is_digit(uint32_t c) { return c >= '0' && c <= '9'; }
__host__ __device__ inline bool is_hex(uint32_t c) {
    return is_digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F');
}

// A JSON string's byte-level grammar (RFC 8259 with RFC 3629 UTF-8, no raw control characters).
// esc: 0 none, 1 after '\', 2..5: hex digits left + 1. utf: bits 0-1 continuation bytes due, bits
// 2-4 the allowed range of the next one (0 80-BF, 1 A0-BF, 2 80-9F, 3 90-BF, 4 80-8F).
// Returns 0 refused, 1 accepted inside the string, 2 the closing quote, and sets *starts when the
// byte begins a code point (a character, an escape, a lead byte).
__host__ __device__ inline int str_byte(uint32_t c, uint32_t& esc, uint32_t& utf, bool& starts) {
    starts = false;
    if ((utf & 3u) != 0u) {
        const uint32_t r = (utf >> 2) & 7u;
        const uint32_t lo = r == 1 ? 0xA0u : (r == 3 ? 0x90u : 0x80u);
        const uint32_t hi = r == 2 ? 0x9Fu : (r == 4 ? 0x8Fu : 0xBFu);
        if (c < lo || c > hi) return 0;
        utf = (utf & 3u) - 1u;  // the following continuation bytes (if any) range over 80-BF
        return 1;
    }
    if (esc == 1u) {
        if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
            esc = 0u;
            return 1;
        }
        if (c == 'u') {
            esc = 5u;
            return 1;
        }
        return 0;
    }
    if (esc >= 2u) {
        if (!is_hex(c)) return 0;
        esc = esc == 2u ? 0u : esc - 1u;
        return 1;
    }
    if (c == '"') return 2;
    if (c == '\\') {
        esc = 1u;
        starts = true;
        return 1;
    }
    if (c < 0x20u) return 0;
    starts = true;
    if (c < 0x80u) return 1;
    if (c >= 0xC2u && c <= 0xDFu) {
        utf = 1u;
        return 1;
    }
    if (c == 0xE0u) { utf = 2u | (1u << 2); return 1; }
    if ((c >= 0xE1u && c <= 0xECu) || c == 0xEEu || c == 0xEFu) { utf = 2u; return 1; }
    if (c == 0xEDu) { utf = 2u | (2u << 2); return 1; }
    if (c == 0xF0u) { utf = 3u | (3u << 2); return 1; }
    if (c >= 0xF1u && c <= 0xF3u) { utf = 3u; return 1; }
    if (c == 0xF4u) { utf = 3u | (4u << 2); return 1; }
    return 0;
}

// Whether an integer being written (sign, magnitude so far, more digits possible) can still end
// inside [lo, hi].
__host__ __device__ inline bool int_viable(bool neg, uint64_t mag, bool more, int64_t lo, int64_t hi) {
    // the values reachable: mag * 10^k .. (mag + 1) * 10^k - 1 for k = 0, 1, ... (k = 0 only when
    // no more digits may follow), mirrored for negative numbers; magnitudes past 2^62 are treated
    // as out of every range
    const uint64_t cap = 1ull << 62;
    uint64_t a = mag, b = mag;
    for (int k = 0; k < 20; ++k) {
        if (a > cap) return false;
        const uint64_t bb = b > cap ? cap : b;
        int64_t vlo, vhi;
        if (neg) {
            vlo = -static_cast<int64_t>(bb);
            vhi = -static_cast<int64_t>(a);
        } else {
            vlo = static_cast<int64_t>(a);
            vhi = static_cast<int64_t>(bb);
        }
        if (vhi >= lo && vlo <= hi) return true;
        if (!more || mag == 0) return false;
        if (a > cap / 10u) return false;  // one more digit passes every range (and must not wrap)
        a = a * 10u;
        b = b > cap / 10u ? cap + 1u : b * 10u + 9u;
    }
    return false;
}

// Whether a '-' may begin an integer of [lo, hi]: some negative value, or -0 (= 0), lies in it.
__host__ __device__ inline bool neg_viable(int64_t lo, int64_t hi) {
    return (lo <= -1 && lo <= hi) || (lo <= 0 && hi >= 0);
}

// One byte through the automaton. S: the frame stack (depth(), top(), at(i) read-only, push(),
// pop(), and mut() for a writable top). Returns false when the byte is refused (S is then
// unspecified: callers work on copies).
template <class S>
struct Machine {
    const Prog& P;
    S& st;
    __host__ __device__ Machine(const Prog& p, S& s) : P(p), st(s) {}

    // the generic node a value of any type that begins with c takes (for N_ANY), else nd
    __host__ __device__ uint32_t concrete(uint32_t nd, uint32_t c) const {
        if (P.nodes[nd].kind != N_ANY) return nd;
        if (c == '{') return P.any_object;
        if (c == '[') return P.any_array;
        if (c == '"') return P.any_string;
        if (c == '-' || is_digit(c)) return P.any_number;
        return P.any_literal;
    }

    // A value of node `nd` begins with byte c (not whitespace); the parent has already moved on
    // to its after-value phase. Pushes the value's frame. Not recursive (device stacks are sized
    // statically): a union's alternatives are never unions themselves (the compiler flattens
    // them and checks it), and an N_ANY resolves to one generic node in one step.
    __host__ __device__ bool begin_value(uint32_t nd, uint32_t c) {
        const Node& U = P.nodes[nd];
        if (U.kind == N_UNION) {
            for (uint32_t i = 0; i < U.n; ++i)  // alternatives begin with different characters
                if (begin_one(concrete(P.ids[U.first + i], c), c)) return true;
            return false;
        }
        return begin_one(concrete(nd, c), c);
    }

    // begin_value for a node that is neither a union nor N_ANY
    __host__ __device__ bool begin_one(uint32_t nd, uint32_t c) {
        const Node& N = P.nodes[nd];
        Frame f{};
        f.node = nd;
        switch (N.kind) {
            case N_OBJECT:
                if (c != '{') return false;
                f.kind = F_OBJ;
                f.phase = O_FIRST;
                f.a = 0xFFu;
                return st.push(f);
            case N_ARRAY:
                if (c != '[') return false;
                f.kind = F_ARR;
                f.phase = A_FIRST;
                return st.push(f);
            case N_STRING:
                if (c != '"') return false;
                f.kind = F_STR;
                f.b = (N.extra != kNone ? P.dfas[N.extra].start : 0xFFFFu) << 8;
                return st.push(f);
            case N_INTEGER:
            case N_NUMBER: {
                f.kind = F_NUM;
                if (c == '-') {
                    if (N.kind == N_INTEGER && !neg_viable(N.lo, N.hi)) return false;
                    f.phase = U_NEG;
                    f.a = 1u;
                } else if (c == '0') {
                    if (N.kind == N_INTEGER && !int_viable(false, 0, false, N.lo, N.hi)) return false;
                    f.phase = U_ZERO;
                } else if (is_digit(c)) {
                    if (N.kind == N_INTEGER && !int_viable(false, c - '0', true, N.lo, N.hi)) return false;
                    f.phase = U_INT;
                    f.m = c - '0';
                } else {
                    return false;
                }
                return st.push(f);
            }
            case N_ENUM: {
                uint64_t cand = 0;
                for (uint32_t i = 0; i < N.n; ++i) {
                    const Lit& L = P.lits[N.first + i];
                    if (L.len > 0 && P.bytes[L.off] == c) cand |= 1ull << i;
                }
                if (cand == 0) return false;
                f.kind = F_LIT;
                f.pos = 1;
                f.m = cand;
                return st.push(f);
            }
            default:
                return false;
        }
    }

    // whether the top NUM / LIT frame is a complete value
    __host__ __device__ bool scalar_complete(const Frame& f) const {
        const Node& N = P.nodes[f.node];
        if (f.kind == F_NUM) {
            if (!(f.phase == U_ZERO || f.phase == U_INT || f.phase == U_FRAC || f.phase == U_EDIG)) return false;
            if (N.kind == N_INTEGER) {
                const int64_t v = f.a ? -static_cast<int64_t>(f.m) : static_cast<int64_t>(f.m);
                return v >= N.lo && v <= N.hi;
            }
            return true;
        }
        for (uint32_t i = 0; i < N.n; ++i)  // F_LIT: a candidate matched to its end
            if (((f.m >> i) & 1ull) && P.lits[N.first + i].len == f.pos) return true;
        return false;
    }

    // the top value is complete: pop it and move its container on
    __host__ __device__ bool value_done() {
        st.pop();
        Frame& p = st.mut();
        if (p.kind == F_ROOT) {
            p.phase = R_DONE;
        } else if (p.kind == F_OBJ) {
            if (p.a != 0xFFu) p.m |= 1ull << p.a;
            p.phase = O_AFTER;
        } else if (p.kind == F_ARR) {
            p.a += 1u;
            p.phase = A_AFTER;
        } else {
            return false;
        }
        return true;
    }

    // the item schema of array position i (kNone: no item may stand there)
    __host__ __device__ uint32_t item_node(const Node& N, uint32_t i) const {
        return i < N.n ? P.ids[N.first + i] : N.extra;
    }

    // properties an object may still take: unseen declared ones, or any when additional ones are allowed
    __host__ __device__ bool more_keys(const Node& N, uint64_t seen) const {
        if (N.extra != kNone) return true;
        const uint64_t all = N.n >= 64 ? ~0ull : ((1ull << N.n) - 1ull);
        return (all & ~seen) != 0ull;
    }

    __host__ __device__ bool step(uint32_t c) {
        for (int guard = 0; guard < 4; ++guard) {  // a completed scalar hands its terminator back once
            if (st.depth() == 0) return false;
            const Frame t = st.top();
            const Node& N = P.nodes[t.node];
            switch (t.kind) {
                case F_ROOT:
                    if (t.phase == R_DONE) return false;  // only the end-of-sequence token follows
                    if (is_ws(c)) return true;
                    return begin_value(t.node, c);
                case F_OBJ: {
                    Frame& f = st.mut();
                    if (is_ws(c)) return true;
                    if (t.phase == O_FIRST || t.phase == O_KEY) {
                        if (c == '}' && t.phase == O_FIRST) {
                            if ((N.required & ~t.m) != 0ull) return false;
                            return value_done();
                        }
                        if (c != '"' || !more_keys(N, t.m)) return false;
                        f.phase = O_COLON;  // after the key
                        Frame k{};
                        k.node = t.node;
                        k.kind = F_KEY;
                        k.pos = 0;
                        k.m = N.n >= 64 ? ~0ull : ((1ull << N.n) - 1ull);
                        k.b = N.extra != kNone ? (1u << 31) : 0u;
                        return st.push(k);
                    }
                    if (t.phase == O_COLON) {
                        if (c != ':') return false;
                        f.phase = O_VALUE;
                        return true;
                    }
                    if (t.phase == O_VALUE) {
                        const uint32_t vn = t.a == 0xFFu ? N.extra : P.props[N.first + t.a].node;
                        f.phase = O_AFTER;  // value_done of the child sets it again
                        return begin_value(vn, c);
                    }
                    // O_AFTER
                    if (c == ',') {
                        if (!more_keys(N, t.m)) return false;
                        f.phase = O_KEY;
                        f.a = 0xFFu;
                        return true;
                    }
                    if (c == '}') {
                        if ((N.required & ~t.m) != 0ull) return false;
                        return value_done();
                    }
                    return false;
                }
                case F_KEY: {
                    Frame& k = st.mut();
                    const bool generic = (t.b >> 31) != 0u;
                    uint32_t esc = t.a, utf = t.b & 0x1Fu;
                    bool starts = false;
                    const int g = str_byte(c, esc, utf, starts);  // a key is a JSON string
                    if (g == 0) return false;
                    if (g == 2) {
                        // the closing quote: a declared name typed exactly, else an additional key
                        uint32_t sel = 0xFFu;
                        for (uint32_t i = 0; i < N.n && i < 64; ++i)
                            if (((t.m >> i) & 1ull) && P.props[N.first + i].name_len == t.pos) sel = i;
                        const Frame& o = st.at(st.depth() - 2);
                        if (sel != 0xFFu) {
                            if ((o.m >> sel) & 1ull) return false;  // a key may not repeat
                        } else if (!generic) {
                            return false;
                        }
                        st.pop();
                        st.mut().a = sel;  // the object frame, now in O_COLON
                        return true;
                    }
                    // a key byte: it extends declared names, or (any key allowed) a generic string
                    uint64_t cand = 0;
                    if (t.pos < 0xFFFFu)
                        for (uint32_t i = 0; i < N.n && i < 64; ++i) {
                            if (!((t.m >> i) & 1ull)) continue;
                            const Prop& pr = P.props[N.first + i];
                            if (t.pos < pr.name_len && P.bytes[pr.name_off + t.pos] == c) cand |= 1ull << i;
                        }
                    // an undeclared key is written without escapes (so it cannot spell a declared
                    // name in another way): the first backslash ends that possibility
                    const bool gen_ok = generic && c != '\\' && esc == 0u;
                    if (cand == 0ull && !gen_ok) return false;
                    if (!gen_ok) {  // only declared names: one not yet seen must stay reachable
                        const Frame& o = st.at(st.depth() - 2);
                        if ((cand & ~o.m) == 0ull) return false;
                    }
                    k.m = cand;
                    k.pos = static_cast<uint16_t>(t.pos < 0xFFFFu ? t.pos + 1u : 0xFFFFu);
                    k.a = esc;
                    k.b = (gen_ok ? 0x80000000u : 0u) | (utf & 0x1Fu);
                    return true;
                }
                case F_ARR: {
                    Frame& f = st.mut();
                    if (is_ws(c)) return true;
                    if (t.phase == A_FIRST || t.phase == A_AFTER) {
                        if (c == ']') {
                            if (static_cast<int64_t>(t.a) < N.lo) return false;
                            return value_done();
                        }
                        if (t.phase == A_AFTER) {
                            if (c != ',') return false;
                            if (static_cast<int64_t>(t.a) >= N.hi || item_node(N, t.a) == kNone) return false;
                            f.phase = A_VALUE;
                            return true;
                        }
                        // A_FIRST: the first item
                    }
                    if (static_cast<int64_t>(t.a) >= N.hi) return false;
                    const uint32_t in = item_node(N, t.a);
                    if (in == kNone) return false;
                    f.phase = A_AFTER;
                    return begin_value(in, c);
                }
                case F_STR: {
                    Frame& f = st.mut();
                    const uint32_t dfa = N.extra;
                    uint32_t esc = t.pos, utf = t.b & 0x1Fu;
                    const uint32_t ds = (t.b >> 8) & 0xFFFFu;
                    if (dfa != kNone) {
                        // a pattern: printable ASCII only, no escapes, each character through the DFA
                        const Dfa& D = P.dfas[dfa];
                        if (c == '"') {
                            if (!P.info[D.info_off + ds].accept) return false;
                            if (static_cast<int64_t>(t.a) < N.lo || static_cast<int64_t>(t.a) > N.hi) return false;
                            return value_done();
                        }
                        if (c < 0x20u || c >= 0x7Fu || c == '\\') return false;
                        const int nx = P.next[D.next_off + ds * 128u + c];
                        if (nx < 0) return false;
                        const DfaInfo& I = P.info[D.info_off + static_cast<uint32_t>(nx)];
                        const int64_t cnt = static_cast<int64_t>(t.a) + 1;
                        if (cnt + I.min_left > N.hi) return false;
                        if (I.max_left != 0xFFFFu && cnt + I.max_left < N.lo) return false;
                        f.a = static_cast<uint32_t>(cnt);
                        f.b = (static_cast<uint32_t>(nx) << 8);
                        return true;
                    }
                    bool starts = false;
                    const int g = str_byte(c, esc, utf, starts);
                    if (g == 0) return false;
                    if (g == 2) {
                        if (static_cast<int64_t>(t.a) < N.lo) return false;
                        return value_done();
                    }
                    uint32_t cnt = t.a;
                    if (starts) {
                        if (static_cast<int64_t>(cnt) >= N.hi) return false;
                        ++cnt;
                    }
                    f.pos = static_cast<uint16_t>(esc);
                    f.a = cnt;
                    f.b = (t.b & ~0x1Fu) | (utf & 0x1Fu);
                    return true;
                }
                case F_NUM: {
                    Frame& f = st.mut();
                    const bool integer = N.kind == N_INTEGER;
                    const bool neg = t.a != 0u;
                    switch (t.phase) {
                        case U_NEG:
                            if (c == '0') {
                                if (integer && !int_viable(true, 0, false, N.lo, N.hi)) break;
                                f.phase = U_ZERO;
                                return true;
                            }
                            if (is_digit(c)) {
                                if (integer && !int_viable(true, c - '0', true, N.lo, N.hi)) break;
                                f.phase = U_INT;
                                f.m = c - '0';
                                return true;
                            }
                            return false;
                        case U_ZERO:
                        case U_INT:
                            if (t.phase == U_INT && is_digit(c)) {
                                const uint64_t nm = t.m > (1ull << 60) ? (1ull << 62) : t.m * 10u + (c - '0');
                                if (integer && !int_viable(neg, nm, true, N.lo, N.hi)) return false;
                                f.m = nm;
                                return true;
                            }
                            if (!integer && c == '.') {
                                f.phase = U_DOT;
                                return true;
                            }
                            if (!integer && (c == 'e' || c == 'E')) {
                                f.phase = U_EXP;
                                return true;
                            }
                            break;  // a terminator
                        case U_DOT:
                            if (!is_digit(c)) return false;
                            f.phase = U_FRAC;
                            return true;
                        case U_FRAC:
                            if (is_digit(c)) return true;
                            if (c == 'e' || c == 'E') {
                                f.phase = U_EXP;
                                return true;
                            }
                            break;
                        case U_EXP:
                            if (c == '+' || c == '-') {
                                f.phase = U_ESIGN;
                                return true;
                            }
                            if (!is_digit(c)) return false;
                            f.phase = U_EDIG;
                            return true;
                        case U_ESIGN:
                            if (!is_digit(c)) return false;
                            f.phase = U_EDIG;
                            return true;
                        case U_EDIG:
                            if (is_digit(c)) return true;
                            break;
                        default:
                            return false;
                    }
                    // c cannot extend the number: it must end it, then the container takes c
                    if (!scalar_complete(t)) return false;
                    if (!value_done()) return false;
                    continue;
                }
                case F_LIT: {
                    uint64_t cand = 0;
                    for (uint32_t i = 0; i < N.n && i < 64; ++i) {
                        if (!((t.m >> i) & 1ull)) continue;
                        const Lit& L = P.lits[N.first + i];
                        if (t.pos < L.len && P.bytes[L.off + t.pos] == c) cand |= 1ull << i;
                    }
                    if (cand != 0ull) {
                        Frame& f = st.mut();
                        f.m = cand;
                        f.pos = static_cast<uint16_t>(t.pos + 1u);
                        return true;
                    }
                    if (!scalar_complete(t)) return false;
                    if (!value_done()) return false;
                    continue;
                }
                default:
                    return false;
            }
            return false;
        }
        return false;
    }

    // whether the text so far is a complete document (the end-of-sequence token may follow): the
    // root is done, or a complete number / literal is the root's value
    __host__ __device__ bool complete() const {
        const uint32_t d = st.depth();
        if (d == 0) return false;
        const Frame& t = st.top();
        if (t.kind == F_ROOT) return t.phase == R_DONE;
        if (d == 2 && (t.kind == F_NUM || t.kind == F_LIT)) return scalar_complete(t);
        return false;
    }
};

// The full stack of a State (host checks and the advance kernels).
struct FullStack {
    State& s;
    __host__ __device__ explicit FullStack(State& st) : s(st) {}
    __host__ __device__ uint32_t depth() const { return s.depth; }
    __host__ __device__ const Frame& top() const { return s.f[s.depth - 1]; }
    __host__ __device__ const Frame& at(uint32_t i) const { return s.f[i]; }
    __host__ __device__ Frame& mut() { return s.f[s.depth - 1]; }
    __host__ __device__ bool push(const Frame& f) {
        if (s.depth >= static_cast<uint32_t>(kMaxDepth)) return false;
        s.f[s.depth++] = f;
        return true;
    }
    __host__ __device__ void pop() { --s.depth; }
};

// The row's stack read-only, with the frames a token changes or pushes kept in a small overlay
// (the mask walks: one per token and row, most touching only the top frame or two).
template <int OV>
struct OverlayStack {
    const State& base;
    uint32_t base_n;  // base frames still below the overlay
    uint32_t ov_n;
    Frame ov[OV];
    __host__ __device__ explicit OverlayStack(const State& b) : base(b), base_n(b.depth), ov_n(0) {}
    __host__ __device__ uint32_t depth() const { return base_n + ov_n; }
    __host__ __device__ const Frame& top() const { return ov_n ? ov[ov_n - 1] : base.f[base_n - 1]; }
    __host__ __device__ const Frame& at(uint32_t i) const { return i < base_n ? base.f[i] : ov[i - base_n]; }
    __host__ __device__ Frame& mut() {
        if (ov_n == 0) {  // copy the base's top into the overlay (it is changed there)
            ov[0] = base.f[base_n - 1];
            --base_n;
            ov_n = 1;
        }
        return ov[ov_n - 1];
    }
    __host__ __device__ bool push(const Frame& f) {
        if (ov_n >= static_cast<uint32_t>(OV) || depth() >= static_cast<uint32_t>(kMaxDepth)) return false;
        ov[ov_n++] = f;
        return true;
    }
    __host__ __device__ void pop() {
        if (ov_n) --ov_n;
        else --base_n;
    }
};

// Whether a row state can be walked safely: its depth and every frame's node and kind lie in
// range, and string frames under a pattern hold a state of their DFA. States made by
// sixi_schema_reset / sixi_schema_advance always pass; the kernels treat any other as dead.
__host__ __device__ inline bool state_ok(const Prog& P, const State& s) {
    if (s.depth == 0u) return true;  // finished (or never started): nothing may follow
    if (s.depth > static_cast<uint32_t>(kMaxDepth)) return false;
    for (uint32_t i = 0; i < s.depth; ++i) {
        const Frame& f = s.f[i];
        if (f.node >= P.n_nodes || f.kind > F_LIT || (i == 0) != (f.kind == F_ROOT)) return false;
        const Node& N = P.nodes[f.node];
        if (f.kind == F_STR && N.kind == N_STRING && N.extra != kNone) {
            if (N.extra >= P.n_dfas || ((f.b >> 8) & 0xFFFFu) >= P.dfas[N.extra].n_states) return false;
        }
        if ((f.kind == F_OBJ || f.kind == F_KEY) && N.kind != N_OBJECT) return false;
        if (f.kind == F_KEY && (s.f[i - 1].kind != F_OBJ || s.f[i - 1].node != f.node)) return false;
        if (f.kind == F_OBJ && f.a != 0xFFu && f.a >= N.n) return false;
        if (f.kind == F_ARR && N.kind != N_ARRAY) return false;
        if (f.kind == F_LIT && N.kind != N_ENUM) return false;
        if (f.kind == F_NUM && N.kind != N_INTEGER && N.kind != N_NUMBER) return false;
        if (f.kind == F_STR && N.kind != N_STRING) return false;
    }
    return true;
}

__host__ __device__ inline void start_state(State& s, uint32_t root) {
    s.depth = 1;
    s.failed = 0;
    for (int i = 0; i < 6; ++i) s.pad[i] = 0;
    Frame r{};
    r.node = root;
    r.kind = F_ROOT;
    r.phase = R_START;
    s.f[0] = r;
}

}  // namespace schema
}  // namespace sixi_b200
