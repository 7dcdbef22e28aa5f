// smp_schema.cu - `response_format: json_schema`: the schema compiler (host), the automaton's
// kernels (masks, advance, reset) and the C ABI of include/sixi_schema.h.
//
// The compiler turns the schema's JSON text into a program of nodes (smp_schema_auto.cuh): objects
// with their declared properties (key texts, value nodes, the required set and the node of
// additional properties), arrays (prefix items, the item node, the count bounds), strings (length
// bounds and an optional DFA for a pattern or format), integers with bounds, numbers, enum / const
// literals in compact JSON (booleans and null are such literals), unions (anyOf, type lists) and
// "any value". $ref targets are compiled once and may be recursive. allOf is merged into one
// schema before compiling. Patterns become DFAs over printable ASCII by subset construction from
// a Thompson NFA, trimmed to the states from which an accepting state is reachable.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <utility>
#include <vector>

#include "../../include/sixi_schema.h"
#include "smp_schema_auto.cuh"

namespace sixi_b200 {
namespace schema {
namespace {

// ------------------------------------------------------------------------------------ JSON text
struct JV {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    bool b = false;
    std::string s;  // STR: the decoded string (UTF-8); NUM: the number as written
    std::vector<JV> a;
    std::vector<std::pair<std::string, JV>> o;
    const JV* get(const std::string& k) const {
        for (const auto& kv : o)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct Parser {
    const char* p;
    const char* e;
    std::string err;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = std::string("JSON schema: not valid JSON (") + m + ")";
        return false;
    }
    static void put_utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(uint32_t& v) {
        v = 0;
        for (int i = 0; i < 4; ++i) {
            if (p >= e) return false;
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else return false;
        }
        return true;
    }
    bool str(std::string& out) {
        if (p >= e || *p != '"') return fail("string expected");
        ++p;
        while (p < e && *p != '"') {
            const unsigned char c = static_cast<unsigned char>(*p++);
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') {
                out += static_cast<char>(c);
                continue;
            }
            if (p >= e) return fail("unterminated escape");
            const char x = *p++;
            switch (x) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t v;
                    if (!hex4(v)) return fail("bad \\u escape");
                    if (v >= 0xD800 && v < 0xDC00 && p + 6 <= e && p[0] == '\\' && p[1] == 'u') {
                        p += 2;
                        uint32_t w;
                        if (!hex4(w) || w < 0xDC00 || w > 0xDFFF) return fail("bad surrogate pair");
                        v = 0x10000 + ((v - 0xD800) << 10) + (w - 0xDC00);
                    }
                    put_utf8(out, v);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JV& v, int depth) {
        if (depth > 200) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("unexpected end");
        const char c = *p;
        if (c == '{') {
            ++p;
            v.t = JV::OBJ;
            ws();
            if (p < e && *p == '}') {
                ++p;
                return true;
            }
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= e || *p != ':') return fail("':' expected");
                ++p;
                JV x;
                if (!value(x, depth + 1)) return false;
                v.o.emplace_back(std::move(k), std::move(x));
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == '}') { ++p; return true; }
                return fail("',' or '}' expected");
            }
        }
        if (c == '[') {
            ++p;
            v.t = JV::ARR;
            ws();
            if (p < e && *p == ']') {
                ++p;
                return true;
            }
            for (;;) {
                JV x;
                if (!value(x, depth + 1)) return false;
                v.a.push_back(std::move(x));
                ws();
                if (p < e && *p == ',') { ++p; continue; }
                if (p < e && *p == ']') { ++p; return true; }
                return fail("',' or ']' expected");
            }
        }
        if (c == '"') {
            v.t = JV::STR;
            return str(v.s);
        }
        auto lit = [&](const char* w, JV::Type t, bool b) {
            const size_t n = std::strlen(w);
            if (static_cast<size_t>(e - p) < n || std::strncmp(p, w, n) != 0) return fail("unknown literal");
            p += n;
            v.t = t;
            v.b = b;
            return true;
        };
        if (c == 't') return lit("true", JV::BOOL, true);
        if (c == 'f') return lit("false", JV::BOOL, false);
        if (c == 'n') return lit("null", JV::NUL, false);
        const char* s0 = p;  // number
        if (p < e && *p == '-') ++p;
        if (p < e && *p == '0') {
            ++p;
        } else if (p < e && *p >= '1' && *p <= '9') {
            while (p < e && *p >= '0' && *p <= '9') ++p;
        } else {
            return fail("value expected");
        }
        if (p < e && *p == '.') {
            ++p;
            if (p >= e || *p < '0' || *p > '9') return fail("digits expected after '.'");
            while (p < e && *p >= '0' && *p <= '9') ++p;
        }
        if (p < e && (*p == 'e' || *p == 'E')) {
            ++p;
            if (p < e && (*p == '+' || *p == '-')) ++p;
            if (p >= e || *p < '0' || *p > '9') return fail("exponent digits expected");
            while (p < e && *p >= '0' && *p <= '9') ++p;
        }
        v.t = JV::NUM;
        v.s.assign(s0, p);
        return true;
    }
};

void escape_into(std::string& out, const std::string& s) {  // JSON string content, minimal escapes
    static const char* hx = "0123456789abcdef";
    for (unsigned char c : s) {
        if (c == '"') out += "\\\"";
        else if (c == '\\') out += "\\\\";
        else if (c == '\n') out += "\\n";
        else if (c == '\r') out += "\\r";
        else if (c == '\t') out += "\\t";
        else if (c == '\b') out += "\\b";
        else if (c == '\f') out += "\\f";
        else if (c < 0x20) {
            out += "\\u00";
            out += hx[c >> 4];
            out += hx[c & 15];
        } else {
            out += static_cast<char>(c);
        }
    }
}

void compact(std::string& out, const JV& v) {
    switch (v.t) {
        case JV::NUL: out += "null"; break;
        case JV::BOOL: out += v.b ? "true" : "false"; break;
        case JV::NUM: out += v.s; break;
        case JV::STR:
            out += '"';
            escape_into(out, v.s);
            out += '"';
            break;
        case JV::ARR:
            out += '[';
            for (size_t i = 0; i < v.a.size(); ++i) {
                if (i) out += ',';
                compact(out, v.a[i]);
            }
            out += ']';
            break;
        case JV::OBJ:
            out += '{';
            for (size_t i = 0; i < v.o.size(); ++i) {
                if (i) out += ',';
                out += '"';
                escape_into(out, v.o[i].first);
                out += "\":";
                compact(out, v.o[i].second);
            }
            out += '}';
            break;
    }
}

bool num_is_integer(const std::string& s) {  // an integer value (1, -3, 2.0, 1e2)
    const double d = std::strtod(s.c_str(), nullptr);
    return std::isfinite(d) && std::floor(d) == d;
}

// ------------------------------------------------------------------------------------ patterns
// AST of a restricted regular expression over printable ASCII (0x20-0x7E without '"' and '\\',
// the characters a pattern-constrained string may hold unescaped).
struct RNode {
    enum K { SET, CAT, ALT, REP, EMPTY } k = EMPTY;
    std::vector<int> kids;
    uint64_t set[2] = {0, 0};  // SET: 128-bit character set
    int lo = 0, hi = 0;        // REP: bounds (hi = -1: unbounded)
};

struct Regex {
    std::vector<RNode> n;
    const char* p;
    const char* e;
    std::string err;

    int add(RNode x) {
        n.push_back(std::move(x));
        return static_cast<int>(n.size()) - 1;
    }
    static void set_add(RNode& r, int c) {
        if (c >= 0x20 && c < 0x7F && c != '"' && c != '\\') r.set[c >> 6] |= 1ull << (c & 63);
    }
    static void set_range(RNode& r, int a, int b) {
        for (int c = a; c <= b; ++c) set_add(r, c);
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool esc_class(RNode& r, char c) {  // \d \w \s \D ... and escaped literals
        switch (c) {
            case 'd': set_range(r, '0', '9'); return true;
            case 'w':
                set_range(r, '0', '9');
                set_range(r, 'a', 'z');
                set_range(r, 'A', 'Z');
                set_add(r, '_');
                return true;
            case 's': set_add(r, ' '); return true;  // the only whitespace a pattern string holds unescaped
            case 'D': case 'W': case 'S': {
                RNode t;
                esc_class(t, static_cast<char>(c - 'A' + 'a'));
                for (int x = 0x20; x < 0x7F; ++x)
                    if (!((t.set[x >> 6] >> (x & 63)) & 1ull)) set_add(r, x);
                return true;
            }
            default:
                if (std::strchr(".^$|?*+()[]{}/-\\\"", c) != nullptr || c == ' ') {
                    set_add(r, c);
                    return true;
                }
                return fail("unsupported escape in pattern");
        }
    }
    int atom() {
        if (p >= e) return fail("pattern ends early"), -1;
        const char c = *p++;
        RNode r;
        r.k = RNode::SET;
        if (c == '(') {
            if (p + 1 < e && p[0] == '?' && p[1] == ':') p += 2;
            const int x = alt();
            if (x < 0) return -1;
            if (p >= e || *p != ')') return fail("')' expected in pattern"), -1;
            ++p;
            return x;
        }
        if (c == '.') {
            set_range(r, 0x20, 0x7E);
            return add(r);
        }
        if (c == '\\') {
            if (p >= e) return fail("pattern ends in an escape"), -1;
            if (!esc_class(r, *p++)) return -1;
            return add(r);
        }
        if (c == '[') {
            bool neg = false;
            if (p < e && *p == '^') {
                neg = true;
                ++p;
            }
            RNode s;
            bool first = true;
            while (p < e && (*p != ']' || first)) {
                first = false;
                int a = static_cast<unsigned char>(*p++);
                if (a == '\\') {
                    if (p >= e) return fail("pattern ends in an escape"), -1;
                    const char x = *p++;
                    if (x == 'd' || x == 'w' || x == 's' || x == 'D' || x == 'W' || x == 'S') {
                        if (!esc_class(s, x)) return -1;
                        continue;
                    }
                    a = static_cast<unsigned char>(x);
                }
                if (p + 1 < e && *p == '-' && p[1] != ']') {
                    ++p;
                    int b = static_cast<unsigned char>(*p++);
                    if (b == '\\') {
                        if (p >= e) return fail("pattern ends in an escape"), -1;
                        b = static_cast<unsigned char>(*p++);
                    }
                    if (b < a) return fail("bad range in pattern"), -1;
                    set_range(s, a, b);
                } else {
                    set_add(s, a);
                }
            }
            if (p >= e) return fail("']' expected in pattern"), -1;
            ++p;
            if (neg) {
                for (int x = 0x20; x < 0x7F; ++x)
                    if (!((s.set[x >> 6] >> (x & 63)) & 1ull)) set_add(r, x);
            } else {
                r.set[0] = s.set[0];
                r.set[1] = s.set[1];
            }
            return add(r);
        }
        if (std::strchr("?*+{|)", c) != nullptr) return fail("misplaced operator in pattern"), -1;
        if (c == '^' || c == '$') return fail("'^' / '$' only at the ends of a pattern"), -1;
        set_add(r, static_cast<unsigned char>(c));
        return add(r);
    }
    int quantified() {
        int x = atom();
        if (x < 0) return -1;
        while (p < e && (*p == '*' || *p == '+' || *p == '?' || *p == '{')) {
            RNode r;
            r.k = RNode::REP;
            r.kids = {x};
            const char q = *p++;
            if (q == '*') { r.lo = 0; r.hi = -1; }
            else if (q == '+') { r.lo = 1; r.hi = -1; }
            else if (q == '?') { r.lo = 0; r.hi = 1; }
            else {
                auto num = [&](int& v) {
                    if (p >= e || *p < '0' || *p > '9') return false;
                    v = 0;
                    while (p < e && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
                    return v <= 256;
                };
                if (!num(r.lo)) return fail("bad {m,n} in pattern"), -1;
                r.hi = r.lo;
                if (p < e && *p == ',') {
                    ++p;
                    if (p < e && *p == '}') r.hi = -1;
                    else if (!num(r.hi) || r.hi < r.lo) return fail("bad {m,n} in pattern"), -1;
                }
                if (p >= e || *p != '}') return fail("bad {m,n} in pattern"), -1;
                ++p;
            }
            x = add(r);
        }
        return x;
    }
    int seq() {
        RNode r;
        r.k = RNode::CAT;
        while (p < e && *p != '|' && *p != ')') {
            const int x = quantified();
            if (x < 0) return -1;
            r.kids.push_back(x);
        }
        return add(r);
    }
    int alt() {
        RNode r;
        r.k = RNode::ALT;
        int x = seq();
        if (x < 0) return -1;
        r.kids.push_back(x);
        while (p < e && *p == '|') {
            ++p;
            x = seq();
            if (x < 0) return -1;
            r.kids.push_back(x);
        }
        return add(r);
    }
};

struct Nfa {
    struct St {
        std::vector<int> eps;
        uint64_t set[2] = {0, 0};
        int to = -1;
    };
    std::vector<St> s;
    int add() {
        s.emplace_back();
        return static_cast<int>(s.size()) - 1;
    }
    // fragment of AST node x from state `in`; returns its out state
    int emit(const Regex& R, int x, int in) {
        const RNode& r = R.n[x];
        switch (r.k) {
            case RNode::EMPTY: return in;
            case RNode::SET: {
                const int o = add();
                s[in].set[0] = r.set[0];  // a state with a character edge has no other edge
                s[in].set[1] = r.set[1];
                s[in].to = o;
                return o;
            }
            case RNode::CAT: {
                int cur = in;
                for (int k : r.kids) {
                    const int nx = add();
                    s[cur].eps.push_back(nx);
                    cur = emit(R, k, nx);
                }
                return cur;
            }
            case RNode::ALT: {
                const int o = add();
                for (int k : r.kids) {
                    const int b = add();
                    s[in].eps.push_back(b);
                    const int be = emit(R, k, b);
                    s[be].eps.push_back(o);
                }
                return o;
            }
            case RNode::REP: {
                int cur = in;
                for (int i = 0; i < r.lo; ++i) {
                    const int b = add();
                    s[cur].eps.push_back(b);
                    cur = emit(R, r.kids[0], b);
                }
                if (r.hi < 0) {  // then any number more
                    const int loop = add(), o = add();
                    s[cur].eps.push_back(loop);
                    s[loop].eps.push_back(o);
                    const int b = add();
                    s[loop].eps.push_back(b);
                    const int be = emit(R, r.kids[0], b);
                    s[be].eps.push_back(loop);
                    return o;
                }
                const int o = add();
                for (int i = r.lo; i < r.hi; ++i) {  // optional copies
                    s[cur].eps.push_back(o);
                    const int b = add();
                    s[cur].eps.push_back(b);
                    cur = emit(R, r.kids[0], b);
                }
                s[cur].eps.push_back(o);
                return o;
            }
        }
        return in;
    }
    void closure(std::set<int>& x) const {
        std::vector<int> st(x.begin(), x.end());
        while (!st.empty()) {
            const int q = st.back();
            st.pop_back();
            for (int y : s[q].eps)
                if (x.insert(y).second) st.push_back(y);
        }
    }
};

constexpr int kMaxDfaStates = 4096;

// pattern (anchored) -> DFA tables appended to next / info; returns an empty string or the error
std::string build_dfa(const std::string& pat, std::vector<int16_t>& next, std::vector<DfaInfo>& info, Dfa& out) {
    if (pat.size() < 2 || pat.front() != '^' || pat.back() != '$') return "pattern must be anchored with ^ and $";
    Regex R;
    const std::string body = pat.substr(1, pat.size() - 2);
    R.p = body.data();
    R.e = body.data() + body.size();
    const int root = R.alt();
    if (root < 0 || R.p != R.e) return R.err.empty() ? "unsupported pattern syntax" : R.err;
    Nfa N;
    const int s0 = N.add();
    const int fin = N.emit(R, root, s0);
    if (N.s.size() > 200000) return "pattern too large";
    std::map<std::set<int>, int> ids;
    std::vector<std::set<int>> sets;
    std::vector<std::vector<int>> tr;
    std::set<int> st0{s0};
    N.closure(st0);
    ids[st0] = 0;
    sets.push_back(st0);
    for (size_t i = 0; i < sets.size(); ++i) {
        tr.emplace_back(128, -1);
        for (int c = 0x20; c < 0x7F; ++c) {
            if (c == '"' || c == '\\') continue;
            std::set<int> nx;
            for (int q : sets[i])
                if (N.s[q].to >= 0 && ((N.s[q].set[c >> 6] >> (c & 63)) & 1ull)) nx.insert(N.s[q].to);
            if (nx.empty()) continue;
            N.closure(nx);
            auto it = ids.find(nx);
            int id;
            if (it == ids.end()) {
                if (static_cast<int>(sets.size()) >= kMaxDfaStates) return "pattern needs too many states";
                id = static_cast<int>(sets.size());
                ids[nx] = id;
                sets.push_back(nx);
            } else {
                id = it->second;
            }
            tr[i][c] = id;
        }
    }
    const int ns = static_cast<int>(sets.size());
    std::vector<int> acc(ns, 0);
    for (int i = 0; i < ns; ++i) acc[i] = sets[i].count(fin) ? 1 : 0;
    // live states (an accepting state is reachable) and the fewest characters to one
    std::vector<int> dist(ns, -1);
    std::vector<std::vector<int>> rev(ns);
    for (int i = 0; i < ns; ++i)
        for (int c = 0; c < 128; ++c)
            if (tr[i][c] >= 0) rev[tr[i][c]].push_back(i);
    std::vector<int> q;
    for (int i = 0; i < ns; ++i)
        if (acc[i]) {
            dist[i] = 0;
            q.push_back(i);
        }
    for (size_t h = 0; h < q.size(); ++h)
        for (int pr : rev[q[h]])
            if (dist[pr] < 0) {
                dist[pr] = dist[q[h]] + 1;
                q.push_back(pr);
            }
    if (dist[0] < 0) return "pattern matches no string";
    for (int i = 0; i < ns; ++i)
        for (int c = 0; c < 128; ++c)
            if (tr[i][c] >= 0 && dist[tr[i][c]] < 0) tr[i][c] = -1;  // no dead ends
    // the most characters to an accepting state (unbounded where a cycle of live states is reachable)
    std::vector<int> mx(ns, -2), color(ns, 0);  // -2 unknown, -1 unbounded
    std::vector<std::pair<int, int>> stk;
    for (int r0 = 0; r0 < ns; ++r0) {
        if (dist[r0] < 0 || color[r0]) continue;
        stk.push_back({r0, 0});
        color[r0] = 1;
        while (!stk.empty()) {
            auto& [u, c] = stk.back();
            if (c < 128) {
                const int v = tr[u][c++];
                if (v < 0) continue;
                if (color[v] == 1) {
                    mx[u] = -1;  // on the current path: a cycle
                } else if (color[v] == 0) {
                    color[v] = 1;
                    stk.push_back({v, 0});
                }
                continue;
            }
            int best = acc[u] ? 0 : -3;
            bool unb = mx[u] == -1;
            for (int cc = 0; cc < 128 && !unb; ++cc) {
                const int v = tr[u][cc];
                if (v < 0) continue;
                if (mx[v] == -1) unb = true;
                else if (mx[v] >= 0) best = std::max(best, mx[v] + 1);
            }
            mx[u] = unb ? -1 : best;
            color[u] = 2;
            stk.pop_back();
        }
    }
    out.next_off = static_cast<uint32_t>(next.size());
    out.info_off = static_cast<uint32_t>(info.size());
    out.n_states = static_cast<uint32_t>(ns);
    out.start = 0;
    for (int i = 0; i < ns; ++i)
        for (int c = 0; c < 128; ++c) next.push_back(static_cast<int16_t>(tr[i][c]));
    for (int i = 0; i < ns; ++i) {
        DfaInfo d{};
        d.accept = static_cast<uint16_t>(acc[i]);
        d.min_left = static_cast<uint16_t>(dist[i] < 0 ? 0xFFFF : std::min(dist[i], 0xFFFE));
        d.max_left = static_cast<uint16_t>(mx[i] < 0 ? 0xFFFF : std::min(mx[i], 0xFFFE));
        info.push_back(d);
    }
    return std::string();
}

const char* format_pattern(const std::string& f) {
    if (f == "date") return "^[0-9]{4}-(0[1-9]|1[0-2])-(0[1-9]|[12][0-9]|3[01])$";
    if (f == "time")
        return "^([01][0-9]|2[0-3]):[0-5][0-9]:([0-5][0-9]|60)(\\.[0-9]+)?([Zz]|[+-]([01][0-9]|2[0-3]):[0-5][0-9])$";
    if (f == "date-time")
        return "^[0-9]{4}-(0[1-9]|1[0-2])-(0[1-9]|[12][0-9]|3[01])[Tt]([01][0-9]|2[0-3]):[0-5][0-9]:([0-5][0-9]|60)"
               "(\\.[0-9]+)?([Zz]|[+-]([01][0-9]|2[0-3]):[0-5][0-9])$";
    if (f == "uuid") return "^[0-9a-fA-F]{8}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{12}$";
    return nullptr;
}

// ------------------------------------------------------------------------------------ compiler
constexpr int64_t kBig = INT64_MAX / 4;

struct Compiler {
    const JV* root = nullptr;
    std::vector<Node> nodes;
    std::vector<Prop> props;
    std::vector<uint32_t> ids;
    std::vector<Lit> lits;
    std::string bytes;
    std::vector<Dfa> dfas;
    std::vector<int16_t> next;
    std::vector<DfaInfo> info;
    std::map<std::string, uint32_t> refs;
    std::string err;
    uint32_t any_object = 0, any_array = 0, any_string = 0, any_number = 0, any_literal = 0;

    bool fail(const std::string& path, const std::string& m) {
        if (err.empty()) err = "JSON schema: " + path + ": " + m;
        return false;
    }
    uint32_t add(const Node& n) {
        nodes.push_back(n);
        return static_cast<uint32_t>(nodes.size()) - 1;
    }
    uint32_t literal_node(const std::vector<std::string>& texts) {
        Node n{};
        n.kind = N_ENUM;
        n.n = static_cast<uint16_t>(texts.size());
        n.first = static_cast<uint32_t>(lits.size());
        n.extra = kNone;
        for (const auto& t : texts) {
            lits.push_back(Lit{static_cast<uint32_t>(bytes.size()), static_cast<uint32_t>(t.size())});
            bytes += t;
        }
        return add(n);
    }
    void generic_nodes() {
        Node anyn{};
        anyn.kind = N_ANY;
        anyn.extra = kNone;
        add(anyn);  // node 0
        Node o{};
        o.kind = N_OBJECT;
        o.extra = 0;
        any_object = add(o);
        Node a{};
        a.kind = N_ARRAY;
        a.extra = 0;
        a.lo = 0;
        a.hi = kBig;
        any_array = add(a);
        Node s{};
        s.kind = N_STRING;
        s.extra = kNone;
        s.lo = 0;
        s.hi = kBig;
        any_string = add(s);
        Node nb{};
        nb.kind = N_NUMBER;
        nb.extra = kNone;
        any_number = add(nb);
        any_literal = literal_node({"true", "false", "null"});
    }

    // first characters a value of node x may begin with
    void first_chars(uint32_t x, std::set<int>& out, int depth = 0) {
        if (depth > 64) return;
        const Node& n = nodes[x];
        switch (n.kind) {
            case N_ANY: for (const char* c = "{[\"-0123456789tfn"; *c; ++c) out.insert(*c); break;
            case N_OBJECT: out.insert('{'); break;
            case N_ARRAY: out.insert('['); break;
            case N_STRING: out.insert('"'); break;
            case N_INTEGER:
            case N_NUMBER: for (const char* c = "-0123456789"; *c; ++c) out.insert(*c); break;
            case N_ENUM:
                for (uint32_t i = 0; i < n.n; ++i) out.insert(static_cast<unsigned char>(bytes[lits[n.first + i].off]));
                break;
            case N_UNION:
                for (uint32_t i = 0; i < n.n; ++i) first_chars(ids[n.first + i], out, depth + 1);
                break;
        }
    }

    uint32_t make_union(const std::vector<uint32_t>& alts, const std::string& path, bool& ok) {
        if (alts.size() == 1) return alts[0];
        std::set<int> seen;
        for (uint32_t a : alts) {
            std::set<int> f;
            first_chars(a, f);
            for (int c : f)
                if (!seen.insert(c).second) {
                    ok = fail(path, "anyOf / type alternatives that begin with the same character are not supported");
                    return 0;
                }
        }
        Node u{};
        u.kind = N_UNION;
        u.n = static_cast<uint16_t>(alts.size());
        u.first = static_cast<uint32_t>(ids.size());
        u.extra = kNone;
        for (uint32_t a : alts) ids.push_back(a);
        return add(u);
    }

    static bool is_annotation(const std::string& k) {
        return k == "title" || k == "description" || k == "default" || k == "examples" || k == "$schema" ||
               k == "$id" || k == "$comment" || k == "$defs" || k == "definitions";
    }
    static bool is_known(const std::string& k) {
        static const char* known[] = {"type", "properties", "required", "additionalProperties", "items", "prefixItems",
                                      "minItems", "maxItems", "enum", "const", "anyOf", "allOf", "$ref", "minimum",
                                      "maximum", "exclusiveMinimum", "exclusiveMaximum", "minLength", "maxLength",
                                      "pattern", "format"};
        for (const char* x : known)
            if (k == x) return true;
        return is_annotation(k);
    }

    const JV* resolve(const std::string& ref, const std::string& path) {
        if (ref == "#") return root;
        const std::string p1 = "#/$defs/", p2 = "#/definitions/";
        std::string name, sect;
        if (ref.compare(0, p1.size(), p1) == 0) {
            name = ref.substr(p1.size());
            sect = "$defs";
        } else if (ref.compare(0, p2.size(), p2) == 0) {
            name = ref.substr(p2.size());
            sect = "definitions";
        } else {
            fail(path, "$ref '" + ref + "' is not supported (only '#' and '#/$defs/<name>')");
            return nullptr;
        }
        const JV* defs = root->t == JV::OBJ ? root->get(sect) : nullptr;
        const JV* t = defs && defs->t == JV::OBJ ? defs->get(name) : nullptr;
        if (t == nullptr) fail(path, "$ref '" + ref + "' does not resolve");
        return t;
    }

    // allOf: one schema holding every branch's keywords (objects merge their properties and
    // required sets, bounds take the stricter value, equal keywords stay)
    bool merge_into(JV& acc, const JV& b, const std::string& path, int depth) {
        if (depth > 32) return fail(path, "allOf nests too deep");
        if (b.t == JV::BOOL) return b.b ? true : fail(path, "schema false in allOf matches nothing");
        if (b.t != JV::OBJ) return fail(path, "a schema must be an object or a boolean");
        const JV* bref = b.get("$ref");
        if (bref != nullptr) {
            if (bref->t != JV::STR) return fail(path, "$ref must be a string");
            const JV* t = resolve(bref->s, path);
            if (t == nullptr) return false;
            if (!merge_into(acc, *t, path, depth + 1)) return false;
        }
        for (const auto& kv : b.o) {
            const std::string& k = kv.first;
            if (k == "$ref" || is_annotation(k)) continue;
            if (k == "allOf") {
                if (kv.second.t != JV::ARR) return fail(path, "allOf must be an array");
                for (const JV& x : kv.second.a)
                    if (!merge_into(acc, x, path + "/allOf", depth + 1)) return false;
                continue;
            }
            JV* cur = nullptr;
            for (auto& e : acc.o)
                if (e.first == k) cur = &e.second;
            if (cur == nullptr) {
                acc.o.emplace_back(k, kv.second);
                continue;
            }
            if (k == "properties") {
                if (cur->t != JV::OBJ || kv.second.t != JV::OBJ) return fail(path, "properties must be an object");
                for (const auto& pv : kv.second.o) {
                    JV* have = nullptr;
                    for (auto& e : cur->o)
                        if (e.first == pv.first) have = &e.second;
                    if (have == nullptr) {
                        cur->o.push_back(pv);
                    } else {  // both constrain the property: allOf of the two
                        JV al;
                        al.t = JV::OBJ;
                        JV arr;
                        arr.t = JV::ARR;
                        arr.a = {*have, pv.second};
                        al.o.emplace_back("allOf", arr);
                        *have = al;
                    }
                }
            } else if (k == "required") {
                for (const JV& r : kv.second.a) {
                    bool dup = false;
                    for (const JV& x : cur->a) dup |= x.t == JV::STR && x.s == r.s;
                    if (!dup) cur->a.push_back(r);
                }
            } else if (k == "minimum" || k == "exclusiveMinimum" || k == "minLength" || k == "minItems" ||
                       k == "maximum" || k == "exclusiveMaximum" || k == "maxLength" || k == "maxItems") {
                if (cur->t != JV::NUM || kv.second.t != JV::NUM) return fail(path, "'" + k + "' must be a number");
                const double x = std::strtod(cur->s.c_str(), nullptr), y = std::strtod(kv.second.s.c_str(), nullptr);
                const bool takes_max = k.find("min") != std::string::npos || k.find("Min") != std::string::npos;
                if (takes_max ? y > x : y < x) *cur = kv.second;
            } else if (k == "additionalProperties") {
                if (kv.second.t == JV::BOOL && !kv.second.b) *cur = kv.second;
                else if (!(cur->t == JV::BOOL)) {
                    std::string a, bb;
                    compact(a, *cur);
                    compact(bb, kv.second);
                    if (a != bb) return fail(path, "allOf: conflicting additionalProperties schemas are not supported");
                }
            } else {
                std::string a, bb;
                compact(a, *cur);
                compact(bb, kv.second);
                if (a != bb) return fail(path, "allOf: conflicting '" + k + "' is not supported");
            }
        }
        return true;
    }

    bool allof_closed_ok(const JV& s, const JV& merged, const std::string& path, int depth) {
        const JV* mp = merged.get("properties");
        if (mp == nullptr || depth > 32) return true;
        std::vector<const JV*> branches{&s};
        if (const JV* al = s.get("allOf"))
            for (const JV& b : al->a) branches.push_back(&b);
        for (const JV* b : branches) {
            const JV* x = b;
            if (x->t == JV::OBJ && x->get("$ref") != nullptr && x->get("$ref")->t == JV::STR) {
                x = resolve(x->get("$ref")->s, path);
                if (x == nullptr) return false;
            }
            if (x->t != JV::OBJ) continue;
            const JV* ap = x->get("additionalProperties");
            if (ap == nullptr || !(ap->t == JV::BOOL && !ap->b)) continue;
            const JV* bp = x->get("properties");
            for (const auto& kv : mp->o)
                if (bp == nullptr || bp->get(kv.first) == nullptr)
                    return fail(path, "allOf: a branch with additionalProperties false does not declare '" +
                                          kv.first + "' (not supported)");
        }
        return true;
    }

    bool count_kw(const JV& s, const char* k, int64_t& v, const std::string& path) {
        const JV* x = s.get(k);
        if (x == nullptr) return true;
        if (x->t != JV::NUM || !num_is_integer(x->s) || std::strtod(x->s.c_str(), nullptr) < 0)
            return fail(path, std::string("'") + k + "' must be a non-negative integer");
        v = static_cast<int64_t>(std::strtod(x->s.c_str(), nullptr));
        return true;
    }

    uint32_t compile(const JV& s, const std::string& path, bool& ok, int depth = 0) {
        if (!ok) return 0;
        if (depth > 64) {
            ok = fail(path, "schema nests too deep");
            return 0;
        }
        if (s.t == JV::BOOL) {
            if (s.b) return 0;
            ok = fail(path, "schema false matches nothing");
            return 0;
        }
        if (s.t != JV::OBJ) {
            ok = fail(path, "a schema must be an object or a boolean");
            return 0;
        }
        for (const auto& kv : s.o)
            if (!is_known(kv.first)) {
                ok = fail(path, "keyword '" + kv.first + "' is not supported");
                return 0;
            }
        int validation = 0;
        for (const auto& kv : s.o) validation += is_annotation(kv.first) ? 0 : 1;
        if (const JV* r = s.get("$ref")) {
            if (validation > 1) {
                ok = fail(path, "$ref together with other keywords is not supported");
                return 0;
            }
            if (r->t != JV::STR) {
                ok = fail(path, "$ref must be a string");
                return 0;
            }
            auto it = refs.find(r->s);
            if (it != refs.end()) return it->second;
            const JV* t = resolve(r->s, path);
            if (t == nullptr) {
                ok = false;
                return 0;
            }
            Node ph{};
            ph.kind = N_ANY;
            ph.extra = kNone;
            const uint32_t id = add(ph);  // the target's node, filled in below (recursion sees this id)
            refs[r->s] = id;
            const uint32_t x = compile(*t, r->s, ok, depth + 1);
            if (!ok) return 0;
            nodes[id] = nodes[x];
            return id;
        }
        if (s.get("allOf") != nullptr) {
            JV m;
            m.t = JV::OBJ;
            if (!merge_into(m, s, path, depth)) {
                ok = false;
                return 0;
            }
            // a branch with additionalProperties false refuses every property it does not declare,
            // so the merged object is the allOf only when that branch declares them all
            if (!allof_closed_ok(s, m, path, depth)) {
                ok = false;
                return 0;
            }
            return compile(m, path, ok, depth + 1);
        }
        if (const JV* any = s.get("anyOf")) {
            if (validation > 1) {
                ok = fail(path, "anyOf together with other keywords is not supported");
                return 0;
            }
            if (any->t != JV::ARR || any->a.empty()) {
                ok = fail(path, "anyOf must be a non-empty array");
                return 0;
            }
            std::vector<uint32_t> alts;
            for (size_t i = 0; i < any->a.size(); ++i) {
                const uint32_t x = compile(any->a[i], path + "/anyOf/" + std::to_string(i), ok, depth + 1);
                if (!ok) return 0;
                if (nodes[x].kind == N_UNION) {  // flatten nested unions
                    for (uint32_t j = 0; j < nodes[x].n; ++j) alts.push_back(ids[nodes[x].first + j]);
                } else {
                    alts.push_back(x);
                }
            }
            return make_union(alts, path, ok);
        }
        // the value types this schema admits
        std::vector<std::string> types;
        if (const JV* t = s.get("type")) {
            if (t->t == JV::STR) {
                types.push_back(t->s);
            } else if (t->t == JV::ARR && !t->a.empty()) {
                for (const JV& x : t->a) {
                    if (x.t != JV::STR) {
                        ok = fail(path, "type must be a name or a list of names");
                        return 0;
                    }
                    types.push_back(x.s);
                }
            } else {
                ok = fail(path, "type must be a name or a list of names");
                return 0;
            }
            for (const auto& x : types)
                if (x != "object" && x != "array" && x != "string" && x != "integer" && x != "number" &&
                    x != "boolean" && x != "null") {
                    ok = fail(path, "unknown type '" + x + "'");
                    return 0;
                }
        }
        const JV* en = s.get("enum");
        const JV* cn = s.get("const");
        if (en != nullptr || cn != nullptr) {
            std::vector<const JV*> vals;
            if (cn != nullptr) vals.push_back(cn);
            if (en != nullptr) {
                if (en->t != JV::ARR || en->a.empty()) {
                    ok = fail(path, "enum must be a non-empty array");
                    return 0;
                }
                if (cn == nullptr)
                    for (const JV& x : en->a) vals.push_back(&x);
                else {  // const and enum: the const value, if the enum holds it
                    std::string c0;
                    compact(c0, *cn);
                    bool in = false;
                    for (const JV& x : en->a) {
                        std::string t;
                        compact(t, x);
                        in |= t == c0;
                    }
                    if (!in) vals.clear();
                }
            }
            std::vector<std::string> texts;
            for (const JV* v : vals) {
                const char* tn = v->t == JV::OBJ ? "object" : v->t == JV::ARR ? "array" : v->t == JV::STR ? "string"
                                 : v->t == JV::BOOL ? "boolean" : v->t == JV::NUL ? "null"
                                 : (num_is_integer(v->s) ? "integer" : "number");
                bool typed = types.empty();
                for (const auto& t : types)
                    typed |= t == tn || (t == "number" && std::strcmp(tn, "integer") == 0);
                if (!typed) continue;
                std::string txt;
                compact(txt, *v);
                if (std::find(texts.begin(), texts.end(), txt) == texts.end()) texts.push_back(txt);
            }
            if (texts.empty()) {
                ok = fail(path, "enum / const admits no value");
                return 0;
            }
            if (texts.size() > 64) {
                ok = fail(path, "more than 64 enum values are not supported");
                return 0;
            }
            return literal_node(texts);
        }
        if (types.empty()) {  // infer the type from the keywords present
            const bool o = s.get("properties") || s.get("required") || s.get("additionalProperties");
            const bool a = s.get("items") || s.get("prefixItems") || s.get("minItems") || s.get("maxItems");
            const bool st = s.get("minLength") || s.get("maxLength") || s.get("pattern") || s.get("format");
            const bool i = s.get("minimum") || s.get("maximum") || s.get("exclusiveMinimum") || s.get("exclusiveMaximum");
            if (o + a + st + i > 1) {
                ok = fail(path, "keywords of several types without 'type' are not supported");
                return 0;
            }
            if (o) types.push_back("object");
            else if (a) types.push_back("array");
            else if (st) types.push_back("string");
            else if (i) types.push_back("integer");
            else return 0;  // any value
        }
        if (std::find(types.begin(), types.end(), "number") != types.end())
            types.erase(std::remove(types.begin(), types.end(), std::string("integer")), types.end());
        std::vector<uint32_t> alts;
        for (const auto& t : types) {
            const uint32_t x = compile_type(s, t, path, ok, depth);
            if (!ok) return 0;
            alts.push_back(x);
        }
        return make_union(alts, path, ok);
    }

    uint32_t compile_type(const JV& s, const std::string& t, const std::string& path, bool& ok, int depth) {
        if (t == "boolean") return literal_node({"true", "false"});
        if (t == "null") return literal_node({"null"});
        if (t == "number") {
            if (s.get("minimum") || s.get("maximum") || s.get("exclusiveMinimum") || s.get("exclusiveMaximum")) {
                ok = fail(path, "bounds on non-integers are not supported");
                return 0;
            }
            return any_number;
        }
        if (t == "integer") {
            Node n{};
            n.kind = N_INTEGER;
            n.extra = kNone;
            double lo = -9.2e18, hi = 9.2e18;
            auto bound = [&](const char* k, double& v, bool lower, bool excl) {
                const JV* x = s.get(k);
                if (x == nullptr) return true;
                if (x->t != JV::NUM) return fail(path, std::string("'") + k + "' must be a number");
                const double d = std::strtod(x->s.c_str(), nullptr);
                double b = lower ? std::ceil(d) : std::floor(d);
                if (excl && b == d) b += lower ? 1.0 : -1.0;
                v = lower ? std::max(v, b) : std::min(v, b);
                return true;
            };
            if (!bound("minimum", lo, true, false) || !bound("exclusiveMinimum", lo, true, true) ||
                !bound("maximum", hi, false, false) || !bound("exclusiveMaximum", hi, false, true)) {
                ok = false;
                return 0;
            }
            const double cap = 4.0e18;  // magnitudes the automaton tracks exactly
            if (lo > hi || lo > cap || hi < -cap) {
                ok = fail(path, "integer bounds admit no value");
                return 0;
            }
            n.lo = static_cast<int64_t>(std::max(lo, -cap));
            n.hi = static_cast<int64_t>(std::min(hi, cap));
            return add(n);
        }
        if (t == "string") {
            Node n{};
            n.kind = N_STRING;
            n.extra = kNone;
            n.lo = 0;
            n.hi = kBig;
            if (!count_kw(s, "minLength", n.lo, path) || !count_kw(s, "maxLength", n.hi, path)) {
                ok = false;
                return 0;
            }
            if (n.lo > n.hi) {
                ok = fail(path, "minLength above maxLength");
                return 0;
            }
            const JV* pat = s.get("pattern");
            const JV* fmt = s.get("format");
            if (pat && fmt) {
                ok = fail(path, "pattern together with format is not supported");
                return 0;
            }
            std::string re;
            if (pat) {
                if (pat->t != JV::STR) {
                    ok = fail(path, "pattern must be a string");
                    return 0;
                }
                re = pat->s;
            } else if (fmt) {
                const char* f = fmt->t == JV::STR ? format_pattern(fmt->s) : nullptr;
                if (f == nullptr) {
                    ok = fail(path, "format '" + (fmt->t == JV::STR ? fmt->s : std::string("?")) + "' is not supported");
                    return 0;
                }
                re = f;
            }
            if (!re.empty()) {
                Dfa d{};
                const std::string e = build_dfa(re, next, info, d);
                if (!e.empty()) {
                    ok = fail(path, e);
                    return 0;
                }
                const DfaInfo& i0 = info[d.info_off + d.start];
                if (i0.min_left > n.hi || (i0.max_left != 0xFFFF && i0.max_left < n.lo)) {
                    ok = fail(path, "pattern and length bounds admit no string");
                    return 0;
                }
                n.extra = static_cast<uint32_t>(dfas.size());
                dfas.push_back(d);
            }
            return add(n);
        }
        if (t == "array") {
            Node n{};
            n.kind = N_ARRAY;
            n.lo = 0;
            n.hi = kBig;
            if (!count_kw(s, "minItems", n.lo, path) || !count_kw(s, "maxItems", n.hi, path)) {
                ok = false;
                return 0;
            }
            std::vector<uint32_t> pre;
            if (const JV* pi = s.get("prefixItems")) {
                if (pi->t != JV::ARR) {
                    ok = fail(path, "prefixItems must be an array");
                    return 0;
                }
                for (size_t i = 0; i < pi->a.size(); ++i) {
                    pre.push_back(compile(pi->a[i], path + "/prefixItems/" + std::to_string(i), ok, depth + 1));
                    if (!ok) return 0;
                }
            }
            uint32_t items = 0;  // absent: any value
            if (const JV* it = s.get("items")) {
                if (it->t == JV::BOOL && !it->b) items = kNone;
                else items = compile(*it, path + "/items", ok, depth + 1);
                if (!ok) return 0;
            }
            if (items == kNone && n.lo > static_cast<int64_t>(pre.size())) {
                ok = fail(path, "minItems above the items allowed");
                return 0;
            }
            if (n.lo > n.hi) {
                ok = fail(path, "minItems above maxItems");
                return 0;
            }
            n.n = static_cast<uint16_t>(pre.size());
            n.first = static_cast<uint32_t>(ids.size());
            for (uint32_t x : pre) ids.push_back(x);
            n.extra = items;
            return add(n);
        }
        // object
        Node n{};
        n.kind = N_OBJECT;
        std::vector<std::pair<std::string, uint32_t>> ps;
        if (const JV* pr = s.get("properties")) {
            if (pr->t != JV::OBJ) {
                ok = fail(path, "properties must be an object");
                return 0;
            }
            for (const auto& kv : pr->o) {
                const uint32_t x = compile(kv.second, path + "/properties/" + kv.first, ok, depth + 1);
                if (!ok) return 0;
                ps.emplace_back(kv.first, x);
            }
        }
        uint32_t addl = 0;  // absent: any additional property
        if (const JV* ap = s.get("additionalProperties")) {
            if (ap->t == JV::BOOL) addl = ap->b ? 0 : kNone;
            else addl = compile(*ap, path + "/additionalProperties", ok, depth + 1);
            if (!ok) return 0;
        }
        uint64_t req = 0;
        if (const JV* rq = s.get("required")) {
            if (rq->t != JV::ARR) {
                ok = fail(path, "required must be an array");
                return 0;
            }
            for (const JV& r : rq->a) {
                if (r.t != JV::STR) {
                    ok = fail(path, "required must hold property names");
                    return 0;
                }
                size_t i = 0;
                while (i < ps.size() && ps[i].first != r.s) ++i;
                if (i == ps.size()) {  // required but not declared: an additional property, named
                    if (addl == kNone) {
                        ok = fail(path, "required property '" + r.s + "' is not allowed by additionalProperties");
                        return 0;
                    }
                    ps.emplace_back(r.s, addl);
                }
                if (i >= 64) {
                    ok = fail(path, "more than 64 properties are not supported");
                    return 0;
                }
                req |= 1ull << i;
            }
        }
        if (ps.size() > 64) {
            ok = fail(path, "more than 64 properties are not supported");
            return 0;
        }
        n.n = static_cast<uint16_t>(ps.size());
        n.first = static_cast<uint32_t>(props.size());
        n.extra = addl;
        n.required = req;
        for (const auto& p : ps) {
            std::string key;
            escape_into(key, p.first);
            props.push_back(Prop{static_cast<uint32_t>(bytes.size()), static_cast<uint32_t>(key.size()), p.second, 0});
            bytes += key;
        }
        return add(n);
    }
};

// ------------------------------------------------------------------------------------ kernels
constexpr int kMaskThreads = 256;
constexpr uint32_t kTokSpecial = 1u, kTokEos = 2u;

struct TokInfo {       // what the mask tables test of a token, in one 8-byte load
    uint8_t flags;     // kTokSpecial / kTokEos
    uint8_t first;     // first byte (0 for an empty token)
    uint8_t second;    // second byte (0 for a shorter token)
    uint8_t pad;
    uint16_t plain;    // code points of a token that is a plain string body, else kNotPlain
    uint16_t pad2;
};
static_assert(sizeof(TokInfo) == 8, "token record");
struct SVocab {
    const uint8_t* bytes;
    const uint64_t* off;
    const uint8_t* flags;   // kTokSpecial / kTokEos
    const TokInfo* info;
    uint32_t vocab;
};
constexpr uint16_t kNotPlain = 0xFFFFu;

// Code points of a token that a string in its plain state (no escape or UTF-8 sequence open)
// takes whole and stays plain after: no quote, backslash or control byte, complete UTF-8 sequences.
// kNotPlain otherwise (the token needs the full walk).
uint16_t plain_code_points(const uint8_t* b, size_t n) {
    if (n == 0) return kNotPlain;
    uint32_t esc = 0, utf = 0, cp = 0;
    for (size_t i = 0; i < n; ++i) {
        if (b[i] == '\\') return kNotPlain;
        bool starts = false;
        if (str_byte(b[i], esc, utf, starts) != 1) return kNotPlain;
        cp += starts ? 1u : 0u;
    }
    return (esc == 0u && (utf & 3u) == 0u && cp < kNotPlain) ? static_cast<uint16_t>(cp) : kNotPlain;
}

__global__ void schema_reset_kernel(State* s, uint32_t n, uint32_t root) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n) start_state(s[r], root);
}

constexpr uint32_t kTileWords = 64;    // mask words per tile of a block (2,048 tokens)
constexpr uint32_t kQueueCap = 8192;   // queued walks (a walk phase runs when a tile could overflow it)
constexpr uint32_t kProgSmem = 48 * 1024;  // programs up to this size are walked from shared memory
constexpr uint32_t kWordsPerIter = 4;  // mask words a warp tests per iteration

// Whether the row at state `st` takes token `id` (not EOS, not special): its bytes walked on an
// overlay of the stack.
__device__ __noinline__ bool walk_token(const Prog& P, const SVocab& V, const State& st, uint32_t id) {
    const uint64_t b0 = V.off[id], b1 = V.off[id + 1];
    OverlayStack<SIXI_SCHEMA_MASK_OPENS> ov(st);
    Machine<OverlayStack<SIXI_SCHEMA_MASK_OPENS>> m(P, ov);
    bool ok = b1 > b0;
    for (uint64_t j = b0; j < b1 && ok; ++j) ok = m.step(V.bytes[j]);
    return ok;
}

// One block per (row, vocabulary slice): the row's state in shared memory, per-state tables of
// first bytes (and of bytes after a space), tokens decided by those tables or queued for a walk of
// their bytes on an overlay of the stack, 32 verdicts per mask word.
__global__ void __launch_bounds__(kMaskThreads, 3) schema_mask_kernel(const Prog PG, const SVocab V, const State* states,
                                                                   uint32_t* masks, uint64_t stride, uint32_t prog_in_smem) {
    // The automaton's tables are read by every step of every walk, in dependent chains: a copy in
    // shared memory keeps them off the global-memory latency (the program is a few KB for a
    // typical schema; larger ones are walked from global memory).
    extern __shared__ __align__(16) uint8_t sprog[];
    if (prog_in_smem) {
        const uint4* src4 = reinterpret_cast<const uint4*>(PG.base);
        for (uint32_t i = threadIdx.x; i < PG.base_bytes / 16u; i += blockDim.x) reinterpret_cast<uint4*>(sprog)[i] = src4[i];
    }
    const Prog P = prog_in_smem ? rebase(PG, sprog) : PG;
    static_assert(kMaskThreads >= 256, "one thread per first byte");
    __shared__ State st;
    __shared__ uint32_t st_ok, eos_ok;
    __shared__ int32_t str_room;   // a plain-string top frame: code points it may still take, else -1
    __shared__ uint32_t first_ok[8];  // bytes the state takes as a token's first byte
    __shared__ uint32_t after_sp[8];  // bytes it takes after a space (most tokens start with one)
    __shared__ uint32_t qid[kQueueCap];    // tokens of the tile that need a walk
    __shared__ uint32_t qn;
    const uint32_t row = blockIdx.y;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&states[row]);
    for (uint32_t i = threadIdx.x; i < sizeof(State) / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(&st)[i] = src[i];
    if (threadIdx.x < 8) first_ok[threadIdx.x] = 0u;
    if (threadIdx.x >= 8 && threadIdx.x < 16) after_sp[threadIdx.x - 8] = 0u;
    __syncthreads();
    if (threadIdx.x == 0) st_ok = state_ok(P, st) ? 1u : 0u;
    __syncthreads();
    const uint32_t words = (V.vocab + 31u) / 32u;
    uint32_t* out = masks + static_cast<uint64_t>(row) * stride;
    const bool dead = st.failed != 0u || st.depth == 0u || st_ok == 0u;  // no token for a malformed state
    if (!dead) {
        // The first-byte table (one step of the automaton per byte) rejects most tokens of a state
        // without a walk; it is exact for the first byte, so a token it passes is walked in full.
        if (threadIdx.x < 256) {
            OverlayStack<SIXI_SCHEMA_MASK_OPENS> ov(st);
            Machine<OverlayStack<SIXI_SCHEMA_MASK_OPENS>> m(P, ov);
            if (m.step(threadIdx.x)) atomicOr(&first_ok[threadIdx.x >> 5], 1u << (threadIdx.x & 31u));
            OverlayStack<SIXI_SCHEMA_MASK_OPENS> ov2(st);
            Machine<OverlayStack<SIXI_SCHEMA_MASK_OPENS>> m2(P, ov2);
            if (m2.step(' ') && m2.step(threadIdx.x)) atomicOr(&after_sp[threadIdx.x >> 5], 1u << (threadIdx.x & 31u));
        }
        if (threadIdx.x == 0) {
            OverlayStack<SIXI_SCHEMA_MASK_OPENS> ov(st);
            Machine<OverlayStack<SIXI_SCHEMA_MASK_OPENS>> m(P, ov);
            eos_ok = m.complete() ? 1u : 0u;
            // A string in its plain state without a pattern: a plain token of n code points is
            // allowed exactly when the length bound admits n more (str_byte accepts every byte).
            const Frame& t = st.f[st.depth - 1];
            const Node& N = P.nodes[t.node];
            const bool plain = t.kind == F_STR && N.extra == kNone && t.pos == 0u && (t.b & 0x1Fu) == 0u;
            const int64_t room = N.hi - static_cast<int64_t>(t.a);
            str_room = plain ? static_cast<int32_t>(room < 0 ? 0 : (room > 0x7FFFFFFF ? 0x7FFFFFFF : room)) : -1;
        }
    }
    __syncthreads();
    // Tiles of kTileWords mask words of this block's contiguous range: the table tests decide most
    // tokens at once; the rest are queued and walked by the whole block together, so that a walk
    // does not hold up a warp of decided tokens; the tile's words are written once at the end.
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t wpb = (words + gridDim.x - 1u) / gridDim.x;
    const uint32_t w_begin = blockIdx.x * wpb;
    const uint32_t w_end = w_begin + wpb < words ? w_begin + wpb : words;
    // Queued walks run once for the block's whole range (or when the queue could overflow): a
    // walk phase leaves most threads waiting at the barrier, so there should be as few as can be.
    auto walk_queue = [&]() {
        const uint32_t nq = qn;
        for (uint32_t i = threadIdx.x; i < nq; i += kMaskThreads) {
            const uint32_t id = qid[i];
            if (walk_token(P, V, st, id)) atomicOr(&out[id / 32u], 1u << (id & 31u));
        }
        __syncthreads();
        if (threadIdx.x == 0) qn = 0u;
        __syncthreads();
    };
    if (threadIdx.x == 0) qn = 0u;
    __syncthreads();
    for (uint32_t t0 = w_begin; t0 < w_end; t0 += kTileWords) {
        const uint32_t nw = w_end - t0 < kTileWords ? w_end - t0 : kTileWords;
        const uint32_t q_now = qn;  // every thread reads it before any thread adds to it again
        __syncthreads();
        if (q_now + kTileWords * 32u > kQueueCap) walk_queue();
        // each warp takes kWordsPerIter words at a time, their records loaded together; the
        // decided bits go out at once, the walks' bits are OR-ed in later
        for (uint32_t wi0 = warp * kWordsPerIter; wi0 < nw; wi0 += kWordsPerIter * (kMaskThreads / 32)) {
            TokInfo ti[kWordsPerIter];
#pragma unroll
            for (uint32_t u = 0; u < kWordsPerIter; ++u) {
                const uint32_t id = (t0 + wi0 + u) * 32u + lane;
                ti[u] = (wi0 + u < nw && id < V.vocab) ? V.info[id] : TokInfo{kTokSpecial, 0, 0, 0, kNotPlain, 0};
            }
#pragma unroll
            for (uint32_t u = 0; u < kWordsPerIter; ++u) {
                const uint32_t wi = wi0 + u;
                if (wi >= nw) break;  // warp-uniform
                const uint32_t id = (t0 + wi) * 32u + lane;
                bool ok = false, walk = false;
                if (!dead) {
                    const uint32_t c0 = ti[u].first, c1 = ti[u].second;
                    if (ti[u].flags & kTokEos) {
                        ok = eos_ok != 0u;
                    } else if (ti[u].flags & kTokSpecial) {
                        ok = false;  // also ids past the vocabulary
                    } else if (!((first_ok[c0 >> 5] >> (c0 & 31u)) & 1u)) {
                        ok = false;  // also every empty token (byte 0 is never a first byte)
                    } else if (c0 == ' ' && c1 != 0u && !((after_sp[c1 >> 5] >> (c1 & 31u)) & 1u)) {
                        ok = false;  // refused at its second byte (c1 = 0: a one-byte token)
                    } else if (str_room >= 0 && ti[u].plain != kNotPlain) {
                        ok = static_cast<int32_t>(ti[u].plain) <= str_room;
                    } else {
                        walk = true;
                    }
                }
                const unsigned wm = __ballot_sync(0xFFFFFFFFu, walk);
                uint32_t base = 0u;
                if (lane == 0 && wm != 0u) base = atomicAdd(&qn, static_cast<uint32_t>(__popc(wm)));
                base = __shfl_sync(0xFFFFFFFFu, base, 0);
                if (walk) qid[base + static_cast<uint32_t>(__popc(wm & ((1u << lane) - 1u)))] = id;  // < kQueueCap
                const unsigned word = __ballot_sync(0xFFFFFFFFu, ok);
                if (lane == 0) out[t0 + wi] = word;
            }
        }
        __syncthreads();
    }
    walk_queue();
    for (uint32_t w = words + blockIdx.x * blockDim.x + threadIdx.x; w < stride && blockIdx.x == 0; w += blockDim.x)
        out[w] = 0u;
}

__device__ bool apply_token(const Prog& P, const SVocab& V, State& s, int32_t tok) {
    if (tok < 0 || static_cast<uint32_t>(tok) >= V.vocab || s.failed || s.depth == 0) return false;
    const uint8_t fl = V.flags[tok];
    if (fl & kTokEos) {
        FullStack fs(s);
        Machine<FullStack> m(P, fs);
        if (!m.complete()) return false;
        s.depth = 0;  // finished: nothing may follow
        return true;
    }
    const uint64_t b0 = V.off[tok], b1 = V.off[tok + 1];
    if ((fl & kTokSpecial) || b1 == b0) return false;
    State t = s;
    FullStack fs(t);
    Machine<FullStack> m(P, fs);
    for (uint64_t j = b0; j < b1; ++j)
        if (!m.step(V.bytes[j])) return false;
    s = t;
    return true;
}

__global__ void schema_advance_kernel(const Prog P, const SVocab V, State* states, uint32_t n_rows, const int32_t* tokens,
                                      uint64_t token_stride, const int32_t* n_tokens, int32_t* out_status) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    State s = states[r];
    const int32_t n = n_tokens ? n_tokens[r] : 1;
    int32_t status = SIXI_OK;
    if (!state_ok(P, s)) {  // a malformed state is frozen, not walked
        s.failed = 1u;
        if (s.depth > static_cast<uint32_t>(kMaxDepth)) s.depth = 0u;
        states[r] = s;
        if (out_status) out_status[r] = SIXI_INVALID_ARGUMENT;
        return;
    }
    for (int32_t j = 0; j < n; ++j) {
        if (!apply_token(P, V, s, tokens[static_cast<uint64_t>(r) * token_stride + j])) {
            s.failed = 1u;
            status = SIXI_INVALID_ARGUMENT;
            break;
        }
    }
    states[r] = s;
    if (out_status) out_status[r] = status;
}

}  // namespace
}  // namespace schema
}  // namespace sixi_b200

using namespace sixi_b200::schema;

struct sixi_schema {
    int32_t device;
    uint32_t vocab;
    uint32_t root, any_object, any_array, any_string, any_number, any_literal;
    // host copies (sixi_schema_check_text)
    std::vector<Node> nodes;
    std::vector<Prop> props;
    std::vector<uint32_t> ids;
    std::vector<Lit> lits;
    std::string bytes;
    std::vector<Dfa> dfas;
    std::vector<int16_t> next;
    std::vector<DfaInfo> info;
    // device copies
    void* d_prog = nullptr;  // one allocation holding every table
    Prog dprog{};
    uint8_t* d_vbytes = nullptr;
    uint64_t* d_voff = nullptr;
    uint8_t* d_vflags = nullptr;
    TokInfo* d_vinfo = nullptr;

    Prog host_prog() const {
        Prog p{};
        p.nodes = nodes.data();
        p.props = props.data();
        p.ids = ids.data();
        p.lits = lits.data();
        p.bytes = reinterpret_cast<const uint8_t*>(bytes.data());
        p.dfas = dfas.data();
        p.next = next.data();
        p.info = info.data();
        p.root = root;
        p.any_object = any_object;
        p.any_array = any_array;
        p.any_string = any_string;
        p.any_number = any_number;
        p.any_literal = any_literal;
        p.n_nodes = static_cast<uint32_t>(nodes.size());
        p.n_dfas = static_cast<uint32_t>(dfas.size());
        return p;
    }

    // Unions whose alternatives are unions (possible through a $ref to an anyOf) take their
    // alternatives' alternatives instead, so that the automaton never nests unions. Their first
    // characters were checked disjoint over the nested alternatives already.
    void flatten_unions() {
        for (size_t u = 0; u < nodes.size(); ++u) {
            if (nodes[u].kind != N_UNION) continue;
            std::vector<uint32_t> work(ids.begin() + nodes[u].first, ids.begin() + nodes[u].first + nodes[u].n), flat;
            bool nested = false;
            for (int guard = 0; !work.empty() && guard < 65536; ++guard) {
                const uint32_t x = work.back();
                work.pop_back();
                if (x < nodes.size() && nodes[x].kind == N_UNION && x != u) {
                    nested = true;
                    for (uint32_t j = 0; j < nodes[x].n; ++j) work.push_back(ids[nodes[x].first + j]);
                } else {
                    flat.push_back(x);
                }
            }
            if (!nested || flat.size() > 0xFFFFu) continue;
            nodes[u].first = static_cast<uint32_t>(ids.size());
            nodes[u].n = static_cast<uint16_t>(flat.size());
            ids.insert(ids.end(), flat.begin(), flat.end());
        }
    }

    // Every index the automaton follows lies inside its table (the device walks trust them).
    bool tables_ok() const {
        const size_t nn = nodes.size();
        auto node_ok = [&](uint32_t x) { return x < nn; };
        if (!node_ok(root) || !node_ok(any_object) || !node_ok(any_array) || !node_ok(any_string) ||
            !node_ok(any_number) || !node_ok(any_literal))
            return false;
        for (const Dfa& d : dfas) {
            if (d.n_states == 0) continue;  // the placeholder entry of a program without patterns
            if (d.start >= d.n_states || static_cast<size_t>(d.next_off) + d.n_states * 128ull > next.size() ||
                static_cast<size_t>(d.info_off) + d.n_states > info.size())
                return false;
            for (size_t i = 0; i < d.n_states * 128ull; ++i)
                if (next[d.next_off + i] >= static_cast<int32_t>(d.n_states)) return false;
        }
        for (const Node& n : nodes) {
            switch (n.kind) {
                case N_ANY: break;
                case N_OBJECT:
                    if (static_cast<size_t>(n.first) + n.n > props.size() || (n.extra != kNone && !node_ok(n.extra)))
                        return false;
                    for (uint32_t i = 0; i < n.n; ++i) {
                        const Prop& pr = props[n.first + i];
                        if (!node_ok(pr.node) || static_cast<size_t>(pr.name_off) + pr.name_len > bytes.size()) return false;
                    }
                    break;
                case N_ARRAY:
                    if (static_cast<size_t>(n.first) + n.n > ids.size() || (n.extra != kNone && !node_ok(n.extra)))
                        return false;
                    for (uint32_t i = 0; i < n.n; ++i)
                        if (!node_ok(ids[n.first + i])) return false;
                    break;
                case N_STRING:
                    if (n.extra != kNone && (n.extra >= dfas.size() || dfas[n.extra].n_states == 0)) return false;
                    break;
                case N_INTEGER:
                case N_NUMBER: break;
                case N_ENUM:
                    if (static_cast<size_t>(n.first) + n.n > lits.size() || n.n > 64) return false;
                    for (uint32_t i = 0; i < n.n; ++i) {
                        const Lit& l = lits[n.first + i];
                        if (static_cast<size_t>(l.off) + l.len > bytes.size()) return false;
                    }
                    break;
                case N_UNION:
                    if (static_cast<size_t>(n.first) + n.n > ids.size()) return false;
                    for (uint32_t i = 0; i < n.n; ++i)
                        if (!node_ok(ids[n.first + i]) || nodes[ids[n.first + i]].kind == N_UNION) return false;
                    break;
                default: return false;
            }
        }
        return true;
    }
    SVocab svocab() const { return SVocab{d_vbytes, d_voff, d_vflags, d_vinfo, vocab}; }
};

namespace {

struct DevGuard {
    int prev = 0;
    explicit DevGuard(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DevGuard() { cudaSetDevice(prev); }
};

int32_t from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return SIXI_OK;
    if (e == cudaErrorMemoryAllocation) return SIXI_OUT_OF_MEMORY_VRAM;
    return SIXI_BACKEND_ERROR;
}

template <class T>
size_t table_bytes(const std::vector<T>& v) {
    return (v.size() * sizeof(T) + 255) / 256 * 256 + 256;
}

}  // namespace

extern "C" {

int32_t sixi_schema_compile(int32_t device, const char* schema_json, size_t schema_len, const uint8_t* host_bytes,
                            const uint64_t* host_offsets, uint32_t vocab, const uint8_t* host_flags, int32_t eos_id,
                            char* err, size_t err_cap, sixi_schema** out) {
    auto set_err = [&](const std::string& m) {
        if (err != nullptr && err_cap > 0) {
            const size_t n = std::min(m.size(), err_cap - 1);
            std::memcpy(err, m.data(), n);
            err[n] = '\0';
        }
    };
    if (out == nullptr || schema_json == nullptr || (vocab > 0 && (host_bytes == nullptr || host_offsets == nullptr)) ||
        (eos_id >= 0 && static_cast<uint32_t>(eos_id) >= vocab)) {
        set_err("invalid argument");
        return SIXI_INVALID_ARGUMENT;
    }
    *out = nullptr;
    Parser ps{schema_json, schema_json + schema_len, {}};
    JV doc;
    if (!ps.value(doc, 0)) {
        set_err(ps.err);
        return SIXI_INVALID_ARGUMENT;
    }
    ps.ws();
    if (ps.p != ps.e) {
        set_err("JSON schema: not valid JSON (text after the schema)");
        return SIXI_INVALID_ARGUMENT;
    }
    Compiler c;
    c.root = &doc;
    c.generic_nodes();
    bool ok = true;
    const uint32_t root = c.compile(doc, "#", ok);
    if (!ok) {
        set_err(c.err);
        return SIXI_INVALID_ARGUMENT;
    }
    std::unique_ptr<sixi_schema> g(new sixi_schema());
    g->device = device;
    g->vocab = vocab;
    g->root = root;
    g->any_object = c.any_object;
    g->any_array = c.any_array;
    g->any_string = c.any_string;
    g->any_number = c.any_number;
    g->any_literal = c.any_literal;
    g->nodes = std::move(c.nodes);
    g->props = std::move(c.props);
    g->ids = std::move(c.ids);
    g->lits = std::move(c.lits);
    g->bytes = std::move(c.bytes);
    g->dfas = std::move(c.dfas);
    g->next = std::move(c.next);
    g->info = std::move(c.info);
    for (auto* v : {&g->ids}) if (v->empty()) v->push_back(0);  // non-null tables
    if (g->props.empty()) g->props.push_back(Prop{});
    if (g->lits.empty()) g->lits.push_back(Lit{});
    if (g->bytes.empty()) g->bytes.push_back('\0');
    if (g->dfas.empty()) g->dfas.push_back(Dfa{});
    if (g->next.empty()) g->next.push_back(-1);
    if (g->info.empty()) g->info.push_back(DfaInfo{});
    g->flatten_unions();
    if (!g->tables_ok()) {
        set_err("JSON schema: internal error (inconsistent compiled program)");
        return SIXI_BACKEND_ERROR;
    }
    if (device >= 0) {  // device copies of the program and the vocabulary
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) {
            set_err("invalid device");
            return SIXI_INVALID_ARGUMENT;
        }
        DevGuard dg(device);
        const size_t sz = table_bytes(g->nodes) + table_bytes(g->props) + table_bytes(g->ids) + table_bytes(g->lits) +
                          (g->bytes.size() + 511) / 256 * 256 + table_bytes(g->dfas) + table_bytes(g->next) +
                          table_bytes(g->info);
        cudaError_t e = cudaMalloc(&g->d_prog, sz);
        uint8_t* p = static_cast<uint8_t*>(g->d_prog);
        size_t o = 0;
        auto put = [&](const void* src, size_t bytes_n, size_t room) -> const void* {
            const void* at = p + o;
            if (e == cudaSuccess) e = cudaMemcpy(p + o, src, bytes_n, cudaMemcpyHostToDevice);
            o += room;
            return at;
        };
        Prog dp = g->host_prog();
        if (e == cudaSuccess) {
            dp.nodes = static_cast<const Node*>(put(g->nodes.data(), g->nodes.size() * sizeof(Node), table_bytes(g->nodes)));
            dp.props = static_cast<const Prop*>(put(g->props.data(), g->props.size() * sizeof(Prop), table_bytes(g->props)));
            dp.ids = static_cast<const uint32_t*>(put(g->ids.data(), g->ids.size() * 4, table_bytes(g->ids)));
            dp.lits = static_cast<const Lit*>(put(g->lits.data(), g->lits.size() * sizeof(Lit), table_bytes(g->lits)));
            dp.bytes = static_cast<const uint8_t*>(put(g->bytes.data(), g->bytes.size(), (g->bytes.size() + 511) / 256 * 256));
            dp.dfas = static_cast<const Dfa*>(put(g->dfas.data(), g->dfas.size() * sizeof(Dfa), table_bytes(g->dfas)));
            dp.next = static_cast<const int16_t*>(put(g->next.data(), g->next.size() * 2, table_bytes(g->next)));
            dp.info = static_cast<const DfaInfo*>(put(g->info.data(), g->info.size() * sizeof(DfaInfo), table_bytes(g->info)));
        }
        dp.base = static_cast<const uint8_t*>(g->d_prog);
        dp.base_bytes = static_cast<uint32_t>(o);
        g->dprog = dp;
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(schema_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kProgSmem));
        std::vector<uint8_t> fl(vocab + 1, 0);
        for (uint32_t i = 0; i < vocab; ++i) fl[i] = host_flags && (host_flags[i] & 1u) ? kTokSpecial : 0;
        if (eos_id >= 0) fl[static_cast<uint32_t>(eos_id)] = kTokEos;
        const uint64_t nb = vocab ? host_offsets[vocab] : 0;
        if (e == cudaSuccess) e = cudaMalloc(&g->d_vbytes, nb + 16);
        if (e == cudaSuccess) e = cudaMalloc(&g->d_voff, (static_cast<size_t>(vocab) + 1) * 8);
        if (e == cudaSuccess) e = cudaMalloc(&g->d_vflags, vocab + 16);
        if (e == cudaSuccess && nb) e = cudaMemcpy(g->d_vbytes, host_bytes, nb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(g->d_voff, host_offsets, (static_cast<size_t>(vocab) + 1) * 8, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(g->d_vflags, fl.data(), vocab, cudaMemcpyHostToDevice);
        // per token: flags, first two bytes and, for plain string bodies, code points (mask tables)
        std::vector<TokInfo> info(vocab + 1, TokInfo{0, 0, 0, 0, kNotPlain, 0});
        for (uint32_t i = 0; i < vocab; ++i) {
            const uint64_t b0 = host_offsets[i], b1 = host_offsets[i + 1];
            info[i].flags = fl[i];
            if (b1 > b0) {
                info[i].first = host_bytes[b0];
                if (b1 > b0 + 1) info[i].second = host_bytes[b0 + 1];
                info[i].plain = plain_code_points(host_bytes + b0, static_cast<size_t>(b1 - b0));
            }
        }
        if (e == cudaSuccess) e = cudaMalloc(&g->d_vinfo, sizeof(TokInfo) * (static_cast<size_t>(vocab) + 1));
        if (e == cudaSuccess) e = cudaMemcpy(g->d_vinfo, info.data(), sizeof(TokInfo) * vocab, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            sixi_schema_destroy(g.release());
            set_err("device allocation failed");
            return from_cuda(e);
        }
    }
    *out = g.release();
    set_err("");
    return SIXI_OK;
}

void sixi_schema_destroy(sixi_schema* g) {
    if (g == nullptr) return;
    if (g->device >= 0) {
        DevGuard dg(g->device);
        cudaFree(g->d_prog);
        cudaFree(g->d_vbytes);
        cudaFree(g->d_voff);
        cudaFree(g->d_vflags);
        cudaFree(g->d_vinfo);
    }
    delete g;
}

uint32_t sixi_schema_vocab_size(const sixi_schema* g) { return g ? g->vocab : 0u; }

int32_t sixi_schema_reset(const sixi_schema* g, sixi_schema_state* states, uint32_t n_rows, void* stream) {
    if (g == nullptr || g->device < 0 || (n_rows > 0 && states == nullptr)) return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard dg(g->device);
    schema_reset_kernel<<<(n_rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<State*>(states), n_rows, g->root);
    return from_cuda(cudaGetLastError());
}

int32_t sixi_schema_fill_masks(const sixi_schema* g, const sixi_schema_state* states, uint32_t n_rows,
                               uint32_t* mask_words, uint64_t mask_stride, void* stream) {
    if (g == nullptr || g->device < 0 || (n_rows > 0 && (states == nullptr || mask_words == nullptr)) ||
        mask_stride < (g->vocab + 31u) / 32u || n_rows > 65535u)
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard dg(g->device);
    const uint32_t words = (g->vocab + 31u) / 32u;
    uint32_t bx = (words + (kMaskThreads / 32) - 1) / (kMaskThreads / 32);
    const uint32_t want = std::max(1u, 592u / n_rows);  // about four blocks per SM over the batch
    bx = std::min(bx, want);
    const uint32_t in_smem = g->dprog.base_bytes <= kProgSmem ? 1u : 0u;
    schema_mask_kernel<<<dim3(bx, n_rows), kMaskThreads, in_smem ? g->dprog.base_bytes : 0u,
                         static_cast<cudaStream_t>(stream)>>>(g->dprog, g->svocab(), reinterpret_cast<const State*>(states),
                                                              mask_words, mask_stride, in_smem);
    return from_cuda(cudaGetLastError());
}

int32_t sixi_schema_advance(const sixi_schema* g, sixi_schema_state* states, uint32_t n_rows, const int32_t* tokens,
                            uint64_t token_stride, const int32_t* n_tokens, int32_t* out_status, void* stream) {
    if (g == nullptr || g->device < 0 || (n_rows > 0 && (states == nullptr || tokens == nullptr))) return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard dg(g->device);
    schema_advance_kernel<<<(n_rows + 63) / 64, 64, 0, static_cast<cudaStream_t>(stream)>>>(
        g->dprog, g->svocab(), reinterpret_cast<State*>(states), n_rows, tokens, token_stride, n_tokens, out_status);
    return from_cuda(cudaGetLastError());
}

int32_t sixi_schema_check_text(const sixi_schema* g, const uint8_t* text, size_t len) {
    if (g == nullptr || (len > 0 && text == nullptr)) return 0;
    const Prog P = g->host_prog();
    std::unique_ptr<State> s(new State());
    start_state(*s, g->root);
    FullStack fs(*s);
    Machine<FullStack> m(P, fs);
    for (size_t i = 0; i < len; ++i)
        if (!m.step(text[i])) return 0;
    return m.complete() ? 2 : 1;
}

}  // extern "C"
