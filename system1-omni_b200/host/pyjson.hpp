// Request JSON for the worker-side processing (processing.cpp), as the reference's request
// contract reads and writes it (src/models/qwen3_5/native/src/json.rs):
//   parse: strict RFC 8259 (valid UTF-8, no NaN / Infinity, no lone surrogates, nesting
//          below 128), keys repeated in one object rejected, object key order kept,
//          integers that fit 64 bits kept as integers, other numbers as finite doubles;
//   dumps: Python's json.dumps(value, ensure_ascii=False[, sort_keys=True]): separators
//          ", " and ": ", floats as Python's repr.
#pragma once

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace s1json {

struct Value {
    enum Kind { NUL, BOOL, INT, FLOAT, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    int64_t i = 0;
    bool neg_u = false;  // INT: u holds a value above INT64_MAX
    uint64_t u = 0;
    double f = 0;
    std::string s;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;  // insertion order

    bool is_str() const { return kind == STR; }
    bool is_obj() const { return kind == OBJ; }
    bool is_arr() const { return kind == ARR; }
    bool is_null() const { return kind == NUL; }
    const Value* get(const std::string& k) const {
        if (kind != OBJ) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

// ---- UTF-8 ----
inline void put_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
        out += (char)cp;
    } else if (cp < 0x800) {
        out += (char)(0xC0 | (cp >> 6));
        out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
        out += (char)(0xE0 | (cp >> 12));
        out += (char)(0x80 | ((cp >> 6) & 0x3F));
        out += (char)(0x80 | (cp & 0x3F));
    } else {
        out += (char)(0xF0 | (cp >> 18));
        out += (char)(0x80 | ((cp >> 12) & 0x3F));
        out += (char)(0x80 | ((cp >> 6) & 0x3F));
        out += (char)(0x80 | (cp & 0x3F));
    }
}

// Decodes one code point at s[i]; false on invalid UTF-8 (overlong, surrogate, > U+10FFFF).
inline bool next_utf8(const std::string& s, size_t& i, uint32_t& cp) {
    const unsigned char c = (unsigned char)s[i];
    int n;
    uint32_t min;
    if (c < 0x80) {
        cp = c;
        i++;
        return true;
    } else if ((c & 0xE0) == 0xC0) {
        n = 1, cp = c & 0x1F, min = 0x80;
    } else if ((c & 0xF0) == 0xE0) {
        n = 2, cp = c & 0x0F, min = 0x800;
    } else if ((c & 0xF8) == 0xF0) {
        n = 3, cp = c & 0x07, min = 0x10000;
    } else {
        return false;
    }
    if (i + n >= s.size()) return false;  // the continuation bytes s[i + 1 .. i + n]
    for (int k = 1; k <= n; k++) {
        const unsigned char d = (unsigned char)s[i + k];
        if ((d & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (d & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += n + 1;
    return true;
}

inline bool valid_utf8(const std::string& s) {
    size_t i = 0;
    uint32_t cp;
    while (i < s.size())
        if (!next_utf8(s, i, cp)) return false;
    return true;
}

// ---- parse ----
class Parser {
public:
    explicit Parser(const std::string& t) : s_(t) {}
    bool parse(Value& out, std::string& err) {
        if (!valid_utf8(s_)) return fail(err, "invalid UTF-8");
        ws();
        if (!value(out, 0)) return fail(err, err_);
        ws();
        if (i_ != s_.size()) return fail(err, "trailing characters");
        return true;
    }

private:
    const std::string& s_;
    size_t i_ = 0;
    std::string err_ = "invalid JSON";

    static bool fail(std::string& err, const std::string& what) {
        err = what;
        return false;
    }
    bool bad(const char* what) {
        err_ = what;
        return false;
    }
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if (s_.compare(i_, n, w) != 0) return false;
        i_ += n;
        return true;
    }
    bool hex4(uint32_t& v) {
        if (i_ + 4 > s_.size()) return false;
        v = 0;
        for (int k = 0; k < 4; k++) {
            const char c = s_[i_ + k];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        i_ += 4;
        return true;
    }
    bool string(std::string& out) {
        if (i_ >= s_.size() || s_[i_] != '"') return bad("expected a string");
        i_++;
        while (true) {
            if (i_ >= s_.size()) return bad("unterminated string");
            const unsigned char c = (unsigned char)s_[i_];
            if (c == '"') {
                i_++;
                return true;
            }
            if (c < 0x20) return bad("control character in string");
            if (c != '\\') {
                out += (char)c;
                i_++;
                continue;
            }
            if (++i_ >= s_.size()) return bad("unterminated escape");
            const char e = s_[i_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return bad("invalid \\u escape");
                    if (cp >= 0xD800 && cp <= 0xDBFF) {
                        uint32_t lo;
                        if (!(lit("\\u") && hex4(lo) && lo >= 0xDC00 && lo <= 0xDFFF)) return bad("lone surrogate");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
                        return bad("lone surrogate");
                    }
                    put_utf8(out, cp);
                    break;
                }
                default: return bad("invalid escape");
            }
        }
    }
    bool number(Value& v) {
        const size_t a = i_;
        if (i_ < s_.size() && s_[i_] == '-') i_++;
        if (i_ >= s_.size()) return bad("invalid number");
        if (s_[i_] == '0') {
            i_++;
        } else if (s_[i_] >= '1' && s_[i_] <= '9') {
            while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
        } else {
            return bad("invalid number");
        }
        bool integral = true;
        if (i_ < s_.size() && s_[i_] == '.') {
            integral = false;
            i_++;
            if (i_ >= s_.size() || !isdigit((unsigned char)s_[i_])) return bad("invalid number");
            while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
        }
        if (i_ < s_.size() && (s_[i_] == 'e' || s_[i_] == 'E')) {
            integral = false;
            i_++;
            if (i_ < s_.size() && (s_[i_] == '+' || s_[i_] == '-')) i_++;
            if (i_ >= s_.size() || !isdigit((unsigned char)s_[i_])) return bad("invalid number");
            while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
        }
        const std::string text = s_.substr(a, i_ - a);
        if (integral) {
            errno = 0;
            char* end = nullptr;
            if (text[0] == '-') {
                const long long x = strtoll(text.c_str(), &end, 10);
                if (errno == 0) {
                    v.kind = Value::INT;
                    v.i = x;
                    return true;
                }
            } else {
                const unsigned long long x = strtoull(text.c_str(), &end, 10);
                if (errno == 0) {
                    v.kind = Value::INT;
                    if (x > (unsigned long long)INT64_MAX) {
                        v.neg_u = true;
                        v.u = x;
                    } else {
                        v.i = (int64_t)x;
                    }
                    return true;
                }
            }
        }
        const double d = strtod(text.c_str(), nullptr);
        if (!std::isfinite(d)) return bad("number out of range");
        v.kind = Value::FLOAT;
        v.f = d;
        return true;
    }
    bool value(Value& v, int depth) {
        if (depth >= 128) return bad("recursion limit exceeded");
        if (i_ >= s_.size()) return bad("unexpected end");
        const char c = s_[i_];
        if (c == '{') {
            v.kind = Value::OBJ;
            i_++;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') {
                i_++;
                return true;
            }
            while (true) {
                ws();
                std::string k;
                if (!string(k)) return false;
                for (const auto& kv : v.obj)
                    if (kv.first == k) return bad("key repeated in an object");
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') return bad("expected ':'");
                i_++;
                ws();
                v.obj.emplace_back(std::move(k), Value());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    i_++;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') {
                    i_++;
                    return true;
                }
                return bad("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Value::ARR;
            i_++;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') {
                i_++;
                return true;
            }
            while (true) {
                ws();
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    i_++;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') {
                    i_++;
                    return true;
                }
                return bad("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Value::STR;
            return string(v.s);
        }
        if (lit("true")) {
            v.kind = Value::BOOL;
            v.b = true;
            return true;
        }
        if (lit("false")) {
            v.kind = Value::BOOL;
            return true;
        }
        if (lit("null")) return true;
        return number(v);
    }
};

inline bool parse(const std::string& text, Value& out, std::string& err) {
    Parser p(text);
    return p.parse(out, err);
}

// ---- dumps ----
// Python's repr of a finite double: the shortest digits that read back to the same value,
// fixed notation for decimal exponents -4 .. 15 (with ".0" when integral), else
// d[.ddd]e+XX / e-XX with at least two exponent digits.
inline std::string float_repr(double x) {
    if (x == 0) return std::signbit(x) ? "-0.0" : "0.0";
    char buf[64];
    int p = 1;
    for (; p <= 17; p++) {
        snprintf(buf, sizeof(buf), "%.*e", p - 1, x);
        if (strtod(buf, nullptr) == x) break;
    }
    // buf: [-]d[.ddd]e[+-]XX
    std::string t(buf);
    const bool neg = t[0] == '-';
    if (neg) t.erase(0, 1);
    const size_t epos = t.find('e');
    std::string digits = t.substr(0, epos);
    const int exp = atoi(t.c_str() + epos + 1);
    digits.erase(std::remove(digits.begin(), digits.end(), '.'), digits.end());
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    std::string out = neg ? "-" : "";
    if (exp >= -4 && exp < 16) {
        if (exp < 0) {
            out += "0." + std::string((size_t)(-exp - 1), '0') + digits;
        } else if ((int)digits.size() <= exp + 1) {
            out += digits + std::string((size_t)(exp + 1 - (int)digits.size()), '0') + ".0";
        } else {
            out += digits.substr(0, (size_t)exp + 1) + "." + digits.substr((size_t)exp + 1);
        }
    } else {
        out += digits.substr(0, 1);
        if (digits.size() > 1) out += "." + digits.substr(1);
        char e[16];
        snprintf(e, sizeof(e), "e%c%02d", exp < 0 ? '-' : '+', exp < 0 ? -exp : exp);
        out += e;
    }
    return out;
}

inline void dump_string(std::string& out, const std::string& s) {
    out += '"';
    for (unsigned char c : s) {
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            case '\b': out += "\\b"; break;
            case '\f': out += "\\f"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    snprintf(b, sizeof(b), "\\u%04x", c);
                    out += b;
                } else {
                    out += (char)c;
                }
        }
    }
    out += '"';
}

inline void dump(std::string& out, const Value& v, bool sort_keys) {
    switch (v.kind) {
        case Value::NUL: out += "null"; break;
        case Value::BOOL: out += v.b ? "true" : "false"; break;
        case Value::INT: out += v.neg_u ? std::to_string(v.u) : std::to_string(v.i); break;
        case Value::FLOAT: out += float_repr(v.f); break;
        case Value::STR: dump_string(out, v.s); break;
        case Value::ARR:
            out += '[';
            for (size_t k = 0; k < v.arr.size(); k++) {
                if (k) out += ", ";
                dump(out, v.arr[k], sort_keys);
            }
            out += ']';
            break;
        case Value::OBJ: {
            std::vector<const std::pair<std::string, Value>*> items;
            for (const auto& kv : v.obj) items.push_back(&kv);
            if (sort_keys)  // code point order = byte order of UTF-8
                std::stable_sort(items.begin(), items.end(),
                                 [](const auto* a, const auto* b) { return a->first < b->first; });
            out += '{';
            for (size_t k = 0; k < items.size(); k++) {
                if (k) out += ", ";
                dump_string(out, items[k]->first);
                out += ": ";
                dump(out, items[k]->second, sort_keys);
            }
            out += '}';
            break;
        }
    }
}

inline std::string dumps(const Value& v, bool sort_keys = false) {
    std::string out;
    dump(out, v, sort_keys);
    return out;
}

}  // namespace s1json
