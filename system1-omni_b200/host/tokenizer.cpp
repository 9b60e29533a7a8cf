// Worker-side tokenizer: the byte-level BPE tokenizer of the Qwen family, read from a
// Hugging Face tokenizer.json, as the reference's worker runs it through the third-party
// `tokenizers` crate (pinned =0.22.2, src/models/open_jev/native/Cargo.toml:14;
// Processor::load / encode_questions, src/models/open_jev/native/src/processing.rs:41-60,
// 141-200). The published algorithm, restated:
//   1. added tokens (every entry of "added_tokens": matched first, leftmost-longest, on the
//      raw text when "normalized" is false, on the normalized text otherwise);
//   2. the normalizer (NFC, or none);
//   3. the pre-tokenizer: Split on the Qwen2 pattern (isolated) then ByteLevel without
//      its own regex; the pattern
//        (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
//      is matched by hand below, alternative by alternative in order, with the
//      backtracking the regex engine does;
//   4. ByteLevel: the UTF-8 bytes of each piece through the GPT-2 byte-to-character map;
//   5. BPE: repeatedly merge the adjacent pair with the lowest merge rank (ties: leftmost),
//      then look each symbol up in the vocabulary.
// The tokenizer.json shapes the Qwen tokenizers use are accepted, plus the word-level shape
// the reference's own processing tests build (WordLevel model, WhitespaceSplit
// pre-tokenizer, a TemplateProcessing post-processor adding special tokens); anything
// else is refused at load rather than tokenized differently.
#include "tokenizer.hpp"

#include <algorithm>
#include <fstream>
#include <queue>
#include <sstream>
#include <unordered_map>

#include "pyjson.hpp"

namespace s1tok {
namespace {

#include "unicode_data.inc"

const char* kQwenPattern =
    "(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";

template <size_t N>
bool in_ranges(const uint32_t (&r)[N][2], uint32_t cp) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < r[mid][0]) hi = mid;
        else if (cp > r[mid][1]) lo = mid + 1;
        else return true;
    }
    return false;
}

bool is_letter(uint32_t cp) { return in_ranges(kLetters, cp); }
bool is_number(uint32_t cp) { return in_ranges(kNumbers, cp); }
// Unicode White_Space (the regex \s)
bool is_space(uint32_t cp) {
    return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
           (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
           cp == 0x3000;
}
bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }

int combining_class(uint32_t cp) {
    size_t lo = 0, hi = sizeof(kCombining) / sizeof(kCombining[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < kCombining[mid][0]) hi = mid;
        else if (cp > kCombining[mid][1]) lo = mid + 1;
        else return (int)kCombining[mid][2];
    }
    return 0;
}

// Hangul syllables: decomposition and composition by arithmetic (Unicode 3.12)
constexpr uint32_t SBase = 0xAC00, LBase = 0x1100, VBase = 0x1161, TBase = 0x11A7;
constexpr uint32_t LCount = 19, VCount = 21, TCount = 28, NCount = VCount * TCount, SCount = LCount * NCount;

void decompose(uint32_t cp, std::vector<uint32_t>& out) {
    if (cp >= SBase && cp < SBase + SCount) {
        const uint32_t s = cp - SBase;
        out.push_back(LBase + s / NCount);
        out.push_back(VBase + (s % NCount) / TCount);
        if (s % TCount) out.push_back(TBase + s % TCount);
        return;
    }
    size_t lo = 0, hi = sizeof(kDecomp) / sizeof(kDecomp[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (cp < kDecomp[mid][0]) hi = mid;
        else if (cp > kDecomp[mid][0]) lo = mid + 1;
        else {
            for (uint32_t k = 0; k < kDecomp[mid][2]; k++) out.push_back(kDecompData[kDecomp[mid][1] + k]);
            return;
        }
    }
    out.push_back(cp);
}

bool compose_pair(uint32_t a, uint32_t b, uint32_t& c) {
    if (a >= LBase && a < LBase + LCount && b >= VBase && b < VBase + VCount) {
        c = SBase + ((a - LBase) * VCount + (b - VBase)) * TCount;
        return true;
    }
    if (a >= SBase && a < SBase + SCount && (a - SBase) % TCount == 0 && b > TBase && b < TBase + TCount) {
        c = a + (b - TBase);
        return true;
    }
    size_t lo = 0, hi = sizeof(kCompose) / sizeof(kCompose[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (a < kCompose[mid][0] || (a == kCompose[mid][0] && b < kCompose[mid][1])) hi = mid;
        else if (a > kCompose[mid][0] || b > kCompose[mid][1]) lo = mid + 1;
        else {
            c = kCompose[mid][2];
            return true;
        }
    }
    return false;
}

std::vector<uint32_t> to_cps(const std::string& s) {
    std::vector<uint32_t> out;
    size_t i = 0;
    uint32_t cp;
    while (i < s.size()) {
        if (!s1json::next_utf8(s, i, cp)) {
            cp = 0xFFFD;  // (inputs are validated UTF-8; kept total)
            i++;
        }
        out.push_back(cp);
    }
    return out;
}

std::string to_utf8(const std::vector<uint32_t>& cps, size_t a, size_t b) {
    std::string out;
    for (size_t i = a; i < b; i++) s1json::put_utf8(out, cps[i]);
    return out;
}

// NFC: canonical decomposition, canonical ordering, canonical composition (UAX #15).
std::vector<uint32_t> to_nfc(const std::vector<uint32_t>& in) {
    std::vector<uint32_t> d;
    d.reserve(in.size());
    for (uint32_t cp : in) decompose(cp, d);
    // canonical ordering: stable sort of each run of non-starters by class
    for (size_t i = 0; i < d.size();) {
        if (combining_class(d[i]) == 0) {
            i++;
            continue;
        }
        size_t j = i;
        while (j < d.size() && combining_class(d[j]) != 0) j++;
        std::stable_sort(d.begin() + i, d.begin() + j,
                         [](uint32_t a, uint32_t b) { return combining_class(a) < combining_class(b); });
        i = j;
    }
    // composition: a character joins the last starter unless a character between them has
    // class 0 or a class >= its own (after canonical ordering the last one between has the
    // largest class of them)
    std::vector<uint32_t> out;
    out.reserve(d.size());
    long starter = -1;  // index in out of the last starter
    for (uint32_t cp : d) {
        const int cc = combining_class(cp);
        if (starter >= 0) {
            const bool adjacent = (size_t)starter + 1 == out.size();
            const int between = adjacent ? -1 : combining_class(out.back());
            uint32_t comp;
            if ((adjacent || (between != 0 && between < cc)) && compose_pair(out[(size_t)starter], cp, comp)) {
                out[(size_t)starter] = comp;
                continue;
            }
        }
        if (cc == 0) starter = (long)out.size();
        out.push_back(cp);
    }
    return out;
}

// One match of the Qwen2 pre-tokenizer pattern at i (always at least one code point).
size_t match_piece(const std::vector<uint32_t>& c, size_t i) {
    const size_t n = c.size();
    auto letter = [&](size_t k) { return k < n && is_letter(c[k]); };
    auto lower = [&](size_t k) { return k < n ? (c[k] < 0x80 ? (uint32_t)tolower((int)c[k]) : c[k]) : 0u; };
    // (?i:'s|'t|'re|'ve|'m|'ll|'d)
    if (c[i] == '\'') {
        const uint32_t a = lower(i + 1), b = lower(i + 2);
        const bool s_ = a == 's' || (i + 1 < n && c[i + 1] == 0x17F);  // long s folds to s
        if (s_ || a == 't' || a == 'm' || a == 'd') return 2;
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    }
    // [^\r\n\p{L}\p{N}]?\p{L}+
    {
        size_t k = i;
        if (!is_crlf(c[k]) && !is_letter(c[k]) && !is_number(c[k]) && letter(k + 1)) k++;
        if (letter(k)) {
            while (letter(k)) k++;
            return k - i;
        }
    }
    // \p{N}
    if (is_number(c[i])) return 1;
    // ' '?[^\s\p{L}\p{N}]+[\r\n]*
    {
        auto other = [&](size_t k) { return k < n && !is_space(c[k]) && !is_letter(c[k]) && !is_number(c[k]); };
        size_t k = i;
        if (c[k] == ' ' && other(k + 1)) k++;
        if (other(k)) {
            while (other(k)) k++;
            while (k < n && is_crlf(c[k])) k++;
            return k - i;
        }
    }
    // whitespace run from i
    size_t j = i;
    while (j < n && is_space(c[j])) j++;
    if (j > i) {
        // \s*[\r\n]+ : up to and including the run's last CR / LF
        for (size_t k = j; k > i; k--)
            if (is_crlf(c[k - 1])) return k - i;
        // \s+(?!\S)
        if (j == n) return j - i;
        if (j - i >= 2) return j - i - 1;
        // \s+
        return j - i;
    }
    return 1;  // not reached: every code point falls in one of the classes above
}

// GPT-2's byte-to-character map of the ByteLevel pre-tokenizer.
std::vector<std::string> byte_map() {
    std::vector<int> bs;
    for (int b = '!'; b <= '~'; b++) bs.push_back(b);
    for (int b = 0xA1; b <= 0xAC; b++) bs.push_back(b);
    for (int b = 0xAE; b <= 0xFF; b++) bs.push_back(b);
    std::vector<uint32_t> cs(256, 0);
    std::vector<bool> have(256, false);
    for (int b : bs) {
        cs[b] = (uint32_t)b;
        have[b] = true;
    }
    uint32_t extra = 0;
    for (int b = 0; b < 256; b++)
        if (!have[b]) cs[b] = 256 + extra++;
    std::vector<std::string> out(256);
    for (int b = 0; b < 256; b++) s1json::put_utf8(out[b], cs[b]);
    return out;
}

bool read_file(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

}  // namespace

struct Tokenizer::Impl {
    struct Added {
        std::string text;
        uint32_t id;
        bool normalized;
    };
    std::vector<Added> added;
    bool nfc = false;
    bool ignore_merges = false;
    bool word_level = false;       // WordLevel model over WhitespaceSplit pieces
    long unk = -1;                 // WordLevel unknown-token id
    std::vector<long> template_;   // post-processor: ids to add, -1 for the sequence itself
    std::unordered_map<std::string, uint32_t> vocab;
    std::unordered_map<std::string, uint32_t> ranks;  // "a\x01b" -> merge rank
    std::vector<std::string> bytes = byte_map();

    // Splits `text` on added tokens (those with the given normalized flag); appends (piece,
    // id or -1) in order.
    void split_added(const std::string& text, bool normalized, std::vector<std::pair<std::string, long>>& out) const {
        size_t i = 0, start = 0;
        while (i < text.size()) {
            size_t best = 0;
            long id = -1;
            for (const auto& a : added)
                if (a.normalized == normalized && a.text.size() > best && text.compare(i, a.text.size(), a.text) == 0) {
                    best = a.text.size();
                    id = a.id;
                }
            if (best) {
                if (i > start) out.emplace_back(text.substr(start, i - start), -1);
                out.emplace_back(text.substr(i, best), id);
                i += best;
                start = i;
            } else {
                i++;
            }
        }
        if (start < text.size()) out.emplace_back(text.substr(start), -1);
    }

    void bpe(const std::string& word, std::vector<uint32_t>& ids, std::string& err) const {
        if (ignore_merges) {
            auto it = vocab.find(word);
            if (it != vocab.end()) {
                ids.push_back(it->second);
                return;
            }
        }
        // symbols: the word's characters (each a byte-map character)
        std::vector<std::string> sym;
        {
            size_t i = 0;
            uint32_t cp;
            while (i < word.size()) {
                const size_t a = i;
                s1json::next_utf8(word, i, cp);
                sym.push_back(word.substr(a, i - a));
            }
        }
        std::vector<int> prev(sym.size()), next(sym.size());  // links of the surviving symbols
        std::vector<bool> alive(sym.size(), true);
        for (size_t k = 0; k < sym.size(); k++) {
            prev[k] = (int)k - 1;
            next[k] = k + 1 < sym.size() ? (int)k + 1 : -1;
        }
        struct Cand {
            uint32_t rank;
            int pos;
            std::string left, right;
            bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
        };
        std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> q;
        auto push = [&](int a) {
            const int b = next[a];
            if (a < 0 || b < 0) return;
            auto it = ranks.find(sym[a] + '\x01' + sym[b]);
            if (it != ranks.end()) q.push({it->second, a, sym[a], sym[b]});
        };
        for (size_t k = 0; k + 1 < sym.size(); k++) push((int)k);
        while (!q.empty()) {
            Cand c = q.top();
            q.pop();
            const int a = c.pos, b = next[a];
            // stale: the pair changed since it was queued
            if (!alive[a] || b < 0 || sym[a] != c.left || sym[b] != c.right) continue;
            sym[a] += sym[b];
            alive[b] = false;
            next[a] = next[b];
            if (next[b] >= 0) prev[next[b]] = a;
            if (prev[a] >= 0) push(prev[a]);
            push(a);
        }
        for (int k = sym.empty() ? -1 : 0; k >= 0; k = next[k]) {  // the first symbol always survives
            auto it = vocab.find(sym[k]);
            if (it == vocab.end()) {
                err = "symbol not in the vocabulary";
                return;
            }
            ids.push_back(it->second);
        }
    }

    bool encode(const std::string& text, std::vector<uint32_t>& ids, std::string& err) const {
        if (!s1json::valid_utf8(text)) {
            err = "text is not valid UTF-8";
            return false;
        }
        std::vector<std::pair<std::string, long>> raw;
        split_added(text, false, raw);
        for (const auto& part : raw) {
            if (part.second >= 0) {
                ids.push_back((uint32_t)part.second);
                continue;
            }
            std::vector<uint32_t> cps = to_cps(part.first);
            if (nfc) cps = to_nfc(cps);
            std::vector<std::pair<std::string, long>> norm;
            split_added(to_utf8(cps, 0, cps.size()), true, norm);
            for (const auto& piece : norm) {
                if (piece.second >= 0) {
                    ids.push_back((uint32_t)piece.second);
                    continue;
                }
                const std::vector<uint32_t> c = to_cps(piece.first);
                if (word_level) {  // whitespace-separated words, each a vocabulary entry or the unknown token
                    for (size_t i = 0; i < c.size();) {
                        while (i < c.size() && is_space(c[i])) i++;
                        size_t j = i;
                        while (j < c.size() && !is_space(c[j])) j++;
                        if (j > i) {
                            auto it = vocab.find(to_utf8(c, i, j));
                            if (it != vocab.end()) {
                                ids.push_back(it->second);
                            } else if (unk >= 0) {
                                ids.push_back((uint32_t)unk);
                            } else {
                                err = "word not in the vocabulary";
                                return false;
                            }
                        }
                        i = j;
                    }
                    continue;
                }
                for (size_t i = 0; i < c.size();) {
                    const size_t len = match_piece(c, i);
                    const std::string utf8 = to_utf8(c, i, i + len);
                    std::string mapped;
                    for (unsigned char byte : utf8) mapped += bytes[byte];
                    bpe(mapped, ids, err);
                    if (!err.empty()) return false;
                    i += len;
                }
            }
        }
        return true;
    }
};

Tokenizer::Tokenizer() : impl_(new Impl) {}
Tokenizer::~Tokenizer() { delete impl_; }

bool Tokenizer::load(const std::string& path, std::string& err) {
    std::string text;
    if (!read_file(path, text)) {
        err = "cannot read " + path;
        return false;
    }
    s1json::Value j;
    if (!s1json::parse(text, j, err)) {
        err = "tokenizer.json: " + err;
        return false;
    }
    auto fail = [&](const std::string& what) {
        err = "tokenizer.json: " + what;
        return false;
    };
    // added tokens
    if (const auto* at = j.get("added_tokens")) {
        if (!at->is_arr()) return fail("added_tokens must be an array");
        for (const auto& a : at->arr) {
            const auto* content = a.get("content");
            const auto* id = a.get("id");
            if (!content || !content->is_str() || !id || id->kind != s1json::Value::INT) return fail("bad added token");
            for (const char* flag : {"lstrip", "rstrip", "single_word"}) {
                const auto* f = a.get(flag);
                if (f && f->kind == s1json::Value::BOOL && f->b) return fail(std::string("added token ") + flag);
            }
            const auto* norm = a.get("normalized");
            impl_->added.push_back({content->s, (uint32_t)id->i, norm && norm->kind == s1json::Value::BOOL && norm->b});
        }
    }
    // normalizer: none or NFC (alone or as the only member of a sequence)
    if (const auto* n = j.get("normalizer"); n && !n->is_null()) {
        const auto* type = n->get("type");
        const s1json::Value* one = n;
        if (type && type->s == "Sequence") {
            const auto* list = n->get("normalizers");
            if (!list || !list->is_arr() || list->arr.size() != 1) return fail("unsupported normalizer");
            one = &list->arr[0];
            type = one->get("type");
        }
        if (!type || type->s != "NFC") return fail("unsupported normalizer");
        impl_->nfc = true;
    }
    // pre-tokenizer: Split on the Qwen2 pattern (isolated), then ByteLevel without its regex;
    // or WhitespaceSplit (word-level tokenizers)
    const auto* pre = j.get("pre_tokenizer");
    const bool whitespace = pre && pre->get("type") && pre->get("type")->s == "WhitespaceSplit";
    if (!whitespace) {
        const auto* p = pre;
        const auto* list = p ? p->get("pretokenizers") : nullptr;
        if (!p || !list || !list->is_arr() || list->arr.size() != 2) return fail("unsupported pre-tokenizer");
        const auto& split = list->arr[0];
        const auto& bl = list->arr[1];
        const auto* st = split.get("type");
        const auto* pat = split.get("pattern");
        const auto* rx = pat ? pat->get("Regex") : nullptr;
        const auto* beh = split.get("behavior");
        const auto* inv = split.get("invert");
        if (!st || st->s != "Split" || !rx || rx->s != kQwenPattern || !beh || beh->s != "Isolated" ||
            (inv && inv->kind == s1json::Value::BOOL && inv->b))
            return fail("unsupported pre-tokenizer split");
        const auto* bt = bl.get("type");
        const auto* ur = bl.get("use_regex");
        const auto* aps = bl.get("add_prefix_space");
        if (!bt || bt->s != "ByteLevel" || (ur && ur->b) || (aps && aps->b))
            return fail("unsupported byte-level pre-tokenizer");
    }
    // post-processor: none, ByteLevel (adds nothing), or a single-sequence TemplateProcessing
    if (const auto* pp = j.get("post_processor"); pp && !pp->is_null()) {
        const auto* t = pp->get("type");
        if (t && t->s == "TemplateProcessing") {
            const auto* single = pp->get("single");
            const auto* specials = pp->get("special_tokens");
            if (!single || !single->is_arr()) return fail("TemplateProcessing needs a single template");
            for (const auto& piece : single->arr) {
                if (const auto* sp = piece.get("SpecialToken")) {
                    const auto* name = sp->get("id");
                    const auto* entry = specials && name ? specials->get(name->s) : nullptr;
                    const auto* list = entry ? entry->get("ids") : nullptr;
                    if (!list || !list->is_arr()) return fail("template special token without ids");
                    for (const auto& id : list->arr) impl_->template_.push_back((long)id.i);
                } else if (const auto* sq = piece.get("Sequence")) {
                    const auto* id = sq->get("id");
                    if (!id || id->s != "A") return fail("template sequence must be A");
                    impl_->template_.push_back(-1);
                } else {
                    return fail("unsupported template piece");
                }
            }
        } else if (!t || t->s != "ByteLevel") {
            return fail("unsupported post-processor");
        }
    }
    const auto* m = j.get("model");
    if (whitespace) {  // word-level: a vocabulary of whole words and an unknown token
        if (!m || !m->get("type") || m->get("type")->s != "WordLevel") return fail("WhitespaceSplit needs WordLevel");
        const auto* vocab = m->get("vocab");
        if (!vocab || !vocab->is_obj()) return fail("WordLevel needs a vocab");
        for (const auto& kv : vocab->obj) impl_->vocab[kv.first] = (uint32_t)kv.second.i;
        if (const auto* u = m->get("unk_token"); u && u->is_str()) {
            auto it = impl_->vocab.find(u->s);
            if (it == impl_->vocab.end()) return fail("unk_token not in the vocab");
            impl_->unk = it->second;
        }
        impl_->word_level = true;
        return true;
    }
    // model: byte-level BPE without unknown-token or byte fallbacks or affixes
    if (!m || !m->get("type") || m->get("type")->s != "BPE") return fail("model must be BPE");
    for (const char* k : {"dropout", "unk_token", "continuing_subword_prefix", "end_of_word_suffix"}) {
        const auto* v = m->get(k);
        if (v && !v->is_null()) return fail(std::string("unsupported BPE ") + k);
    }
    if (const auto* bf = m->get("byte_fallback"); bf && bf->b) return fail("unsupported BPE byte_fallback");
    if (const auto* im = m->get("ignore_merges")) impl_->ignore_merges = im->kind == s1json::Value::BOOL && im->b;
    const auto* vocab = m->get("vocab");
    const auto* merges = m->get("merges");
    if (!vocab || !vocab->is_obj() || !merges || !merges->is_arr()) return fail("BPE needs vocab and merges");
    for (const auto& kv : vocab->obj) {
        if (kv.second.kind != s1json::Value::INT) return fail("vocab ids must be integers");
        impl_->vocab[kv.first] = (uint32_t)kv.second.i;
    }
    uint32_t rank = 0;
    for (const auto& mg : merges->arr) {
        std::string a, b;
        if (mg.is_arr() && mg.arr.size() == 2 && mg.arr[0].is_str() && mg.arr[1].is_str()) {
            a = mg.arr[0].s;
            b = mg.arr[1].s;
        } else if (mg.is_str() && mg.s.find(' ') != std::string::npos) {
            a = mg.s.substr(0, mg.s.find(' '));
            b = mg.s.substr(mg.s.find(' ') + 1);
        } else {
            return fail("bad merge");
        }
        impl_->ranks.emplace(a + '\x01' + b, rank++);
    }
    return true;
}

bool Tokenizer::encode(const std::string& text, std::vector<uint32_t>& ids, std::string& err) const {
    ids.clear();
    err.clear();
    if (impl_->template_.empty()) return impl_->encode(text, ids, err);
    std::vector<uint32_t> seq;
    if (!impl_->encode(text, seq, err)) return false;
    for (long t : impl_->template_) {
        if (t < 0) ids.insert(ids.end(), seq.begin(), seq.end());
        else ids.push_back((uint32_t)t);
    }
    return true;
}

std::string trim(const std::string& s) {
    const std::vector<uint32_t> c = to_cps(s);
    size_t a = 0, b = c.size();
    while (a < b && is_space(c[a])) a++;
    while (b > a && is_space(c[b - 1])) b--;
    return to_utf8(c, a, b);
}

}  // namespace s1tok
