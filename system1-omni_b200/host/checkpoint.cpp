// Checkpoint loading of the C++ host: a Hugging Face Qwen3.5 language-model folder
// (config.json + model.safetensors or model.safetensors.index.json shards) and the
// Open-Jev export manifest (open_jev_export.json: the trained scorer head).
//
// Follows the reference's loader (src/models/qwen3_5/native/src/model.rs:96-226 for the
// configuration, :267-397 for the weights; src/models/open_jev/native/src/executor.rs and
// engine.rs:125-177 for the head): tensors under the "model.language_model.", "model." or
// empty prefix (the one holding embed_tokens.weight), bf16 everywhere except A_log and
// the GDN output-norm weight, which current HF folders store in fp32 and which are rounded
// once to bf16 (round to nearest even; non-finite values are an error). Each tensor is read
// from its file and handed to s1_model_set_weight under this host's parameter name, which
// places it in the stacked projection groups (and the gate/up interleave).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/s1_model.h"

namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, true/false/null) ----
struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;
    const Json* get(const std::string& k) const {
        if (kind != OBJ) return nullptr;
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
};

struct Parser {
    const std::string& s;
    size_t i = 0;
    bool ok = true;
    explicit Parser(const std::string& t) : s(t) {}
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) i++;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if (s.compare(i, n, w) == 0) {
            i += n;
            return true;
        }
        return false;
    }
    std::string string() {
        std::string out;
        if (s[i] != '"') {
            ok = false;
            return out;
        }
        i++;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\' && i < s.size()) {
                const char e = s[i++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {  // keep \uXXXX as UTF-8 (basic plane)
                        if (i + 4 > s.size()) {
                            ok = false;
                            return out;
                        }
                        const unsigned cp = (unsigned)strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                        i += 4;
                        if (cp < 0x80) {
                            out += (char)cp;
                        } else if (cp < 0x800) {
                            out += (char)(0xC0 | (cp >> 6));
                            out += (char)(0x80 | (cp & 0x3F));
                        } else {
                            out += (char)(0xE0 | (cp >> 12));
                            out += (char)(0x80 | ((cp >> 6) & 0x3F));
                            out += (char)(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i >= s.size()) ok = false;
        i++;
        return out;
    }
    Json value(int depth = 0) {
        Json v;
        ws();
        if (i >= s.size() || depth > 64) {
            ok = false;
            return v;
        }
        const char c = s[i];
        if (c == '{') {
            v.kind = Json::OBJ;
            i++;
            ws();
            if (i < s.size() && s[i] == '}') {
                i++;
                return v;
            }
            while (ok) {
                ws();
                std::string k = string();
                ws();
                if (i >= s.size() || s[i] != ':') {
                    ok = false;
                    break;
                }
                i++;
                v.obj[k] = value(depth + 1);
                ws();
                if (i < s.size() && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < s.size() && s[i] == '}') {
                    i++;
                    break;
                }
                ok = false;
            }
        } else if (c == '[') {
            v.kind = Json::ARR;
            i++;
            ws();
            if (i < s.size() && s[i] == ']') {
                i++;
                return v;
            }
            while (ok) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (i < s.size() && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < s.size() && s[i] == ']') {
                    i++;
                    break;
                }
                ok = false;
            }
        } else if (c == '"') {
            v.kind = Json::STR;
            v.str = string();
        } else if (lit("true")) {
            v.kind = Json::BOOL;
            v.b = true;
        } else if (lit("false")) {
            v.kind = Json::BOOL;
        } else if (lit("null")) {
            v.kind = Json::NUL;
        } else {
            char* end = nullptr;
            v.num = strtod(s.c_str() + i, &end);
            if (end == s.c_str() + i) {
                ok = false;
                return v;
            }
            v.kind = Json::NUM;
            i = (size_t)(end - s.c_str());
        }
        return v;
    }
};

bool parse_json(const std::string& text, Json& out) {
    Parser p(text);
    out = p.value();
    p.ws();
    return p.ok && p.i == text.size();
}

bool read_file(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

thread_local std::string g_error;
int fail(const std::string& msg) {
    g_error = msg;
    return -1;
}

// ---- safetensors ----
struct Entry {
    std::string file, hf, name, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0, data_start = 0;  // payload bytes [data_start + begin, data_start + end)
};

int read_header(const std::string& path, std::vector<Entry>& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail("cannot open " + path);
    uint64_t n = 0;
    f.read(reinterpret_cast<char*>(&n), 8);
    if (!f || n == 0 || n > (1ull << 30)) return fail("bad safetensors header in " + path);
    std::string text(n, '\0');
    f.read(&text[0], (std::streamsize)n);
    if (!f) return fail("short safetensors header in " + path);
    Json h;
    if (!parse_json(text, h) || h.kind != Json::OBJ) return fail("unreadable safetensors header in " + path);
    for (const auto& kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const Json& t = kv.second;
        const Json *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
        if (!dt || !sh || !off || off->arr.size() != 2) return fail("bad entry " + kv.first + " in " + path);
        Entry e;
        e.file = path;
        e.hf = kv.first;
        e.dtype = dt->str;
        for (const Json& d : sh->arr) e.shape.push_back((int64_t)d.num);
        e.begin = (uint64_t)off->arr[0].num;
        e.end = (uint64_t)off->arr[1].num;
        e.data_start = 8 + n;
        out.push_back(e);
    }
    return 0;
}

// HF name (prefix removed) -> this host's parameter name, "" when not a language-model weight.
std::string map_name(const std::string& hf) {
    if (hf == "embed_tokens.weight") return "embed";
    if (hf == "norm.weight") return "final_norm";
    if (hf.compare(0, 7, "layers.") != 0) return "";
    const size_t dot = hf.find('.', 7);
    if (dot == std::string::npos) return "";
    const std::string layer = hf.substr(7, dot - 7), rest = hf.substr(dot + 1);
    for (char c : layer)
        if (c < '0' || c > '9') return "";
    static const std::map<std::string, std::string> leaf = {
        {"input_layernorm.weight", "input_norm"},
        {"post_attention_layernorm.weight", "post_norm"},
        {"mlp.gate_proj.weight", "gate"},
        {"mlp.up_proj.weight", "up"},
        {"mlp.down_proj.weight", "down"},
        {"linear_attn.in_proj_qkv.weight", "in_qkv"},
        {"linear_attn.in_proj_z.weight", "in_z"},
        {"linear_attn.in_proj_b.weight", "in_b"},
        {"linear_attn.in_proj_a.weight", "in_a"},
        {"linear_attn.conv1d.weight", "conv"},
        {"linear_attn.A_log", "A_log"},
        {"linear_attn.dt_bias", "dt_bias"},
        {"linear_attn.norm.weight", "norm"},
        {"linear_attn.out_proj.weight", "out"},
        {"self_attn.q_proj.weight", "q"},
        {"self_attn.k_proj.weight", "k"},
        {"self_attn.v_proj.weight", "v"},
        {"self_attn.o_proj.weight", "o"},
        {"self_attn.q_norm.weight", "q_norm"},
        {"self_attn.k_norm.weight", "k_norm"},
    };
    auto it = leaf.find(rest);
    return it == leaf.end() ? "" : "l" + layer + "." + it->second;
}

bool fp32_allowed(const std::string& name) {
    const size_t dot = name.rfind('.');
    const std::string leaf = dot == std::string::npos ? name : name.substr(dot + 1);
    return leaf == "A_log" || leaf == "norm";
}

// The language-model tensors of a checkpoint folder, mapped and checked (dtype rules).
int plan(const std::string& dir, std::vector<Entry>& out) {
    std::vector<std::string> files;
    std::string index;
    if (read_file(dir + "/model.safetensors.index.json", index)) {
        Json j;
        if (!parse_json(index, j) || !j.get("weight_map")) return fail("unreadable model.safetensors.index.json");
        std::set<std::string> uniq;
        for (const auto& kv : j.get("weight_map")->obj) uniq.insert(kv.second.str);
        files.assign(uniq.begin(), uniq.end());
    } else {
        files.push_back("model.safetensors");
    }
    std::vector<Entry> all;
    for (const auto& f : files)
        if (read_header(dir + "/" + f, all)) return -1;
    std::string prefix;
    bool found = false;
    for (const char* p : {"model.language_model.", "model.", ""}) {
        for (const Entry& e : all)
            if (e.hf == std::string(p) + "embed_tokens.weight") {
                prefix = p;
                found = true;
                break;
            }
        if (found) break;
    }
    if (!found) return fail("no embed_tokens.weight in the checkpoint");
    for (Entry& e : all) {
        if (e.hf.compare(0, prefix.size(), prefix) != 0) continue;
        e.name = map_name(e.hf.substr(prefix.size()));
        if (e.name.empty()) continue;
        if (e.dtype != "BF16" && !(e.dtype == "F32" && fp32_allowed(e.name)))
            return fail(e.hf + " is " + e.dtype + ", not bfloat16");
        out.push_back(e);
    }
    return 0;
}

// Shape of every weight the model's configuration holds (HF row-major shapes).
std::map<std::string, std::vector<int64_t>> expected_shapes(const s1_config& c) {
    const int64_t H = c.hidden, I = c.intermediate, hv = c.lin_v_heads, kd = (int64_t)c.lin_k_heads * c.lin_k_dim,
                  vd = (int64_t)c.lin_v_heads * c.lin_v_dim, conv = 2 * kd + vd, hd = c.head_dim;
    std::map<std::string, std::vector<int64_t>> s;
    s["embed"] = {c.vocab, H};
    s["final_norm"] = {H};
    for (int i = 0; i < c.n_layers; i++) {
        const std::string p = "l" + std::to_string(i) + ".";
        s[p + "input_norm"] = {H};
        s[p + "post_norm"] = {H};
        s[p + "gate"] = {I, H};
        s[p + "up"] = {I, H};
        s[p + "down"] = {H, I};
        if (c.layer_types[i] == 0) {
            s[p + "in_qkv"] = {conv, H};
            s[p + "in_z"] = {vd, H};
            s[p + "in_b"] = {hv, H};
            s[p + "in_a"] = {hv, H};
            s[p + "conv"] = {conv, 1, 4};
            s[p + "A_log"] = {hv};
            s[p + "dt_bias"] = {hv};
            s[p + "norm"] = {c.lin_v_dim};
            s[p + "out"] = {H, vd};
        } else {
            s[p + "q"] = {2 * c.heads * hd, H};
            s[p + "k"] = {c.kv_heads * hd, H};
            s[p + "v"] = {c.kv_heads * hd, H};
            s[p + "o"] = {H, c.heads * hd};
            s[p + "q_norm"] = {hd};
            s[p + "k_norm"] = {hd};
        }
    }
    return s;
}

std::string shape_text(const std::vector<int64_t>& v) {
    std::string t = "[";
    for (size_t d = 0; d < v.size(); d++) t += (d ? ", " : "") + std::to_string(v[d]);
    return t + "]";
}

// Entries against the configuration: shapes (conv also as [C, 4]), payload sizes, and
// every expected weight present exactly once.
int check_plan(const std::vector<Entry>& entries, const s1_config& c) {
    auto want = expected_shapes(c);
    std::set<std::string> seen;
    for (const Entry& e : entries) {
        auto it = want.find(e.name);
        if (it == want.end()) return fail(e.hf + " has no place in the model's configuration");
        if (!seen.insert(e.name).second) return fail(e.hf + " appears twice");
        std::vector<int64_t> got = e.shape;
        if (it->second.size() == 3 && got.size() == 2) got.insert(got.begin() + 1, 1);
        if (got != it->second)
            return fail(e.hf + " has shape " + shape_text(e.shape) + ", the model expects " + shape_text(it->second));
        uint64_t elems = 1;
        for (int64_t d : e.shape) elems *= (uint64_t)d;
        if (e.end < e.begin || e.end - e.begin != elems * (e.dtype == "F32" ? 4 : 2))
            return fail(e.hf + ": payload size does not match its shape");
    }
    for (const auto& kv : want)
        if (!seen.count(kv.first)) return fail("the checkpoint lacks " + kv.first);
    return 0;
}

uint16_t bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

int set_head(void* model, const Json& manifest, int labels, int hidden) {
    const Json *w = manifest.get("head_weight"), *b = manifest.get("head_bias");
    if (!w || !b) return fail("open_jev_export.json has no head_weight / head_bias");
    std::vector<float> W, B;
    if (w->kind == Json::ARR && !w->arr.empty() && w->arr[0].kind == Json::ARR) {
        for (const Json& row : w->arr)
            for (const Json& x : row.arr) W.push_back((float)x.num);
    } else {
        for (const Json& x : w->arr) W.push_back((float)x.num);
    }
    if (b->kind == Json::ARR)
        for (const Json& x : b->arr) B.push_back((float)x.num);
    else
        B.push_back((float)b->num);
    if ((int)W.size() != labels * hidden || (int)B.size() != labels)
        return fail("head shape does not match the model (" + std::to_string(labels) + " x " +
                    std::to_string(hidden) + ")");
    for (float x : W)
        if (!std::isfinite(x)) return fail("non-finite scorer head");
    for (float x : B)
        if (!std::isfinite(x)) return fail("non-finite scorer head");
    if (s1_model_set_weight(model, "head_w", W.data(), W.size() * 4)) return fail(s1_model_error(model));
    if (s1_model_set_weight(model, "head_b", B.data(), B.size() * 4)) return fail(s1_model_error(model));
    return 0;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* s1_checkpoint_error(void) { return g_error.c_str(); }

__attribute__((visibility("default"))) int s1_config_from_hf(const char* config_json, s1_config* out,
                                                            int* layer_types, int max_layers) {
    if (!config_json || !out || !layer_types || max_layers <= 0) return fail("invalid argument");
    std::string text;
    if (!read_file(config_json, text)) return fail(std::string("cannot read ") + config_json);
    Json root;
    if (!parse_json(text, root) || root.kind != Json::OBJ) return fail("unreadable config.json");
    const Json* c = root.get("text_config") ? root.get("text_config") : &root;
    auto num = [&](const char* k, double dflt, bool required) -> double {
        const Json* v = c->get(k);
        if (v && v->kind == Json::NUM) return v->num;
        if (required) g_error = std::string("config.json has no ") + k;
        return required ? NAN : dflt;
    };
    s1_config cfg{};
    cfg.hidden = (int)num("hidden_size", 0, true);
    cfg.intermediate = (int)num("intermediate_size", 0, true);
    cfg.n_layers = (int)num("num_hidden_layers", 0, true);
    cfg.lin_k_heads = (int)num("linear_num_key_heads", 0, true);
    cfg.lin_v_heads = (int)num("linear_num_value_heads", 0, true);
    cfg.lin_k_dim = (int)num("linear_key_head_dim", 128, false);
    cfg.lin_v_dim = (int)num("linear_value_head_dim", 128, false);
    cfg.heads = (int)num("num_attention_heads", 0, true);
    cfg.kv_heads = (int)num("num_key_value_heads", 0, true);
    cfg.head_dim = (int)num("head_dim", 256, false);
    cfg.vocab = (int)num("vocab_size", 0, true);
    cfg.eps = (float)num("rms_norm_eps", 1e-6, false);
    if (cfg.hidden <= 0 || cfg.intermediate <= 0 || cfg.n_layers <= 0 || cfg.heads <= 0 || cfg.kv_heads <= 0 ||
        cfg.lin_k_heads <= 0 || cfg.lin_v_heads <= 0 || cfg.vocab <= 0)
        return fail(g_error.empty() ? "config.json: missing or invalid sizes" : g_error);
    if ((int)num("linear_conv_kernel_dim", 4, false) != 4) return fail("linear_conv_kernel_dim must be 4");
    // rotary: rope_parameters {rope_theta, partial_rotary_factor} or the same keys at top level
    const Json* rp = c->get("rope_parameters") ? c->get("rope_parameters") : c->get("rope_scaling");
    auto rope = [&](const char* k, double dflt) {
        if (rp && rp->get(k) && rp->get(k)->kind == Json::NUM) return rp->get(k)->num;
        const Json* v = c->get(k);
        return v && v->kind == Json::NUM ? v->num : dflt;
    };
    cfg.theta = rope("rope_theta", 1e7);
    const double factor = rope("partial_rotary_factor", 0.25);
    cfg.rotary_half = (int)std::lround(cfg.head_dim * factor / 2);
    if (cfg.n_layers > max_layers) return fail("more layers than the caller's layer_types buffer");
    const Json* lt = c->get("layer_types");
    if (lt && lt->kind == Json::ARR) {
        if ((int)lt->arr.size() != cfg.n_layers) return fail("layer_types does not have num_hidden_layers entries");
        for (int i = 0; i < cfg.n_layers; i++) {
            const std::string& t = lt->arr[i].str;
            if (t == "linear_attention")
                layer_types[i] = 0;
            else if (t == "full_attention")
                layer_types[i] = 1;
            else
                return fail("unknown layer type " + t);
        }
    } else {
        const int interval = (int)num("full_attention_interval", 4, false);
        for (int i = 0; i < cfg.n_layers; i++) layer_types[i] = (i + 1) % interval == 0 ? 1 : 0;
    }
    cfg.layer_types = layer_types;
    cfg.labels = 1;
    *out = cfg;
    return 0;
}

// One line per mapped tensor: "<name> <hf name> <dtype> <d0>x<d1>..."; returns the bytes
// the full listing needs (including the terminating zero), or -1.
__attribute__((visibility("default"))) long s1_checkpoint_list(const char* dir, char* out, size_t cap) {
    if (!dir) return fail("invalid argument");
    std::vector<Entry> entries;
    if (plan(dir, entries)) return -1;
    std::string text;
    for (const Entry& e : entries) {
        text += e.name + " " + e.hf + " " + e.dtype + " ";
        for (size_t d = 0; d < e.shape.size(); d++) text += (d ? "x" : "") + std::to_string(e.shape[d]);
        text += "\n";
    }
    if (out && cap > 0) {
        const size_t n = std::min(cap - 1, text.size());
        memcpy(out, text.data(), n);
        out[n] = 0;
    }
    return (long)text.size() + 1;
}

__attribute__((visibility("default"))) int s1_checkpoint_check(const char* dir, const s1_config* cfg) {
    if (!dir || !cfg || !cfg->layer_types || cfg->n_layers <= 0) return fail("invalid argument");
    std::vector<Entry> entries;
    if (plan(dir, entries)) return -1;
    return check_plan(entries, *cfg);
}

__attribute__((visibility("default"))) int s1_model_load_checkpoint(void* model, const char* dir) {
    if (!model || !dir) return fail("invalid argument");
    std::vector<Entry> entries;
    if (plan(dir, entries)) return -1;
    s1_config cfg{};
    if (s1_model_get_config(model, &cfg)) return fail("invalid model");
    if (check_plan(entries, cfg)) return -1;
    std::vector<char> buf;
    std::vector<uint16_t> conv;
    for (const Entry& e : entries) {
        std::ifstream f(e.file, std::ios::binary);
        const uint64_t n = e.end - e.begin;
        buf.resize(n);
        f.seekg((std::streamoff)(e.data_start + e.begin));
        f.read(buf.data(), (std::streamsize)n);
        if (!f) return fail("short read of " + e.hf);
        const void* data = buf.data();
        size_t bytes = n;
        if (e.dtype == "F32") {  // A_log / GDN norm: rounded once to bf16
            conv.resize(n / 4);
            for (size_t i = 0; i < n / 4; i++) {
                float x;
                memcpy(&x, buf.data() + 4 * i, 4);
                if (!std::isfinite(x)) return fail("non-finite " + e.hf);
                conv[i] = bf16_rne(x);
            }
            data = conv.data();
            bytes = conv.size() * 2;
        }
        if (s1_model_set_weight(model, e.name.c_str(), data, bytes))
            return fail(e.hf + ": " + s1_model_error(model));
    }
    return 0;
}

__attribute__((visibility("default"))) int s1_model_load_head(void* model, const char* manifest_json, int labels,
                                                             int hidden) {
    if (!model || !manifest_json) return fail("invalid argument");
    std::string text;
    if (!read_file(manifest_json, text)) return fail(std::string("cannot read ") + manifest_json);
    Json m;
    if (!parse_json(text, m) || m.kind != Json::OBJ) return fail("unreadable export manifest");
    return set_head(model, m, labels, hidden);
}

}  // extern "C"
