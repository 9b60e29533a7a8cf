// Worker-side request processing of the decision model: the request contract (questions
// -> candidate prompts), tokenization of every candidate, and the calibrated response.
// Restates the reference's open_jev worker:
//   contract::compile / answer (src/models/open_jev/native/src/contract.rs:98-289),
//   Processor::prepare, encode_questions and ResponseContext::finish
//   (src/models/open_jev/native/src/processing.rs:65-200),
//   the request JSON rules of src/models/qwen3_5/native/src/json.rs (pyjson.hpp).
// Candidates are tokenized on a pool of host threads (the reference batches chunks of 16
// through the tokenizer's own thread pool) and validated in request order, so the first
// over-long candidate is the one reported whatever the threads' timing.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "pyjson.hpp"
#include "s1_processing.h"
#include "tokenizer.hpp"

namespace {

thread_local std::string g_error;

struct Checkpoint {
    const char* name;
    const char* model_id;
    const char* base_revision;
    const char* alias;
};

// The pinned checkpoints the worker serves (contract.rs:28-51).
const Checkpoint kCheckpoints[] = {
    {"Open-Jev-27B-v1.1", "Qwen/Qwen3.8-27B", "1d4bf0f2ff6012fd82039f2fa52739d0dd7c60c0", "open-jev-27b-v1.1"},
    {"Open-Jev-9B", "Qwen/Qwen3.5-9B", "c202236235762e1c871ad0ccb60c8ee5ba337b9a", "open-jev-9b"},
};

enum class Kind { Choice, Score, Noul };

struct Question {
    std::string id;
    Kind kind;
    std::vector<std::string> keys;
    std::vector<std::string> prompts;
    s1json::Value legend;  // Score: {"0": level, ...}
};

struct Processor {
    s1tok::Tokenizer tokenizer;
    const Checkpoint* checkpoint = &kCheckpoints[0];
    std::string prefix, suffix;
    double temperature = 1.0;
    size_t max_length = 4096;
    bool parallel = true;
};

struct Prepared {
    const Checkpoint* checkpoint;
    std::vector<Question> questions;
    std::vector<std::vector<std::vector<uint32_t>>> ids;
    size_t input_tokens = 0, candidates = 0;
    double temperature;
    size_t max_length;
    std::chrono::steady_clock::time_point start;
};

bool err(const std::string& what) {
    g_error = what;
    return false;
}

// Python json.dumps(ensure_ascii=False, sort_keys=True), or the string itself.
std::string render(const s1json::Value& v) { return v.is_str() ? v.s : s1json::dumps(v, true); }

bool description(const s1json::Value& v, std::string& out) {
    if (!(v.is_str() || v.is_obj() || v.is_arr()))
        return err("instructions and descriptions must be text, an object, or an array");
    out = render(v);
    return true;
}

bool serves(const Checkpoint* c, const std::string& model) {
    return model == c->model_id || model == "open-jev" || model == "jev-latest" || model == c->alias;
}

bool compile(const std::string& raw, const Checkpoint* ck, std::vector<Question>& result) {
    s1json::Value request;
    std::string perr;
    if (!s1json::parse(raw, request, perr)) return err("request body is not valid JSON: " + perr);
    if (!request.is_obj()) return err("request body must be a JSON object");
    const s1json::Value* model = request.get("model");
    if (model && !model->is_null() && !(model->is_str() && serves(ck, model->s)))
        return err("requested model is not loaded");
    const s1json::Value* state = request.get("state");
    if (!state) return err("request requires state");
    if (!(state->is_str() || state->is_obj() || state->is_arr()))
        return err("state must be text, a JSON object, or an array");
    const s1json::Value* questions = request.get("questions");
    if (!questions || !questions->is_obj()) return err("questions must be an object");
    if (questions->obj.empty() || questions->obj.size() > 4096)
        return err("questions must be nonempty and within the server question limit");
    size_t candidates = 0;
    const s1json::Value null;
    for (const auto& [id, def] : questions->obj) {
        if (!def.is_obj()) return err("question definition must be an object");
        const s1json::Value* ins = def.get("instructions");
        std::string instructions;
        if (!description(ins ? *ins : null, instructions)) return false;
        const s1json::Value* crit = def.get("criteria");
        const s1json::Value& criteria = crit ? *crit : null;
        const s1json::Value* type = def.get("type");
        Question q;
        q.id = id;
        std::vector<std::string> options;
        if (type && type->is_str() && type->s == "choice") {
            if (!criteria.is_obj()) return err("Choice requires an object");
            if (criteria.obj.empty() || criteria.obj.size() > 255)
                return err("Choice requires between 1 and 255 candidates");
            for (const auto& [name, value] : criteria.obj) {
                if (value.is_null()) {
                    options.push_back(name);
                } else {
                    std::string d;
                    if (!description(value, d)) return false;
                    options.push_back(name + ": " + d);
                }
                q.keys.push_back(name);
            }
            q.kind = Kind::Choice;
        } else if (type && type->is_str() && type->s == "score") {
            if (!criteria.is_arr()) return err("Score requires an array");
            if (criteria.arr.size() < 2 || criteria.arr.size() > 10)
                return err("Score requires 2 to 10 descriptive levels");
            q.legend.kind = s1json::Value::OBJ;
            for (size_t i = 0; i < criteria.arr.size(); i++) {
                q.keys.push_back(std::to_string(i));
                q.legend.obj.emplace_back(std::to_string(i), criteria.arr[i]);
                std::string d;
                if (!description(criteria.arr[i], d)) return false;
                options.push_back(d);
            }
            q.kind = Kind::Score;
        } else if (type && type->is_str() && type->s == "noul") {
            if (!criteria.is_null()) {
                if (!criteria.is_obj() || criteria.obj.size() != 2 || !criteria.get("true") || !criteria.get("false"))
                    return err("Noul criteria must contain true and false descriptions");
                std::string t, f;
                if (!description(*criteria.get("true"), t) || !description(*criteria.get("false"), f)) return false;
                instructions += "\nYes means: " + t + "\nNo means: " + f;
            }
            q.kind = Kind::Noul;
            q.keys = {"false", "true"};
        } else {
            return err("question type must be choice, score, or noul");
        }
        const std::string prefix = "Context:\n" + render(*state) + "\n\nQuestion: " + instructions + "\n";
        if (q.kind == Kind::Noul) {
            q.prompts.push_back(prefix + "Is the answer to this question yes? Answer Yes or No.");
        } else {
            for (const auto& o : options)
                q.prompts.push_back(prefix + "Proposed answer: " + o +
                                    "\nIs this proposed answer correct? Answer Yes or No.");
        }
        candidates += q.prompts.size();
        if (candidates > 65536) return err("request exceeds the candidate limit");
        result.push_back(std::move(q));
    }
    return true;
}

bool encode_all(const Processor& p, Prepared& r) {
    struct Job {
        size_t q, c;
        std::string text;
        std::vector<uint32_t> ids;
        std::string error;
        bool ok = false;
    };
    std::vector<Job> jobs;
    for (size_t qi = 0; qi < r.questions.size(); qi++)
        for (size_t ci = 0; ci < r.questions[qi].prompts.size(); ci++)
            jobs.push_back({qi, ci, p.prefix + s1tok::trim(r.questions[qi].prompts[ci]) + p.suffix, {}, {}, false});
    auto run = [&](size_t j) { jobs[j].ok = p.tokenizer.encode(jobs[j].text, jobs[j].ids, jobs[j].error); };
    const size_t workers = p.parallel ? std::min<size_t>(std::max(1u, std::thread::hardware_concurrency()), 32) : 1;
    if (workers <= 1 || jobs.size() < 2) {
        for (size_t j = 0; j < jobs.size(); j++) run(j);
    } else {
        std::atomic<size_t> next{0};
        std::vector<std::thread> pool;
        for (size_t w = 0; w < std::min(workers, jobs.size()); w++)
            pool.emplace_back([&] {
                for (size_t j = next++; j < jobs.size(); j = next++) run(j);
            });
        for (auto& t : pool) t.join();
    }
    r.ids.assign(r.questions.size(), {});
    for (size_t qi = 0; qi < r.questions.size(); qi++) r.ids[qi].resize(r.questions[qi].prompts.size());
    for (auto& j : jobs) {  // request order: the first failing candidate is the one reported
        if (!j.ok) return err(j.error);
        if (j.ids.size() > p.max_length)
            return err("question " + r.questions[j.q].id + ": " + std::to_string(j.ids.size()) +
                       " tokens exceeds max_length=" + std::to_string(p.max_length) + "; no silent truncation");
        r.input_tokens += j.ids.size();
        r.candidates++;
        r.ids[j.q][j.c] = std::move(j.ids);
    }
    return true;
}

s1json::Value num(double x) {
    s1json::Value v;
    v.kind = s1json::Value::FLOAT;
    v.f = x;
    return v;
}
s1json::Value str(const std::string& s) {
    s1json::Value v;
    v.kind = s1json::Value::STR;
    v.s = s;
    return v;
}
s1json::Value integer(long long i) {
    s1json::Value v;
    v.kind = s1json::Value::INT;
    v.i = i;
    return v;
}
s1json::Value boolean(bool b) {
    s1json::Value v;
    v.kind = s1json::Value::BOOL;
    v.b = b;
    return v;
}

// Calibrated normalisation across the complete question's candidates (contract.rs:226-289).
bool answer(const Question& q, const std::vector<float>& logits, double temperature, s1json::Value& out) {
    if (!(std::isfinite(temperature) && temperature > 0)) return err("invalid temperature");
    if (logits.size() != q.keys.size()) return err("invalid logits");
    for (float v : logits)
        if (!std::isfinite(v)) return err("invalid logits");
    float mx = -INFINITY;
    for (float v : logits) mx = std::max(mx, v);
    std::vector<double> probs;
    for (float v : logits) probs.push_back(std::exp(((double)v - (double)mx) / temperature));
    double total = 0;
    for (double pr : probs) total += pr;
    for (double& pr : probs) pr /= total;
    out = s1json::Value();
    out.kind = s1json::Value::OBJ;
    if (q.kind == Kind::Noul) {
        out.obj.emplace_back("type", str("noul"));
        out.obj.emplace_back("noul", num(probs[1]));
        return true;
    }
    size_t mode = 0;  // the first maximum wins ties
    for (size_t i = 1; i < probs.size(); i++)
        if (probs[i] > probs[mode]) mode = i;
    s1json::Value probabilities;
    probabilities.kind = s1json::Value::OBJ;
    for (size_t i = 0; i < probs.size(); i++) probabilities.obj.emplace_back(q.keys[i], num(probs[i]));
    const double n = (double)probs.size();
    if (q.kind == Kind::Choice) {
        const double confidence = probs.size() == 1 ? 1.0 : (probs[mode] - 1.0 / n) / (1.0 - 1.0 / n);
        out.obj.emplace_back("type", str("choice"));
        out.obj.emplace_back("choice", str(q.keys[mode]));
        out.obj.emplace_back("probabilities", probabilities);
        out.obj.emplace_back("confidence", num(confidence));
        return true;
    }
    double score = 0, distance = 0, uniform = 0;
    for (size_t i = 0; i < probs.size(); i++) {
        score += (double)i * probs[i];
        distance += (double)(i > mode ? i - mode : mode - i) * probs[i];
    }
    const double center = (n - 1.0) / 2.0;
    for (size_t i = 0; i < probs.size(); i++) uniform += std::fabs((double)i - center);
    uniform /= n;
    out.obj.emplace_back("type", str("score"));
    out.obj.emplace_back("score", num(score));
    out.obj.emplace_back("probabilities", probabilities);
    out.obj.emplace_back("confidence", num(std::max(0.0, 1.0 - distance / uniform)));
    out.obj.emplace_back("legend", q.legend);
    return true;
}

char* dup(const std::string& s) {
    char* out = static_cast<char*>(malloc(s.size() + 1));
    if (out) memcpy(out, s.c_str(), s.size() + 1);
    return out;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* s1_processing_error(void) { return g_error.c_str(); }

__attribute__((visibility("default"))) void* s1_tokenizer_load(const char* path) {
    if (!path) return nullptr;
    auto* t = new s1tok::Tokenizer;
    if (!t->load(path, g_error)) {
        delete t;
        return nullptr;
    }
    return t;
}

__attribute__((visibility("default"))) void s1_tokenizer_free(void* t) { delete static_cast<s1tok::Tokenizer*>(t); }

__attribute__((visibility("default"))) int s1_tokenizer_encode(void* t, const char* text, size_t len, uint32_t* ids,
                                                              size_t cap, size_t* count) {
    if (!t || (!text && len) || !count) return -1;
    std::vector<uint32_t> out;
    if (!static_cast<s1tok::Tokenizer*>(t)->encode(std::string(text ? text : "", len), out, g_error)) return -1;
    *count = out.size();
    if (out.size() > cap || (!ids && !out.empty())) return out.size() > cap ? 1 : -1;
    std::copy(out.begin(), out.end(), ids);
    return 0;
}

__attribute__((visibility("default"))) void* s1_processor_create(const char* tokenizer_json, const char* checkpoint,
                                                                const char* chat_prefix, const char* chat_suffix,
                                                                double temperature, size_t max_length, int parallel) {
    if (!tokenizer_json) return nullptr;
    auto p = std::make_unique<Processor>();
    if (!p->tokenizer.load(tokenizer_json, g_error)) return nullptr;
    p->checkpoint = nullptr;
    for (const auto& c : kCheckpoints)
        if (checkpoint && (strcmp(checkpoint, c.name) == 0 || strcmp(checkpoint, c.model_id) == 0))
            p->checkpoint = &c;
    if (!p->checkpoint) {
        g_error = "expected an Open-Jev-27B-v1.1 or Open-Jev-9B export";
        return nullptr;
    }
    p->prefix = chat_prefix ? chat_prefix : "";
    p->suffix = chat_suffix ? chat_suffix : "";
    p->temperature = temperature;
    p->max_length = max_length;
    p->parallel = parallel != 0;
    return p.release();
}

__attribute__((visibility("default"))) void s1_processor_free(void* p) { delete static_cast<Processor*>(p); }

__attribute__((visibility("default"))) int s1_processor_set(void* pp, size_t max_length, int parallel) {
    auto* p = static_cast<Processor*>(pp);
    if (!p) return -1;
    p->max_length = max_length;
    p->parallel = parallel != 0;
    return 0;
}

__attribute__((visibility("default"))) void* s1_processor_prepare(void* pp, const char* raw, size_t len) {
    auto* p = static_cast<Processor*>(pp);
    if (!p || (!raw && len)) return nullptr;
    auto r = std::make_unique<Prepared>();
    r->checkpoint = p->checkpoint;
    r->temperature = p->temperature;
    r->max_length = p->max_length;
    if (!compile(std::string(raw ? raw : "", len), p->checkpoint, r->questions)) return nullptr;
    r->start = std::chrono::steady_clock::now();
    if (!encode_all(*p, *r)) return nullptr;
    return r.release();
}

__attribute__((visibility("default"))) void s1_prepared_free(void* r) { delete static_cast<Prepared*>(r); }

__attribute__((visibility("default"))) size_t s1_prepared_questions(void* r) {
    return r ? static_cast<Prepared*>(r)->questions.size() : 0;
}

__attribute__((visibility("default"))) size_t s1_prepared_candidates(void* rp, size_t q) {
    auto* r = static_cast<Prepared*>(rp);
    return r && q < r->questions.size() ? r->questions[q].prompts.size() : 0;
}

__attribute__((visibility("default"))) const uint32_t* s1_prepared_ids(void* rp, size_t q, size_t c, size_t* count) {
    auto* r = static_cast<Prepared*>(rp);
    if (!r || q >= r->ids.size() || c >= r->ids[q].size() || !count) return nullptr;
    *count = r->ids[q][c].size();
    return r->ids[q][c].data();
}

__attribute__((visibility("default"))) const char* s1_prepared_prompt(void* rp, size_t q, size_t c) {
    auto* r = static_cast<Prepared*>(rp);
    if (!r || q >= r->questions.size() || c >= r->questions[q].prompts.size()) return nullptr;
    return r->questions[q].prompts[c].c_str();
}

__attribute__((visibility("default"))) char* s1_prepared_finish(void* rp, const float* logits, size_t n,
                                                              const char* policy, int shared, int across_questions,
                                                              long long saved_tokens) {
    auto* r = static_cast<Prepared*>(rp);
    if (!r || (!logits && n)) {
        g_error = "invalid logit rows";
        return nullptr;
    }
    // Noul questions score one candidate; its answer's logits are [false = 0, true = score]
    size_t need = 0;
    for (const auto& q : r->questions) need += q.prompts.size();
    if (n != need) {
        g_error = "invalid logit rows";
        return nullptr;
    }
    s1json::Value answers;
    answers.kind = s1json::Value::OBJ;
    size_t at = 0;
    for (const auto& q : r->questions) {
        std::vector<float> row(logits + at, logits + at + q.prompts.size());
        at += q.prompts.size();
        if (q.kind == Kind::Noul) row.insert(row.begin(), 0.0f);
        s1json::Value a;
        if (!answer(q, row, r->temperature, a)) return nullptr;
        answers.obj.emplace_back(q.id, a);
    }
    const double seconds =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - r->start).count();
    s1json::Value body, usage, meta, cache;
    body.kind = usage.kind = meta.kind = cache.kind = s1json::Value::OBJ;
    const bool used = shared != 0;
    cache.obj.emplace_back("policy", str(policy && *policy ? policy : "default"));
    cache.obj.emplace_back("enabled", boolean(used));
    cache.obj.emplace_back("scope", str(!used ? "none" : across_questions ? "across_questions" : "within_question"));
    cache.obj.emplace_back("saved_tokens", integer(saved_tokens));
    usage.obj.emplace_back("input_tokens", integer((long long)r->input_tokens));
    usage.obj.emplace_back("output_tokens", integer(0));
    meta.obj.emplace_back("method", str("native_merged_lora_decision_head"));
    meta.obj.emplace_back("temperature", num(r->temperature));
    meta.obj.emplace_back("candidate_sequences", integer((long long)r->candidates));
    meta.obj.emplace_back("inference_seconds", num(seconds));
    meta.obj.emplace_back("base_revision", str(r->checkpoint->base_revision));
    meta.obj.emplace_back("max_length", integer((long long)r->max_length));
    meta.obj.emplace_back("prefix_cache", cache);
    body.obj.emplace_back("model", str(r->checkpoint->model_id));
    body.obj.emplace_back("answers", answers);
    body.obj.emplace_back("usage", usage);
    body.obj.emplace_back("metadata", meta);
    return dup(s1json::dumps(body));
}

// The calibrated answer of one question from a full logit row (one per key: a Noul
// question's [false, true]), as contract::answer (contract.rs:226-289).
__attribute__((visibility("default"))) char* s1_prepared_answer(void* rp, size_t question, const float* logits,
                                                              size_t n, double temperature) {
    auto* r = static_cast<Prepared*>(rp);
    if (!r || question >= r->questions.size() || (!logits && n)) {
        g_error = "invalid arguments";
        return nullptr;
    }
    s1json::Value a;
    if (!answer(r->questions[question], std::vector<float>(logits, logits + n), temperature, a)) return nullptr;
    return dup(s1json::dumps(a));
}

__attribute__((visibility("default"))) void s1_string_free(char* s) { free(s); }

}  // extern "C"
