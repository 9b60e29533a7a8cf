// libs1_model.so: the Qwen3.5 hybrid decision-model prefill host (C++ above the cs1_* ABI).
//
// Mirrors the reference's Rust Model (src/models/qwen3_5/native/src/model.rs) for the
// decision path: one weight arena with the projection groups stacked (qkv|z|b|a,
// q|k|v, gate|up; model.rs:251-265), per-pack scratch, the layer loop of
// run_with_attention (model.rs:3178-3727), packed candidates with per-sequence
// positions and state (model.rs:1548-1632), the shared-prefix fork of GDN state, conv
// history and attention K/V (model.rs:1664-1907), the final-token scorer head
// (open_jev executor.rs:59-71) and CUDA graphs keyed by the length vector
// (model.rs:1583-1614). The cs1 library is bound by dlopen with the ABI-9 check,
// required and optional symbols, like the reference's loader (cuda.rs:279-383, 495-698);
// additive symbols of this build (fused projections, packed conv/GDN, scorer head)
// are used when present, otherwise the reference's per-sequence call sequence runs.
#include "s1_model.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <map>
#include <string>
#include <type_traits>
#include <vector>

namespace {

thread_local std::string g_create_error;

// ---------------------------------------------------------------- the ABI ----
struct Api {
    void* handle = nullptr;
    uint32_t (*abi_version)();
    const char* (*error_string)(int);
    int (*set_device)(int);
    int (*malloc_)(void**, size_t);
    int (*free_)(void*);
    int (*stream_create)(void**);
    int (*stream_sync)(void*);
    int (*stream_destroy)(void*);
    int (*graph_begin)(void*);
    int (*graph_end)(void*, void**);
    int (*graph_launch)(void*, void*);
    int (*graph_destroy)(void*);
    int (*upload)(void*, const void*, size_t, void*);
    int (*download)(void*, const void*, size_t, void*);
    int (*copy_dd)(void*, const void*, size_t, void*);
    int (*copy2d)(void*, size_t, const void*, size_t, size_t, size_t, void*);
    int (*embed)(const int32_t*, const void*, void*, int, int, void*);
    int (*rms_norm)(const void*, const void*, void*, int, int, float, void*);
    int (*add_rms_norm)(void*, const void*, const void*, void*, int, int, float, void*);
    int (*gated_rms_norm)(const void*, const void*, int, const void*, void*, int, int, int, float, void*);
    int (*gdn_conv)(const void*, int, const void*, void*, void*, void*, int, int, int, void*);
    int (*gdn_conv_prefix)(const void*, const void*, int, const void*, void*, void*, void*, int, int, int, void*);
    int (*gdn_gates)(const void*, const void*, int, const void*, const void*, void*, float*, int, int, void*);
    size_t (*gdn_workspace_floats)(int, int);
    int (*gdn_prefill)(const void*, const void*, const void*, const float*, const void*, void*, float*, int, int,
                       int, float, void*);
    int (*gdn_prefill_x)(const void*, const void*, const void*, const float*, const void*, void*, float*, int, int,
                         int, float, const void*, void*, void*);
    int (*attn_prep)(const void*, const void*, int, const void*, const void*, const void*, const void*, void*, void*,
                     void*, int, int, int, int, int, float, void*);
    int (*attention_gated)(const void*, const void*, const void*, int, const void*, void*, int, int, int, int, float,
                           void*);
    int (*silu_mul)(const void*, int, void*, int, int, void*);
    void* (*gemm_create)(size_t);
    void (*gemm_destroy)(void*);
    int (*gemm)(void*, const void*, const void*, void*, int, int, int, int, void*);
    // optional (reference)
    size_t (*gdn_batch_workspace_floats)(int, int, int) = nullptr;
    int (*gdn_prefill_batch)(const void*, const void*, const void*, const float*, const void*, void*, float*, size_t,
                             const size_t*, size_t, int, int, float, void*) = nullptr;
    int (*attention_gated_shared)(const void*, const void*, const void*, int, const void*, void*, const void*,
                                  const void*, int, int, int, int, int, float, void*) = nullptr;
    // additive (this build)
    int (*gdn_conv_batch)(const void*, const void*, int, const void*, void*, void*, void*, const size_t*, size_t, int,
                          int, void*) = nullptr;
    int (*gdn_prefill_batch_x)(const void*, const void*, const void*, const float*, const void*, void*, float*,
                               size_t, const size_t*, size_t, int, int, float, const void*, int, void*,
                               void*) = nullptr;
    int (*attention_gated_shared_batch)(const void*, const void*, const void*, int, const void*, void*, const void*,
                                        const void*, const size_t*, size_t, int, int, int, int, float,
                                        void*) = nullptr;
    int (*attention_gated_batch)(const void*, const void*, const void*, int, const void*, void*, const size_t*,
                                 size_t, int, int, int, float, void*) = nullptr;
    // the GDN front end (conv + SiLU + q/k inverse norms + gates in one launch) and the
    // prefill that takes its norms
    int (*gdn_front_batch)(const void*, const void*, int, const void*, void*, void*, void*, float*, float*,
                           const void*, const void*, const void*, const void*, void*, float*, int, const size_t*,
                           size_t, int, int, void*) = nullptr;
    int (*gdn_prefill_batch_xn)(const void*, const void*, const void*, const float*, const void*, const float*,
                                const float*, void*, const size_t*, size_t, int, int, float, const void*, int, void*,
                                void*) = nullptr;
    // most sequences one batched launch takes: 256 in this build, 16 in the reference (ops.h:83-94)
    int max_batch = 16;
    int (*gemm_residual)(void*, const void*, const void*, void*, int, int, int, int, void*) = nullptr;
    int (*gemm_swiglu)(void*, const void*, const void*, void*, int, int, int, int, void*) = nullptr;
    int (*head_score)(const void*, int, const int32_t*, int, const float*, const float*, int, int, float*,
                      void*) = nullptr;
    int (*fill_random)(void*, size_t, int, uint64_t, float, float, int, void*) = nullptr;
    // additive: the capacity path (device-resident batch descriptor; one graph per capacity)
    size_t (*batch_desc_bytes)() = nullptr;
    int (*batch_desc_pack)(const size_t*, size_t, void*, size_t) = nullptr;
    int (*embed_dyn)(const int32_t*, const void*, void*, int, int, const void*, void*) = nullptr;
    int (*rms_norm_dyn)(const void*, const void*, void*, int, int, float, const void*, void*) = nullptr;
    int (*gated_rms_norm_dyn)(const void*, const void*, int, const void*, void*, int, int, int, float, const void*,
                              void*) = nullptr;
    int (*gemm_dyn)(void*, const void*, const void*, void*, int, int, int, int, int, const void*, void*) = nullptr;
    int (*gdn_prefill_dyn)(const void*, const void*, const void*, const float*, const void*, const float*,
                           const float*, void*, int, int, int, int, float, const void*, int, void*, const void*,
                           void*) = nullptr;
    int (*gdn_front_dyn)(const void*, const void*, int, const void*, void*, void*, void*, float*, float*, const void*,
                         const void*, const void*, const void*, void*, float*, int, int, int, int, int, const void*,
                         void*) = nullptr;
    int (*attn_prep_dyn)(const void*, const void*, int, const void*, const void*, const void*, const void*, void*,
                         void*, void*, int, int, int, int, int, float, const void*, void*) = nullptr;
    int (*attention_dyn)(const void*, const void*, const void*, int, const void*, void*, const void*, const void*, int,
                         int, int, int, int, int, float, const void*, void*) = nullptr;
    int (*head_score_dyn)(const void*, int, const int32_t*, int, const float*, const float*, int, int, float*,
                          const void*, void*) = nullptr;
    int (*clear_tail_dyn)(void*, size_t, size_t, int, int, const void*, void*) = nullptr;
    bool has_dyn() const {
        return batch_desc_bytes && batch_desc_pack && clear_tail_dyn && gdn_front_dyn && embed_dyn && rms_norm_dyn &&
               gated_rms_norm_dyn && gemm_dyn && gdn_prefill_dyn && attn_prep_dyn && attention_dyn && head_score_dyn;
    }
};

template <typename F>
bool bind(void* h, const char* name, F& fn, bool required, std::string& err) {
    void* p = dlsym(h, name);
    if (!p && required) {
        err = std::string("missing required symbol ") + name;
        return false;
    }
    fn = reinterpret_cast<F>(p);
    return true;
}

// `spec` is "library" or "library;aux": symbols of this build that a library lacks
// (the random weight fill used by benchmarks) may come from the aux library.
bool load_api(const char* spec, Api& a, std::string& err) {
    std::string primary(spec), aux;
    const size_t semi = primary.find(';');
    if (semi != std::string::npos) {
        aux = primary.substr(semi + 1);
        primary = primary.substr(0, semi);
    }
    const char* path = primary.c_str();
    a.handle = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!a.handle) {
        err = std::string("dlopen failed: ") + dlerror();
        return false;
    }
    void* h = a.handle;
    if (!bind(h, "cs1_abi_version", a.abi_version, true, err)) return false;
    if (a.abi_version() != 9) {
        err = "cs1 ABI version " + std::to_string(a.abi_version()) + ", expected 9";
        return false;
    }
#define REQ(sym, field) \
    if (!bind(h, sym, a.field, true, err)) return false
    REQ("cs1_error_string", error_string);
    REQ("cs1_set_device", set_device);
    REQ("cs1_malloc", malloc_);
    REQ("cs1_free", free_);
    REQ("cs1_stream_create", stream_create);
    REQ("cs1_stream_sync", stream_sync);
    REQ("cs1_stream_destroy", stream_destroy);
    REQ("cs1_graph_begin", graph_begin);
    REQ("cs1_graph_end", graph_end);
    REQ("cs1_graph_launch", graph_launch);
    REQ("cs1_graph_destroy", graph_destroy);
    REQ("cs1_upload", upload);
    REQ("cs1_download", download);
    REQ("cs1_copy_dd", copy_dd);
    REQ("cs1_copy2d", copy2d);
    REQ("cs1_embed", embed);
    REQ("cs1_rms_norm", rms_norm);
    REQ("cs1_add_rms_norm", add_rms_norm);
    REQ("cs1_gated_rms_norm", gated_rms_norm);
    REQ("cs1_gdn_conv", gdn_conv);
    REQ("cs1_gdn_gates", gdn_gates);
    REQ("cs1_gdn_workspace_floats", gdn_workspace_floats);
    REQ("cs1_gdn_prefill", gdn_prefill);
    REQ("cs1_gdn_prefill_x", gdn_prefill_x);
    REQ("cs1_attn_prep", attn_prep);
    REQ("cs1_attention_gated", attention_gated);
    REQ("cs1_silu_mul", silu_mul);
    REQ("cs1_gemm_create", gemm_create);
    REQ("cs1_gemm_destroy", gemm_destroy);
    REQ("cs1_gemm", gemm);
#undef REQ
    bind(h, "cs1_gdn_conv_prefix", a.gdn_conv_prefix, false, err);
    bind(h, "cs1_gdn_batch_workspace_floats", a.gdn_batch_workspace_floats, false, err);
    bind(h, "cs1_gdn_prefill_batch", a.gdn_prefill_batch, false, err);
    bind(h, "cs1_attention_gated_shared", a.attention_gated_shared, false, err);
    bind(h, "cs1_gdn_conv_batch", a.gdn_conv_batch, false, err);
    bind(h, "cs1_gdn_prefill_batch_x", a.gdn_prefill_batch_x, false, err);
    bind(h, "cs1_attention_gated_shared_batch", a.attention_gated_shared_batch, false, err);
    bind(h, "cs1_attention_gated_batch", a.attention_gated_batch, false, err);
    bind(h, "cs1_gemm_residual", a.gemm_residual, false, err);
    bind(h, "cs1_gemm_swiglu", a.gemm_swiglu, false, err);
    bind(h, "cs1_head_score", a.head_score, false, err);
    bind(h, "cs1_fill_random", a.fill_random, false, err);
    bind(h, "cs1_batch_desc_bytes", a.batch_desc_bytes, false, err);
    bind(h, "cs1_batch_desc_pack", a.batch_desc_pack, false, err);
    bind(h, "cs1_embed_dyn", a.embed_dyn, false, err);
    bind(h, "cs1_rms_norm_dyn", a.rms_norm_dyn, false, err);
    bind(h, "cs1_gated_rms_norm_dyn", a.gated_rms_norm_dyn, false, err);
    bind(h, "cs1_gemm_dyn", a.gemm_dyn, false, err);
    bind(h, "cs1_gdn_prefill_dyn", a.gdn_prefill_dyn, false, err);
    bind(h, "cs1_attn_prep_dyn", a.attn_prep_dyn, false, err);
    bind(h, "cs1_attention_dyn", a.attention_dyn, false, err);
    bind(h, "cs1_head_score_dyn", a.head_score_dyn, false, err);
    bind(h, "cs1_clear_tail_dyn", a.clear_tail_dyn, false, err);
    bind(h, "cs1_gdn_front_dyn", a.gdn_front_dyn, false, err);
    bind(h, "cs1_gdn_front_batch", a.gdn_front_batch, false, err);
    bind(h, "cs1_gdn_prefill_batch_xn", a.gdn_prefill_batch_xn, false, err);
    a.max_batch = a.gdn_prefill_batch_x ? 256 : 16;
    if (!a.fill_random && !aux.empty()) {
        void* ah = dlopen(aux.c_str(), RTLD_NOW | RTLD_LOCAL);
        if (ah) bind(ah, "cs1_fill_random", a.fill_random, false, err);
    }
    return true;
}

// ------------------------------------------------------------------ model ----
constexpr size_t ALIGN = 256;
inline size_t up(size_t x) { return (x + ALIGN - 1) / ALIGN * ALIGN; }

struct Region {
    size_t off = 0;
    size_t elems = 0;
    bool f32 = false;
};

struct Layer {
    int type = 0;
    Region input_norm, post_norm;
    Region in_proj, conv, A_log, dt_bias, norm, out;  // GDN
    Region qkv, q_norm, k_norm, o;                    // attention
    Region gate_up, down;
};

struct Batch {
    std::vector<size_t> lengths;
    int prefix = 0;        // shared prefix length for suffix passes (positions start there)
    bool capture = false;  // capture prefix state (prefix pass)
    bool cp = false;       // context-parallel piece: prefix state from rank - 1, own state to rank + 1
    size_t rows = 0;
    // capacity path: launches sized for (cap_rows, cap_seqs), the batch read from the
    // device descriptor, so one captured graph serves every batch of that capacity
    bool dyn = false;
    int cap_rows = 0, cap_seqs = 0;
};

// NCCL, bound at run time (the library torch or the system provides) for the
// context-parallel prefill.
struct Nccl {
    void* lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

bool load_nccl(const char* path, Nccl& n, std::string& err) {
    n.lib = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!n.lib) {
        err = std::string("cannot load NCCL: ") + dlerror();
        return false;
    }
    bool ok = true;
    auto sym = [&](const char* name, auto& fn) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(n.lib, name));
        if (!fn) {
            ok = false;
            err = std::string("NCCL has no ") + name;
        }
    };
    sym("ncclGetUniqueId", n.get_unique_id);
    sym("ncclCommInitRank", n.comm_init_rank);
    sym("ncclCommDestroy", n.comm_destroy);
    sym("ncclSend", n.send);
    sym("ncclRecv", n.recv);
    sym("ncclAllGather", n.all_gather);
    sym("ncclGroupStart", n.group_start);
    sym("ncclGroupEnd", n.group_end);
    sym("ncclGetErrorString", n.error_string);
    return ok;
}

struct Model {
    Api api;
    s1_config cfg{};
    std::vector<int> types;
    int device = 0;
    void* stream = nullptr;
    void* gemm = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    std::vector<Layer> layers;
    Region embed, final_norm, head_w, head_b;
    bool fused = false;
    int cap_tokens = 0, cap_seqs = 0;
    // widths
    int conv = 0, kd = 0, vd = 0, gdn_in = 0, attn_q = 0, attn_in = 0, kvd = 0, qd = 0;
    // scratch
    uint8_t* scratch = nullptr;
    size_t s_ids, s_cos, s_sin, s_res, s_x, s_delta, s_gdn_in, s_lq, s_lk, s_lv, s_beta, s_g, s_lo, s_ln, s_attn_in,
        s_aq, s_agate, s_ak, s_ao, s_gate_up, s_act, s_rows, s_logits, s_ws, s_rnq, s_rnk;
    size_t ws_bytes = 0;
    // shared-prefix buffers (allocated on first use)
    uint8_t* prefix_buf = nullptr;
    std::vector<size_t> p_state, p_tail, p_k, p_v;
    int prefix_len = 0;
    // host tables
    std::vector<uint16_t> cos_table, sin_table;  // [positions][half] bf16 bits
    int table_positions = 0;
    // graphs
    bool graphs = false;
    // capacity path (s1_model_set_dynamic): the batch descriptor in device memory
    bool dynamic = false;
    uint8_t* desc = nullptr;
    size_t desc_bytes = 0;
    std::map<std::vector<size_t>, void*> graph_cache;
    std::deque<std::vector<size_t>> graph_order;
    // context parallelism: rank of `cp_world` processes that split one prompt in order
    Nccl nccl;
    ncclComm_t comm = nullptr;
    int cp_rank = 0, cp_world = 1;
    uint8_t* cp_state = nullptr;  // this rank's final GDN state of the current layer, sent on
    int64_t* cp_table = nullptr;  // (status, start, len, 0) of every rank, then this rank's own row
    // staged batch for run_staged
    Batch staged;
    bool have_staged = false;
    long launches = 0;
    std::string err;

    uint8_t* S(size_t off) const { return scratch + off; }
    uint8_t* W(const Region& r) const { return arena + r.off; }
};

int fail(Model* m, int code, const std::string& what) {
    m->err = what + " (code " + std::to_string(code) + ": " +
             (code > 0 && m->api.error_string ? m->api.error_string(code) : "host error") + ")";
    return code ? code : -1;
}

#define CK(expr, what)                                  \
    do {                                                \
        const int _rc = (expr);                         \
        if (_rc != 0) return fail(m, _rc, what);        \
    } while (0)

uint16_t f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// Rotary tables for positions [0, n): float32 inverse frequencies 1/theta^(2i/2half),
// float32 angle, float64 cos/sin rounded to float32 then bf16 (inputs.rs:178-204).
void ensure_tables(Model* m, int n) {
    if (n <= m->table_positions) return;
    const int half = m->cfg.rotary_half;
    std::vector<float> inv(half);
    for (int i = 0; i < half; i++)
        inv[i] = 1.0f / std::pow((float)m->cfg.theta, (float)(2 * i) / (float)(2 * half));
    m->cos_table.resize((size_t)n * half);
    m->sin_table.resize((size_t)n * half);
    for (int p = 0; p < n; p++)
        for (int i = 0; i < half; i++) {
            const double ang = (double)(inv[i] * (float)p);
            m->cos_table[(size_t)p * half + i] = f2bf((float)std::cos(ang));
            m->sin_table[(size_t)p * half + i] = f2bf((float)std::sin(ang));
        }
    m->table_positions = n;
}

Region take(size_t& at, size_t elems, bool f32 = false) {
    Region r;
    r.off = at;
    r.elems = elems;
    r.f32 = f32;
    at = up(at + elems * (f32 ? 4 : 2));
    return r;
}

void layout_weights(Model* m) {
    const s1_config& c = m->cfg;
    const size_t H = c.hidden, I = c.intermediate;
    size_t at = 0;
    m->embed = take(at, (size_t)c.vocab * H);
    m->layers.resize(c.n_layers);
    for (int i = 0; i < c.n_layers; i++) {
        Layer& L = m->layers[i];
        L.type = m->types[i];
        L.input_norm = take(at, H);
        L.post_norm = take(at, H);
        if (L.type == 0) {
            L.in_proj = take(at, (size_t)m->gdn_in * H);
            L.conv = take(at, (size_t)m->conv * 4);
            L.A_log = take(at, c.lin_v_heads);
            L.dt_bias = take(at, c.lin_v_heads);
            L.norm = take(at, c.lin_v_dim);
            L.out = take(at, H * (size_t)m->vd);
        } else {
            L.qkv = take(at, (size_t)m->attn_in * H);
            L.q_norm = take(at, c.head_dim);
            L.k_norm = take(at, c.head_dim);
            L.o = take(at, H * (size_t)m->qd);
        }
        L.gate_up = take(at, 2 * I * H);
        L.down = take(at, H * I);
    }
    m->final_norm = take(at, H);
    m->head_w = take(at, (size_t)c.labels * H, true);
    m->head_b = take(at, c.labels, true);
    m->arena_bytes = at;
}

int layout_scratch(Model* m) {
    const s1_config& c = m->cfg;
    const size_t T = m->cap_tokens, H = c.hidden, I = c.intermediate;
    size_t at = 0;
    auto t = [&](size_t bytes) {
        const size_t o = at;
        at = up(at + bytes);
        return o;
    };
    m->s_ids = t(T * 4);
    m->s_cos = t(T * c.rotary_half * 2);
    m->s_sin = t(T * c.rotary_half * 2);
    m->s_res = t(T * H * 2);
    m->s_x = t(T * H * 2);
    m->s_delta = t(T * H * 2);
    m->s_gdn_in = t(T * m->gdn_in * 2);
    m->s_lq = t(T * m->kd * 2);
    m->s_lk = t(T * m->kd * 2);
    m->s_lv = t(T * m->vd * 2);
    m->s_beta = t(T * c.lin_v_heads * 2);
    m->s_g = t(T * c.lin_v_heads * 4);
    m->s_rnq = t(T * c.lin_k_heads * 4);  // the front end's inverse norms of q and k
    m->s_rnk = t(T * c.lin_k_heads * 4);
    m->s_lo = t(T * m->vd * 2);
    m->s_ln = t(T * m->vd * 2);
    m->s_attn_in = t(T * m->attn_in * 2);
    m->s_aq = t(T * m->qd * 2);
    m->s_agate = t(T * m->qd * 2);
    m->s_ak = t(T * m->kvd * 2);
    m->s_ao = t(T * m->qd * 2);
    m->s_gate_up = t(m->fused ? 0 : T * 2 * I * 2);
    m->s_act = t(T * I * 2);
    m->s_rows = t((size_t)m->cap_seqs * 4);
    m->s_logits = t((size_t)m->cap_seqs * c.labels * 4);
    size_t floats = 0;
    if (m->api.gdn_batch_workspace_floats) {
        floats = m->api.gdn_batch_workspace_floats(m->cap_tokens, c.lin_v_heads, std::min(m->cap_seqs, 256));
        if (!floats) floats = m->api.gdn_batch_workspace_floats(m->cap_tokens, c.lin_v_heads, std::min(m->cap_seqs, 16));
    }
    floats = std::max(floats, m->api.gdn_workspace_floats(m->cap_tokens, c.lin_v_heads));
    m->ws_bytes = floats * 4 + 1024;
    m->s_ws = t(m->ws_bytes);
    void* p = nullptr;
    CK(m->api.malloc_(&p, at), "scratch allocation");
    m->scratch = static_cast<uint8_t*>(p);
    return 0;
}

// ------------------------------------------------------------- the forward ----
int gemm_store(Model* m, size_t x, const Region& w, size_t y, int M, int N, int K, bool dyn = false) {
    m->launches++;
    if (dyn) return m->api.gemm_dyn(m->gemm, m->S(x), m->W(w), m->S(y), M, N, K, N, 0, m->desc, m->stream);
    return m->api.gemm(m->gemm, m->S(x), m->W(w), m->S(y), M, N, K, N, m->stream);
}

// residual += x w^T, then x_next = rms_norm(residual, norm_w). On the capacity path M is
// the capacity and the batch's rows come from the descriptor.
int project_residual(Model* m, size_t x, const Region& w, int M, int K, const Region& norm_w, bool dyn = false) {
    const s1_config& c = m->cfg;
    if (dyn) {
        m->launches += 2;
        CK(m->api.gemm_dyn(m->gemm, m->S(x), m->W(w), m->S(m->s_res), M, c.hidden, K, c.hidden, 1, m->desc,
                           m->stream),
           "residual projection");
        CK(m->api.rms_norm_dyn(m->S(m->s_res), m->W(norm_w), m->S(m->s_x), M, c.hidden, c.eps, m->desc, m->stream),
           "rms norm");
        return 0;
    }
    if (m->fused) {
        m->launches += 2;
        CK(m->api.gemm_residual(m->gemm, m->S(x), m->W(w), m->S(m->s_res), M, c.hidden, K, c.hidden, m->stream),
           "residual projection");
        CK(m->api.rms_norm(m->S(m->s_res), m->W(norm_w), m->S(m->s_x), M, c.hidden, c.eps, m->stream), "rms norm");
        return 0;
    }
    CK(gemm_store(m, x, w, m->s_delta, M, c.hidden, K), "projection");
    m->launches++;
    CK(m->api.add_rms_norm(m->S(m->s_res), m->S(m->s_delta), m->W(norm_w), m->S(m->s_x), M, c.hidden, c.eps,
                           m->stream),
       "add rms norm");
    return 0;
}

// One NCCL group on the model stream: `send` to rank + 1 and / or receive into `recv`
// from rank - 1 (either may be null).
int cp_xfer(Model* m, const void* send, size_t send_bytes, void* recv, size_t recv_bytes, const char* what) {
    Nccl& n = m->nccl;
    const auto st = static_cast<cudaStream_t>(m->stream);
    ncclResult_t r = n.group_start();
    if (r == ncclSuccess && send) r = n.send(send, send_bytes, ncclUint8, m->cp_rank + 1, m->comm, st);
    if (r == ncclSuccess && recv) r = n.recv(recv, recv_bytes, ncclUint8, m->cp_rank - 1, m->comm, st);
    const ncclResult_t e = n.group_end();
    if (r == ncclSuccess) r = e;
    if (r != ncclSuccess) return fail(m, -1, std::string(what) + ": " + n.error_string(r));
    return 0;
}

// Layers [first, last) of a staged batch. From layer 0 the residual stream starts at the
// embedding of the staged ids; from a later layer it is whatever s_res holds (a
// residual stream handed in by s1_model_run_layers).
int run_layers(Model* m, const Batch& b, int first = 0, int last = -1) {
    const s1_config& c = m->cfg;
    if (last < 0) last = c.n_layers;
    const int T = (int)b.rows;
    const int n = (int)b.lengths.size();
    // capacity path: launches sized for cap_rows rows and cap_seqs sequences, the batch
    // itself read from the device descriptor (m->desc)
    const bool dyn = b.dyn;
    const int TL = dyn ? b.cap_rows : T;
    std::vector<size_t> offs(n + 1, 0);
    for (int i = 0; i < n; i++) offs[i + 1] = offs[i] + b.lengths[i];
    const float gdn_scale = 1.0f / std::sqrt((float)c.lin_k_dim);
    const float attn_scale = 1.0f / std::sqrt((float)c.head_dim);
    const bool suffix = b.prefix > 0 && !b.capture;
    const bool cp_send = b.cp && m->cp_rank + 1 < m->cp_world, cp_recv = b.cp && m->cp_rank > 0;
    if (first == 0) {
        m->launches++;
        const int32_t* ids = static_cast<const int32_t*>((const void*)m->S(m->s_ids));
        CK(dyn ? m->api.embed_dyn(ids, m->W(m->embed), m->S(m->s_res), TL, c.hidden, m->desc, m->stream)
               : m->api.embed(ids, m->W(m->embed), m->S(m->s_res), T, c.hidden, m->stream),
           "embed");
    }
    m->launches++;
    CK(dyn ? m->api.rms_norm_dyn(m->S(m->s_res), m->W(m->layers[first].input_norm), m->S(m->s_x), TL, c.hidden,
                                 c.eps, m->desc, m->stream)
           : m->api.rms_norm(m->S(m->s_res), m->W(m->layers[first].input_norm), m->S(m->s_x), T, c.hidden, c.eps,
                             m->stream),
       "input norm");
    if (dyn) {
        // Rows just past the batch that a last GDN chunk or attention key tile reads (masked
        // there, but they must be finite): zero, as the host-length launches' tensor-map
        // bounds give them. Nothing on the capacity path writes past the batch afterwards.
        const int margin = 256;
        const struct { size_t off; size_t ld, width; } tails[] = {
            {m->s_lq, (size_t)m->kd * 2, (size_t)m->kd * 2},
            {m->s_lk, (size_t)m->kd * 2, (size_t)m->kd * 2},
            {m->s_lv, (size_t)m->vd * 2, (size_t)m->vd * 2},
            {m->s_ak, (size_t)m->kvd * 2, (size_t)m->kvd * 2},
            {m->s_attn_in + (size_t)(m->attn_q + m->kvd) * 2, (size_t)m->attn_in * 2, (size_t)m->kvd * 2}};
        for (const auto& t : tails) {
            m->launches++;
            CK(m->api.clear_tail_dyn(m->S(t.off), t.ld, t.width, TL, margin, m->desc, m->stream), "clear tail rows");
        }
    }
    int gi = 0, ai = 0;  // index of the layer among the GDN / attention layers (prefix buffers)
    for (int li = 0; li < first; li++) (m->types[li] == 0 ? gi : ai)++;
    for (int li = first; li < last; li++) {
        const Layer& L = m->layers[li];
        if (L.type == 0) {
            CK(gemm_store(m, m->s_x, L.in_proj, m->s_gdn_in, TL, m->gdn_in, c.hidden, dyn), "gdn input projection");
            const int ld = m->gdn_in;
            uint8_t* gin = m->S(m->s_gdn_in);
            if (cp_send || cp_recv) {  // the last three pre-conv rows go to the next piece's conv
                const int rc = cp_xfer(m, cp_send ? gin + (size_t)(T - 3) * ld * 2 : nullptr, (size_t)3 * ld * 2,
                                       cp_recv ? m->prefix_buf + m->p_tail[gi] : nullptr, (size_t)3 * ld * 2,
                                       "conv history exchange");
                if (rc) return rc;
            }
            const void* hist = suffix ? m->prefix_buf + m->p_tail[gi] : nullptr;
            const size_t zoff = (size_t)m->conv * 2, boff = zoff + (size_t)m->vd * 2,
                         aoff = boff + (size_t)c.lin_v_heads * 2;
            float* rnq = reinterpret_cast<float*>(m->S(m->s_rnq));
            float* rnk = reinterpret_cast<float*>(m->S(m->s_rnk));
            // the fused front end: conv + SiLU, q/k inverse norms and gates in one launch
            const bool front = dyn || (m->api.gdn_front_batch && m->api.gdn_prefill_batch_xn && n <= m->api.max_batch);
            if (dyn) {
                m->launches++;
                CK(m->api.gdn_front_dyn(gin, hist, ld, m->W(L.conv), m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv), rnq,
                                        rnk, gin + boff, gin + aoff, m->W(L.A_log), m->W(L.dt_bias), m->S(m->s_beta),
                                        reinterpret_cast<float*>(m->S(m->s_g)), c.lin_v_heads, TL, b.cap_seqs, m->kd,
                                        m->vd, m->desc, m->stream),
                   "gdn front end");
            } else if (front) {
                m->launches++;
                CK(m->api.gdn_front_batch(gin, hist, ld, m->W(L.conv), m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv), rnq,
                                          rnk, gin + boff, gin + aoff, m->W(L.A_log), m->W(L.dt_bias),
                                          m->S(m->s_beta), reinterpret_cast<float*>(m->S(m->s_g)), c.lin_v_heads,
                                          b.lengths.data(), n, m->kd, m->vd, m->stream),
                   "gdn front end");
            } else if (m->api.gdn_conv_batch && n <= m->api.max_batch) {
                m->launches++;
                CK(m->api.gdn_conv_batch(gin, hist, ld, m->W(L.conv), m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv),
                                         b.lengths.data(), n, m->kd, m->vd, m->stream),
                   "gdn conv");
            } else {
                for (int s = 0; s < n; s++) {
                    m->launches++;
                    const size_t o = offs[s];
                    if (hist && m->api.gdn_conv_prefix) {
                        CK(m->api.gdn_conv_prefix(gin + o * ld * 2, hist, ld, m->W(L.conv), m->S(m->s_lq) + o * m->kd * 2,
                                                  m->S(m->s_lk) + o * m->kd * 2, m->S(m->s_lv) + o * m->vd * 2,
                                                  (int)b.lengths[s], m->kd, m->vd, m->stream),
                           "gdn conv prefix");
                    } else {
                        if (hist) return fail(m, -1, "library has no prefix convolution");
                        CK(m->api.gdn_conv(gin + o * ld * 2, ld, m->W(L.conv), m->S(m->s_lq) + o * m->kd * 2,
                                           m->S(m->s_lk) + o * m->kd * 2, m->S(m->s_lv) + o * m->vd * 2,
                                           (int)b.lengths[s], m->kd, m->vd, m->stream),
                           "gdn conv");
                    }
                }
            }
            if (!front) {
                m->launches++;
                CK(m->api.gdn_gates(gin + boff, gin + aoff, ld, m->W(L.A_log), m->W(L.dt_bias), m->S(m->s_beta),
                                    reinterpret_cast<float*>(m->S(m->s_g)), T, c.lin_v_heads, m->stream),
                   "gdn gates");
            }
            float* ws = reinterpret_cast<float*>(m->S(m->s_ws));
            const size_t state_bytes = (size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim * 4;
            if (cp_recv) {  // the previous piece's final state of this layer
                const int rc = cp_xfer(m, nullptr, 0, m->prefix_buf + m->p_state[gi], state_bytes, "state receive");
                if (rc) return rc;
            }
            const void* s_in = suffix ? m->prefix_buf + m->p_state[gi] : nullptr;
            void* s_out = b.capture ? m->prefix_buf + m->p_state[gi] : cp_send ? m->cp_state : nullptr;
            if (dyn) {
                m->launches++;
                CK(m->api.gdn_prefill_dyn(m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv),
                                          reinterpret_cast<const float*>(m->S(m->s_g)), m->S(m->s_beta), rnq, rnk,
                                          m->S(m->s_lo), TL, b.cap_seqs, c.lin_v_heads, c.lin_k_heads, gdn_scale, s_in,
                                          0, nullptr, m->desc, m->stream),
                   "gdn prefill");
            } else if (front) {
                m->launches++;
                CK(m->api.gdn_prefill_batch_xn(m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv),
                                               reinterpret_cast<const float*>(m->S(m->s_g)), m->S(m->s_beta), rnq, rnk,
                                               m->S(m->s_lo), b.lengths.data(), n, c.lin_v_heads, c.lin_k_heads,
                                               gdn_scale, s_in, 0, s_out, m->stream),
                   "gdn prefill");
            } else if (m->api.gdn_prefill_batch_x && n <= m->api.max_batch) {
                m->launches += 2;
                CK(m->api.gdn_prefill_batch_x(m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv),
                                              reinterpret_cast<const float*>(m->S(m->s_g)), m->S(m->s_beta),
                                              m->S(m->s_lo), ws, m->ws_bytes, b.lengths.data(), n, c.lin_v_heads,
                                              c.lin_k_heads, gdn_scale, s_in, 0, s_out, m->stream),
                   "gdn prefill");
            } else if (!s_in && !s_out && m->api.gdn_prefill_batch && n >= 2 && n <= 16) {
                m->launches += 3;
                CK(m->api.gdn_prefill_batch(m->S(m->s_lq), m->S(m->s_lk), m->S(m->s_lv),
                                            reinterpret_cast<const float*>(m->S(m->s_g)), m->S(m->s_beta),
                                            m->S(m->s_lo), ws, m->ws_bytes, b.lengths.data(), n, c.lin_v_heads,
                                            c.lin_k_heads, gdn_scale, m->stream),
                   "gdn prefill batch");
            } else {
                for (int s = 0; s < n; s++) {
                    const size_t o = offs[s];
                    m->launches += 3;
                    CK(m->api.gdn_prefill_x(m->S(m->s_lq) + o * m->kd * 2, m->S(m->s_lk) + o * m->kd * 2,
                                            m->S(m->s_lv) + o * m->vd * 2,
                                            reinterpret_cast<const float*>(m->S(m->s_g)) + o * c.lin_v_heads,
                                            m->S(m->s_beta) + o * c.lin_v_heads * 2, m->S(m->s_lo) + o * m->vd * 2,
                                            ws, (int)b.lengths[s], c.lin_v_heads, c.lin_k_heads, gdn_scale, s_in,
                                            s_out, m->stream),
                       "gdn prefill");
                }
            }
            if (cp_send) {
                const int rc = cp_xfer(m, m->cp_state, state_bytes, nullptr, 0, "state send");
                if (rc) return rc;
            }
            m->launches++;
            CK(dyn ? m->api.gated_rms_norm_dyn(m->S(m->s_lo), gin + zoff, ld, m->W(L.norm), m->S(m->s_ln), TL,
                                               c.lin_v_heads, c.lin_v_dim, c.eps, m->desc, m->stream)
                   : m->api.gated_rms_norm(m->S(m->s_lo), gin + zoff, ld, m->W(L.norm), m->S(m->s_ln), T,
                                           c.lin_v_heads, c.lin_v_dim, c.eps, m->stream),
               "gated norm");
            if (b.capture) {
                // the last three pre-conv rows of the prefix, in rows of ld
                const int P = (int)b.rows;
                m->launches++;
                CK(m->api.copy2d(m->prefix_buf + m->p_tail[gi], (size_t)ld * 2, gin + (size_t)(P - 3) * ld * 2,
                                 (size_t)ld * 2, (size_t)m->conv * 2, 3, m->stream),
                   "capture conv history");
            }
            CK(project_residual(m, m->s_ln, L.out, TL, m->vd, L.post_norm, dyn), "gdn output projection");
            gi++;
        } else {
            CK(gemm_store(m, m->s_x, L.qkv, m->s_attn_in, TL, m->attn_in, c.hidden, dyn), "attention input projection");
            const int ld = m->attn_in;
            uint8_t* ain = m->S(m->s_attn_in);
            uint8_t* kptr = ain + (size_t)m->attn_q * 2;
            uint8_t* vptr = kptr + (size_t)m->kvd * 2;
            m->launches++;
            CK(dyn ? m->api.attn_prep_dyn(ain, kptr, ld, m->W(L.q_norm), m->W(L.k_norm), m->S(m->s_cos), m->S(m->s_sin),
                                          m->S(m->s_aq), m->S(m->s_agate), m->S(m->s_ak), TL, c.heads, c.kv_heads,
                                          c.head_dim, c.rotary_half, c.eps, m->desc, m->stream)
                   : m->api.attn_prep(ain, kptr, ld, m->W(L.q_norm), m->W(L.k_norm), m->S(m->s_cos), m->S(m->s_sin),
                                      m->S(m->s_aq), m->S(m->s_agate), m->S(m->s_ak), T, c.heads, c.kv_heads,
                                      c.head_dim, c.rotary_half, c.eps, m->stream),
               "attention prep");
            const size_t kv_prefix = (size_t)b.prefix * m->kvd * 2;
            if (cp_recv) {  // K (normed, rotated) and V of every earlier piece
                int rc = cp_xfer(m, nullptr, 0, m->prefix_buf + m->p_k[ai], kv_prefix, "prefix K receive");
                if (!rc) rc = cp_xfer(m, nullptr, 0, m->prefix_buf + m->p_v[ai], kv_prefix, "prefix V receive");
                if (rc) return rc;
            }
            const void* pk = suffix ? m->prefix_buf + m->p_k[ai] : nullptr;
            const void* pv = suffix ? m->prefix_buf + m->p_v[ai] : nullptr;
            if (dyn) {
                m->launches++;
                CK(m->api.attention_dyn(m->S(m->s_aq), m->S(m->s_ak), vptr, ld, m->S(m->s_agate), m->S(m->s_ao), pk,
                                        pv, suffix ? b.prefix : 0, TL, b.cap_seqs, c.heads, c.kv_heads, c.head_dim,
                                        attn_scale, m->desc, m->stream),
                   "attention");
            } else if (suffix && m->api.attention_gated_shared_batch && n <= m->api.max_batch) {
                m->launches++;
                CK(m->api.attention_gated_shared_batch(m->S(m->s_aq), m->S(m->s_ak), vptr, ld, m->S(m->s_agate),
                                                       m->S(m->s_ao), pk, pv, b.lengths.data(), n, b.prefix,
                                                       c.heads, c.kv_heads, c.head_dim, attn_scale, m->stream),
                   "shared attention batch");
            } else if (!suffix && m->api.attention_gated_batch && n >= 2 && n <= m->api.max_batch) {
                m->launches++;
                CK(m->api.attention_gated_batch(m->S(m->s_aq), m->S(m->s_ak), vptr, ld, m->S(m->s_agate),
                                                m->S(m->s_ao), b.lengths.data(), n, c.heads, c.kv_heads, c.head_dim,
                                                attn_scale, m->stream),
                   "attention batch");
            } else {
                for (int s = 0; s < n; s++) {
                    const size_t o = offs[s];
                    m->launches++;
                    if (suffix) {
                        if (!m->api.attention_gated_shared) return fail(m, -1, "library has no shared attention");
                        CK(m->api.attention_gated_shared(m->S(m->s_aq) + o * m->qd * 2, m->S(m->s_ak) + o * m->kvd * 2,
                                                         vptr + o * ld * 2, ld, m->S(m->s_agate) + o * m->qd * 2,
                                                         m->S(m->s_ao) + o * m->qd * 2, pk, pv, (int)b.lengths[s],
                                                         b.prefix, c.heads, c.kv_heads, c.head_dim, attn_scale,
                                                         m->stream),
                           "shared attention");
                    } else {
                        CK(m->api.attention_gated(m->S(m->s_aq) + o * m->qd * 2, m->S(m->s_ak) + o * m->kvd * 2,
                                                  vptr + o * ld * 2, ld, m->S(m->s_agate) + o * m->qd * 2,
                                                  m->S(m->s_ao) + o * m->qd * 2, (int)b.lengths[s], c.heads,
                                                  c.kv_heads, c.head_dim, attn_scale, m->stream),
                           "attention");
                    }
                }
            }
            if (b.capture) {
                const int P = (int)b.rows;
                m->launches += 2;
                CK(m->api.copy_dd(m->prefix_buf + m->p_k[ai], m->S(m->s_ak), (size_t)P * m->kvd * 2, m->stream),
                   "capture prefix K");
                CK(m->api.copy2d(m->prefix_buf + m->p_v[ai], (size_t)m->kvd * 2, vptr, (size_t)ld * 2,
                                 (size_t)m->kvd * 2, P, m->stream),
                   "capture prefix V");
            }
            if (cp_send) {  // this piece's K and V after the received ones, all to the next piece
                m->launches += 2;
                CK(m->api.copy_dd(m->prefix_buf + m->p_k[ai] + kv_prefix, m->S(m->s_ak), (size_t)T * m->kvd * 2,
                                  m->stream),
                   "append K");
                CK(m->api.copy2d(m->prefix_buf + m->p_v[ai] + kv_prefix, (size_t)m->kvd * 2, vptr, (size_t)ld * 2,
                                 (size_t)m->kvd * 2, T, m->stream),
                   "append V");
                const size_t bytes = kv_prefix + (size_t)T * m->kvd * 2;
                int rc = cp_xfer(m, m->prefix_buf + m->p_k[ai], bytes, nullptr, 0, "prefix K send");
                if (!rc) rc = cp_xfer(m, m->prefix_buf + m->p_v[ai], bytes, nullptr, 0, "prefix V send");
                if (rc) return rc;
            }
            CK(project_residual(m, m->s_ao, L.o, TL, m->qd, L.post_norm, dyn), "attention output projection");
            ai++;
        }
        const Region& next = li + 1 < c.n_layers ? m->layers[li + 1].input_norm : m->final_norm;
        if (dyn) {
            m->launches++;
            CK(m->api.gemm_dyn(m->gemm, m->S(m->s_x), m->W(L.gate_up), m->S(m->s_act), TL, 2 * c.intermediate,
                               c.hidden, c.intermediate, 2, m->desc, m->stream),
               "gate/up projection");
        } else if (m->fused) {
            m->launches++;
            CK(m->api.gemm_swiglu(m->gemm, m->S(m->s_x), m->W(L.gate_up), m->S(m->s_act), T, c.intermediate,
                                  c.hidden, c.intermediate, m->stream),
               "gate/up projection");
        } else {
            CK(gemm_store(m, m->s_x, L.gate_up, m->s_gate_up, T, 2 * c.intermediate, c.hidden), "gate/up projection");
            m->launches++;
            CK(m->api.silu_mul(m->S(m->s_gate_up), 2 * c.intermediate, m->S(m->s_act), T, c.intermediate, m->stream),
               "silu mul");
        }
        CK(project_residual(m, m->s_act, L.down, TL, c.intermediate, next, dyn), "down projection");
    }
    return 0;
}

// Without cs1_head_score the head runs on the host after downloading each last row,
// as the reference's executor does (executor.rs:59-71); logits land in host_logits.
int host_head(Model* m, int n, float* logits) {
    const s1_config& c = m->cfg;
    std::vector<int32_t> rows(n);
    CK(m->api.download(rows.data(), m->S(m->s_rows), (size_t)n * 4, m->stream), "download rows");
    std::vector<float> W((size_t)c.labels * c.hidden), bias(c.labels);
    CK(m->api.download(W.data(), m->W(m->head_w), W.size() * 4, m->stream), "download head");
    CK(m->api.download(bias.data(), m->W(m->head_b), bias.size() * 4, m->stream), "download bias");
    std::vector<uint16_t> row(c.hidden);
    for (int i = 0; i < n; i++) {
        CK(m->api.download(row.data(), m->S(m->s_x) + (size_t)rows[i] * c.hidden * 2, (size_t)c.hidden * 2,
                           m->stream),
           "download last row");
        for (int l = 0; l < c.labels; l++) {
            double acc = 0.0;
            for (int d = 0; d < c.hidden; d++) {
                const uint32_t u = (uint32_t)row[d] << 16;
                float h;
                std::memcpy(&h, &u, 4);
                acc += (double)W[(size_t)l * c.hidden + d] * (double)h;
            }
            logits[(size_t)i * c.labels + l] = (float)acc + bias[l];
        }
    }
    return 0;
}

int run_head(Model* m, const Batch& b) {
    const s1_config& c = m->cfg;
    const int n = (int)b.lengths.size();
    if (!m->api.head_score) return 0;  // host head after the forward (host_head)
    m->launches++;
    if (b.dyn) {
        CK(m->api.head_score_dyn(m->S(m->s_x), c.hidden, reinterpret_cast<const int32_t*>(m->S(m->s_rows)), b.cap_seqs,
                                 reinterpret_cast<const float*>(m->W(m->head_w)),
                                 reinterpret_cast<const float*>(m->W(m->head_b)), c.labels, c.hidden,
                                 reinterpret_cast<float*>(m->S(m->s_logits)), m->desc, m->stream),
           "scorer head");
        return 0;
    }
    CK(m->api.head_score(m->S(m->s_x), c.hidden, reinterpret_cast<const int32_t*>(m->S(m->s_rows)), n,
                         reinterpret_cast<const float*>(m->W(m->head_w)), reinterpret_cast<const float*>(m->W(m->head_b)),
                         c.labels, c.hidden, reinterpret_cast<float*>(m->S(m->s_logits)), m->stream),
       "scorer head");
    return 0;
}

// Upload ids, per-row rotary tables and the last-token rows of a batch; on the capacity
// path (s1_model_set_dynamic) also its descriptor, after choosing the capacities: rows
// rounded up to an eighth of their power-of-two octave (a multiple of 64, at most the
// model's: at most 12.5% of launched rows idle, eight capacities per octave), sequences
// to a power of two.
int stage_inputs(Model* m, const int32_t* ids, Batch& b) {
    // Every id indexes the embedding table, so one out of range would read past it on the
    // device: the batch is refused before anything is copied or launched.
    for (size_t i = 0; i < b.rows; i++)
        if (ids[i] < 0 || ids[i] >= m->cfg.vocab)
            return fail(m, -1, "token id " + std::to_string(ids[i]) + " at row " + std::to_string(i) +
                                   " is outside [0, vocab = " + std::to_string(m->cfg.vocab) + ")");
    const int half = m->cfg.rotary_half;
    const int n = (int)b.lengths.size();
    size_t maxpos = 0;
    for (size_t len : b.lengths) maxpos = std::max(maxpos, len);
    ensure_tables(m, (int)(b.prefix + maxpos));
    std::vector<uint16_t> cs(b.rows * half), sn(b.rows * half);
    std::vector<int32_t> rows(n);
    size_t r = 0;
    for (int s = 0; s < n; s++) {
        for (size_t i = 0; i < b.lengths[s]; i++, r++) {
            const size_t pos = (b.capture ? 0 : b.prefix) + i;
            std::memcpy(&cs[r * half], &m->cos_table[pos * half], half * 2);
            std::memcpy(&sn[r * half], &m->sin_table[pos * half], half * 2);
        }
        rows[s] = (int32_t)(r - 1);
    }
    CK(m->api.upload(m->S(m->s_ids), ids, b.rows * 4, m->stream), "upload ids");
    CK(m->api.upload(m->S(m->s_cos), cs.data(), cs.size() * 2, m->stream), "upload cos");
    CK(m->api.upload(m->S(m->s_sin), sn.data(), sn.size() * 2, m->stream), "upload sin");
    CK(m->api.upload(m->S(m->s_rows), rows.data(), rows.size() * 4, m->stream), "upload rows");
    b.dyn = m->dynamic && m->desc && !b.capture && !b.cp && n <= 256;
    if (b.dyn) {
        int octave = 64;
        while (octave * 2 <= (int)b.rows) octave <<= 1;
        const int step = std::max(64, octave / 8);
        b.cap_rows = std::min(((int)b.rows + step - 1) / step * step, m->cap_tokens);
        int q = 1;
        while (q < n) q <<= 1;
        b.cap_seqs = std::min(q, std::min(m->cap_seqs, 256));
        std::vector<uint8_t> d(m->desc_bytes);
        if (m->api.batch_desc_pack(b.lengths.data(), b.lengths.size(), d.data(), d.size()) != 0)
            return fail(m, -1, "batch descriptor");
        CK(m->api.upload(m->desc, d.data(), d.size(), m->stream), "upload batch descriptor");
    }
    return 0;
}

// A graph serves the batches of its key: on the capacity path every batch of its
// capacities and prefix (the last field cannot be a capture flag), else one length vector.
std::vector<size_t> graph_key(const Batch& b) {
    if (b.dyn) return {(size_t)b.cap_rows, (size_t)b.cap_seqs, (size_t)b.prefix, SIZE_MAX};
    std::vector<size_t> k = b.lengths;
    k.push_back((size_t)b.prefix);
    k.push_back(b.capture ? 1 : 0);
    return k;
}

// Run the layers and the head of a staged batch, eagerly or through a cached graph.
int execute(Model* m, const Batch& b, bool head) {
    m->launches = 0;
    if (!m->graphs || b.capture) {
        int rc = run_layers(m, b);
        if (!rc && head) rc = run_head(m, b);
        return rc;
    }
    std::vector<size_t> key = graph_key(b);
    key.push_back(head ? 1 : 0);
    auto it = m->graph_cache.find(key);
    if (it != m->graph_cache.end()) {
        CK(m->api.graph_launch(it->second, m->stream), "graph launch");
        return 0;
    }
    int rc = run_layers(m, b);
    if (!rc && head) rc = run_head(m, b);
    if (rc) return rc;
    const long eager = m->launches;
    // capture the same sequence for the next call with this length vector
    if (m->api.graph_begin(m->stream) == 0) {
        int crc = run_layers(m, b);
        if (!crc && head) crc = run_head(m, b);
        void* exec = nullptr;
        const int erc = m->api.graph_end(m->stream, &exec);
        if (!crc && !erc && exec) {
            if (m->graph_cache.size() >= 64) {
                auto old = m->graph_cache.find(m->graph_order.front());
                if (old != m->graph_cache.end()) {
                    m->api.graph_destroy(old->second);
                    m->graph_cache.erase(old);
                }
                m->graph_order.pop_front();
            }
            m->graph_cache[key] = exec;
            m->graph_order.push_back(key);
        } else if (exec) {
            m->api.graph_destroy(exec);
        }
    }
    m->launches = eager;
    m->err.clear();
    return 0;
}

// Destroy every cached graph: a captured graph holds the device addresses it ran on.
void drop_graphs(Model* m) {
    for (auto& kv : m->graph_cache) m->api.graph_destroy(kv.second);
    m->graph_cache.clear();
    m->graph_order.clear();
}

int ensure_prefix(Model* m, int P) {
    if (m->prefix_buf && P <= m->prefix_len) return 0;
    if (m->prefix_buf) {
        // Graphs of suffix passes read the prefix buffer being freed: replaying one would
        // touch freed device memory, so they go with it (after the stream has drained).
        CK(m->api.stream_sync(m->stream), "sync before prefix reallocation");
        drop_graphs(m);
        m->api.free_(m->prefix_buf);
    }
    m->prefix_buf = nullptr;
    const s1_config& c = m->cfg;
    size_t at = 0;
    m->p_state.clear();
    m->p_tail.clear();
    m->p_k.clear();
    m->p_v.clear();
    for (int li = 0; li < c.n_layers; li++) {
        if (m->types[li] == 0) {
            m->p_state.push_back(at);
            at = up(at + (size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim * 4);
            m->p_tail.push_back(at);
            at = up(at + (size_t)3 * m->gdn_in * 2);
        } else {
            m->p_k.push_back(at);
            at = up(at + (size_t)P * m->kvd * 2);
            m->p_v.push_back(at);
            at = up(at + (size_t)P * m->kvd * 2);
        }
    }
    void* p = nullptr;
    CK(m->api.malloc_(&p, at), "prefix allocation");
    m->prefix_buf = static_cast<uint8_t*>(p);
    m->prefix_len = P;
    return 0;
}

int read_outputs(Model* m, const Batch& b, float* logits, float* hidden) {
    const s1_config& c = m->cfg;
    const int n = (int)b.lengths.size();
    if (logits && !m->api.head_score) {
        const int rc = host_head(m, n, logits);
        if (rc) return rc;
    } else if (logits) {
        CK(m->api.download(logits, m->S(m->s_logits), (size_t)n * c.labels * 4, m->stream), "download logits");
    } else {
        CK(m->api.stream_sync(m->stream), "sync");
    }
    if (hidden) {
        std::vector<uint16_t> row(c.hidden);
        size_t r = 0;
        for (int s = 0; s < n; s++) {
            r += b.lengths[s];
            CK(m->api.download(row.data(), m->S(m->s_x) + (r - 1) * c.hidden * 2, (size_t)c.hidden * 2, m->stream),
               "download hidden");
            for (int d = 0; d < c.hidden; d++) {
                const uint32_t u = (uint32_t)row[d] << 16;
                std::memcpy(&hidden[(size_t)s * c.hidden + d], &u, 4);
            }
        }
    }
    return 0;
}

int check_batch(Model* m, const size_t* lengths, size_t count, Batch& b) {
    if (!lengths || count == 0) return fail(m, -1, "empty batch");
    if ((int)count > m->cap_seqs) return fail(m, -1, "more sequences than the model's capacity");
    b.lengths.assign(lengths, lengths + count);
    b.rows = 0;
    for (size_t i = 0; i < count; i++) {
        if (lengths[i] == 0) return fail(m, -1, "empty sequence");
        b.rows += lengths[i];
    }
    if (b.rows > (size_t)m->cap_tokens) return fail(m, -1, "more tokens than the model's capacity");
    return 0;
}

}  // namespace

// ====================================================================== C API ====
extern "C" {

__attribute__((visibility("default"))) void* s1_model_create(const char* path, const s1_config* cfg, int device,
                                                             int max_tokens, int max_seqs) {
    if (!path || !cfg || cfg->n_layers <= 0 || !cfg->layer_types || max_tokens <= 0 || max_seqs <= 0) {
        g_create_error = "invalid arguments";
        return nullptr;
    }
    if (cfg->lin_k_dim != 128 || cfg->lin_v_dim != 128 || cfg->head_dim != 256) {
        g_create_error = "head dims must be 128 (GDN) and 256 (attention)";
        return nullptr;
    }
    auto* m = new Model;
    std::string err;
    if (!load_api(path, m->api, err)) {
        g_create_error = err;
        delete m;
        return nullptr;
    }
    m->cfg = *cfg;
    m->types.assign(cfg->layer_types, cfg->layer_types + cfg->n_layers);
    m->cfg.layer_types = m->types.data();
    m->device = device;
    m->cap_tokens = max_tokens;
    m->cap_seqs = max_seqs;
    m->kd = cfg->lin_k_heads * cfg->lin_k_dim;
    m->vd = cfg->lin_v_heads * cfg->lin_v_dim;
    m->conv = 2 * m->kd + m->vd;
    m->gdn_in = m->conv + m->vd + 2 * cfg->lin_v_heads;
    m->qd = cfg->heads * cfg->head_dim;
    m->attn_q = 2 * m->qd;
    m->kvd = cfg->kv_heads * cfg->head_dim;
    m->attn_in = m->attn_q + 2 * m->kvd;
    m->fused = m->api.gemm_residual && m->api.gemm_swiglu && cfg->intermediate % 128 == 0;
    auto bail = [&](const std::string& what, int rc) {
        g_create_error = what + " (code " + std::to_string(rc) + ")";
        s1_model_destroy(m);
        return nullptr;
    };
    int rc = m->api.set_device(device);
    if (rc) return bail("set device", rc);
    rc = m->api.stream_create(&m->stream);
    if (rc) return bail("stream", rc);
    layout_weights(m);
    void* p = nullptr;
    rc = m->api.malloc_(&p, m->arena_bytes);
    if (rc) return bail("weight arena allocation", rc);
    m->arena = static_cast<uint8_t*>(p);
    if (layout_scratch(m)) return bail(m->err, -1);
    m->gemm = m->api.gemm_create(32u << 20);
    if (!m->gemm) return bail("gemm handle", -1);
    return m;
}

__attribute__((visibility("default"))) void s1_model_destroy(void* mp) {
    auto* m = static_cast<Model*>(mp);
    if (!m) return;
    if (m->stream) m->api.stream_sync(m->stream);
    drop_graphs(m);
    if (m->gemm) m->api.gemm_destroy(m->gemm);
    if (m->arena) m->api.free_(m->arena);
    if (m->scratch) m->api.free_(m->scratch);
    if (m->prefix_buf) m->api.free_(m->prefix_buf);
    if (m->cp_state) m->api.free_(m->cp_state);
    if (m->cp_table) m->api.free_(m->cp_table);
    if (m->desc) m->api.free_(m->desc);
    if (m->comm) m->nccl.comm_destroy(m->comm);
    if (m->stream) m->api.stream_destroy(m->stream);
    // the library stays loaded: CUDA state it owns must outlive this model
    delete m;
}

__attribute__((visibility("default"))) const char* s1_model_error(void* mp) {
    auto* m = static_cast<Model*>(mp);
    return m ? m->err.c_str() : g_create_error.c_str();
}

// Copies one named parameter between the host and the arena (to_device: upload).
static int weight_io(Model* m, const char* name, void* data, size_t bytes, bool to_device) {
    const s1_config& c = m->cfg;
    const size_t H = c.hidden, I = c.intermediate;
    std::string n(name);
    auto put = [&](const Region& r, size_t row0, size_t rows, size_t cols) -> int {
        const size_t eb = r.f32 ? 4 : 2;
        if (bytes != rows * cols * eb) return fail(m, -1, "size mismatch for " + n);
        if (to_device)
            CK(m->api.upload(m->W(r) + row0 * cols * eb, data, bytes, m->stream), "upload " + n);
        else
            CK(m->api.download(data, m->W(r) + row0 * cols * eb, bytes, m->stream), "download " + n);
        return 0;
    };
    if (n == "embed") return put(m->embed, 0, c.vocab, H);
    if (n == "final_norm") return put(m->final_norm, 0, 1, H);
    if (n == "head_w") return put(m->head_w, 0, c.labels, H);
    if (n == "head_b") return put(m->head_b, 0, 1, c.labels);
    int li = -1;
    char leaf[64] = {0};
    if (std::sscanf(name, "l%d.%63s", &li, leaf) != 2 || li < 0 || li >= c.n_layers)
        return fail(m, -1, "unknown parameter " + n);
    const Layer& L = m->layers[li];
    const std::string f(leaf);
    if (f == "input_norm") return put(L.input_norm, 0, 1, H);
    if (f == "post_norm") return put(L.post_norm, 0, 1, H);
    if (f == "down") return put(L.down, 0, H, I);
    if (f == "gate" || f == "up") {
        if (bytes != I * H * 2) return fail(m, -1, "size mismatch for " + n);
        if (!m->fused) return put(L.gate_up, f == "gate" ? 0 : I, I, H);
        // interleave in blocks of 128 rows: [gate b | up b] for b = 0, 1, ...
        uint8_t* host = static_cast<uint8_t*>(data);
        for (size_t b = 0; b < I / 128; b++) {
            const size_t dst_row = 256 * b + (f == "gate" ? 0 : 128);
            if (to_device)
                CK(m->api.upload(m->W(L.gate_up) + dst_row * H * 2, host + b * 128 * H * 2, 128 * H * 2, m->stream),
                   "upload " + n);
            else
                CK(m->api.download(host + b * 128 * H * 2, m->W(L.gate_up) + dst_row * H * 2, 128 * H * 2, m->stream),
                   "download " + n);
        }
        return 0;
    }
    if (L.type == 0) {
        const size_t hv = c.lin_v_heads;
        if (f == "in_qkv") return put(L.in_proj, 0, m->conv, H);
        if (f == "in_z") return put(L.in_proj, m->conv, m->vd, H);
        if (f == "in_b") return put(L.in_proj, m->conv + m->vd, hv, H);
        if (f == "in_a") return put(L.in_proj, m->conv + m->vd + hv, hv, H);
        if (f == "conv") return put(L.conv, 0, m->conv, 4);
        if (f == "A_log") return put(L.A_log, 0, 1, hv);
        if (f == "dt_bias") return put(L.dt_bias, 0, 1, hv);
        if (f == "norm") return put(L.norm, 0, 1, c.lin_v_dim);
        if (f == "out") return put(L.out, 0, H, m->vd);
    } else {
        if (f == "q") return put(L.qkv, 0, m->attn_q, H);
        if (f == "k") return put(L.qkv, m->attn_q, m->kvd, H);
        if (f == "v") return put(L.qkv, m->attn_q + m->kvd, m->kvd, H);
        if (f == "q_norm") return put(L.q_norm, 0, 1, c.head_dim);
        if (f == "k_norm") return put(L.k_norm, 0, 1, c.head_dim);
        if (f == "o") return put(L.o, 0, H, m->qd);
    }
    return fail(m, -1, "unknown parameter " + n);
}

__attribute__((visibility("default"))) int s1_model_set_weight(void* mp, const char* name, const void* data,
                                                              size_t bytes) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !name || !data) return -1;
    return weight_io(m, name, const_cast<void*>(data), bytes, true);
}

__attribute__((visibility("default"))) int s1_model_get_weight(void* mp, const char* name, void* data,
                                                              size_t bytes) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !name || !data) return -1;
    return weight_io(m, name, data, bytes, false);
}

__attribute__((visibility("default"))) int s1_model_init_random(void* mp, uint64_t seed, float std_) {
    auto* m = static_cast<Model*>(mp);
    if (!m) return -1;
    if (!m->api.fill_random) return fail(m, -1, "library has no cs1_fill_random");
    uint64_t k = seed * 0x9E3779B97F4A7C15ull;
    auto fill = [&](const Region& r, int kind, float a, float b) -> int {
        k += 0xD1B54A32D192ED03ull;
        CK(m->api.fill_random(m->W(r), r.elems, kind, k, a, b, r.f32 ? 1 : 0, m->stream), "random fill");
        return 0;
    };
    // gate and up rows are drawn per logical 128-row block, so the stacked (gate | up) and
    // the interleaved (fused SwiGLU) layouts hold the same logical weights
    auto fill_gate_up = [&](const Layer& L) -> int {
        const size_t H = m->cfg.hidden, I = m->cfg.intermediate, blk = 128;
        const uint64_t kg = (k += 0xD1B54A32D192ED03ull), ku = (k += 0xD1B54A32D192ED03ull);
        for (size_t b = 0; b * blk < I; b++) {
            const size_t rows = std::min(blk, I - b * blk);
            const size_t gate_row = m->fused ? 2 * blk * b : blk * b;
            const size_t up_row = m->fused ? 2 * blk * b + blk : I + blk * b;
            CK(m->api.fill_random(m->W(L.gate_up) + gate_row * H * 2, rows * H, 0, kg + b, 0.f, std_, 0, m->stream),
               "random fill");
            CK(m->api.fill_random(m->W(L.gate_up) + up_row * H * 2, rows * H, 0, ku + b, 0.f, std_, 0, m->stream),
               "random fill");
        }
        return 0;
    };
    int rc = fill(m->embed, 0, 0.f, std_);
    for (const Layer& L : m->layers) {
        if (rc) return rc;
        rc = fill(L.input_norm, 0, 0.f, 0.1f) || fill(L.post_norm, 0, 0.f, 0.1f) || fill_gate_up(L) ||
             fill(L.down, 0, 0.f, std_);
        if (rc) return rc;
        if (L.type == 0)
            rc = fill(L.in_proj, 0, 0.f, std_) || fill(L.conv, 1, -0.5f, 0.5f) || fill(L.A_log, 2, 1.f, 16.f) ||
                 fill(L.dt_bias, 0, 1.f, 0.1f) || fill(L.norm, 0, 1.f, 0.1f) || fill(L.out, 0, 0.f, std_);
        else
            rc = fill(L.qkv, 0, 0.f, std_) || fill(L.q_norm, 0, 0.f, 0.1f) || fill(L.k_norm, 0, 0.f, 0.1f) ||
                 fill(L.o, 0, 0.f, std_);
    }
    if (rc) return rc;
    rc = fill(m->final_norm, 0, 0.f, 0.1f) || fill(m->head_w, 0, 0.f, std_) || fill(m->head_b, 0, 0.f, std_);
    if (rc) return rc;
    CK(m->api.stream_sync(m->stream), "random init");
    return 0;
}

__attribute__((visibility("default"))) int s1_model_forward(void* mp, const int32_t* ids, const size_t* lengths,
                                                           size_t count, float* logits, float* hidden) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !ids) return -1;
    Batch b;
    int rc = check_batch(m, lengths, count, b);
    if (rc) return rc;
    rc = stage_inputs(m, ids, b);
    if (rc) return rc;
    rc = execute(m, b, true);
    if (rc) return rc;
    return read_outputs(m, b, logits, hidden);
}

__attribute__((visibility("default"))) int s1_model_run_layers(void* mp, const int32_t* ids, const size_t* lengths,
                                                              size_t count, int first, int last, uint16_t* residual) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !ids || !residual) return -1;
    if (first < 0 || last <= first || last > m->cfg.n_layers) return fail(m, -1, "layer range out of bounds");
    Batch b;
    int rc = check_batch(m, lengths, count, b);
    if (rc) return rc;
    rc = stage_inputs(m, ids, b);
    if (rc) return rc;
    const size_t bytes = b.rows * (size_t)m->cfg.hidden * 2;
    CK(m->api.upload(m->S(m->s_res), residual, bytes, m->stream), "upload residual");
    m->launches = 0;
    rc = run_layers(m, b, first, last);
    if (rc) return rc;
    CK(m->api.download(residual, m->S(m->s_res), bytes, m->stream), "download residual");
    return 0;
}

__attribute__((visibility("default"))) int s1_model_forward_shared(void* mp, const int32_t* prefix_ids,
                                                                  size_t prefix_len, const int32_t* suffix_ids,
                                                                  const size_t* suffix_lengths, size_t count,
                                                                  float* logits, float* hidden) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !prefix_ids || !suffix_ids) return -1;
    if (prefix_len < 1 || prefix_len > (size_t)m->cap_tokens) return fail(m, -1, "prefix length out of range");
    Batch b;
    int rc = check_batch(m, suffix_lengths, count, b);
    if (rc) return rc;
    // The shared part is the prefix floored to a multiple of 64 tokens (the chunk of the
    // GDN scan and the key tile of the attention kernels), as the reference floors its
    // shared prefixes (batching.rs:29-49); the rest of the prefix is prepended to every
    // suffix, so each candidate's result is that of its full prompt.
    const size_t shared = prefix_len / 64 * 64, rest = prefix_len - shared;
    std::vector<int32_t> ids;
    std::vector<size_t> lens(count);
    ids.reserve(count * rest + b.rows);
    size_t at = 0;
    for (size_t i = 0; i < count; i++) {
        ids.insert(ids.end(), prefix_ids + shared, prefix_ids + prefix_len);
        ids.insert(ids.end(), suffix_ids + at, suffix_ids + at + suffix_lengths[i]);
        at += suffix_lengths[i];
        lens[i] = rest + suffix_lengths[i];
    }
    Batch s;
    rc = check_batch(m, lens.data(), count, s);
    if (rc) return rc;
    if (shared == 0) {  // nothing to share: the full prompts, packed
        rc = stage_inputs(m, ids.data(), s);
        if (!rc) rc = execute(m, s, true);
        return rc ? rc : read_outputs(m, s, logits, hidden);
    }
    rc = ensure_prefix(m, (int)shared);
    if (rc) return rc;
    Batch pre;
    pre.lengths = {shared};
    pre.rows = shared;
    pre.prefix = (int)shared;
    pre.capture = true;
    rc = stage_inputs(m, prefix_ids, pre);
    if (rc) return rc;
    rc = execute(m, pre, false);
    if (rc) return rc;
    s.prefix = (int)shared;
    rc = stage_inputs(m, ids.data(), s);
    if (rc) return rc;
    rc = execute(m, s, true);
    if (rc) return rc;
    return read_outputs(m, s, logits, hidden);
}

__attribute__((visibility("default"))) int s1_model_stage(void* mp, const int32_t* ids, const size_t* lengths,
                                                         size_t count) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !ids) return -1;
    Batch b;
    int rc = check_batch(m, lengths, count, b);
    if (rc) return rc;
    rc = stage_inputs(m, ids, b);
    if (rc) return rc;
    m->staged = b;
    m->have_staged = true;
    return 0;
}

__attribute__((visibility("default"))) int s1_model_run_staged(void* mp) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !m->have_staged) return -1;
    return execute(m, m->staged, true);
}

__attribute__((visibility("default"))) int s1_model_fetch_logits(void* mp, float* logits) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !m->have_staged) return -1;
    return read_outputs(m, m->staged, logits, nullptr);
}

__attribute__((visibility("default"))) int s1_model_set_graphs(void* mp, int enabled) {
    auto* m = static_cast<Model*>(mp);
    if (!m) return -1;
    m->graphs = enabled != 0;
    return 0;
}

__attribute__((visibility("default"))) int s1_model_set_dynamic(void* mp, int enabled) {
    auto* m = static_cast<Model*>(mp);
    if (!m) return -1;
    if (enabled && (!m->api.has_dyn() || !m->fused || !m->api.head_score))
        return fail(m, -1, "the library has no capacity-path entry points");
    if (enabled && !m->desc) {
        m->desc_bytes = m->api.batch_desc_bytes();
        void* p = nullptr;
        CK(m->api.malloc_(&p, m->desc_bytes), "batch descriptor");
        m->desc = static_cast<uint8_t*>(p);
    }
    m->dynamic = enabled != 0;
    return 0;
}

__attribute__((visibility("default"))) int s1_model_graph_count(void* mp) {
    auto* m = static_cast<Model*>(mp);
    return m ? (int)m->graph_cache.size() : -1;
}

__attribute__((visibility("default"))) void* s1_model_stream(void* mp) {
    auto* m = static_cast<Model*>(mp);
    return m ? m->stream : nullptr;
}

__attribute__((visibility("default"))) long s1_model_last_launches(void* mp) {
    auto* m = static_cast<Model*>(mp);
    return m ? m->launches : -1;
}

__attribute__((visibility("default"))) int s1_model_fused(void* mp) {
    auto* m = static_cast<Model*>(mp);
    return m ? (m->fused ? 1 : 0) : -1;
}

__attribute__((visibility("default"))) int s1_cp_unique_id(const char* nccl_library, void* id_out) {
    if (!id_out) return -1;
    Nccl n;
    std::string err;
    if (!load_nccl(nccl_library, n, err)) {
        g_create_error = err;
        return -1;
    }
    ncclUniqueId id;
    if (n.get_unique_id(&id) != ncclSuccess) {
        g_create_error = "ncclGetUniqueId failed";
        return -1;
    }
    std::memcpy(id_out, &id, sizeof(id));
    return 0;
}

__attribute__((visibility("default"))) int s1_model_cp_init(void* mp, const char* nccl_library, const void* id,
                                                           int rank, int world) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !id || world < 2 || rank < 0 || rank >= world) return -1;
    if (m->comm) return fail(m, -1, "context parallelism is already initialised");
    std::string err;
    if (!load_nccl(nccl_library, m->nccl, err)) return fail(m, -1, err);
    CK(m->api.set_device(m->device), "set device");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = m->nccl.comm_init_rank(&m->comm, world, uid, rank);
    if (r != ncclSuccess) {
        m->comm = nullptr;
        return fail(m, -1, std::string("ncclCommInitRank: ") + m->nccl.error_string(r));
    }
    void* p = nullptr;
    const s1_config& c = m->cfg;
    CK(m->api.malloc_(&p, (size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim * 4), "state buffer");
    m->cp_state = static_cast<uint8_t*>(p);
    CK(m->api.malloc_(&p, (size_t)(world + 1) * 4 * sizeof(int64_t)), "piece table");
    m->cp_table = static_cast<int64_t*>(p);
    m->cp_rank = rank;
    m->cp_world = world;
    return 0;
}

__attribute__((visibility("default"))) int s1_model_forward_cp(void* mp, const int32_t* ids, size_t len, size_t start,
                                                              float* logits, float* hidden) {
    auto* m = static_cast<Model*>(mp);
    if (!m) return -1;
    if (!m->comm) return fail(m, -1, "context parallelism is not initialised");
    const bool last = m->cp_rank + 1 == m->cp_world;
    // Every rank checks its own piece, then all ranks exchange (status, start, len) and
    // apply the same verdict before any transfer: a rank that refused alone would leave
    // its peers waiting in NCCL sends and receives that have no timeout.
    const int status = s1_cp_piece_status(ids, len, start, m->cp_rank, m->cp_world, m->cfg.vocab,
                                          (size_t)m->cap_tokens);
    const int64_t mine[4] = {status, (int64_t)start, (int64_t)len, 0};
    int64_t* own = m->cp_table + (size_t)m->cp_world * 4;
    CK(m->api.upload(own, mine, sizeof(mine), m->stream), "upload piece row");
    const ncclResult_t r = m->nccl.all_gather(own, m->cp_table, 4, ncclInt64, m->comm,
                                              static_cast<cudaStream_t>(m->stream));
    if (r != ncclSuccess) return fail(m, -1, std::string("piece exchange: ") + m->nccl.error_string(r));
    std::vector<int64_t> table((size_t)m->cp_world * 4);
    CK(m->api.download(table.data(), m->cp_table, table.size() * sizeof(int64_t), m->stream), "download pieces");
    char why[256];
    if (s1_cp_agree(table.data(), m->cp_world, why, sizeof(why)) != 0) return fail(m, -1, why);
    int rc = ensure_prefix(m, (int)(start + len));
    if (rc) return rc;
    Batch b;
    b.lengths = {len};
    b.rows = len;
    b.prefix = (int)start;
    b.cp = true;
    rc = stage_inputs(m, ids, b);
    if (rc) return rc;
    m->launches = 0;
    rc = run_layers(m, b);
    if (!rc && last) rc = run_head(m, b);
    if (rc) return rc;
    return read_outputs(m, b, last ? logits : nullptr, last ? hidden : nullptr);
}

__attribute__((visibility("default"))) int s1_model_get_config(void* mp, s1_config* out) {
    auto* m = static_cast<Model*>(mp);
    if (!m || !out) return -1;
    *out = m->cfg;
    return 0;
}

}  // extern "C"

// ===================================================== packing policy (host) ====
// Order-keeping launch packing of candidate prompts (open_jev batching.rs:9-25): a
// launch closes before a prompt that would make it hold max_sequences prompts or
// exceed max_tokens tokens; a longer prompt runs alone. Writes range starts into
// starts[] (count + 1 capacity, last = count) and returns the number of ranges.
extern "C" __attribute__((visibility("default"))) int s1_pack_ranges(const size_t* lengths, size_t count,
                                                                    size_t max_sequences, size_t max_tokens,
                                                                    size_t* starts) {
    if (!lengths || !starts || max_sequences == 0) return -1;
    int nr = 0;
    size_t start = 0, tokens = 0;
    for (size_t i = 0; i < count; i++) {
        if (i > start && (i - start == max_sequences || tokens + lengths[i] > max_tokens)) {
            starts[nr++] = start;
            start = i;
            tokens = 0;
        }
        tokens += lengths[i];
    }
    if (start < count) starts[nr++] = start;
    starts[nr] = count;
    return nr;
}

// Common prefix of 2..16 candidates floored to a multiple of 64, or 0 when shorter
// than 512 or when a candidate is shorter than `minimum` (batching.rs:29-49; minimum
// 2049 for long candidates, 512 for packed ones). The prefix always leaves a suffix.
extern "C" __attribute__((visibility("default"))) size_t s1_shared_prefix(const int32_t* const* ids,
                                                                         const size_t* lengths, size_t count,
                                                                         size_t minimum) {
    if (!ids || !lengths || count < 2 || count > 16) return 0;
    size_t shortest = (size_t)-1;
    for (size_t i = 0; i < count; i++) {
        if (lengths[i] < minimum) return 0;
        shortest = std::min(shortest, lengths[i]);
    }
    size_t common = 0;
    for (; common + 1 < shortest; common++) {
        bool same = true;
        for (size_t i = 1; i < count && same; i++) same = ids[i][common] == ids[0][common];
        if (!same) break;
    }
    const size_t aligned = common / 64 * 64;
    return aligned >= 512 ? aligned : 0;
}

// ============================================== context-parallel agreement (host) ====
// The checks one rank makes on its own piece of a context-parallel prompt: 0, or
// -1 no ids, -2 piece length outside [64, cap_tokens], -3 start not a multiple of 64,
// -4 length of a piece before the last not a multiple of 64, -5 rank 0 not at position 0
// (or another rank at 0), -6 a token id outside [0, vocab).
extern "C" __attribute__((visibility("default"))) int s1_cp_piece_status(const int32_t* ids, size_t len,
                                                                        size_t start, int rank, int world,
                                                                        int vocab, size_t cap_tokens) {
    if (!ids) return -1;
    if (len < 64 || len > cap_tokens) return -2;
    if (start % 64 != 0) return -3;
    if (rank + 1 < world && len % 64 != 0) return -4;
    if ((start == 0) != (rank == 0)) return -5;
    for (size_t i = 0; i < len; i++)
        if (ids[i] < 0 || ids[i] >= vocab) return -6;
    return 0;
}

// Every rank's (status, start, len, unused) row, in rank order: 0 when every rank's
// status is 0 and the pieces follow one another (rank r starts where rank r - 1 ends, so
// what rank r - 1 sends is what rank r expects), else -1 with the reason in msg. Every
// rank evaluates the same table and so reaches the same verdict.
extern "C" __attribute__((visibility("default"))) int s1_cp_agree(const int64_t* table, int world, char* msg,
                                                                 size_t cap) {
    auto say = [&](const std::string& s) {
        if (msg && cap) {
            std::strncpy(msg, s.c_str(), cap - 1);
            msg[cap - 1] = 0;
        }
        return -1;
    };
    if (!table || world < 1) return say("no piece table");
    static const char* what[] = {"", "no ids", "piece length out of range", "start not a multiple of 64",
                                 "piece before the last not a multiple of 64 tokens", "rank 0 must hold position 0",
                                 "token id outside [0, vocab)"};
    for (int r = 0; r < world; r++) {
        const int64_t st = table[4 * r];
        if (st != 0) {
            const int k = (st <= -1 && st >= -6) ? (int)-st : 0;
            return say("rank " + std::to_string(r) + " refused its piece: " +
                       (k ? what[k] : ("status " + std::to_string(st))));
        }
    }
    for (int r = 1; r < world; r++) {
        const int64_t want = table[4 * (r - 1) + 1] + table[4 * (r - 1) + 2];
        if (table[4 * r + 1] != want)
            return say("rank " + std::to_string(r) + " starts at " + std::to_string(table[4 * r + 1]) +
                       " but rank " + std::to_string(r - 1) + " ends at " + std::to_string(want));
    }
    if (msg && cap) msg[0] = 0;
    return 0;
}

// ========================================================= request dispatch (host) ====
// Requests over ranks (one process per GPU, each with a full weight replica), longest
// processing time first: requests in decreasing cost (ties: lower index first), each to
// the rank with the least cost assigned so far (ties: lower rank). The greedy's makespan
// is within 4/3 of the optimum. Writes rank_of[n] and, if non-null, loads[ranks]; returns
// 0, or -1 on invalid arguments (a negative or non-finite cost, ranks < 1).
extern "C" __attribute__((visibility("default"))) int s1_dispatch_lpt(const double* costs, size_t n, int ranks,
                                                                     int* rank_of, double* loads) {
    if (ranks < 1 || (n && (!costs || !rank_of))) return -1;
    for (size_t i = 0; i < n; i++)
        if (!(costs[i] >= 0.0) || !std::isfinite(costs[i])) return -1;
    std::vector<size_t> order(n);
    for (size_t i = 0; i < n; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return costs[a] > costs[b]; });
    std::vector<double> load(ranks, 0.0);
    for (size_t i : order) {
        int best = 0;
        for (int r = 1; r < ranks; r++)
            if (load[r] < load[best]) best = r;
        rank_of[i] = best;
        load[best] += costs[i];
    }
    if (loads)
        for (int r = 0; r < ranks; r++) loads[r] = load[r];
    return 0;
}
