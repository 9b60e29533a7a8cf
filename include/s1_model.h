// C interface of libs1_model.so: the Qwen3.5 hybrid decision-model prefill host.
//
// The host side of the reference's worker, rebuilt in C++ above the cs1_* ABI of
// qwen3_5_ops.h (the reference's host is Rust, which this build cannot compile):
//   s1_model_create / set_weight / init_random   Model::load_with_graph and the weight arena
//                                                (src/models/qwen3_5/native/src/model.rs:945-1076, 316-397)
//   s1_model_forward                             Model::forward_batch -> forward_batch_layout ->
//                                                run_with_attention (model.rs:1505, 1548-1632, 3178-3727)
//                                                plus DecisionHead::score per candidate
//                                                (src/models/open_jev/native/src/executor.rs:59-71)
//   s1_model_forward_shared                      Model::try_forward_shared_prefix ->
//                                                shared_prefix_with_original_rows (model.rs:1634-1907)
//   s1_model_set_graphs                          the CUDA-graph cache keyed by the length vector
//                                                (model.rs:1583-1614, 1959)
//   s1_model_set_dynamic                         device-side batching: graphs keyed by capacity
//                                                (replaces the host grouping of open_jev
//                                                executor/batched.rs:28-31)
// The model binds a cs1_* library by path at run time (dlopen, ABI version 9 check,
// required + optional symbols), as the reference's loader does (cuda.rs:673-698), so
// the same host drives this build's library or any other ABI-9 library.
//
// Errors: functions return 0 on success, else a cs1/CUDA error code or -1 for a host
// error; s1_model_error() describes the last one. Not thread-safe: one caller at a time
// per model (the reference serialises its Model behind a mutex, executor.rs:127).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct s1_config {
    int hidden;          // H
    int intermediate;    // I (multiple of 128 for the fused SwiGLU projection)
    int n_layers;
    const int* layer_types;  // n_layers entries: 0 = Gated DeltaNet, 1 = gated full attention
    int lin_k_heads;     // GDN key heads (HK)
    int lin_v_heads;     // GDN value heads (HV)
    int lin_k_dim;       // 128
    int lin_v_dim;       // 128
    int heads;           // attention query heads
    int kv_heads;        // attention key/value heads
    int head_dim;        // 256
    int rotary_half;     // 32 (rotary on the first 64 dims)
    double theta;        // rotary base
    float eps;           // RMSNorm epsilon
    int vocab;
    int labels;          // scorer-head rows
} s1_config;

// Binds the cs1 library at `cs1_library_path` ("lib" or "lib;aux", where aux may supply
// cs1_fill_random for libraries without it), selects `device`, allocates the weight
// arena and scratch for packs of up to max_tokens rows and max_seqs sequences.
// Returns null on failure (s1_model_error(NULL) then describes it).
void* s1_model_create(const char* cs1_library_path, const s1_config* cfg, int device, int max_tokens,
                      int max_seqs);
void s1_model_destroy(void* model);
const char* s1_model_error(void* model);

// Parameter names: "embed", "final_norm", "head_w" (f32 [labels,H]), "head_b" (f32 [labels]),
// and per layer i "l<i>.<leaf>" with leaf in input_norm, post_norm, gate, up, down and
// GDN: in_qkv, in_z, in_b, in_a, conv, A_log, dt_bias, norm, out;
// attention: q, k, v, q_norm, k_norm, o. Data are host bf16 (f32 for the head),
// row-major in the Transformers shapes; `bytes` must match.
int s1_model_set_weight(void* model, const char* name, const void* host_data, size_t bytes);
// The inverse: copy a parameter, in the same layout, back to host memory.
int s1_model_get_weight(void* model, const char* name, void* host_data, size_t bytes);
// Fill every parameter on the device from a counter-based generator (benchmarks):
// matrices ~ N(0, std), zero-centred norms ~ N(0, 0.1), gated-norm weight ~ 1 + N(0, 0.1),
// conv ~ U(-0.5, 0.5), A_log = log U(1, 16), dt_bias ~ 1 + N(0, 0.1).
int s1_model_init_random(void* model, uint64_t seed, float std);

// Packed independent candidates: ids concatenated [sum lengths] (host), lengths[count].
// Writes logits [count, labels] (host f32) and, if hidden is non-null, each candidate's
// final-norm last-token row [count, H] (host f32).
int s1_model_forward(void* model, const int32_t* ids, const size_t* lengths, size_t count, float* logits,
                     float* hidden);
// One shared prefix, computed once, then `count` suffixes continued from its GDN
// states, conv history and attention K/V. The shared part is the prefix floored to a
// multiple of 64 tokens (the reference floors shared prefixes the same way); the rest of
// the prefix is prepended to every suffix, so each candidate's logits are those of its
// full prompt (prefix + suffix) run alone. A prefix under 64 tokens is not shared at all.
int s1_model_forward_shared(void* model, const int32_t* prefix_ids, size_t prefix_len, const int32_t* suffix_ids,
                            const size_t* suffix_lengths, size_t count, float* logits, float* hidden);

// Resident inputs (benchmarks): stage ids and lengths on the device once, then run the
// forward on the model stream without host copies; fetch the logits afterwards.
int s1_model_stage(void* model, const int32_t* ids, const size_t* lengths, size_t count);
int s1_model_run_staged(void* model);
int s1_model_fetch_logits(void* model, float* logits);

// Layers [first, last) of a packed batch, eagerly, starting from a given residual stream
// instead of the embedding (layer-by-layer comparisons of two cs1 libraries or against an
// oracle). residual: host bf16 bits [sum lengths, H], the stream entering layer `first`;
// overwritten with the stream leaving layer last - 1. ids give the positions' rotary rows
// and are range-checked as in s1_model_forward.
int s1_model_run_layers(void* model, const int32_t* ids, const size_t* lengths, size_t count, int first, int last,
                        uint16_t* residual);

// CUDA graphs for repeated length vectors (default off): 0 = eager, 1 = capture/replay.
int s1_model_set_graphs(void* model, int enabled);
// Device-side batching (default off; needs the library's cs1_*_dyn entry points): every
// forward other than a prefix-capture pass and a context-parallel piece sizes its launches
// for capacities (rows rounded up to an eighth of their power-of-two octave, a multiple of
// 64; sequences to a power of two)
// and reads the batch from a descriptor in device memory uploaded with the ids, so with
// graphs on one captured graph per (capacities, shared prefix) serves every length vector
// that fits, instead of one per length vector (the reference's cache, model.rs:1583-1614).
// Logits and hidden rows are the same bits either way.
int s1_model_set_dynamic(void* model, int enabled);
// Graphs held in the model's cache.
int s1_model_graph_count(void* model);
// The model's cudaStream_t (for timing with events on the launching stream).
void* s1_model_stream(void* model);
// Kernel launches the last forward issued through the cs1 library (eager count).
long s1_model_last_launches(void* model);
// Fused projections (cs1_gemm_residual / cs1_gemm_swiglu) in use: 1 yes, 0 no.
int s1_model_fused(void* model);
// The model's configuration (layer_types points into the model; valid while it lives).
int s1_model_get_config(void* model, s1_config* out);

// ---- context-parallel prefill of one prompt over several GPUs (one process each) ----
// The prompt is split in order into one piece per rank; rank r runs every layer on its
// piece and receives from rank r - 1, per layer, what a shared prefix would hand it (the
// GDN layer's final fp32 state and last three pre-conv rows, the attention layer's K and V
// of all earlier pieces), sending its own on to rank r + 1 (NCCL point-to-point on the
// model stream, so the ranks pipeline layer by layer). With pieces on 64-token boundaries
// the last rank's logits equal those of the whole prompt on one GPU, bit for bit.
// NCCL is bound at run time: nccl_library null or "" means "libnccl.so.2".
int s1_cp_unique_id(const char* nccl_library, void* id_out);  // 128 bytes, made on one rank
int s1_model_cp_init(void* model, const char* nccl_library, const void* id, int rank, int world);
// ids[len]: this rank's piece, starting at prompt position `start` (0 on rank 0, a multiple
// of 64; every piece but the last a multiple of 64 long). logits [labels] and hidden [H]
// are written on the last rank only.
int s1_model_forward_cp(void* model, const int32_t* ids, size_t len, size_t start, float* logits, float* hidden);

// Before any transfer, forward_cp has every rank check its own piece and exchange
// (status, start, len) with the others (one NCCL all-gather); if any rank refuses, or the
// pieces do not follow one another, every rank returns the same error. The two steps,
// callable without a GPU:
// the checks on one rank's piece: 0, or a negative code (-1 no ids, -2 length outside
// [64, cap_tokens], -3 start not a multiple of 64, -4 a piece before the last not a
// multiple of 64 long, -5 rank 0 not at position 0, -6 a token id outside [0, vocab));
int s1_cp_piece_status(const int32_t* ids, size_t len, size_t start, int rank, int world, int vocab,
                       size_t cap_tokens);
// the verdict on all ranks' rows (status, start, len, 0) in rank order: 0, or -1 with the
// reason written to msg (capacity cap).
int s1_cp_agree(const int64_t* table, int world, char* msg, size_t cap);

// ---- checkpoints (src/models/qwen3_5/native/src/model.rs:96-226, 267-397) ----
// A Hugging Face Qwen3.5 config.json (or its text_config) as an s1_config; layer_types
// receives the per-layer kinds (capacity max_layers). labels is set to 1 (the Open-Jev
// scalar head); change it for another head. Returns 0, or -1 (s1_checkpoint_error()).
int s1_config_from_hf(const char* config_json, s1_config* out, int* layer_types, int max_layers);
// Load every language-model weight of a checkpoint folder (model.safetensors, or the
// shards of model.safetensors.index.json; tensors under "model.language_model.",
// "model." or no prefix) into the model; fp32 A_log and GDN-norm weights are rounded
// once to bf16, any other non-bf16 tensor is an error, and so is a weight of the model's
// configuration that the folder lacks or a tensor whose shape differs from the model's.
int s1_model_load_checkpoint(void* model, const char* dir);
// The scorer head of an export manifest (open_jev_export.json: head_weight, head_bias;
// a flat list for one label or [labels][hidden]).
int s1_model_load_head(void* model, const char* manifest_json, int labels, int hidden);
// The tensors a checkpoint folder maps to ("<name> <hf name> <dtype> <shape>" lines; no
// GPU needed). Returns the bytes of the full text, or -1.
long s1_checkpoint_list(const char* dir, char* out, size_t cap);
// The checks s1_model_load_checkpoint makes before reading any payload (tensor set,
// shapes, dtypes, payload sizes) against a configuration, without a model or a GPU.
int s1_checkpoint_check(const char* dir, const s1_config* cfg);
const char* s1_checkpoint_error(void);

// ---- packing policy (host integer logic, no GPU) ----
// Launch ranges of candidates (src/models/open_jev/native/src/batching.rs:9-25): writes
// the start of each range to starts[] (capacity count + 1; starts[ranges] = count) and
// returns the number of ranges, or -1 on invalid arguments.
int s1_pack_ranges(const size_t* lengths, size_t count, size_t max_sequences, size_t max_tokens, size_t* starts);
// Shared prefix of 2..16 candidates (batching.rs:29-49): the common prefix floored to a
// multiple of 64, or 0 if under 512 or if any candidate is shorter than `minimum`.
size_t s1_shared_prefix(const int32_t* const* ids, const size_t* lengths, size_t count, size_t minimum);

// ---- request dispatch over GPUs (host integer/float logic, no GPU) ----
// Each GPU holds a full weight replica and serves the requests given to it; requests go
// to ranks longest processing time first by token cost (s1omni.request_cost): requests
// in decreasing cost, each to the least-loaded rank (ties: lower index / lower rank).
// Writes rank_of[n] and, if non-null, the per-rank cost totals loads[ranks]. Returns 0,
// or -1 for ranks < 1 or a negative / non-finite cost. Replaces the reference's
// per-worker grouping of queued requests (src/runtime/src/batching.rs:94-125,
// src/models/open_jev/native/src/executor/batched.rs:28-31) one level up: across
// the per-GPU workers.
int s1_dispatch_lpt(const double* costs, size_t n, int ranks, int* rank_of, double* loads);

#ifdef __cplusplus
}
#endif
