// C interface of libqwen3_5_cuda.so, the B200 (sm_100a) build.
//
// Drop-in for the reference library of the same name (InferMatrixLab/system1-omni,
// src/backends/cuda/qwen3_5/ops.h, ABI 9): the same symbols, argument meanings,
// return conventions and ownership rules, so the reference's Rust loader
// (src/models/qwen3_5/native/src/cuda.rs:297-383 required, :495-661 optional)
// binds it unchanged. Each declaration names the reference declaration it
// replaces as `ops.h:<line>`.
//
// Conventions (ops.h:1-9): tensors are row-major bfloat16 unless noted; every
// operation queues work on `stream` (a cudaStream_t) and returns a cudaError_t
// (0 = success); invalid shapes return cudaErrorInvalidValue (1) before any launch;
// empty inputs (T == 0) are no-ops. Host arrays (lengths) are consumed before the
// call returns and passed to kernels by value, so CUDA graph capture records them.
// Workspace and outputs are caller-owned; no operation frees caller memory.
//
// Additive symbols of this build (not in the reference; callers that do not
// resolve them are unaffected) are marked "additive".
#pragma once

#include <stddef.h>
#include <stdint.h>

#define CS1_ABI_VERSION 9

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

// ---- runtime ----
uint32_t cs1_abi_version(void);                                   // ops.h:24
const char* cs1_error_string(int code);                           // ops.h:25
int cs1_set_device(int device);                                   // ops.h:26
int cs1_get_device(int* device);                                  // ops.h:27
// Set *flag to 0, then to 1 if any of the n bf16 values is NaN or infinite.
int cs1_bf16_finite(const void* x, size_t n, uint32_t* flag, void* stream);   // ops.h:29
int cs1_malloc(void** ptr, size_t bytes);                         // ops.h:30
int cs1_free(void* ptr);                                          // ops.h:31
int cs1_stream_create(void** stream);                             // ops.h:32
int cs1_stream_sync(void* stream);                                // ops.h:33
int cs1_stream_destroy(void* stream);                             // ops.h:34
int cs1_graph_begin(void* stream);                                // ops.h:35
int cs1_graph_end(void* stream, void** exec);                     // ops.h:36
int cs1_graph_launch(void* exec, void* stream);                   // ops.h:37
int cs1_graph_destroy(void* exec);                                // ops.h:38
int cs1_upload(void* dst, const void* src, size_t bytes, void* stream);     // ops.h:40 (copies, then waits)
int cs1_download(void* dst, const void* src, size_t bytes, void* stream);   // ops.h:41 (copies, then waits)
int cs1_copy_dd(void* dst, const void* src, size_t bytes, void* stream);    // ops.h:43
int cs1_copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
               void* stream);                                     // ops.h:46
// Additive: bit mask of bounded device waits that gave up (1 producer, 2 MMA issuer,
// 4 epilogue, 8 other) since the last clear; a set bit means a kernel abandoned its
// work and its outputs are not valid.
uint32_t cs1_fault_status(int clear);
// Additive, no counterpart in the reference: a self-test of that reporting. One thread
// waits, with the kernels' bounded wait cut to `cycles` (1e3 .. 4e9), on a barrier nothing
// completes, gives up and sets bit 8; no copy or MMA is in flight. Returns the launch status.
int cs1_wait_selftest(long long cycles, void* stream);

// ---- operations ----
int cs1_embed(const int32_t* ids, const void* table, void* out, int T, int D, void* stream);   // ops.h:51
int cs1_rms_norm(const void* x, const void* w, void* out, int rows, int D, float eps, void* stream);   // ops.h:54
int cs1_add_rms_norm(void* residual, const void* delta, const void* w, void* out, int rows, int D, float eps,
                     void* stream);                               // ops.h:57
int cs1_gated_rms_norm(const void* x, const void* z, int ldz, const void* w, void* out, int T, int H, int D,
                       float eps, void* stream);                  // ops.h:62
int cs1_gdn_conv(const void* qkv, int ld, const void* w, void* q, void* k, void* v, int T, int key_dim,
                 int value_dim, void* stream);                    // ops.h:67
int cs1_gdn_conv_vector(const void* qkv, int ld, const void* w, void* q, void* k, void* v, int T, int key_dim,
                        int value_dim, void* stream);             // ops.h:70
int cs1_gdn_conv_prefix(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                        int T, int key_dim, int value_dim, void* stream);   // ops.h:74
// Additive: causal conv of `count` (<= 256) packed sequences in one launch. Every
// sequence starts from zero history, or, if `history` is non-null, from the same three
// pre-conv rows [3, ld] (the tail of a shared prefix). lengths: host array.
int cs1_gdn_conv_batch(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                       const size_t* lengths, size_t count, int key_dim, int value_dim, void* stream);
int cs1_attention_gated_shared(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                               const void* prefix_k, const void* prefix_v, int suffix, int prefix, int Hq,
                               int Hk, int Dh, float scale, void* stream);   // ops.h:78
int cs1_attention_gated_shared_batch(const void* q, const void* k, const void* v, int ldv, const void* gate,
                                     void* out, const void* prefix_k, const void* prefix_v,
                                     const size_t* lengths, size_t count, int prefix, int Hq, int Hk, int Dh,
                                     float scale, void* stream);  // ops.h:85
int cs1_attention_gated_batch(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                              const size_t* lengths, size_t count, int Hq, int Hk, int Dh, float scale,
                              void* stream);                      // ops.h:92
int cs1_gdn_gates(const void* b, const void* a, int ld, const void* A_log, const void* dt_bias, void* beta,
                  float* g, int T, int H, void* stream);          // ops.h:98
// Additive: the GDN front end in one launch: cs1_gdn_conv_batch (causal conv + SiLU of q, k,
// v), the inverse L2 norm of every (row, head) of q and k (rnorm_q, rnorm_k: [T, key_dim /
// 128] float32, rsqrt(sum y^2 + 1e-6) over the head's bf16 outputs) and cs1_gdn_gates of
// the same rows (b, a: gate columns in rows of ld; H gates). key_dim a multiple of 128.
int cs1_gdn_front_batch(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                        float* rnorm_q, float* rnorm_k, const void* b, const void* a, const void* A_log,
                        const void* dt_bias, void* beta, float* g, int H, const size_t* lengths, size_t count,
                        int key_dim, int value_dim, void* stream);
// Additive: cs1_gdn_prefill_batch_x with the front end's inverse norms of q and k in place
// of the prefill's own (no workspace).
int cs1_gdn_prefill_batch_xn(const void* q, const void* k, const void* v, const float* g, const void* beta,
                             const float* rnorm_q, const float* rnorm_k, void* o, const size_t* lengths, size_t count,
                             int H, int HK, float scale, const void* state_in, int state_stride, void* state_out,
                             void* stream);
size_t cs1_gdn_batch_workspace_floats(int tokens, int H, int count);   // ops.h:104
int cs1_gdn_prefill_batch(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                          float* workspace, size_t workspace_bytes, const size_t* lengths, size_t count, int H,
                          int HK, float scale, void* stream);     // ops.h:105
int cs1_gdn_prefill_batch_shared(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                 void* o, float* workspace, size_t workspace_bytes, const size_t* lengths,
                                 size_t count, int H, int HK, float scale, const void* state,
                                 void* stream);                   // ops.h:109
size_t cs1_gdn_workspace_floats(int T, int H);                    // ops.h:112
void* cs1_gdn_fp32_create(size_t workspace_bytes);                // ops.h:115
void cs1_gdn_fp32_destroy(void* context);                         // ops.h:116
size_t cs1_gdn_fp32_workspace_floats(int T, int H);               // ops.h:117
int cs1_gdn_prefill_fp32(void* context, const void* q, const void* k, const void* v, const float* g,
                         const void* beta, void* o, float* workspace, int T, int H, int HK, float scale,
                         void* stream);                           // ops.h:118
// Additive: the FP32 operator with float32 output o [T,H,128] and an optional
// explicit float32 state (s_in null = zero; s_out null = skip), [H,128,128].
int cs1_gdn_prefill_fp32_x(void* context, const void* q, const void* k, const void* v, const float* g,
                           const void* beta, float* o, float* workspace, int T, int H, int HK, float scale,
                           const float* s_in, float* s_out, void* stream);
int cs1_gdn_prefill(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                    float* workspace, int T, int H, int HK, float scale, void* stream);   // ops.h:121
// Additive, no counterpart in the reference: cs1_gdn_prefill for callers that cannot
// allocate device memory (a host that may not call cudaMalloc on the path where it runs
// the prefill). The workspace is a fixed 64 MiB device array inside this library, held by
// every GPU that loads it until exit, so T x H is limited: roughly
// ceil(T / 64) * H <= 910 (T <= 1152 at 48 heads, 1792 at 32, 3584 at 16); larger
// sizes return cudaErrorInvalidValue before any launch. The first call on a device looks
// up the array's device address (make it before any stream capture). The array keeps the
// last call's contents; nothing needs clearing, but calls that overlap on the GPU (other
// streams, other host threads) race on it. Allocates nothing.
int cs1_gdn_prefill_noalloc(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                            int T, int H, int HK, float scale, void* stream);
int cs1_gdn_prefill_wide(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                         float* workspace, int T, int H, int HK, float scale, void* stream);   // ops.h:126
int cs1_gdn_prefill_x(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                      float* workspace, int T, int H, int HK, float scale, const void* s_in, void* s_out,
                      void* stream);                              // ops.h:134
// Additive: packed sequences with per-sequence initial states. state_in: null (zero),
// or [count,H,128,128] float32 (state_stride 1) or one shared [H,128,128] (state_stride 0);
// state_out: null or [count,H,128,128]. Workspace as cs1_gdn_batch_workspace_floats.
int cs1_gdn_prefill_batch_x(const void* q, const void* k, const void* v, const float* g, const void* beta,
                            void* o, float* workspace, size_t workspace_bytes, const size_t* lengths,
                            size_t count, int H, int HK, float scale, const void* state_in, int state_stride,
                            void* state_out, void* stream);
int cs1_attn_prep(const void* qg, const void* kr, int ld, const void* qw, const void* kw, const void* cos,
                  const void* sin, void* q, void* gate, void* k, int T, int Hq, int Hk, int Dh, int half,
                  float eps, void* stream);                       // ops.h:141
int cs1_attention(const void* q, const void* k, const void* v, int ldv, void* out, int T, int Hq, int Hk, int Dh,
                  float scale, void* stream);                     // ops.h:147
int cs1_attention_gated(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out, int T,
                        int Hq, int Hk, int Dh, float scale, void* stream);   // ops.h:153
int cs1_attention_gated_bidirectional(const void* q, const void* k, const void* v, int ldv, const void* gate,
                                      void* out, int T, int Hq, int Hk, int Dh, float scale,
                                      void* stream);              // ops.h:159
int cs1_attention_gated_prefix_bidirectional(const void* q, const void* k, const void* v, int ldv,
                                             const void* gate, void* out, int T, int state, int Hq, int Hk,
                                             int Dh, float scale, void* stream);   // ops.h:167
int cs1_attention_gated_prefix(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                               int T, int Hq, int Hk, int Dh, float scale, int q_base, void* stream);   // ops.h:174
int cs1_sigmoid_gate(void* x, const void* gate, size_t n, void* stream);   // ops.h:179
int cs1_silu_mul(const void* gate_up, int ld, void* out, int T, int I, void* stream);   // ops.h:182

// GEMM handles (ops.h:187-217). The tcgen05 kernels need no library workspace and
// reduce every output in an order independent of M, the row index and the tile
// width, so every handle kind is row-invariant and all handles are compatible.
void* cs1_gemm_create(size_t workspace_bytes);                    // ops.h:186
void* cs1_gemm_create_fixed(size_t workspace_bytes, int reference_m);   // ops.h:192
void* cs1_gemm_create_matched(size_t workspace_bytes, int reference_m);   // ops.h:196
int cs1_gemm_compatible(void* ordinary, void* matched, int M, int N, int K);   // ops.h:197
void cs1_gemm_destroy(void* gemm);                                // ops.h:198
int cs1_gemm_enable_equivalent_tiles(void* gemm);                 // ops.h:203
int cs1_gemm(void* gemm, const void* x, const void* w, void* y, int M, int N, int K, int ldy, void* stream);   // ops.h:204
int cs1_gemm_packed(void* gemm, const void* x, const void* w, void* y, const size_t* lengths, size_t count, int N,
                    int K, void* stream);                         // ops.h:208
int cs1_gemm_reuse_check(void* gemm, const size_t* original_rows, size_t originals, const size_t* target_rows,
                         size_t targets, int N, int K);           // ops.h:214
int cs1_gemm_reuse(void* gemm, const void* x, const void* w, void* y, int M, int N, int K, int original_M,
                   void* stream);                                 // ops.h:216
// Additive: residual[M,N] (rows of ldr) = bf16(residual + bf16(x w^T)), the decoder
// residual add fused into the projection epilogue.
int cs1_gemm_residual(void* gemm, const void* x, const void* w, void* residual, int M, int N, int K, int ldr,
                      void* stream);
// Additive: out[M,I] (rows of ldo) = bf16(bf16(silu(bf16(x g^T))) * bf16(x u^T)) where w
// [2I,K] holds gate and up rows interleaved in blocks of 128 (rows 256b..256b+127 are
// gate rows 128b.., rows 256b+128.. the matching up rows). I a multiple of 128.
int cs1_gemm_swiglu(void* gemm, const void* x, const void* w, void* out, int M, int I, int K, int ldo,
                    void* stream);

// Additive: final-token scorer head (open_jev executor.rs:59-71 for each of L labels):
// logits[i,l] = f32(sum_d f64(W[l,d]) * f64(hidden[rows[i], d])) + bias[l].
// hidden bf16 [*, D] in rows of ldh; rows int32 [n] on the device; W f32 [L,D];
// bias f32 [L]; logits f32 [n,L].
int cs1_head_score(const void* hidden, int ldh, const int32_t* rows, int n, const float* W, const float* bias,
                   int L, int D, float* logits, void* stream);

// Additive: fill n elements (dtype 0 bf16, 1 f32) from a counter-based generator keyed
// by (seed, index): kind 0 a + b*N(0,1), 1 U(a,b), 2 log U(a,b). For benchmark weights.
int cs1_fill_random(void* dst, size_t n, int kind, uint64_t seed, float a, float b, int dtype, void* stream);

// ---- capacity path (additive) ----
// Device-side batching: the `*_dyn` entry points size their launches for capacities
// (cap_rows packed rows, cap_seqs sequences) and take the batch itself from a descriptor
// in device memory (`desc`: cs1_batch_desc_bytes() bytes, 16-byte aligned, filled on the
// host by cs1_batch_desc_pack and copied to the device before the launches run). A CUDA
// graph captured once per capacity therefore serves every batch that fits it, where the
// reference captures one graph per length vector (model.rs:1583-1614) and groups requests
// on the host (open_jev executor/batched.rs:28-31). Rows past the descriptor's count
// inside the capacity are scratch: they may be read and written, their values are
// unspecified. Each result equals its host-length entry point's bit for bit.
size_t cs1_batch_desc_bytes(void);
// lengths: host array of `count` (1..256) nonzero sequence lengths.
int cs1_batch_desc_pack(const size_t* lengths, size_t count, void* out, size_t bytes);
int cs1_embed_dyn(const int32_t* ids, const void* table, void* out, int cap_rows, int D, const void* desc,
                  void* stream);
// Zero width_bytes of rows [rows, min(rows + margin, cap_rows)) of x (rows of ld_bytes; both
// multiples of 16, x 16-byte aligned): the rows just past the batch that a last GDN chunk
// or attention key tile reads (masked, but they must be finite; the host-length entry
// points read zeros there through their tensor-map bounds).
int cs1_clear_tail_dyn(void* x, size_t ld_bytes, size_t width_bytes, int cap_rows, int margin, const void* desc,
                       void* stream);
int cs1_rms_norm_dyn(const void* x, const void* w, void* out, int cap_rows, int D, float eps, const void* desc,
                     void* stream);
int cs1_add_rms_norm_dyn(void* residual, const void* delta, const void* w, void* out, int cap_rows, int D,
                         float eps, const void* desc, void* stream);
int cs1_gated_rms_norm_dyn(const void* x, const void* z, int ldz, const void* w, void* out, int cap_rows, int H,
                           int D, float eps, const void* desc, void* stream);
// epilogue: 0 store (cs1_gemm), 1 residual (cs1_gemm_residual), 2 SwiGLU (cs1_gemm_swiglu,
// N = 2I interleaved rows).
int cs1_gemm_dyn(void* gemm, const void* x, const void* w, void* y, int cap_rows, int N, int K, int ldy,
                 int epilogue, const void* desc, void* stream);
int cs1_gdn_conv_dyn(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                     int cap_rows, int cap_seqs, int key_dim, int value_dim, const void* desc, void* stream);
int cs1_gdn_gates_dyn(const void* b, const void* a, int ld, const void* A_log, const void* dt_bias, void* beta,
                      float* g, int cap_rows, int H, const void* desc, void* stream);
// state_in / state_out as cs1_gdn_prefill_batch_x; no workspace. rnorm_q, rnorm_k: the
// inverse norms from cs1_gdn_front_dyn, or both null (computed in the prefill).
int cs1_gdn_prefill_dyn(const void* q, const void* k, const void* v, const float* g, const void* beta,
                        const float* rnorm_q, const float* rnorm_k, void* o, int cap_rows, int cap_seqs, int H,
                        int HK, float scale, const void* state_in, int state_stride, void* state_out, const void* desc,
                        void* stream);
// cs1_gdn_front_batch on the capacity path.
int cs1_gdn_front_dyn(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                      float* rnorm_q, float* rnorm_k, const void* b, const void* a, const void* A_log,
                      const void* dt_bias, void* beta, float* g, int H, int cap_rows, int cap_seqs, int key_dim,
                      int value_dim, const void* desc, void* stream);
int cs1_attn_prep_dyn(const void* qg, const void* kr, int ld, const void* qw, const void* kw, const void* cos,
                      const void* sin, void* q, void* gate, void* k, int cap_rows, int Hq, int Hk, int Dh, int half,
                      float eps, const void* desc, void* stream);
// prefix 0: cs1_attention_gated_batch; prefix > 0: cs1_attention_gated_shared_batch.
int cs1_attention_dyn(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                      const void* prefix_k, const void* prefix_v, int prefix, int cap_rows, int cap_seqs, int Hq,
                      int Hk, int Dh, float scale, const void* desc, void* stream);
// The first (descriptor's sequence count) of cap_n candidates are scored; rows: device
// int32 [cap_n] rows of `hidden`, or null for each sequence's final row.
int cs1_head_score_dyn(const void* hidden, int ldh, const int32_t* rows, int cap_n, const float* W,
                       const float* bias, int L, int D, float* logits, const void* desc, void* stream);

// ---- vision (ops.h:231-236): required by the reference loader; this library does
// not implement the vision path and returns cudaErrorNotSupported ----
int cs1_vision_linear(void* gemm, const void* x, const void* w, const void* bias, void* y, int M, int N, int K,
                      void* stream);
int cs1_gemm_f32(void* gemm, const float* x, const float* w, float* y, int M, int N, int K, void* stream);
int cs1_vision_norm(const void* x, const void* w, const void* b, void* y, int rows, int d, void* stream);
int cs1_vision_position(void* x, const void* table, const int* indices, const float* weights, int n, void* stream);
int cs1_vision_rope(const void* qkv, const float* co, const float* si, void* q, void* k, int n, void* stream);
int cs1_vision_attention(const void* q, const void* k, const void* v, void* out, int n, void* stream);
int cs1_vision_bias(void* x, const void* bias, size_t n, int d, void* stream);               // ops.h:233
int cs1_vision_gelu(void* x, size_t n, int exact, void* stream);                             // ops.h:234
int cs1_vision_add(void* x, const void* delta, size_t n, void* stream);                      // ops.h:235
int cs1_vision_to_float(const void* x, float* out, size_t n, void* stream);                  // ops.h:236
int cs1_vision_lora_add(void* x, const float* delta, size_t n, float scale, void* stream);   // ops.h:237

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
