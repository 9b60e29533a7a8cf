// Declarations shared by the two Gated DeltaNet translation units (gdn.cu, gdn_fp32.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "ops_internal.h"

namespace s1 {
namespace gdn {

constexpr int C = 64;   // chunk length
constexpr int K = 128;  // key head dim
constexpr int V = 128;  // value head dim

// Packed sequences plus the first chunk slot of each (slots = chunks over the pack).
struct GdnTable {
    SeqTable seq;
    int chunk_base[MAX_SEQS + 1];
    int max_chunks;
};
bool make_gdn_table(GdnTable& g, const SeqTable& t);

// Workspace regions; element type bf16 (scan operands) or fp32 (FP32 operator).
// Index [head * slots + slot] selects one chunk's tile.
struct Work {
    void* w;       // [.., 64 t][128 k]
    void* qd;      // [.., 64 t][128 k]
    void* p;       // [.., 64 t][64 j]
    void* kdt;     // [.., 128 k][64 t]
    void* ut;      // [.., 128 v][64 t]
    float* decay;  // [..] e^{cum_last}
    long slots;
};

struct Layout {
    long w, qd, p, kdt, ut, decay, total;
    Layout(long slots, int H, bool f32);
};

size_t workspace_bytes_for(long slots, int H, bool f32);

// The bf16 chunked prefill over packed sequences (gdn.cu): the fused kernel, which
// ignores the workspace arguments.
int run(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o, void* workspace,
        size_t workspace_bytes, const SeqTable& seqs, int H, int HK, float scale, const void* s_in,
        long s_in_stride, void* s_out, cudaStream_t st);
// The fused kernel: preparation and scan of a (head, sequence) in one CTA (gdn_fused.cu).
// On the capacity path (dyn non-null) `seqs` stands for the capacity (offset[count] =
// cap_rows: tensor-map extents) and the grid covers cap_seqs sequences. rnorm_q, rnorm_k:
// the front end's inverse norms of q and k ([T, HK] float32), or both null (computed here).
int run_fused(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
              const SeqTable& seqs, int H, int HK, float scale, const void* s_in, long s_in_stride, void* s_out,
              cudaStream_t st, const DevBatch* dyn = nullptr, int cap_seqs = 0, const float* rnorm_q = nullptr,
              const float* rnorm_k = nullptr);
// The two-kernel form with its tiles in a caller-provided (1024-byte aligned) workspace of
// workspace_bytes (gdn.cu).
int run_two_pass(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                 void* workspace, size_t workspace_bytes, const SeqTable& seqs, int H, int HK, float scale,
                 const void* s_in, long s_in_stride, void* s_out, cudaStream_t st);

}  // namespace gdn
}  // namespace s1
