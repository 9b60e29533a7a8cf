// Internal declarations shared by the translation units of libqwen3_5_cuda.so.
// The public C ABI is include/qwen3_5_ops.h at the repository root.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/qwen3_5_ops.h"

namespace s1 {

// Packed sequences of one launch, passed to kernels by value (CUDA graph capture
// records it): sequence i covers rows [offset[i], offset[i+1]).
constexpr int MAX_SEQS = 256;
struct SeqTable {
    int count;
    int max_len;
    int offset[MAX_SEQS + 1];
    int order[MAX_SEQS];  // sequence indices by decreasing length (longest work scheduled first)
};

// Build a table from host lengths; false if count is 0 or above MAX_SEQS, a length is
// zero, or the rows overflow int.
bool make_table(SeqTable& t, const size_t* lengths, size_t count);

#ifdef __CUDACC__
// Sequence index of row `row` (binary search over the offsets).
__device__ __forceinline__ int seq_of(const SeqTable& t, int row) {
    int lo = 0, hi = t.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (t.offset[mid] <= row) lo = mid; else hi = mid - 1;
    }
    return lo;
}
#endif

}  // namespace s1
