// Internal declarations shared by the translation units of libqwen3_5_cuda.so.
// The public C ABI is include/qwen3_5_ops.h at the repository root.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#include <cuda_runtime.h>
#endif

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
    // prefix sums of 128-row query blocks in `order`: the blocks of sequence order[i] are
    // [qcum[i], qcum[i + 1]) (the attention kernel's work index, found by a uniform search)
    int qcum[MAX_SEQS + 1];
};

// Build a table from host lengths; false if count is 0 or above MAX_SEQS, a length is
// zero, or the rows overflow int.
bool make_table(SeqTable& t, const size_t* lengths, size_t count);

// The batch descriptor of the capacity path (the `*_dyn` entry points): the packed rows
// and the sequence table in device memory, written by one host-to-device copy before the
// launches (or a captured graph of them) run. Launch geometry comes from the caller's
// capacities (rows, sequences), the work from the descriptor, so one captured graph
// serves every batch within its capacities.
struct DevBatch {
    int rows;  // packed rows of the batch, <= the capacity the launches were sized for
    int pad[3];
    SeqTable tab;
};

#ifdef __CUDACC__
// Programmatic dependent launch. The forward's kernels are launched with programmatic
// stream serialisation, so a kernel's CTAs may start while the previous kernel's last
// CTAs still run: everything before grid_dep_wait() (barrier set-up, tensor-memory
// allocation, descriptor prefetch) overlaps that tail, and nothing before it touches
// global memory. grid_dep_wait() returns once the previous kernel has completed and its
// writes are visible; grid_dep_launch() lets the next kernel's CTAs be scheduled.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();  // always on (a build with -DS1_TUNING reads S1_PDL=0 to turn it off)
int sm_count();  // multiprocessors of the current device (148 when the query fails)

// Launch with the programmatic-serialisation attribute (see grid_dep_wait); the kernel
// must call grid_dep_wait() before its first global-memory access. The attribute is set
// for eager launches only: inside a captured CUDA graph it measured slower (the graph
// already removes the launch gaps it hides), so captured launches keep plain order.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool capturing = cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() && !capturing ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Rows to process: the descriptor's when a launch runs on the capacity path, else the
// launch's own count.
__device__ __forceinline__ int dyn_rows(const DevBatch* d, int rows) {
    return d ? min(d->rows, rows) : rows;
}

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
