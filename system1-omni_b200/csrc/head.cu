// Final-token scorer head: gathers each candidate's last hidden row and applies the
// learned label head, so only n x L float32 scores leave the GPU.
//
//   logits[i, l] = f32( sum_d f64(W[l, d]) * f64(hidden[rows[i], d]) ) + bias[l]
//
// The arithmetic of the reference's scalar head (open_jev executor.rs:59-71: a
// float64 dot product rounded to float32, plus a float32 bias), one row per label;
// one warp per (candidate, label), float64 partial sums reduced across the warp.
#include "common.cuh"
#include "ops_internal.h"

namespace s1 {
namespace {

__global__ void head_kernel(const bf16* __restrict__ hidden, int ldh, const int32_t* __restrict__ rows, int n,
                            const float* __restrict__ W, const float* __restrict__ bias, int L, int D,
                            float* __restrict__ logits, const DevBatch* dyn) {
    grid_dep_wait();
    grid_dep_launch();
    if (dyn) n = min(n, dyn->tab.count);
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= n * L) return;
    const int i = w / L, l = w % L;
    // the capacity path without a row list scores each sequence's final row
    const int r = rows ? rows[i] : dyn->tab.offset[i + 1] - 1;
    const bf16* h = hidden + (size_t)r * ldh;
    const float* wr = W + (size_t)l * D;
    double acc = 0.0;
    for (int d = lane; d < D; d += 32) acc += (double)wr[d] * (double)f32(h[d]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) logits[(size_t)i * L + l] = (float)acc + bias[l];
}

}  // namespace
}  // namespace s1

using namespace s1;

extern "C" int cs1_head_score(const void* hidden, int ldh, const int32_t* rows, int n, const float* W,
                              const float* bias, int L, int D, float* logits, void* stream) {
    if (!hidden || !rows || !W || !bias || !logits || n < 0 || L <= 0 || D <= 0 || ldh < D) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    const long warps = (long)n * L;
    return launch_pdl(head_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                      static_cast<const bf16*>(hidden), ldh, rows, n, W, bias, L, D, logits,
                      static_cast<const DevBatch*>(nullptr));
}

extern "C" int cs1_head_score_dyn(const void* hidden, int ldh, const int32_t* rows, int cap_n, const float* W,
                                  const float* bias, int L, int D, float* logits, const void* desc, void* stream) {
    if (!desc || !hidden || !W || !bias || !logits || cap_n <= 0 || cap_n > MAX_SEQS || L <= 0 || D <= 0 || ldh < D)
        return cudaErrorInvalidValue;
    const long warps = (long)cap_n * L;
    return launch_pdl(head_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                      static_cast<const bf16*>(hidden), ldh, rows, cap_n, W, bias, L, D, logits,
                      static_cast<const DevBatch*>(desc));
}
