// Shared device helpers of libqwen3_5_cuda.so (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s1 {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float f32(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ bf16 to_bf16(float x) { return __float2bfloat16_rn(x); }
// A float rounded through bfloat16, the value PyTorch keeps after a bfloat16 op.
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Eight floats rounded through bfloat16 in pairs: one cvt.rn.bf16x2.f32 per two values
// (the scalar conversion issues at half that rate), same values as rbf on each.
__device__ __forceinline__ void rbf8(float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 f = __bfloat1622float2(__floats2bfloat162_rn(v[i], v[i + 1]));
        v[i] = f.x;
        v[i + 1] = f.y;
    }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

// Sum over the block (blockDim.x a multiple of 32); every thread gets the total.
__device__ __forceinline__ float block_sum(float x, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    x = warp_sum(x);
    if (lane == 0) scratch[warp] = x;
    __syncthreads();
    float t = lane < warps ? scratch[lane] : 0.f;
    t = warp_sum(t);
    __syncthreads();
    return t;
}

// PyTorch's float32 SiLU and sigmoid.
__device__ __forceinline__ float silu(float x) { return x / (1.f + expf(-x)); }
// SiLU with the hardware exp2 / reciprocal approximations (relative error ~1e-7, far
// below the bf16 rounding that follows it) for the bandwidth-bound kernels, where the
// accurate expf and IEEE division would make them instruction-bound.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }


// Eight bfloat16 values moved as one 16-byte access.
struct alignas(16) Pack8 {
    __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const Pack8& p, float out[8]) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __bfloat1622float2(p.h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ Pack8 pack8(const float in[8]) {
    Pack8 p;
#pragma unroll
    for (int i = 0; i < 4; i++) p.h[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
    return p;
}
__device__ __forceinline__ Pack8 ld8(const bf16* p) { return *reinterpret_cast<const Pack8*>(p); }
__device__ __forceinline__ void st8(bf16* p, const Pack8& v) { *reinterpret_cast<Pack8*>(p) = v; }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace s1
