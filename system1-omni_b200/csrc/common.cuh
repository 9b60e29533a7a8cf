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

// SiLU with the hardware exp2 / reciprocal approximations (relative error ~1e-7, far
// below the bf16 rounding that follows it) for the bandwidth-bound kernels, where the
// accurate expf and IEEE division would make them instruction-bound.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }
// PyTorch's float32 sigmoid.
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

// 16-byte asynchronous global -> shared copy (zero-filled when !valid; gmem must still be
// a valid address), its group commit and waits.
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Packed fp32 pairs: Blackwell's f32x2 arithmetic does two lanes of a 64-bit register
// pair in one instruction, each lane rounded exactly like the scalar operation.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
// Maximum of three (one instruction on sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// bf16 rounding of a pair (one paired conversion), back in fp32.
__device__ __forceinline__ float2 rbf2(float2 v) { return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y)); }
// Sigmoid of a pair from 1 / (1 + 2^(-y log2 e)) with the hardware base-2 exponential and
// reciprocal (relative error ~1e-7).
__device__ __forceinline__ float2 sigmoid2_fast(float2 y) {
    constexpr float kLog2e = 1.4426950408889634f;
    const float2 t = mul2(y, make_float2(-kLog2e, -kLog2e));
    float2 e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(t.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(t.y));
    const float2 d = add2(e, make_float2(1.f, 1.f));
    float2 r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
    return r;
}
// The same SiLU for one value, operation for operation (so a scalar and a packed caller
// round identically): the SwiGLU of the GEMM epilogues and of cs1_silu_mul. Within one
// bf16 ulp of PyTorch's float32 SiLU after rounding to bf16, except for x < -87.34: there
// 1 + e^-x exceeds 2^126, the flush-to-zero reciprocal gives 0 and the result is -0 where
// the exact value has a magnitude below 1.1e-36.
__device__ __forceinline__ float silu_hw(float y) {
    constexpr float kLog2e = 1.4426950408889634f;
    float e, r;
    const float t = y * -kLog2e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(e + 1.f));
    return y * r;
}
// SiLU of a pair from the identity y / (1 + 2^(-y log2 e)) with the hardware base-2
// exponential and reciprocal (relative error ~1e-7, far below the bf16 rounding that
// follows): one packed multiply, add and multiply and two special-function operations
// per lane; rounds lane for lane like silu_hw.
__device__ __forceinline__ float2 silu2_fast(float2 y) {
    constexpr float kLog2e = 1.4426950408889634f;
    const float2 t = mul2(y, make_float2(-kLog2e, -kLog2e));
    float2 e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(t.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(t.y));
    const float2 d = add2(e, make_float2(1.f, 1.f));
    float2 r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
    return mul2(y, r);
}
}  // namespace s1
