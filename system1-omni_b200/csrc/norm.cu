// Row normalisations of the Qwen3.5 prefill (bandwidth-bound, 16-byte accesses).
//
//  cs1_rms_norm       out = bf16(x * rsqrt(mean(x^2) + eps) * (1 + w))      (Qwen3_5RMSNorm)
//  cs1_add_rms_norm   residual = bf16(residual + delta); out = rms_norm(residual)
//  cs1_gated_rms_norm GDN output norm, rows of 128:
//                     bf16(bf16(w * bf16(x / rms(x))) * silu(z))          (Qwen3_5RMSNormGated)
// Rounding points follow the reference kernels (norm.cu:11-139 of the reference);
// the fp32 sum of squares is reduced in a different order (tree over packs).
#include "common.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(norm)

namespace s1 {
namespace {

constexpr int NT = 256;       // threads per row block
constexpr int MAXP = 4;       // packs of 8 cached per thread: D <= 8192

// Rows wider than the warp kernel takes (5,120 < D <= 8,192): a CTA per row.
template <bool Add>
__global__ void __launch_bounds__(NT) rms_kernel(bf16* __restrict__ res, const bf16* __restrict__ delta,
                                                 const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                 bf16* __restrict__ out, int D, float eps) {
    __shared__ float scratch[32];
    const size_t row = blockIdx.x;
    const int packs = D >> 3;
    // the weights are loaded with the row, ahead of the reduction
    Pack8 wp[MAXP];
#pragma unroll
    for (int i = 0; i < MAXP; i++) {
        const int pk = threadIdx.x + i * NT;
        if (pk < packs) wp[i] = ld8(w + (size_t)pk * 8);
    }
    float v[MAXP][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXP; i++) {
        const int pk = threadIdx.x + i * NT;
        if (pk < packs) {
            const size_t off = row * D + (size_t)pk * 8;
            if constexpr (Add) {
                float a[8], b[8];
                unpack8(ld8(res + off), a);
                unpack8(ld8(delta + off), b);
#pragma unroll
                for (int e = 0; e < 8; e++) v[i][e] = rbf(a[e] + b[e]);
                st8(res + off, pack8(v[i]));
            } else {
                unpack8(ld8(x + off), v[i]);
            }
#pragma unroll
            for (int e = 0; e < 8; e++) ss = fmaf(v[i][e], v[i][e], ss);
        }
    }
    const float inv = rsqrtf(block_sum(ss, scratch) / D + eps);
#pragma unroll
    for (int i = 0; i < MAXP; i++) {
        const int pk = threadIdx.x + i * NT;
        if (pk < packs) {
            float wv[8], o[8];
            unpack8(wp[i], wv);
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = v[i][e] * inv * (1.f + wv[e]);
            st8(out + row * D + (size_t)pk * 8, pack8(o));
        }
    }
}

constexpr int PPL = 20;  // packs of 8 per lane in the warp-per-row kernel: D <= 5120

// One warp per row for D <= 32 * 8 * PPL, rows staged in shared memory: each warp owns a
// ring of row slots (the residual and the delta row for the add variant, one slot; two slots
// otherwise); its lane 0 copies the warp's next row in by bulk copies while the warp
// normalises the current one, so a row's bytes are in flight without registers and the warps
// never wait for one another. The weights sit in shared memory, loaded once per CTA; each
// warp walks rows with a grid stride; one CTA of 8 warps per SM.
constexpr int RB_WARPS = 8;
__host__ __device__ constexpr int rb_warps(bool) { return RB_WARPS; }
__host__ __device__ constexpr int rb_stages(bool add) { return add ? 1 : 2; }
__host__ __device__ constexpr int rb_smem(bool add, int D) {
    return D * 2 + rb_warps(add) * rb_stages(add) * (add ? 2 : 1) * D * 2 + 8 * rb_warps(add) * rb_stages(add);
}
template <bool Add>
__global__ void __launch_bounds__(rb_warps(Add) * 32, 1) rms_bulk_kernel(bf16* __restrict__ res, const bf16* __restrict__ delta,
                                                                 const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                                 bf16* __restrict__ out, int rows, int D, float eps,
                                                                 const DevBatch* dyn) {
    constexpr int W = rb_warps(Add), BUFS = Add ? 2 : 1, RB_STAGES = rb_stages(Add);
    extern __shared__ __align__(128) uint8_t rsm[];
    const int packs = D >> 3, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t row_bytes = (uint32_t)D * 2;
    const Pack8* wsm = reinterpret_cast<const Pack8*>(rsm);
    uint8_t* ring = rsm + row_bytes + (size_t)warp * RB_STAGES * BUFS * row_bytes;
    const uint32_t bars = tc::smem_u32(rsm) + row_bytes + W * RB_STAGES * BUFS * row_bytes + 8u * warp * RB_STAGES;
    if (lane == 0)
        for (int st = 0; st < RB_STAGES; st++) tc::mbar_init(bars + 8u * st, 1);
    tc::mbar_fence_init();
    grid_dep_wait();
    grid_dep_launch();
    rows = dyn_rows(dyn, rows);
    for (int i = threadIdx.x; i < packs; i += blockDim.x) reinterpret_cast<Pack8*>(rsm)[i] = ld8(w + (size_t)i * 8);
    __syncthreads();
    const int g0 = blockIdx.x * W + warp, gstep = gridDim.x * W;
    const bf16* src0 = Add ? res : x;
    auto issue = [&](int k) {  // the warp's k-th row into stage k % RB_STAGES
        const int row = g0 + k * gstep, st = k % RB_STAGES;
        const uint32_t bar = bars + 8u * st, dst = tc::smem_u32(ring + (size_t)st * BUFS * row_bytes);
        tc::mbar_expect_tx(bar, BUFS * row_bytes);
        tc::bulk_load(dst, src0 + (size_t)row * D, row_bytes, bar);
        if constexpr (Add) tc::bulk_load(dst + row_bytes, delta + (size_t)row * D, row_bytes, bar);
    };
    if (lane == 0)
        for (int k = 0; k < RB_STAGES && g0 + k * gstep < rows; k++) issue(k);
    int k = 0;
    for (; g0 + k * gstep < rows; k++) {
        const int row = g0 + k * gstep, st = k % RB_STAGES;
        const bool waited = tc::mbar_wait(bars + 8u * st, (uint32_t)(k / RB_STAGES) & 1u);
        if (__any_sync(0xffffffffu, !waited)) {
            if (lane == 0) atomicOr(&g_fault_word, tc::FAULT_WAIT_OTHER);
            break;
        }
        const Pack8* a = reinterpret_cast<const Pack8*>(ring + (size_t)st * BUFS * row_bytes);
        const size_t off = (size_t)row * D;
        Pack8 v[PPL];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < PPL; i++) {
            const int pk = lane + 32 * i;
            if (pk < packs) {
                float f[8];
                if constexpr (Add) {
                    float fb[8];
                    unpack8(a[pk], f);
                    unpack8(a[packs + pk], fb);
#pragma unroll
                    for (int e = 0; e < 8; e++) f[e] += fb[e];
                    v[i] = pack8(f);
                    st8(res + off + (size_t)pk * 8, v[i]);
                    unpack8(v[i], f);
                } else {
                    v[i] = a[pk];
                    unpack8(v[i], f);
                }
#pragma unroll
                for (int e = 0; e < 8; e++) ss = fmaf(f[e], f[e], ss);
            }
        }
        // the stage is read: lane 0 refills it with the warp's row RB_STAGES ahead
        __syncwarp();
        if (lane == 0 && g0 + (k + RB_STAGES) * gstep < rows) {
            tc::fence_async_smem();
            issue(k + RB_STAGES);
        }
        const float inv = rsqrtf(warp_sum(ss) / D + eps);
#pragma unroll
        for (int i = 0; i < PPL; i++) {
            const int pk = lane + 32 * i;
            if (pk < packs) {
                float f[8], wv[8], o[8];
                unpack8(v[i], f);
                unpack8(wsm[pk], wv);
#pragma unroll
                for (int e = 0; e < 8; e++) o[e] = f[e] * inv * (1.f + wv[e]);
                st8(out + off + (size_t)pk * 8, pack8(o));
            }
        }
    }
    if (lane == 0 && g0 + k * gstep < rows) {
        // a wait gave up: the copies still in flight land before the CTA's memory is released
        for (int j = k; j < k + RB_STAGES && g0 + j * gstep < rows; j++)
            (void)tc::mbar_wait(bars + 8u * (j % RB_STAGES), (uint32_t)(j / RB_STAGES) & 1u);
    }
}

// Any D: scalar path, two passes over the row.
template <bool Add>
__global__ void __launch_bounds__(NT) rms_scalar_kernel(bf16* __restrict__ res, const bf16* __restrict__ delta,
                                                        const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                        bf16* __restrict__ out, int D, float eps) {
    __shared__ float scratch[32];
    const size_t row = blockIdx.x;
    const bf16* src = Add ? res : x;
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += NT) {
        float val;
        if constexpr (Add) {
            const bf16 r = to_bf16(f32(res[row * D + i]) + f32(delta[row * D + i]));
            res[row * D + i] = r;
            val = f32(r);
        } else {
            val = f32(src[row * D + i]);
        }
        ss = fmaf(val, val, ss);
    }
    const float inv = rsqrtf(block_sum(ss, scratch) / D + eps);
    for (int i = threadIdx.x; i < D; i += NT) out[row * D + i] = to_bf16(f32(src[row * D + i]) * inv * (1.f + f32(w[i])));
}

constexpr int G_ROWS = 8;  // (token, head) rows per warp and group: half a warp per row of 128

// The gated norm over a grid-stride loop of G_ROWS-row groups per warp, with each lane's
// x and z chunks of the next two groups fetched by cp.async into a per-lane ring of
// shared memory while the current group is computed (each lane reads back only its own
// slots, so no barrier).
constexpr int GA_WARPS = 8, GA_STAGES = 3;
constexpr int GA_SLOTS = G_ROWS;  // per lane and stage: G_ROWS / 2 x chunks, then as many z chunks
constexpr int GA_SMEM = GA_WARPS * GA_STAGES * GA_SLOTS * 32 * 16;

__global__ void __launch_bounds__(GA_WARPS * 32) gated_async_kernel(const bf16* __restrict__ x,
                                                                  const bf16* __restrict__ z, int ldz,
                                                                  const bf16* __restrict__ w, bf16* __restrict__ out,
                                                                  int rows, int H, float eps, const DevBatch* dyn) {
    extern __shared__ Pack8 gring[];  // [GA_WARPS][GA_STAGES][GA_SLOTS][32]
    grid_dep_wait();
    grid_dep_launch();
    if (dyn) rows = min(rows, dyn->rows * H);
    const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4, wib = threadIdx.x >> 5;
    const int groups = (rows + G_ROWS - 1) / G_ROWS;
    const int g0 = blockIdx.x * GA_WARPS + wib, gstep = gridDim.x * GA_WARPS;
    Pack8* ring = gring + (size_t)wib * GA_STAGES * GA_SLOTS * 32 + lane;
    auto issue = [&](int k) {  // the k-th group of this warp into stage k % GA_STAGES
        const int g = g0 + k * gstep;
        Pack8* dst = ring + (k % GA_STAGES) * GA_SLOTS * 32;
#pragma unroll
        for (int i = 0; i < G_ROWS / 2; i++) {
            const int row = g * G_ROWS + 2 * i + half;
            const bool ok = g < groups && row < rows;
            const int r = ok ? row : 0;
            cp_async16_zfill(dst + i * 32, x + (size_t)r * 128 + hl * 8, ok);
            cp_async16_zfill(dst + (G_ROWS / 2 + i) * 32, z + (size_t)(r / H) * ldz + (size_t)(r % H) * 128 + hl * 8,
                             ok);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);
    float2 w2[4];
    {
        const Pack8 wp = ld8(w + hl * 8);
#pragma unroll
        for (int p = 0; p < 4; p++) w2[p] = __bfloat1622float2(wp.h[p]);
    }
    for (int k = 0; g0 + k * gstep < groups; k++) {
        cp_async_wait1();
        issue(k + 2);  // past the end it only commits zero-filled slots of a later stage
        const Pack8* src = ring + (k % GA_STAGES) * GA_SLOTS * 32;
        const int row0 = (g0 + k * gstep) * G_ROWS;
#pragma unroll
        for (int i = 0; i < G_ROWS / 2; i++) {
            const int row = row0 + 2 * i + half;
            const Pack8 xv = src[i * 32], zv = src[(G_ROWS / 2 + i) * 32];
            float2 v[4];
            float ss = 0.f;
#pragma unroll
            for (int p = 0; p < 4; p++) {
                v[p] = __bfloat1622float2(xv.h[p]);
                ss = fmaf(v[p].x, v[p].x, ss);
                ss = fmaf(v[p].y, v[p].y, ss);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = rsqrtf(ss / 128.f + eps);
            const float2 inv2 = make_float2(inv, inv);
            Pack8 o8;
#pragma unroll
            for (int p = 0; p < 4; p++) {
                // bf16(bf16(w * bf16(x * inv)) * silu(z)), lane for lane the scalar roundings
                const float2 y = mul2(rbf2(mul2(rbf2(mul2(v[p], inv2)), w2[p])),
                                      silu2_fast(__bfloat1622float2(zv.h[p])));
                o8.h[p] = __floats2bfloat162_rn(y.x, y.y);
            }
            if (row < rows) st8(out + (size_t)row * 128 + hl * 8, o8);
        }
    }
    cp_async_wait_all();
}

__global__ void gated_scalar_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, int ldz,
                                    const bf16* __restrict__ w, bf16* __restrict__ out, int rows, int H, float eps) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const size_t base = (size_t)row * 128;
    const size_t zb = (size_t)(row / H) * ldz + (size_t)(row % H) * 128;
    float ss = 0.f;
    for (int i = lane; i < 128; i += 32) ss = fmaf(f32(x[base + i]), f32(x[base + i]), ss);
    const float inv = rsqrtf(warp_sum(ss) / 128.f + eps);
    for (int i = lane; i < 128; i += 32)
        out[base + i] = to_bf16(rbf(f32(w[i]) * rbf(f32(x[base + i]) * inv)) * silu_hw(f32(z[zb + i])));
}

bool vec_ok(int D, const void* a, const void* b, const void* c, const void* d) {
    return D % 8 == 0 && D <= 8 * NT * MAXP && aligned16(a) && aligned16(b) && aligned16(c) && aligned16(d);
}

}  // namespace
}  // namespace s1

using namespace s1;

namespace s1 {
namespace {

int rms_norm(const void* x, const void* w, void* out, int rows, int D, float eps, const DevBatch* dyn,
             void* stream) {
    if (rows < 0 || D <= 0) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    auto st = static_cast<cudaStream_t>(stream);
    auto X = static_cast<const bf16*>(x);
    auto Wt = static_cast<const bf16*>(w);
    auto O = static_cast<bf16*>(out);
    if (vec_ok(D, x, w, out, out) && D <= 256 * PPL) {
        static const cudaError_t configured =
            cudaFuncSetAttribute(rms_bulk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 rb_smem(false, 256 * PPL));
        if (configured != cudaSuccess) return configured;
        const int need = (rows + rb_warps(false) - 1) / rb_warps(false);
        return launch_pdl(rms_bulk_kernel<false>, dim3(need < sm_count() ? need : sm_count()),
                          dim3(rb_warps(false) * 32), (size_t)rb_smem(false, D), st, static_cast<bf16*>(nullptr),
                          static_cast<const bf16*>(nullptr), X, Wt, O, rows, D, eps, dyn);
    }
    if (dyn) return cudaErrorInvalidValue;  // the capacity path needs the staged warp-per-row kernel
    if (vec_ok(D, x, w, out, out))
        rms_kernel<false><<<rows, NT, 0, st>>>(nullptr, nullptr, X, Wt, O, D, eps);
    else
        rms_scalar_kernel<false><<<rows, NT, 0, st>>>(nullptr, nullptr, X, Wt, O, D, eps);
    return cudaGetLastError();
}

int add_rms_norm(void* residual, const void* delta, const void* w, void* out, int rows, int D, float eps,
                 const DevBatch* dyn, void* stream) {
    if (rows < 0 || D <= 0) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    auto st = static_cast<cudaStream_t>(stream);
    auto R = static_cast<bf16*>(residual);
    auto Dl = static_cast<const bf16*>(delta);
    auto Wt = static_cast<const bf16*>(w);
    auto O = static_cast<bf16*>(out);
    if (vec_ok(D, residual, delta, w, out) && D <= 256 * PPL) {
        static const cudaError_t configured =
            cudaFuncSetAttribute(rms_bulk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 rb_smem(true, 256 * PPL));
        if (configured != cudaSuccess) return configured;
        const int need = (rows + rb_warps(true) - 1) / rb_warps(true);
        return launch_pdl(rms_bulk_kernel<true>, dim3(need < sm_count() ? need : sm_count()),
                          dim3(rb_warps(true) * 32), (size_t)rb_smem(true, D), st, R, Dl,
                          static_cast<const bf16*>(nullptr), Wt, O, rows, D, eps, dyn);
    }
    if (dyn) return cudaErrorInvalidValue;
    if (vec_ok(D, residual, delta, w, out))
        rms_kernel<true><<<rows, NT, 0, st>>>(R, Dl, nullptr, Wt, O, D, eps);
    else
        rms_scalar_kernel<true><<<rows, NT, 0, st>>>(R, Dl, nullptr, Wt, O, D, eps);
    return cudaGetLastError();
}

int gated_rms_norm(const void* x, const void* z, int ldz, const void* w, void* out, int T, int H, int D, float eps,
                   const DevBatch* dyn, void* stream) {
    if (D != 128 || T < 0 || H <= 0 || ldz < H * D) return cudaErrorInvalidValue;
    const int rows = T * H;
    if (rows == 0) return cudaSuccess;
    constexpr int WARPS = 8;
    auto st = static_cast<cudaStream_t>(stream);
    const uintptr_t bits = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(z) |
                           reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out);
    if (ldz % 8 == 0 && (bits & 15) == 0) {
        static const cudaError_t configured =
            cudaFuncSetAttribute(gated_async_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GA_SMEM);
        if (configured != cudaSuccess) return configured;
        const int groups = (rows + G_ROWS - 1) / G_ROWS;
        const int need = (groups + GA_WARPS - 1) / GA_WARPS;
        const int grid = need < sm_count() * 2 ? need : sm_count() * 2;  // two resident per SM
        return launch_pdl(gated_async_kernel, dim3(grid), dim3(GA_WARPS * 32), GA_SMEM, st,
                          static_cast<const bf16*>(x), static_cast<const bf16*>(z), ldz, static_cast<const bf16*>(w),
                          static_cast<bf16*>(out), rows, H, eps, dyn);
    }
    if (dyn) return cudaErrorInvalidValue;
    // operands not on 16-byte boundaries: one warp per row, scalar accesses
    gated_scalar_kernel<<<(rows + WARPS - 1) / WARPS, WARPS * 32, 0, st>>>(static_cast<const bf16*>(x),
        static_cast<const bf16*>(z), ldz, static_cast<const bf16*>(w), static_cast<bf16*>(out), rows, H, eps);
    return cudaGetLastError();
}

}  // namespace
}  // namespace s1

extern "C" int cs1_rms_norm(const void* x, const void* w, void* out, int rows, int D, float eps, void* stream) {
    return rms_norm(x, w, out, rows, D, eps, nullptr, stream);
}

extern "C" int cs1_add_rms_norm(void* residual, const void* delta, const void* w, void* out, int rows, int D,
                                float eps, void* stream) {
    return add_rms_norm(residual, delta, w, out, rows, D, eps, nullptr, stream);
}

extern "C" int cs1_gated_rms_norm(const void* x, const void* z, int ldz, const void* w, void* out, int T, int H,
                                  int D, float eps, void* stream) {
    return gated_rms_norm(x, z, ldz, w, out, T, H, D, eps, nullptr, stream);
}

extern "C" int cs1_rms_norm_dyn(const void* x, const void* w, void* out, int cap_rows, int D, float eps,
                                const void* desc, void* stream) {
    if (!desc) return cudaErrorInvalidValue;
    return rms_norm(x, w, out, cap_rows, D, eps, static_cast<const DevBatch*>(desc), stream);
}

extern "C" int cs1_add_rms_norm_dyn(void* residual, const void* delta, const void* w, void* out, int cap_rows, int D,
                                    float eps, const void* desc, void* stream) {
    if (!desc) return cudaErrorInvalidValue;
    return add_rms_norm(residual, delta, w, out, cap_rows, D, eps, static_cast<const DevBatch*>(desc), stream);
}

extern "C" int cs1_gated_rms_norm_dyn(const void* x, const void* z, int ldz, const void* w, void* out, int cap_rows,
                                      int H, int D, float eps, const void* desc, void* stream) {
    if (!desc) return cudaErrorInvalidValue;
    return gated_rms_norm(x, z, ldz, w, out, cap_rows, H, D, eps, static_cast<const DevBatch*>(desc), stream);
}
