// Chunked Gated DeltaNet prefill (chunks of 64 tokens, K = V = 128 per head).
//
// Recurrence, per value head h (key head h / (H / HK)), q and k L2-normalised, q scaled:
//   S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T,   o_t = S_t^T q_t
// in the chunk (WY / UT-transform) form of Transformers' torch_chunk_gated_delta_rule:
//   per chunk: cum = cumsum(g); A_ij = beta_i k_i.k_j e^{cum_i - cum_j} (j < i); T = (I + A)^-1
//              u = T diag(beta) v;  w = T diag(beta) (k e^cum);  qd = q e^cum;  kd = k e^{last - cum}
//              P_ij = q_i.k_j e^{cum_i - cum_j} (j <= i)
//   scan:      v_new = u - w S;  o = qd S + P v_new;  S = e^{last} S + kd^T v_new
//
// Two kernels:
//  1. gdn_prep_tc (parallel over chunk x head x sequence): everything that does not
//     depend on the state, written to the workspace in the layouts the scan's
//     tensor-core operands want (qd [64 t][128 k] K-major, w^T [128 k][64 t] and
//     kd [64 t][128 k] read MN-major, P [64 t][64 j], u^T [128 v][64 t]) as bfloat16,
//     plus e^{last} per chunk.
//  2. gdn_scan (one CTA per head x sequence, serial over chunks) on tcgen05:
//     the state is kept transposed, S^T [v][k], so that TMEM lane = value column v
//     and every contraction is an M = 128, K-major MMA:
//        (wS)^T  [v][t] = S^T w^T           (qd S)^T [v][t] = S^T qd^T
//        (P v_new)^T [v][t] += v_new^T P^T   (kd^T v_new)^T [v][k] = v_new^T kd
//     Thread v holds row v of S^T in fp32 registers across chunks, writes its bf16
//     copy to shared memory as the MMA operand, forms v_new = bf16(u - wS) from
//     TMEM, and applies S = e^{last} S + update. w, qd, P, kd^T arrive by TMA,
//     double-buffered one chunk ahead.
// Rounding points follow the reference kernel (gdn_prefill.cu:1-15 of the reference):
// u, w, qd, kd, P, the per-chunk state copy and v_new in bfloat16, state and
// accumulations in fp32.
//
// The FP32 operator (cs1_gdn_prefill_fp32) runs a float32 CUDA-core prep
// (gdn_prep<true>, w [t][k] and kd^T [k][t] layouts) and its own float32 scan.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstring>
#include <new>
#include <type_traits>

#include "common.cuh"
#include "gdn.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(gdn)

namespace s1 {
namespace gdn {

using namespace s1::tc;

bool make_gdn_table(GdnTable& g, const SeqTable& t) {
    g.seq = t;
    int slots = 0;
    for (int i = 0; i < t.count; i++) {
        g.chunk_base[i] = slots;
        const int len = t.offset[i + 1] - t.offset[i];
        slots += (len + C - 1) / C;
    }
    g.chunk_base[t.count] = slots;
    g.max_chunks = (t.max_len + C - 1) / C;
    return true;
}

Layout::Layout(long slots, int H, bool f32) {
    const long e = f32 ? 4 : 2;
    const long n = (long)H * slots;
    long at = 0;
    auto take = [&](long bytes) {
        const long off = at;
        at = (at + bytes + 1023) / 1024 * 1024;
        return off;
    };
    w = take(n * C * K * e);
    qd = take(n * C * K * e);
    p = take(n * C * C * e);
    kdt = take(n * K * C * e);
    ut = take(n * V * C * e);
    decay = take(n * 4);
    total = at;
}

// ---------------------------------------------------------------- prep ----
// 256 threads; shared: kn, qn fp32 [64][129]; A/T fp32 [64][65] x 2; tb fp32 [64][65];
// staged bf16-rounded k e^cum and v as fp32 [64][129].
constexpr int PREP_THREADS = 256;
constexpr int LDK = K + 1;
constexpr int LDC = C + 1;
constexpr int PREP_SMEM = (3 * C * LDK + 3 * C * LDC + 5 * C) * 4;

template <bool F32>
__global__ void __launch_bounds__(PREP_THREADS) gdn_prep(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                          const bf16* __restrict__ v, const float* __restrict__ g,
                                                          const bf16* __restrict__ beta, Work ws, GdnTable tab,
                                                          int H, int HK, float scale) {
    using OutT = typename std::conditional<F32, float, bf16>::type;
    const int seq = blockIdx.z;
    const int start = tab.seq.offset[seq];
    const int len = tab.seq.offset[seq + 1] - start;
    const int c = blockIdx.x;
    if (c * C >= len) return;
    const int h = blockIdx.y, hk = h / (H / HK);
    const long slot = (long)h * ws.slots + tab.chunk_base[seq] + c;
    const int t0 = start + c * C;
    const int n = min(C, len - c * C);

    extern __shared__ float sm[];
    float* kn = sm;                 // [C][LDK] normalised k
    float* qn = kn + C * LDK;       // [C][LDK] normalised, scaled q
    float* st = qn + C * LDK;       // [C][LDK] staging: bf16(k e^cum) then v
    float* A = st + C * LDK;        // [C][LDC]
    float* Tm = A + C * LDC;        // [C][LDC]
    float* tb = Tm + C * LDC;       // [C][LDC]  T diag(beta) (bf16-rounded unless F32)
    float* cum = tb + C * LDC;      // [C]
    float* bet = cum + C;
    float* ecum = bet + C;
    float* erem = ecum + C;
    float* gg = erem + C;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid < C) {
        gg[tid] = tid < n ? g[(size_t)(t0 + tid) * H + h] : 0.f;
        bet[tid] = tid < n ? f32(beta[(size_t)(t0 + tid) * H + h]) : 0.f;
    }
    __syncthreads();
    if (tid == 0) {
        float s = 0.f;
        for (int i = 0; i < C; i++) {
            s += gg[i];
            cum[i] = s;
        }
        ws.decay[slot] = expf(s);
    }
    __syncthreads();
    if (tid < C) {
        ecum[tid] = expf(cum[tid]);
        erem[tid] = expf(cum[C - 1] - cum[tid]);
    }
    // L2 norms: one warp per row, lane covers 4 dims.
    for (int r = warp; r < C; r += PREP_THREADS / 32) {
        float kx[4], qx[4], ks = 0.f, qs = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int d = lane + 32 * e;
            kx[e] = r < n ? f32(k[((size_t)(t0 + r) * HK + hk) * K + d]) : 0.f;
            qx[e] = r < n ? f32(q[((size_t)(t0 + r) * HK + hk) * K + d]) : 0.f;
            ks = fmaf(kx[e], kx[e], ks);
            qs = fmaf(qx[e], qx[e], qs);
        }
        ks = warp_sum(ks);
        qs = warp_sum(qs);
        const float kinv = rsqrtf(ks + 1e-6f), qinv = rsqrtf(qs + 1e-6f) * scale;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int d = lane + 32 * e;
            kn[r * LDK + d] = kx[e] * kinv;
            qn[r * LDK + d] = qx[e] * qinv;
        }
    }
    __syncthreads();

    // Pair products: A (strictly lower, with beta_i and the decay) and P (lower incl. diagonal).
    OutT* P = reinterpret_cast<OutT*>(ws.p) + slot * C * C;
    for (int x = tid; x < C * C; x += PREP_THREADS) {
        const int i = x / C, j = x % C;
        float a = 0.f, p = 0.f;
        if (j <= i) {
            const float* ki = kn + i * LDK;
            const float* qi = qn + i * LDK;
            const float* kj = kn + j * LDK;
            float dk = 0.f, dq = 0.f;
#pragma unroll 8
            for (int d = 0; d < K; d++) {
                dk = fmaf(ki[d], kj[d], dk);
                dq = fmaf(qi[d], kj[d], dq);
            }
            const float dec = expf(cum[i] - cum[j]);
            if (j < i) a = bet[i] * dk * dec;
            p = dq * dec;
        }
        A[i * LDC + j] = a;
        if constexpr (F32) P[x] = p; else P[x] = to_bf16(p);
    }
    __syncthreads();

    // T = (I + A)^-1 by forward substitution, one column per thread.
    if (tid < C) {
        const int j = tid;
        for (int r = 0; r < C; r++) {
            float acc = r == j ? 1.f : 0.f;
            for (int m = j; m < r; m++) acc = fmaf(-A[r * LDC + m], Tm[m * LDC + j], acc);
            Tm[r * LDC + j] = r < j ? 0.f : acc;
        }
    }
    __syncthreads();
    for (int x = tid; x < C * C; x += PREP_THREADS) {
        const int i = x / C, j = x % C;
        const float val = Tm[i * LDC + j] * bet[j];
        tb[i * LDC + j] = F32 ? val : rbf(val);
    }
    // k e^cum staged (bf16-rounded unless F32)
    for (int x = tid; x < C * K; x += PREP_THREADS) {
        const int j = x / K, d = x % K;
        const float val = kn[j * LDK + d] * ecum[j];
        st[j * LDK + d] = F32 ? val : rbf(val);
    }
    __syncthreads();

    // w[t][d] = sum_j tb[t][j] kw[j][d]; thread: d = tid % 128, rows t = tid/128 + 2i
    OutT* W = reinterpret_cast<OutT*>(ws.w) + slot * C * K;
    {
        const int d = tid & 127, tg = tid >> 7;
        for (int t = tg; t < C; t += 2) {
            float acc = 0.f;
            for (int j = 0; j <= t; j++) acc = fmaf(tb[t * LDC + j], st[j * LDK + d], acc);
            if constexpr (F32) W[t * K + d] = acc; else W[t * K + d] = to_bf16(acc);
        }
    }
    // qd[t][d] and kd^T[d][t]
    OutT* QD = reinterpret_cast<OutT*>(ws.qd) + slot * C * K;
    OutT* KDT = reinterpret_cast<OutT*>(ws.kdt) + slot * K * C;
    for (int x = tid; x < C * K; x += PREP_THREADS) {
        const int t = x / K, d = x % K;
        const float a = qn[t * LDK + d] * ecum[t];
        if constexpr (F32) QD[x] = a; else QD[x] = to_bf16(a);
        const int d2 = x / C, t2 = x % C;
        const float b = kn[t2 * LDK + d2] * erem[t2];
        if constexpr (F32) KDT[x] = b; else KDT[x] = to_bf16(b);
    }
    __syncthreads();
    // v staged, then u^T[v][t] = sum_j tb[t][j] v[j][v]
    for (int x = tid; x < C * V; x += PREP_THREADS) {
        const int j = x / V, d = x % V;
        st[j * LDK + d] = j < n ? f32(v[((size_t)(t0 + j) * H + h) * V + d]) : 0.f;
    }
    __syncthreads();
    OutT* UT = reinterpret_cast<OutT*>(ws.ut) + slot * V * C;
    {
        const int d = tid & 127, tg = tid >> 7;
        for (int t = tg; t < C; t += 2) {
            float acc = 0.f;
            for (int j = 0; j <= t; j++) acc = fmaf(tb[t * LDC + j], st[j * LDK + d], acc);
            if constexpr (F32) UT[d * C + t] = acc; else UT[d * C + t] = to_bf16(acc);
        }
    }
}

// ------------------------------------------------------- prep on tcgen05 ----
// One CTA (256 threads, 2 per SM) per (chunk slot, head) over all packed sequences;
// every operand is used in the layout it is produced in (no transposes):
//  1. v arrives by TMA in an MN-major bf16 tile (rows = token j). Each warp loads 8 rows
//     of q and k (8-byte lane accesses) and normalises them (k / |k|, q / |q| * scale)
//     into a K-major TF32 operand tile (128B swizzle) while one thread forms the
//     sequential fp32 cumsum of g. MMA1 is issued, then qd = bf16(qn e^cum) and
//     kd = bf16(kn e^(last-cum)) go to the workspace and kw = bf16(kn e^cum) into an
//     MN-major operand tile.
//  2. MMA1 (kind::tf32, M=128, N=64, K=128): D[i][j] = [kn;qn]_i . kn_j in TMEM, read by
//     all 8 warps (one column half each): lanes 0..63 give A_ij = beta_i kk_ij
//     e^(cum_i-cum_j) (j < i); lanes 64..127 give P_tj = qk_tj e^(cum_t-cum_j) (j <= t),
//     staged as bf16 and stored as one contiguous 8 KB tile.
//  3. T = (I + A)^-1 blockwise on CUDA cores in fp32: 16x16 diagonal substitutions, then
//     block rows T_ij = -T_ii sum_k A_ik T_kj in 4-column register tiles (each sum in the
//     order of the plain loops); tb = bf16(T diag(beta)) as a K-major tile.
//  4. MMA2 (kind::f16, A MN-major, M=128, N=64, K=64): u^T = v^T tb^T and w^T = kw^T tb^T;
//     the TMEM rows are staged in shared memory and stored as contiguous 16 KB tiles.
// Rows past a sequence's end have beta = 0, so their tb columns are zero and whatever v
// rows the TMA brings there (the next sequence's, or zero fill) do not reach u.
// Workspace layouts written: qd [t][k], kd [t][k], P [t][j], u^T [v][t], w^T [k][t].
constexpr int TP_THREADS = 256;
constexpr int LDT = C + 4;                       // fp32 row stride of A and T (16-byte aligned rows)
constexpr int TP_KQ = 0;                         // 4 x [128][32 fp32] = 64 KB; then A, T, scratch; then u^T / w^T staging
constexpr int TP_KW = 65536;                     // kw, MN-major: 2 blocks x [64 j][64 d] bf16 = 16 KB
constexpr int TP_VB = TP_KW + 16384;             // v,  MN-major: 2 blocks x [64 j][64 v] bf16 = 16 KB
constexpr int TP_TB = TP_VB + 16384;             // P staging, then tb K-major [64 t][64 j] bf16 = 8 KB
constexpr int TP_VEC = TP_TB + 8192;             // cum, bet, ecum, erem, gg [64] each
constexpr int TP_BAR = TP_VEC + 5 * C * 4;
constexpr int TP_SMEM = TP_BAR + 64 + 1024;
constexpr int TP_A = 0;                          // inside the KQ region once MMA1 is done
constexpr int TP_T = TP_A + C * LDT * 4;
constexpr int TP_S = TP_T + C * LDT * 4;         // inverse scratch [3][16][16] fp32
constexpr uint32_t MN_BLOCK = 8192;              // 64 K-rows x 128 B: stride between 64-wide MN blocks

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Byte offset of bf16 element (k_row, mn) in an MN-major 128B-swizzled tile made of
// 64-wide MN blocks of [64 K-rows][128 B].
__device__ __forceinline__ uint32_t mn_off(int krow, int mn) {
    return (uint32_t)(mn >> 6) * MN_BLOCK + sw128_offset(krow, (mn & 63) >> 3) + (uint32_t)((mn & 7) << 1);
}

__global__ void __launch_bounds__(TP_THREADS, 2)
    gdn_prep_tc(const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q, const bf16* __restrict__ k,
                const float* __restrict__ g, const bf16* __restrict__ beta, Work ws, GdnTable tab, int H, int HK,
                float scale) {
    // blockIdx.x enumerates the chunk slots of all packed sequences (no idle CTAs)
    const int slot_in_pack = blockIdx.x;
    int seq = 0;
    {
        int lo = 0, hi = tab.seq.count - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (tab.chunk_base[mid] <= slot_in_pack) lo = mid; else hi = mid - 1;
        }
        seq = lo;
    }
    const int start = tab.seq.offset[seq];
    const int len = tab.seq.offset[seq + 1] - start;
    const int c = slot_in_pack - tab.chunk_base[seq];
    const int h = blockIdx.y, hk = h / (H / HK);
    const long slot = (long)h * ws.slots + slot_in_pack;
    const int t0 = start + c * C;
    const int n = min(C, len - c * C);

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* sm = smem_raw + (base - raw);
    float* A = reinterpret_cast<float*>(sm + TP_A);
    float* Tm = reinterpret_cast<float*>(sm + TP_T);
    float* S = reinterpret_cast<float*>(sm + TP_S);
    float* cum = reinterpret_cast<float*>(sm + TP_VEC);
    float* bet = cum + C;
    float* ecum = bet + C;
    float* erem = ecum + C;
    float* gg = erem + C;
    const uint32_t bar = base + TP_BAR, vbar = base + TP_BAR + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + TP_BAR + 16);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    grid_dep_wait();
    grid_dep_launch();
    // global loads first: g and beta of the chunk, this warp's 8 rows of k and q
    float gval = 0.f, bval = 0.f;
    if (tid < n) {
        gval = g[(size_t)(t0 + tid) * H + h];
        bval = f32(beta[(size_t)(t0 + tid) * H + h]);
    }
    const int d0 = lane * 4;
    uint2 kr[8], qr[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = warp * 8 + i;
        if (r < n) {
            kr[i] = *reinterpret_cast<const uint2*>(k + ((size_t)(t0 + r) * HK + hk) * K + d0);
            qr[i] = *reinterpret_cast<const uint2*>(q + ((size_t)(t0 + r) * HK + hk) * K + d0);
        } else {
            kr[i] = make_uint2(0u, 0u);
            qr[i] = make_uint2(0u, 0u);
        }
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_init(vbar, 1);
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), 256);
        tmem_relinquish();
    }
    if (tid < C) {
        gg[tid] = gval;
        bet[tid] = bval;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) {
        // v rows t0..t0+63 of head h into the MN-major tile
        mbar_expect_tx(vbar, 2 * MN_BLOCK);
        tma_load_3d(base + TP_VB, &vmap, vbar, 0, h, t0);
        tma_load_3d(base + TP_VB + MN_BLOCK, &vmap, vbar, 64, h, t0);
        // sequential fp32 sum (the reference's order), from registers
        float gv[C];
#pragma unroll
        for (int i = 0; i < C; i++) gv[i] = gg[i];
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < C; i++) {
            s += gv[i];
            cum[i] = s;
        }
        ws.decay[slot] = expf(s);
    }
    // 1. norms and the TF32 operand rows: dims d0..d0+3 = one 16-byte chunk of sub-tile d0 / 32
    float kinv[8], qinv[8];
    const uint32_t chunk = (uint32_t)((d0 & 31) >> 2);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = warp * 8 + i;
        float kx[4], qx[4];
        const __nv_bfloat162* kp = reinterpret_cast<const __nv_bfloat162*>(&kr[i]);
        const __nv_bfloat162* qp = reinterpret_cast<const __nv_bfloat162*>(&qr[i]);
        const float2 k01 = __bfloat1622float2(kp[0]), k23 = __bfloat1622float2(kp[1]);
        const float2 q01 = __bfloat1622float2(qp[0]), q23 = __bfloat1622float2(qp[1]);
        kx[0] = k01.x; kx[1] = k01.y; kx[2] = k23.x; kx[3] = k23.y;
        qx[0] = q01.x; qx[1] = q01.y; qx[2] = q23.x; qx[3] = q23.y;
        float ks = 0.f, qs = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            ks = fmaf(kx[e], kx[e], ks);
            qs = fmaf(qx[e], qx[e], qs);
        }
        ks = warp_sum(ks);
        qs = warp_sum(qs);
        kinv[i] = rsqrtf(ks + 1e-6f);
        qinv[i] = rsqrtf(qs + 1e-6f) * scale;
        *reinterpret_cast<float4*>(sm + TP_KQ + (d0 >> 5) * 16384 + sw128_offset(r, chunk)) =
            make_float4(tf32_rna(kx[0] * kinv[i]), tf32_rna(kx[1] * kinv[i]), tf32_rna(kx[2] * kinv[i]),
                        tf32_rna(kx[3] * kinv[i]));
        *reinterpret_cast<float4*>(sm + TP_KQ + (d0 >> 5) * 16384 + sw128_offset(C + r, chunk)) =
            make_float4(tf32_rna(qx[0] * qinv[i]), tf32_rna(qx[1] * qinv[i]), tf32_rna(qx[2] * qinv[i]),
                        tf32_rna(qx[3] * qinv[i]));
    }
    fence_async_smem();
    __syncthreads();  // cum and the TF32 tile are complete
    if (tid == 0) {
        tc_fence_after();
        constexpr uint32_t ID = idesc(128, 64, AB_TF32);
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            const uint32_t a = base + TP_KQ + (uint32_t)(kk >> 2) * 16384 + (uint32_t)(kk & 3) * 32;
            mma_tf32(tmem, desc_sw128(a), desc_sw128(a), ID, kk > 0);
        }
        mma_commit(bar);
    }
    if (tid < C) {
        ecum[tid] = expf(cum[tid]);
        erem[tid] = expf(cum[C - 1] - cum[tid]);
    }
    __syncthreads();
    {
        bf16* QD = static_cast<bf16*>(ws.qd) + slot * C * K;
        bf16* KD = static_cast<bf16*>(ws.kdt) + slot * C * K;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = warp * 8 + i;
            float kn[4], qn[4];
            const __nv_bfloat162* kp = reinterpret_cast<const __nv_bfloat162*>(&kr[i]);
            const __nv_bfloat162* qp = reinterpret_cast<const __nv_bfloat162*>(&qr[i]);
            const float2 k01 = __bfloat1622float2(kp[0]), k23 = __bfloat1622float2(kp[1]);
            const float2 q01 = __bfloat1622float2(qp[0]), q23 = __bfloat1622float2(qp[1]);
            kn[0] = k01.x * kinv[i]; kn[1] = k01.y * kinv[i]; kn[2] = k23.x * kinv[i]; kn[3] = k23.y * kinv[i];
            qn[0] = q01.x * qinv[i]; qn[1] = q01.y * qinv[i]; qn[2] = q23.x * qinv[i]; qn[3] = q23.y * qinv[i];
            const float ec = ecum[r], er = erem[r];
            uint2 o;
            o.x = pack_bf16x2(qn[0] * ec, qn[1] * ec);
            o.y = pack_bf16x2(qn[2] * ec, qn[3] * ec);
            *reinterpret_cast<uint2*>(QD + (size_t)r * K + d0) = o;
            o.x = pack_bf16x2(kn[0] * er, kn[1] * er);
            o.y = pack_bf16x2(kn[2] * er, kn[3] * er);
            *reinterpret_cast<uint2*>(KD + (size_t)r * K + d0) = o;
            o.x = pack_bf16x2(kn[0] * ec, kn[1] * ec);
            o.y = pack_bf16x2(kn[2] * ec, kn[3] * ec);
            *reinterpret_cast<uint2*>(sm + TP_KW + mn_off(r, d0)) = o;
        }
    }
    fence_async_smem();  // kw is read by MMA2
    bool ok = mbar_wait(bar, 0);  // every thread: MMA1 done, the KQ region is free
    if (!ok && lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
    tc_fence_after();
    // 2. A rows (TMEM lanes 0..63) and P rows (lanes 64..127); warp w reads lane quarter
    //    w % 4, columns 32 * (w / 4) .. +31
    {
        const int q4 = warp & 3, j0 = (warp >> 2) * 32;
        const int row = q4 * 32 + lane;
        float d[32];
        tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)j0, d);
        tmem_ld_wait();
        if (row < C) {
            const int i = row;
            const float ci = cum[i], bi = bet[i];
            float* arow = A + i * LDT + j0;
#pragma unroll
            for (int j4 = 0; j4 < 8; j4++) {
                float f[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int j = j0 + j4 * 4 + e;
                    f[e] = j < i ? bi * d[j4 * 4 + e] * __expf(ci - cum[j]) : 0.f;
                }
                *reinterpret_cast<float4*>(arow + j4 * 4) = make_float4(f[0], f[1], f[2], f[3]);
            }
        } else {
            const int t = row - C;
            const float ct = cum[t];
#pragma unroll
            for (int c8 = 0; c8 < 4; c8++) {
                float f[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int j = j0 + c8 * 8 + e;
                    f[e] = j <= t ? d[c8 * 8 + e] * __expf(ct - cum[j]) : 0.f;
                }
                const int ch = (j0 >> 3) + c8;  // 16-byte chunk of the 128-byte P row
                *reinterpret_cast<Pack8*>(sm + TP_TB + t * 128 + ((ch ^ (t & 7)) << 4)) = pack8(f);
            }
        }
    }
    __syncthreads();
    {
        bf16* P = static_cast<bf16*>(ws.p) + slot * C * C;
        for (int u = tid; u < C * C / 8; u += TP_THREADS) {
            const int t = u >> 3, c8 = u & 7;
            st8(P + t * C + c8 * 8, *reinterpret_cast<const Pack8*>(sm + TP_TB + t * 128 + ((c8 ^ (t & 7)) << 4)));
        }
    }
    // 3. T = (I + A)^-1. Diagonal 16x16 blocks: one thread per (block, column).
    if (tid < C) {
        const int b = tid >> 4, col = tid & 15, o = b * 16;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; r++) {
            float acc = r == col ? 1.f : 0.f;
#pragma unroll
            for (int m = 0; m < r; m++) acc = fmaf(-A[(o + r) * LDT + o + m], x[m], acc);
            x[r] = r < col ? 0.f : acc;
        }
#pragma unroll
        for (int r = 0; r < 16; r++) Tm[(o + r) * LDT + o + col] = x[r];
    }
    for (int x = tid; x < C * C; x += TP_THREADS) {
        const int i = x / C, j = x % C;
        if ((j >> 4) > (i >> 4)) Tm[i * LDT + j] = 0.f;
    }
    __syncthreads();
    // block rows bi = 1..3: S_bj = sum_{kb = bj}^{bi-1} A_(bi,kb) T_(kb,bj), then
    // T_(bi,bj) = -T_(bi,bi) S_bj; thread = (bj, row r, 4 columns)
#pragma unroll
    for (int bi = 1; bi < 4; bi++) {
        const int bj = tid >> 6, r = (tid >> 2) & 15, c4 = (tid & 3) * 4;
        if (tid < bi * 64) {
            const float* arow = A + (16 * bi + r) * LDT;
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            for (int kb = bj; kb < bi; kb++) {
#pragma unroll
                for (int m = 0; m < 16; m++) {
                    const float av = arow[16 * kb + m];
                    const float4 tv = *reinterpret_cast<const float4*>(Tm + (16 * kb + m) * LDT + 16 * bj + c4);
                    a0 = fmaf(av, tv.x, a0);
                    a1 = fmaf(av, tv.y, a1);
                    a2 = fmaf(av, tv.z, a2);
                    a3 = fmaf(av, tv.w, a3);
                }
            }
            *reinterpret_cast<float4*>(S + (bj * 16 + r) * 16 + c4) = make_float4(a0, a1, a2, a3);
        }
        __syncthreads();
        if (tid < bi * 64) {
            const float* trow = Tm + (16 * bi + r) * LDT + 16 * bi;
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int m = 0; m < 16; m++) {
                if (m <= r) {
                    const float tv = trow[m];
                    const float4 sv = *reinterpret_cast<const float4*>(S + (bj * 16 + m) * 16 + c4);
                    a0 = fmaf(tv, sv.x, a0);
                    a1 = fmaf(tv, sv.y, a1);
                    a2 = fmaf(tv, sv.z, a2);
                    a3 = fmaf(tv, sv.w, a3);
                }
            }
            *reinterpret_cast<float4*>(Tm + (16 * bi + r) * LDT + 16 * bj + c4) = make_float4(-a0, -a1, -a2, -a3);
        }
        __syncthreads();
    }
    // tb = bf16(T diag(beta)), K-major [64 t][64 j]
    for (int u = tid; u < C * C / 8; u += TP_THREADS) {
        const int t = u >> 3, j0 = (u & 7) * 8;
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = Tm[t * LDT + j0 + e] * bet[j0 + e];
        *reinterpret_cast<Pack8*>(sm + TP_TB + sw128_offset(t, j0 >> 3)) = pack8(f);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        if (!mbar_wait(vbar, 0)) atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
        constexpr uint32_t ID = idesc_major(128, 64, AB_BF16, 1, 0);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint64_t bdesc = desc_sw128(base + TP_TB + (uint32_t)kk * 32);
            const uint32_t koff = (uint32_t)kk * 2048;
            mma_bf16(tmem + 64, desc_sw128_mn(base + TP_VB + koff, MN_BLOCK, 1024), bdesc, ID, kk > 0);
            mma_bf16(tmem + 128, desc_sw128_mn(base + TP_KW + koff, MN_BLOCK, 1024), bdesc, ID, kk > 0);
        }
        mma_commit(bar);
    }
    __syncwarp();
    if (!mbar_wait(bar, 1)) {
        if (lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
    }
    tc_fence_after();
    // 4. u^T rows (warps 0-3) and w^T rows (warps 4-7) staged in the free KQ region
    {
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;  // TMEM lane = v (u^T) or k (w^T)
        float x[64];
        const uint32_t col = warp < 4 ? 64u : 128u;
        tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + col, *reinterpret_cast<float(*)[32]>(x));
        tmem_ld32(tmem + ((uint32_t)(q4 * 32) << 16) + col + 32, *reinterpret_cast<float(*)[32]>(x + 32));
        tmem_ld_wait();
        uint8_t* stg = sm + TP_KQ + (warp < 4 ? 0 : 16384) + row * 128;
#pragma unroll
        for (int c8 = 0; c8 < 8; c8++) *reinterpret_cast<Pack8*>(stg + ((c8 ^ (row & 7)) << 4)) = pack8(x + c8 * 8);
    }
    __syncthreads();
    // one contiguous 16 KB tile each: u^T [128 v][64 t] and w^T [128 k][64 t]
    for (int u = tid; u < 2 * V * C / 8; u += TP_THREADS) {
        const int which = u >> 10, row = (u >> 3) & 127, c8 = u & 7;
        bf16* dst = static_cast<bf16*>(which ? ws.w : ws.ut) + (slot * V + row) * C + c8 * 8;
        st8(dst, *reinterpret_cast<const Pack8*>(sm + TP_KQ + which * 16384 + row * 128 + ((c8 ^ (row & 7)) << 4)));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ---------------------------------------------------------------- scan ----
// One CTA per (head, sequence), longest sequences first; two CTAs per SM.
// 160 threads: warps 0..3 own TMEM lanes = value columns 0..127, warp 4 lane 0 issues TMA
// and MMA. The fp32 state S^T [v][k] lives in tensor memory (columns 128..255) and is
// accumulated there by the update MMA; per chunk each thread reads its state row, writes
// the bf16 copy the next MMAs read from shared memory, and writes back e^{last} S before
// the update MMA adds (kd^T v_new)^T onto it.
// TMEM columns: [0,64) (wS)^T, [64,128) o^T, [128,256) S^T.
// Shared memory (1024-aligned tiles, 128B swizzle):
//   ST   S^T bf16 [128 v][128 k] as two [128][64] K-major sub-tiles     32 KB
//   VN   v_new^T bf16 [128 v][64 t] K-major                             16 KB
//   one operand buffer: W = w^T [128 k][64 t] MN-major, QD [64 t][128 k] K-major
//   (2 sub-tiles), P [64 t][64 j] K-major, KD [64 t][128 k] MN-major (2 blocks)   56 KB
constexpr int SCAN_THREADS = 160;
constexpr int SUB64 = 64 * 128;        // bytes of a [64 rows][64 bf16] tile
constexpr int SUB128 = 128 * 128;      // bytes of a [128 rows][64 bf16] tile
constexpr int OFF_ST = 0;
constexpr int OFF_VN = OFF_ST + 2 * SUB128;
constexpr int OFF_BUF = OFF_VN + SUB128;
constexpr int BUF_W = 0, BUF_QD = 2 * SUB64, BUF_P = 4 * SUB64, BUF_KDT = 5 * SUB64;
constexpr int BUF_BYTES = 5 * SUB64 + SUB128;
constexpr int OFF_BAR = OFF_BUF + BUF_BYTES;
constexpr int SCAN_SMEM = OFF_BAR + 128 + 1024;
constexpr uint32_t TX_BYTES = BUF_BYTES;

struct ScanMaps {
    CUtensorMap w, qd, p, kdt;
};

__global__ void __launch_bounds__(SCAN_THREADS, 2)
    gdn_scan(const __grid_constant__ ScanMaps maps, Work ws, GdnTable tab, bf16* __restrict__ o, int H,
             const float* __restrict__ s_in, long s_in_stride, float* __restrict__ s_out) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + OFF_BAR;
    const uint32_t full = bars, empty = bars + 8;
    const uint32_t s_ready = bars + 16, ws_done = bars + 24, vn_ready = bars + 32, upd_done = bars + 40;
    const uint32_t drain = bars + 48;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 64);

    const int h = blockIdx.x, seq = tab.seq.order[blockIdx.y];
    const int start = tab.seq.offset[seq];
    const int len = tab.seq.offset[seq + 1] - start;
    const int NC = (len + C - 1) / C;
    const long slot0 = (long)h * ws.slots + tab.chunk_base[seq];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(full, 1);
        mbar_init(empty, 1);
        mbar_init(s_ready, 4);  // one arrive per epilogue warp
        mbar_init(ws_done, 1);
        mbar_init(vn_ready, 4);
        mbar_init(upd_done, 1);
        mbar_init(drain, 1);
        mbar_fence_init();
    }
    if (warp == 4) {
        tmem_alloc(smem_u32(tmem_slot), 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 4) {
        if (lane == 0) {
            constexpr uint32_t ID64 = idesc(128, 64, AB_BF16);
            constexpr uint32_t ID64_BMN = idesc_major(128, 64, AB_BF16, 0, 1);
            constexpr uint32_t ID128_BMN = idesc_major(128, 128, AB_BF16, 0, 1);
            const uint32_t buf = base + OFF_BUF;
            auto issue_load = [&](int c) {
                const int row = (int)((slot0 + c) * C);
                mbar_expect_tx(full, TX_BYTES);
                tma_load_2d(buf + BUF_W, &maps.w, full, 0, (int)((slot0 + c) * K));  // w^T [128 k][64 t]
                tma_load_2d(buf + BUF_QD, &maps.qd, full, 0, row);
                tma_load_2d(buf + BUF_QD + SUB64, &maps.qd, full, 64, row);
                tma_load_2d(buf + BUF_P, &maps.p, full, 0, row);
                tma_load_2d(buf + BUF_KDT, &maps.kdt, full, 0, row);  // kd [64 t][128 k], two 64-wide blocks
                tma_load_2d(buf + BUF_KDT + SUB64, &maps.kdt, full, 64, row);
            };
            int issued = 0;
            if (NC > 0) issue_load(0), issued++;
            for (int c = 0; c < NC; c++) {
                const uint32_t cp = (uint32_t)c & 1u;
                if (!mbar_wait(full, cp) || !mbar_wait(s_ready, cp)) {
                    atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                    break;
                }
                tc_fence_after();
                // (wS)^T -> cols [0,64), (qd S)^T -> cols [64,128); K = 128 over two sub-tiles
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t sub = (uint32_t)(kk >> 2), off = (uint32_t)(kk & 3) * 32;
                    const uint64_t a = desc_sw128(base + OFF_ST + sub * SUB128 + off);
                    mma_bf16(tmem + 0, a, desc_sw128_mn(buf + BUF_W + (uint32_t)kk * 2048, SUB64, 1024), ID64_BMN,
                             kk > 0);
                    mma_bf16(tmem + 64, a, desc_sw128(buf + BUF_QD + sub * SUB64 + off), ID64, kk > 0);
                }
                mma_commit(ws_done);
                if (!mbar_wait(vn_ready, cp)) {
                    atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                    break;
                }
                tc_fence_after();
                // o^T += v_new^T P^T ; S^T += v_new^T kd  (K = 64 tokens; S^T holds e^{last} S)
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t off = (uint32_t)kk * 32;
                    const uint64_t a = desc_sw128(base + OFF_VN + off);
                    mma_bf16(tmem + 64, a, desc_sw128(buf + BUF_P + off), ID64, 1);
                    mma_bf16(tmem + 128, a, desc_sw128_mn(buf + BUF_KDT + (uint32_t)kk * 2048, SUB64, 1024),
                             ID128_BMN, 1);
                }
                mma_commit(upd_done);
                mma_commit(empty);
                if (c + 1 < NC) {
                    if (!mbar_wait(empty, cp)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                        break;
                    }
                    issue_load(c + 1);
                    issued++;
                }
            }
            mma_commit(drain);
            (void)mbar_wait(drain, 0);
            if (issued > 0) (void)mbar_wait(full, (uint32_t)(issued - 1) & 1u);
        }
    } else {
        // Thread v = threadIdx.x owns TMEM lane v: row v of S^T and column v of o.
        const int vcol = threadIdx.x;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        {
            // initial state into TMEM (zero or s_in column v)
            const float* si = s_in ? s_in + (long)seq * s_in_stride + (size_t)h * K * V : nullptr;
#pragma unroll
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = si ? si[(size_t)(q4 * 32 + i) * V + vcol] : 0.f;
                tmem_st32(lane_addr + 128 + q4 * 32, x);
            }
            tmem_st_wait();
        }
        const bf16* UT = reinterpret_cast<const bf16*>(ws.ut);
        uint8_t* st_tile = smem + OFF_ST;
        uint8_t* vn_tile = smem + OFF_VN;
        uint4 ur4[8];  // this chunk's u^T row (128 bytes)
        auto load_u = [&](int c) {
            const uint4* ur = reinterpret_cast<const uint4*>(UT + ((slot0 + c) * V + vcol) * C);
#pragma unroll
            for (int i = 0; i < 8; i++) ur4[i] = ur[i];
        };
        // Chunk c's pass over the state row: the bf16 copy the first MMAs read, then e^{last} S
        // written back for the update MMA; one arrive per warp on s_ready.
        auto state_pass = [&](int c) {
            const float dec = ws.decay[slot0 + c];
#pragma unroll
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
                tmem_ld32(lane_addr + 128 + q4 * 32, x);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int ch = q4 * 4 + i;  // 16-byte chunk of the 256-byte row
                    *reinterpret_cast<Pack8*>(st_tile + (ch >> 3) * SUB128 + sw128_offset(vcol, ch & 7)) =
                        pack8(x + i * 8);
                }
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] *= dec;
                tmem_st32(lane_addr + 128 + q4 * 32, x);
            }
            tmem_st_wait();
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_ready);
        };
        if (NC > 0) {
            load_u(0);
            state_pass(0);
        }
        for (int c = 0; c < NC; c++) {
            const uint32_t cp = (uint32_t)c & 1u;
            // A wait that gives up does not leave the loop on its own: the group decides
            // together at the named barrier below, so no thread waits there for one that left.
            // tcgen05.ld is warp-collective: the wait outcome is made warp-uniform
            bool ok = __all_sync(0xffffffffu, mbar_wait(ws_done, cp));
            tc_fence_after();
            // v_new = bf16(u - wS)
#pragma unroll
            for (int half = 0; half < 2; half++) {
                if (!ok) break;  // warp-uniform
                float ws_[32];
                tmem_ld32(lane_addr + half * 32, ws_);
                float u[32];
#pragma unroll
                for (int i = 0; i < 4; i++) unpack8(*reinterpret_cast<const Pack8*>(&ur4[half * 4 + i]), u + i * 8);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) f[e] = u[i * 8 + e] - ws_[i * 8 + e];
                    *reinterpret_cast<Pack8*>(vn_tile + sw128_offset(vcol, half * 4 + i)) = pack8(f);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(vn_ready);
            ok = __all_sync(0xffffffffu, ok && mbar_wait(upd_done, cp));
            tc_fence_after();
            // o rows of this chunk into the v_new tile (free: the update MMAs have read it) right
            // away -- the next chunk's first MMAs rewrite these TMEM columns -- then the next
            // chunk's state pass (it gates those MMAs); the o rows leave as 16-byte row segments
            // while the MMAs run
            const int rows = min(C, len - c * C);
            bf16* ost = reinterpret_cast<bf16*>(vn_tile);
            if (ok) {  // warp-uniform
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float ov[32];
                    tmem_ld32(lane_addr + 64 + half * 32, ov);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) ost[(half * 32 + i) * V + vcol] = to_bf16(ov[i]);
                }
            }
            if (ok && c + 1 < NC) {
                load_u(c + 1);
                state_pass(c + 1);
            }
            if (bar_any(1, 128, !ok)) {
                atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
                break;
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int u = vcol + i * 128;  // 16-byte unit: row u / 16, columns (u % 16) * 8
                const int t = u >> 4, v8 = (u & 15) * 8;
                if (t < rows)
                    st8(o + ((size_t)(start + c * C + t) * H + h) * V + v8,
                        *reinterpret_cast<const Pack8*>(ost + t * V + v8));
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the tile takes the next v_new
        }
        if (s_out) {
            float* so = s_out + (long)seq * (long)H * K * V + (size_t)h * K * V;
#pragma unroll
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
                tmem_ld32(lane_addr + 128 + q4 * 32, x);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) so[(size_t)(q4 * 32 + i) * V + vcol] = x[i];
            }
        }
        tc_fence_before();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// The bf16 prefill: the fused kernel (gdn_fused.cu), which needs no workspace.
int run(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o, void* workspace,
        size_t workspace_bytes, const SeqTable& seqs, int H, int HK, float scale, const void* s_in,
        long s_in_stride, void* s_out, cudaStream_t st) {
    (void)workspace;
    (void)workspace_bytes;
    return run_fused(q, k, v, g, beta, o, seqs, H, HK, scale, s_in, s_in_stride, s_out, st);
}

// The two-kernel form (gdn_prep_tc, then gdn_scan) with its tiles in a caller-provided
// workspace. Zero-token sequences never reach the kernels; s_out for an empty call is a copy.
int run_two_pass(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                 void* workspace, size_t workspace_bytes, const SeqTable& seqs, int H, int HK, float scale,
                 const void* s_in, long s_in_stride, void* s_out, cudaStream_t st) {
    if (!q || !k || !v || !g || !beta || !o || !workspace || H <= 0 || HK <= 0 || H % HK) return cudaErrorInvalidValue;
    GdnTable tab;
    make_gdn_table(tab, seqs);
    const long slots = tab.chunk_base[seqs.count];
    const Layout L(slots, H, false);
    if ((size_t)L.total > workspace_bytes) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(workspace) & 1023) != 0) return cudaErrorInvalidValue;
    static const cudaError_t configured = [] {
        cudaError_t e = cudaFuncSetAttribute(gdn_prep_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TP_SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN_SMEM);
        return e;
    }();
    if (configured != cudaSuccess) return configured;
    uint8_t* b = static_cast<uint8_t*>(workspace);
    Work ws{b + L.w, b + L.qd, b + L.p, b + L.kdt, b + L.ut, reinterpret_cast<float*>(b + L.decay), slots};
    CUtensorMap vmap;
    if (int e = host::make_map_3d_bf16(&vmap, v, V, H, (uint64_t)seqs.offset[seqs.count], V, (uint64_t)H * V, 64, 64))
        return e;
    cudaError_t e = launch_pdl(gdn_prep_tc, dim3((unsigned)slots, H), dim3(TP_THREADS), TP_SMEM, st, vmap,
                               static_cast<const bf16*>(q), static_cast<const bf16*>(k), g,
                               static_cast<const bf16*>(beta), ws, tab, H, HK, scale);
    if (e != cudaSuccess) return e;
    ScanMaps maps;
    const uint64_t rows64 = (uint64_t)H * slots * C, rows128 = (uint64_t)H * slots * K;
    int r = host::make_map_2d(&maps.w, ws.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows128, C, C, 128, 64,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (!r) r = host::make_map_2d(&maps.qd, ws.qd, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows64, K, K, 64, 64,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (!r) r = host::make_map_2d(&maps.p, ws.p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows64, C, C, 64, 64,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (!r) r = host::make_map_2d(&maps.kdt, ws.kdt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows64, K, K, 64, 64,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (r) return r;
    return launch_pdl(gdn_scan, dim3(H, seqs.count), dim3(SCAN_THREADS), SCAN_SMEM, st, maps, ws, tab,
                      static_cast<bf16*>(o), H, static_cast<const float*>(s_in), s_in_stride,
                      static_cast<float*>(s_out));
}

size_t workspace_bytes_for(long slots, int H, bool f32) { return (size_t)Layout(slots, H, f32).total + 1024; }

// ------------------------------------------------------------ FP32 scan ----
// The FP32 operator: same prep with float32 outputs, then a float32 CUDA-core scan.
// One CTA per (head, sequence, 32 value columns); S [128 k][32 v] in shared memory.
constexpr int F32_THREADS = 256;
constexpr int F32_VB = 32;
constexpr int F32_SMEM = (C * K * 2 + C * C + K * C + F32_VB * C + K * F32_VB + C * F32_VB) * 4;

template <typename OutT>
__global__ void __launch_bounds__(F32_THREADS) gdn_scan_f32(Work ws, GdnTable tab, OutT* __restrict__ o, int H,
                                                            const float* __restrict__ s_in, long s_in_stride,
                                                            float* __restrict__ s_out) {
    extern __shared__ float fs[];
    float* w = fs;                  // [64][128]
    float* qd = w + C * K;          // [64][128]
    float* P = qd + C * K;          // [64][64]
    float* kdt = P + C * C;         // [128][64]
    float* ut = kdt + K * C;        // [32 v][64 t]
    float* S = ut + F32_VB * C;     // [128 k][32 v]
    float* vn = S + K * F32_VB;     // [64 t][32 v]
    const int h = blockIdx.x, seq = blockIdx.y, v0 = blockIdx.z * F32_VB;
    const int start = tab.seq.offset[seq];
    const int len = tab.seq.offset[seq + 1] - start;
    const int NC = (len + C - 1) / C;
    const long slot0 = (long)h * ws.slots + tab.chunk_base[seq];
    const int tid = threadIdx.x;
    for (int x = tid; x < K * F32_VB; x += F32_THREADS) {
        const int kk = x / F32_VB, vv = x % F32_VB;
        S[x] = s_in ? s_in[(long)seq * s_in_stride + ((size_t)h * K + kk) * V + v0 + vv] : 0.f;
    }
    const float* Wg = static_cast<const float*>(ws.w);
    const float* Qg = static_cast<const float*>(ws.qd);
    const float* Pg = static_cast<const float*>(ws.p);
    const float* Kg = static_cast<const float*>(ws.kdt);
    const float* Ug = static_cast<const float*>(ws.ut);
    for (int c = 0; c < NC; c++) {
        const long slot = slot0 + c;
        __syncthreads();
        for (int x = tid; x < C * K; x += F32_THREADS) {
            w[x] = Wg[slot * C * K + x];
            qd[x] = Qg[slot * C * K + x];
            kdt[x] = Kg[slot * K * C + x];
        }
        for (int x = tid; x < C * C; x += F32_THREADS) P[x] = Pg[slot * C * C + x];
        for (int x = tid; x < F32_VB * C; x += F32_THREADS) ut[x] = Ug[(slot * V + v0) * C + x];
        __syncthreads();
        // v_new[t][v] = u[t][v] - sum_k w[t][k] S[k][v]
        for (int x = tid; x < C * F32_VB; x += F32_THREADS) {
            const int t = x / F32_VB, vv = x % F32_VB;
            float acc = 0.f;
            for (int kk = 0; kk < K; kk++) acc = fmaf(w[t * K + kk], S[kk * F32_VB + vv], acc);
            vn[x] = ut[vv * C + t] - acc;
        }
        __syncthreads();
        // o[t][v] = sum_k qd[t][k] S[k][v] + sum_j P[t][j] v_new[j][v]
        const int rows = min(C, len - c * C);
        for (int x = tid; x < C * F32_VB; x += F32_THREADS) {
            const int t = x / F32_VB, vv = x % F32_VB;
            float a = 0.f, b = 0.f;
            for (int kk = 0; kk < K; kk++) a = fmaf(qd[t * K + kk], S[kk * F32_VB + vv], a);
            for (int j = 0; j <= t; j++) b = fmaf(P[t * C + j], vn[j * F32_VB + vv], b);
            if (t < rows) {
                const float val = a + b;
                OutT* dst = o + ((size_t)(start + c * C + t) * H + h) * V + v0 + vv;
                if constexpr (sizeof(OutT) == 4) *dst = val; else *dst = to_bf16(val);
            }
        }
        __syncthreads();
        // S = e^{last} S + kd^T v_new
        const float dec = ws.decay[slot];
        for (int x = tid; x < K * F32_VB; x += F32_THREADS) {
            const int kk = x / F32_VB, vv = x % F32_VB;
            float acc = 0.f;
            for (int t = 0; t < C; t++) acc = fmaf(kdt[kk * C + t], vn[t * F32_VB + vv], acc);
            S[x] = S[x] * dec + acc;
        }
    }
    __syncthreads();
    if (s_out)
        for (int x = tid; x < K * F32_VB; x += F32_THREADS) {
            const int kk = x / F32_VB, vv = x % F32_VB;
            s_out[(long)seq * H * K * V + ((size_t)h * K + kk) * V + v0 + vv] = S[x];
        }
}

int run_f32(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o, bool o_f32,
            void* workspace, size_t workspace_bytes, const SeqTable& seqs, int H, int HK, float scale,
            const void* s_in, long s_in_stride, void* s_out, cudaStream_t st) {
    if (!q || !k || !v || !g || !beta || !o || !workspace || H <= 0 || HK <= 0 || H % HK) return cudaErrorInvalidValue;
    GdnTable tab;
    make_gdn_table(tab, seqs);
    const long slots = tab.chunk_base[seqs.count];
    const Layout L(slots, H, true);
    if ((size_t)L.total > workspace_bytes) return cudaErrorInvalidValue;
    static const cudaError_t configured = [] {
        cudaError_t e = cudaFuncSetAttribute(gdn_prep<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_scan_f32<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, F32_SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_scan_f32<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, F32_SMEM);
        return e;
    }();
    if (configured != cudaSuccess) return configured;
    uint8_t* b = static_cast<uint8_t*>(workspace);
    Work ws{b + L.w, b + L.qd, b + L.p, b + L.kdt, b + L.ut, reinterpret_cast<float*>(b + L.decay), slots};
    gdn_prep<true><<<dim3(tab.max_chunks, H, seqs.count), PREP_THREADS, PREP_SMEM, st>>>(
        static_cast<const bf16*>(q), static_cast<const bf16*>(k), static_cast<const bf16*>(v), g,
        static_cast<const bf16*>(beta), ws, tab, H, HK, scale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const dim3 grid(H, seqs.count, V / F32_VB);
    if (o_f32)
        gdn_scan_f32<float><<<grid, F32_THREADS, F32_SMEM, st>>>(ws, tab, static_cast<float*>(o), H,
            static_cast<const float*>(s_in), s_in_stride, static_cast<float*>(s_out));
    else
        gdn_scan_f32<bf16><<<grid, F32_THREADS, F32_SMEM, st>>>(ws, tab, static_cast<bf16*>(o), H,
            static_cast<const float*>(s_in), s_in_stride, static_cast<float*>(s_out));
    return cudaGetLastError();
}

}  // namespace gdn
}  // namespace s1

using namespace s1;

namespace {

// Workspace pointers handed in by callers are 256-byte aligned (cudaMalloc); the
// TMA tiles want 1024: round up inside the caller's buffer.
void* align1k(void* p, size_t& bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uintptr_t r = (a + 1023) & ~(uintptr_t)1023;
    const size_t skip = r - a;
    bytes = bytes > skip ? bytes - skip : 0;
    return reinterpret_cast<void*>(r);
}

int single(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
           float* workspace, int T, int H, int HK, float scale, const void* s_in, void* s_out, void* stream) {
    if (T < 0 || HK <= 0 || H <= 0 || H % HK != 0) return cudaErrorInvalidValue;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (T == 0) {
        if (!s_out) return cudaSuccess;
        const size_t bytes = (size_t)H * 128 * 128 * sizeof(float);
        return s_in ? cudaMemcpyAsync(s_out, s_in, bytes, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(s_out, 0, bytes, st);
    }
    SeqTable tab;
    const size_t len = (size_t)T;
    make_table(tab, &len, 1);
    size_t bytes = gdn::workspace_bytes_for((T + 63) / 64, H, false);
    void* ws = align1k(workspace, bytes);
    return gdn::run(q, k, v, g, beta, o, ws, bytes, tab, H, HK, scale, s_in, 0, s_out, st);
}

}  // namespace

extern "C" {

size_t cs1_gdn_workspace_floats(int T, int H) {
    if (T <= 0 || H <= 0) return 0;
    return (gdn::workspace_bytes_for((T + 63) / 64, H, false) + 3) / 4;
}

int cs1_gdn_prefill(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                    float* workspace, int T, int H, int HK, float scale, void* stream) {
    return single(q, k, v, g, beta, o, workspace, T, H, HK, scale, nullptr, nullptr, stream);
}

int cs1_gdn_prefill_wide(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                         float* workspace, int T, int H, int HK, float scale, void* stream) {
    return single(q, k, v, g, beta, o, workspace, T, H, HK, scale, nullptr, nullptr, stream);
}

int cs1_gdn_prefill_x(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                      float* workspace, int T, int H, int HK, float scale, const void* s_in, void* s_out,
                      void* stream) {
    return single(q, k, v, g, beta, o, workspace, T, H, HK, scale, s_in, s_out, stream);
}

size_t cs1_gdn_batch_workspace_floats(int tokens, int H, int count) {
    if (tokens <= 0 || H <= 0 || count <= 0 || count > MAX_SEQS || tokens > INT_MAX - count * 64) return 0;
    const long slots = (tokens + 63) / 64 + count;
    return (gdn::workspace_bytes_for(slots, H, false) + 3) / 4;
}

int cs1_gdn_prefill_batch_x(const void* q, const void* k, const void* v, const float* g, const void* beta,
                            void* o, float* workspace, size_t workspace_bytes, const size_t* lengths,
                            size_t count, int H, int HK, float scale, const void* state_in, int state_stride,
                            void* state_out, void* stream) {
    SeqTable tab;
    if (!make_table(tab, lengths, count) || (state_stride != 0 && state_stride != 1)) return cudaErrorInvalidValue;
    size_t bytes = workspace_bytes;
    void* ws = align1k(workspace, bytes);
    const long stride = state_stride ? (long)H * 128 * 128 : 0;
    return gdn::run(q, k, v, g, beta, o, ws, bytes, tab, H, HK, scale, state_in, stride, state_out,
                    static_cast<cudaStream_t>(stream));
}

int cs1_gdn_prefill_batch_xn(const void* q, const void* k, const void* v, const float* g, const void* beta,
                             const float* rnorm_q, const float* rnorm_k, void* o, const size_t* lengths, size_t count,
                             int H, int HK, float scale, const void* state_in, int state_stride, void* state_out,
                             void* stream) {
    SeqTable tab;
    if (!rnorm_q || !rnorm_k || !make_table(tab, lengths, count) || (state_stride != 0 && state_stride != 1))
        return cudaErrorInvalidValue;
    const long stride = state_stride ? (long)H * 128 * 128 : 0;
    return gdn::run_fused(q, k, v, g, beta, o, tab, H, HK, scale, state_in, stride, state_out,
                          static_cast<cudaStream_t>(stream), nullptr, 0, rnorm_q, rnorm_k);
}

int cs1_gdn_prefill_dyn(const void* q, const void* k, const void* v, const float* g, const void* beta,
                        const float* rnorm_q, const float* rnorm_k, void* o, int cap_rows, int cap_seqs, int H, int HK,
                        float scale, const void* state_in, int state_stride, void* state_out, const void* desc,
                        void* stream) {
    if (!desc || cap_rows <= 0 || (state_stride != 0 && state_stride != 1)) return cudaErrorInvalidValue;
    SeqTable cap;  // tensor-map extents only
    memset(&cap, 0, sizeof(cap));
    cap.count = 1;
    cap.offset[1] = cap_rows;
    const long stride = state_stride ? (long)H * 128 * 128 : 0;
    return gdn::run_fused(q, k, v, g, beta, o, cap, H, HK, scale, state_in, stride, state_out,
                          static_cast<cudaStream_t>(stream), static_cast<const DevBatch*>(desc), cap_seqs, rnorm_q,
                          rnorm_k);
}

int cs1_gdn_prefill_batch_shared(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                 void* o, float* workspace, size_t workspace_bytes, const size_t* lengths,
                                 size_t count, int H, int HK, float scale, const void* state, void* stream) {
    return cs1_gdn_prefill_batch_x(q, k, v, g, beta, o, workspace, workspace_bytes, lengths, count, H, HK, scale,
                                   state, 0, nullptr, stream);
}

int cs1_gdn_prefill_batch(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
                          float* workspace, size_t workspace_bytes, const size_t* lengths, size_t count, int H,
                          int HK, float scale, void* stream) {
    return cs1_gdn_prefill_batch_x(q, k, v, g, beta, o, workspace, workspace_bytes, lengths, count, H, HK, scale,
                                   nullptr, 0, nullptr, stream);
}

// ---- FP32 operator (ops.h:116-121): float32 normalised q/k, recurrent state and
// intermediates; bfloat16 output. The context records the device it was made on. ----
struct Fp32Context {
    int device;
    size_t bytes;
};

void* cs1_gdn_fp32_create(size_t workspace_bytes) {
    auto* c = new (std::nothrow) Fp32Context;
    if (!c) return nullptr;
    c->bytes = workspace_bytes;
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    return c;
}

void cs1_gdn_fp32_destroy(void* context) { delete static_cast<Fp32Context*>(context); }

size_t cs1_gdn_fp32_workspace_floats(int T, int H) {
    if (T <= 0 || T > 65536 || H <= 0 || H > 256) return 0;
    return (gdn::workspace_bytes_for((T + 63) / 64, H, true) + 3) / 4;
}

static int fp32_call(void* context, const void* q, const void* k, const void* v, const float* g, const void* beta,
                     void* o, bool o_f32, float* workspace, int T, int H, int HK, float scale, const float* s_in,
                     float* s_out, void* stream) {
    if (!context || !workspace || !q || !k || !v || !g || !beta || !o || !cs1_gdn_fp32_workspace_floats(T, H) ||
        HK <= 0 || H % HK != 0 || !(scale > 0.f) || !(scale < INFINITY))
        return cudaErrorInvalidValue;
    SeqTable tab;
    const size_t len = (size_t)T;
    make_table(tab, &len, 1);
    size_t bytes = gdn::workspace_bytes_for((T + 63) / 64, H, true);
    void* ws = align1k(workspace, bytes);
    return gdn::run_f32(q, k, v, g, beta, o, o_f32, ws, bytes, tab, H, HK, scale, s_in, 0, s_out,
                        static_cast<cudaStream_t>(stream));
}

int cs1_gdn_prefill_fp32(void* context, const void* q, const void* k, const void* v, const float* g,
                         const void* beta, void* o, float* workspace, int T, int H, int HK, float scale,
                         void* stream) {
    return fp32_call(context, q, k, v, g, beta, o, false, workspace, T, H, HK, scale, nullptr, nullptr, stream);
}

int cs1_gdn_prefill_fp32_x(void* context, const void* q, const void* k, const void* v, const float* g,
                           const void* beta, float* o, float* workspace, int T, int H, int HK, float scale,
                           const float* s_in, float* s_out, void* stream) {
    return fp32_call(context, q, k, v, g, beta, o, true, workspace, T, H, HK, scale, s_in, s_out, stream);
}

}  // extern "C"
