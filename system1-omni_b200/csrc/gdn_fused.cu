// Chunked Gated DeltaNet prefill in one kernel: the per-chunk preparation and the state
// scan of a (value head, sequence) run in the same CTA, warp-specialised, so nothing of a
// chunk goes through global memory between them.
//
// Recurrence and chunk form as in gdn.cu (Transformers' torch_chunk_gated_delta_rule,
// chunks of 64): per chunk, with cum = cumsum(g), k^ = k / |k|, q^ = q / |q| * scale,
//   A_ij = beta_i k^_i.k^_j e^{cum_i - cum_j} (j < i),  T = (I + A)^-1,
//   tb = bf16(T diag(beta)),  u = bf16(tb v),  w = bf16(tb bf16(k^ e^cum)),
//   qd = bf16(q^ e^cum),  kd = bf16(k^ e^{last - cum}),  P_tj = bf16(q^_t.k^_j e^{cum_t - cum_j}),
//   v_new = bf16(u - w S),  o = qd S + P v_new,  S = e^{last} S + kd^T v_new.
// The bf16 rounding points are those of the reference kernel (gdn_prefill.cu:1-15 of the
// reference). The pair products k.k and q.k are taken on the raw bf16 rows (exact
// products, fp32 sums) and scaled by the inverse norms afterwards, instead of on
// TF32-rounded normalised rows: the same quantities, with fewer rounding steps.
//
// One CTA (512 threads, one per SM: ~205 KB of shared memory, all 512 TMEM columns) per
// (value head, sequence), longest sequences first, walking the chunks in order:
//   warp 0       TMA producer: q and k rows of the key head (double-buffered), v rows of
//                the value head (single buffer, refilled as soon as its MMA has read it, on
//                its own barrier so that the next q and k do not wait for it)
//   warp 1       scan MMA issuer:  (wS)^T, (qd S)^T = S^T [w^T | qd^T]   (A = S^T in TMEM)
//                                  o^T += v_new^T P^T,  S^T += v_new^T kd  (A = v_new^T in TMEM)
//   warp 2       prep MMA issuer:  D1 = [k; q] k^T                         (raw bf16, K = 128)
//                                  u^T = v^T tb^T,  w^T = kw^T tb^T        (K = 64)
//   warp 3       vector warp, ahead of the preparation: g and beta of the chunk, the
//                sequential cumsum of g, e^cum, e^{last - cum} and the decay e^{last}
//   warps 4-7    scan epilogue, thread = value column v = TMEM lane: per chunk the bf16
//                copy of S^T (the next MMA's A operand, written to TMEM) and e^{last} S^T,
//                v_new^T = bf16(bf16(u) - wS) (TMEM), the next chunk's qd and kd operand
//                tiles, o rows straight to global memory
//   warps 8-15   preparation of the next chunk while the scan runs: norms, kw, A and P from
//                D1, the 64 x 64 inverse by block doubling (8 x 8 diagonal blocks by
//                substitution, then the blocks below the diagonal at 16, 32 and 64) written
//                out as tb, then w (from TMEM)
// TMEM columns: [0,128) S^T fp32 | [128,192) S^T bf16 pairs | [192,256) wS fp32, then
// v_new^T bf16 pairs | [256,320) o^T fp32 | [320,384) D1 fp32, then w^T fp32 |
// [384,512) u^T fp32, two chunk buffers.
// Every wait is bounded (tc.cuh); a wait that gives up records a fault bit and sets an
// abort flag that stops every role at its next chunk, after which the CTA drains its
// copies and MMAs and frees its tensor memory. Each mbarrier has one producing role whose
// arrivals are ordered behind the waits of its consumers, so no waiter can fall two phases
// behind (which a parity wait would misread); the one hand-off without that order, the
// norms of the next chunk read by the scan warps, is a monotonic counter.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "gdn.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(gdn_fused)

namespace s1 {
namespace gdnf {

using namespace s1::tc;
using gdn::C;
using gdn::K;
using gdn::V;

constexpr int THREADS = 512;
constexpr int PREP0 = 8;        // first preparation warp
constexpr int NPREP = 256;      // preparation threads (warps 8-15)
constexpr int BAR_SCAN = 1, BAR_PREP = 2;  // named barriers (0 is __syncthreads)
constexpr int LDT = C + 4;      // fp32 row stride of A and T

// shared memory (offsets from a 1024-byte aligned base)
constexpr int BOX = 64 * 128;                 // one [64 rows][64 bf16] swizzled box, 8 KB
constexpr int KQ_TILE = 4 * BOX;              // [k box0 | q box0 | k box1 | q box1]: two [128][64] A tiles
constexpr int OFF_KQ = 0;                     // two slots
constexpr int OFF_V = OFF_KQ + 2 * KQ_TILE;   // v [64 j][128 v] as two MN blocks
constexpr int OFF_KW = OFF_V + 2 * BOX;       // k^ e^cum [64 j][128 k] as two MN blocks
constexpr int OFF_TB = OFF_KW + 2 * BOX;      // tb [64 t][64 j] K-major
constexpr int OFF_W = OFF_TB + BOX;           // w^T [128 k][64 t]: the MN-major B operand of (wS)^T, two chunk buffers
constexpr int OFF_QD = OFF_W + 4 * BOX;       // qd [64 t][128 k] K-major (two sub-tiles)
constexpr int OFF_KD = OFF_QD + 2 * BOX;      // kd [64 t][128 k] MN-major (two blocks)
constexpr int OFF_P = OFF_KD + 2 * BOX;       // P [64 t][64 j] K-major, two chunk buffers
constexpr int OFF_A = OFF_P + 2 * BOX;        // A fp32 [64][LDT]
constexpr int LDD = 36;                       // fp32 row stride of the diagonal blocks of T
constexpr int OFF_T = OFF_A + C * LDT * 4;    // T's two diagonal 32 x 32 blocks, fp32 [2][32][LDD]
constexpr int OFF_X = OFF_T + 2 * 32 * LDD * 4;  // inverse scratch [32][32] fp32
constexpr int OFF_VEC = OFF_X + 32 * 32 * 4;  // per-chunk vectors (floats)
// two chunk slots of VEC_SLOT floats: cum * log2(e), beta, e^cum, e^{last - cum}, g
// (scratch), written by the vector warp, and the inverse norms of k and q (q's times the
// scale), written by the preparation; the decay e^{last} in a ring of four chunks
constexpr int VEC_CUM2 = 0, VEC_BET = 64, VEC_ECUM = 128, VEC_EREM = 192, VEC_G = 256, VEC_KINV = 320,
              VEC_QINV = 384, VEC_SLOT = 448;
constexpr int VEC_DECAY = 2 * VEC_SLOT;
constexpr int OFF_BAR = OFF_VEC + (VEC_DECAY + 8) * 4;
constexpr int NBAR = 40;
constexpr int SMEM = OFF_BAR + NBAR * 8 + 64 + 1024;

// TMEM columns
constexpr uint32_t TM_S = 0, TM_ST = 128, TM_WS = 192, TM_O = 256, TM_D1 = 320, TM_U = 384;

// barrier indices (8 bytes each)
enum Bar : int {
    B_IN_FULL = 0,      // [2] q, k (slot) landed
    B_IN_KQ_FREE = 2,   // [2] preparation and scan warps done with the q, k slot (count 12)
    B_IN_V_FREE = 4,    // MMA2 read v
    B_D1_FULL = 5,      // MMA1 done
    B_D1W_FREE = 6,     // prep read w^T out of the D1 columns (count 8)
    B_TB_READY = 7,     // tb and kw tiles written (count 8)
    B_MMA2_DONE = 8,    // u^T and w^T in TMEM
    B_U_FREE = 9,       // [2] scan read u^T of the slot (count 4)
    B_OPS_READY = 11,   // [2] w of the chunk written into the slot by the preparation (count 8)
    B_S_READY = 14,     // S^T bf16 copy and e^{last} S^T written (count 4)
    B_WS_DONE = 15,     // (wS)^T and (qd S)^T in TMEM
    B_VN_READY = 16,    // v_new^T written (count 4)
    B_UPD_DONE = 17,    // o^T and S^T updated
    B_DRAIN_SCAN = 18,
    B_DRAIN_PREP = 19,
    B_VEC_READY = 20,   // [2] the vector warp wrote the slot's vectors (count 1)
    B_VEC_FREE = 22,    // [2] preparation and scan warps are done with the slot (count 12)
    B_DEC_READY = 24,   // [4] the chunk's decay is in the ring (count 1)
    B_QD_READY = 29,    // qd of the chunk written by the scan warps (count 4)
    B_KD_READY = 30,    // kd of the chunk written by the scan warps (count 4)
    B_W_FREE = 32,      // [2] the first scan MMAs read the slot's w
    B_P_FREE = 34,      // [2] the second scan MMAs read the slot's P
    B_OPS2_READY = 36,  // [2] P of the chunk written into the slot by the preparation (count 8)
    B_V_FULL = 38,      // v landed (its own barrier: q and k need not wait for v's buffer)
};

struct Maps {
    CUtensorMap q, k, v;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fail(uint32_t bit, volatile int* abort_flag) {
    atomicOr(&g_fault_word, bit);
    *abort_flag = 1;
}

template <bool Dyn>
__global__ void __launch_bounds__(THREADS, 1)
    gdn_fused(const __grid_constant__ Maps maps, const float* __restrict__ g, const bf16* __restrict__ beta,
              const __grid_constant__ SeqTable tab, bf16* __restrict__ o, int H, int HK, float scale,
              const float* __restrict__ s_in, long s_in_stride, float* __restrict__ s_out, const DevBatch* dyn,
              const float* __restrict__ rnq, const float* __restrict__ rnk) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* sm = smem_raw + (base - raw);
    float* vec = reinterpret_cast<float*>(sm + OFF_VEC);
    const uint32_t bars = base + OFF_BAR;
    auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + NBAR * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + OFF_BAR + NBAR * 8 + 16);
    // chunks whose norms are in (monotonic; the scan warps read them to form qd and kd)
    volatile int* norms_done = reinterpret_cast<volatile int*>(sm + OFF_BAR + NBAR * 8 + 20);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // the capacity path (dyn): the table is the descriptor's, the grid covers the capacity
    int seq, start, len;
    if constexpr (Dyn) {
        if ((int)blockIdx.y >= dyn->tab.count) return;  // past the batch: nothing allocated or armed
        seq = dyn->tab.order[blockIdx.y];
        start = dyn->tab.offset[seq];
        len = dyn->tab.offset[seq + 1] - start;
    } else {
        seq = tab.order[blockIdx.y];
        start = tab.offset[seq];
        len = tab.offset[seq + 1] - start;
    }
    const int h = blockIdx.x;
    const int hk = h / (H / HK);
    const int NC = (len + C - 1) / C;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(B_IN_FULL + i), 1);
            mbar_init(bar(B_IN_KQ_FREE + i), 12);
            mbar_init(bar(B_U_FREE + i), 4);
            mbar_init(bar(B_VEC_READY + i), 1);
            mbar_init(bar(B_VEC_FREE + i), 12);
            mbar_init(bar(B_OPS_READY + i), 8);
            mbar_init(bar(B_W_FREE + i), 1);
            mbar_init(bar(B_P_FREE + i), 1);
            mbar_init(bar(B_OPS2_READY + i), 8);
        }
        for (int i = 0; i < 4; i++) mbar_init(bar(B_DEC_READY + i), 1);
        mbar_init(bar(B_IN_V_FREE), 1);
        mbar_init(bar(B_V_FULL), 1);
        mbar_init(bar(B_D1_FULL), 1);
        mbar_init(bar(B_D1W_FREE), 8);
        mbar_init(bar(B_TB_READY), 8);
        mbar_init(bar(B_MMA2_DONE), 1);
        mbar_init(bar(B_S_READY), 4);
        mbar_init(bar(B_WS_DONE), 1);
        mbar_init(bar(B_VN_READY), 4);
        mbar_init(bar(B_UPD_DONE), 1);
        mbar_init(bar(B_DRAIN_SCAN), 1);
        mbar_init(bar(B_DRAIN_PREP), 1);
        mbar_init(bar(B_QD_READY), 4);
        mbar_init(bar(B_KD_READY), 4);
        *abort_flag = 0;
        *norms_done = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&maps.q);
            tma_prefetch_desc(&maps.k);
            tma_prefetch_desc(&maps.v);
            int issued = 0, issued_v = 0;
            for (int c = 0; c < NC; c++) {
                if (*abort_flag) break;
                const int slot = c & 1;
                const int t0 = start + c * C;
                // q and k into their slot as soon as it is free; v (one buffer) once the
                // previous chunk's MMA2 has read it, on its own barrier
                if (!mbar_wait(bar(B_IN_KQ_FREE + slot), (uint32_t)((c >> 1) + 1) & 1u)) {
                    fail(FAULT_WAIT_PRODUCER, abort_flag);
                    break;
                }
                const uint32_t kq = base + OFF_KQ + slot * KQ_TILE, full = bar(B_IN_FULL + slot);
                mbar_expect_tx(full, 4 * BOX);
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    tma_load_3d(kq + b * 2 * BOX, &maps.k, full, 64 * b, hk, t0);
                    tma_load_3d(kq + b * 2 * BOX + BOX, &maps.q, full, 64 * b, hk, t0);
                }
                issued++;
                if (!mbar_wait(bar(B_IN_V_FREE), (uint32_t)(c + 1) & 1u)) {
                    fail(FAULT_WAIT_PRODUCER, abort_flag);
                    break;
                }
                mbar_expect_tx(bar(B_V_FULL), 2 * BOX);
#pragma unroll
                for (int b = 0; b < 2; b++) tma_load_3d(base + OFF_V + b * BOX, &maps.v, bar(B_V_FULL), 64 * b, h, t0);
                issued_v++;
            }
            // the copies in flight land before the CTA can leave
            for (int c = issued > 2 ? issued - 2 : 0; c < issued; c++)
                (void)mbar_wait(bar(B_IN_FULL + (c & 1)), (uint32_t)(c >> 1) & 1u);
            if (issued_v > 0) (void)mbar_wait(bar(B_V_FULL), (uint32_t)(issued_v - 1) & 1u);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- scan MMAs
        if (lane == 0) {
            constexpr uint32_t ID_W = idesc_major(128, 64, AB_BF16, 0, 1);    // B = w^T, MN-major
            constexpr uint32_t ID_K64 = idesc(128, 64, AB_BF16);              // B = qd or P, K-major
            constexpr uint32_t ID_KD = idesc_major(128, 128, AB_BF16, 0, 1);  // B = kd, MN-major, N = 128
            bool ok = true;
            for (int c = 0; c < NC; c++) {
                if (*abort_flag) break;
                const uint32_t par = (uint32_t)c & 1u, spar = (uint32_t)(c >> 1) & 1u;
                const int slot = c & 1;
                if (!mbar_wait(bar(B_OPS_READY + slot), spar) || !mbar_wait(bar(B_QD_READY), par) ||
                    !mbar_wait(bar(B_S_READY), par)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t a = tmem + TM_ST + (uint32_t)kk * 8;
                    mma_bf16_ts(tmem + TM_WS, a, desc_sw128_mn(base + OFF_W + slot * 2 * BOX + kk * 2048, BOX, 1024),
                                ID_W, kk > 0);
                    mma_bf16_ts(tmem + TM_O, a, desc_sw128(base + OFF_QD + (kk >> 2) * BOX + (kk & 3) * 32), ID_K64,
                                kk > 0);
                }
                mma_commit(bar(B_WS_DONE));
                mma_commit(bar(B_W_FREE + slot));
                if (!mbar_wait(bar(B_VN_READY), par) || !mbar_wait(bar(B_OPS2_READY + slot), spar) ||
                    !mbar_wait(bar(B_KD_READY), par)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t pt = base + OFF_P + (uint32_t)(c & 1) * BOX;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint32_t a = tmem + TM_WS + (uint32_t)kk * 8;
                    mma_bf16_ts(tmem + TM_O, a, desc_sw128(pt + kk * 32), ID_K64, 1);
                    mma_bf16_ts(tmem + TM_S, a, desc_sw128_mn(base + OFF_KD + kk * 2048, BOX, 1024), ID_KD, 1);
                }
                mma_commit(bar(B_UPD_DONE));
                mma_commit(bar(B_P_FREE + slot));
            }
            if (!ok) fail(FAULT_WAIT_MMA, abort_flag);
            mma_commit(bar(B_DRAIN_SCAN));
            (void)mbar_wait(bar(B_DRAIN_SCAN), 0);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- preparation MMAs
        if (lane == 0) {
            constexpr uint32_t ID_D1 = idesc(128, 64, AB_BF16);
            constexpr uint32_t ID_2 = idesc_major(128, 64, AB_BF16, 1, 0);  // A MN-major (v, kw), B = tb K-major
            bool ok = true;
            for (int c = 0; c < NC; c++) {
                if (*abort_flag) break;
                const int slot = c & 1;
                const uint32_t kq = base + OFF_KQ + slot * KQ_TILE;
                if (!mbar_wait(bar(B_IN_FULL + slot), (uint32_t)(c >> 1) & 1u) ||
                    !mbar_wait(bar(B_D1W_FREE), (uint32_t)(c + 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // D1 = [k; q] k^T on the raw rows: A = [k box | q box] (128 rows), B = its k box
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t t = kq + (kk >> 2) * 2 * BOX + (kk & 3) * 32;
                    mma_bf16(tmem + TM_D1, desc_sw128(t), desc_sw128(t), ID_D1, kk > 0);
                }
                mma_commit(bar(B_D1_FULL));
                if (!mbar_wait(bar(B_TB_READY), (uint32_t)c & 1u) ||
                    !mbar_wait(bar(B_U_FREE + slot), (uint32_t)((c >> 1) + 1) & 1u) ||
                    !mbar_wait(bar(B_V_FULL), (uint32_t)c & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // u^T = v^T tb^T into this chunk's u buffer; w^T = kw^T tb^T over the D1 columns
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const uint64_t b = desc_sw128(base + OFF_TB + kk * 32);
                    mma_bf16(tmem + TM_U + (uint32_t)slot * 64, desc_sw128_mn(base + OFF_V + kk * 2048, BOX, 1024), b,
                             ID_2, kk > 0);
                    mma_bf16(tmem + TM_D1, desc_sw128_mn(base + OFF_KW + kk * 2048, BOX, 1024), b, ID_2, kk > 0);
                }
                mma_commit(bar(B_MMA2_DONE));
                mma_commit(bar(B_IN_V_FREE));
            }
            if (!ok) fail(FAULT_WAIT_MMA, abort_flag);
            mma_commit(bar(B_DRAIN_PREP));
            (void)mbar_wait(bar(B_DRAIN_PREP), 0);
        }
    } else if (warp == 3) {
        // ---------------------------------------------------------------- vector warp
        // Per chunk, ahead of the preparation: g and beta of the chunk (rows past the
        // sequence's end: 0), the sequential fp32 cumsum of g (the reference's order),
        // cum * log2(e), e^cum, e^{last - cum} and the decay e^{last}.
        // With the front end's inverse norms (rnk, rnq: [T, HK]) it also fills the chunk's
        // norm vectors (q's times the scale); rows past the sequence get 0.
        float gn[2] = {0.f, 0.f}, bn[2] = {0.f, 0.f};  // this lane's rows lane, lane + 32 of the next chunk
        float kn[2] = {0.f, 0.f}, qn[2] = {0.f, 0.f};
        auto fetch = [&](int c) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int row = c * C + lane + 32 * i;
                gn[i] = row < len ? g[(size_t)(start + row) * H + h] : 0.f;
                bn[i] = row < len ? f32(beta[(size_t)(start + row) * H + h]) : 0.f;
                if (rnk) {
                    kn[i] = row < len ? rnk[(size_t)(start + row) * HK + hk] : 0.f;
                    qn[i] = row < len ? rnq[(size_t)(start + row) * HK + hk] * scale : 0.f;
                }
            }
        };
        fetch(0);
        for (int c = 0; c < NC; c++) {
            if (*abort_flag) break;
            const int slot = c & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_VEC_FREE + slot), (uint32_t)((c >> 1) + 1) & 1u))) {
                if (lane == 0) fail(FAULT_WAIT_OTHER, abort_flag);
                break;
            }
            float* vs = vec + slot * VEC_SLOT;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                vs[VEC_G + lane + 32 * i] = gn[i];
                vs[VEC_BET + lane + 32 * i] = bn[i];
                if (rnk) {
                    vs[VEC_KINV + lane + 32 * i] = kn[i];
                    vs[VEC_QINV + lane + 32 * i] = qn[i];
                }
            }
            if (c + 1 < NC) fetch(c + 1);  // in flight behind this chunk's arithmetic
            __syncwarp();
            if (lane == 0) {
                float gv[C];
#pragma unroll
                for (int i = 0; i < C; i++) gv[i] = vs[VEC_G + i];
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < C; i++) {
                    acc += gv[i];
                    gv[i] = acc;
                }
#pragma unroll
                for (int i = 0; i < C; i++) vs[VEC_G + i] = gv[i];  // cum
                vec[VEC_DECAY + (c & 3)] = expf(acc);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int t = lane + 32 * i;
                const float ct = vs[VEC_G + t];
                vs[VEC_CUM2 + t] = ct * 1.4426950408889634f;
                vs[VEC_ECUM + t] = expf(ct);
                vs[VEC_EREM + t] = expf(vs[VEC_G + C - 1] - ct);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(B_VEC_READY + slot));
                mbar_arrive(bar(B_DEC_READY + (c & 3)));
            }
        }
    } else if (warp >= 4 && warp < PREP0) {
        // ---------------------------------------------------------------- scan epilogue
        const int v = threadIdx.x - 128;
        const uint32_t lrow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        {
            const float* si = s_in ? s_in + (long)seq * s_in_stride + (size_t)h * K * V : nullptr;
#pragma unroll 1
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = si ? si[(size_t)(q4 * 32 + i) * V + v] : 0.f;
                tmem_st32(lrow + TM_S + q4 * 32, x);
            }
            tmem_st_wait();
        }
        // Chunk c's pass over the state row: its bf16 copy (the first MMAs' A operand) and
        // e^{last} S written back for the update MMA to accumulate onto.
        auto state_pass = [&](int c) -> bool {
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_DEC_READY + (c & 3)), (uint32_t)(c >> 2) & 1u))) return false;
            const float dec = vec[VEC_DECAY + (c & 3)];
#pragma unroll 1
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
                uint32_t pk[16];
                tmem_ld32(lrow + TM_S + q4 * 32, x);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; i++) pk[i] = pack_bf16x2(x[2 * i], x[2 * i + 1]);
                tmem_st16(lrow + TM_ST + q4 * 16, pk);
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] *= dec;
                tmem_st32(lrow + TM_S + q4 * 32, x);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_S_READY));
            return true;
        };
        // The o rows of chunk c from this thread's column v of each row. Adjacent lanes swap
        // halves so that each stores two adjacent columns of one row: the even lane rows 2i,
        // the odd lane rows 2i + 1 (a warp writes 64 contiguous bytes of each of two rows per
        // store).
        auto write_o = [&](int c, const uint32_t (&opk)[32]) {
            const int rows = min(C, len - c * C);
            const bool odd = lane & 1;
            uint32_t* dst = reinterpret_cast<uint32_t*>(o + ((size_t)(start + c * C) * H + h) * V + (v & ~1)) +
                            (odd ? (size_t)H * V / 2 : 0);
            const size_t pitch2 = (size_t)H * V;  // two rows, in 32-bit words
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const uint32_t mine = opk[i];  // (row 2i, row 2i + 1) of column v
                const uint32_t other = __shfl_xor_sync(0xffffffffu, odd ? (mine & 0xFFFFu) : (mine >> 16), 1);
                const uint32_t pair = odd ? (other | (mine & 0xFFFF0000u)) : ((mine & 0xFFFFu) | (other << 16));
                if (2 * i + (odd ? 1 : 0) < rows) dst[(size_t)i * pitch2] = pair;
            }
        };
        // qd = bf16(q^ e^cum) and kd = bf16(k^ e^{last - cum}) of chunk c from its q, k rows, once
        // the preparation has their norms (a monotonic count, so no barrier phase can alias)
        auto norms_in = [&](int c) -> bool {
            if (*norms_done <= c) {
                const long long t0 = clock64();
                while (*norms_done <= c)
                    if (clock64() - t0 > S1_WAIT_CYCLES) return false;
            }
            __threadfence_block();
            return true;
        };
        auto form_qd = [&](int c) {
            const int slot = c & 1;
            const uint8_t* kqp = sm + OFF_KQ + slot * KQ_TILE;
            const float* vs = vec + slot * VEC_SLOT;
#pragma unroll 2
            for (int u = v; u < C * 16; u += 128) {
                const int t = u >> 4, b = (u >> 3) & 1, ch = u & 7;
                float qx[8];
                unpack8(*reinterpret_cast<const Pack8*>(kqp + b * 2 * BOX + BOX + sw128_offset(t, ch)), qx);
                const float sc = vs[VEC_QINV + t], ec = vs[VEC_ECUM + t];
#pragma unroll
                for (int e = 0; e < 8; e++) qx[e] = (qx[e] * sc) * ec;
                *reinterpret_cast<Pack8*>(sm + OFF_QD + b * BOX + sw128_offset(t, ch)) = pack8(qx);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_QD_READY));
        };
        auto form_kd = [&](int c) {
            const int slot = c & 1;
            const uint8_t* kqp = sm + OFF_KQ + slot * KQ_TILE;
            const float* vs = vec + slot * VEC_SLOT;
#pragma unroll 2
            for (int u = v; u < C * 16; u += 128) {
                const int t = u >> 4, b = (u >> 3) & 1, ch = u & 7;
                float kx[8];
                unpack8(*reinterpret_cast<const Pack8*>(kqp + b * 2 * BOX + sw128_offset(t, ch)), kx);
                const float sc = vs[VEC_KINV + t], er = vs[VEC_EREM + t];
#pragma unroll
                for (int e = 0; e < 8; e++) kx[e] = (kx[e] * sc) * er;
                *reinterpret_cast<Pack8*>(sm + OFF_KD + b * BOX + sw128_offset(t, ch)) = pack8(kx);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(bar(B_KD_READY));
                mbar_arrive(bar(B_IN_KQ_FREE + slot));
                mbar_arrive(bar(B_VEC_FREE + slot));
            }
        };
        uint32_t opk[32];  // o^T row of the previous chunk, written out behind this chunk's update MMAs
        bool ok = __all_sync(0xffffffffu, norms_in(0));
        if (ok) {
            form_qd(0);
            form_kd(0);
            ok = state_pass(0);
        }
        for (int c = 0; c < NC; c++) {
            if (bar_any(BAR_SCAN, 128, !ok || *abort_flag != 0)) {
                if (!ok && v == 0) fail(FAULT_WAIT_EPILOGUE, abort_flag);
                ok = false;
                break;
            }
            const uint32_t par = (uint32_t)c & 1u;
            // v_new^T = bf16(bf16(u) - (wS)^T), written as bf16 pairs over the (wS)^T columns
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_WS_DONE), par));
            if (ok) {
                tc_fence_after();
                uint32_t pk[32];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    float w16[16], u16[16];
                    tmem_ld16(lrow + TM_WS + q * 16, w16);
                    tmem_ld16(lrow + TM_U + (uint32_t)(c & 1) * 64 + q * 16, u16);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        pk[q * 8 + i] = pack_bf16x2(rbf(u16[2 * i]) - w16[2 * i], rbf(u16[2 * i + 1]) - w16[2 * i + 1]);
                }
                tmem_st32(lrow + TM_WS, *reinterpret_cast<const float(*)[32]>(pk));
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(bar(B_VN_READY));
                    mbar_arrive(bar(B_U_FREE + (c & 1)));
                }
            }
            // the next chunk's qd (the first scan MMAs of this chunk have read the tile), then
            // the previous chunk's o rows, both behind this chunk's update MMAs
            if (ok && c + 1 < NC) {
                ok = __all_sync(0xffffffffu, norms_in(c + 1));
                if (ok) form_qd(c + 1);
            }
            if (c > 0) write_o(c - 1, opk);
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_UPD_DONE), par));
            // o^T of this chunk out of TMEM before the next chunk's first MMAs rewrite it, then
            // the next chunk's state pass (it gates those MMAs) and its kd
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    float ov[32];
                    tmem_ld32(lrow + TM_O + half * 32, ov);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; i++) opk[half * 16 + i] = pack_bf16x2(ov[2 * i], ov[2 * i + 1]);
                }
                if (c + 1 < NC) {
                    ok = state_pass(c + 1);
                    if (ok) form_kd(c + 1);
                }
            }
        }
        if (bar_any(BAR_SCAN, 128, !ok)) {
            if (v == 0 && !*abort_flag) fail(FAULT_WAIT_EPILOGUE, abort_flag);
            ok = false;
        } else {
            write_o(NC - 1, opk);
        }
        if (s_out && ok && !*abort_flag) {
            float* so = s_out + (long)seq * (long)H * K * V + (size_t)h * K * V;
#pragma unroll 1
            for (int q4 = 0; q4 < 4; q4++) {
                float x[32];
                tmem_ld32(lrow + TM_S + q4 * 32, x);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) so[(size_t)(q4 * 32 + i) * V + v] = x[i];
            }
        }
        tc_fence_before();
    } else if (warp >= PREP0) {
        // ---------------------------------------------------------------- preparation
        const int pt = threadIdx.x - PREP0 * 32, pw = warp - PREP0, wq = warp & 3;
        const uint32_t lrow = tmem + ((uint32_t)(wq * 32) << 16);
        float* A = reinterpret_cast<float*>(sm + OFF_A);
        float* Tm = reinterpret_cast<float*>(sm + OFF_T);
        float* X = reinterpret_cast<float*>(sm + OFF_X);
        bool ok = true;
        for (int c = 0; c < NC; c++) {
            if (bar_any(BAR_PREP, NPREP, !ok || *abort_flag != 0)) {
                if (!ok && pt == 0) fail(FAULT_WAIT_OTHER, abort_flag);
                break;
            }
            const int slot = c & 1;
            const uint8_t* kqp = sm + OFF_KQ + slot * KQ_TILE;
            float* vs = vec + slot * VEC_SLOT;
            const float* cum2 = vs + VEC_CUM2;
            const float* bet = vs + VEC_BET;
            const float* ecum = vs + VEC_ECUM;
            float* kinv = vs + VEC_KINV;
            float* qinv = vs + VEC_QINV;
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_IN_FULL + slot), (uint32_t)(c >> 1) & 1u) &&
                                             mbar_wait(bar(B_VEC_READY + slot), (uint32_t)(c >> 1) & 1u));
            // norms: four threads per row (32 dims each: two 16-byte chunks of each box half),
            // rows pt / 4 of k and of q; the same threads then form their part of
            // kw = bf16(k^ e^cum), the MN-major A operand of w^T = kw^T tb^T, while MMA1 runs
            if (ok) {
                const int r = pt >> 2, qq = pt & 3, b = qq >> 1, ch0 = (qq & 1) * 4;
                Pack8 kr[4];
                float kv;
                if (rnk) {  // the front end's norms, already in the slot
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        kr[i] = *reinterpret_cast<const Pack8*>(kqp + b * 2 * BOX + sw128_offset(r, ch0 + i));
                    kv = kinv[r];
                } else {
                    float ks = 0.f, qs = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        float kx[8], qx[8];
                        kr[i] = *reinterpret_cast<const Pack8*>(kqp + b * 2 * BOX + sw128_offset(r, ch0 + i));
                        unpack8(kr[i], kx);
                        unpack8(*reinterpret_cast<const Pack8*>(kqp + b * 2 * BOX + BOX + sw128_offset(r, ch0 + i)),
                                qx);
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            ks = fmaf(kx[e], kx[e], ks);
                            qs = fmaf(qx[e], qx[e], qs);
                        }
                    }
                    ks += __shfl_xor_sync(0xffffffffu, ks, 1);
                    qs += __shfl_xor_sync(0xffffffffu, qs, 1);
                    ks += __shfl_xor_sync(0xffffffffu, ks, 2);
                    qs += __shfl_xor_sync(0xffffffffu, qs, 2);
                    kv = rsqrtf(ks + 1e-6f);
                    if (qq == 0) {
                        kinv[r] = kv;
                        qinv[r] = rsqrtf(qs + 1e-6f) * scale;
                    }
                }
                const float ec = ecum[r];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float f[8];
                    unpack8(kr[i], f);
#pragma unroll
                    for (int e = 0; e < 8; e++) f[e] = (f[e] * kv) * ec;
                    *reinterpret_cast<Pack8*>(sm + OFF_KW + b * BOX + sw128_offset(r, ch0 + i)) = pack8(f);
                }
            }
            named_bar_sync(BAR_PREP, NPREP);  // norms and kw are in
            if (pt == 0) {
                __threadfence_block();
                *norms_done = c + 1;
            }
            // A (rows of k, TMEM lanes 0..63) and P (rows of q, lanes 64..127) from D1;
            // warp pw reads lane quarter pw % 4, columns 32 (pw / 4) .. + 31. P goes into this
            // chunk's buffer once the update MMAs of chunk c - 2 have read it.
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_D1_FULL), (uint32_t)c & 1u) &&
                                                   mbar_wait(bar(B_P_FREE + slot), (uint32_t)((c >> 1) + 1) & 1u));
            if (ok) {
                tc_fence_after();
                const int j0 = (pw >> 2) * 32, row = wq * 32 + lane;
                // the lane quarters of rows 0..31 (k) and 0..31 (q) have nothing left of the
                // diagonal in columns 32..63
                const bool live = (wq & 1) || j0 == 0;
                float d[32];
                tmem_ld32(lrow + TM_D1 + (uint32_t)j0, d);
                tmem_ld_wait();
                if (row < C) {
                    // the off-diagonal block A_10 row-major at A[i][j]; the diagonal blocks
                    // transposed in place, A_bb[i][j] at A[j][i] (conflict-free: lane = i)
                    const int i = row;
                    const bool diag = (i >> 5) == (j0 >> 5);
                    if (live) {
                        const float ci = cum2[i], si = bet[i] * kinv[i];
#pragma unroll
                        for (int j4 = 0; j4 < 8; j4++) {
                            const float4 kv4 = *reinterpret_cast<const float4*>(kinv + j0 + j4 * 4);
                            const float4 cv4 = *reinterpret_cast<const float4*>(cum2 + j0 + j4 * 4);
                            const float kv[4] = {kv4.x, kv4.y, kv4.z, kv4.w}, cv[4] = {cv4.x, cv4.y, cv4.z, cv4.w};
                            float f[4];
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const int j = j0 + j4 * 4 + e;
                                f[e] = j < i ? si * (d[j4 * 4 + e] * kv[e]) * ex2(ci - cv[e]) : 0.f;
                            }
                            if (diag) {
#pragma unroll
                                for (int e = 0; e < 4; e++) A[(j0 + j4 * 4 + e) * LDT + i] = f[e];
                            } else {
                                *reinterpret_cast<float4*>(A + i * LDT + j0 + j4 * 4) = make_float4(f[0], f[1], f[2], f[3]);
                            }
                        }
                    }
                } else {
                    const int t = row - C;
                    uint8_t* pt_tile = sm + OFF_P + slot * BOX;
                    const float ct = cum2[t], st_ = qinv[t];
#pragma unroll
                    for (int c8 = 0; c8 < 4; c8++) {
                        float f[8], kv[8], cv[8];
                        *reinterpret_cast<float4*>(kv) = *reinterpret_cast<const float4*>(kinv + j0 + c8 * 8);
                        *reinterpret_cast<float4*>(kv + 4) = *reinterpret_cast<const float4*>(kinv + j0 + c8 * 8 + 4);
                        *reinterpret_cast<float4*>(cv) = *reinterpret_cast<const float4*>(cum2 + j0 + c8 * 8);
                        *reinterpret_cast<float4*>(cv + 4) = *reinterpret_cast<const float4*>(cum2 + j0 + c8 * 8 + 4);
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const int j = j0 + c8 * 8 + e;
                            f[e] = (live && j <= t) ? (d[c8 * 8 + e] * st_) * kv[e] * ex2(ct - cv[e]) : 0.f;
                        }
                        *reinterpret_cast<Pack8*>(pt_tile + sw128_offset(t, (j0 >> 3) + c8)) = pack8(f);
                    }
                }
                fence_async_smem();  // P (and kw) are read by MMAs
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(bar(B_OPS2_READY + slot));
                    mbar_arrive(bar(B_IN_KQ_FREE + slot));  // MMA1 is done and the norms pass read k, q
                }
            }
            named_bar_sync(BAR_PREP, NPREP);  // A complete
            // T = (I + A)^-1 by block doubling, written out as tb = bf16(T diag(beta)) (K-major
            // [64 t][64 j]) as the entries become final. Level 0: the eight 8 x 8 diagonal
            // blocks by right-looking substitution, one thread per (block, column). Levels 1 and
            // 2: the block below the diagonal of each 16 x 16, then 32 x 32 diagonal block,
            // T_10 = -T_11 (A_10 T_00), one thread per entry (two at level 2). Level 3, the 32 x 32
            // block below the two diagonal ones, follows in the same form. Inside the diagonal
            // 32-blocks A(r, c) sits at A[c][r] (transposed) and T(r, c) at Tm[r][c mod 32];
            // every entry above the diagonal of those blocks is written as 0, so the sums below
            // run over whole blocks.
            uint8_t* tb = sm + OFF_TB;
            bf16* tcol = reinterpret_cast<bf16*>(tb);
            auto put_tb = [&](int t, int jj, float tv) {
                tcol[(sw128_offset(t, jj >> 3) >> 1) + (jj & 7)] = to_bf16(tv * bet[jj]);
            };
            auto adiag = [&](int r, int cc) { return A[cc * LDT + r]; };
            auto tdiag = [&](int r, int cc) -> float& { return Tm[r * LDD + (cc & 31)]; };
            if (ok && pt < C) {
                const int o8 = (pt >> 3) * 8, col = pt & 7;
                float x[8];
#pragma unroll
                for (int r = 0; r < 8; r++) x[r] = r == col ? 1.f : 0.f;
#pragma unroll
                for (int m = 0; m < 7; m++) {
                    const float xm = x[m];
#pragma unroll
                    for (int r = m + 1; r < 8; r++) x[r] = fmaf(-adiag(o8 + r, o8 + m), xm, x[r]);
                }
#pragma unroll
                for (int r = 0; r < 8; r++) {
                    const float tv = r < col ? 0.f : x[r];
                    tdiag(o8 + r, o8 + col) = tv;
                    put_tb(o8 + r, o8 + col, tv);
                }
            } else if (ok) {
                // zeros: the six 8 x 8 blocks above the diagonal ones inside each 32-block (Tm and
                // tb), four entries per thread, and tb's upper block (rows 0..31, columns 32..63)
                const int u = pt - C;
#pragma unroll
                for (int e4 = 0; e4 < 4; e4++) {
                    const int e = u + (NPREP - C) * e4, b = e / 384, rem = e - b * 384, blk = rem >> 6;
                    const int bi = blk < 3 ? 0 : blk < 5 ? 1 : 2, bj = blk < 3 ? blk + 1 : blk < 5 ? blk - 1 : 3;
                    const int r = b * 32 + bi * 8 + ((rem >> 3) & 7), cc = b * 32 + bj * 8 + (rem & 7);
                    tdiag(r, cc) = 0.f;
                    put_tb(r, cc, 0.f);
                }
                if (u < 32 * 4) {
                    const int t = u >> 2, ch = 4 + (u & 3);
                    *reinterpret_cast<uint4*>(tb + sw128_offset(t, ch)) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            named_bar_sync(BAR_PREP, NPREP);
            // levels 1 (8 -> 16) and 2 (16 -> 32), each sum unrolled over its block so that
            // the loads are in flight together
            auto join = [&](auto hb_c) {
                constexpr int HB = decltype(hb_c)::value;  // size of the blocks being joined
                constexpr int PER = HB * HB, N = HB == 8 ? 1 : 2, TPJ = PER / N;
                const int pair = pt / TPJ, o0 = pair * 2 * HB, o1 = o0 + HB;
                const int idx = (pt - pair * TPJ) * N, i = idx / HB, j0 = idx % HB;
                float* xs = X + pair * PER;
                float acc[N];
#pragma unroll
                for (int e = 0; e < N; e++) acc[e] = 0.f;
                // (entry pairs, N = 2, are read as float2: j0 is even)
                auto pair2 = [](const float* p2) { return *reinterpret_cast<const float2*>(p2); };
#pragma unroll
                for (int m = 0; m < HB; m++) {
                    const float a = adiag(o1 + i, o0 + m);
                    if constexpr (N == 2) {
                        const float2 t2 = pair2(&tdiag(o0 + m, o0 + j0));
                        acc[0] = fmaf(a, t2.x, acc[0]);
                        acc[1] = fmaf(a, t2.y, acc[1]);
                    } else {
                        acc[0] = fmaf(a, tdiag(o0 + m, o0 + j0), acc[0]);
                    }
                }
#pragma unroll
                for (int e = 0; e < N; e++) xs[idx + e] = acc[e];
                named_bar_sync(BAR_PREP, NPREP);
#pragma unroll
                for (int e = 0; e < N; e++) acc[e] = 0.f;
                const float* trow = &tdiag(o1 + i, o1);  // row o1 + i of the diagonal block, 16-byte aligned
#pragma unroll
                for (int m4 = 0; m4 < HB; m4 += 4) {
                    const float4 t4 = *reinterpret_cast<const float4*>(trow + m4);
                    const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
                    for (int e4 = 0; e4 < 4; e4++) {
                        const int m = m4 + e4;
                        if constexpr (N == 2) {
                            const float2 x2 = pair2(xs + m * HB + j0);
                            acc[0] = fmaf(tv[e4], x2.x, acc[0]);
                            acc[1] = fmaf(tv[e4], x2.y, acc[1]);
                        } else {
                            acc[0] = fmaf(tv[e4], xs[m * HB + j0], acc[0]);
                        }
                    }
                }
                if (ok) {
#pragma unroll
                    for (int e = 0; e < N; e++) {
                        tdiag(o1 + i, o0 + j0 + e) = -acc[e];
                        put_tb(o1 + i, o0 + j0 + e, -acc[e]);
                    }
                }
                named_bar_sync(BAR_PREP, NPREP);
            };
            join(std::integral_constant<int, 8>{});
            join(std::integral_constant<int, 16>{});
            // X = A_10 T_00, then T_10 = -T_11 X; thread = (row r, 4 columns c4)
            {
                const int r = pt >> 3, c4 = (pt & 7) * 4;
                const float* arow = A + (32 + r) * LDT;
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 2
                for (int m4 = 0; m4 < 32; m4 += 4) {
                    const float4 av4 = *reinterpret_cast<const float4*>(arow + m4);
                    const float av[4] = {av4.x, av4.y, av4.z, av4.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float4 tv = *reinterpret_cast<const float4*>(Tm + (m4 + e) * LDD + c4);
                        a0 = fmaf(av[e], tv.x, a0);
                        a1 = fmaf(av[e], tv.y, a1);
                        a2 = fmaf(av[e], tv.z, a2);
                        a3 = fmaf(av[e], tv.w, a3);
                    }
                }
                *reinterpret_cast<float4*>(X + r * 32 + c4) = make_float4(a0, a1, a2, a3);
                named_bar_sync(BAR_PREP, NPREP);
                const float* trow = Tm + (32 + r) * LDD;
                a0 = a1 = a2 = a3 = 0.f;
                for (int m4 = 0; m4 <= r; m4 += 4) {  // T_11 is lower triangular: rows r >= m
                    const float4 tv4 = *reinterpret_cast<const float4*>(trow + m4);
                    const float tv[4] = {tv4.x, tv4.y, tv4.z, tv4.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float4 xv = *reinterpret_cast<const float4*>(X + (m4 + e) * 32 + c4);
                        const float t_ = m4 + e <= r ? tv[e] : 0.f;
                        a0 = fmaf(t_, xv.x, a0);
                        a1 = fmaf(t_, xv.y, a1);
                        a2 = fmaf(t_, xv.z, a2);
                        a3 = fmaf(t_, xv.w, a3);
                    }
                }
                if (ok) {
                    const int t = 32 + r;
                    uint2 pk;
                    pk.x = pack_bf16x2(-a0 * bet[c4], -a1 * bet[c4 + 1]);
                    pk.y = pack_bf16x2(-a2 * bet[c4 + 2], -a3 * bet[c4 + 3]);
                    *reinterpret_cast<uint2*>(tb + sw128_offset(t, c4 >> 3) + (c4 & 7) * 2) = pk;
                }
            }
            fence_async_smem();
            tc_fence_before();  // the D1 loads are complete before MMA2 rewrites those columns
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(bar(B_TB_READY));
            // w^T from TMEM (lane = k) into this chunk's MN-major [128 k][64 t] operand tile, once
            // the first scan MMAs of chunk c - 2 have read it
            ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(B_MMA2_DONE), (uint32_t)c & 1u) &&
                                                   mbar_wait(bar(B_W_FREE + slot), (uint32_t)((c >> 1) + 1) & 1u));
            if (ok) {
                tc_fence_after();
                const int t0w = (pw >> 2) * 32, kr = wq * 32 + lane;
                float x[32];
                tmem_ld32(lrow + TM_D1 + (uint32_t)t0w, x);
                tmem_ld_wait();
#pragma unroll
                for (int c4 = 0; c4 < 4; c4++)
                    *reinterpret_cast<Pack8*>(sm + OFF_W + slot * 2 * BOX + sw128_offset(kr, (t0w >> 3) + c4)) =
                        pack8(x + 8 * c4);
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(bar(B_OPS_READY + slot));
                    mbar_arrive(bar(B_D1W_FREE));
                    mbar_arrive(bar(B_VEC_FREE + slot));
                }
            }
        }
        tc_fence_before();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace gdnf

namespace gdn {

// The fused prefill over packed sequences (no workspace). Defined for the layouts of
// cs1_gdn_prefill: q, k [rows][HK][128], v, o [rows][H][128] bf16, g [rows][H] fp32,
// beta [rows][H] bf16; s_in / s_out [count][H][128][128] fp32 (s_in_stride 0: one state
// for every sequence).
int run_fused(const void* q, const void* k, const void* v, const float* g, const void* beta, void* o,
              const SeqTable& seqs, int H, int HK, float scale, const void* s_in, long s_in_stride, void* s_out,
              cudaStream_t st, const DevBatch* dyn, int cap_seqs, const float* rnorm_q, const float* rnorm_k) {
    using namespace gdnf;
    if (!q || !k || !v || !g || !beta || !o || H <= 0 || HK <= 0 || H % HK || H > 65535 || seqs.count > 65535)
        return cudaErrorInvalidValue;
    if (dyn && (cap_seqs <= 0 || cap_seqs > MAX_SEQS)) return cudaErrorInvalidValue;
    if ((rnorm_q == nullptr) != (rnorm_k == nullptr)) return cudaErrorInvalidValue;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return cudaErrorInvalidValue;
    static const cudaError_t configured =
        cudaFuncSetAttribute(gdn_fused<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (configured != cudaSuccess) return configured;
    static const cudaError_t configured_dyn =
        cudaFuncSetAttribute(gdn_fused<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (configured_dyn != cudaSuccess) return configured_dyn;
    const uint64_t rows = (uint64_t)seqs.offset[seqs.count];
    Maps maps;
    int e = host::make_map_3d_bf16(&maps.q, q, K, HK, rows, K, (uint64_t)HK * K, 64, 64);
    if (!e) e = host::make_map_3d_bf16(&maps.k, k, K, HK, rows, K, (uint64_t)HK * K, 64, 64);
    if (!e) e = host::make_map_3d_bf16(&maps.v, v, V, H, rows, V, (uint64_t)H * V, 64, 64);
    if (e) return e;
    return launch_pdl(dyn ? gdn_fused<true> : gdn_fused<false>, dim3(H, dyn ? cap_seqs : seqs.count), dim3(THREADS), SMEM, st, maps, g,
                      static_cast<const bf16*>(beta), seqs, static_cast<bf16*>(o), H, HK, scale,
                      static_cast<const float*>(s_in), s_in_stride, static_cast<float*>(s_out), dyn, rnorm_q, rnorm_k);
}

}  // namespace gdn
}  // namespace s1
