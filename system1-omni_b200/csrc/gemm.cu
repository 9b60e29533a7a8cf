// Projection GEMMs of the Qwen3.5 prefill on Blackwell tensor cores.
//
//   y[M, N] = x[M, K] * w[N, K]^T     bf16 in, fp32 accumulate in tensor memory, bf16 out
//
// One persistent, warp-specialised kernel per (tile width, epilogue):
//   warp 0      TMA producer: 128x64 A and BNx64 B tiles (128-byte swizzle) into a
//               ring of shared-memory stages, completion counted on mbarriers
//   warp 1      allocates tensor memory, one thread issues tcgen05.mma (M=128, N=BN,
//               K=16) into one of two TMEM accumulators and commits to mbarriers
//   warps 2..5  epilogue: tcgen05.ld of their 32 TMEM lanes (= 32 output rows),
//               bf16 conversion and the fused epilogue, stores to global memory;
//               the accumulator is released while the next tile's MMAs run in the
//               other one.
// Tiles are walked in groups of GROUP_M row blocks so that the CTAs resident at
// one time share A rows and B rows in L2.
//
// Every output element's K reduction runs in the same order whatever M, the row
// index or the tile width, so a row's result does not depend on how rows were
// packed (the property cs1_gemm_create_fixed promises in the reference's ops.h).
//
// Fused epilogues (additive symbols):
//   cs1_gemm_residual: residual = bf16(residual + bf16(x w^T))   (decoder residual add)
//   cs1_gemm_swiglu:   out = bf16(bf16(silu(gate)) * up), with gate and up rows of w
//                      interleaved in blocks of 128 (SwiGLU of the MLP)
#include <algorithm>
#include <cstdlib>
#include <new>
#include <string>

#include "common.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(gemm)

namespace s1 {
namespace gemm {

using namespace s1::tc;

constexpr int BM = 128, BK = 64, THREADS = 192, GROUP_M = 16;
enum Epi : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2 };

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int STG_OFFSET = STAGES * STAGE_BYTES;   // epilogue staging, 4 warps x 32 rows x 80 B
    static constexpr int BAR_OFFSET = STG_OFFSET + 4 * 32 * 80;
    static constexpr int SMEM = BAR_OFFSET + 256 + 1024;  // barriers + TMEM address + alignment slack
};

struct Params {
    bf16* y;
    int ldy;
    int M, N, K;
    int tiles_m, tiles_n;
    int group;  // > 0: tiles walked in groups of `group` row blocks; < 0: groups of -group column blocks
    const DevBatch* dyn;  // capacity path: M is the capacity, the batch's rows come from here
};

// Tile t -> (row block m, column block n). With group g > 0 the CTAs resident at one time
// share g row blocks of A and sweep the columns; with g < 0 they share -g column blocks
// of B and sweep the rows.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group, int& m, int& n) {
    if (group > 0) {
        const int per_group = group * tiles_n;
        const int gi = t / per_group;
        const int first = gi * group;
        const int gm = min(group, tiles_m - first);
        const int r = t - gi * per_group;
        m = first + r % gm;
        n = r / gm;
    } else {
        const int g = -group;
        const int per_group = g * tiles_m;
        const int gi = t / per_group;
        const int first = gi * g;
        const int gn = min(g, tiles_n - first);
        const int r = t - gi * per_group;
        n = first + r % gn;
        m = r / gn;
    }
}

// Epilogue store of one warp's 32 rows x 32 columns: lane i holds row row0 + i (v: its
// 32 columns, the STORE / RESIDUAL accumulator or the finished SwiGLU output). The block
// goes through a private shared-memory tile (rows 80 bytes apart: the 16-byte chunks of
// any 8 rows fall in distinct bank groups) and leaves as 64-byte row segments, so a warp
// store writes whole 32-byte sectors of 8 rows instead of 16 bytes of 32 rows. The
// residual is read the same way; numerics as before: bf16(acc), bf16(res + bf16(acc)).
template <int EPI>
__device__ __forceinline__ void store_block(uint8_t* stg, const float (&v)[32], bf16* y, int ldy, int row0,
                                            int M, int col, int out_n, int lane) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = v[j * 8 + e];
        *reinterpret_cast<Pack8*>(stg + lane * 80 + j * 16) = pack8(f);
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int ch = lane + 32 * j, i = ch >> 2, part = ch & 3;
        const int row = row0 + i, c = col + part * 8;
        if (row < M && c + 8 <= out_n) {
            const Pack8 val = *reinterpret_cast<const Pack8*>(stg + i * 80 + part * 16);
            bf16* dst = y + (size_t)row * ldy + c;
            if constexpr (EPI == EPI_RESIDUAL) {
                float r[8], a[8];
                unpack8(ld8(dst), r);
                unpack8(val, a);
#pragma unroll
                for (int e = 0; e < 8; e++) r[e] += a[e];
                st8(dst, pack8(r));
            } else {
                st8(dst, val);
            }
        }
    }
    __syncwarp();
}

template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Params p) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + C::BAR_OFFSET;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * C::STAGES + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * C::STAGES + 2 + a); };
    const uint32_t drain = bars + 8u * (2 * C::STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BAR_OFFSET + 8 * (2 * C::STAGES + 5));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (p.dyn) {  // capacity path: only the batch's row blocks
        p.M = min(p.M, p.dyn->rows);
        p.tiles_m = (p.M + BM - 1) / BM;
    }
    const int num_tiles = p.tiles_m * p.tiles_n;
    const int KB = (p.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 4);
        }
        mbar_init(drain, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int m, n;
                tile_coords(t, p.tiles_m, p.tiles_n, p.group, m, n);
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(empty(s), ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
                        ok = false;
                        break;
                    }
                    const uint32_t a_dst = base + s * C::STAGE_BYTES;
                    mbar_expect_tx(full(s), C::STAGE_BYTES);
                    tma_load_2d(a_dst, &map_a, full(s), kb * BK, m * BM);
                    tma_load_2d(a_dst + C::A_BYTES, &map_b, full(s), kb * BK, n * BN);
                    issued++;
                    if (++s == C::STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            // Drain: every load this thread issued has landed before the CTA exits.
            const long pending = issued < C::STAGES ? issued : C::STAGES;
            for (long i = 0; i < pending; i++) {
                if (--s < 0) {
                    s = C::STAGES - 1;
                    ph ^= 1;
                }
                (void)mbar_wait(full(s), ph);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc(BM, BN, AB_BF16);
            int s = 0, acc = 0;
            uint32_t ph = 0, acc_ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(tempty(acc), acc_ph ^ 1)) {
                    atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(full(s), ph)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = base + s * C::STAGE_BYTES;
                    const uint64_t ad = desc_sw128(a_addr), bd = desc_sw128(a_addr + C::A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        mma_bf16(d, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
                    mma_commit(empty(s));
                    if (++s == C::STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(tfull(acc));
                if (++acc == 2) {
                    acc = 0;
                    acc_ph ^= 1;
                }
            }
            // All MMAs of this CTA complete before tensor memory is freed.
            mma_commit(drain);
            (void)mbar_wait(drain, 0);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
        int acc = 0;
        uint32_t acc_ph = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int m, n;
            tile_coords(t, p.tiles_m, p.tiles_n, p.group, m, n);
            if (!mbar_wait(tfull(acc), acc_ph)) {
                if (lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int row0 = m * BM + q * 32;  // this warp's 32 rows
            const uint32_t tcol = lane_addr + acc * BN;
            uint8_t* stg = smem + C::STG_OFFSET + q * 32 * 80;
            if constexpr (EPI == EPI_SWIGLU) {
                // columns [0, BN/2) are gate rows, [BN/2, BN) the matching up rows
                const int out_col0 = n * (BN / 2);
#pragma unroll 1
                for (int c = 0; c < BN / 64; c++) {
                    float g[32], u[32];
                    tmem_ld32(tcol + c * 32, g);
                    tmem_ld32(tcol + BN / 2 + c * 32, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e++) g[e] = rbf(silu_hw(rbf(g[e]))) * rbf(u[e]);
                    store_block<EPI>(stg, g, p.y, p.ldy, row0, p.M, out_col0 + c * 32, p.N / 2, lane);
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    float v[32];
                    tmem_ld32(tcol + c * 32, v);
                    tmem_ld_wait();
                    store_block<EPI>(stg, v, p.y, p.ldy, row0, p.M, n * BN + c * 32, p.N, lane);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(acc));
            if (++acc == 2) {
                acc = 0;
                acc_ph ^= 1;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x 256 tile. Each CTA loads its own 128 rows of A and one half (128 rows) of B
// per stage (32 KB instead of 48 KB for the same per-SM MMA work), the even (leader)
// CTA issues M=256 N=256 MMAs that read both CTAs' shared memory, and each CTA holds
// its 128 accumulator rows in its own tensor memory for its own epilogue.
//   - TMA completions of both CTAs count on the leader's full barrier;
//   - the leader's commits arrive on both CTAs' empty / tmem-full barriers (multicast
//     commit, no multicast loads);
//   - both CTAs' epilogue warps arrive on the leader's tmem-empty barrier.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;
constexpr int P_B_BYTES = 128 * BK * 2;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_STG_OFFSET = P_STAGES * P_STAGE_BYTES;  // epilogue staging, 4 warps x 32 rows x 80 B
constexpr int P_BAR_OFFSET = P_STG_OFFSET + 4 * 32 * 80;
constexpr int P_SMEM = P_BAR_OFFSET + 256 + 1024;
constexpr int P_GROUP_M = 16;


template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Params p) {
    constexpr int BN = 256;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + P_BAR_OFFSET;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (P_STAGES + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * P_STAGES + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * P_STAGES + 2 + a); };
    const uint32_t drain = bars + 8u * (2 * P_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P_BAR_OFFSET + 8 * (2 * P_STAGES + 5));

    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (p.dyn) {  // capacity path: only the batch's row blocks (both CTAs of a pair agree)
        p.M = min(p.M, p.dyn->rows);
        p.tiles_m = (p.M + 255) / 256;
    }
    const int num_tiles = p.tiles_m * p.tiles_n;
    const int KB = (p.K + BK - 1) / BK;
    const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 8);
        }
        mbar_init(drain, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), 2 * BN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any remote arrive or TMA completion
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            bool ok = true;
            for (int t = cid; t < num_tiles && ok; t += nclusters) {
                int m, n;
                tile_coords(t, p.tiles_m, p.tiles_n, p.group, m, n);
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(empty(s), ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
                        ok = false;
                        break;
                    }
                    const uint32_t a_dst = base + s * P_STAGE_BYTES;
                    if (leader) mbar_expect_tx(full(s), 2 * P_STAGE_BYTES);
                    tma_load_2d_pair(a_dst, &map_a, full(s), kb * BK, m * 256 + (int)rank * 128);
                    tma_load_2d_pair(a_dst + P_A_BYTES, &map_b, full(s), kb * BK, n * BN + (int)rank * 128);
                    issued++;
                    if (++s == P_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (leader) {
                // every load of both CTAs has landed (all complete on the leader's barriers)
                const long pending = issued < P_STAGES ? issued : P_STAGES;
                for (long i = 0; i < pending; i++) {
                    if (--s < 0) {
                        s = P_STAGES - 1;
                        ph ^= 1;
                    }
                    (void)mbar_wait(full(s), ph);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            if (leader) {
                constexpr uint32_t IDESC = idesc(256, BN, AB_BF16);
                int s = 0, acc = 0;
                uint32_t ph = 0, acc_ph = 0;
                bool ok = true;
                for (int t = cid; t < num_tiles && ok; t += nclusters) {
                    if (!mbar_wait(tempty(acc), acc_ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + acc * BN;
                    for (int kb = 0; kb < KB; kb++) {
                        if (!mbar_wait(full(s), ph)) {
                            atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = base + s * P_STAGE_BYTES;
                        const uint64_t ad = desc_sw128(a_addr), bd = desc_sw128(a_addr + P_A_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / 16; k++)
                            mma_bf16_pair(d, ad + 2 * k, bd + 2 * k, IDESC, (kb | k) != 0);
                        mma_commit_pair(empty(s), 3);
                        if (++s == P_STAGES) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit_pair(tfull(acc), 3);
                    if (++acc == 2) {
                        acc = 0;
                        acc_ph ^= 1;
                    }
                }
                mma_commit_pair(drain, 3);
            }
            // both CTAs: the leader's MMAs (which write this CTA's tensor memory) are done
            (void)mbar_wait(drain, 0);
        }
    } else {
        const int q = warp & 3;
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
        const uint32_t leader_tempty0 = map_to_rank(tempty(0), 0), leader_tempty1 = map_to_rank(tempty(1), 0);
        int acc = 0;
        uint32_t acc_ph = 0;
        for (int t = cid; t < num_tiles; t += nclusters) {
            int m, n;
            tile_coords(t, p.tiles_m, p.tiles_n, p.group, m, n);
            if (!mbar_wait(tfull(acc), acc_ph)) {
                if (lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int row0 = m * 256 + (int)rank * 128 + q * 32;  // this warp's 32 rows
            const uint32_t tcol = lane_addr + acc * BN;
            uint8_t* stg = smem + P_STG_OFFSET + q * 32 * 80;
            if constexpr (EPI == EPI_SWIGLU) {
                const int out_col0 = n * (BN / 2);
#pragma unroll 1
                for (int c = 0; c < BN / 64; c++) {
                    float g[32], u[32];
                    tmem_ld32(tcol + c * 32, g);
                    tmem_ld32(tcol + BN / 2 + c * 32, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e++) g[e] = rbf(silu_hw(rbf(g[e]))) * rbf(u[e]);
                    store_block<EPI>(stg, g, p.y, p.ldy, row0, p.M, out_col0 + c * 32, p.N / 2, lane);
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    float v[32];
                    tmem_ld32(tcol + c * 32, v);
                    tmem_ld_wait();
                    store_block<EPI>(stg, v, p.y, p.ldy, row0, p.M, n * BN + c * 32, p.N, lane);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
            if (++acc == 2) {
                acc = 0;
                acc_ph ^= 1;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BN);
    }
}

// ---------------------------------------------------------------------------
// Swapped-operand variant for few rows of x (short prompts): the MMA's M side is 128
// rows of w (output columns) and its N side NT rows of x (a multiple of 16 up to 256),
// D^T[128 w rows][NT rows of x], so the rows of x are covered at a granularity of 16
// instead of 128 and the tile count can be matched to the SMs. The K reduction of each
// output element has the same order as in the other kernels. Epilogue warps own TMEM
// lanes = output columns; each stages 32 rows x 32 columns in shared memory and stores
// 64-byte row segments. A SwiGLU tile holds a gate block of w and its up block (two
// accumulators; NT <= 128).
constexpr int S_STAGES = 4;
constexpr int S_STAGE_BYTES = 48 * 1024;
constexpr int S_STG_OFFSET = S_STAGES * S_STAGE_BYTES;  // 4 warps x [32][32] bf16 staging
constexpr int S_BAR_OFFSET = S_STG_OFFSET + 4 * 2048;
constexpr int S_SMEM = S_BAR_OFFSET + 256 + 1024;

struct SwapParams {
    bf16* y;
    int ldy;
    int M, N, K;  // M rows of x, N rows of w (both halves for SwiGLU)
    int nt;       // rows of x per tile
    int tiles_w, tiles_t;
    int full;     // tiles done whole (whole waves); the rest are split along x
    int split;    // parts per remaining tile, of `sub` rows of x each
    int sub;
    int items;    // full + (tiles_w * tiles_t - full) * split
    int units;    // SMs (CTA pairs for the pair kernel) the split plan spreads a partial wave over
    const DevBatch* dyn;  // capacity path: M is the capacity, the batch's rows come from here
};

// Whole waves of tiles stay whole; the tiles of a last partial wave are split along x
// into parts of at least 64 rows so that they spread over the idle SMs.
__host__ __device__ inline void swap_split(int tiles, int sms, int nt, int& full, int& split, int& sub) {
    full = tiles / sms * sms;
    const int rem = tiles - full;
    split = 1;
    if (rem > 0) {
        const int by_sms = (sms + rem - 1) / rem;
        const int by_rows = nt / 64 > 1 ? nt / 64 : 1;
        split = by_sms < by_rows ? by_sms : by_rows;
        while (split > 1 && rem * split > sms) split--;
    }
    sub = ((nt + split - 1) / split + 15) & ~15;
    if (split == 1) full = tiles;
}

// The capacity path's plan for the batch's rows (the same plan the host makes for them).
__device__ __forceinline__ void swap_dyn(SwapParams& p) {
    if (!p.dyn) return;
    p.M = min(p.M, p.dyn->rows);
    p.tiles_t = (p.M + p.nt - 1) / p.nt;
    const int tiles = p.tiles_w * p.tiles_t;
    swap_split(tiles, p.units, p.nt, p.full, p.split, p.sub);
    p.items = p.full + (tiles - p.full) * p.split;
}

// Work item -> (w tile, first row of x, rows of x). Items past `full` are parts of the
// last partial wave's tiles, so that wave spreads over every SM; a part can be empty.
__device__ __forceinline__ void swap_item(const SwapParams& p, int t, int& wt, int& x0, int& rows) {
    int tile = t, part = 0, span = p.nt;
    if (t >= p.full) {
        const int u = t - p.full;
        tile = p.full + u / p.split;
        part = u - (u / p.split) * p.split;
        span = p.sub;
    }
    wt = tile / p.tiles_t;
    const int tt = tile - wt * p.tiles_t;
    x0 = tt * p.nt + part * span;
    rows = min(min(span, p.nt - part * span), p.M - x0);
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_swap_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                     SwapParams p) {
    constexpr bool SW = EPI == EPI_SWIGLU;
    constexpr int A_BYTES = BM * BK * 2;
    constexpr uint32_t B_OFF = SW ? 2 * A_BYTES : A_BYTES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + S_BAR_OFFSET;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (S_STAGES + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * S_STAGES + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * S_STAGES + 2 + a); };
    const uint32_t drain = bars + 8u * (2 * S_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S_BAR_OFFSET + 8 * (2 * S_STAGES + 5));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    swap_dyn(p);
    const int num_tiles = p.items;
    const int KB = (p.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 4);
        }
        mbar_init(drain, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_w);
        tma_prefetch_desc(&map_x);
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
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            bool ok = true;
            const uint32_t tx = B_OFF + (uint32_t)p.nt * BK * 2;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int wt, x0, rows;
                swap_item(p, t, wt, x0, rows);
                if (rows <= 0) continue;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(empty(s), ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
                        ok = false;
                        break;
                    }
                    const uint32_t dst = base + s * S_STAGE_BYTES;
                    mbar_expect_tx(full(s), tx);
                    tma_load_2d(dst, &map_w, full(s), kb * BK, SW ? wt * 256 : wt * BM);
                    if constexpr (SW) tma_load_2d(dst + A_BYTES, &map_w, full(s), kb * BK, wt * 256 + BM);
                    tma_load_2d(dst + B_OFF, &map_x, full(s), kb * BK, x0);
                    issued++;
                    if (++s == S_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            const long pending = issued < S_STAGES ? issued : S_STAGES;
            for (long i = 0; i < pending; i++) {
                if (--s < 0) {
                    s = S_STAGES - 1;
                    ph ^= 1;
                }
                (void)mbar_wait(full(s), ph);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int s = 0, acc = 0;
            uint32_t ph = 0, acc_ph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                int wt, x0, rows;
                swap_item(p, t, wt, x0, rows);
                if (rows <= 0) continue;
                const uint32_t id = idesc(BM, (rows + 15) & ~15, AB_BF16);
                if (!mbar_wait(tempty(acc), acc_ph ^ 1)) {
                    atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * 256;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(full(s), ph)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = base + s * S_STAGE_BYTES;
                    const uint64_t ad = desc_sw128(a_addr), bd = desc_sw128(a_addr + B_OFF);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) {
                        mma_bf16(d, ad + 2 * k, bd + 2 * k, id, (kb | k) != 0);
                        if constexpr (SW) mma_bf16(d + 128, desc_sw128(a_addr + A_BYTES) + 2 * k, bd + 2 * k, id,
                                                   (kb | k) != 0);
                    }
                    mma_commit(empty(s));
                    if (++s == S_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                mma_commit(tfull(acc));
                if (++acc == 2) {
                    acc = 0;
                    acc_ph ^= 1;
                }
            }
            mma_commit(drain);
            (void)mbar_wait(drain, 0);
        }
    } else {
        const int q = warp & 3;
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
        bf16* stg = reinterpret_cast<bf16*>(smem + S_STG_OFFSET + q * 2048);  // [32 rows of x][32 columns]
        const int out_n = SW ? p.N / 2 : p.N;
        int acc = 0;
        uint32_t acc_ph = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            int wt, row0, rows;
            swap_item(p, t, wt, row0, rows);
            if (rows <= 0) continue;
            if (!mbar_wait(tfull(acc), acc_ph)) {
                if (lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int col0 = wt * BM + q * 32;  // this warp's 32 output columns
#pragma unroll 1
            for (int c = 0; c * 32 < rows; c++) {
                float v[32];
                tmem_ld32(lane_addr + acc * 256 + c * 32, v);
                if constexpr (SW) {
                    float u[32];
                    tmem_ld32(lane_addr + acc * 256 + 128 + c * 32, u);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = rbf(silu_hw(rbf(v[i]))) * rbf(u[i]);
                } else {
                    tmem_ld_wait();
                }
                // STORE: bf16(acc); RESIDUAL: bf16(acc), added to the residual below; SwiGLU: the output
#pragma unroll
                for (int i = 0; i < 32; i++) stg[i * 32 + lane] = to_bf16(v[i]);
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int ch = lane + 32 * j, i = ch >> 2, part = ch & 3;
                    const int r = c * 32 + i, row = row0 + r, col = col0 + part * 8;
                    if (r < rows && col + 8 <= out_n) {  // rows of this tile only (r < rows implies row < M)
                        const Pack8 val = *reinterpret_cast<const Pack8*>(stg + i * 32 + part * 8);
                        bf16* dst = p.y + (size_t)row * p.ldy + col;
                        if constexpr (EPI == EPI_RESIDUAL) {
                            float r[8], a[8];
                            unpack8(ld8(dst), r);
                            unpack8(val, a);
#pragma unroll
                            for (int e = 0; e < 8; e++) r[e] += a[e];
                            st8(dst, pack8(r));
                        } else {
                            st8(dst, val);
                        }
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(acc));
            if (++acc == 2) {
                acc = 0;
                acc_ph ^= 1;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair swapped-operand variant: a cluster of two CTAs computes 256 rows of w (the
// MMA's M side, 128 per CTA) x N rows of x (N a multiple of 16, at most NT <= 256; each
// CTA loads N/2 of them, cta_group::2 splits the MMA's N side in halves). Per SM and
// MMA cycle it reads 8192 / N + 32 bytes of operands from shared memory, against
// 8192 / N + 64 for the single-CTA swapped kernel, and its tile of x is twice as wide.
// Work items, the split of the last partial wave and the epilogue follow the swapped
// kernel. SwiGLU: CTA r of a pair takes, from the 256-row block (gate 128 | up 128) of
// w, gate rows 64r .. 64r+63 into its A rows 0..63 and the up rows of the same output
// columns into A rows 64..127, so TMEM lanes l and l + 64 hold gate and up of one output
// column; the epilogue warps holding them (q and q + 2) pass rounded values through
// shared memory, each computing the outputs of every other 32-row chunk of x.
constexpr int SP_A_BYTES = BM * BK * 2;  // 128 rows of w
constexpr int SP_B_MAX = 128 * BK * 2;   // up to 128 rows of x (N <= 256)
constexpr int SP_STAGE_BYTES = SP_A_BYTES + SP_B_MAX;
template <int EPI>
struct SPCfg {
    static constexpr bool SW = EPI == EPI_SWIGLU;
    static constexpr int STAGES = SW ? 5 : 6;
    static constexpr int STG_OFFSET = STAGES * SP_STAGE_BYTES;  // 4 warps x [32][32] bf16 staging
    // SwiGLU exchange: per warp up to 4 chunks x [32 rows of x][32 lanes] bf16 for its partner
    static constexpr int XCH_OFFSET = STG_OFFSET + 4 * 2048;
    static constexpr int BAR_OFFSET = XCH_OFFSET + (SW ? 4 * 8192 : 0);
    static constexpr int SMEM = BAR_OFFSET + 256 + 1024;
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_swap_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                          SwapParams p) {
    using C = SPCfg<EPI>;
    constexpr bool SW = C::SW;
    constexpr int SP_STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + C::BAR_OFFSET;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (SP_STAGES + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * SP_STAGES + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * SP_STAGES + 2 + a); };
    const uint32_t drain = bars + 8u * (2 * SP_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::BAR_OFFSET + 8 * (2 * SP_STAGES + 5));

    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    swap_dyn(p);
    const int num_items = p.items;
    const int KB = (p.K + BK - 1) / BK;
    const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SP_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 8);
        }
        mbar_init(drain, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_w);
        tma_prefetch_desc(&map_x);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any remote arrive or TMA completion
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long issued = 0;
            bool ok = true;
            const uint32_t tx = 2u * (SP_A_BYTES + (uint32_t)(p.nt / 2) * BK * 2);
            for (int t = cid; t < num_items && ok; t += nclusters) {
                int wt, x0, rows;
                swap_item(p, t, wt, x0, rows);
                if (rows <= 0) continue;
                const int n_half = ((rows + 15) & ~15) / 2;
                // rows of w: SwiGLU gate 64r.. and up 128+64r.. of block wt; else 128r.. of tile wt
                const int w0 = SW ? wt * 256 + 64 * (int)rank : wt * 256 + 128 * (int)rank;
                const int w1 = SW ? w0 + 128 : w0 + 64;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(empty(s), ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
                        ok = false;
                        break;
                    }
                    const uint32_t dst = base + s * SP_STAGE_BYTES;
                    if (leader) mbar_expect_tx(full(s), tx);
                    tma_load_2d_pair(dst, &map_w, full(s), kb * BK, w0);
                    tma_load_2d_pair(dst + SP_A_BYTES / 2, &map_w, full(s), kb * BK, w1);
                    tma_load_2d_pair(dst + SP_A_BYTES, &map_x, full(s), kb * BK, x0 + (int)rank * n_half);
                    issued++;
                    if (++s == SP_STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (leader) {
                // every load of both CTAs has landed (all complete on the leader's barriers)
                const long pending = issued < SP_STAGES ? issued : SP_STAGES;
                for (long i = 0; i < pending; i++) {
                    if (--s < 0) {
                        s = SP_STAGES - 1;
                        ph ^= 1;
                    }
                    (void)mbar_wait(full(s), ph);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            if (leader) {
                int s = 0, acc = 0;
                uint32_t ph = 0, acc_ph = 0;
                bool ok = true;
                for (int t = cid; t < num_items && ok; t += nclusters) {
                    int wt, x0, rows;
                    swap_item(p, t, wt, x0, rows);
                    if (rows <= 0) continue;
                    const uint32_t id = idesc(256, (rows + 15) & ~15, AB_BF16);
                    if (!mbar_wait(tempty(acc), acc_ph ^ 1)) {
                        atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + acc * 256;
                    for (int kb = 0; kb < KB; kb++) {
                        if (!mbar_wait(full(s), ph)) {
                            atomicOr(&g_fault_word, FAULT_WAIT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = base + s * SP_STAGE_BYTES;
                        const uint64_t ad = desc_sw128(a_addr), bd = desc_sw128(a_addr + SP_A_BYTES);
#pragma unroll
                        for (int k = 0; k < BK / 16; k++) mma_bf16_pair(d, ad + 2 * k, bd + 2 * k, id, (kb | k) != 0);
                        mma_commit_pair(empty(s), 3);
                        if (++s == SP_STAGES) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit_pair(tfull(acc), 3);
                    if (++acc == 2) {
                        acc = 0;
                        acc_ph ^= 1;
                    }
                }
                mma_commit_pair(drain, 3);
            }
            // both CTAs: the leader's MMAs (which write this CTA's tensor memory) are done
            (void)mbar_wait(drain, 0);
        }
    } else {
        const int q = warp & 3;
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
        bf16* stg = reinterpret_cast<bf16*>(smem + C::STG_OFFSET + q * 2048);  // [32 rows of x][32 columns]
        // SwiGLU partners: warps q and q ^ 2 (gate lanes 32q.., up lanes 64 + 32q..)
        bf16* xsend = reinterpret_cast<bf16*>(smem + C::XCH_OFFSET + q * 8192);
        const bf16* xrecv = reinterpret_cast<const bf16*>(smem + C::XCH_OFFSET + (q ^ 2) * 8192);
        const uint32_t leader_tempty0 = map_to_rank(tempty(0), 0), leader_tempty1 = map_to_rank(tempty(1), 0);
        const int out_n = SW ? p.N / 2 : p.N;
        int acc = 0;
        uint32_t acc_ph = 0;
        for (int t = cid; t < num_items; t += nclusters) {
            int wt, row0, rows;
            swap_item(p, t, wt, row0, rows);
            if (rows <= 0) continue;
            bool bad = !__all_sync(0xffffffffu, mbar_wait(tfull(acc), acc_ph));
            if (SW) bad = bar_any(1 + (q & 1), 64, bad);  // the exchange partners leave together
            if (bad) {
                if (lane == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
                break;
            }
            tc_fence_after();
            // this warp's 32 output columns
            const int col0 = SW ? wt * 128 + 64 * (int)rank + (q & 1) * 32 : wt * 256 + 128 * (int)rank + q * 32;
            const uint32_t tacc = lane_addr + acc * 256;
            const int chunks = (rows + 31) / 32;
            // SwiGLU: the gate warp finishes the even chunks of 32 rows of x, the up warp the
            // odd ones; each first hands its partner the bf16-rounded values of the others
            const int own = SW ? (q < 2 ? 0 : 1) : 0, step = SW ? 2 : 1;
            if constexpr (SW) {
#pragma unroll 1
                for (int c = 1 - own; c < chunks; c += 2) {
                    float v[32];
                    tmem_ld32(tacc + c * 32, v);
                    tmem_ld_wait();
                    bf16* dst = xsend + (c >> 1) * 1024;
#pragma unroll
                    for (int i = 0; i < 32; i++) dst[i * 32 + lane] = to_bf16(v[i]);
                }
                named_bar_sync(1 + (q & 1), 64);
            }
#pragma unroll 1
            for (int c = own; c < chunks; c += step) {
                float v[32];
                tmem_ld32(tacc + c * 32, v);
                tmem_ld_wait();
                if constexpr (SW) {
                    const bf16* src = xrecv + (c >> 1) * 1024;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float o = f32(src[i * 32 + lane]);
                        v[i] = q < 2 ? rbf(silu_hw(rbf(v[i]))) * o : rbf(silu_hw(o)) * rbf(v[i]);
                    }
                }
                // STORE: bf16(acc); RESIDUAL: bf16(acc), added to the residual below; SwiGLU: the output
#pragma unroll
                for (int i = 0; i < 32; i++) stg[i * 32 + lane] = to_bf16(v[i]);
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int ch = lane + 32 * j, i = ch >> 2, part = ch & 3;
                    const int r = c * 32 + i, row = row0 + r, col = col0 + part * 8;
                    if (r < rows && col + 8 <= out_n) {  // rows of this item only (r < rows implies row < M)
                        const Pack8 val = *reinterpret_cast<const Pack8*>(stg + i * 32 + part * 8);
                        bf16* dst = p.y + (size_t)row * p.ldy + col;
                        if constexpr (EPI == EPI_RESIDUAL) {
                            float r8[8], a8[8];
                            unpack8(ld8(dst), r8);
                            unpack8(val, a8);
#pragma unroll
                            for (int e = 0; e < 8; e++) r8[e] += a8[e];
                            st8(dst, pack8(r8));
                        } else {
                            st8(dst, val);
                        }
                    }
                }
                __syncwarp();
            }
            if constexpr (SW) named_bar_sync(1 + (q & 1), 64);  // partner done reading before the next item's writes
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
            if (++acc == 2) {
                acc = 0;
                acc_ph ^= 1;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// Any shape: one thread per output, fp32 accumulation in K order. Used only when
// a shape or pointer misses the tensor-map alignment rules.
template <int EPI>
__global__ void gemm_simt_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* y, int ldy, int M,
                                 int N, int K) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
    if (m >= M) return;
    const int out_n = EPI == EPI_SWIGLU ? N / 2 : N;
    if (n >= out_n) return;
    const bf16* xr = x + (size_t)m * K;
    auto dot = [&](int row) {
        const bf16* wr = w + (size_t)row * K;
        float acc = 0.f;
        for (int k = 0; k < K; k++) acc = fmaf(f32(xr[k]), f32(wr[k]), acc);
        return acc;
    };
    if constexpr (EPI == EPI_SWIGLU) {
        const int blk = n / 128, j = n % 128;
        const float g = rbf(dot(blk * 256 + j)), u = rbf(dot(blk * 256 + 128 + j));
        y[(size_t)m * ldy + n] = to_bf16(rbf(silu_hw(g)) * u);
    } else if constexpr (EPI == EPI_RESIDUAL) {
        bf16* d = y + (size_t)m * ldy + n;
        *d = to_bf16(f32(*d) + rbf(dot(n)));
    } else {
        y[(size_t)m * ldy + n] = to_bf16(dot(n));
    }
}

struct Handle {
    int device = 0;
    int sms = 148;
    int fixed_m = 0;
    // The fields below are fixed in product builds; a build with -DS1_TUNING (build.py
    // --tuning) reads them from S1_GEMM_PAIRS, S1_GEMM_GROUP, S1_GEMM_SWAP, S1_GEMM_KERNEL
    // (pair | row256 | row128 | swap | swap2) and S1_GEMM_NT to calibrate the kernel choice.
    bool pairs = true;  // CTA-pair kernels for large M
    int group = 0;      // tile grouping (0: the kernels' defaults)
    bool swap = true;   // swapped-operand kernel for few rows
    // forced kernel (0 = the wave model's choice) and the swapped kernels' rows of x per tile
    int force = 0, force_nt = 0;
};
enum Force : int { FORCE_NONE = 0, FORCE_PAIR, FORCE_ROW256, FORCE_ROW128, FORCE_SWAP, FORCE_SWAP2 };

template <int BN, int EPI>
int launch_tc(const Handle* h, const void* x, const void* w, void* y, int M, int N, int K, int ldy,
              cudaStream_t st, const DevBatch* dyn) {
    using C = Cfg<BN>;
    static const cudaError_t configured =
        cudaFuncSetAttribute(gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (configured != cudaSuccess) return configured;
    CUtensorMap ma, mb;
    int e = host::make_map_2d(&ma, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, K, BM, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    e = host::make_map_2d(&mb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, BN, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    Params p;
    p.y = static_cast<bf16*>(y);
    p.ldy = ldy;
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = (M + BM - 1) / BM;
    p.tiles_n = (N + BN - 1) / BN;
    p.group = h->group ? h->group : GROUP_M;
    p.dyn = dyn;
    const int tiles = p.tiles_m * p.tiles_n;
    const int grid = std::min(tiles, h->sms);
    return launch_pdl(gemm_kernel<BN, EPI>, dim3(grid), dim3(THREADS), C::SMEM, st, ma, mb, p);
}

template <int EPI>
int launch_pair(const Handle* h, const void* x, const void* w, void* y, int M, int N, int K, int ldy,
                cudaStream_t st, const DevBatch* dyn) {
    static const cudaError_t configured =
        cudaFuncSetAttribute(gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
    if (configured != cudaSuccess) return configured;
    CUtensorMap ma, mb;
    int e = host::make_map_2d(&ma, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, K, 128, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    e = host::make_map_2d(&mb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, 128, BK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    Params p;
    p.y = static_cast<bf16*>(y);
    p.ldy = ldy;
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = (M + 255) / 256;
    p.tiles_n = (N + 255) / 256;
    p.group = h->group ? h->group : P_GROUP_M;
    p.dyn = dyn;
    const int tiles = p.tiles_m * p.tiles_n;
    const int grid = 2 * std::min(tiles, h->sms / 2);
    return launch_pdl(gemm_pair_kernel<EPI>, dim3(grid), dim3(THREADS), P_SMEM, st, ma, mb, p);
}


template <int EPI>
int launch_swap(const Handle* h, const void* x, const void* w, void* y, int M, int N, int K, int ldy, int nt,
                cudaStream_t st, const DevBatch* dyn) {
    static const cudaError_t configured =
        cudaFuncSetAttribute(gemm_swap_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_SMEM);
    if (configured != cudaSuccess) return configured;
    CUtensorMap mw, mx;
    int e = host::make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, BM, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    e = host::make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, K, (uint32_t)nt, BK,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    SwapParams p;
    p.y = static_cast<bf16*>(y);
    p.ldy = ldy;
    p.M = M;
    p.N = N;
    p.K = K;
    p.nt = nt;
    p.tiles_w = EPI == EPI_SWIGLU ? N / 256 : (N + BM - 1) / BM;
    p.tiles_t = (M + nt - 1) / nt;
    const int tiles = p.tiles_w * p.tiles_t;
    swap_split(tiles, h->sms, nt, p.full, p.split, p.sub);
    p.items = p.full + (tiles - p.full) * p.split;
    p.units = h->sms;
    p.dyn = dyn;
    // the capacity path's plan is made in the kernel: every SM may get an item
    const int grid = dyn ? h->sms : std::min(p.items, h->sms);
    return launch_pdl(gemm_swap_kernel<EPI>, dim3(grid), dim3(THREADS), S_SMEM, st, mw, mx, p);
}

template <int EPI>
int launch_swap_pair(const Handle* h, const void* x, const void* w, void* y, int M, int N, int K, int ldy, int nt,
                     cudaStream_t st, const DevBatch* dyn) {
    static const cudaError_t configured =
        cudaFuncSetAttribute(gemm_swap_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SPCfg<EPI>::SMEM);
    if (configured != cudaSuccess) return configured;
    CUtensorMap mw, mx;
    int e = host::make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, 64, BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    e = host::make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, K, (uint32_t)(nt / 2), BK,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (e) return e;
    SwapParams p;
    p.y = static_cast<bf16*>(y);
    p.ldy = ldy;
    p.M = M;
    p.N = N;
    p.K = K;
    p.nt = nt;
    p.tiles_w = EPI == EPI_SWIGLU ? N / 256 : (N + 255) / 256;
    p.tiles_t = (M + nt - 1) / nt;
    const int tiles = p.tiles_w * p.tiles_t, pairs = h->sms / 2;
    swap_split(tiles, pairs, nt, p.full, p.split, p.sub);
    p.items = p.full + (tiles - p.full) * p.split;
    p.units = pairs;
    p.dyn = dyn;
    const int grid = 2 * (dyn ? pairs : std::min(p.items, pairs));
    return launch_pdl(gemm_swap_pair_kernel<EPI>, dim3(grid), dim3(THREADS), SPCfg<EPI>::SMEM, st,
                      mw, mx, p);
}

// Best token tile of the swapped kernel and its estimated time in the units of the
// kernel choice below (waves x per-tile time relative to a 256 x 256 CTA-pair tile).
// A tile of 128 w rows x nt rows costs nt / 256 of a 128 x 256 single-CTA tile, scaled up
// where its operand bytes per MMA cycle (8192 / nt + 64; SwiGLU 8192 / nt + 32) exceed
// what the 128 x 256 tiles sustain (~90 B / cycle / SM). Constants fitted to sweeps of the
// 27B shapes with each kernel forced in turn (a -DS1_TUNING build).
double swap_cost(int M, int N, int epi, int sms, int& best_nt) {
    const bool sw = epi == EPI_SWIGLU;
    const long tiles_w = sw ? N / 256 : (N + BM - 1) / BM;
    double best = 1e30;
    best_nt = 0;
    for (int nt = 32; nt <= (sw ? 128 : 256); nt += 16) {
        const long tiles = tiles_w * ((M + nt - 1) / nt);
        int full, split, sub;
        swap_split((int)tiles, sms, nt, full, split, sub);
        const long whole = tiles / sms;  // whole waves; a partial one costs sub / nt of a wave
        const double waves = (double)whole + (tiles > whole * sms ? (double)sub / nt : 0.0);
        const double rate = 8192.0 / nt + (sw ? 32.0 : 64.0);
        const double eff = rate > 90.0 ? rate / 90.0 : 1.0;
        const double c = waves * 1.2 * (sw ? 2.0 : 1.0) * nt / 256.0 * eff;
        if (c < best) {
            best = c;
            best_nt = nt;
        }
    }
    return best;
}

// The same for the CTA-pair swapped kernel: a pair tile of 256 w rows x nt rows of x is
// nt / 256 of a 256 x 256 pair tile; operand bytes per MMA cycle and SM 8192 / nt + 32.
double swap_pair_cost(int M, int N, int epi, int sms, int& best_nt) {
    const long tiles_w = epi == EPI_SWIGLU ? N / 256 : (N + 255) / 256;
    const int pairs = sms / 2;
    double best = 1e30;
    best_nt = 0;
    for (int nt = 32; nt <= 256; nt += 16) {
        const long tiles = tiles_w * ((M + nt - 1) / nt);
        int full, split, sub;
        swap_split((int)tiles, pairs, nt, full, split, sub);
        const long whole = tiles / pairs;
        const double waves = (double)whole + (tiles > whole * pairs ? (double)sub / nt : 0.0);
        const double rate = 8192.0 / nt + 32.0;
        const double eff = rate > 70.0 ? rate / 70.0 : 1.0;
        const double c = waves * 1.15 * nt / 256.0 * eff;
        if (c < best) {
            best = c;
            best_nt = nt;
        }
    }
    return best;
}

int run(const Handle* h, const void* x, const void* w, void* y, int M, int N, int K, int ldy, int epi,
        cudaStream_t st, const DevBatch* dyn = nullptr) {
    if (!h || M < 0 || N <= 0 || K <= 0 || !x || !w || !y) return cudaErrorInvalidValue;
    const int out_n = epi == EPI_SWIGLU ? N / 2 : N;
    if (ldy < out_n) return cudaErrorInvalidValue;
    if (epi == EPI_SWIGLU && N % 256 != 0) return cudaErrorInvalidValue;
    if (M == 0) return cudaSuccess;
    const bool tc_ok = K % 8 == 0 && N % 8 == 0 && ldy % 8 == 0 && aligned16(x) && aligned16(w) && aligned16(y);
    if (!tc_ok) {
        if (dyn) return cudaErrorInvalidValue;  // the capacity path needs the tensor-core kernels
        const dim3 grid((out_n + 127) / 128, M);
        switch (epi) {
            case EPI_SWIGLU:
                gemm_simt_kernel<EPI_SWIGLU><<<grid, 128, 0, st>>>(static_cast<const bf16*>(x),
                    static_cast<const bf16*>(w), static_cast<bf16*>(y), ldy, M, N, K);
                break;
            case EPI_RESIDUAL:
                gemm_simt_kernel<EPI_RESIDUAL><<<grid, 128, 0, st>>>(static_cast<const bf16*>(x),
                    static_cast<const bf16*>(w), static_cast<bf16*>(y), ldy, M, N, K);
                break;
            default:
                gemm_simt_kernel<EPI_STORE><<<grid, 128, 0, st>>>(static_cast<const bf16*>(x),
                    static_cast<const bf16*>(w), static_cast<bf16*>(y), ldy, M, N, K);
        }
        return cudaGetLastError();
    }
    // Kernel choice by waves: a wave of the CTA-pair kernel is sms/2 tiles of 256x256, of
    // the single-CTA kernels sms tiles of 128x256 or 128x128. The pair kernel does the same
    // per-SM work per tile about 15% faster, the 128-wide kernel half the work about 20%
    // slower; pick the smallest estimated time (waves x relative tile time).
    const long pair_tiles = (long)((M + 255) / 256) * ((N + 255) / 256);
    const long t256 = (long)((M + BM - 1) / BM) * ((N + 255) / 256);
    const long t128 = (long)((M + BM - 1) / BM) * ((N + 127) / 128);
    const long slots = h->sms;
    const double c_pair = (double)((pair_tiles + slots / 2 - 1) / (slots / 2)) * 1.0;
    const double c_256 = (double)((t256 + slots - 1) / slots) * 1.15;
    const double c_128 = (double)((t128 + slots - 1) / slots) * 0.6;
    int nt = 0, nt2 = 0;
    double c_swap = h->swap ? swap_cost(M, N, epi, (int)slots, nt) : 1e30;
    double c_swap2 = h->swap && h->pairs ? swap_pair_cost(M, N, epi, (int)slots, nt2) : 1e30;
    double cp = c_pair, c2 = c_256, c1 = epi == EPI_SWIGLU ? 1e30 : c_128;
    if (h->force != FORCE_NONE) {  // tuning override: make the forced kernel the cheapest
        cp = h->force == FORCE_PAIR ? 0.0 : 1e30;
        c2 = h->force == FORCE_ROW256 ? 0.0 : 1e30;
        c1 = h->force == FORCE_ROW128 && epi != EPI_SWIGLU ? 0.0 : 1e30;
        c_swap = h->force == FORCE_SWAP ? 0.0 : 1e30;
        c_swap2 = h->force == FORCE_SWAP2 ? 0.0 : 1e30;
        if (h->force == FORCE_SWAP) {
            const int cap = epi == EPI_SWIGLU ? 128 : 256;
            nt = 0;
            if (h->force_nt >= 16 && h->force_nt <= cap && h->force_nt % 16 == 0) nt = h->force_nt;
            if (nt == 0) nt = 128;
        }
        if (h->force == FORCE_SWAP2) {
            nt2 = 0;
            if (h->force_nt >= 32 && h->force_nt <= 256 && h->force_nt % 16 == 0) nt2 = h->force_nt;
            if (nt2 == 0) nt2 = 256;
        }
        if ((h->force == FORCE_PAIR || h->force == FORCE_SWAP2) && !h->pairs) cp = c_swap2 = 1e30;
        if (cp != 0.0 && c2 != 0.0 && c1 != 0.0 && c_swap != 0.0 && c_swap2 != 0.0)
            c2 = 0.0;  // not applicable: 128 x 256
    }
    if (nt2 > 0 && c_swap2 < cp && c_swap2 < c2 && c_swap2 < c1 && c_swap2 <= c_swap) {
        switch (epi) {
            case EPI_SWIGLU:
                return launch_swap_pair<EPI_SWIGLU>(h, x, w, y, M, N, K, ldy, nt2, st, dyn);
            case EPI_RESIDUAL:
                return launch_swap_pair<EPI_RESIDUAL>(h, x, w, y, M, N, K, ldy, nt2, st, dyn);
            default:
                return launch_swap_pair<EPI_STORE>(h, x, w, y, M, N, K, ldy, nt2, st, dyn);
        }
    }
    if (nt > 0 && c_swap < cp && c_swap < c2 && c_swap < c1) {
        switch (epi) {
            case EPI_SWIGLU:
                return launch_swap<EPI_SWIGLU>(h, x, w, y, M, N, K, ldy, nt, st, dyn);
            case EPI_RESIDUAL:
                return launch_swap<EPI_RESIDUAL>(h, x, w, y, M, N, K, ldy, nt, st, dyn);
            default:
                return launch_swap<EPI_STORE>(h, x, w, y, M, N, K, ldy, nt, st, dyn);
        }
    }
    if (h->pairs && cp <= c2 && cp <= c1) {
        switch (epi) {
            case EPI_SWIGLU:
                return launch_pair<EPI_SWIGLU>(h, x, w, y, M, N, K, ldy, st, dyn);
            case EPI_RESIDUAL:
                return launch_pair<EPI_RESIDUAL>(h, x, w, y, M, N, K, ldy, st, dyn);
            default:
                return launch_pair<EPI_STORE>(h, x, w, y, M, N, K, ldy, st, dyn);
        }
    }
    const bool wide = epi == EPI_SWIGLU || c2 <= c1;
    switch (epi) {
        case EPI_SWIGLU:
            return launch_tc<256, EPI_SWIGLU>(h, x, w, y, M, N, K, ldy, st, dyn);
        case EPI_RESIDUAL:
            return wide ? launch_tc<256, EPI_RESIDUAL>(h, x, w, y, M, N, K, ldy, st, dyn)
                        : launch_tc<128, EPI_RESIDUAL>(h, x, w, y, M, N, K, ldy, st, dyn);
        default:
            return wide ? launch_tc<256, EPI_STORE>(h, x, w, y, M, N, K, ldy, st, dyn)
                        : launch_tc<128, EPI_STORE>(h, x, w, y, M, N, K, ldy, st, dyn);
    }
}

}  // namespace gemm
}  // namespace s1

using namespace s1;

extern "C" {

void* cs1_gemm_create(size_t workspace_bytes) {
    (void)workspace_bytes;  // the tcgen05 kernels need no library workspace
    auto* h = new (std::nothrow) gemm::Handle;
    if (!h) return nullptr;
    if (cudaGetDevice(&h->device) != cudaSuccess) {
        delete h;
        return nullptr;
    }
    h->sms = host::num_sms();
#ifdef S1_TUNING
    // tuning builds only (build.py --tuning): kernel overrides for calibrating the wave model
    const char* env = getenv("S1_GEMM_PAIRS");
    h->pairs = !(env && env[0] == '0');
    const char* grp = getenv("S1_GEMM_GROUP");
    if (grp) h->group = atoi(grp);
    const char* sw = getenv("S1_GEMM_SWAP");
    h->swap = !(sw && sw[0] == '0');
    if (const char* f = getenv("S1_GEMM_KERNEL")) {
        const std::string k(f);
        h->force = k == "pair" ? gemm::FORCE_PAIR : k == "row256" ? gemm::FORCE_ROW256
                 : k == "row128" ? gemm::FORCE_ROW128 : k == "swap" ? gemm::FORCE_SWAP
                 : k == "swap2" ? gemm::FORCE_SWAP2 : gemm::FORCE_NONE;
    }
    if (const char* nt = getenv("S1_GEMM_NT")) h->force_nt = atoi(nt);
#endif
    return h;
}

void* cs1_gemm_create_fixed(size_t workspace_bytes, int reference_m) {
    if (reference_m <= 0) return nullptr;
    auto* h = static_cast<gemm::Handle*>(cs1_gemm_create(workspace_bytes));
    if (h) h->fixed_m = reference_m;
    return h;
}

void* cs1_gemm_create_matched(size_t workspace_bytes, int reference_m) {
    return cs1_gemm_create_fixed(workspace_bytes, reference_m);
}

// Every handle runs the same M-independent kernels, so any two are compatible.
int cs1_gemm_compatible(void* ordinary, void* matched, int M, int N, int K) {
    (void)ordinary;
    (void)matched;
    return (M >= 0 && N > 0 && K > 0) ? 1 : 0;
}

void cs1_gemm_destroy(void* gemm) { delete static_cast<gemm::Handle*>(gemm); }

int cs1_gemm_enable_equivalent_tiles(void* gemm) { return gemm ? 1 : -1; }

int cs1_gemm(void* gemm, const void* x, const void* w, void* y, int M, int N, int K, int ldy, void* stream) {
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, y, M, N, K, ldy, gemm::EPI_STORE,
                     static_cast<cudaStream_t>(stream));
}

int cs1_gemm_packed(void* gemm, const void* x, const void* w, void* y, const size_t* lengths, size_t count, int N,
                    int K, void* stream) {
    if (!lengths || count == 0) return cudaErrorInvalidValue;
    size_t rows = 0;
    for (size_t i = 0; i < count; i++) {
        if (lengths[i] == 0) return cudaErrorInvalidValue;
        rows += lengths[i];
    }
    if (rows > 0x7FFFFFFF) return cudaErrorInvalidValue;
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, y, (int)rows, N, K, N, gemm::EPI_STORE,
                     static_cast<cudaStream_t>(stream));
}

int cs1_gemm_reuse_check(void* gemm, const size_t* original_rows, size_t originals, const size_t* target_rows,
                         size_t targets, int N, int K) {
    if (!gemm || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    (void)original_rows;
    (void)originals;
    (void)target_rows;
    (void)targets;
    return 0;
}

int cs1_gemm_reuse(void* gemm, const void* x, const void* w, void* y, int M, int N, int K, int original_M,
                   void* stream) {
    (void)original_M;
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, y, M, N, K, N, gemm::EPI_STORE,
                     static_cast<cudaStream_t>(stream));
}

int cs1_gemm_residual(void* gemm, const void* x, const void* w, void* residual, int M, int N, int K, int ldr,
                      void* stream) {
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, residual, M, N, K, ldr, gemm::EPI_RESIDUAL,
                     static_cast<cudaStream_t>(stream));
}

int cs1_gemm_swiglu(void* gemm, const void* x, const void* w, void* out, int M, int I, int K, int ldo,
                    void* stream) {
    if (I <= 0 || I % 128 != 0) return cudaErrorInvalidValue;
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, out, M, 2 * I, K, ldo, gemm::EPI_SWIGLU,
                     static_cast<cudaStream_t>(stream));
}

int cs1_gemm_dyn(void* gemm, const void* x, const void* w, void* y, int cap_rows, int N, int K, int ldy,
                 int epilogue, const void* desc, void* stream) {
    if (!desc || cap_rows <= 0 || epilogue < gemm::EPI_STORE || epilogue > gemm::EPI_SWIGLU)
        return cudaErrorInvalidValue;
    if (epilogue == gemm::EPI_SWIGLU && (N <= 0 || N % 256 != 0)) return cudaErrorInvalidValue;
    return gemm::run(static_cast<const gemm::Handle*>(gemm), x, w, y, cap_rows, N, K, ldy, epilogue,
                     static_cast<cudaStream_t>(stream), static_cast<const DevBatch*>(desc));
}

}  // extern "C"
