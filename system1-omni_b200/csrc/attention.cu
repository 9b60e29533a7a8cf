// Full-attention layers of the Qwen3.5 prefill: q/k preparation and gated GQA
// flash attention (head dim 256).
//
// attn_prep (prep_fast_kernel): one warp per 4 (token, head) units; each lane holds 8
// consecutive dims (one 16-byte load). Per-head zero-centred RMSNorm (one bf16 rounding),
// then partial rotary embedding on the first 2*half dims (rotate_half; each product and
// the sum rounded to bf16 as Transformers does in bf16); the partner of dim d < half
// (dim d + half) sits in lane ^ (half / 8). The gate half of each q row is copied out.
//
// flash attention (flash_tc): tcgen05 MMAs with S, P and O in tensor memory, fed by TMA;
// see the comment above the kernel. One kernel serves every entry point through its
// arguments: packed sequences (a SeqTable), an immutable shared prefix K/V read before
// each sequence's own rows (positions continue after it), a windowed first query row,
// and the bidirectional / prefix-bidirectional masks. Operands must start on 16-byte
// boundaries and a shared prefix must be whole 64-key tiles; other calls are refused
// with cudaErrorInvalidValue before any launch.
#include <climits>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(attention)

namespace s1 {
namespace attn {

constexpr int DH = 256;

// ---------------------------------------------------------------- prep ----
constexpr int PREP_UNITS = 4;  // (token, head) units per warp, loads of all issued first
// Aligned: Hq and Hk multiples of PREP_UNITS, so a warp's units are heads of one token and
// all of q or all of k (one rotary row, no bounds or token checks per unit).
template <bool Aligned>
__global__ void __launch_bounds__(256, 3) prep_fast_kernel(const bf16* __restrict__ qg, const bf16* __restrict__ kr, int ld,
                                 const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                 const bf16* __restrict__ cosb, const bf16* __restrict__ sinb, bf16* __restrict__ q,
                                 bf16* __restrict__ gate, bf16* __restrict__ k, int T, int Hq, int Hk, int half,
                                 float eps, const DevBatch* dyn) {
    grid_dep_wait();
    grid_dep_launch();
    T = dyn_rows(dyn, T);
    const int unit0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * PREP_UNITS;
    const int lane = threadIdx.x & 31;
    const int heads = Hq + Hk;
    const int units = T * heads;
    if (unit0 >= units) return;
    const int d0 = lane * 8;
    const bool rotated = d0 < 2 * half;  // a lane's 8 dims are all rotated or all passed through
    int ti[PREP_UNITS], hi[PREP_UNITS];
    {
        int t = unit0 / heads, hh = unit0 - t * heads;
#pragma unroll
        for (int i = 0; i < PREP_UNITS; i++) {
            ti[i] = t;
            hi[i] = hh;
            if (Aligned) {
                hh++;
            } else if (++hh == heads) {
                hh = 0;
                t++;
            }
        }
    }
    const int n = Aligned ? PREP_UNITS : min(PREP_UNITS, units - unit0);
    Pack8 xr[PREP_UNITS], gr[PREP_UNITS];
#pragma unroll
    for (int i = 0; i < PREP_UNITS; i++) {
        if (Aligned || i < n) {
            const bf16* row = qg + (size_t)ti[i] * ld;
            if (Aligned ? hi[0] < Hq : hi[i] < Hq) {
                const bf16* src = row + hi[i] * 2 * DH;
                xr[i] = ld8(src + d0);
                gr[i] = ld8(src + DH + d0);
            } else {
                xr[i] = ld8(kr + (size_t)ti[i] * ld + (hi[i] - Hq) * DH + d0);
            }
        }
    }
    const int f = d0 & (half - 1);  // half is a power of two (checked on the host)
    Pack8 ca, sa;
    if (rotated) {
        ca = ld8(cosb + (size_t)ti[0] * half + f);
        sa = ld8(sinb + (size_t)ti[0] * half + f);
    }
    const float sgn = d0 < half ? -1.f : 1.f;  // rotate-half: -x2 for the first half, +x1 for the second
    float2 cs[4], sn[4];
    auto rot_rows = [&](const Pack8& c8, const Pack8& s8) {
#pragma unroll
        for (int p = 0; p < 4; p++) {
            cs[p] = __bfloat1622float2(c8.h[p]);
            const float2 sv = __bfloat1622float2(s8.h[p]);
            sn[p] = make_float2(sgn * sv.x, sgn * sv.y);
        }
    };
    if (rotated) rot_rows(ca, sa);
#pragma unroll
    for (int i = 0; i < PREP_UNITS; i++) {
        if (!Aligned && i >= n) break;  // uniform over the warp
        const bool is_q = Aligned ? hi[0] < Hq : hi[i] < Hq;
        float2 x[4];
        float ss = 0.f;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            x[p] = __bfloat1622float2(xr[i].h[p]);
            ss = fmaf(x[p].x, x[p].x, ss);
            ss = fmaf(x[p].y, x[p].y, ss);
        }
        const float inv = rsqrtf(warp_sum(ss) / DH + eps);
        const float2 inv2 = make_float2(inv, inv);
        const Pack8 wv = ld8((is_q ? qw : kw) + d0);  // this unit's norm weight (L1-resident, 512 bytes)
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const float2 w = __bfloat1622float2(wv.h[p]);
            x[p] = rbf2(mul2(mul2(x[p], inv2), make_float2(1.f + w.x, 1.f + w.y)));
        }
        if (!Aligned && rotated && i > 0 && ti[i] != ti[i - 1])  // the warp's second token: its rotary rows
            rot_rows(ld8(cosb + (size_t)ti[i] * half + f), ld8(sinb + (size_t)ti[i] * half + f));
        Pack8 out;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const float2 partner = make_float2(__shfl_xor_sync(0xffffffffu, x[p].x, half / 8),
                                               __shfl_xor_sync(0xffffffffu, x[p].y, half / 8));
            if (rotated) {
                // bf16(x cos) + bf16(rotate_half(x) sin), rounded once more by the pack
                const float2 y = add2(rbf2(mul2(x[p], cs[p])), rbf2(mul2(partner, sn[p])));
                out.h[p] = __floats2bfloat162_rn(y.x, y.y);
            } else {
                out.h[p] = __floats2bfloat162_rn(x[p].x, x[p].y);
            }
        }
        if (is_q) {
            st8(q + ((size_t)ti[i] * Hq + hi[i]) * DH + d0, out);
            st8(gate + ((size_t)ti[i] * Hq + hi[i]) * DH + d0, gr[i]);
        } else {
            st8(k + ((size_t)ti[i] * Hk + hi[i] - Hq) * DH + d0, out);
        }
    }
}

// ---------------------------------------------------------------- flash ----
struct Args {
    const bf16* q;
    const bf16* k;
    const bf16* v;
    int ldv;
    const bf16* gate;
    bf16* out;
    const bf16* pk;   // shared prefix K [P][Hk][DH] (or null)
    const bf16* pv;   // shared prefix V [P][Hk][DH]
    int P;            // prefix length (positions of own rows start at P)
    int q_base;       // first own query row computed (multiple of BM... any value)
    int state;        // prefix-bidirectional boundary (0 = none)
    int Hq, Hk;
    float scale_log2;
    int gated, causal;
};

// ------------------------------------------------------- flash (tcgen05) ----
// A CTA takes 128 queries of one head. Per 128-key tile j:
//   S_j = Q K_j^T   tcgen05.mma M=128 N=128 K=256 into one of two TMEM buffers
//   softmax         4 warps, thread = query row = TMEM lane: masked row max, exp2,
//                   bf16 P_j into tensor memory over S_j (the A operand of PV_j)
//   O += P_j V_j    tcgen05.mma M=128 N=256 K=128 into TMEM (V as an MN-major B operand)
// The MMA thread issues S_{j+1} before PV_j, so the tensor pipe computes the next
// scores while the softmax warps work. O is rescaled only when a row's maximum grows
// by more than 2^8 over the base its probabilities were taken against (the sum l uses
// the same base, so the quotient is unchanged; p <= 2^8 loses nothing in bf16).
// Q, K and V arrive by TMA (128-byte swizzle, one head per box, prefix K/V from their
// own tensor maps); K is released per 64-dim block as soon as its MMAs have completed.
// Warp 0: TMA producer; warp 1: TMEM allocation and MMA issue; warps 2-5: softmax and
// the epilogue (O / l staged through shared memory, gate applied on coalesced rows).
namespace tca {

constexpr int BM = 128, BN = 128, THREADS = 192;
constexpr int SUB = 128 * 128;  // one [128 rows][64 bf16] swizzled tile, 16 KB
constexpr int OFF_Q = 0, OFF_K = 4 * SUB, OFF_V = 8 * SUB, OFF_BAR = 12 * SUB;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t ID_S = tc::idesc(128, BN, tc::AB_BF16);
constexpr uint32_t ID_O = tc::idesc_major(128, DH, tc::AB_BF16, 0, 1);
constexpr float RESCALE_LOG2 = 8.f;

struct Maps {
    CUtensorMap q, k, v, pk, pv;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ int query_blocks(const SeqTable& tab, int i, int q_base) {
    const int rows = tab.offset[i + 1] - tab.offset[i] - q_base;
    return rows > 0 ? (rows + BM - 1) / BM : 0;
}

// P lives in tensor memory. The softmax warps write bf16 P_j over the first 64 columns of
// its own S buffer (two keys per 32-bit column) and PV_j reads its A operand from there, so
// P is double-buffered with S: the softmax of tile j + 1 does not wait for PV_j (only a
// rescale of O does), and S_{j+2} is issued into a buffer once PV_j, its last reader, is
// complete.
// Dyn: the capacity path. The table is the descriptor's in device memory and the grid is
// sized for the capacity; CTAs past the batch's query blocks return at once.
template <bool Dyn>
__global__ void __launch_bounds__(THREADS, 1)
    flash_tc(const __grid_constant__ Maps maps, Args a, const __grid_constant__ SeqTable tab_arg, const DevBatch* dyn) {
    using namespace tc;
    const SeqTable& tab = Dyn ? dyn->tab : tab_arg;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    const uint32_t bars = base + OFF_BAR;
    const uint32_t q_full = bars, k_full = bars + 8, k_empty = bars + 40, v_full = bars + 72, v_empty = bars + 80;
    const uint32_t s_full = bars + 88, s_free = bars + 104, pv_done = bars + 128;
    const uint32_t drain = bars + 136, pv_done1 = bars + 144;
    // PV_i completion: one barrier per S/P buffer (parity (i >> 1) & 1), so that a waiter is
    // never two phases behind (the softmax does not wait for every PV)
    auto pv_bar = [&](int i) { return (i & 1) ? pv_done1 : pv_done; };
    auto pv_par = [&](int i) { return (uint32_t)(i >> 1) & 1u; };
    int* info = reinterpret_cast<int*>(smem + OFF_BAR + 160);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 192);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0 && a.q_base == 0) {
        // blockIdx.y -> (sequence, query block): sequences in the table's order (longest
        // first), the blocks of one sequence last-first (the most key tiles first), by a
        // binary search of the block prefix sums (every access the same for the warp)
        if (lane == 0) {
            const int target = blockIdx.y;
            info[0] = -1;
            if (target < tab.qcum[tab.count]) {
                int lo = 0, hi = tab.count;  // qcum[lo] <= target < qcum[hi]
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (tab.qcum[mid] <= target)
                        lo = mid;
                    else
                        hi = mid;
                }
                info[0] = tab.order[lo];
                info[1] = tab.qcum[lo + 1] - 1 - target;
            }
        }
    } else if (warp == 0) {
        // the same mapping for a first query row q_base > 0 (blocks counted from it)
        const int target = blockIdx.y;
        if (Dyn && lane == 0) info[0] = -1;
        __syncwarp();
        int cnt[8], local = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int pos = lane * 8 + e;
            cnt[e] = pos < tab.count ? query_blocks(tab, tab.order[pos], a.q_base) : 0;
            local += cnt[e];
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int first = incl - local;
        if (target >= first && target < incl) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                if (target >= first && target < first + cnt[e]) {
                    info[0] = tab.order[lane * 8 + e];
                    info[1] = cnt[e] - 1 - (target - first);
                }
                first += cnt[e];
            }
        }
    }
    if constexpr (Dyn) {
        __syncthreads();
        if (info[0] < 0) return;  // past the batch: nothing allocated or armed yet
    }
    if (threadIdx.x == 32) {
        mbar_init(q_full, 1);
        for (int d = 0; d < 4; d++) {
            mbar_init(k_full + 8 * d, 1);
            mbar_init(k_empty + 8 * d, 1);
        }
        mbar_init(v_full, 1);
        mbar_init(v_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(s_full + 8, 1);
        mbar_init(s_free, 4);  // one arrive per softmax warp
        mbar_init(s_free + 8, 4);
        mbar_init(pv_done, 1);
        mbar_init(pv_done1, 1);
        mbar_init(drain, 1);
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
    const int seq = info[0], qb = info[1];
    const int h = blockIdx.x, hk = h / (a.Hq / a.Hk);
    const int off = tab.offset[seq];
    const int len = tab.offset[seq + 1] - off;
    const int q0 = a.q_base + qb * BM;  // first own query row of this block
    const int P = a.P;
    const int total = P + len;          // keys visible to this sequence
    const int qpos0 = P + q0;           // position of the block's first query
    const int kv_end = a.causal ? min(total, qpos0 + BM) : total;
    const int n = (kv_end + BN - 1) / BN;

    if (warp == 0) {
        if (lane == 0) {
            int kc[4] = {0, 0, 0, 0}, vc = 0;
            bool ok = true;
            mbar_expect_tx(q_full, 4 * SUB);
#pragma unroll
            for (int d = 0; d < 4; d++) tma_load_3d(base + OFF_Q + d * SUB, &maps.q, q_full, d * 64, h, off + q0);
            auto load_kv = [&](uint32_t dst, const CUtensorMap* own, const CUtensorMap* pre, uint32_t bar, int d,
                               int j) {
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int key0 = j * BN + hf * 64;  // P is a multiple of 64: a half is all prefix or all own
                    if (key0 < P)
                        tma_load_3d(dst + hf * (SUB / 2), pre, bar, d * 64, hk, key0);
                    else
                        tma_load_3d(dst + hf * (SUB / 2), own, bar, d * 64, hk, off + key0 - P);
                }
            };
            // order of use: K_0, K_1, V_0, K_2, V_1, ... (S_{j+1} is issued before PV_j)
            for (int j = 0; ok && j <= n; j++) {
                if (j < n) {
                    for (int d = 0; d < 4 && ok; d++) {
                        if (j > 0 && !mbar_wait(k_empty + 8 * d, (uint32_t)(j - 1) & 1u)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(k_full + 8 * d, SUB);
                        load_kv(base + OFF_K + d * SUB, &maps.k, &maps.pk, k_full + 8 * d, d, j);
                        kc[d]++;
                    }
                }
                if (ok && j > 0) {
                    const int t = j - 1;
                    if (t > 0 && !mbar_wait(v_empty, (uint32_t)(t - 1) & 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(v_full, 4 * SUB);
#pragma unroll
                    for (int d = 0; d < 4; d++) load_kv(base + OFF_V + d * SUB, &maps.v, &maps.pv, v_full, d, t);
                    vc++;
                }
            }
            if (!ok) atomicOr(&g_fault_word, FAULT_WAIT_PRODUCER);
            // the copies still in flight land before this CTA can leave
            (void)mbar_wait(q_full, 0);
            for (int d = 0; d < 4; d++)
                if (kc[d] > 0) (void)mbar_wait(k_full + 8 * d, (uint32_t)(kc[d] - 1) & 1u);
            if (vc > 0) (void)mbar_wait(v_full, (uint32_t)(vc - 1) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0);
            tc_fence_after();
            auto pv = [&](int i) -> bool {
                // P_i is announced on its buffer's own barrier, so the softmax running a tile
                // ahead cannot complete a second phase before this wait
                const bool p_ok = mbar_wait(s_free + 8 * (i & 1), (uint32_t)(i >> 1) & 1u);
                if (!p_ok || !mbar_wait(v_full, (uint32_t)i & 1u)) return false;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint64_t vd = desc_sw128_mn(base + OFF_V + kk * 2048, SUB, 1024);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    // 16 keys = 8 packed columns of P_i
                    mma_bf16_ts(tmem + 256, tmem + (uint32_t)((i & 1) * BN + kk * 8), vd, ID_O, acc);
                }
                mma_commit(v_empty);
                mma_commit(pv_bar(i));
                return true;
            };
            for (int j = 0; ok && j < n; j++) {
                const int b = j & 1;
                // buffer b is free once PV_{j-2}, the last reader of P_{j-2} in it, has completed
                // (PV_{j-1} is not issued yet, so the parity names PV_{j-2})
                if (j >= 2 && !mbar_wait(pv_bar(j - 2), pv_par(j - 2))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int d = 0; d < 4; d++) {
                    if (!mbar_wait(k_full + 8 * d, (uint32_t)j & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16(tmem + b * BN, desc_sw128(base + OFF_Q + d * SUB + kk * 32),
                                 desc_sw128(base + OFF_K + d * SUB + kk * 32), ID_S, (d | kk) ? 1u : 0u);
                    mma_commit(k_empty + 8 * d);
                }
                if (!ok) break;
                mma_commit(s_full + 8 * b);
                if (j >= 1) ok = pv(j - 1);
            }
            if (ok && n > 0) ok = pv(n - 1);
            if (!ok) atomicOr(&g_fault_word, FAULT_WAIT_MMA);
            mma_commit(drain);
            (void)mbar_wait(drain, 0);
        }
    } else {
        const int wq = warp & 3;  // this warp's quarter of the TMEM lanes
        const int r = wq * 32 + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(wq * 32) << 16);
        const int qpos = qpos0 + r;
        const float sl2 = a.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n; j++) {
            const int b = j & 1;
            // tcgen05.ld/st are warp-collective: every wait outcome is made warp-uniform
            if (!__all_sync(0xffffffffu, mbar_wait(s_full + 8 * b, (uint32_t)(j >> 1) & 1u))) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (j == n - 1 && a.gated) {
                // S_{n-1} is complete, so no MMA reads the K tile any more: fetch this thread's
                // gate units of the output pass into it, behind the last softmax and PV
                const int t = threadIdx.x - 64, chunk = t & 31;
                bf16* gs = reinterpret_cast<bf16*>(smem + OFF_K);
#pragma unroll 8
                for (int i = 0; i < BM / 4; i++) {
                    const int row = (t >> 5) + 4 * i, lrow = min(q0 + row, len - 1);
                    cp_async16_zfill(gs + row * DH + chunk * 8, a.gate + ((size_t)(off + lrow) * a.Hq + h) * DH + chunk * 8,
                                     q0 + row < len);
                }
                cp_async_commit();
            }
            float s[4][32];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld32(lane_addr + b * BN + c * 32, s[c]);
            tmem_ld_wait();
            const int k0 = j * BN;
            bool full = k0 + BN <= total;
            if (a.causal)
                full = full && k0 + BN - 1 <= qpos;
            else if (a.state > 0 && qpos < a.state)
                full = full && k0 + BN <= a.state;
            // row maximum over 8 independent chains (one warp per SMSP: no other warp hides
            // the latency of a 128-long dependent chain)
            float m8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) m8[i] = -INFINITY;
            if (full) {  // three-input max: 16 per chain instead of 32
#pragma unroll
                for (int c = 0; c < 4; c++)
#pragma unroll
                    for (int e = 0; e < 32; e += 16)
#pragma unroll
                        for (int i = 0; i < 8; i++) m8[i] = max3(m8[i], s[c][e + i], s[c][e + 8 + i]);
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++)
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        const int key = k0 + c * 32 + e;
                        bool vis = key < total;
                        if (a.causal)
                            vis = vis && key <= qpos;
                        else if (a.state > 0 && qpos < a.state)
                            vis = vis && key < a.state;
                        s[c][e] = vis ? s[c][e] : -INFINITY;
                        m8[e & 7] = fmaxf(m8[e & 7], s[c][e]);
                    }
            }
            float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            mx *= sl2;
            const bool grow = mx > m + RESCALE_LOG2;
            // PV_{j-1} must be complete before O is rescaled; PV_{j-2} is, since S_j was issued
            // after it
            if (j > 0 && __any_sync(0xffffffffu, grow) &&
                !__all_sync(0xffffffffu, mbar_wait(pv_bar(j - 1), pv_par(j - 1)))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float alpha = grow ? ex2(m - mx) : 1.f;
            l *= alpha;
            if (grow) m = mx;
            // the warp rescales its 32 rows of O together (factor 1 for rows that keep their base)
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
                for (int c = 0; c < DH / 32; c++) {
                    float o[32];
                    tmem_ld32(lane_addr + 256 + c * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] *= alpha;
                    tmem_st32(lane_addr + 256 + c * 32, o);
                }
                tmem_st_wait();
            }
            const float nm = m == -INFINITY ? 0.f : -m;
            float2 l2[4];  // row-sum chains of keys e = 2p, 2p + 1 (mod 8), in f32x2 pairs
#pragma unroll
            for (int i = 0; i < 4; i++) l2[i] = make_float2(0.f, 0.f);
            const float2 sl22 = make_float2(sl2, sl2), nm2 = make_float2(nm, nm);
            uint32_t pk[32];  // 64 keys of P as bf16 pairs (one tcgen05.st of 32 columns)
#pragma unroll
            for (int c = 0; c < 4; c++) {
#pragma unroll
                for (int g8 = 0; g8 < 4; g8++) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; e += 2) {
                        const float2 t = fma2(make_float2(s[c][g8 * 8 + e], s[c][g8 * 8 + e + 1]), sl22, nm2);
                        f[e] = ex2(t.x);
                        f[e + 1] = ex2(t.y);
                        l2[e >> 1] = add2(l2[e >> 1], make_float2(f[e], f[e + 1]));
                    }
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const __nv_bfloat162 h2 = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
                        pk[(c & 1) * 16 + g8 * 4 + e] = *reinterpret_cast<const uint32_t*>(&h2);
                    }
                }
                if (c & 1) tmem_st32(lane_addr + b * BN + (c >> 1) * 32, *reinterpret_cast<const float(*)[32]>(pk));
            }
            l += ((l2[0].x + l2[0].y) + (l2[1].x + l2[1].y)) + ((l2[2].x + l2[2].y) + (l2[3].x + l2[3].y));
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free + 8 * b);
        }
        if (ok && n > 0) ok = mbar_wait(pv_bar(n - 1), pv_par(n - 1));
        tc_fence_after();
        if (bar_any(1, 128, !ok)) {  // uniform over the four warps: the loads below are collective
            if (r == 0) atomicOr(&g_fault_word, FAULT_WAIT_EPILOGUE);
        } else {
            // bf16(O / l) into the Q tile (free: every MMA has completed), row r with its
            // 16-byte chunks rotated by r so that the row-per-thread writes spread over banks
            const float inv = 1.f / l;
            bf16* stage = reinterpret_cast<bf16*>(smem + OFF_Q);
#pragma unroll 1
            for (int c = 0; c < DH / 32; c++) {
                float o[32];
                tmem_ld32(lane_addr + 256 + c * 32, o);
                tmem_ld_wait();
#pragma unroll
                for (int g8 = 0; g8 < 4; g8++) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) f[e] = o[g8 * 8 + e] * inv;
                    const int chunk = c * 4 + g8;
                    st8(stage + r * DH + ((chunk ^ r) & 31) * 8, pack8(f));
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const int t = threadIdx.x - 64, chunk = t & 31;
            const bf16* gs = reinterpret_cast<const bf16*>(smem + OFF_K);
            if (a.gated) cp_async_wait_all();  // this thread's own gate units (fetched at the last tile)
            // groups of 8 rows: the group's shared-memory loads (all unconditional, the staging
            // tile is whole) are written before its stores, since a store through the generic
            // output pointer may alias shared memory as far as the compiler knows and no load
            // written after it could be issued ahead of it; only stores past the end are skipped
            const int rows = min(BM, len - q0);
            constexpr int GR = 8;
#pragma unroll 1
            for (int i0 = 0; i0 < BM / 4; i0 += GR) {
                Pack8 xv[GR], gv[GR];
#pragma unroll
                for (int u = 0; u < GR; u++) {
                    const int row = (t >> 5) + 4 * (i0 + u);
                    xv[u] = ld8(stage + row * DH + ((chunk ^ row) & 31) * 8);
                    if (a.gated) gv[u] = ld8(gs + row * DH + chunk * 8);
                }
#pragma unroll
                for (int u = 0; u < GR; u++) {
                    const int row = (t >> 5) + 4 * (i0 + u);
                    const size_t o_off = ((size_t)(off + q0 + row) * a.Hq + h) * DH + chunk * 8;
                    if (a.gated) {
                        Pack8 y;
#pragma unroll
                        for (int p2 = 0; p2 < 4; p2++) {
                            // out = x * bf16(sigmoid(gate))
                            const float2 sg = rbf2(sigmoid2_fast(__bfloat1622float2(gv[u].h[p2])));
                            const float2 o2 = mul2(__bfloat1622float2(xv[u].h[p2]), sg);
                            y.h[p2] = __floats2bfloat162_rn(o2.x, o2.y);
                        }
                        if (row < rows) st8(a.out + o_off, y);
                    } else if (row < rows) {
                        st8(a.out + o_off, xv[u]);
                    }
                }
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

int launch_tc(const Args& a, const SeqTable& tab, int blocks, const DevBatch* dyn, cudaStream_t st) {
    static const cudaError_t configured =
        cudaFuncSetAttribute(flash_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (configured != cudaSuccess) return configured;
    static const cudaError_t configured_dyn =
        cudaFuncSetAttribute(flash_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (configured_dyn != cudaSuccess) return configured_dyn;
    const int rows = tab.offset[tab.count];
    Maps maps;
    memset(&maps, 0, sizeof(maps));
    int e = host::make_map_3d_bf16(&maps.q, a.q, DH, a.Hq, rows, DH, (uint64_t)a.Hq * DH, 64, BM);
    if (!e) e = host::make_map_3d_bf16(&maps.k, a.k, DH, a.Hk, rows, DH, (uint64_t)a.Hk * DH, 64, 64);
    if (!e) e = host::make_map_3d_bf16(&maps.v, a.v, DH, a.Hk, rows, DH, (uint64_t)a.ldv, 64, 64);
    if (!e && a.P > 0) e = host::make_map_3d_bf16(&maps.pk, a.pk, DH, a.Hk, a.P, DH, (uint64_t)a.Hk * DH, 64, 64);
    if (!e && a.P > 0) e = host::make_map_3d_bf16(&maps.pv, a.pv, DH, a.Hk, a.P, DH, (uint64_t)a.Hk * DH, 64, 64);
    if (e) return e;
    return launch_pdl(dyn ? flash_tc<true> : flash_tc<false>, dim3(a.Hq, blocks), dim3(THREADS), SMEM, st, maps, a,
                      tab, dyn);
}

}  // namespace tca

// `tab` holds the batch, or, on the capacity path (dyn non-null), one sequence of
// cap_rows rows standing for the capacity, with `cap_seqs` sequences at most: the grid
// then covers every batch that fits (sum of ceil(L_i / BM) <= cap_rows / BM + cap_seqs).
int launch(Args a, const SeqTable& tab, cudaStream_t st, const DevBatch* dyn = nullptr, int cap_seqs = 0) {
    if (a.Hq <= 0 || a.Hk <= 0 || a.Hq % a.Hk || a.ldv % 8 || a.ldv < a.Hk * DH) return cudaErrorInvalidValue;
    int max_rows = 0, blocks = 0;
    for (int i = 0; i < tab.count; i++) {
        const int rows = tab.offset[i + 1] - tab.offset[i] - a.q_base;
        max_rows = max(max_rows, rows);
        if (rows > 0) blocks += (rows + tca::BM - 1) / tca::BM;
    }
    if (max_rows <= 0) return cudaSuccess;
    if (dyn) {
        if (a.q_base != 0 || cap_seqs <= 0 || cap_seqs > MAX_SEQS) return cudaErrorInvalidValue;
        blocks = tab.offset[tab.count] / tca::BM + cap_seqs;
    }
    // TMA tiles: every operand starts on a 16-byte boundary and the shared prefix is whole
    // 64-key tiles (the reference's own shared-prefix entry point asks the same of it)
    const bool aligned = aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.out) &&
                         (!a.gated || aligned16(a.gate)) &&
                         (a.P == 0 || (a.P % 64 == 0 && aligned16(a.pk) && aligned16(a.pv)));
    if (!aligned) return cudaErrorInvalidValue;
    return tca::launch_tc(a, tab, blocks, dyn, st);
}

Args make_args(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out, int Hq, int Hk,
               float scale, bool causal) {
    Args a{};
    a.q = static_cast<const bf16*>(q);
    a.k = static_cast<const bf16*>(k);
    a.v = static_cast<const bf16*>(v);
    a.ldv = ldv;
    a.gate = static_cast<const bf16*>(gate);
    a.out = static_cast<bf16*>(out);
    a.Hq = Hq;
    a.Hk = Hk;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.gated = gate != nullptr;
    a.causal = causal;
    return a;
}

int single(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out, int T, int Hq, int Hk,
           int Dh, float scale, int q_base, bool causal, int state, bool need_gate, void* stream) {
    if (Dh != DH || T < 0 || !q || !k || !v || !out) return cudaErrorInvalidValue;
    if (q_base < 0 || q_base > T || (need_gate && !gate && T > 0)) return cudaErrorInvalidValue;
    if (T == q_base) return cudaSuccess;
    SeqTable tab;
    const size_t len = (size_t)T;
    make_table(tab, &len, 1);
    Args a = make_args(q, k, v, ldv, gate, out, Hq, Hk, scale, causal);
    a.q_base = q_base;
    a.state = state;
    return launch(a, tab, static_cast<cudaStream_t>(stream));
}

}  // namespace attn
}  // namespace s1

using namespace s1;

extern "C" {

int cs1_attn_prep(const void* qg, const void* kr, int ld, const void* qw, const void* kw, const void* cos,
                  const void* sin, void* q, void* gate, void* k, int T, int Hq, int Hk, int Dh, int half, float eps,
                  void* stream) {
    if (ld % 8 != 0 || T < 0 || Hq < 1 || Hk < 1) return cudaErrorInvalidValue;
    if (Dh != attn::DH || half <= 0 || half % 8 != 0 || 2 * half > Dh || ((half / 8) & (half / 8 - 1)))
        return cudaErrorInvalidValue;
    const long units = (long)T * (Hq + Hk);
    if (units == 0) return cudaSuccess;
    if (units > INT_MAX - 64) return cudaErrorInvalidValue;
    const long warps = (units + attn::PREP_UNITS - 1) / attn::PREP_UNITS;
    if (!aligned16(qg) || !aligned16(kr) || !aligned16(qw) || !aligned16(kw) || !aligned16(q) || !aligned16(gate) ||
        !aligned16(k))
        return cudaErrorInvalidValue;
    if (!aligned16(cos) || !aligned16(sin)) return cudaErrorInvalidValue;
    constexpr int WPB = 8;
    // (Hq >= Hk >= 1, so Hq + Hk >= 2: the PREP_UNITS = 4 units of a warp fall in at most two tokens)
    const bool aligned = Hq % attn::PREP_UNITS == 0 && Hk % attn::PREP_UNITS == 0;
    return launch_pdl(aligned ? attn::prep_fast_kernel<true> : attn::prep_fast_kernel<false>,
                      dim3((unsigned)((warps + WPB - 1) / WPB)), dim3(WPB * 32), 0,
                      static_cast<cudaStream_t>(stream), static_cast<const bf16*>(qg), static_cast<const bf16*>(kr),
                      ld, static_cast<const bf16*>(qw), static_cast<const bf16*>(kw), static_cast<const bf16*>(cos),
                      static_cast<const bf16*>(sin), static_cast<bf16*>(q), static_cast<bf16*>(gate),
                      static_cast<bf16*>(k), T, Hq, Hk, half, eps, static_cast<const DevBatch*>(nullptr));
}

int cs1_attn_prep_dyn(const void* qg, const void* kr, int ld, const void* qw, const void* kw, const void* cos,
                      const void* sin, void* q, void* gate, void* k, int cap_rows, int Hq, int Hk, int Dh, int half,
                      float eps, const void* desc, void* stream) {
    if (!desc || ld % 8 != 0 || cap_rows < 0 || Hq < 1 || Hk < 1) return cudaErrorInvalidValue;
    if (Dh != attn::DH || half <= 0 || half % 8 != 0 || 2 * half > Dh || ((half / 8) & (half / 8 - 1)))
        return cudaErrorInvalidValue;
    const long units = (long)cap_rows * (Hq + Hk);
    if (units == 0) return cudaSuccess;
    if (units > INT_MAX - 64) return cudaErrorInvalidValue;
    const long warps = (units + attn::PREP_UNITS - 1) / attn::PREP_UNITS;
    if (!aligned16(qg) || !aligned16(kr) || !aligned16(qw) || !aligned16(kw) || !aligned16(q) || !aligned16(gate) ||
        !aligned16(k) || !aligned16(cos) || !aligned16(sin))
        return cudaErrorInvalidValue;
    constexpr int WPB = 8;
    const bool aligned = Hq % attn::PREP_UNITS == 0 && Hk % attn::PREP_UNITS == 0;
    return launch_pdl(aligned ? attn::prep_fast_kernel<true> : attn::prep_fast_kernel<false>,
                      dim3((unsigned)((warps + WPB - 1) / WPB)), dim3(WPB * 32), 0,
                      static_cast<cudaStream_t>(stream), static_cast<const bf16*>(qg), static_cast<const bf16*>(kr),
                      ld, static_cast<const bf16*>(qw), static_cast<const bf16*>(kw), static_cast<const bf16*>(cos),
                      static_cast<const bf16*>(sin), static_cast<bf16*>(q), static_cast<bf16*>(gate),
                      static_cast<bf16*>(k), cap_rows, Hq, Hk, half, eps, static_cast<const DevBatch*>(desc));
}

int cs1_attention(const void* q, const void* k, const void* v, int ldv, void* out, int T, int Hq, int Hk, int Dh,
                  float scale, void* stream) {
    return attn::single(q, k, v, ldv, nullptr, out, T, Hq, Hk, Dh, scale, 0, true, 0, false, stream);
}

int cs1_attention_gated(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out, int T,
                        int Hq, int Hk, int Dh, float scale, void* stream) {
    return attn::single(q, k, v, ldv, gate, out, T, Hq, Hk, Dh, scale, 0, true, 0, true, stream);
}

int cs1_attention_gated_bidirectional(const void* q, const void* k, const void* v, int ldv, const void* gate,
                                      void* out, int T, int Hq, int Hk, int Dh, float scale, void* stream) {
    return attn::single(q, k, v, ldv, gate, out, T, Hq, Hk, Dh, scale, 0, false, 0, true, stream);
}

int cs1_attention_gated_prefix_bidirectional(const void* q, const void* k, const void* v, int ldv, const void* gate,
                                             void* out, int T, int state, int Hq, int Hk, int Dh, float scale,
                                             void* stream) {
    if (state <= 0 || state >= T || !gate) return cudaErrorInvalidValue;
    return attn::single(q, k, v, ldv, gate, out, T, Hq, Hk, Dh, scale, 0, false, state, true, stream);
}

int cs1_attention_gated_prefix(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                               int T, int Hq, int Hk, int Dh, float scale, int q_base, void* stream) {
    if (q_base % 64) return cudaErrorInvalidValue;
    return attn::single(q, k, v, ldv, gate, out, T, Hq, Hk, Dh, scale, q_base, true, 0, true, stream);
}

int cs1_attention_gated_shared(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                               const void* prefix_k, const void* prefix_v, int suffix, int prefix, int Hq, int Hk,
                               int Dh, float scale, void* stream) {
    if (!q || !k || !v || !gate || !out || !prefix_k || !prefix_v || suffix <= 0 || prefix <= 0 || prefix % 64 ||
        prefix > INT_MAX - suffix || Dh != attn::DH)
        return cudaErrorInvalidValue;
    SeqTable tab;
    const size_t len = (size_t)suffix;
    make_table(tab, &len, 1);
    attn::Args a = attn::make_args(q, k, v, ldv, gate, out, Hq, Hk, scale, true);
    a.pk = static_cast<const bf16*>(prefix_k);
    a.pv = static_cast<const bf16*>(prefix_v);
    a.P = prefix;
    return attn::launch(a, tab, static_cast<cudaStream_t>(stream));
}

int cs1_attention_gated_shared_batch(const void* q, const void* k, const void* v, int ldv, const void* gate,
                                     void* out, const void* prefix_k, const void* prefix_v, const size_t* lengths,
                                     size_t count, int prefix, int Hq, int Hk, int Dh, float scale, void* stream) {
    SeqTable tab;
    if (!q || !k || !v || !gate || !out || Dh != attn::DH || prefix < 0 || !make_table(tab, lengths, count))
        return cudaErrorInvalidValue;
    if (prefix > 0 && (!prefix_k || !prefix_v)) return cudaErrorInvalidValue;
    attn::Args a = attn::make_args(q, k, v, ldv, gate, out, Hq, Hk, scale, true);
    a.pk = static_cast<const bf16*>(prefix_k);
    a.pv = static_cast<const bf16*>(prefix_v);
    a.P = prefix;
    return attn::launch(a, tab, static_cast<cudaStream_t>(stream));
}

int cs1_attention_gated_batch(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                              const size_t* lengths, size_t count, int Hq, int Hk, int Dh, float scale,
                              void* stream) {
    return cs1_attention_gated_shared_batch(q, k, v, ldv, gate, out, nullptr, nullptr, lengths, count, 0, Hq, Hk,
                                            Dh, scale, stream);
}

int cs1_attention_dyn(const void* q, const void* k, const void* v, int ldv, const void* gate, void* out,
                      const void* prefix_k, const void* prefix_v, int prefix, int cap_rows, int cap_seqs, int Hq,
                      int Hk, int Dh, float scale, const void* desc, void* stream) {
    if (!desc || !q || !k || !v || !gate || !out || Dh != attn::DH || prefix < 0 || cap_rows <= 0)
        return cudaErrorInvalidValue;
    if (prefix > 0 && (!prefix_k || !prefix_v)) return cudaErrorInvalidValue;
    SeqTable cap;  // launch geometry and tensor-map extents only
    memset(&cap, 0, sizeof(cap));
    cap.count = 1;
    cap.offset[1] = cap_rows;
    attn::Args a = attn::make_args(q, k, v, ldv, gate, out, Hq, Hk, scale, true);
    a.pk = static_cast<const bf16*>(prefix_k);
    a.pv = static_cast<const bf16*>(prefix_v);
    a.P = prefix;
    return attn::launch(a, cap, static_cast<cudaStream_t>(stream), static_cast<const DevBatch*>(desc), cap_seqs);
}

}  // extern "C"
