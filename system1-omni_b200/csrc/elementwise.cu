// Embedding gather, the Gated DeltaNet front end (causal depthwise conv1d + SiLU,
// gates) and the elementwise activations of the Qwen3.5 prefill. All are
// bandwidth-bound: 16-byte accesses, grids sized by rows x packs.
//
// Rounding points follow the reference's elementwise.cu:
//   conv   y = bf16(silu(bf16(sum_j w[c,j] x[t-3+j,c])))    (F.conv1d then F.silu, both bf16)
//   gates  beta = bf16(sigmoid(b)); g = -exp(A_log) softplus(a + dt_bias) (fp32, threshold 20)
//   silu   out = bf16(bf16(silu(gate)) * up)
#include <climits>
#include <type_traits>

#include "common.cuh"
#include "ops_internal.h"
#include "tc.cuh"

S1_FAULT_WORD(elementwise)

namespace s1 {

bool make_table(SeqTable& t, const size_t* lengths, size_t count) {
    if (!lengths || count == 0 || count > (size_t)MAX_SEQS) return false;
    t.count = (int)count;
    t.max_len = 0;
    size_t rows = 0;
    t.offset[0] = 0;
    for (size_t i = 0; i < count; i++) {
        if (lengths[i] == 0 || lengths[i] > (size_t)INT_MAX - rows) return false;
        rows += lengths[i];
        t.offset[i + 1] = (int)rows;
        if ((int)lengths[i] > t.max_len) t.max_len = (int)lengths[i];
    }
    // stable insertion sort by decreasing length (count <= 256)
    for (size_t i = 0; i < count; i++) {
        int j = (int)i;
        while (j > 0 && lengths[t.order[j - 1]] < lengths[i]) {
            t.order[j] = t.order[j - 1];
            j--;
        }
        t.order[j] = (int)i;
    }
    t.qcum[0] = 0;
    for (size_t i = 0; i < count; i++) t.qcum[i + 1] = t.qcum[i] + (int)((lengths[t.order[i]] + 127) / 128);
    return true;
}

namespace {

constexpr int THREADS = 256;

__global__ void embed_kernel(const int32_t* __restrict__ ids, const Pack8* __restrict__ table,
                             Pack8* __restrict__ out, int packs, int T, const DevBatch* dyn) {
    grid_dep_wait();
    grid_dep_launch();
    T = dyn_rows(dyn, T);
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
        const size_t id = (size_t)ids[t];
        for (int i = threadIdx.x; i < packs; i += blockDim.x) out[(size_t)t * packs + i] = table[id * packs + i];
    }
}

// Channels per thread over a run of `run` consecutive rows: the weights are loaded once and
// the three previous input rows slide through registers, so every input row is read once
// (plus three rows of window per run). A run that crosses into a new sequence restarts its
// window from zeros (or from the three rows of `history`, shared by every sequence). The
// split into runs does not change any output bit.

// NP channel pairs per thread: 4 (16-byte accesses) or 2 (8-byte accesses, about half the
// registers, so more warps per SM keep loads in flight).
template <int NP>
struct alignas(4 * NP) PackN {
    __nv_bfloat162 h[NP];
};

// The GDN front end (Front): besides q, k and v, the inverse L2 norm of every (row, head)
// of q and k, rsqrt(sum y^2 + 1e-6) over the bf16 outputs y of the head (the norm the GDN
// prefill applies in fp32, here reduced across the head's lanes), and, in one extra CTA
// column per run of rows, the gates of those rows: beta = bf16(sigmoid(b)) and
// g = -exp(A_log) softplus(a + dt_bias) (the arithmetic of cs1_gdn_gates).
struct FrontArgs {
    float* rnq;  // [T, HK] inverse norms of q
    float* rnk;  // [T, HK] inverse norms of k
    const bf16* b;
    const bf16* a;  // gate inputs, rows of ld (the conv input's row stride)
    const bf16* A_log;
    const bf16* dt_bias;
    bf16* beta;  // [T, H]
    float* g;    // [T, H]
    int H;
};

// Gates of items [i0, i1) of rows t_begin.. (item i = row t_begin + i / H, head i % H), out
// of line so that its registers do not count against the conv's.
__device__ __noinline__ void front_gates(const FrontArgs& fr, int ld, int t_begin, int i0, int i1) {
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const int t = t_begin + i / fr.H, h = i % fr.H;
        const size_t src = (size_t)t * ld + h;
        fr.beta[(size_t)t * fr.H + h] = to_bf16(sigmoid(f32(fr.b[src])));
        const float x = f32(fr.a[src]) + f32(fr.dt_bias[h]);
        const float sp = x > 20.f ? x : log1pf(expf(x));
        fr.g[(size_t)t * fr.H + h] = -expf(f32(fr.A_log[h])) * sp;
    }
}

// The conv kernel takes 4 channels per thread (one 8-byte pack); a CTA of 128 threads covers
// 128 packs of a run of rows. Each CTA's slice of a row (contiguous) is copied into a ring of
// CB_STAGES batches of 8 rows by bulk copies, so up to 32 KB per CTA are in flight without
// holding registers; the threads read their packs from shared memory. The warps do not wait
// for one another: each counts itself out of a batch's stage when it is done with it, and the
// last of the four issues the copies of the batch CB_STAGES ahead into that stage.
constexpr int CB_STAGES = 4;
constexpr int CB_WARPS = 4;
constexpr int CB_ROW = 128 * 8;               // bytes of a row slice (128 threads x 8 bytes)
constexpr int CB_STAGE = 8 * CB_ROW;          // 8 rows
// ring | full barriers | per-stage warp counts | batches issued | abort flag
constexpr int CB_BAR = CB_STAGES * CB_STAGE;
constexpr int CB_CNT = CB_BAR + 8 * CB_STAGES;
constexpr int CB_SMEM = CB_CNT + 4 * CB_STAGES + 8;

template <bool Dyn, bool Front>
__global__ void __launch_bounds__(128, 6) conv_vec_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ history, int ld_,
                                const bf16* __restrict__ w, bf16* __restrict__ q, bf16* __restrict__ k,
                                bf16* __restrict__ v, int key_packs, int value_packs, int run,
                                const __grid_constant__ SeqTable tab_arg, const DevBatch* dyn,
                                const __grid_constant__ FrontArgs fr) {
    constexpr int NP = 2;  // channel pairs per thread
    using P = PackN<NP>;
    const SeqTable& tab = Dyn ? dyn->tab : tab_arg;  // the capacity path's table is in device memory
    constexpr int CH = 2 * NP;  // channels per thread
    grid_dep_wait();
    grid_dep_launch();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;  // pack of CH channels
    const int packs = 2 * key_packs + value_packs;
    // lanes past the last pack stay for the ring's counts and barriers
    const bool active = c < packs;
    // Front: a q or k pack (warp-uniform: a head's packs are whole warps), whose rows' sums
    // of squares are taken
    const bool qk = Front && c < 2 * key_packs;
    // channel pairs (2p, 2p + 1) in f32x2 lanes: wt[p][j] = tap j of both channels
    float2 wt[NP][4];
#pragma unroll
    for (int i = 0; i < NP; i++) {
        float f[8];
        if (active) unpack8(ld8(w + (size_t)c * CH * 4 + i * 8), f);  // channels 2i, 2i + 1, four taps each
#pragma unroll
        for (int j = 0; j < 4; j++) wt[i][j] = active ? make_float2(f[j], f[4 + j]) : make_float2(0.f, 0.f);
    }
    bf16* dst;
    int dst_ld;
    if (!active) {
        dst = nullptr;
        dst_ld = 0;
    } else if (c < key_packs) {
        dst = q + (size_t)c * CH;
        dst_ld = key_packs * CH;
    } else if (c < 2 * key_packs) {
        dst = k + (size_t)(c - key_packs) * CH;
        dst_ld = key_packs * CH;
    } else {
        dst = v + (size_t)(c - 2 * key_packs) * CH;
        dst_ld = value_packs * CH;
    }
    const int T = tab.offset[tab.count];
    const int t_begin = blockIdx.y * run;
    const int t_end = min(T, t_begin + run);
    if (t_begin >= T) return;
    int s = seq_of(tab, t_begin);
    int next = tab.offset[s + 1];
    const bf16* col = qkv + (size_t)c * CH;
    auto ld = [&](const bf16* p) { return *reinterpret_cast<const P*>(p); };
    float2 x1[NP], x2[NP], x3[NP];  // rows t-3, t-2, t-1
    auto unpack = [](const P& p, float2 (&o)[NP]) {
#pragma unroll
        for (int i = 0; i < NP; i++) o[i] = __bfloat1622float2(p.h[i]);
    };
    auto window = [&](int t) {
        // load the three rows before t inside its sequence (history or zeros before the start)
        const int pos = t - tab.offset[s];
#pragma unroll
        for (int back = 3; back >= 1; back--) {
            float2(&dw)[NP] = back == 3 ? x1 : back == 2 ? x2 : x3;
            if (pos >= back) {
                unpack(ld(col + (size_t)(t - back) * ld_), dw);
            } else if (history) {
                unpack(ld(history + (size_t)(3 - back + pos) * ld_ + (size_t)c * CH), dw);
            } else {
#pragma unroll
                for (int i = 0; i < NP; i++) dw[i] = make_float2(0.f, 0.f);
            }
        }
    };
    // the ring, its barriers and counts
    extern __shared__ __align__(128) uint8_t cbuf[];
    const int batches = (t_end - t_begin + 7) / 8;
    const uint32_t ring = tc::smem_u32(cbuf), bars = ring + CB_BAR;
    int* cnt = reinterpret_cast<int*>(cbuf + CB_CNT);
    volatile int* issued = reinterpret_cast<volatile int*>(cbuf + CB_CNT + 4 * CB_STAGES);
    volatile int* abort_flag = issued + 1;
    const int slice = min(128, packs - (int)blockIdx.x * 128) * (int)sizeof(P);
    const int lane = threadIdx.x & 31;
    auto issue = [&](int b) {
        const int st = b % CB_STAGES, r0 = t_begin + 8 * b, nr = min(8, t_end - r0);
        const uint32_t bar = bars + 8u * st;
        tc::mbar_expect_tx(bar, (uint32_t)(nr * slice));
        const bf16* src = qkv + (size_t)blockIdx.x * 128 * CH + (size_t)r0 * ld_;
        for (int i = 0; i < nr; i++)
            tc::bulk_load(ring + st * CB_STAGE + i * CB_ROW, src + (size_t)i * ld_, (uint32_t)slice, bar);
        *issued = b + 1;
    };
    {
        if (threadIdx.x == 0) {
            for (int i = 0; i < CB_STAGES; i++) {
                tc::mbar_init(bars + 8u * i, 1);
                cnt[i] = 0;
            }
            *issued = 0;
            *abort_flag = 0;
            tc::mbar_fence_init();
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int b = 0; b < min(CB_STAGES, batches); b++) issue(b);
    }
    if (active) window(t_begin);
    // rows in batches of 8 (one stage of the ring each)
    for (int bi = 0; bi < batches; bi++) {
        const int tb = t_begin + 8 * bi;
        {
            const int st = bi % CB_STAGES;
            const bool waited = tc::mbar_wait(bars + 8u * st, (uint32_t)(bi / CB_STAGES) & 1u);
            // warp-uniform decisions: a wait that gave up here, or another warp's
            const bool timeout = __any_sync(0xffffffffu, !waited);
            if (timeout || __any_sync(0xffffffffu, *abort_flag != 0)) {
                if (timeout && lane == 0) {
                    atomicOr(&g_fault_word, tc::FAULT_WAIT_OTHER);
                    *abort_flag = 1;
                }
                break;
            }
        }
        // this warp is done with the batch's stage: the last warp out refills it
        auto release = [&]() {
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                const int st = bi % CB_STAGES;
                if (atomicAdd(&cnt[st], 1) == CB_WARPS - 1) {
                    cnt[st] = 0;
                    if (bi + CB_STAGES < batches) {
                        tc::fence_async_smem();
                        issue(bi + CB_STAGES);
                    }
                }
            }
        };
        if (active) {
        float ss8[8];  // Front: this thread's part of each row's sum of squares
#pragma unroll
        for (int i = 0; i < 8; i++) ss8[i] = 0.f;
        // one row: the conv over the window and row i of the batch, its store, the row's
        // part of the sum of squares, the window moved on by one row
        auto row = [&](int i, auto with_ss) {
            const int t = tb + i;
            float2 x0[NP];  // row i of the batch's stage, read where it is used
            unpack(*reinterpret_cast<const P*>(cbuf + (bi % CB_STAGES) * CB_STAGE + i * CB_ROW +
                                               threadIdx.x * sizeof(P)), x0);
            P out;
#pragma unroll
            for (int p = 0; p < NP; p++) {
                // the reference's tap order: w0 x[t-3] + w1 x[t-2] + w2 x[t-1] + w3 x[t], fp32
                float2 acc = mul2(wt[p][0], x1[p]);
                acc = fma2(wt[p][1], x2[p], acc);
                acc = fma2(wt[p][2], x3[p], acc);
                acc = fma2(wt[p][3], x0[p], acc);
                const float2 y = silu2_fast(rbf2(acc));
                out.h[p] = __floats2bfloat162_rn(y.x, y.y);
            }
            *reinterpret_cast<P*>(dst + (size_t)t * dst_ld) = out;
            if constexpr (decltype(with_ss)::value) {
                float2 sq = make_float2(0.f, 0.f);
#pragma unroll
                for (int p = 0; p < NP; p++) {
                    const float2 yy = __bfloat1622float2(out.h[p]);
                    sq = fma2(yy, yy, sq);
                }
                ss8[i] = sq.x + sq.y;
            }
#pragma unroll
            for (int p = 0; p < NP; p++) {
                x1[p] = x2[p];
                x2[p] = x3[p];
                x3[p] = x0[p];
            }
        };
        using SS = std::integral_constant<bool, Front>;
        using NoSS = std::false_type;
        if (tb + 8 <= t_end && next >= tb + 8) {
            // the common batch: eight rows of one sequence, straight-line code (the window
            // lives in renamed registers, no moves); sums of squares for q and k only
            if (qk) {
#pragma unroll
                for (int i = 0; i < 8; i++) row(i, SS{});
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) row(i, NoSS{});
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int t = tb + i;
                if (t >= t_end) break;
                if (t == next) {
                    s++;
                    next = tab.offset[s + 1];
                    window(t);
                }
                if (qk)
                    row(i, SS{});
                else
                    row(i, NoSS{});
            }
        }
        if constexpr (Front) {
            // q and k packs: a head is LANES = 128 / CH consecutive lanes of one warp (heads start
            // on pack multiples of LANES), so the branch and the shuffles are warp-uniform. The
            // eight rows' sums are reduced together: three exchange steps halve the values a lane
            // holds (lane bit LANES/2 -> rows +4, LANES/4 -> +2, LANES/8 -> +1), then plain steps
            // finish each sum; lanes whose bits below LANES/8 are 0 hold one row's total.
            constexpr int LANES = 128 / CH;
            if (qk) {
                const int lane = threadIdx.x & 31;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const bool hi = lane & (LANES / 2);
                    const float send = hi ? ss8[k] : ss8[k + 4], keep = hi ? ss8[k + 4] : ss8[k];
                    ss8[k] = keep + __shfl_xor_sync(0xffffffffu, send, LANES / 2);
                }
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const bool hi = lane & (LANES / 4);
                    const float send = hi ? ss8[k] : ss8[k + 2], keep = hi ? ss8[k + 2] : ss8[k];
                    ss8[k] = keep + __shfl_xor_sync(0xffffffffu, send, LANES / 4);
                }
                {
                    const bool hi = lane & (LANES / 8);
                    const float send = hi ? ss8[0] : ss8[1], keep = hi ? ss8[1] : ss8[0];
                    ss8[0] = keep + __shfl_xor_sync(0xffffffffu, send, LANES / 8);
                }
#pragma unroll
                for (int o = LANES / 16; o > 0; o >>= 1) ss8[0] += __shfl_xor_sync(0xffffffffu, ss8[0], o);
                const int row = ((lane & (LANES / 2)) ? 4 : 0) + ((lane & (LANES / 4)) ? 2 : 0) +
                                ((lane & (LANES / 8)) ? 1 : 0);
                const int t = tb + row;
                if ((lane & (LANES / 8 - 1)) == 0 && t < t_end) {
                    const int HK = key_packs / LANES, head = c / LANES;
                    float* dn = head < HK ? fr.rnq : fr.rnk;
                    dn[(size_t)t * HK + (head < HK ? head : head - HK)] = rsqrtf(ss8[0] + 1e-6f);
                }
            }
        }
        }
        release();
    }
    {
        // after a wait gave up: the copies still in flight (the last CB_STAGES issued) land
        // before the CTA's shared memory is released
        __syncthreads();
        if (threadIdx.x == 0 && *abort_flag) {
            const int n = *issued;
            for (int b = max(0, n - CB_STAGES); b < n; b++)
                (void)tc::mbar_wait(bars + 8u * (b % CB_STAGES), (uint32_t)(b / CB_STAGES) & 1u);
        }
        if constexpr (Front) {
            // the gates of this run's rows, shared out over the CTAs of v packs (which have no
            // norms to take), or over every CTA when there are none
            const int groups = (packs + 127) / 128, first_v = min(groups, (2 * key_packs + 127) / 128);
            const int g0 = first_v < groups ? first_v : 0, ng = groups - g0;
            if ((int)blockIdx.x >= g0) {
                const int items = (t_end - t_begin) * fr.H, per = (items + ng - 1) / ng;
                const int i0 = ((int)blockIdx.x - g0) * per;
                front_gates(fr, ld_, t_begin, i0, min(items, i0 + per));
            }
        }
    }
}

__global__ void conv_scalar_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ history, int ld,
                                   const bf16* __restrict__ w, bf16* __restrict__ q, bf16* __restrict__ k,
                                   bf16* __restrict__ v, int key_dim, int value_dim, SeqTable tab) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int channels = 2 * key_dim + value_dim;
    if (c >= channels) return;
    const int T = tab.offset[tab.count];
    for (int t = blockIdx.y; t < T; t += gridDim.y) {
        const int s = seq_of(tab, t);
        const int pos = t - tab.offset[s];
        float acc = 0.f;
        for (int j = 0; j < 4; j++) {
            const int back = 3 - j;
            float x = 0.f;
            if (pos >= back)
                x = f32(qkv[(size_t)(t - back) * ld + c]);
            else if (history)
                x = f32(history[(size_t)(3 - back + pos) * ld + c]);
            acc = fmaf(f32(w[c * 4 + j]), x, acc);
        }
        const bf16 y = to_bf16(silu_hw(rbf(acc)));
        if (c < key_dim)
            q[(size_t)t * key_dim + c] = y;
        else if (c < 2 * key_dim)
            k[(size_t)t * key_dim + c - key_dim] = y;
        else
            v[(size_t)t * value_dim + c - 2 * key_dim] = y;
    }
}

__global__ void gates_kernel(const bf16* __restrict__ b, const bf16* __restrict__ a, int ld,
                             const bf16* __restrict__ A_log, const bf16* __restrict__ dt_bias,
                             bf16* __restrict__ beta, float* __restrict__ g, long n, int H, const DevBatch* dyn) {
    grid_dep_wait();
    grid_dep_launch();
    if (dyn) n = min(n, (long)dyn->rows * H);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const int h = (int)(i % H);
        const size_t src = (size_t)(i / H) * ld + h;
        beta[i] = to_bf16(sigmoid(f32(b[src])));
        const float x = f32(a[src]) + f32(dt_bias[h]);
        const float sp = x > 20.f ? x : log1pf(expf(x));
        g[i] = -expf(f32(A_log[h])) * sp;
    }
}

__global__ void sigmoid_gate_kernel(bf16* __restrict__ x, const bf16* __restrict__ gate, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = to_bf16(f32(x[i]) * rbf(sigmoid(f32(gate[i]))));
}

// Grid (column packs / blockDim.x, row pairs): a thread takes one 8-column pack of two
// rows, with the four loads in flight together.
__global__ void silu_mul_vec_kernel(const bf16* __restrict__ gu, int ld, bf16* __restrict__ out, int I, long T) {
    const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (j >= I) return;
    for (long t0 = 2 * (long)blockIdx.y; t0 < T; t0 += 2 * (long)gridDim.y) {
        Pack8 gp[2], up[2];
#pragma unroll
        for (int r = 0; r < 2; r++)
            if (t0 + r < T) {
                gp[r] = ld8(gu + (t0 + r) * ld + j);
                up[r] = ld8(gu + (t0 + r) * ld + I + j);
            }
#pragma unroll
        for (int r = 0; r < 2; r++)
            if (t0 + r < T) {
                Pack8 o;
#pragma unroll
                for (int p = 0; p < 4; p++) {  // bf16(bf16(silu(g)) * u), in f32x2 pairs
                    const float2 y = mul2(rbf2(silu2_fast(__bfloat1622float2(gp[r].h[p]))),
                                          __bfloat1622float2(up[r].h[p]));
                    o.h[p] = __floats2bfloat162_rn(y.x, y.y);
                }
                st8(out + (t0 + r) * I + j, o);
            }
    }
}

__global__ void silu_mul_scalar_kernel(const bf16* __restrict__ gu, int ld, bf16* __restrict__ out, int I, long T) {
    const long n = T * I;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long t = i / I;
        const int j = (int)(i % I);
        out[i] = to_bf16(rbf(silu_hw(f32(gu[t * ld + j]))) * f32(gu[t * ld + I + j]));
    }
}

__global__ void finite_kernel(const uint16_t* __restrict__ x, size_t n, uint32_t* flag) {
    bool bad = false;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        bad |= (x[i] & 0x7f80u) == 0x7f80u;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicExch(flag, 1u);
}

unsigned grid_for(size_t n) {
    const size_t b = (n + THREADS - 1) / THREADS;
    return (unsigned)(b < 148 * 32 ? (b ? b : 1) : 148 * 32);
}

// `tab` holds the batch, or, on the capacity path (dyn non-null), only its capacity
// (offset[count] = cap_rows) while the kernels read the batch from the descriptor.
int conv_launch(const void* qkv, const void* history, int ld, const void* w, void* q, void* k, void* v,
                const SeqTable& tab, int key_dim, int value_dim, const DevBatch* dyn, cudaStream_t st,
                const FrontArgs* front = nullptr) {
    const int T = tab.offset[tab.count];
    const int rows = T < 65535 ? T : 65535;
    const bool vec = key_dim % 8 == 0 && value_dim % 8 == 0 && ld % 8 == 0 && aligned16(qkv) && aligned16(w) &&
                     aligned16(q) && aligned16(k) && aligned16(v) && (!history || aligned16(history));
    if (vec) {
        // 4 channels per thread (one 8-byte pack): with key and value widths multiples of 8,
        // every CTA's row slice (up to 128 packs) is a multiple of 16 bytes, as the ring's
        // bulk copies need
        const int tpacks = (2 * key_dim + value_dim) / 4;
        const long groups = (tpacks + 127) / 128;
        // Runs of 64 rows, shortened (to 32, then 16) while the grid is below two waves of
        // resident CTAs (6 per SM): a short prompt's CTAs each wait on a few batches in series,
        // so more and shorter runs finish sooner.
        const long waves2 = 2L * sm_count() * 6;
        int run = 64;
        while (run > 16 && groups * ((T + run - 1) / run) < waves2 && (T + run / 2 - 1) / (run / 2) <= 65535)
            run /= 2;
        if ((T + run - 1) / run > 65535) return cudaErrorInvalidValue;
        FrontArgs fr{};
        if (front) fr = *front;
        void (*kernel)(const bf16*, const bf16*, int, const bf16*, bf16*, bf16*, bf16*, int, int, int, SeqTable,
                       const DevBatch*, FrontArgs);
        if (front)
            kernel = dyn ? conv_vec_kernel<true, true> : conv_vec_kernel<false, true>;
        else
            kernel = dyn ? conv_vec_kernel<true, false> : conv_vec_kernel<false, false>;
        return launch_pdl(kernel, dim3((unsigned)groups, (T + run - 1) / run), dim3(128), (size_t)CB_SMEM, st,
                          static_cast<const bf16*>(qkv), static_cast<const bf16*>(history), ld,
                          static_cast<const bf16*>(w), static_cast<bf16*>(q), static_cast<bf16*>(k),
                          static_cast<bf16*>(v), key_dim / 4, value_dim / 4, run, tab, dyn, fr);
    } else {
        // the capacity path and the front end need the vector kernel
        if (dyn || front) return cudaErrorInvalidValue;
        const int ch = 2 * key_dim + value_dim;
        conv_scalar_kernel<<<dim3((ch + 127) / 128, rows), 128, 0, st>>>(
            static_cast<const bf16*>(qkv), static_cast<const bf16*>(history), ld, static_cast<const bf16*>(w),
            static_cast<bf16*>(q), static_cast<bf16*>(k), static_cast<bf16*>(v), key_dim, value_dim, tab);
    }
    return cudaGetLastError();
}

}  // namespace
}  // namespace s1

using namespace s1;

extern "C" int cs1_embed(const int32_t* ids, const void* table, void* out, int T, int D, void* stream) {
    if (D <= 0 || D % 8 != 0 || T < 0) return cudaErrorInvalidValue;
    if (T == 0) return cudaSuccess;
    if (!aligned16(table) || !aligned16(out)) return cudaErrorInvalidValue;
    const int grid = T < 65535 ? T : 65535;
    return launch_pdl(embed_kernel, dim3(grid), dim3(128), 0, static_cast<cudaStream_t>(stream), ids,
                      static_cast<const Pack8*>(table), static_cast<Pack8*>(out), D / 8, T,
                      static_cast<const DevBatch*>(nullptr));
}

extern "C" int cs1_gdn_conv(const void* qkv, int ld, const void* w, void* q, void* k, void* v, int T, int key_dim,
                            int value_dim, void* stream) {
    if (T < 0 || key_dim < 0 || value_dim < 0 || ld < 2 * key_dim + value_dim) return cudaErrorInvalidValue;
    if (T == 0 || 2 * key_dim + value_dim == 0) return cudaSuccess;
    SeqTable tab;
    const size_t len = (size_t)T;
    make_table(tab, &len, 1);
    return conv_launch(qkv, nullptr, ld, w, q, k, v, tab, key_dim, value_dim, nullptr,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cs1_gdn_conv_vector(const void* qkv, int ld, const void* w, void* q, void* k, void* v, int T,
                                   int key_dim, int value_dim, void* stream) {
    return cs1_gdn_conv(qkv, ld, w, q, k, v, T, key_dim, value_dim, stream);
}

extern "C" int cs1_gdn_conv_prefix(const void* qkv, const void* history, int ld, const void* w, void* q, void* k,
                                   void* v, int T, int key_dim, int value_dim, void* stream) {
    if (!qkv || !history || !w || !q || !k || !v || T <= 0 || key_dim <= 0 || value_dim <= 0 ||
        ld < 2 * key_dim + value_dim)
        return cudaErrorInvalidValue;
    SeqTable tab;
    const size_t len = (size_t)T;
    make_table(tab, &len, 1);
    return conv_launch(qkv, history, ld, w, q, k, v, tab, key_dim, value_dim, nullptr,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cs1_gdn_conv_batch(const void* qkv, const void* history, int ld, const void* w, void* q, void* k,
                                  void* v, const size_t* lengths, size_t count, int key_dim, int value_dim,
                                  void* stream) {
    SeqTable tab;
    if (!qkv || !w || !q || !k || !v || key_dim <= 0 || value_dim <= 0 || ld < 2 * key_dim + value_dim ||
        !make_table(tab, lengths, count))
        return cudaErrorInvalidValue;
    return conv_launch(qkv, history, ld, w, q, k, v, tab, key_dim, value_dim, nullptr,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cs1_gdn_gates(const void* b, const void* a, int ld, const void* A_log, const void* dt_bias,
                             void* beta, float* g, int T, int H, void* stream) {
    if (T < 0 || H < 0 || ld < H) return cudaErrorInvalidValue;
    const long n = (long)T * H;
    if (n == 0) return cudaSuccess;
    return launch_pdl(gates_kernel, dim3(grid_for(n)), dim3(THREADS), 0, static_cast<cudaStream_t>(stream),
                      static_cast<const bf16*>(b), static_cast<const bf16*>(a), ld, static_cast<const bf16*>(A_log),
                      static_cast<const bf16*>(dt_bias), static_cast<bf16*>(beta), g, n, H,
                      static_cast<const DevBatch*>(nullptr));
}

namespace s1 {
namespace {
int front_args(FrontArgs& fr, float* rnorm_q, float* rnorm_k, const void* b, const void* a, const void* A_log,
               const void* dt_bias, void* beta, float* g, int H) {
    if (!rnorm_q || !rnorm_k || !b || !a || !A_log || !dt_bias || !beta || !g || H <= 0) return cudaErrorInvalidValue;
    fr.rnq = rnorm_q;
    fr.rnk = rnorm_k;
    fr.b = static_cast<const bf16*>(b);
    fr.a = static_cast<const bf16*>(a);
    fr.A_log = static_cast<const bf16*>(A_log);
    fr.dt_bias = static_cast<const bf16*>(dt_bias);
    fr.beta = static_cast<bf16*>(beta);
    fr.g = g;
    fr.H = H;
    return cudaSuccess;
}
}  // namespace
}  // namespace s1

extern "C" int cs1_gdn_front_batch(const void* qkv, const void* history, int ld, const void* w, void* q, void* k,
                                   void* v, float* rnorm_q, float* rnorm_k, const void* b, const void* a,
                                   const void* A_log, const void* dt_bias, void* beta, float* g, int H,
                                   const size_t* lengths, size_t count, int key_dim, int value_dim, void* stream) {
    SeqTable tab;
    FrontArgs fr{};
    if (!qkv || !w || !q || !k || !v || key_dim <= 0 || key_dim % 128 || value_dim <= 0 ||
        ld < 2 * key_dim + value_dim || ld < H || !make_table(tab, lengths, count) ||
        front_args(fr, rnorm_q, rnorm_k, b, a, A_log, dt_bias, beta, g, H) != cudaSuccess)
        return cudaErrorInvalidValue;
    return conv_launch(qkv, history, ld, w, q, k, v, tab, key_dim, value_dim, nullptr,
                       static_cast<cudaStream_t>(stream), &fr);
}

// ---- capacity path ----

extern "C" int cs1_gdn_front_dyn(const void* qkv, const void* history, int ld, const void* w, void* q, void* k,
                                 void* v, float* rnorm_q, float* rnorm_k, const void* b, const void* a,
                                 const void* A_log, const void* dt_bias, void* beta, float* g, int H, int cap_rows,
                                 int cap_seqs, int key_dim, int value_dim, const void* desc, void* stream) {
    FrontArgs fr{};
    if (!desc || !qkv || !w || !q || !k || !v || key_dim <= 0 || key_dim % 128 || value_dim <= 0 ||
        ld < 2 * key_dim + value_dim || ld < H || cap_rows <= 0 || cap_seqs <= 0 || cap_seqs > MAX_SEQS ||
        front_args(fr, rnorm_q, rnorm_k, b, a, A_log, dt_bias, beta, g, H) != cudaSuccess)
        return cudaErrorInvalidValue;
    SeqTable cap;  // launch geometry only
    memset(&cap, 0, sizeof(cap));
    cap.count = 1;
    cap.offset[1] = cap_rows;
    return conv_launch(qkv, history, ld, w, q, k, v, cap, key_dim, value_dim, static_cast<const DevBatch*>(desc),
                       static_cast<cudaStream_t>(stream), &fr);
}

namespace s1 {
namespace {
// Zero `width` bytes (a multiple of 16) of rows [rows, min(rows + margin, cap_rows)) of a
// strided matrix, rows from the descriptor.
__global__ void clear_tail_kernel(uint8_t* __restrict__ x, size_t ld, size_t width, int cap_rows, int margin,
                                  const DevBatch* __restrict__ dyn) {
    grid_dep_wait();
    grid_dep_launch();
    const int r0 = dyn->rows, r1 = min(r0 + margin, cap_rows);
    const size_t packs = width / 16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)(r1 - r0) * packs;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = (size_t)r0 + i / packs, p = i % packs;
        *reinterpret_cast<uint4*>(x + r * ld + p * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
}
}  // namespace
}  // namespace s1

extern "C" int cs1_clear_tail_dyn(void* x, size_t ld_bytes, size_t width_bytes, int cap_rows, int margin,
                                  const void* desc, void* stream) {
    if (!desc || !x || cap_rows < 0 || margin < 0 || width_bytes % 16 || ld_bytes % 16 || width_bytes > ld_bytes ||
        !aligned16(x))
        return cudaErrorInvalidValue;
    if (cap_rows == 0 || margin == 0 || width_bytes == 0) return cudaSuccess;
    const size_t n = (size_t)margin * (width_bytes / 16);
    return launch_pdl(clear_tail_kernel, dim3(grid_for(n)), dim3(THREADS), 0, static_cast<cudaStream_t>(stream),
                      static_cast<uint8_t*>(x), ld_bytes, width_bytes, cap_rows, margin,
                      static_cast<const DevBatch*>(desc));
}

extern "C" size_t cs1_batch_desc_bytes(void) { return sizeof(DevBatch); }

extern "C" int cs1_batch_desc_pack(const size_t* lengths, size_t count, void* out, size_t bytes) {
    if (!out || bytes < sizeof(DevBatch)) return cudaErrorInvalidValue;
    DevBatch d;
    memset(&d, 0, sizeof(d));
    if (!make_table(d.tab, lengths, count)) return cudaErrorInvalidValue;
    d.rows = d.tab.offset[d.tab.count];
    memcpy(out, &d, sizeof(d));
    return cudaSuccess;
}

extern "C" int cs1_embed_dyn(const int32_t* ids, const void* table, void* out, int cap_rows, int D, const void* desc,
                             void* stream) {
    if (!desc || D <= 0 || D % 8 != 0 || cap_rows < 0) return cudaErrorInvalidValue;
    if (cap_rows == 0) return cudaSuccess;
    if (!aligned16(table) || !aligned16(out)) return cudaErrorInvalidValue;
    const int grid = cap_rows < 65535 ? cap_rows : 65535;
    return launch_pdl(embed_kernel, dim3(grid), dim3(128), 0, static_cast<cudaStream_t>(stream), ids,
                      static_cast<const Pack8*>(table), static_cast<Pack8*>(out), D / 8, cap_rows,
                      static_cast<const DevBatch*>(desc));
}

extern "C" int cs1_gdn_conv_dyn(const void* qkv, const void* history, int ld, const void* w, void* q, void* k,
                                void* v, int cap_rows, int cap_seqs, int key_dim, int value_dim, const void* desc,
                                void* stream) {
    if (!desc || !qkv || !w || !q || !k || !v || key_dim <= 0 || value_dim <= 0 || ld < 2 * key_dim + value_dim ||
        cap_rows <= 0 || cap_seqs <= 0 || cap_seqs > MAX_SEQS)
        return cudaErrorInvalidValue;
    SeqTable cap;  // launch geometry only
    memset(&cap, 0, sizeof(cap));
    cap.count = 1;
    cap.offset[1] = cap_rows;
    return conv_launch(qkv, history, ld, w, q, k, v, cap, key_dim, value_dim, static_cast<const DevBatch*>(desc),
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cs1_gdn_gates_dyn(const void* b, const void* a, int ld, const void* A_log, const void* dt_bias,
                                 void* beta, float* g, int cap_rows, int H, const void* desc, void* stream) {
    if (!desc || cap_rows < 0 || H < 0 || ld < H) return cudaErrorInvalidValue;
    const long n = (long)cap_rows * H;
    if (n == 0) return cudaSuccess;
    return launch_pdl(gates_kernel, dim3(grid_for(n)), dim3(THREADS), 0, static_cast<cudaStream_t>(stream),
                      static_cast<const bf16*>(b), static_cast<const bf16*>(a), ld, static_cast<const bf16*>(A_log),
                      static_cast<const bf16*>(dt_bias), static_cast<bf16*>(beta), g, n, H,
                      static_cast<const DevBatch*>(desc));
}

extern "C" int cs1_sigmoid_gate(void* x, const void* gate, size_t n, void* stream) {
    if (n == 0) return cudaSuccess;
    sigmoid_gate_kernel<<<grid_for(n), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<bf16*>(x), static_cast<const bf16*>(gate), n);
    return cudaGetLastError();
}

extern "C" int cs1_silu_mul(const void* gate_up, int ld, void* out, int T, int I, void* stream) {
    if (T < 0 || I < 0 || ld < 2 * I) return cudaErrorInvalidValue;
    const long n = (long)T * I;
    if (n == 0) return cudaSuccess;
    auto st = static_cast<cudaStream_t>(stream);
    if (I % 8 == 0 && ld % 8 == 0 && aligned16(gate_up) && aligned16(out))
    {
        const unsigned cols = (unsigned)((I / 8 + THREADS - 1) / THREADS);
        const long pairs = ((long)T + 1) / 2;
        const unsigned rows = (unsigned)(pairs < 65535 ? pairs : 65535);
        silu_mul_vec_kernel<<<dim3(cols, rows), THREADS, 0, st>>>(static_cast<const bf16*>(gate_up), ld,
                                                                  static_cast<bf16*>(out), I, T);
    }
    else
        silu_mul_scalar_kernel<<<grid_for(n), THREADS, 0, st>>>(static_cast<const bf16*>(gate_up), ld,
                                                                 static_cast<bf16*>(out), I, T);
    return cudaGetLastError();
}

extern "C" int cs1_bf16_finite(const void* x, size_t n, uint32_t* flag, void* stream) {
    auto st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(uint32_t), st);
    if (e != cudaSuccess) return e;
    if (n) finite_kernel<<<grid_for(n), THREADS, 0, st>>>(static_cast<const uint16_t*>(x), n, flag);
    return cudaGetLastError();
}

// ---- counter-based random fill (weights for benchmarks; not a Transformers init) ----
namespace s1 {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float unit(uint64_t bits) { return ((bits >> 40) + 0.5f) * (1.0f / 16777216.0f); }

// kind 0: a + b * N(0,1) (Box-Muller); 1: U(a, b); 2: log U(a, b). dtype 0 bf16, 1 f32.
__global__ void fill_kernel(void* dst, size_t n, int kind, uint64_t seed, float a, float b, int dtype) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t r1 = mix64(seed ^ mix64(2 * i)), r2 = mix64(seed ^ mix64(2 * i + 1));
        float x;
        if (kind == 0) {
            const float u1 = unit(r1), u2 = unit(r2);
            x = a + b * sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
        } else {
            x = a + (b - a) * unit(r1);
            if (kind == 2) x = logf(x);
        }
        if (dtype == 0) static_cast<bf16*>(dst)[i] = to_bf16(x);
        else static_cast<float*>(dst)[i] = x;
    }
}

}  // namespace
}  // namespace s1

extern "C" int cs1_fill_random(void* dst, size_t n, int kind, uint64_t seed, float a, float b, int dtype,
                               void* stream) {
    if (!dst || kind < 0 || kind > 2 || dtype < 0 || dtype > 1) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    s1::fill_kernel<<<s1::grid_for(n), s1::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(dst, n, kind, seed, a, b,
                                                                                        dtype);
    return cudaGetLastError();
}
