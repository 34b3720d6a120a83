// Kernel (c): block-sparse causal FlashAttention forward on sm_100a tensor cores.
// Q, K and V are read in their natural [rows, heads, head_dim] layout (V as an MN-major operand).
//
// One CTA per (128-row query tile, query head); two CTAs share an SM (each holds 256 of the 512
// tensor-memory columns), so one CTA's softmax overlaps the other's MMAs.  Warp roles:
//   warps 0-3  softmax + epilogue: thread r owns query row r = TMEM lane r
//   warp 4     TMA producer: Q once, then K and V tiles of each walked key tile into
//              mbarrier-guarded stage rings (no multicast)
//   warp 5     TMEM allocator and single-thread tcgen05.mma issuer
// Per key tile t (128 keys: one 128-key block or two 64-key blocks of the block list, walked from
// the last list entry to the first like the reference, kai_fa_fp8_tma.py:149-162):
//   S  = Q K^T            tcgen05.mma, A and B from shared memory, fp32 accumulator in TMEM
//   softmax (online, exp2 domain, scale folded: kai_fa_fp8.py:76-77) -> P written back into the S
//   columns of TMEM (e4m3 after scaling by 448, or bf16); O rescaled in TMEM when the row max grows
//   O += P V              tcgen05.mma, A = P from TMEM, B = V tile from shared memory (MN-major)
// Epilogue: O * out_scale / rowsum -> bf16 (0 for a row with no visible key, kai_fa_fp8.py:259-264).
// Every mbarrier wait is bounded (sa_common.cuh); on expiry the CTA drains its copies and MMAs,
// frees TMEM and exits with a status bit set.
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "attn_common.cuh"
#include "sa_common.cuh"

namespace sa {
namespace {

template <bool FP8>
struct Cfg {
    static constexpr int E = FP8 ? 1 : 2;                 // bytes per operand element
    static constexpr int D = 128;                         // head_dim
    static constexpr int BM = 128;                        // query rows per tile (TMEM lanes)
    static constexpr int BN = 64;                         // keys per S tile
    static constexpr int NST = FP8 ? 4 : 2;               // K+V^T stages of BN keys
    static constexpr int UK = FP8 ? 32 : 16;              // MMA K per instruction
    static constexpr int QK_STEPS = D / UK;
    static constexpr int PV_STEPS = BN / UK;
    static constexpr int REG_ELEMS = 128 / E;             // head_dim elements per 128-byte swizzle row
    static constexpr int NREG = D / REG_ELEMS;            // swizzle regions along head_dim
    static constexpr int Q_REG = BM * 128;                // bytes of one Q region (128 rows x 128 B)
    static constexpr int K_REG = BN * 128;                // bytes of one K region (64 rows x 128 B)
    static constexpr int Q_BYTES = NREG * Q_REG;
    static constexpr int K_BYTES = NREG * K_REG;
    static constexpr int V_REG = BN * 128;                // one V region: 64 keys x 128 B of head_dim
    static constexpr int V_BYTES = NREG * V_REG;          // V tile [64 keys][128 d], d contiguous
    static constexpr int STAGE = K_BYTES + V_BYTES;
    static constexpr int SMEM_TILES = Q_BYTES + NST * STAGE;
    static constexpr int SMEM_BYTES = SMEM_TILES + 1024 /*barriers*/ + 1024 /*alignment*/;
    static constexpr uint32_t FMT = FP8 ? 0u : 1u;
    static constexpr uint32_t IDESC_QK = instr_desc(128, BN, FMT);
    // P.V: B = V tile read MN-major (d contiguous), so V is consumed in its natural layout
    static constexpr uint32_t IDESC_PV = instr_desc(128, D, FMT) | (1u << 16);
    static constexpr uint32_t TMEM_COLS = 256;
    static constexpr uint32_t S_COL0 = 0;                 // S/P buffer b at S_COL0 + b * BN

    static constexpr uint32_t O_COL = 128;
    static constexpr int THREADS = 192;
    // Rescale O only when the running row max grows by more than this (log2 units).  bf16 P can
    // exceed 1 safely; e4m3 P (scaled to 448) cannot, so the FP8 kernel rescales on every increase.
    static constexpr float RESCALE_SLACK = FP8 ? 0.f : 8.f;
};


// exponential pairs in eight computed on the FMA pipe (FP8).  1 measured fastest on the power-capped
// benchmark chunk (11.52 ms vs 11.69 / 11.70 ms for 2 / 3 on one box; with the polling waits the
// attention launch took 11.46-11.53 ms against 11.63-11.64 for 0 and 11.60-11.64 for 2).
#ifndef SA_TILE_EXP_POLY
#define SA_TILE_EXP_POLY 1
#endif
constexpr int TILE_EXP_POLY = SA_TILE_EXP_POLY;

// Paged K/V (BF16 kernel).  The BF16 kernel has two K/V stages, so the load of tile u+2 starts
// only once O += P(u) V_u has freed its stage and sits on the critical path: everything a paged
// stage needs beyond the TMA issue is worked out before the stage-empty wait.  Lane i < 64 / box_rows
// owns box i of the tile (keys kb + i * box_rows ..): the TMA coordinates of its page (slot, page),
// or an out-of-range page coordinate (zero fill) when the box starts at or past kv_len or its page
// id is outside [0, num_pages) (SA_DEV_BAD_PAGE).  `tail` is the box that holds the last key when
// kv_len ends inside it (-1 otherwise).
struct PagedBox {
    int slot, page, tail;
    bool bad;
};

__device__ __forceinline__ PagedBox paged_box(const Params& p, int kb, int lane) {
    PagedBox b;
    const int key0 = kb + (lane << p.box_shift);
    b.slot = 0;
    b.page = p.num_pages;
    bool bad = false;
    if (lane < (64 >> p.box_shift) && key0 < p.kv_len) {
        const int pi = p.page_shift >= 0 ? key0 >> p.page_shift : key0 / p.page;
        const int id = __ldg(p.pages + pi);
        bad = static_cast<unsigned>(id) >= static_cast<unsigned>(p.num_pages);
        b.page = bad ? p.num_pages : id;
        b.slot = key0 - pi * p.page;
    }
    b.bad = __any_sync(0xffffffffu, bad);
    b.tail = (p.last_box0 >= kb && p.last_box0 < kb + 64) ? (p.last_box0 - kb) >> p.box_shift : -1;
    return b;
}

// One K/V stage of a paged cache, after the stage-empty wait.  The tail box is read by the warp's
// lanes with plain 16-byte loads instead of TMA (rows past kv_len written as zeros, as TMA's bounds
// give a contiguous K/V), stored at the 128-byte-swizzled places TMA would use (16-byte chunk c of
// tile row R at chunk c ^ (R % 8) of the row) and fenced for the tensor cores.  Lane 0 then arms the
// stage barrier with the remaining bytes and every lane issues the 4D TMA loads of its own box.
template <class C>
__device__ __forceinline__ void load_paged_stage(const Params& p, uint8_t* dst, uint32_t full, const CUtensorMap* tmK,
                                                 const CUtensorMap* tmV, int kb, int hk, int lane, const PagedBox& b,
                                                 volatile int* kb_slot) {
    static_assert(C::E == 2, "paged stages are bf16");
    const int br = 1 << p.box_shift;
    if (b.bad && lane == 0 && p.status) atomicOr(p.status, SA_DEV_BAD_PAGE);
    uint32_t tail_bytes = 0;
    if (b.tail >= 0) {
        const int tp = __shfl_sync(0xffffffffu, b.page, b.tail);
        const int slot0 = __shfl_sync(0xffffffffu, b.slot, b.tail);
        const bool tp_ok = tp < p.num_pages;
        const int valid = p.kv_len - p.last_box0;
        const int chunks = br * 16;                          // 16-byte chunks of the box's K rows (and V rows)
        for (int i = lane; i < 2 * chunks; i += 32) {
            const bool isv = i >= chunks;
            const int ii = isv ? i - chunks : i;
            const int rr = ii >> 4, c = ii & 15;
            const int R = b.tail * br + rr;                  // row of the 64-key tile
            uint4 val = make_uint4(0u, 0u, 0u, 0u);
            if (rr < valid && tp_ok) {
                const uint16_t* base = isv ? p.vc : p.kc;
                val = *reinterpret_cast<const uint4*>(base + static_cast<int64_t>(tp) * p.kv_ps +
                                                      static_cast<int64_t>(slot0 + rr) * p.kv_rs +
                                                      static_cast<int64_t>(hk) * p.kv_hs + c * 8);
            }
            const int reg = c >> 3, cc = c & 7;
            uint8_t* d = dst + (isv ? C::K_BYTES + reg * C::V_REG : reg * C::K_REG) + R * 128 + ((cc ^ (R & 7)) << 4);
            *reinterpret_cast<uint4*>(d) = val;
        }
        fence_proxy_async_smem();
        tail_bytes = static_cast<uint32_t>(2 * br * 256);
    }
    __syncwarp();
    if (lane == 0) {
        *kb_slot = kb;
        mbar_arrive_expect_tx(full, C::STAGE - tail_bytes);
    }
    __syncwarp();
    if (lane < (64 >> p.box_shift) && lane != b.tail) {
#pragma unroll
        for (int r = 0; r < C::NREG; ++r) {
            tma_load_4d(smem_u32(dst + r * C::K_REG + lane * br * 128), tmK, full, r * C::REG_ELEMS, hk, b.slot, b.page);
            tma_load_4d(smem_u32(dst + C::K_BYTES + r * C::V_REG + lane * br * 128), tmV, full, r * C::REG_ELEMS, hk,
                        b.slot, b.page);
        }
    }
    __syncwarp();
}

// One 64-key tile of a softmax warp (thread r owns query row r = TMEM lane r): waits for S(gt),
// loads its 64 columns, masks invisible keys (diagonal, kv_len, rows outside the tile's list half),
// updates the running max (exp2 domain, scale folded) and row sum, writes P into the S columns (e4m3
// x448 or bf16), rescales O in TMEM when the max grew (not on a unit's first tile), and arrives on
// P(gt).  gt counts the tiles the CTA has walked (S/P buffer and barrier parities).  Returns false
// when a bounded wait gave up.
template <bool FP8>
__device__ __forceinline__ bool softmax_tile(const Params& p, int gt, bool first, int kb, uint32_t rm, uint32_t tS0,
                                             uint32_t tO, int qpos_min, int vis, uint32_t my_half, float sl2,
                                             float pbias, float& m_run, float& l_run, uint64_t* bS, uint64_t* bP,
                                             uint64_t* bO, volatile int* abort_flag) {
    using C = Cfg<FP8>;
        const int b = gt & 1;
        bool ok = __all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bS + b), (gt >> 1) & 1, abort_flag, p.status, SA_DEV_WAIT_S));
        if (!ok) return false;
        tc_fence_after();
        const uint32_t tS = tS0 + b * C::BN;
        float x[64];
        {
            uint32_t u[64];
            tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(u));
            tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(u[i]);
        }
        if (rm != 3u || kb + 63 > qpos_min || kb + 63 >= p.kv_len) {
            const int lim = (rm & my_half) ? vis - kb : -1;      // visible columns: c <= lim
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (c > lim) x[c] = -INFINITY;
        }
        float mx;
        {
            float a[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = fmax3(x[i], x[8 + i], x[16 + i]);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = fmax3(a[i], x[24 + i], x[32 + i]);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = fmax3(a[i], x[40 + i], x[48 + i]);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = fmaxf(a[i], x[56 + i]);
            mx = fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
        }
        // running max used for the exponentials; grows (with an O rescale) only past the slack
        const float cand = mx * sl2;
        const bool grow = cand > m_run + C::RESCALE_SLACK || m_run == -INFINITY;
        const float m_new = grow ? fmaxf(m_run, cand) : m_run;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = ex2_approx(m_run - m_use);
        const float2 sl2v = make_float2(sl2, sl2), biasv = make_float2(pbias - m_use, pbias - m_use);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        auto exp_pair = [&](int c) -> float2 {
            const float2 e = ffma2(make_float2(x[c], x[c + 1]), sl2v, biasv);
            // FP8: TILE_EXP_POLY pairs in eight on the FMA pipe, easing the MUFU unit (exp2_poly's
            // 7.5e-5 relative error is far below e4m3's rounding)
            const bool on_fma = FP8 && ((c >> 1) & 7) >= 8 - TILE_EXP_POLY;
            const float2 pr = on_fma ? exp2_poly2(e) : make_float2(ex2_approx(e.x), ex2_approx(e.y));
            acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pr);
            return pr;
        };
        if constexpr (FP8) {
            // 64 keys -> 16 columns of 4 e4m3 values (key 4c+i in byte i of column c)
            uint32_t pk[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float2 p01 = exp_pair(4 * c);
                const float2 p23 = exp_pair(4 * c + 2);
                pk[c] = static_cast<uint32_t>(pack_e4m3x2(p01.x, p01.y)) |
                        (static_cast<uint32_t>(pack_e4m3x2(p23.x, p23.y)) << 16);
            }
            tmem_st16(tS, pk);
        } else {
            // 64 keys -> 32 columns of 2 bf16 values (key 2c+i in half i of column c)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const float2 pr = exp_pair(32 * hh + 2 * c);
                    pk[c] = pack_bf16x2(pr.x, pr.y);
                }
                tmem_st16(tS + 16 * hh, pk);
            }
        }
        const float2 s01 = fadd2(acc[0], acc[1]), s23 = fadd2(acc[2], acc[3]);
        l_run = l_run * alpha + ((s01.x + s01.y) + (s23.x + s23.y));
        m_run = m_new;
        if (!first && __any_sync(0xffffffffu, alpha < 1.f)) {
            // O rescale: wait until O += P(gt-1) V has completed, then scale in TMEM.  S(gt)
            // being complete implies O += P(gt-2) V is, so the barrier is at most one phase
            // behind and the parity wait is unambiguous.
            ok = __all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bO), (gt - 1) & 1, abort_flag, p.status, SA_DEV_WAIT_O));
            if (!ok) return false;
            tc_fence_after();
            uint32_t u[128];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * c));
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 128; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_st32(tO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * c));
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(bP + b));
    return ok;
}

// Row r of split tail unit tu (tile m, head h): combines the step ranges' partial outputs, one warp
// per row, lane l holding head_dim columns 4l..4l+3.  With M the largest running max of the ranges
// and w_s = 2^(m_s - M): out = (sum_s w_s O_s) * out_scale / (sum_s w_s l_s), 0 for a row with no
// visible key (as the unsplit epilogue).  The partials of the other CTAs are read past L1.
__device__ __forceinline__ void merge_split_row(const Params& p, int tu, int h, int m, int r, int lane,
                                                float out_scale) {
    const int qrow = m * 128 + r - p.q_front;
    if (qrow < 0 || qrow >= p.n_q) return;
    const float* ml_base = p.part + static_cast<int64_t>(p.n_tail) * p.splits * (128 * 128);
    const int64_t u0 = static_cast<int64_t>(tu) * p.splits;
    float M = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, __ldcg(ml_base + ((u0 + sp) * 128 + r) * 2));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < p.splits; ++sp) {
        const float ms = __ldcg(ml_base + ((u0 + sp) * 128 + r) * 2);
        const float ls = __ldcg(ml_base + ((u0 + sp) * 128 + r) * 2 + 1);
        if (!(ls > 0.f)) continue;
        const float w = ex2_approx(ms - M);
        L += w * ls;
        const float4 o = __ldcg(reinterpret_cast<const float4*>(p.part + ((u0 + sp) * 128 + r) * 128) + lane);
        acc.x += w * o.x;
        acc.y += w * o.y;
        acc.z += w * o.z;
        acc.w += w * o.w;
    }
    const float inv = L > 0.f ? out_scale / L : 0.f;
    uint16_t* orow = reinterpret_cast<uint16_t*>(p.out) + static_cast<int64_t>(qrow) * p.o_row_stride +
                     static_cast<int64_t>(h) * p.o_head_stride;
    *reinterpret_cast<uint2*>(orow + 4 * lane) =
        make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
}

// SPLIT: the split-launch instantiation (1D grid of whole and tail units, step ranges, partial
// outputs); the default instantiation keeps the 2D grid and whole walks with none of that code.
template <bool FP8, bool SPLIT>
__global__ void __launch_bounds__(192, 2) attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                          const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV, const Params p) {
    using C = Cfg<FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sKV = sQ + C::Q_BYTES;                                // stage s: K at s*STAGE, V^T after it
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + C::NST * C::STAGE);
    uint64_t* bQ = bars;
    uint64_t* bFull = bars + 1;
    uint64_t* bEmpty = bFull + C::NST;
    // Barrier phases: a parity wait is only unambiguous while the barrier is at most one phase ahead
    // of its waiter, so the S and P hand-offs use one barrier per S/P buffer (tile t uses t & 1).
    uint64_t* bS = bEmpty + C::NST;                                // [2] S(t) ready
    uint64_t* bP = bS + 2;                                         // [2] P(t) written
    uint64_t* bO = bP + 2;                                         // one phase per O += P V
    uint64_t* bOF = bO + 1;                                        // single phase: last O += P V done
    uint64_t* bDrain = bOF + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDrain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // Per-stage tile descriptor written by the producer before it arms the stage's full barrier:
    // key base of the 64-key tile, KEY_END after the last tile.  The MMA warp reads it after
    // waiting on that barrier.
    volatile int* tile_kb = const_cast<int*>(reinterpret_cast<volatile int*>(abort_flag + 1));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // unit (tile m, head h) and, for a tail unit of a split launch, this CTA's range of its walk
    int m, h, split = 0, tail_unit = -1;
    if constexpr (SPLIT) {
        int u = static_cast<int>(blockIdx.x);
        if (u >= p.n_whole) {
            const int j = u - p.n_whole;
            tail_unit = j / p.splits;
            split = j - tail_unit * p.splits;
            u = p.n_whole + tail_unit;
        }
        h = u / p.n_tiles;
        m = p.n_tiles - 1 - (u - h * p.n_tiles);                     // late (heavier) tiles first
    } else {
        m = p.n_tiles - 1 - static_cast<int>(blockIdx.x);
        h = blockIdx.y;
    }
    const int g = p.H / p.Hk;
    const int hk = h / g;
    int step0 = 0, step1 = INT_MAX;
    bool partial = false;                                            // write O, max, sum to `part`
    if constexpr (SPLIT) {
        const int steps = tail_unit >= 0 ? walk_steps(p, h, m) : 0;
        if (tail_unit >= 0) split_range(p, steps, split, step0, step1);
        if (step1 <= step0) return;                                  // a split of an unsplit unit
        partial = tail_unit >= 0 && steps >= p.split_min_steps;
    }

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(bQ), 1);
        for (int i = 0; i < C::NST; ++i) { mbar_init(smem_u32(bFull + i), 1); mbar_init(smem_u32(bEmpty + i), 1); }
        mbar_init(smem_u32(bS), 1);
        mbar_init(smem_u32(bS + 1), 1);
        mbar_init(smem_u32(bP), 128);
        mbar_init(smem_u32(bP + 1), 128);
        mbar_init(smem_u32(bO), 1);
        mbar_init(smem_u32(bOF), 1);
        mbar_init(smem_u32(bDrain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---------------------------------------------------------------- TMA producer (warp-uniform;
        // one elected lane issues)
        {
            Walker w = make_walker(p, h, m, step0, step1 - step0);
            int kb;
            uint32_t rm;
            bool have = w.template next<SPLIT>(kb, rm);
            int par[C::NST];
            bool used[C::NST];
            for (int i = 0; i < C::NST; ++i) { par[i] = 0; used[i] = false; }
            if (have && elect_one()) {
                tma_prefetch_desc(&tmK);
                tma_prefetch_desc(&tmV);
                mbar_arrive_expect_tx(smem_u32(bQ), C::Q_BYTES);
                const int qrow0 = m * 128 - p.q_front;
                for (int r = 0; r < C::NREG; ++r)
                    tma_load_3d(smem_u32(sQ + r * C::Q_REG), &tmQ, smem_u32(bQ), r * C::REG_ELEMS, h, qrow0);
            }
            __syncwarp();
            bool paged = false;
            if constexpr (!FP8) paged = p.pages != nullptr;
            for (int t = 0;; ++t, have = w.template next<SPLIT>(kb, rm)) {
                const int st = t % C::NST;
                // paged K/V: the tile's boxes are worked out while the stage drains
                PagedBox pbox{0, 0, -1, false};
                if (paged && have) pbox = paged_box(p, kb, lane);
                if (!__all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bEmpty + st), ((t / C::NST) & 1) ^ 1, abort_flag,
                                                        p.status, SA_DEV_WAIT_KV)))
                    break;
                if (!have) {                                          // end of the walk
                    if (elect_one()) {
                        tile_kb[st] = KEY_END;
                        mbar_arrive(smem_u32(bFull + st));
                    }
                    __syncwarp();
                    break;
                }
                uint8_t* dst = sKV + st * C::STAGE;
                if constexpr (!FP8) {
                    if (paged) {
                        load_paged_stage<C>(p, dst, smem_u32(bFull + st), &tmK, &tmV, kb, hk, lane, pbox,
                                            tile_kb + st);
                        par[st] = (t / C::NST) & 1;
                        used[st] = true;
                        continue;
                    }
                }
                if (elect_one()) {
                    tile_kb[st] = kb;
                    mbar_arrive_expect_tx(smem_u32(bFull + st), C::STAGE);
                    for (int r = 0; r < C::NREG; ++r) {
                        tma_load_3d(smem_u32(dst + r * C::K_REG), &tmK, smem_u32(bFull + st), r * C::REG_ELEMS, hk, kb);
                        tma_load_3d(smem_u32(dst + C::K_BYTES + r * C::V_REG), &tmV, smem_u32(bFull + st),
                                    r * C::REG_ELEMS, hk, kb);
                    }
                }
                __syncwarp();
                par[st] = (t / C::NST) & 1;
                used[st] = true;
            }
            if (w.bad && lane == 0 && p.status) atomicOr(p.status, SA_DEV_BAD_LIST);
            if (*abort_flag) {
                // let the copies already issued land before the CTA can exit
                mbar_drain(smem_u32(bQ), 0);
                for (int i = 0; i < C::NST; ++i)
                    if (used[i]) mbar_drain(smem_u32(bFull + i), par[i]);
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---------------------------------------------------------------- MMA issuer (warp-uniform;
        // one elected lane issues each tcgen05.mma / commit)
        //
        // Issue order: S(0), S(1), then for each tile u: O += P(u) V_u immediately followed by
        // S(u+2) = Q K_{u+2}^T into the S buffer P(u) was just read from (the tcgen05 operations of
        // one CTA execute in issue order).  The critical path of the pipeline is P(u) written ->
        // S(u+2) ready, so with three or more stages the wait for tile u+2's K and V is taken before
        // the wait for P(u) and only the two issues sit on that path.  With two stages tile u+2
        // reuses tile u's stage, which only O += P(u) V_u releases, so there it waits afterwards.
        {
            constexpr bool EARLY_FETCH = C::NST >= 3;
            const uint32_t q_base = smem_u32(sQ);
            bool ok = true;
            int T = INT_MAX;                                          // tiles in the walk, once known
            auto fetch = [&](int t) -> bool {                         // wait for tile t's stage
                const int st = t % C::NST;
                if (!__all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bFull + st), (t / C::NST) & 1, abort_flag,
                                                             p.status, SA_DEV_WAIT_KV)))
                    return false;
                if (tile_kb[st] == KEY_END) T = t;
                return true;
            };
            auto issue_qk = [&](int t) {
                tc_fence_after();
                const uint32_t k_base = smem_u32(sKV + (t % C::NST) * C::STAGE);
                if (elect_one()) {
#pragma unroll
                    for (int s = 0; s < C::QK_STEPS; ++s) {
                        const uint32_t qoff = (s / 4) * C::Q_REG + (s % 4) * 32;
                        const uint32_t koff = (s / 4) * C::K_REG + (s % 4) * 32;
                        mma_ss<FP8>(tmem + C::S_COL0 + (t & 1) * C::BN, smem_desc_kmajor(q_base + qoff, 128),
                                    smem_desc_kmajor(k_base + koff, 128), C::IDESC_QK, s > 0 ? 1u : 0u);
                    }
                    tc_commit(smem_u32(bS + (t & 1)));
                }
                __syncwarp();
            };
            auto issue_pv = [&](int u) -> bool {
                if (!__all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bP + (u & 1)), (u >> 1) & 1, abort_flag,
                                                             p.status, SA_DEV_WAIT_P)))
                    return false;
                tc_fence_after();
                const int su = u % C::NST;
                const uint32_t v_base = smem_u32(sKV + su * C::STAGE + C::K_BYTES);
                const uint32_t a_tm = tmem + C::S_COL0 + (u & 1) * C::BN;
                if (elect_one()) {
                    // K step s covers keys UK*s.. of the tile: UK rows of 128 B, a whole number of
                    // 8-row swizzle atoms; head_dim blocks of 128 B are V_REG apart
#pragma unroll
                    for (int s = 0; s < C::PV_STEPS; ++s)
                        mma_ts<FP8>(tmem + C::O_COL, a_tm + s * 8,
                                    smem_desc_mnmajor(v_base + s * C::UK * 128, C::V_REG), C::IDESC_PV,
                                    (u > 0 || s > 0) ? 1u : 0u);
                    tc_commit(smem_u32(bEmpty + su));
                    tc_commit(smem_u32(bO));
                }
                __syncwarp();
                return true;
            };
            ok = fetch(0);
            if (ok && T > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bQ), 0, abort_flag, p.status, SA_DEV_WAIT_Q));
                if (ok) issue_qk(0);
                if (ok) ok = fetch(1);
                if (ok && T > 1) issue_qk(1);
            }
            for (int u = 0; ok && u < T; ++u) {
                const int nx = u + 2;
                if (EARLY_FETCH && T > nx && !(ok = fetch(nx))) break;
                if (!(ok = issue_pv(u))) break;
                if (!EARLY_FETCH && T > nx && !(ok = fetch(nx))) break;
                if (T > nx) issue_qk(nx);
            }
            if (ok && T > 0 && elect_one()) tc_commit(smem_u32(bOF));
            __syncwarp();
            if (*abort_flag) {
                if (elect_one()) tc_commit(smem_u32(bDrain));
                __syncwarp();
                mbar_drain(smem_u32(bDrain), 0);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- softmax + epilogue (warps 0-3)
        const int r = threadIdx.x;                                   // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t tO = tmem + lane_off + C::O_COL;
        const int qpos = p.q_offset + m * 128 + r;
        const int qpos_min = p.q_offset + m * 128;
        const int vis = min(qpos, p.kv_len - 1);                     // visible keys: position <= vis
        const uint32_t my_half = r >= 64 ? 2u : 1u;
        float sl2, out_scale;
        if constexpr (FP8) {
            sl2 = p.softmax_scale * __ldg(p.q_scale + h * p.qss) * __ldg(p.k_scale + hk * p.kss) * LOG2E;
            out_scale = __ldg(p.v_scale + hk * p.vss);
        } else {
            sl2 = p.softmax_scale * LOG2E;
            out_scale = 1.f;
        }
        const float pbias = FP8 ? LOG2_448 : 0.f;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        int t = 0;
        // The softmax threads walk the block lists themselves (the same walk as the producer's), one
        // tile ahead, instead of waiting on the stage barrier for the producer's tile descriptor.
        Walker walk = make_walker(p, h, m, step0, step1 - step0);
        int kb_next;
        uint32_t rm_next;
        bool have_next = walk.template next<SPLIT>(kb_next, rm_next);
        for (;; ++t) {
            if (!have_next) break;
            const int kb = kb_next;
            const uint32_t rm = rm_next;
            have_next = walk.template next<SPLIT>(kb_next, rm_next);
            ok = softmax_tile<FP8>(p, t, t == 0, kb, rm, tmem + lane_off + C::S_COL0, tO, qpos_min, vis, my_half, sl2,
                                   pbias, m_run, l_run, bS, bP, bO, abort_flag);
            if (!ok) break;
        }
        const int T = t;
        // ---------------------------------------------------------------- epilogue
        // (the per-PV barrier cannot be used here: the MMA warp may still be two PVs behind)
        const bool have_o = __all_sync(0xffffffffu, ok && T > 0 &&
                                       mbar_wait(smem_u32(bOF), 0, abort_flag, p.status, SA_DEV_WAIT_O));
        if (have_o) tc_fence_after();
        if (SPLIT && partial) {
            // unnormalised fp32 O row, running max (log2 units) and row sum of this step range
            const int64_t u = static_cast<int64_t>(tail_unit) * p.splits + split;
            float* ml = p.part + static_cast<int64_t>(p.n_tail) * p.splits * (128 * 128) + (u * 128 + r) * 2;
            ml[0] = have_o ? m_run : -INFINITY;
            ml[1] = have_o ? l_run : 0.f;
            if (have_o) {
                float4* orow4 = reinterpret_cast<float4*>(p.part + (u * 128 + r) * 128);
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t u32[32];
                    tmem_ld32(tO + c * 32, u32);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        orow4[c * 8 + i] = make_float4(__uint_as_float(u32[4 * i]), __uint_as_float(u32[4 * i + 1]),
                                                       __uint_as_float(u32[4 * i + 2]), __uint_as_float(u32[4 * i + 3]));
                }
            }
            __threadfence();                              // partials visible before the arrival count
        }
        const float inv = (have_o && l_run > 0.f) ? out_scale / l_run : 0.f;
        const int qrow = m * 128 + r - p.q_front;
        const bool row_ok = !partial && qrow >= 0 && qrow < p.n_q;
        uint16_t* orow = reinterpret_cast<uint16_t*>(p.out) + static_cast<int64_t>(qrow) * p.o_row_stride +
                         static_cast<int64_t>(h) * p.o_head_stride;
#pragma unroll 1
        for (int c = 0; c < (partial ? 0 : 4); ++c) {
            uint32_t u[32];
            if (have_o) {
                tmem_ld32(tO + c * 32, u);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) u[i] = 0u;
            }
            if (row_ok) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    pk[i] = pack_bf16x2(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
                uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if constexpr (SPLIT) {
        // the last range of a split unit to finish combines the unit's rows (no second launch)
        if (partial) {
            __shared__ int merge_here;
            if (threadIdx.x == 0) {
                int* arrived = reinterpret_cast<int*>(p.part + static_cast<int64_t>(p.n_tail) * p.splits * (128 * 128 + 256));
                merge_here = atomicAdd(arrived + tail_unit, 1) == p.splits - 1;
            }
            __syncthreads();
            if (merge_here) {
                __threadfence();
                float out_scale = 1.f;
                if constexpr (FP8) out_scale = __ldg(p.v_scale + hk * p.vss);
                for (int r = warp; r < 128; r += C::THREADS / 32) merge_split_row(p, tail_unit, h, m, r, lane, out_scale);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps and launch
// ------------------------------------------------------------------------------------------------
// Which kernel serves an FP8 call: this file's one-tile kernel, or the paired-tile kernel
// (attn_pair.cu) when SA_ATTN_KERNEL=pair (read once per process; measured slower on the benchmark
// shapes, kept as an option).  BF16 always uses the one-tile kernel.
bool use_pair_kernel() {
    static bool pair = false;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* e = std::getenv("SA_ATTN_KERNEL");
        if (e && !std::strcmp(e, "pair")) pair = true;
    });
    return pair;
}

// A paged K/V cache (BF16 kernel): k and v are the cache bases, krs/khs (= vrs/vhs) the slot and
// head strides, page_stride the element stride between pages.
struct PagedKV {
    const int32_t* pages;
    int page, num_pages;
    int64_t page_stride;
};

// Split walks: `splits` step ranges per tail unit over a caller-provided fp32 workspace (`part`);
// tail_units < 0: the partial last wave of this GPU.
struct SplitOpts {
    int splits, tail_units;
    void* part;
    int64_t part_bytes;
};

// Units run whole and tail units (split) of a split launch: the last tail_units units of the
// launch order, or (tail_units < 0) the partial last wave of 2 resident CTAs per SM on the current
// device (none for less than one wave).
void split_plan(int n_tiles, int H, int splits, int tail_units, int* n_whole, int* n_tail) {
    const int units = n_tiles * H;
    *n_whole = units;
    *n_tail = 0;
    if (splits <= 1) return;
    if (tail_units >= 0) {
        *n_tail = std::min(tail_units, units);
    } else {
        const int slots = 2 * num_sms();
        if (units >= slots) *n_tail = units - (units / slots) * slots;
    }
    *n_whole = units - *n_tail;
}

int64_t split_workspace_bytes(int n_tiles, int H, int splits, int tail_units) {
    int n_whole, n_tail;
    split_plan(n_tiles, H, splits, tail_units, &n_whole, &n_tail);
    // per tail unit and range: O rows and (max, sum) pairs; then one arrival counter per tail unit
    const int64_t floats = static_cast<int64_t>(n_tail) * splits * (128 * 128 + 256);
    return floats * static_cast<int64_t>(sizeof(float)) + ((static_cast<int64_t>(n_tail) * 4 + 15) & ~15ll);
}

template <bool FP8>
int launch_attn(const void* q, int64_t qrs, int64_t qhs, const void* k, int64_t krs, int64_t khs, const void* v,
                int64_t vrs, int64_t vhs, void* out, int64_t ors, int64_t ohs, int n_q, int H, int Hk, int D, int kv_len,
                int q_front, int q_offset, const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                int kv_block, const float* qsc, int qss, const float* ksc, int kss, const float* vsc, int vss,
                float softmax_scale, int32_t* status, cudaStream_t stream, const PagedKV* paged = nullptr,
                const SplitOpts* split = nullptr) {
    using C = Cfg<FP8>;
    const char* name = paged ? "sa_attn_fwd_bf16_paged" : FP8 ? "sa_attn_fwd_fp8" : "sa_attn_fwd_bf16";
    if (D != 128) return fail(SA_ERR_UNSUPPORTED, "%s: head_dim %d (only 128)", name, D);
    if (n_q < 0 || H <= 0 || Hk <= 0 || H % Hk || kv_len <= 0 || q_front < 0 || q_front >= 128 || q_offset < 0)
        return fail(SA_ERR_ARG, "%s: bad sizes", name);
    if (counts && (!lists || (kv_block != 64 && kv_block != 128) || list_stride < 1))
        return fail(SA_ERR_ARG, "%s: block lists need lists, kv_block 64|128", name);
    if (counts && q_block != 128 && !(q_block == 64 && kv_block == 64))
        return fail(SA_ERR_UNSUPPORTED, "%s: q_block %d with kv_block %d (q_block 128, or 64 with kv_block 64)",
                    name, q_block, kv_block);
    if (!q || !k || !v || !out) return fail(SA_ERR_ARG, "%s: null pointer", name);
    if (FP8 && (!qsc || !ksc || !vsc)) return fail(SA_ERR_ARG, "%s: null scale pointer", name);
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const int E = C::E;
    if (!a16(q) || !a16(k) || !a16(v) || !a16(out) || (qrs * E) % 16 || (qhs * E) % 16 || (krs * E) % 16 ||
        (khs * E) % 16 || (vrs * E) % 16 || (vhs * E) % 16 || (ors * 2) % 16 || (ohs * 2) % 16)
        return fail(SA_ERR_ALIGN, "%s: pointers must be 16-byte aligned and strides multiples of 16 bytes", name);
    if (split && split->splits > 1) {                   // checked before any driver or device call
        if (split->splits > 16) return fail(SA_ERR_ARG, "%s: splits %d (at most 16)", name, split->splits);
        const int64_t need = split_workspace_bytes((q_front + n_q + 127) / 128, H, split->splits, split->tail_units);
        if (need > 0 && (!split->part || (reinterpret_cast<uintptr_t>(split->part) & 15) || split->part_bytes < need))
            return fail(SA_ERR_ARG, "%s: split workspace needs %lld bytes (16-byte aligned)", name,
                        static_cast<long long>(need));
    }
    int box_rows = 0;
    if (paged) {
        if (FP8) return fail(SA_ERR_UNSUPPORTED, "%s: paged K/V is bf16 only", name);
        if (!paged->pages || paged->num_pages <= 0) return fail(SA_ERR_ARG, "%s: page table and num_pages > 0 required", name);
        if (paged->page <= 0 || !(paged->page % 64 == 0 || paged->page == 8 || paged->page == 16 || paged->page == 32))
            return fail(SA_ERR_UNSUPPORTED, "%s: page_size %d (8, 16, 32 or a multiple of 64)", name, paged->page);
        if ((paged->page_stride * E) % 16 || krs != vrs || khs != vhs)
            return fail(SA_ERR_ALIGN, "%s: page stride multiple of 16 bytes, K and V with the same strides", name);
        box_rows = std::min(paged->page, 64);
    }
    if (n_q == 0) return SA_OK;
    const int n_tiles = (q_front + n_q + 127) / 128;
    CUtensorMap tmQ, tmK, tmV;
    int rc;
    const CUtensorMapSwizzle sw128 = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = encode3d(&tmQ, FP8, q, D, H, n_q > 0 ? n_q : 1, qhs * E, qrs * E, C::REG_ELEMS, 1, 128, sw128, "q"))) return rc;
    if (paged) {
        const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Hk), static_cast<uint64_t>(paged->page),
                                  static_cast<uint64_t>(paged->num_pages)};
        const uint64_t strides[3] = {static_cast<uint64_t>(khs * E), static_cast<uint64_t>(krs * E),
                                     static_cast<uint64_t>(paged->page_stride * E)};
        const uint32_t box[4] = {static_cast<uint32_t>(C::REG_ELEMS), 1u, static_cast<uint32_t>(box_rows), 1u};
        if ((rc = encode_nd(&tmK, FP8, k, 4, dims, strides, box, sw128, "k pages"))) return rc;
        if ((rc = encode_nd(&tmV, FP8, v, 4, dims, strides, box, sw128, "v pages"))) return rc;
    } else {
        if ((rc = encode3d(&tmK, FP8, k, D, Hk, kv_len, khs * E, krs * E, C::REG_ELEMS, 1, C::BN, sw128, "k"))) return rc;
        if ((rc = encode3d(&tmV, FP8, v, D, Hk, kv_len, vhs * E, vrs * E, C::REG_ELEMS, 1, C::BN, sw128, "v"))) return rc;
    }
    Params p{};
    if (paged) {
        p.pages = paged->pages;
        p.page = paged->page;
        p.box_rows = box_rows;
        p.num_pages = paged->num_pages;
        p.kc = static_cast<const uint16_t*>(k);
        p.vc = static_cast<const uint16_t*>(v);
        p.kv_ps = paged->page_stride;
        p.kv_rs = krs;
        p.kv_hs = khs;
        p.box_shift = box_rows == 8 ? 3 : box_rows == 16 ? 4 : box_rows == 32 ? 5 : 6;
        p.page_shift = -1;
        for (int sh = 0; sh < 31; ++sh)
            if (paged->page == (1 << sh)) p.page_shift = sh;
        p.last_box0 = kv_len % box_rows ? ((kv_len - 1) / box_rows) * box_rows : -1;
    }
    p.counts = counts;
    p.lists = lists;
    p.list_stride = list_stride;
    p.out = out;
    p.o_row_stride = ors;
    p.o_head_stride = ohs;
    p.n_q = n_q;
    p.H = H;
    p.Hk = Hk;
    p.kv_len = kv_len;
    p.q_front = q_front;
    p.q_offset = q_offset;
    p.n_tiles = n_tiles;
    p.kv_block = counts ? kv_block : 64;
    p.q_block = counts ? q_block : 128;
    p.list_rows_per_head = counts ? (q_front + n_q + p.q_block - 1) / p.q_block : 0;
    p.q_scale = qsc;
    p.k_scale = ksc;
    p.v_scale = vsc;
    p.qss = qss;
    p.kss = kss;
    p.vss = vss;
    p.softmax_scale = softmax_scale;
    p.status = status;
    p.splits = 1;
    if (split && split->splits > 1) {
        int n_whole, n_tail;
        split_plan(n_tiles, H, split->splits, split->tail_units, &n_whole, &n_tail);
        if (n_tail > 0 && !(FP8 && use_pair_kernel())) {   // the paired-tile kernel runs its units whole
            p.splits = split->splits;
            p.split_min_steps = 32 * split->splits;
            p.n_whole = n_whole;
            p.n_tail = n_tail;
            p.part = static_cast<float*>(split->part);
        }
    }
    if constexpr (FP8) {
        if (use_pair_kernel()) return launch_attn_pair<true>(tmQ, tmK, tmV, p, stream, name);
    }
    static PerContext attr;                                  // shared-memory opt-in, once per device context
    int dev = 0;
    void* ctx = nullptr;
    if ((rc = current_device_context(name, &dev, &ctx))) return rc;
    {
        std::lock_guard<std::mutex> lock(attr.mu);
        if (attr.ctx[dev] != ctx) {
            cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<FP8, false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(attn_fwd_kernel<FP8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
            if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
            attr.ctx[dev] = ctx;
        }
    }
    if (p.splits > 1) {
        cudaError_t e = cudaMemsetAsync(p.part + static_cast<int64_t>(p.n_tail) * p.splits * (128 * 128 + 256), 0,
                                        sizeof(int) * static_cast<size_t>(p.n_tail), stream);
        if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
        attn_fwd_kernel<FP8, true><<<p.n_whole + p.n_tail * p.splits, C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK,
                                                                                                        tmV, p);
    } else {
        attn_fwd_kernel<FP8, false><<<dim3(n_tiles, H), C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, p);
    }
    return check_launch(name);
}

}  // namespace
}  // namespace sa

extern "C" int sa_attn_fwd_fp8(const uint8_t* q, int64_t q_row_stride, int64_t q_head_stride, const uint8_t* k,
                               int64_t k_row_stride, int64_t k_head_stride, const uint8_t* v, int64_t v_row_stride,
                               int64_t v_head_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                               int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                               const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                               int kv_block, const float* q_scale, int q_scale_stride, const float* k_scale,
                               int k_scale_stride, const float* v_scale, int v_scale_stride, float softmax_scale,
                               int32_t* status, void* stream) {
    return sa::launch_attn<true>(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, v, v_row_stride,
                                 v_head_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                 kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, q_scale,
                                 q_scale_stride, k_scale, k_scale_stride, v_scale, v_scale_stride, softmax_scale, status,
                                 static_cast<cudaStream_t>(stream));
}

extern "C" int sa_attn_split_count(int n_q, int q_front, int num_heads) {
    if (n_q <= 0 || num_heads <= 0 || q_front < 0) return 1;
    // (tile, head) units of nearly equal cost T over 2 resident CTAs per SM: the full waves run
    // whole; the partial last wave's units run as k pieces of T / k, taking ceil(tail * k / slots)
    // rounds.  The k with the shortest total, if it saves at least 5%; 1 for less than one wave.
    const int64_t units = static_cast<int64_t>((q_front + n_q + 127) / 128) * num_heads;
    const int64_t slots = 2ll * sa::num_sms();
    if (units < slots) return 1;
    const int64_t waves = units / slots, tail = units - waves * slots;
    if (tail == 0) return 1;
    int best = 1;
    double best_t = static_cast<double>(waves + 1);
    const double base = best_t;
    for (int k = 2; k <= 8; ++k) {
        const double t = static_cast<double>(waves) + static_cast<double>((tail * k + slots - 1) / slots) / k;
        if (t < best_t - 1e-9) {
            best = k;
            best_t = t;
        }
    }
    return best_t <= base * 0.95 ? best : 1;
}

extern "C" int64_t sa_attn_split_workspace_bytes(int n_q, int q_front, int num_heads, int splits, int tail_units) {
    if (n_q <= 0 || num_heads <= 0 || splits <= 1) return 0;
    return sa::split_workspace_bytes((q_front + n_q + 127) / 128, num_heads, splits, tail_units);
}

extern "C" int sa_attn_fwd_fp8_split(const uint8_t* q, int64_t q_row_stride, int64_t q_head_stride, const uint8_t* k,
                                     int64_t k_row_stride, int64_t k_head_stride, const uint8_t* v,
                                     int64_t v_row_stride, int64_t v_head_stride, void* out, int64_t o_row_stride,
                                     int64_t o_head_stride, int n_q, int num_heads, int num_kv_heads, int head_dim,
                                     int kv_len, int q_front, int q_offset, const int32_t* counts,
                                     const int32_t* lists, int64_t list_stride, int q_block, int kv_block,
                                     const float* q_scale, int q_scale_stride, const float* k_scale,
                                     int k_scale_stride, const float* v_scale, int v_scale_stride,
                                     float softmax_scale, int32_t* status, int splits, int tail_units,
                                     void* workspace, int64_t workspace_bytes, void* stream) {
    const sa::SplitOpts so{splits, tail_units, workspace, workspace_bytes};
    return sa::launch_attn<true>(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, v, v_row_stride,
                                 v_head_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                 kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, q_scale,
                                 q_scale_stride, k_scale, k_scale_stride, v_scale, v_scale_stride, softmax_scale, status,
                                 static_cast<cudaStream_t>(stream), nullptr, &so);
}

extern "C" int sa_attn_fwd_bf16_paged(const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k_cache,
                                      const void* v_cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                      const int32_t* page_table, int page_size, int num_pages, void* out,
                                      int64_t o_row_stride, int64_t o_head_stride, int n_q, int num_heads,
                                      int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                                      const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                                      int kv_block, float softmax_scale, int32_t* status, void* stream) {
    const sa::PagedKV pg{page_table, page_size, num_pages, page_stride};
    return sa::launch_attn<false>(q, q_row_stride, q_head_stride, k_cache, row_stride, head_stride, v_cache, row_stride,
                                  head_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                  kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, nullptr, 0,
                                  nullptr, 0, nullptr, 0, softmax_scale, status, static_cast<cudaStream_t>(stream), &pg);
}

extern "C" int sa_attn_fwd_bf16(const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k,
                                int64_t k_row_stride, int64_t k_head_stride, const void* v, int64_t v_row_stride,
                                int64_t v_head_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                                int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                                const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                                int kv_block, float softmax_scale, int32_t* status, void* stream) {
    return sa::launch_attn<false>(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, v, v_row_stride,
                                  v_head_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                  kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, nullptr, 0,
                                  nullptr, 0, nullptr, 0, softmax_scale, status, static_cast<cudaStream_t>(stream));
}
