// Kernel (c), paired-tile form: block-sparse causal FlashAttention forward on sm_100a tensor cores,
// two 128-row query tiles per CTA sharing every K/V stage.
//
// A CTA owns one work unit: two query tiles that read the same KV head - two query heads of one
// GQA group at the same 128-row tile, or (odd group sizes) two neighbouring tiles of one head.  The
// tiles' block lists are merged into one descending walk of 64-key blocks (the union; every block
// carries a mask of the tiles and 64-row halves that selected it), two blocks per 128-key step.
// The producer loads each step's K and V once into a stage ring; each query tile runs its own
// online softmax over the steps it selected.  One CTA per SM (all 512 tensor-memory columns):
//
//   TMEM columns   [0,128) S/P of tile 0   [128,256) S/P of tile 1
//                  [256,384) O of tile 0   [384,512) O of tile 1
//   warps 0-3      softmax + epilogue of tile 0 (thread r owns row r = TMEM lane r)
//   warps 4-7      softmax + epilogue of tile 1
//   warp 8         TMA producer: Q tiles once, then K and V of each step (two 64-key halves each)
//   warp 9         TMEM allocator and single-thread tcgen05.mma issuer
//   warps 10-11    idle (they complete the warpgroup that holds the producer and the issuer)
//
// Per step u the issuer runs  O0 += P0(u-1) V(u-1),  S0(u) = Q0 K(u)^T,  O1 += P1(u-1) V(u-1),
// S1(u) = Q1 K(u)^T  (each only for a tile that selected the step), so one tile's P.V and next
// Q.K^T run on the tensor core while the other tile's softmax works: the two softmax warpgroups
// alternate and every step keeps N = 128 for both contractions.  P is written back into the S
// columns (e4m3 x 448, or bf16), the next S of a tile overwrites them only after the P.V that reads
// them (tcgen05 operations of one thread execute in issue order).
//
// Every mbarrier wait is bounded (sa_common.cuh); on expiry the CTA drains its copies and MMAs,
// frees TMEM, writes zeros for its rows and sets a status bit.
//
// FP8 only, selected with SA_ATTN_KERNEL=pair.  On the benchmark shapes it runs 2-5% slower than the
// one-tile kernel of attn_fwd.cu (the default): a tile waits for its own P.V and next Q.K^T before
// each step (its S columns hold P), and the exponentials, not the tensor core, bound both designs.
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
struct PCfg {
    static constexpr int E = FP8 ? 1 : 2;                 // bytes per operand element
    static constexpr int D = 128;                         // head_dim
    static constexpr int BM = 128;                        // query rows per tile (TMEM lanes)
    static constexpr int BN = 128;                        // keys per step (two 64-key halves)
    static constexpr int HALF = 64;
    static constexpr int NST = FP8 ? 5 : 2;               // K+V stages
    static constexpr int UK = FP8 ? 32 : 16;              // MMA K per instruction
    static constexpr int QK_STEPS = D / UK;
    static constexpr int PV_STEPS = BN / UK;
    static constexpr int REG_ELEMS = 128 / E;             // head_dim elements per 128-byte swizzle row
    static constexpr int NREG = D / REG_ELEMS;            // swizzle regions along head_dim
    static constexpr int Q_REG = BM * 128;                // one Q region: 128 rows x 128 B
    static constexpr int Q_BYTES = NREG * Q_REG;
    static constexpr int K_REG = BN * 128;                // one K region: 128 keys x 128 B (halves at +8 KB)
    static constexpr int K_BYTES = NREG * K_REG;
    static constexpr int V_REG = BN * 128;                // one V region: 128 keys x 128 B of head_dim
    static constexpr int V_BYTES = NREG * V_REG;
    static constexpr int HALF_BYTES = HALF * 128;         // one 64-key half of one region
    static constexpr int STAGE = K_BYTES + V_BYTES;
    static constexpr int SMEM_TILES = 2 * Q_BYTES + NST * STAGE;
    static constexpr int SMEM_BYTES = SMEM_TILES + 1024 /*barriers*/ + 1024 /*alignment*/;
    static constexpr uint32_t FMT = FP8 ? 0u : 1u;
    static constexpr uint32_t IDESC_QK = instr_desc(128, BN, FMT);
    static constexpr uint32_t IDESC_PV = instr_desc(128, D, FMT) | (1u << 16);   // B (V) MN-major
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int THREADS = 384;
    // TMEM columns of tile i: S/P at s_col(i), O at o_col(i)
    __host__ __device__ static constexpr uint32_t s_col(int i) { return 128u * i; }
    __host__ __device__ static constexpr uint32_t o_col(int i) { return 256u + 128u * i; }
    // Rescale O only when the running row max grows by more than this (log2 units); e4m3 P (scaled
    // to 448) must stay <= 448, so the FP8 kernel rescales on every increase.
    static constexpr float RESCALE_SLACK = FP8 ? 0.f : 8.f;
    // FP8: of every 8 exponential pairs, EXP_POLY are computed with the polynomial on the FMA pipe
    // and the rest on the MUFU unit
#ifndef SA_EXP_POLY
#define SA_EXP_POLY 2
#endif
    static constexpr int EXP_POLY = SA_EXP_POLY;
};

// ------------------------------------------------------------------------------------------------
// Walk of one query tile: descending 64-key block ids, each with a 2-bit mask of the tile's 64-row
// halves that selected it (both halves for 128-row block lists and the dense walk).
// ------------------------------------------------------------------------------------------------
struct TileWalk {
    const int32_t* a;
    const int32_t* b;
    int ia, ib, va, vb;
    int mode;            // 0 absent tile, 1 dense, 2 list of 64-key blocks, 3 list of 128-key blocks,
                         // 4 two lists of 64-key blocks (one per 64-row half)
    int half;            // mode 3: 1 = the upper half of block va comes next
    int dense_next;      // mode 1: next 64-key block id
    int blk_lim;         // entries at or above this are invalid (their key base would overflow)
    bool bad;

    // list entry i (-1 once the list is exhausted); a negative entry maps above every valid block,
    // so that it is walked (first) as an invalid block: masked out and reported
    __device__ __forceinline__ static int load(const int32_t* p, int i) {
        if (i < 0) return -1;
        const int v = __ldg(p + i);
        return v < 0 ? INT_MAX - 1 : v;
    }

    __device__ __forceinline__ int peek() const {
        switch (mode) {
            case 1: return dense_next;
            case 2: return va;
            case 3: return va < 0 ? -1 : (va >= blk_lim ? INT_MAX - 2 + half : 2 * va + half);
            case 4: return max(va, vb);
            default: return -1;
        }
    }
    // Consume 64-key block `blk` if it is this walk's next one; returns the row-half mask (0 if not).
    __device__ __forceinline__ uint32_t take(int blk) {
        if (blk < 0 || peek() != blk) return 0u;
        if (mode == 1) {
            --dense_next;
            return 3u;
        }
        if (mode == 2) {
            --ia;
            va = load(a, ia);
            return 3u;
        }
        if (mode == 3) {
            if (half == 1) {
                half = 0;
            } else {
                half = 1;
                --ia;
                va = load(a, ia);
            }
            return 3u;
        }
        uint32_t m = 0;
        if (va == blk) { m |= 1u; --ia; va = load(a, ia); }
        if (vb == blk) { m |= 2u; --ib; vb = load(b, ib); }
        return m;
    }
};

__device__ __forceinline__ TileWalk make_tile_walk(const Params& p, int h, int m) {
    TileWalk w;
    w.a = w.b = nullptr;
    w.ia = w.ib = -1;
    w.va = w.vb = -1;
    w.half = 1;
    w.dense_next = -1;
    w.bad = false;
    w.blk_lim = KEY_NONE / max(p.kv_block, 64);
    if (h < 0) {
        w.mode = 0;
        return w;
    }
    if (!p.counts) {
        w.mode = 1;
        const int keys = min(p.q_offset + (m + 1) * 128, p.kv_len);
        w.dense_next = keys > 0 ? (keys + 63) / 64 - 1 : -1;
        return w;
    }
    if (p.q_block == 128) {
        w.mode = p.kv_block == 128 ? 3 : 2;
        const int64_t row = static_cast<int64_t>(h) * p.list_rows_per_head + m;
        w.a = p.lists + row * p.list_stride;
        w.ia = max(__ldg(p.counts + row), 0) - 1;
        w.va = TileWalk::load(w.a, w.ia);
    } else {
        w.mode = 4;
        const int64_t row0 = static_cast<int64_t>(h) * p.list_rows_per_head + 2 * m;
        w.a = p.lists + row0 * p.list_stride;
        w.ia = max(__ldg(p.counts + row0), 0) - 1;
        if (2 * m + 1 < p.list_rows_per_head) {
            w.b = p.lists + (row0 + 1) * p.list_stride;
            w.ib = max(__ldg(p.counts + row0 + 1), 0) - 1;
        }
        w.va = TileWalk::load(w.a, w.ia);
        w.vb = w.b ? TileWalk::load(w.b, w.ib) : -1;
    }
    return w;
}

// One step of the merged walk: two 64-key halves (key base KEY_NONE when absent or invalid) and,
// per half, a 4-bit mask (bits 0-1: tile 0's row halves, bits 2-3: tile 1's).
struct Step {
    int kb[2];
    uint32_t mk[2];
};

struct PairWalk {
    TileWalk w[2];
    bool bad;

    __device__ __forceinline__ bool next_half(int& kb, uint32_t& mk, int kvb) {
        const int blk = max(w[0].peek(), w[1].peek());
        if (blk < 0) return false;
        mk = w[0].take(blk) | (w[1].take(blk) << 2);
        // invalid entries (negative or past the key range) were mapped above every valid block
        const bool ok = blk < KEY_NONE / 64;
        if (!ok) bad = true;
        kb = ok ? blk * 64 : KEY_NONE;
        (void)kvb;
        return true;
    }
    __device__ __forceinline__ bool next(Step& s, int kvb) {
        if (!next_half(s.kb[0], s.mk[0], kvb)) return false;
        if (!next_half(s.kb[1], s.mk[1], kvb)) {
            s.kb[1] = KEY_NONE;
            s.mk[1] = 0u;
        }
        return true;
    }
};



// Unit -> (head, tile) of its two query tiles (head -1: absent).  Units run in groups of
// UNIT_TILES consecutive query tiles from the last group to the first (late tiles hold the most
// blocks), and within a group KV head by KV head, so the CTAs resident at one time read the keys and
// values of a few KV heads (they stay in L2) while heavy tiles still start first.
constexpr int UNIT_TILES = 8;

__device__ __forceinline__ void unit_tiles(const Params& p, int unit, int (&h)[2], int (&m)[2]) {
    const int g = p.H / p.Hk;
    const bool even = (g & 1) == 0;
    // per (KV head, tile): g/2 head pairs; odd g: g heads, tiles taken two at a time
    const int per_kv = even ? g / 2 : g;
    const int tile_slots = even ? p.n_tiles : (p.n_tiles + 1) / 2;      // tiles, or tile pairs
    const int grp_span = even ? UNIT_TILES : UNIT_TILES / 2;
    const int n_groups = (tile_slots + grp_span - 1) / grp_span;
    // the top group (run first) may hold fewer slots than grp_span; the groups below it are full
    const int top_span = tile_slots - (n_groups - 1) * grp_span;
    const int top_units = top_span * p.Hk * per_kv;
    int grp, rem, span;
    if (unit < top_units) {
        grp = n_groups - 1;
        rem = unit;
        span = top_span;
    } else {
        const int u2 = unit - top_units, full_units = grp_span * p.Hk * per_kv;
        grp = n_groups - 2 - u2 / full_units;
        rem = u2 % full_units;
        span = grp_span;
    }
    const int kvh = rem / (span * per_kv);
    rem -= kvh * span * per_kv;
    const int slot = grp * grp_span + (span - 1 - rem / per_kv);         // later slots first
    const int j = rem % per_kv;
    if (even) {
        m[0] = m[1] = slot;
        h[0] = kvh * g + 2 * j;
        h[1] = h[0] + 1;
    } else {
        h[0] = h[1] = kvh * g + j;
        m[0] = 2 * slot;
        m[1] = 2 * slot + 1;
        if (m[1] >= p.n_tiles) h[1] = -1;
    }
}

// Register split: the kernel launches 384 threads x 168 registers (64512); the producer / issuer
// warpgroup gives up 104 per thread (64 left), the two softmax warpgroups take 48 more (216):
// 128 x 64 + 256 x 216 = 63488, within the launch total, so the increase never waits.
__device__ __forceinline__ void reg_dealloc_producer() { asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory"); }
__device__ __forceinline__ void reg_alloc_softmax() { asm volatile("setmaxnreg.inc.sync.aligned.u32 216;" ::: "memory"); }

// Step descriptor in shared memory: the two halves' key bases and masks; kb[0] == KEY_END ends a walk.
struct __align__(16) StepDesc {
    int kb[2];
    uint32_t mk[2];
};

template <bool FP8>
__global__ void __launch_bounds__(384, 1) attn_pair_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                           const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV, const Params p) {
    using C = PCfg<FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                                            // [2][Q_BYTES]
    uint8_t* sKV = sQ + 2 * C::Q_BYTES;                            // stage s: K at s*STAGE, V after it
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + C::NST * C::STAGE);
    uint64_t* bQ = bars;
    uint64_t* bFull = bars + 1;
    uint64_t* bEmpty = bFull + C::NST;
    uint64_t* bS = bEmpty + C::NST;                                // [2] S of tile i ready
    uint64_t* bP = bS + 2;                                         // [2] P of tile i written (128 arrivals)
    uint64_t* bD = bP + 2;                                         // [2] step descriptor of tile i posted
    uint64_t* bOF = bD + 2;                                        // single phase: last MMA done
    uint64_t* bDrain = bOF + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDrain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // descriptors: one per stage (written by the producer before it arms the stage), and a
    // two-entry ring per query tile (written by the issuer before it issues the tile's Q.K^T)
    StepDesc* stage_desc = reinterpret_cast<StepDesc*>(reinterpret_cast<uint8_t*>(bars) + 256);
    StepDesc* tile_desc = stage_desc + C::NST;                     // [2 tiles][2 slots]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int hq[2], mq[2];
    unit_tiles(p, blockIdx.x, hq, mq);
    const int hk = hq[0] / (p.H / p.Hk);

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(bQ), 1);
        for (int i = 0; i < C::NST; ++i) { mbar_init(smem_u32(bFull + i), 1); mbar_init(smem_u32(bEmpty + i), 1); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(bS + i), 1);
            mbar_init(smem_u32(bP + i), 128);
            mbar_init(smem_u32(bD + i), 1);
        }
        mbar_init(smem_u32(bOF), 1);
        mbar_init(smem_u32(bDrain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
        reg_dealloc_producer();
        if (warp == 8) {
            // ------------------------------------------------------------ TMA producer: walks the
            // merged block lists, loads each step's K and V halves, posts the step descriptor
            PairWalk walk{{make_tile_walk(p, hq[0], mq[0]), make_tile_walk(p, hq[1], mq[1])}, false};
            int par[C::NST];
            bool used[C::NST];
            for (int i = 0; i < C::NST; ++i) { par[i] = 0; used[i] = false; }
            if (elect_one()) {
                tma_prefetch_desc(&tmK);
                tma_prefetch_desc(&tmV);
                const int nq = hq[1] >= 0 ? 2 : 1;
                mbar_arrive_expect_tx(smem_u32(bQ), nq * C::Q_BYTES);
                for (int i = 0; i < nq; ++i)
                    for (int r = 0; r < C::NREG; ++r)
                        tma_load_3d(smem_u32(sQ + i * C::Q_BYTES + r * C::Q_REG), &tmQ, smem_u32(bQ),
                                    r * C::REG_ELEMS, hq[i], mq[i] * 128 - p.q_front);
            }
            __syncwarp();
            Step s;
            for (int t = 0;; ++t) {
                const bool have = walk.next(s, p.kv_block);
                const int st = t % C::NST;
                if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(bEmpty + st), ((t / C::NST) & 1) ^ 1, abort_flag,
                                                        p.status, SA_DEV_WAIT_KV)))
                    break;
                if (!have) {                                         // end of the walk
                    if (elect_one()) {
                        stage_desc[st].kb[0] = KEY_END;
                        mbar_arrive(smem_u32(bFull + st));
                    }
                    __syncwarp();
                    break;
                }
                uint8_t* dst = sKV + st * C::STAGE;
                if (elect_one()) {
                    stage_desc[st] = StepDesc{{s.kb[0], s.kb[1]}, {s.mk[0], s.mk[1]}};
                    mbar_arrive_expect_tx(smem_u32(bFull + st), C::STAGE);
                    for (int hf = 0; hf < 2; ++hf) {
                        // an absent half loads keys 0..63 (finite data); its scores are masked out
                        const int kb = s.kb[hf] == KEY_NONE ? 0 : s.kb[hf];
                        for (int r = 0; r < C::NREG; ++r) {
                            tma_load_3d(smem_u32(dst + r * C::K_REG + hf * C::HALF_BYTES), &tmK, smem_u32(bFull + st),
                                        r * C::REG_ELEMS, hk, kb);
                            tma_load_3d(smem_u32(dst + C::K_BYTES + r * C::V_REG + hf * C::HALF_BYTES), &tmV,
                                        smem_u32(bFull + st), r * C::REG_ELEMS, hk, kb);
                        }
                    }
                }
                __syncwarp();
                par[st] = (t / C::NST) & 1;
                used[st] = true;
            }
            if (walk.bad && lane == 0 && p.status) atomicOr(p.status, SA_DEV_BAD_LIST);
            if (*abort_flag) {
                mbar_drain(smem_u32(bQ), 0);
                for (int i = 0; i < C::NST; ++i)
                    if (used[i]) mbar_drain(smem_u32(bFull + i), par[i]);
            }
        } else if (warp == 9) {
            // ------------------------------------------------------------ MMA issuer
            bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bQ), 0, abort_flag, p.status, SA_DEV_WAIT_Q));
            bool pend0 = false, pend1 = false;                       // P.V of the previous step owed
            bool init0 = false, init1 = false;                       // O accumulates after its first P.V
            int cnt0 = 0, cnt1 = 0;                                  // steps taken by tile 0 / 1
            int prev_st = 0;
            bool any = false;
            auto issue_pv = [&](int i, int su, int cnt, bool& init) -> bool {
                if (!__all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bP + i), (cnt - 1) & 1, abort_flag, p.status,
                                                             SA_DEV_WAIT_P)))
                    return false;
                tc_fence_after();
                const uint32_t v_base = smem_u32(sKV + su * C::STAGE + C::K_BYTES);
                const uint32_t a_tm = tmem + C::s_col(i);
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < C::PV_STEPS; ++k)
                        mma_ts<FP8>(tmem + C::o_col(i), a_tm + k * (C::UK * C::E / 4),
                                    smem_desc_mnmajor(v_base + k * C::UK * 128, C::V_REG), C::IDESC_PV,
                                    (init || k > 0) ? 1u : 0u);
                }
                __syncwarp();
                init = true;
                return true;
            };
            auto post = [&](int i, int cnt, const StepDesc& d) {     // hand tile i its step descriptor
                if (elect_one()) {
                    tile_desc[2 * i + (cnt & 1)] = d;
                    mbar_arrive(smem_u32(bD + i));
                }
                __syncwarp();
            };
            auto issue_qk = [&](int i, int st) {
                const uint32_t q_base = smem_u32(sQ + i * C::Q_BYTES);
                const uint32_t k_base = smem_u32(sKV + st * C::STAGE);
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < C::QK_STEPS; ++k) {
                        const uint32_t off = (k * C::UK * C::E / 128) * C::Q_REG + (k * C::UK * C::E) % 128;
                        const uint32_t koff = (k * C::UK * C::E / 128) * C::K_REG + (k * C::UK * C::E) % 128;
                        mma_ss<FP8>(tmem + C::s_col(i), smem_desc_kmajor(q_base + off, 128),
                                    smem_desc_kmajor(k_base + koff, 128), C::IDESC_QK, k > 0 ? 1u : 0u);
                    }
                    tc_commit(smem_u32(bS + i));
                }
                __syncwarp();
            };
            const StepDesc end_desc{{KEY_END, KEY_END}, {0u, 0u}};
            for (int u = 0; ok; ++u) {
                const int st = u % C::NST;
                if (pend0 && !(ok = issue_pv(0, prev_st, cnt0, init0))) break;
                pend0 = false;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait_spin(smem_u32(bFull + st), (u / C::NST) & 1, abort_flag,
                                                                  p.status, SA_DEV_WAIT_KV))))
                    break;
                const StepDesc d = stage_desc[st];
                if (d.kb[0] == KEY_END) {
                    if (pend1 && !(ok = issue_pv(1, prev_st, cnt1, init1))) break;
                    pend1 = false;
                    break;
                }
                tc_fence_after();
                any = true;
                const bool use0 = ((d.mk[0] | d.mk[1]) & 3u) != 0u, use1 = ((d.mk[0] | d.mk[1]) & 12u) != 0u;
                if (use0) {
                    post(0, cnt0, d);
                    issue_qk(0, st);
                    ++cnt0;
                    pend0 = true;
                }
                if (pend1 && !(ok = issue_pv(1, prev_st, cnt1, init1))) break;
                pend1 = false;
                if (u > 0) {
                    if (elect_one()) tc_commit(smem_u32(bEmpty + prev_st));   // both P.V of step u-1 issued
                    __syncwarp();
                }
                if (use1) {
                    post(1, cnt1, d);
                    issue_qk(1, st);
                    ++cnt1;
                    pend1 = true;
                }
                prev_st = st;
            }
            if (ok) {
                // end markers for the softmax warpgroups (their last P arrived before the last P.V)
                post(0, cnt0, end_desc);
                post(1, cnt1, end_desc);
                if (any) {
                    if (elect_one()) tc_commit(smem_u32(bOF));
                    __syncwarp();
                }
            }
            if (*abort_flag) {
                if (elect_one()) tc_commit(smem_u32(bDrain));
                __syncwarp();
                mbar_drain(smem_u32(bDrain), 0);
            }
        }
        __syncwarp();
    } else {
        reg_alloc_softmax();
        // ---------------------------------------------------------------- softmax + epilogue
        const int i = warp >> 2;                                     // query tile of this warpgroup
        const int r = threadIdx.x & 127;                             // row within the tile
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + C::s_col(i);
        const uint32_t tO = tmem + lane_off + C::o_col(i);
        const int h = hq[i], m = mq[i];
        const bool present = h >= 0;
        const int qpos = p.q_offset + m * 128 + r;
        const int qpos_min = p.q_offset + m * 128;
        const int vis = min(qpos, p.kv_len - 1);                     // visible keys: position <= vis
        const uint32_t my_bit = 1u << (2 * i + (r >= 64 ? 1 : 0));
        float sl2 = 0.f, out_scale = 1.f;
        if (present) {
            if constexpr (FP8) {
                sl2 = p.softmax_scale * __ldg(p.q_scale + h * p.qss) * __ldg(p.k_scale + hk * p.kss) * LOG2E;
                out_scale = __ldg(p.v_scale + hk * p.vss);
            } else {
                sl2 = p.softmax_scale * LOG2E;
            }
        }
        const float pbias = FP8 ? LOG2_448 : 0.f;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = present;
        int t = 0;                                                   // steps this tile took
        while (ok) {
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bD + i), t & 1, abort_flag, p.status, SA_DEV_WAIT_S));
            if (!ok) break;
            const StepDesc d = tile_desc[2 * i + (t & 1)];
            if (d.kb[0] == KEY_END) break;
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bS + i), t & 1, abort_flag, p.status, SA_DEV_WAIT_S));
            if (!ok) break;
            tc_fence_after();
            uint32_t u[128];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * c));
            tmem_wait_ld();
            // masking: a half this row did not select, keys past the row's position or past kv_len
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int kb = d.kb[hf];
                const bool sel = (d.mk[hf] & my_bit) != 0u;
                if (!sel || kb + 63 > qpos_min || kb + 63 >= p.kv_len) {
                    const int lim = sel ? vis - kb : -1;             // visible columns: c <= lim
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (c > lim) u[64 * hf + c] = 0xff800000u;  // -inf
                }
            }
            float mx;
            {
                float a[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    a[j] = fmax3(__uint_as_float(u[j]), __uint_as_float(u[16 + j]), __uint_as_float(u[32 + j]));
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    a[j] = fmax3(a[j], __uint_as_float(u[48 + j]), __uint_as_float(u[64 + j]));
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    a[j] = fmax3(a[j], __uint_as_float(u[80 + j]), __uint_as_float(u[96 + j]));
#pragma unroll
                for (int j = 0; j < 16; ++j) a[j] = fmaxf(a[j], __uint_as_float(u[112 + j]));
#pragma unroll
                for (int j = 0; j < 5; ++j) a[j] = fmax3(a[3 * j], a[3 * j + 1], a[3 * j + 2]);
                mx = fmax3(fmax3(a[0], a[1], a[2]), fmaxf(a[3], a[4]), a[15]);
            }
            const float cand = mx * sl2;
            const bool grow = cand > m_run + C::RESCALE_SLACK || m_run == -INFINITY;
            const float m_new = grow ? fmaxf(m_run, cand) : m_run;
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = ex2_approx(m_run - m_use);
            const float2 sl2v = make_float2(sl2, sl2), biasv = make_float2(pbias - m_use, pbias - m_use);
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
            auto exp_pair = [&](int c) -> float2 {
                const float2 e = ffma2(make_float2(__uint_as_float(u[c]), __uint_as_float(u[c + 1])), sl2v, biasv);
                // FP8: EXP_POLY pairs in 8 on the FMA pipe (exp2_poly's 7.5e-5 relative error is far
                // below e4m3's rounding), easing the MUFU unit
                const bool on_fma = FP8 && ((c >> 1) & 7) >= 8 - C::EXP_POLY;
                const float2 pr = on_fma ? exp2_poly2(e) : make_float2(ex2_approx(e.x), ex2_approx(e.y));
                acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pr);
                return pr;
            };
            if constexpr (FP8) {
                // 128 keys -> 32 columns of 4 e4m3 values (key 4c+j in byte j of column c)
                uint32_t pk[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float2 p01 = exp_pair(4 * c);
                    const float2 p23 = exp_pair(4 * c + 2);
                    pk[c] = static_cast<uint32_t>(pack_e4m3x2(p01.x, p01.y)) |
                            (static_cast<uint32_t>(pack_e4m3x2(p23.x, p23.y)) << 16);
                }
                tmem_st32(tS, pk);
            } else {
                // 128 keys -> 64 columns of 2 bf16 values (key 2c+j in half j of column c)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t pk[32];
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const float2 pr = exp_pair(64 * hh + 2 * c);
                        pk[c] = pack_bf16x2(pr.x, pr.y);
                    }
                    tmem_st32(tS + 32 * hh, pk);
                }
            }
            const float2 s01 = fadd2(acc[0], acc[1]), s23 = fadd2(acc[2], acc[3]);
            l_run = l_run * alpha + ((s01.x + s01.y) + (s23.x + s23.y));
            m_run = m_new;
            if (t > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
                // O rescale in TMEM.  S(t) complete implies the P.V of this tile's previous step is
                // complete (the issuer issued it before this step's Q.K^T), and this step's P.V waits
                // for the P barrier below.
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[64];
                    tmem_ld32(tO + 64 * c, *reinterpret_cast<uint32_t(*)[32]>(o));
                    tmem_ld32(tO + 64 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 64; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
                    tmem_st32(tO + 64 * c, *reinterpret_cast<uint32_t(*)[32]>(o));
                    tmem_st32(tO + 64 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(bP + i));
            ++t;
        }
        // ---------------------------------------------------------------- epilogue
        const bool have_o = __all_sync(0xffffffffu, present && ok && t > 0 &&
                                       mbar_wait(smem_u32(bOF), 0, abort_flag, p.status, SA_DEV_WAIT_O));
        if (have_o) tc_fence_after();
        const float inv = (have_o && l_run > 0.f) ? out_scale / l_run : 0.f;
        const int qrow = m * 128 + r - p.q_front;
        const bool row_ok = present && qrow >= 0 && qrow < p.n_q;
        uint16_t* orow = reinterpret_cast<uint16_t*>(p.out) + static_cast<int64_t>(qrow) * p.o_row_stride +
                         static_cast<int64_t>(h) * p.o_head_stride;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            if (have_o) {
                tmem_ld32(tO + c * 32, o);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = 0u;
            }
            if (row_ok) {
                uint32_t pk[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    pk[j] = pack_bf16x2(__uint_as_float(o[2 * j]) * inv, __uint_as_float(o[2 * j + 1]) * inv);
                uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                for (int j = 0; j < 4; ++j) dst[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace

// Paired-tile launch; the caller (launch_attn) has validated the arguments and built the tensor maps
// with 64-row K/V boxes.
template <bool FP8>
int launch_attn_pair(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV, const Params& p,
                     cudaStream_t stream, const char* name) {
    using C = PCfg<FP8>;
    static PerContext attr;                                  // shared-memory opt-in, once per device context
    int dev = 0;
    void* ctx = nullptr;
    if (int rc = current_device_context(name, &dev, &ctx)) return rc;
    {
        std::lock_guard<std::mutex> lock(attr.mu);
        if (attr.ctx[dev] != ctx) {
            cudaError_t e = cudaFuncSetAttribute(attn_pair_kernel<FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::SMEM_BYTES);
            if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
            attr.ctx[dev] = ctx;
        }
    }
    const int g = p.H / p.Hk;
    const int units = (g % 2 == 0) ? p.n_tiles * (p.H / 2) : ((p.n_tiles + 1) / 2) * p.H;
    attn_pair_kernel<FP8><<<units, C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, p);
    return check_launch(name);
}

template int launch_attn_pair<true>(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const Params&,
                                    cudaStream_t, const char*);

}  // namespace sa
