// Kernel (c): block-sparse causal FlashAttention forward on sm_100a tensor cores.
//
// One CTA per (128-row query tile, query head); two CTAs share an SM (each holds 256 of the 512
// tensor-memory columns), so one CTA's softmax overlaps the other's MMAs.  Warp roles:
//   warps 0-3  softmax + epilogue: thread r owns query row r = TMEM lane r
//   warp 4     TMA producer: Q once, then K and V^T tiles of each walked key tile into
//              mbarrier-guarded stage rings (no multicast)
//   warp 5     TMEM allocator and single-thread tcgen05.mma issuer
// Per key tile t (128 keys: one 128-key block or two 64-key blocks of the block list, walked from
// the last list entry to the first like the reference, kai_fa_fp8_tma.py:149-162):
//   S  = Q K^T            tcgen05.mma, A and B from shared memory, fp32 accumulator in TMEM
//   softmax (online, exp2 domain, scale folded: kai_fa_fp8.py:76-77) -> P written back into the S
//   columns of TMEM (e4m3 after scaling by 448, or bf16); O rescaled in TMEM when the row max grows
//   O += P V              tcgen05.mma, A = P from TMEM, B = V^T tile from shared memory
// Epilogue: O * out_scale / rowsum -> bf16 (0 for a row with no visible key, kai_fa_fp8.py:259-264).
// Every mbarrier wait is bounded (sa_common.cuh); on expiry the CTA drains its copies and MMAs,
// frees TMEM and exits with a status bit set.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "sa_common.cuh"

namespace sa {
namespace {

constexpr int KEY_NONE = 1 << 30;   // key base of an absent half tile: every key masked, TMA zero-fills
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LOG2_448 = 8.807354922057604f;

template <bool FP8>
struct Cfg {
    static constexpr int E = FP8 ? 1 : 2;                 // bytes per operand element
    static constexpr int D = 128;
    static constexpr int BM = 128, BN = 128;
    static constexpr int KST = 2;                         // K stages
    static constexpr int VST = FP8 ? 2 : 1;               // V^T stages
    static constexpr int UK = FP8 ? 32 : 16;              // MMA K per instruction
    static constexpr int QK_STEPS = D / UK;
    static constexpr int PV_STEPS = BN / UK;
    static constexpr int REG_ELEMS = 128 / E;             // head_dim elements per 128-byte swizzle row
    static constexpr int NREG = D / REG_ELEMS;            // swizzle regions along head_dim
    static constexpr int REG_BYTES = 128 * 128;           // one region: 128 rows x 128 B
    static constexpr int Q_BYTES = BM * D * E;
    static constexpr int K_BYTES = BN * D * E;
    static constexpr int VROW = 64 * E;                   // bytes per V^T row of a 64-key chunk
    static constexpr int VCHUNK = D * VROW;               // one 64-key chunk of V^T
    static constexpr int V_BYTES = 2 * VCHUNK;
    static constexpr int SMEM_TILES = Q_BYTES + KST * K_BYTES + VST * V_BYTES;
    static constexpr int SMEM_BYTES = SMEM_TILES + 1024 /*barriers*/ + 1024 /*alignment*/;
    static constexpr uint32_t IDESC = instr_desc(128, 128, FP8 ? 0u : 1u);
    static constexpr uint32_t TMEM_COLS = 256;
    static constexpr uint32_t S_COL = 0, O_COL = 128;
    static constexpr int THREADS = 192;
};

struct Params {
    const int32_t* counts;
    const int32_t* lists;
    int64_t list_stride;
    void* out;
    int64_t o_row_stride, o_head_stride;
    int n_q, H, Hk, kv_len, q_front, q_offset, n_tiles, kv_block;
    const float* q_scale;
    const float* k_scale;
    const float* v_scale;
    int qss, kss, vss;
    float softmax_scale;
    int32_t* status;
};

struct Walk {
    const int32_t* list;   // null: dense causal walk
    int cnt;               // list entries
    int ntiles;            // key tiles to walk
    int nblk;              // dense: 128-key blocks
    int kvb;
};

__device__ __forceinline__ int sanitize_block(int b, int kvb, bool& bad) {
    if (b < 0 || b >= KEY_NONE / kvb) {
        bad = true;
        return KEY_NONE;
    }
    return b * kvb;
}

// Key positions of the two 64-key halves of key tile t.
__device__ __forceinline__ void tile_keys(const Walk& w, int t, int& kb0, int& kb1, bool& bad) {
    if (!w.list) {
        kb0 = (w.nblk - 1 - t) * 128;
        kb1 = kb0 + 64;
    } else if (w.kvb == 128) {
        kb0 = sanitize_block(__ldg(w.list + (w.cnt - 1 - t)), 128, bad);
        kb1 = kb0 == KEY_NONE ? KEY_NONE : kb0 + 64;
    } else {
        const int i = w.cnt - 1 - 2 * t;
        kb0 = sanitize_block(__ldg(w.list + i), 64, bad);
        kb1 = i >= 1 ? sanitize_block(__ldg(w.list + i - 1), 64, bad) : KEY_NONE;
    }
}

template <bool FP8>
__global__ void __launch_bounds__(192, 2) attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                          const __grid_constant__ CUtensorMap tmK,
                                                          const __grid_constant__ CUtensorMap tmV, const Params p) {
    using C = Cfg<FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + C::Q_BYTES;
    uint8_t* sV = sK + C::KST * C::K_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + C::VST * C::V_BYTES);
    // barrier slots
    uint64_t* bQ = bars;
    uint64_t* bKf = bars + 1;
    uint64_t* bKe = bKf + C::KST;
    uint64_t* bVf = bKe + C::KST;
    uint64_t* bVe = bVf + C::VST;
    uint64_t* bS = bVe + C::VST;
    uint64_t* bP = bS + 1;
    uint64_t* bO = bP + 1;
    uint64_t* bDrain = bO + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bDrain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = p.n_tiles - 1 - static_cast<int>(blockIdx.x);     // heavy (late) tiles first
    const int h = blockIdx.y;
    const int g = p.H / p.Hk;
    const int hk = h / g;

    Walk w;
    w.kvb = p.kv_block;
    if (p.counts) {
        const int64_t row = static_cast<int64_t>(h) * p.n_tiles + m;
        w.list = p.lists + row * p.list_stride;
        w.cnt = max(__ldg(p.counts + row), 0);
        w.nblk = 0;
        w.ntiles = p.kv_block == 128 ? w.cnt : (w.cnt + 1) / 2;
    } else {
        w.list = nullptr;
        w.cnt = 0;
        const int last = p.q_offset + (m + 1) * 128;                 // one past the tile's last position
        w.nblk = min((last + 127) / 128, (p.kv_len + 127) / 128);
        w.nblk = max(w.nblk, 0);
        w.ntiles = w.nblk;
    }
    const int T = w.ntiles;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(bQ), 1);
        for (int i = 0; i < C::KST; ++i) { mbar_init(smem_u32(bKf + i), 1); mbar_init(smem_u32(bKe + i), 1); }
        for (int i = 0; i < C::VST; ++i) { mbar_init(smem_u32(bVf + i), 1); mbar_init(smem_u32(bVe + i), 1); }
        mbar_init(smem_u32(bS), 1);
        mbar_init(smem_u32(bP), 128);
        mbar_init(smem_u32(bO), 1);
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
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0 && T > 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            int kpar[C::KST], vpar[C::VST];
            bool kused[C::KST], vused[C::VST];
            for (int i = 0; i < C::KST; ++i) { kpar[i] = 0; kused[i] = false; }
            for (int i = 0; i < C::VST; ++i) { vpar[i] = 0; vused[i] = false; }
            bool bad = false;
            mbar_arrive_expect_tx(smem_u32(bQ), C::Q_BYTES);
            const int qrow0 = m * 128 - p.q_front;
            for (int r = 0; r < C::NREG; ++r)
                tma_load_3d(smem_u32(sQ + r * C::REG_BYTES), &tmQ, smem_u32(bQ), r * C::REG_ELEMS, h, qrow0);
            for (int t = 0; t < T; ++t) {
                int kb0, kb1;
                tile_keys(w, t, kb0, kb1, bad);
                const int ks = t % C::KST;
                if (!mbar_wait(smem_u32(bKe + ks), ((t / C::KST) & 1) ^ 1, abort_flag, p.status, SA_DEV_WAIT_KV)) break;
                uint8_t* kdst = sK + ks * C::K_BYTES;
                mbar_arrive_expect_tx(smem_u32(bKf + ks), C::K_BYTES);
                for (int r = 0; r < C::NREG; ++r) {
                    tma_load_3d(smem_u32(kdst + r * C::REG_BYTES), &tmK, smem_u32(bKf + ks), r * C::REG_ELEMS, hk, kb0);
                    tma_load_3d(smem_u32(kdst + r * C::REG_BYTES + 64 * 128), &tmK, smem_u32(bKf + ks),
                                r * C::REG_ELEMS, hk, kb1);
                }
                kpar[ks] = (t / C::KST) & 1;
                kused[ks] = true;
                const int vs = t % C::VST;
                if (!mbar_wait(smem_u32(bVe + vs), ((t / C::VST) & 1) ^ 1, abort_flag, p.status, SA_DEV_WAIT_KV)) break;
                uint8_t* vdst = sV + vs * C::V_BYTES;
                mbar_arrive_expect_tx(smem_u32(bVf + vs), C::V_BYTES);
                tma_load_3d(smem_u32(vdst), &tmV, smem_u32(bVf + vs), kb0, 0, hk);
                tma_load_3d(smem_u32(vdst + C::VCHUNK), &tmV, smem_u32(bVf + vs), kb1, 0, hk);
                vpar[vs] = (t / C::VST) & 1;
                vused[vs] = true;
            }
            if (*abort_flag) {
                // let the copies already issued land before the CTA can exit
                mbar_drain(smem_u32(bQ), 0);
                for (int i = 0; i < C::KST; ++i)
                    if (kused[i]) mbar_drain(smem_u32(bKf + i), kpar[i]);
                for (int i = 0; i < C::VST; ++i)
                    if (vused[i]) mbar_drain(smem_u32(bVf + i), vpar[i]);
            }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && T > 0) {
            const uint32_t tS = tmem + C::S_COL, tO = tmem + C::O_COL;
            const uint32_t q_base = smem_u32(sQ);
            bool ok = mbar_wait(smem_u32(bQ), 0, abort_flag, p.status, SA_DEV_WAIT_Q);
            for (int t = 0; ok && t < T; ++t) {
                const int ks = t % C::KST;
                if (!mbar_wait(smem_u32(bKf + ks), (t / C::KST) & 1, abort_flag, p.status, SA_DEV_WAIT_KV)) break;
                tc_fence_after();
                const uint32_t k_base = smem_u32(sK + ks * C::K_BYTES);
#pragma unroll
                for (int s = 0; s < C::QK_STEPS; ++s) {
                    const uint32_t off = (s / 4) * C::REG_BYTES + (s % 4) * 32;
                    mma_ss<FP8>(tS, smem_desc_kmajor(q_base + off, 128), smem_desc_kmajor(k_base + off, 128), C::IDESC,
                                s > 0 ? 1u : 0u);
                }
                tc_commit(smem_u32(bS));
                tc_commit(smem_u32(bKe + ks));
                if (!mbar_wait(smem_u32(bP), t & 1, abort_flag, p.status, SA_DEV_WAIT_P)) break;
                const int vs = t % C::VST;
                if (!mbar_wait(smem_u32(bVf + vs), (t / C::VST) & 1, abort_flag, p.status, SA_DEV_WAIT_KV)) break;
                tc_fence_after();
                const uint32_t v_base = smem_u32(sV + vs * C::V_BYTES);
                constexpr int STEPS_PER_CHUNK = 64 / C::UK;
#pragma unroll
                for (int s = 0; s < C::PV_STEPS; ++s) {
                    const uint32_t off = (s / STEPS_PER_CHUNK) * C::VCHUNK + (s % STEPS_PER_CHUNK) * 32;
                    mma_ts<FP8>(tO, tS + s * 8, smem_desc_kmajor(v_base + off, C::VROW), C::IDESC,
                                (t > 0 || s > 0) ? 1u : 0u);
                }
                tc_commit(smem_u32(bVe + vs));
            }
            tc_commit(smem_u32(bO));
            if (*abort_flag) {
                tc_commit(smem_u32(bDrain));
                mbar_drain(smem_u32(bDrain), 0);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- softmax + epilogue (warps 0-3)
        const int r = threadIdx.x;                                   // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t tS = tmem + lane_off + C::S_COL;
        const uint32_t tO = tmem + lane_off + C::O_COL;
        const int qpos = p.q_offset + m * 128 + r;
        const int qpos_min = p.q_offset + m * 128;
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
        bool ok = true, bad = false;
        for (int t = 0; t < T; ++t) {
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bS), t & 1, abort_flag, p.status, SA_DEV_WAIT_S));
            if (!ok) break;
            tc_fence_after();
            float x[128];
            {
                uint32_t u[128];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32 * c));
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 128; ++i) x[i] = __uint_as_float(u[i]);
            }
            int kb0, kb1;
            tile_keys(w, t, kb0, kb1, bad);
            const bool need_mask = (max(kb0, kb1) + 63 > qpos_min) || (max(kb0, kb1) + 63 >= p.kv_len);
            if (need_mask) {
                const int lim = min(qpos, p.kv_len - 1);            // visible keys: kpos <= lim
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const int kpos = (c < 64 ? kb0 : kb1 - 64) + c;
                    if (kpos > lim) x[c] = -INFINITY;
                }
            }
            float mx = x[0];
#pragma unroll
            for (int c = 1; c < 128; ++c) mx = fmaxf(mx, x[c]);
            const float m_new = fmaxf(m_run, mx * sl2);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = ex2_approx(m_run - m_use);
            const float bias = pbias - m_use;
            float rs = 0.f;
            if constexpr (FP8) {
                // 32 keys -> 8 columns of 4 e4m3 values (key 4c+i in byte i of column c)
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    uint32_t pk[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float* xc = x + ch * 32 + 4 * c;
                        const float p0 = ex2_approx(fmaf(xc[0], sl2, bias));
                        const float p1 = ex2_approx(fmaf(xc[1], sl2, bias));
                        const float p2 = ex2_approx(fmaf(xc[2], sl2, bias));
                        const float p3 = ex2_approx(fmaf(xc[3], sl2, bias));
                        rs += (p0 + p1) + (p2 + p3);
                        pk[c] = static_cast<uint32_t>(pack_e4m3x2(p0, p1)) |
                                (static_cast<uint32_t>(pack_e4m3x2(p2, p3)) << 16);
                    }
                    tmem_st8(tS + ch * 8, pk);
                }
            } else {
                // 32 keys -> 16 columns of 2 bf16 values (key 2c+i in half i of column c)
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    uint32_t pk[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const float p0 = ex2_approx(fmaf(x[ch * 32 + 2 * c], sl2, bias));
                        const float p1 = ex2_approx(fmaf(x[ch * 32 + 2 * c + 1], sl2, bias));
                        rs += p0 + p1;
                        pk[c] = pack_bf16x2(p0, p1);
                    }
                    tmem_st16(tS + ch * 16, pk);
                }
            }
            l_run = l_run * alpha + rs;
            m_run = m_new;
            if (t > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {     // O rescale (PV of tile t-1 is complete)
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t u[32];
                    tmem_ld32(tO + c * 32, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
                    tmem_st32(tO + c * 32, u);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(bP));
        }
        if (bad && r == 0 && p.status) atomicOr(p.status, SA_DEV_BAD_LIST);
        // ---------------------------------------------------------------- epilogue
        const bool have_o = __all_sync(0xffffffffu, ok && T > 0 &&
                                       mbar_wait(smem_u32(bO), 0, abort_flag, p.status, SA_DEV_WAIT_O));
        if (have_o) tc_fence_after();
        const float inv = (have_o && l_run > 0.f) ? out_scale / l_run : 0.f;
        const int qrow = m * 128 + r - p.q_front;
        const bool row_ok = qrow >= 0 && qrow < p.n_q;
        uint16_t* orow = reinterpret_cast<uint16_t*>(p.out) + static_cast<int64_t>(qrow) * p.o_row_stride +
                         static_cast<int64_t>(h) * p.o_head_stride;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
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
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps and launch
// ------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

int encode3d(CUtensorMap* map, bool fp8, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
             uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw, const char* what) {
    auto fn = encode_fn();
    if (!fn) return fail(SA_ERR_TMA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1_bytes, s2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(SA_ERR_TMA, "tensor map for %s: error %d (dims %llu %llu %llu strides %llu %llu)", what, (int)r,
                    (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                    (unsigned long long)s1_bytes, (unsigned long long)s2_bytes);
    return SA_OK;
}

template <bool FP8>
int launch_attn(const void* q, int64_t qrs, int64_t qhs, const void* k, int64_t krs, int64_t khs, const void* vt,
                int64_t vths, int64_t vtds, void* out, int64_t ors, int64_t ohs, int n_q, int H, int Hk, int D, int kv_len,
                int q_front, int q_offset, const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                int kv_block, const float* qsc, int qss, const float* ksc, int kss, const float* vsc, int vss,
                float softmax_scale, int32_t* status, cudaStream_t stream) {
    using C = Cfg<FP8>;
    const char* name = FP8 ? "sa_attn_fwd_fp8" : "sa_attn_fwd_bf16";
    if (D != 128) return fail(SA_ERR_UNSUPPORTED, "%s: head_dim %d (only 128)", name, D);
    if (n_q < 0 || H <= 0 || Hk <= 0 || H % Hk || kv_len <= 0 || q_front < 0 || q_front >= 128 || q_offset < 0)
        return fail(SA_ERR_ARG, "%s: bad sizes", name);
    if (counts && (!lists || (kv_block != 64 && kv_block != 128) || list_stride < 1))
        return fail(SA_ERR_ARG, "%s: block lists need lists, kv_block 64|128", name);
    if (counts && q_block != 128) return fail(SA_ERR_UNSUPPORTED, "%s: q_block %d (only 128)", name, q_block);
    if (!q || !k || !vt || !out) return fail(SA_ERR_ARG, "%s: null pointer", name);
    if (FP8 && (!qsc || !ksc || !vsc)) return fail(SA_ERR_ARG, "%s: null scale pointer", name);
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const int E = C::E;
    if (!a16(q) || !a16(k) || !a16(vt) || !a16(out) || (qrs * E) % 16 || (qhs * E) % 16 || (krs * E) % 16 ||
        (khs * E) % 16 || (vths * E) % 16 || (vtds * E) % 16 || (ors * 2) % 16 || (ohs * 2) % 16)
        return fail(SA_ERR_ALIGN, "%s: pointers must be 16-byte aligned and strides multiples of 16 bytes", name);
    if (n_q == 0) return SA_OK;
    const int n_tiles = (q_front + n_q + 127) / 128;
    CUtensorMap tmQ, tmK, tmV;
    int rc;
    const CUtensorMapSwizzle sw128 = CU_TENSOR_MAP_SWIZZLE_128B;
    if ((rc = encode3d(&tmQ, FP8, q, D, H, n_q > 0 ? n_q : 1, qhs * E, qrs * E, C::REG_ELEMS, 1, 128, sw128, "q"))) return rc;
    if ((rc = encode3d(&tmK, FP8, k, D, Hk, kv_len, khs * E, krs * E, C::REG_ELEMS, 1, 64, sw128, "k"))) return rc;
    if ((rc = encode3d(&tmV, FP8, vt, kv_len, D, Hk, vtds * E, vths * E, 64, 128, 1,
                       FP8 ? CU_TENSOR_MAP_SWIZZLE_64B : sw128, "v^T")))
        return rc;
    Params p;
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
    p.kv_block = counts ? kv_block : 128;
    p.q_scale = qsc;
    p.k_scale = ksc;
    p.v_scale = vsc;
    p.qss = qss;
    p.kss = kss;
    p.vss = vss;
    p.softmax_scale = softmax_scale;
    p.status = status;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
    }
    dim3 grid(n_tiles, H);
    attn_fwd_kernel<FP8><<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, p);
    return check_launch(name);
}

}  // namespace
}  // namespace sa

extern "C" int sa_attn_fwd_fp8(const uint8_t* q, int64_t q_row_stride, int64_t q_head_stride, const uint8_t* k,
                               int64_t k_row_stride, int64_t k_head_stride, const uint8_t* vt, int64_t vt_head_stride,
                               int64_t vt_d_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                               int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                               const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                               int kv_block, const float* q_scale, int q_scale_stride, const float* k_scale,
                               int k_scale_stride, const float* v_scale, int v_scale_stride, float softmax_scale,
                               int32_t* status, void* stream) {
    return sa::launch_attn<true>(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, vt, vt_head_stride,
                                 vt_d_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                 kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, q_scale,
                                 q_scale_stride, k_scale, k_scale_stride, v_scale, v_scale_stride, softmax_scale, status,
                                 static_cast<cudaStream_t>(stream));
}

extern "C" int sa_attn_fwd_bf16(const void* q, int64_t q_row_stride, int64_t q_head_stride, const void* k,
                                int64_t k_row_stride, int64_t k_head_stride, const void* vt, int64_t vt_head_stride,
                                int64_t vt_d_stride, void* out, int64_t o_row_stride, int64_t o_head_stride, int n_q,
                                int num_heads, int num_kv_heads, int head_dim, int kv_len, int q_front, int q_offset,
                                const int32_t* counts, const int32_t* lists, int64_t list_stride, int q_block,
                                int kv_block, float softmax_scale, int32_t* status, void* stream) {
    return sa::launch_attn<false>(q, q_row_stride, q_head_stride, k, k_row_stride, k_head_stride, vt, vt_head_stride,
                                  vt_d_stride, out, o_row_stride, o_head_stride, n_q, num_heads, num_kv_heads, head_dim,
                                  kv_len, q_front, q_offset, counts, lists, list_stride, q_block, kv_block, nullptr, 0,
                                  nullptr, 0, nullptr, 0, softmax_scale, status, static_cast<cudaStream_t>(stream));
}
