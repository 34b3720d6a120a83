// Pieces shared by the attention kernels: tile-walk constants, launch parameters, the block-list
// walker, and the host-side TMA descriptor encoder.
#pragma once
#include <cudaTypedefs.h>

#include <climits>
#include <mutex>

#include "sa_common.cuh"

namespace sa {

// Launch parameters of the attention kernels (device pointers, sizes, strides).
struct Params {
    const int32_t* counts;
    const int32_t* lists;
    int64_t list_stride;
    void* out;
    int64_t o_row_stride, o_head_stride;
    int n_q, H, Hk, kv_len, q_front, q_offset, n_tiles, kv_block, q_block, list_rows_per_head;
    const float* q_scale;
    const float* k_scale;
    const float* v_scale;
    int qss, kss, vss;
    float softmax_scale;
    int32_t* status;
    // Split walks (splits > 1, 1D grid): units u = h * n_tiles + i (tile n_tiles-1-i of head h, the
    // launch order of the unsplit grid) below n_whole run whole, one CTA each; the n_tail units after
    // them (the partial last wave) run as `splits` CTAs each.  A tail unit whose walk has at least
    // split_min_steps steps is cut into `splits` contiguous step ranges, each writing its unnormalised
    // fp32 O, running max and row sum to `part`, the last range to finish combining them; a shorter
    // walk runs whole in its first CTA, which writes the output itself, and the others exit at once.
    int splits, split_min_steps, n_whole, n_tail;
    float* part;
    // Paged K/V (BF16 kernel; pages == nullptr: contiguous K/V): key j of the request is slot j % page
    // of cache page pages[j / page].  The tensor maps are then 4D {head_dim, Hk, page, num_pages}
    // with box_rows-row boxes (box_rows = min(page, 64)); kc / vc and the element strides serve the
    // plain loads of the one box that holds the last key when kv_len ends inside it.
    const int32_t* pages;
    int page, box_rows, num_pages;
    int box_shift, page_shift, last_box0;   // log2(box_rows); log2(page) or -1; first key of the
                                            // box holding the last key when kv_len ends inside it, or -1
    const uint16_t* kc;
    const uint16_t* vc;
    int64_t kv_ps, kv_rs, kv_hs;
};

// Paired-tile attention kernel (attn_pair.cu, FP8 only): two 128-row query tiles per CTA sharing
// each K/V stage.  Takes the tensor maps launch_attn built (64-row K/V boxes) and validated
// parameters.
template <bool FP8>
int launch_attn_pair(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV, const Params& p,
                     cudaStream_t stream, const char* name);

namespace {

constexpr int KEY_NONE = 1 << 30;   // key base of an absent tile: every key masked, TMA zero-fills
constexpr int KEY_END = -1;         // stage descriptor after the last tile of a walk
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LOG2_448 = 8.807354922057604f;


// Sequence of 64-key tiles one (head, 128-row query tile) walks, from the last block-list entry
// to the first like the reference (kai_fa_fp8_tma.py:149-162).  Modes: dense causal walk; one
// list of 64- or 128-key blocks for the whole tile; two lists of 64-key blocks, one per 64-row
// half of the tile (the BF16 path's 64-row query blocks), walked as their merged union with a
// per-tile mask of the halves that selected the block.  The producer and every softmax thread
// run the same walk; list heads are loaded one step ahead, so a step never waits on its load.
struct Walker {
    const int32_t* a;
    const int32_t* b;
    int ia, ib;          // list index of the cached head (counting down)
    int va, vb;          // cached list heads (-1 when exhausted)
    int dense_next;      // dense: next 64-key tile base, counting down
    int kvb;
    int blk_lim;         // block ids at or above this are invalid (their key base would overflow)
    int half;            // 128-key blocks: which half of the current block comes next (1 = upper)
    int mode;            // 0 dense, 1 one list, 2 two lists
    int remaining;       // steps left in this walk (a split takes a contiguous range of the steps)
    bool bad;

    __device__ __forceinline__ int load(const int32_t* p, int i) const { return i >= 0 ? __ldg(p + i) : -1; }

    // LIMIT: stop after `remaining` steps (a split walk); whole walks skip the count
    template <bool LIMIT = false>
    __device__ __forceinline__ bool next(int& kbase, uint32_t& rowmask) {
        rowmask = 3u;
        if constexpr (LIMIT) {
            if (remaining <= 0) return false;
            --remaining;
        }
        if (mode == 0) {
            if (dense_next < 0) return false;
            kbase = dense_next;
            dense_next -= 64;
            return true;
        }
        if (mode == 1) {
            if (ia < 0) return false;
            const int blk = va;
            if (blk < 0 || blk >= blk_lim) {
                bad = true;
                kbase = KEY_NONE;
            } else {
                kbase = blk * kvb + (kvb == 128 ? half * 64 : 0);
            }
            if (kvb == 128 && half == 1) {
                half = 0;
            } else {
                half = 1;
                --ia;
                va = load(a, ia);
            }
            return true;
        }
        if (va < 0 && vb < 0) return false;
        const int blk = max(va, vb);
        rowmask = (va == blk ? 1u : 0u) | (vb == blk ? 2u : 0u);
        if (va == blk) { --ia; va = load(a, ia); }
        if (vb == blk) { --ib; vb = load(b, ib); }
        if (blk >= KEY_NONE / 64) {
            bad = true;
            kbase = KEY_NONE;
        } else {
            kbase = blk * 64;
        }
        return true;
    }
};

// Steps of the whole walk of (head h, tile m) in modes 0 and 1 (64-key tiles); -1 in mode 2.
__device__ __forceinline__ int walk_steps(const Params& p, int h, int m) {
    if (!p.counts) {
        const int keys = min(p.q_offset + (m + 1) * 128, p.kv_len);
        return keys > 0 ? (keys + 63) / 64 : 0;
    }
    if (p.q_block != 128) return -1;
    const int64_t row = static_cast<int64_t>(h) * p.list_rows_per_head + m;
    return max(__ldg(p.counts + row), 0) * (p.kv_block == 128 ? 2 : 1);
}

// Step range [begin, end) of split s for a walk of `steps` steps (the whole walk when the unit is
// not split: splits == 1, mode 2, or fewer than split_min_steps steps; empty for s > 0 then).
__device__ __forceinline__ void split_range(const Params& p, int steps, int s, int& begin, int& end) {
    if (p.splits <= 1 || steps < p.split_min_steps) {
        begin = 0;
        end = s == 0 ? INT_MAX : 0;
        return;
    }
    begin = static_cast<int>(static_cast<int64_t>(steps) * s / p.splits);
    end = static_cast<int>(static_cast<int64_t>(steps) * (s + 1) / p.splits);
}

__device__ __forceinline__ Walker make_walker(const Params& p, int h, int m, int skip = 0, int take = INT_MAX) {
    Walker w;
    w.remaining = take;
    w.bad = false;
    w.kvb = p.kv_block;
    w.blk_lim = KEY_NONE / p.kv_block;
    w.half = 1;
    w.a = w.b = nullptr;
    w.ia = w.ib = -1;
    w.va = w.vb = -1;
    w.dense_next = -1;
    if (!p.counts) {
        w.mode = 0;
        const int last = p.q_offset + (m + 1) * 128;              // one past the tile's last position
        const int keys = min(last, p.kv_len);
        w.dense_next = keys > 0 ? ((keys + 63) / 64 - 1) * 64 : -1;
        w.dense_next -= 64 * skip;
    } else if (p.q_block == 128) {
        w.mode = 1;
        const int64_t row = static_cast<int64_t>(h) * p.list_rows_per_head + m;
        w.a = p.lists + row * p.list_stride;
        w.ia = max(__ldg(p.counts + row), 0) - 1;
        if (p.kv_block == 128) {              // two 64-key steps per entry, upper half first
            w.ia -= skip / 2;
            w.half = (skip & 1) ? 0 : 1;
        } else {
            w.ia -= skip;
        }
        w.va = w.load(w.a, w.ia);
    } else {
        w.mode = 2;
        const int r0 = 2 * m, r1 = 2 * m + 1;
        const int64_t row0 = static_cast<int64_t>(h) * p.list_rows_per_head + r0;
        w.a = p.lists + row0 * p.list_stride;
        w.ia = max(__ldg(p.counts + row0), 0) - 1;
        if (r1 < p.list_rows_per_head) {
            w.b = p.lists + (row0 + 1) * p.list_stride;
            w.ib = max(__ldg(p.counts + row0 + 1), 0) - 1;
        }
        w.va = w.load(w.a, w.ia);
        w.vb = w.b ? w.load(w.b, w.ib) : -1;
        if (w.va < -1 || w.vb < -1) {   // negative entries: treat the list as exhausted
            w.bad = true;
            w.va = max(w.va, -1);
            w.vb = max(w.vb, -1);
        }
    }
    return w;
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps
// ------------------------------------------------------------------------------------------------
inline int encode_nd(CUtensorMap* map, bool fp8, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle sw, const char* what) {
    auto fn = encode_fn();
    if (!fn) return fail(SA_ERR_TMA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    CUresult r = fn(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank,
                    const_cast<void*>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SA_ERR_TMA, "tensor map for %s: error %d", what, (int)r);
    return SA_OK;
}

inline int encode3d(CUtensorMap* map, bool fp8, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
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

}  // namespace
}  // namespace sa
