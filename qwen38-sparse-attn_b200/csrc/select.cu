// Kernel (b): dynamic block selection, two launches over a caller-provided workspace.
//
// (b1) score_kernel - logits[h*MB + m][j] = (qm[m, h] . km[h / g, j]) * scale for every causal key
//      block j <= qblk0 + m (sparse_prefill.py:68-74; fp32 like the reference's einsum).  A CTA
//      computes 64 rows (q block, query head pairs of one kv head) x 128 key blocks; each thread an
//      8 x 4 register tile; head_dim is staged through shared memory in 32-wide chunks with
//      cp.async, double buffered, rows padded to 36 floats so that no load conflicts.  Key blocks
//      at or beyond nb_km are scored as zero vectors (the driver's zero padding,
//      sparse_prefill.py:219-221).
// (b2) select_kernel - one warp per output row (per query head or per kv head x q block, or per
//      query head x pair of q blocks), the logits row in registers (lane l holds blocks l, l+32,..):
//      softmax over the causal blocks (fp32, like torch.softmax); tau selection without a sort:
//      the reference keeps the shortest prefix of the probabilities sorted in descending order
//      whose float64-accumulated sum, rounded to fp32, reaches fp32(tau) (sparse_prefill.py:75-77).
//      That prefix is {p > v*} plus the first ties of value v* in ascending block order, where v*
//      is the largest probability whose "mass of all p >= v*" reaches tau; v* is found by
//      bisection on the fp32 bit pattern (probabilities are >= 0, so integer order is value order)
//      with float64 sums.  The diagonal and the sink block are forced per q block before any union
//      (sparse_prefill.py:78-84, :223), then the row is emitted as count / ascending list / 0-1
//      mask.  Rows longer than 2048 blocks take a shared-memory path with the same arithmetic.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "sa_common.cuh"

namespace sa {
namespace {

// ------------------------------------------------------------------------------------------------
// (b1) scores
// ------------------------------------------------------------------------------------------------
constexpr int SC_ROWS = 64, SC_COLS = 128, SC_DC = 32, SC_PAD = 36, SC_THREADS = 256;
constexpr int SC_SMEM = 2 * (SC_ROWS + SC_COLS) * SC_PAD * 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

__global__ void __launch_bounds__(SC_THREADS, 2) score_kernel(
    const float* __restrict__ qm, int64_t qbs, int64_t qhs, const float* __restrict__ km, int64_t khs, int64_t kbs,
    int nb_km, int H, int Hk, int D, int MB, int nb_total, int qblk0, float scale, float* __restrict__ logits,
    int64_t lrs) {
    extern __shared__ __align__(16) float sc_smem[];
    const int g = H / Hk;
    const int hk = blockIdx.z;
    const int R = MB * g;                                         // rows of this kv head: r = m*g + i
    const int r0 = blockIdx.y * SC_ROWS, j0 = blockIdx.x * SC_COLS;
    const int m_last = min(R - 1, r0 + SC_ROWS - 1) / g;
    if (j0 > qblk0 + m_last || j0 >= nb_total) return;           // every block of the tile is in the future
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float* sQ = sc_smem;                                          // [2][SC_ROWS][SC_PAD]
    float* sK = sc_smem + 2 * SC_ROWS * SC_PAD;                   // [2][SC_COLS][SC_PAD]

    // this thread's copies: 2 float4 of the Q tile, 4 of the K tile per chunk
    const float* qsrc[2];
    bool qok[2];
    uint32_t qdst[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int idx = tid + u * SC_THREADS, row = idx >> 3, c4 = idx & 7;
        const int r = r0 + row;
        qok[u] = r < R;
        const int m = qok[u] ? r / g : 0, i = qok[u] ? r - m * g : 0;
        qsrc[u] = qm + static_cast<int64_t>(m) * qbs + static_cast<int64_t>(hk * g + i) * qhs + c4 * 4;
        qdst[u] = smem_u32(sQ + row * SC_PAD + c4 * 4);
    }
    const float* ksrc[4];
    bool kok[4];
    uint32_t kdst[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int idx = tid + u * SC_THREADS, col = idx >> 3, c4 = idx & 7;
        const int j = j0 + col;
        kok[u] = j < nb_km && j < nb_total;
        ksrc[u] = km + static_cast<int64_t>(hk) * khs + static_cast<int64_t>(kok[u] ? j : 0) * kbs + c4 * 4;
        kdst[u] = smem_u32(sK + col * SC_PAD + c4 * 4);
    }
    auto load_chunk = [&](int buf, int d0) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
            cp_async16(qdst[u] + buf * SC_ROWS * SC_PAD * 4, qok[u] ? qsrc[u] + d0 : qm, qok[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            cp_async16(kdst[u] + buf * SC_COLS * SC_PAD * 4, kok[u] ? ksrc[u] + d0 : km, kok[u]);
        cp_async_commit();
    };

    float acc[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
    const int nch = D / SC_DC;
    load_chunk(0, 0);
    for (int ch = 0; ch < nch; ++ch) {
        if (ch + 1 < nch) {
            load_chunk((ch + 1) & 1, (ch + 1) * SC_DC);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float* q = sQ + (ch & 1) * SC_ROWS * SC_PAD + warp * 8 * SC_PAD;     // rows 8w.. (broadcast)
        const float* k = sK + (ch & 1) * SC_COLS * SC_PAD + lane * SC_PAD;          // cols lane + 32c
#pragma unroll
        for (int dd = 0; dd < SC_DC; dd += 4) {
            float4 qa[8], kb[4];
#pragma unroll
            for (int a = 0; a < 8; ++a) qa[a] = *reinterpret_cast<const float4*>(q + a * SC_PAD + dd);
#pragma unroll
            for (int c = 0; c < 4; ++c) kb[c] = *reinterpret_cast<const float4*>(k + c * 32 * SC_PAD + dd);
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    acc[a][c] = fmaf(qa[a].x, kb[c].x, acc[a][c]);
                    acc[a][c] = fmaf(qa[a].y, kb[c].y, acc[a][c]);
                    acc[a][c] = fmaf(qa[a].z, kb[c].z, acc[a][c]);
                    acc[a][c] = fmaf(qa[a].w, kb[c].w, acc[a][c]);
                }
        }
        __syncthreads();                                          // buffer ch&1 is refilled at ch+2
    }
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int r = r0 + warp * 8 + a;
        if (r >= R) break;
        const int m = r / g, i = r - m * g;
        float* out = logits + static_cast<int64_t>((hk * g + i) * MB + m) * lrs;
        const int lim = min(nb_total - 1, qblk0 + m);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int j = j0 + lane + 32 * c;
            if (j <= lim) out[j] = acc[a][c] * scale;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// (b2) selection
// ------------------------------------------------------------------------------------------------
constexpr int SEL_WARPS = 8;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr int SEL_THREADS = SEL_WARPS * 32;
constexpr int SEL_MAX_NPL = 64;   // rows up to 2048 blocks in registers (one warp up to 1024, a warp pair above)

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Number of ties (in ascending block order) that must be kept: ties of value vstar are added to
// `above` one at a time until the fp32-rounded float64 mass reaches tau.
__device__ __forceinline__ int ties_needed(double above, float vstar, int ties, float tau_f) {
    int kt = ties;
    double acc = above;
    for (int k = 1; k <= ties; ++k) {
        acc += static_cast<double>(vstar);
        if (static_cast<float>(acc) >= tau_f) { kt = k; break; }
    }
    return kt;
}

// Register path: selects within one row of nbc <= 32*NPL blocks; returns the kept flags of this
// lane's blocks (bit c <-> block lane + 32c).
// L is a global workspace row (read through the read-only cache) or, with SMEM, a shared-memory row.
template <int NPL, bool SMEM = false>
__device__ uint64_t select_row_regs(const float* __restrict__ L, int nbc, float tau_f, int lane) {
    constexpr bool PRE = NPL <= 16;                               // keep float64 copies in registers
    float p[NPL];
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const int j = lane + 32 * c;
        p[c] = j < nbc ? (SMEM ? L[j] : __ldg(L + j)) : -INFINITY;
    }
    float mx = p[0];
#pragma unroll
    for (int c = 1; c < NPL; ++c) mx = fmaxf(mx, p[c]);
    mx = warp_max_f(mx);
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        p[c] = (lane + 32 * c < nbc) ? expf(p[c] - mx) : 0.f;
        s += p[c];
    }
    s = warp_sum_f(s);
    double pd[PRE ? NPL : 1];
    double t0 = 0.0, t1 = 0.0;
    float pmax = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool valid = lane + 32 * c < nbc;
        p[c] = valid ? __fdiv_rn(p[c], s) : -1.f;                 // -1: not a block of this row
        const double d = valid ? static_cast<double>(p[c]) : 0.0;
        if constexpr (PRE) pd[c] = d;
        if (c & 1) t1 += d; else t0 += d;
        pmax = fmaxf(pmax, p[c]);
    }
    const double tot = warp_sum_d(t0 + t1);
    uint64_t keep = 0;
    if (!(static_cast<float>(tot) >= tau_f)) {                   // tau never reached: every causal block
#pragma unroll
        for (int c = 0; c < NPL; ++c)
            if (lane + 32 * c < nbc) keep |= 1ull << c;
        return keep;
    }
    // largest v (bit pattern) with fp32(sum_{p >= v} p in float64) >= tau: pred(lo) true, pred(hi)
    // false; v* <= max p, so the search starts below max p's successor.
    auto pred64 = [&](uint32_t bits) -> bool {
        const float v = __uint_as_float(bits);
        double m0 = 0.0, m1 = 0.0, m2 = 0.0, m3 = 0.0;
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            double d;
            if constexpr (PRE) d = (p[c] >= v) ? pd[c] : 0.0;
            else d = (p[c] >= v) ? static_cast<double>(p[c]) : 0.0;
            if ((c & 3) == 0) m0 += d;
            else if ((c & 3) == 1) m1 += d;
            else if ((c & 3) == 2) m2 += d;
            else m3 += d;
        }
        return static_cast<float>(warp_sum_d((m0 + m1) + (m2 + m3))) >= tau_f;
    };
    const uint32_t top = __float_as_uint(warp_max_f(pmax)) + 1u;
    // The search itself sums in fp32 (shorter dependency chains, half the shuffles); its boundary
    // is then checked with the float64 predicate, and searched again in float64 in the rare rows
    // where the two disagree there (a mass within fp32 rounding of tau), so the result is the
    // float64 one exactly.
    uint32_t lo = 0u, hi = top;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        const float v = __uint_as_float(mid);
        float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            const float d = (p[c] >= v) ? p[c] : 0.f;
            if ((c & 3) == 0) m0 += d;
            else if ((c & 3) == 1) m1 += d;
            else if ((c & 3) == 2) m2 += d;
            else m3 += d;
        }
        if (warp_sum_f((m0 + m1) + (m2 + m3)) >= tau_f) lo = mid; else hi = mid;
    }
    if (!(pred64(lo) && (hi == top || !pred64(hi)))) {
        lo = 0u;
        hi = top;
        while (hi - lo > 1u) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            if (pred64(mid)) lo = mid; else hi = mid;
        }
    }
    const float vstar = __uint_as_float(lo);
    double above = 0.0;
    int ties = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        above += p[c] > vstar ? static_cast<double>(p[c]) : 0.0;
        ties += (p[c] == vstar);
    }
    above = warp_sum_d(above);
    ties = warp_sum_i(ties);
    const int kt = ties_needed(above, vstar, ties, tau_f);
    int seen = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool tie = p[c] == vstar;
        const uint32_t tb = __ballot_sync(0xffffffffu, tie);
        const int rank = seen + __popc(tb & ((1u << lane) - 1u));
        if (p[c] > vstar || (tie && rank < kt)) keep |= 1ull << c;
        seen += __popc(tb);
    }
    return keep;
}

// Shared-memory path for rows longer than 32*SEL_MAX_NPL blocks: L (the workspace row) is
// overwritten with the probabilities; the selection is OR-ed into bits[] (shared memory).
__device__ void select_row_smem(float* L, int nbc, float tau_f, uint32_t* bits, int lane) {
    float mx = -INFINITY;
    for (int j = lane; j < nbc; j += 32) mx = fmaxf(mx, L[j]);
    mx = warp_max_f(mx);
    float s = 0.f;
    for (int j = lane; j < nbc; j += 32) {
        const float e = expf(L[j] - mx);
        L[j] = e;
        s += e;
    }
    s = warp_sum_f(s);
    double tot = 0.0;
    float pmax = 0.f;
    for (int j = lane; j < nbc; j += 32) {
        const float p = __fdiv_rn(L[j], s);
        L[j] = p;
        tot += static_cast<double>(p);
        pmax = fmaxf(pmax, p);
    }
    tot = warp_sum_d(tot);
    __syncwarp();
    if (!(static_cast<float>(tot) >= tau_f)) {
        for (int j = lane; j < nbc; j += 32) atomicOr(&bits[j >> 5], 1u << (j & 31));
        return;
    }
    uint32_t lo = 0u, hi = __float_as_uint(warp_max_f(pmax)) + 1u;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        const float v = __uint_as_float(mid);
        double m = 0.0;
        for (int j = lane; j < nbc; j += 32) {
            const float p = L[j];
            if (p >= v) m += static_cast<double>(p);
        }
        m = warp_sum_d(m);
        if (static_cast<float>(m) >= tau_f) lo = mid; else hi = mid;
    }
    const float vstar = __uint_as_float(lo);
    double above = 0.0;
    int ties = 0;
    for (int j = lane; j < nbc; j += 32) {
        const float p = L[j];
        if (p > vstar) above += static_cast<double>(p);
        ties += (p == vstar);
    }
    above = warp_sum_d(above);
    ties = warp_sum_i(ties);
    const int kt = ties_needed(above, vstar, ties, tau_f);
    int seen = 0;
    for (int base = 0; base < nbc; base += 32) {
        const int j = base + lane;
        const float p = j < nbc ? L[j] : -1.f;
        const bool tie = (j < nbc) && (p == vstar);
        const uint32_t tb = __ballot_sync(0xffffffffu, tie);
        const int rank = seen + __popc(tb & ((1u << lane) - 1u));
        const bool keep = (j < nbc) && (p > vstar || (tie && rank < kt));
        const uint32_t kb = __ballot_sync(0xffffffffu, keep);
        if (lane == 0 && kb) atomicOr(&bits[base >> 5], kb);
        seen += __popc(tb);
    }
}

struct SelArgs {
    float* logits;
    int64_t lrs;
    int H, Hk, MB, nb_total, qblk0, mode;
    float tau_f;
    int32_t* counts;
    int32_t* lists;
    int64_t list_stride;
    uint8_t* masks;
};

// Output unit -> its first logits row (h0, m0) and the number of rows OR-ed into it: PER_HEAD one
// row; PAIR_UNION rows (h0, m0), (h0, m0 + 1); KV_UNION rows (h0 + i, m0) for the g heads.
__device__ __forceinline__ void unit_rows(const SelArgs& a, int unit, int& h0, int& m0, int& nrows) {
    const int g = a.H / a.Hk;
    if (a.mode == SA_SELECT_PER_HEAD) {
        h0 = unit / a.MB; m0 = unit - h0 * a.MB; nrows = 1;
    } else if (a.mode == SA_SELECT_PAIR_UNION) {
        const int half = a.MB / 2;
        h0 = unit / half; m0 = 2 * (unit - h0 * half); nrows = 2;
    } else {
        const int hk = unit / a.MB;
        m0 = unit - hk * a.MB; h0 = hk * g; nrows = g;
    }
}

template <int NPL>
__global__ void __launch_bounds__(SEL_THREADS) select_kernel(const SelArgs a, int units) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x * SEL_WARPS + warp;
    if (unit >= units) return;
    int h0, m0, nrows;
    unit_rows(a, unit, h0, m0, nrows);
    uint64_t keep = 0;
    for (int k = 0; k < nrows; ++k) {
        const int h = a.mode == SA_SELECT_KV_UNION ? h0 + k : h0;
        const int m = a.mode == SA_SELECT_PAIR_UNION ? m0 + k : m0;
        const int gi = a.qblk0 + m;
        const int nbc = min(gi + 1, a.nb_total);
        uint64_t kr = select_row_regs<NPL>(a.logits + static_cast<int64_t>(h * a.MB + m) * a.lrs, nbc, a.tau_f, lane);
        if (gi < a.nb_total && (gi & 31) == lane) kr |= 1ull << (gi >> 5);     // diagonal
        if (lane == 0) kr |= 1ull;                                             // sink
        keep |= kr;
    }
    int total = 0;
    const int nbw = (a.nb_total + 31) >> 5;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        if (c >= nbw) break;
        const bool on = (keep >> c) & 1ull;
        const uint32_t word = __ballot_sync(0xffffffffu, on);
        const int j = 32 * c + lane;
        if (a.lists && on)
            a.lists[static_cast<int64_t>(unit) * a.list_stride + total + __popc(word & ((1u << lane) - 1u))] = j;
        if (a.masks && j < a.nb_total) a.masks[static_cast<int64_t>(unit) * a.nb_total + j] = on ? 1 : 0;
        total += __popc(word);
    }
    if (a.counts && lane == 0) a.counts[unit] = total;
}

// Long rows: per-warp bit rows in shared memory ([SEL_WARPS][nbw] words).
__global__ void __launch_bounds__(SEL_THREADS) select_kernel_long(const SelArgs a, int units, int nbw) {
    extern __shared__ uint32_t sel_bits[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x * SEL_WARPS + warp;
    if (unit >= units) return;
    uint32_t* bits = sel_bits + warp * nbw;
    for (int w = lane; w < nbw; w += 32) bits[w] = 0u;
    __syncwarp();
    int h0, m0, nrows;
    unit_rows(a, unit, h0, m0, nrows);
    for (int k = 0; k < nrows; ++k) {
        const int h = a.mode == SA_SELECT_KV_UNION ? h0 + k : h0;
        const int m = a.mode == SA_SELECT_PAIR_UNION ? m0 + k : m0;
        const int gi = a.qblk0 + m;
        const int nbc = min(gi + 1, a.nb_total);
        select_row_smem(a.logits + static_cast<int64_t>(h * a.MB + m) * a.lrs, nbc, a.tau_f, bits, lane);
        __syncwarp();
        if (lane == 0) {
            if (gi < a.nb_total) atomicOr(&bits[gi >> 5], 1u << (gi & 31));
            atomicOr(&bits[0], 1u);
        }
        __syncwarp();
    }
    int total = 0;
    for (int w = 0; w < nbw; ++w) {
        const uint32_t word = bits[w];
        const int j = w * 32 + lane;
        const bool on = (word >> lane) & 1u;
        if (a.lists && on)
            a.lists[static_cast<int64_t>(unit) * a.list_stride + total + __popc(word & ((1u << lane) - 1u))] = j;
        if (a.masks && j < a.nb_total) a.masks[static_cast<int64_t>(unit) * a.nb_total + j] = on ? 1 : 0;
        total += __popc(word);
    }
    if (a.counts && lane == 0) a.counts[unit] = total;
}

// Rows of 1025..2048 blocks: two warps per output unit, each holding half of every row in
// registers (half s, lane l: blocks 1024 s + l + 32 c, c < 32).  Their partial sums, maxima and
// counts are combined through double-buffered shared-memory slots with one 64-thread named barrier
// per exchange, so both warps take the same decisions.  (One warp per 2048-block row needs 255
// registers, one CTA per SM, and code too large for the instruction cache.)
constexpr int SPLIT_NPL = 32;
constexpr int SPLIT_BLOCKS = 32 * SPLIT_NPL;                      // blocks per half

struct PairX {
    double* slot;                                                  // [2 buffers][2 halves]
    int bar;                                                       // named barrier id of the pair
    int half;
    int k;                                                         // exchange count
    // v: this warp's value (the same in every lane); returns both halves combined by op
    __device__ __forceinline__ double both(double v, bool take_max) {
        double* sl = slot + (k & 1) * 2;
        if ((threadIdx.x & 31) == 0) sl[half] = v;
        asm volatile("bar.sync %0, 64;" :: "r"(bar) : "memory");
        const double r = take_max ? fmax(sl[0], sl[1]) : sl[0] + sl[1];
        ++k;
        return r;
    }
    __device__ __forceinline__ double sum(double v) { return both(v, false); }
    __device__ __forceinline__ float maxf(float v) { return static_cast<float>(both(static_cast<double>(v), true)); }
};

__device__ uint32_t select_row_split(const float* __restrict__ L, int nbc, float tau_f, int lane, PairX& x) {
    constexpr int NPL = SPLIT_NPL;
    const int base = x.half * SPLIT_BLOCKS;
    float p[NPL];
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const int j = base + lane + 32 * c;
        p[c] = j < nbc ? __ldg(L + j) : -INFINITY;
    }
    float mx = p[0];
#pragma unroll
    for (int c = 1; c < NPL; ++c) mx = fmaxf(mx, p[c]);
    mx = x.maxf(warp_max_f(mx));
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        p[c] = (base + lane + 32 * c < nbc) ? expf(p[c] - mx) : 0.f;
        s += p[c];
    }
    s = static_cast<float>(x.sum(static_cast<double>(warp_sum_f(s))));
    double t0 = 0.0, t1 = 0.0;
    float pmax = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool valid = base + lane + 32 * c < nbc;
        p[c] = valid ? __fdiv_rn(p[c], s) : -1.f;                 // -1: not a block of this row
        const double d = valid ? static_cast<double>(p[c]) : 0.0;
        if (c & 1) t1 += d; else t0 += d;
        pmax = fmaxf(pmax, p[c]);
    }
    const double tot = x.sum(warp_sum_d(t0 + t1));
    uint32_t keep = 0;
    if (!(static_cast<float>(tot) >= tau_f)) {                   // tau never reached: every causal block
#pragma unroll
        for (int c = 0; c < NPL; ++c)
            if (base + lane + 32 * c < nbc) keep |= 1u << c;
        return keep;
    }
    auto pred64 = [&](uint32_t bits) -> bool {
        const float v = __uint_as_float(bits);
        double m0 = 0.0, m1 = 0.0, m2 = 0.0, m3 = 0.0;
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            const double d = (p[c] >= v) ? static_cast<double>(p[c]) : 0.0;
            if ((c & 3) == 0) m0 += d;
            else if ((c & 3) == 1) m1 += d;
            else if ((c & 3) == 2) m2 += d;
            else m3 += d;
        }
        return static_cast<float>(x.sum(warp_sum_d((m0 + m1) + (m2 + m3)))) >= tau_f;
    };
    const uint32_t top = __float_as_uint(x.maxf(warp_max_f(pmax))) + 1u;
    // fp32 search, float64 check of its boundary, float64 search again where they disagree (as in
    // select_row_regs)
    uint32_t lo = 0u, hi = top;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        const float v = __uint_as_float(mid);
        float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            const float d = (p[c] >= v) ? p[c] : 0.f;
            if ((c & 3) == 0) m0 += d;
            else if ((c & 3) == 1) m1 += d;
            else if ((c & 3) == 2) m2 += d;
            else m3 += d;
        }
        if (static_cast<float>(x.sum(static_cast<double>(warp_sum_f((m0 + m1) + (m2 + m3))))) >= tau_f) lo = mid;
        else hi = mid;
    }
    const bool lo_ok = pred64(lo);
    const bool hi_ok = hi == top ? false : pred64(hi);
    if (!(lo_ok && !hi_ok)) {
        lo = 0u;
        hi = top;
        while (hi - lo > 1u) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            if (pred64(mid)) lo = mid; else hi = mid;
        }
    }
    const float vstar = __uint_as_float(lo);
    double above = 0.0;
    int ties = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        above += p[c] > vstar ? static_cast<double>(p[c]) : 0.0;
        ties += (p[c] == vstar);
    }
    above = x.sum(warp_sum_d(above));
    ties = warp_sum_i(ties);
    const int ties_low = static_cast<int>(x.sum(x.half == 0 ? static_cast<double>(ties) : 0.0));
    const int ties_all = static_cast<int>(x.sum(static_cast<double>(ties)));
    const int kt = ties_needed(above, vstar, ties_all, tau_f);
    int seen = x.half ? ties_low : 0;                              // ties are kept in ascending block order
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool tie = p[c] == vstar;
        const uint32_t tb = __ballot_sync(0xffffffffu, tie);
        const int rank = seen + __popc(tb & ((1u << lane) - 1u));
        if (p[c] > vstar || (tie && rank < kt)) keep |= 1u << c;
        seen += __popc(tb);
    }
    return keep;
}

__global__ void __launch_bounds__(SEL_THREADS) select_kernel_split(const SelArgs a, int units) {
    __shared__ double xslot[SEL_WARPS / 2][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = warp >> 1, half = warp & 1;
    const int unit = blockIdx.x * (SEL_WARPS / 2) + pair;
    if (unit >= units) return;                                     // both warps of the pair leave
    PairX x{xslot[pair], 1 + pair, half, 0};
    int h0, m0, nrows;
    unit_rows(a, unit, h0, m0, nrows);
    uint32_t keep = 0;
    const int base = half * SPLIT_BLOCKS;
    for (int k = 0; k < nrows; ++k) {
        const int h = a.mode == SA_SELECT_KV_UNION ? h0 + k : h0;
        const int m = a.mode == SA_SELECT_PAIR_UNION ? m0 + k : m0;
        const int gi = a.qblk0 + m;
        const int nbc = min(gi + 1, a.nb_total);
        uint32_t kr = select_row_split(a.logits + static_cast<int64_t>(h * a.MB + m) * a.lrs, nbc, a.tau_f, lane, x);
        if (gi < a.nb_total && gi >= base && gi < base + SPLIT_BLOCKS && (gi & 31) == lane)
            kr |= 1u << ((gi - base) >> 5);                                  // diagonal
        if (half == 0 && lane == 0) kr |= 1u;                                // sink
        keep |= kr;
    }
    int cnt = 0;
#pragma unroll
    for (int c = 0; c < SPLIT_NPL; ++c) cnt += __popc(__ballot_sync(0xffffffffu, (keep >> c) & 1u));
    const int before = static_cast<int>(x.sum(half == 0 ? static_cast<double>(cnt) : 0.0));
    int total = half ? before : 0;
#pragma unroll
    for (int c = 0; c < SPLIT_NPL; ++c) {
        const int j = base + 32 * c + lane;
        if (base + 32 * c >= a.nb_total) break;
        const bool on = (keep >> c) & 1u;
        const uint32_t word = __ballot_sync(0xffffffffu, on);
        if (a.lists && on)
            a.lists[static_cast<int64_t>(unit) * a.list_stride + total + __popc(word & ((1u << lane) - 1u))] = j;
        if (a.masks && j < a.nb_total) a.masks[static_cast<int64_t>(unit) * a.nb_total + j] = on ? 1 : 0;
        total += __popc(word);
    }
    if (a.counts && half == 1 && lane == 0) a.counts[unit] = total;
}

// ------------------------------------------------------------------------------------------------
// (b') fused selection from the query rows: pooling, scores and tau selection in one launch
// ------------------------------------------------------------------------------------------------
// One CTA per (unit of QB consecutive query blocks, KV head): QB = 2 for the pair union, else 1; its
// R = QB * g rows are the unit's query blocks times the g query heads of the KV head (with per-head
// lists, the units a full wave of resident CTAs leaves over run as CTAs of a subset of the heads).
//  1. pool: mean of the query rows of each block (rows of the chunk only) for the g heads, 16-byte
//     loads along head_dim, rows summed in order per thread and the row groups combined in fixed
//     order; optionally every row read is also written as e4m3 (the FP8 path's q8, fused);
//  2. score: logits[r][j] = scale * qm[r] . km[j] for the unit's causal key blocks, fp32 register
//     tiles over key means staged by TMA, into shared memory (blocks at or past nb_km score 0: the
//     driver's zero padding);
//  3. select: one warp per row with select_row_lean (the decision rule of select_kernel), the
//     diagonal and the sink forced per query block, then the union of the mode and the list emission.
constexpr int FU_THREADS = 256;
constexpr int FU_MAX_FLOATS = 16384;                              // logits rows x padded blocks
// key-means staging of the scores: slices of FS_COLS columns of up to FS_ROWS key blocks, loaded by
// TMA in boxes of FS_BOX rows (32-byte swizzle) into FS_STAGES buffers
constexpr int FS_COLS = 8, FS_ROWS = 2 * FU_THREADS, FS_STAGES = 3, FS_BOX = 256;
constexpr int FS_SLICES = 128 / FS_COLS;
constexpr int FS_STAGE_FLOATS = FS_ROWS * FS_COLS;

// Selection of one row held in shared memory, for the one-pass kernel: the same decision rule as
// select_row_regs with cheaper fp32 arithmetic around it - exponentials as ex2.approx of the
// log2e-scaled difference, one rounded reciprocal instead of a division per block, and the bisection
// sums as multiply-adds by 0/1 - then the float64 check of the boundary and the float64 search where
// it disagrees, which fix the decision exactly for the probabilities computed here.  Those differ
// from torch's softmax by a few ulp, which moves a decision only for blocks whose cumulative mass is
// within ~1e-6 of tau (inside the 1e-4 band of the parity bar).  Bit c of the result <-> block
// lane + 32c.
template <int NPL>
__device__ uint32_t select_row_lean(const float* L, int nbc, float tau_f, int lane) {
    float p[NPL];
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const int j = lane + 32 * c;
        p[c] = j < nbc ? L[j] : -INFINITY;
    }
    float mx = p[0];
#pragma unroll
    for (int c = 1; c < NPL; ++c) mx = fmaxf(mx, p[c]);
    mx = warp_max_f(mx);
    const float off = -mx * LOG2E_F;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        p[c] = (lane + 32 * c < nbc) ? ex2_approx(fmaf(p[c], LOG2E_F, off)) : 0.f;
        if (c & 1) s1 += p[c]; else s0 += p[c];
    }
    const float rs = __frcp_rn(warp_sum_f(s0 + s1));
    double t0 = 0.0, t1 = 0.0;
    float pmax = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool valid = lane + 32 * c < nbc;
        p[c] = valid ? p[c] * rs : -1.f;                          // -1: not a block of this row
        const double d = valid ? static_cast<double>(p[c]) : 0.0;
        if (c & 1) t1 += d; else t0 += d;
        pmax = fmaxf(pmax, p[c]);
    }
    uint32_t keep = 0;
    if (!(static_cast<float>(warp_sum_d(t0 + t1)) >= tau_f)) {   // tau never reached: every causal block
#pragma unroll
        for (int c = 0; c < NPL; ++c)
            if (lane + 32 * c < nbc) keep |= 1u << c;
        return keep;
    }
    auto mass32 = [&](float v) -> float {
        float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
        for (int c = 0; c < NPL; c += 4) {
            m0 = fmaf(p[c] >= v ? 1.f : 0.f, p[c], m0);
            if (c + 1 < NPL) m1 = fmaf(p[c + 1] >= v ? 1.f : 0.f, p[c + 1], m1);
            if (c + 2 < NPL) m2 = fmaf(p[c + 2] >= v ? 1.f : 0.f, p[c + 2], m2);
            if (c + 3 < NPL) m3 = fmaf(p[c + 3] >= v ? 1.f : 0.f, p[c + 3], m3);
        }
        return warp_sum_f((m0 + m1) + (m2 + m3));
    };
    auto pred64 = [&](uint32_t bits) -> bool {
        const float v = __uint_as_float(bits);
        double m0 = 0.0, m1 = 0.0;
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            const double d = (p[c] >= v) ? static_cast<double>(p[c]) : 0.0;
            if (c & 1) m1 += d; else m0 += d;
        }
        return static_cast<float>(warp_sum_d(m0 + m1)) >= tau_f;
    };
    const uint32_t top = __float_as_uint(warp_max_f(pmax)) + 1u;
    uint32_t lo = 0u, hi = top;
    {   // a lower end closer than 0: blocks below v0 = (1 - tau) / (2 nbc) hold less than half of
        // 1 - tau, so mass(>= v0) reaches tau for a row summing to about 1 (checked once)
        const uint32_t v0 = __float_as_uint(0.5f * (1.f - tau_f) / static_cast<float>(nbc));
        if (v0 > 0u && v0 < hi && mass32(__uint_as_float(v0)) >= tau_f) lo = v0;
    }
    // The bisection keeps mass(lo) >= tau > mass(hi).  Once no probability lies strictly between
    // lo and hi, lo is one of the probabilities (else {p >= lo} = {p >= hi}) and the largest whose
    // mass reaches tau - what the remaining steps would converge to - so from the 8th step on the
    // search stops there (checked every 4th step).
    for (int it = 1; hi - lo > 1u; ++it) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        if (mass32(__uint_as_float(mid)) >= tau_f) lo = mid; else hi = mid;
        if (it >= 8 && (it & 3) == 0) {
            const uint32_t span = hi - lo - 1u;                   // bit patterns strictly inside
            bool inside = false;
#pragma unroll
            for (int c = 0; c < NPL; ++c) inside |= __float_as_uint(p[c]) - lo - 1u < span;
            if (!__any_sync(0xffffffffu, inside)) break;
        }
    }
    if (!(pred64(lo) && (hi == top || !pred64(hi)))) {
        lo = 0u;
        hi = top;
        while (hi - lo > 1u) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            if (pred64(mid)) lo = mid; else hi = mid;
        }
    }
    const float vstar = __uint_as_float(lo);
    double above = 0.0;
    int ties = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        above += p[c] > vstar ? static_cast<double>(p[c]) : 0.0;
        ties += (p[c] == vstar);
    }
    above = warp_sum_d(above);
    ties = warp_sum_i(ties);
    const int kt = ties_needed(above, vstar, ties, tau_f);
    int seen = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool tie = p[c] == vstar;
        const uint32_t tb = __ballot_sync(0xffffffffu, tie);
        const int rank = seen + __popc(tb & ((1u << lane) - 1u));
        if (p[c] > vstar || (tie && rank < kt)) keep |= 1u << c;
        seen += __popc(tb);
    }
    return keep;
}

struct FusedArgs {
    const uint16_t* q;
    int64_t qrs, qhs;
    int n, q_start, block, qblk0, MB;
    const float* km;
    int64_t khs, kbs;
    int nb_km, H, Hk, nb_total, nbp;                              // nbp: padded logits row length
    float scale, tau_f;
    int32_t* counts;
    int32_t* lists;
    int64_t list_stride;
    uint8_t* masks;
    uint8_t* q8;
    int64_t q8rs, q8hs;
    const float* inv_scale;
    int iss;
    int* status;                                                  // device status word (SA_DEV_WAIT_KM)
    int n_whole, split;                                           // units run whole; head subsets of the rest
};

__device__ __forceinline__ void emit_row(const FusedArgs& a, int64_t unit, uint32_t keep, int npl, int lane) {
    int total = 0;
    for (int c = 0; c < npl; ++c) {
        const bool on = (keep >> c) & 1u;
        const uint32_t word = __ballot_sync(0xffffffffu, on);
        const int j = 32 * c + lane;
        if (a.lists && on) a.lists[unit * a.list_stride + total + __popc(word & ((1u << lane) - 1u))] = j;
        if (a.masks && j < a.nb_total) a.masks[unit * a.nb_total + j] = on ? 1 : 0;
        total += __popc(word);
    }
    if (a.counts && lane == 0) a.counts[unit] = total;
}

// One slice of key means (columns sl*FS_COLS.., key blocks p0..) as `boxes` TMA boxes into the stage
// buffer at `dst`, completing on `bar`.  Out of line: only thread 0 runs it, and inlined its
// registers would count against the scores loop of every thread.
__device__ __noinline__ void issue_key_slice(const CUtensorMap* map, uint32_t bar, uint32_t dst, int sl, int p0, int boxes,
                                             int hk) {
    mbar_arrive_expect_tx(bar, boxes * FS_BOX * FS_COLS * 4);
    for (int k = 0; k < boxes; ++k) tma_load_3d(dst + k * FS_BOX * FS_COLS * 4, map, bar, sl * FS_COLS, p0 + k * FS_BOX, hk);
}

template <int NPL, int MODE>
__global__ void __launch_bounds__(FU_THREADS, NPL >= 32 ? 2 : 3)
select_fused_kernel(const FusedArgs a, const __grid_constant__ CUtensorMap km_map) {
    constexpr int QB = MODE == SA_SELECT_PAIR_UNION ? 2 : 1;
    extern __shared__ __align__(16) float fu_smem[];
    const int g = a.H / a.Hk;
    const int D = 128;
    // Work unit: (QB query blocks, KV head) in launch order u = hk * units_per_head + i.  The first
    // n_whole CTAs run one unit each; every later unit is run by `split` CTAs, each for gs = g /
    // split of its query heads (per-head lists only, where heads are independent), so that a partial
    // last wave of whole units becomes split times as many smaller CTAs.
    const int ub = blockIdx.x < a.n_whole ? blockIdx.x : a.n_whole + (blockIdx.x - a.n_whole) / a.split;
    const int sub = blockIdx.x < a.n_whole ? 0 : (blockIdx.x - a.n_whole) % a.split;
    const int gs = blockIdx.x < a.n_whole ? g : g / a.split;     // query heads of this CTA
    const int h0s = sub * gs;                                     // the first of them within the group
    const int R = QB * gs;                                        // rows of this CTA (layout below: QB * g)
    const int Rf = QB * g;
    float* qm = fu_smem;                                          // [rows rounded up to 8][D]
    float* logits = qm + ((Rf + 7) & ~7) * D;                     // [rows][nbp]; the pooling partials first
    uint32_t* keepw = reinterpret_cast<uint32_t*>(logits + Rf * a.nbp);  // [rows][32] (unions)
    float* kstage = reinterpret_cast<float*>(keepw + Rf * 32);   // [FS_STAGES][FS_ROWS][FS_COLS] key means,
    kstage += ((1024u - (smem_u32(kstage) & 1023u)) & 1023u) / 4;   // 1024-byte aligned (TMA swizzle atoms)
    __shared__ __align__(8) uint64_t kbar[FS_STAGES];            // stage s full (TMA bytes landed)
    __shared__ int abort_word;
    volatile int* abort_flag = &abort_word;
    const int units_per_head = a.MB / QB;
    const int hk = ub / units_per_head;
    const int m0 = (ub - hk * units_per_head) * QB;              // first query block of the unit
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {                                               // ordered before use by the pooling's barriers
        for (int b = 0; b < FS_STAGES; ++b) mbar_init(smem_u32(&kbar[b]), 1);
        *abort_flag = 0;
        fence_mbar_init();
        if (a.nb_km > 0) tma_prefetch_desc(&km_map);
    }

    // ---------------------------------------------------------------- 1. pool
    for (int i = R * D + tid; i < ((R + 7) & ~7) * D; i += FU_THREADS) qm[i] = 0.f;   // zero pad rows
    {
        const int per_row = gs * 16;                              // (head, 16-byte chunk) pairs of a row
        const int RG = FU_THREADS / per_row;                      // row groups
        const int ty = tid / per_row, tx = tid - ty * per_row;
        const int hl = tx >> 4, c = tx & 15;
        const int h = hk * g + h0s + hl;
        float* partial = logits;                                  // [RG - 1][per_row][8]
        const float inv = a.q8 ? __ldg(a.inv_scale + h * a.iss) : 0.f;
        for (int qb = 0; qb < QB; ++qb) {
            const int b = a.qblk0 + m0 + qb;
            const int lo = max(a.q_start, b * a.block) - a.q_start;
            const int hi = min(a.q_start + a.n, (b + 1) * a.block) - a.q_start;
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
            if (ty < RG) {
                const uint16_t* src = a.q + static_cast<int64_t>(h) * a.qhs + c * 8;
                uint8_t* dst = a.q8 ? a.q8 + static_cast<int64_t>(h) * a.q8hs + c * 8 : nullptr;
                constexpr int BATCH = 8;                          // 8 row loads in flight, summed in order
                for (int base = lo + ty; base < hi; base += BATCH * RG) {
                    uint4 v[BATCH];
#pragma unroll
                    for (int k = 0; k < BATCH; ++k) {
                        const int r = base + k * RG;
                        v[k] = r < hi ? ld_stream(src + static_cast<int64_t>(r) * a.qrs) : make_uint4(0u, 0u, 0u, 0u);
                    }
#pragma unroll
                    for (int k = 0; k < BATCH; ++k) {
                        const int r = base + k * RG;
                        if (r >= hi) break;
                        float f[8];
                        unpack8(v[k], f);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc[i] += f[i];
                        if (dst)
                            *reinterpret_cast<uint2*>(dst + static_cast<int64_t>(r) * a.q8rs) =
                                quant8(f, inv, SA_QUANT_MUL_BF16);
                    }
                }
                if (ty > 0) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) partial[((ty - 1) * per_row + tx) * 8 + i] = acc[i];
                }
            }
            __syncthreads();
            if (ty == 0) {
                for (int k = 1; k < RG; ++k) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] += partial[((k - 1) * per_row + tx) * 8 + i];
                }
                const float cnt = static_cast<float>(max(hi - lo, 1));
                float* o = qm + (qb * gs + hl) * D + c * 8;
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = hi > lo ? __fdiv_rn(acc[i], cnt) : 0.f;
            }
            __syncthreads();
        }
    }
    // the key means may come from the kernel launched just before (programmatic dependent launch)
    grid_dependency_wait();
    // ---------------------------------------------------------------- 2. scores
    // Register tiles: in each pass over up to FS_ROWS key blocks, thread t owns blocks p0 + t and
    // p0 + t + FU_THREADS and, per group of 8 query rows, their 8 x 2 dot products over head_dim,
    // accumulated as (even column, odd column) pairs with packed f32x2 FMAs and added at the end.
    // The pass's key-means rows stream through shared memory in slices of FS_COLS columns (one
    // 32-byte piece of each row), FS_STAGES deep: thread 0 issues the TMA boxes of a slice two
    // slices ahead (rows past nb_km arrive as zeros: the driver's zero padding).  The 32-byte
    // swizzle swaps row j's two 16-byte halves when bit 2 of j is set, so the 8 lanes of a
    // quarter-warp (rows j..j+7) read 8 distinct bank groups.  The query means are read as
    // shared-memory broadcasts.  Waits are bounded: on expiry the CTA records SA_DEV_WAIT_KM, waits
    // (bounded) for the boxes in flight and exits without writing the unit's rows.
    const int nb_max = min(a.qblk0 + m0 + QB, a.nb_total);       // causal blocks of the unit's last q block
    if (a.nb_km == 0) {                                           // no key means: every score is 0
        for (int i = tid; i < R * nb_max; i += FU_THREADS) logits[(i / nb_max) * a.nbp + i % nb_max] = 0.f;
    } else {
        const int R8 = (R + 7) & ~7;
        const int ja = tid, jb = tid + FU_THREADS;                // the thread's rows of a stage buffer
        const int ha = ((ja >> 2) & 1) * 4, hb = ((jb >> 2) & 1) * 4;   // where their columns 0-3 sit
        uint32_t issued = 0, used = 0;                            // slices issued (thread 0) / consumed
        auto issue = [&](int p0, int rows, int sl) {
            const uint32_t b = issued % FS_STAGES;
            issue_key_slice(&km_map, smem_u32(&kbar[b]), smem_u32(kstage + b * FS_STAGE_FLOATS), sl, p0,
                            (rows + FS_BOX - 1) / FS_BOX, hk);
            ++issued;
        };
        bool aborted = false;
        for (int r0 = 0; r0 < R8 && !aborted; r0 += 8) {
            for (int p0 = 0; p0 < nb_max; p0 += FS_ROWS) {
                const int rows = min(FS_ROWS, nb_max - p0);
                if (tid == 0) {
                    issue(p0, rows, 0);
                    issue(p0, rows, 1);
                }
                float2 acc[8][2];
#pragma unroll
                for (int r = 0; r < 8; ++r) acc[r][0] = acc[r][1] = make_float2(0.f, 0.f);
                for (int sl = 0; sl < FS_SLICES; ++sl) {
                    const uint32_t b = used % FS_STAGES;
                    mbar_wait(smem_u32(&kbar[b]), (used / FS_STAGES) & 1, abort_flag, a.status, SA_DEV_WAIT_KM);
                    __syncthreads();                              // all waited; slice sl - 1 consumed by all
                    if (*abort_flag) {                            // the same value for every thread
                        aborted = true;
                        break;
                    }
                    ++used;
                    if (tid == 0 && sl + 2 < FS_SLICES) issue(p0, rows, sl + 2);   // into slice sl - 1's buffer
                    const float* kb = kstage + b * FS_STAGE_FLOATS;
                    const float4 a0 = *reinterpret_cast<const float4*>(kb + ja * FS_COLS + ha);
                    const float4 a1 = *reinterpret_cast<const float4*>(kb + ja * FS_COLS + (ha ^ 4));
                    const float4 b0 = *reinterpret_cast<const float4*>(kb + jb * FS_COLS + hb);
                    const float4 b1 = *reinterpret_cast<const float4*>(kb + jb * FS_COLS + (hb ^ 4));
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        if (r0 + r >= R) break;                   // padding rows (CTA-uniform)
                        const float4 q0 = *reinterpret_cast<const float4*>(qm + (r0 + r) * D + sl * FS_COLS);
                        const float4 q1 = *reinterpret_cast<const float4*>(qm + (r0 + r) * D + sl * FS_COLS + 4);
                        acc[r][0] = ffma2(make_float2(q0.x, q0.y), make_float2(a0.x, a0.y), acc[r][0]);
                        acc[r][1] = ffma2(make_float2(q0.x, q0.y), make_float2(b0.x, b0.y), acc[r][1]);
                        acc[r][0] = ffma2(make_float2(q0.z, q0.w), make_float2(a0.z, a0.w), acc[r][0]);
                        acc[r][1] = ffma2(make_float2(q0.z, q0.w), make_float2(b0.z, b0.w), acc[r][1]);
                        acc[r][0] = ffma2(make_float2(q1.x, q1.y), make_float2(a1.x, a1.y), acc[r][0]);
                        acc[r][1] = ffma2(make_float2(q1.x, q1.y), make_float2(b1.x, b1.y), acc[r][1]);
                        acc[r][0] = ffma2(make_float2(q1.z, q1.w), make_float2(a1.z, a1.w), acc[r][0]);
                        acc[r][1] = ffma2(make_float2(q1.z, q1.w), make_float2(b1.z, b1.w), acc[r][1]);
                    }
                }
                if (aborted) break;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    if (r0 + r >= R) break;
                    float* out = logits + (r0 + r) * a.nbp + p0;
                    if (ja < rows) out[ja] = (p0 + ja < a.nb_km) ? (acc[r][0].x + acc[r][0].y) * a.scale : 0.f;
                    if (jb < rows) out[jb] = (p0 + jb < a.nb_km) ? (acc[r][1].x + acc[r][1].y) * a.scale : 0.f;
                }
                __syncthreads();                                  // the next pass refills the stage buffers
            }
        }
        if (aborted) {                                            // boxes still in flight land before exit
            if (tid == 0)
                for (uint32_t sl = used; sl < issued; ++sl) mbar_drain(smem_u32(&kbar[sl % FS_STAGES]), (sl / FS_STAGES) & 1);
            return;
        }
    }
    __syncthreads();
    // ---------------------------------------------------------------- 3. select
    const int npl_used = (a.nb_total + 31) >> 5;
    for (int r = warp; r < R; r += FU_THREADS / 32) {
        const int qb = r / gs, i = r - qb * gs;
        const int m = m0 + qb;
        const int gi = a.qblk0 + m;
        const int nbc = min(gi + 1, a.nb_total);
        uint32_t keep = select_row_lean<NPL>(logits + r * a.nbp, nbc, a.tau_f, lane);
        if (gi < a.nb_total && (gi & 31) == lane) keep |= 1u << (gi >> 5);     // diagonal
        if (lane == 0) keep |= 1u;                                             // sink
        if (MODE == SA_SELECT_PER_HEAD)
            emit_row(a, static_cast<int64_t>(hk * g + h0s + i) * a.MB + m, keep, npl_used, lane);
        else
            keepw[r * 32 + lane] = keep;
    }
    if (MODE == SA_SELECT_PER_HEAD) return;
    __syncthreads();
    if (MODE == SA_SELECT_KV_UNION) {                             // one row per (KV head, q block)
        if (warp == 0) {
            uint32_t keep = 0;
            for (int i = 0; i < g; ++i) keep |= keepw[i * 32 + lane];
            emit_row(a, static_cast<int64_t>(hk) * a.MB + m0, keep, npl_used, lane);
        }
    } else {                                                      // one row per (query head, q-block pair)
        for (int i = warp; i < g; i += FU_THREADS / 32) {
            const uint32_t keep = keepw[i * 32 + lane] | keepw[(g + i) * 32 + lane];
            emit_row(a, static_cast<int64_t>(hk * g + i) * (a.MB / 2) + m0 / 2, keep, npl_used, lane);
        }
    }
}

// Head-subset tail units of sa_select_q: on unless the environment sets SA_SELECT_SPLIT=0.
bool select_split_enabled() {
    const char* e = getenv("SA_SELECT_SPLIT");
    return !(e && e[0] == '0' && e[1] == 0);
}

int64_t logits_row_stride(int nb_total) { return (static_cast<int64_t>(nb_total) + 31) / 32 * 32; }

// Scratch of sa_select_static: one buffer per device, part of the module image, so that entry
// point needs no allocation.  Every call uses all of it that it needs, hence calls overlapping on a
// device race.
constexpr size_t STATIC_SCRATCH_BYTES = size_t(40) << 20;
static __device__ __align__(256) unsigned char g_select_scratch[STATIC_SCRATCH_BYTES];

}  // namespace
}  // namespace sa

using namespace sa;

extern "C" size_t sa_select_workspace_bytes(int num_heads, int MB, int nb_total) {
    if (num_heads <= 0 || MB <= 0 || nb_total <= 0) return 0;
    return static_cast<size_t>(num_heads) * MB * logits_row_stride(nb_total) * sizeof(float);
}

extern "C" int sa_select(const float* qm, int64_t qm_block_stride, int64_t qm_head_stride, const float* km,
                         int64_t km_head_stride, int64_t km_block_stride, int nb_km, int num_heads, int num_kv_heads,
                         int head_dim, int MB, int nb_total, int qblk0, float scale, float tau, int mode,
                         int32_t* counts, int32_t* lists, int64_t list_stride, uint8_t* masks, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || MB <= 0 || nb_total <= 0 || qblk0 < 0 ||
        nb_km < 0)
        return fail(SA_ERR_ARG, "sa_select: bad sizes");
    const int g = num_heads / num_kv_heads;
    if (head_dim <= 0 || head_dim % SC_DC) return fail(SA_ERR_UNSUPPORTED, "sa_select: head_dim %% %d", SC_DC);
    if (!qm || (!km && nb_km > 0)) return fail(SA_ERR_ARG, "sa_select: null pointer");
    if ((reinterpret_cast<uintptr_t>(km) & 15) || km_block_stride % 4 || km_head_stride % 4 ||
        (reinterpret_cast<uintptr_t>(qm) & 15) || qm_block_stride % 4 || qm_head_stride % 4)
        return fail(SA_ERR_ALIGN, "sa_select: qm and km must be 16-byte aligned with strides %% 4 == 0");
    if (mode < 0 || mode > 2) return fail(SA_ERR_ARG, "sa_select: bad mode");
    if (mode == SA_SELECT_PAIR_UNION && (MB % 2)) return fail(SA_ERR_ARG, "sa_select: pair union needs even MB");
    if (lists && list_stride < nb_total) return fail(SA_ERR_ARG, "sa_select: list_stride < nb_total");
    const size_t need = sa_select_workspace_bytes(num_heads, MB, nb_total);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
        return fail(SA_ERR_ARG, "sa_select: workspace of %zu bytes (16-byte aligned) needed", need);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* L = static_cast<float*>(workspace);
    const int64_t lrs = logits_row_stride(nb_total);

    cudaError_t e = cudaSuccess;
    {
        static PerContext attr;                                   // shared-memory opt-in, once per device context
        int dev = 0;
        void* ctx = nullptr;
        if (int rc = current_device_context("sa_select", &dev, &ctx)) return rc;
        std::lock_guard<std::mutex> lock(attr.mu);
        if (attr.ctx[dev] != ctx) {
            e = cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SC_SMEM);
            if (e != cudaSuccess) return fail(SA_ERR_CUDA, "sa_select: %s", cudaGetErrorString(e));
            attr.ctx[dev] = ctx;
        }
    }
    dim3 sgrid((nb_total + SC_COLS - 1) / SC_COLS, (MB * g + SC_ROWS - 1) / SC_ROWS, num_kv_heads);
    score_kernel<<<sgrid, SC_THREADS, SC_SMEM, s>>>(qm, qm_block_stride, qm_head_stride, km, km_head_stride,
                                                   km_block_stride, nb_km, num_heads, num_kv_heads, head_dim, MB,
                                                   nb_total, qblk0, scale, L, lrs);
    int rc = check_launch("score_kernel");
    if (rc) return rc;

    const SelArgs a{L, lrs, num_heads, num_kv_heads, MB, nb_total, qblk0, mode, static_cast<float>(tau),
                    counts, lists, list_stride, masks};
    const int units = (mode == SA_SELECT_PER_HEAD) ? num_heads * MB
                    : (mode == SA_SELECT_PAIR_UNION) ? num_heads * (MB / 2) : num_kv_heads * MB;
    const int blocks = (units + SEL_WARPS - 1) / SEL_WARPS;
    const int npl = (nb_total + 31) / 32;
    if (npl <= 4) select_kernel<4><<<blocks, SEL_THREADS, 0, s>>>(a, units);
    else if (npl <= 8) select_kernel<8><<<blocks, SEL_THREADS, 0, s>>>(a, units);
    else if (npl <= 16) select_kernel<16><<<blocks, SEL_THREADS, 0, s>>>(a, units);
    else if (npl <= 32) select_kernel<32><<<blocks, SEL_THREADS, 0, s>>>(a, units);
    else if (npl <= 2 * SPLIT_NPL) select_kernel_split<<<(units + SEL_WARPS / 2 - 1) / (SEL_WARPS / 2), SEL_THREADS, 0, s>>>(a, units);
    else {
        const size_t smem = static_cast<size_t>(SEL_WARPS) * npl * sizeof(uint32_t);
        if (smem > 227 * 1024) return fail(SA_ERR_UNSUPPORTED, "sa_select: %d key blocks", nb_total);
        if (smem > 48 * 1024) {
            e = cudaFuncSetAttribute(select_kernel_long, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return fail(SA_ERR_CUDA, "sa_select: %s", cudaGetErrorString(e));
        }
        select_kernel_long<<<blocks, SEL_THREADS, smem, s>>>(a, units, npl);
    }
    return check_launch("select_kernel");
}

extern "C" int sa_select_q(const void* q, int64_t q_row_stride, int64_t q_head_stride, int n, int q_start, int block,
                           int qblk0, int MB, const float* km, int64_t km_head_stride, int64_t km_block_stride,
                           int nb_km, int num_heads, int num_kv_heads, int head_dim, int nb_total, float scale,
                           float tau, int mode, int32_t* counts, int32_t* lists, int64_t list_stride, uint8_t* masks,
                           uint8_t* q8, int64_t q8_row_stride, int64_t q8_head_stride, const float* inv_scale,
                           int inv_scale_stride, int32_t* status, void* stream) {
    const char* name = "sa_select_q";
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || MB <= 0 || nb_total <= 0 || qblk0 < 0 ||
        nb_km < 0 || n < 0 || q_start < 0 || block <= 0)
        return fail(SA_ERR_ARG, "%s: bad sizes", name);
    if (mode < 0 || mode > 2) return fail(SA_ERR_ARG, "%s: bad mode", name);
    if (mode == SA_SELECT_PAIR_UNION && (MB % 2)) return fail(SA_ERR_ARG, "%s: pair union needs even MB", name);
    if (lists && list_stride < nb_total) return fail(SA_ERR_ARG, "%s: list_stride < nb_total", name);
    if (q_start < qblk0 * block || (n > 0 && q_start + n > (qblk0 + MB) * block))
        return fail(SA_ERR_ARG, "%s: query rows outside the query blocks", name);
    const int g = num_heads / num_kv_heads;
    const int QB = mode == SA_SELECT_PAIR_UNION ? 2 : 1;
    const int R = QB * g;
    const int npl = (nb_total + 31) / 32;
    const int nbp = npl * 32;
    // shapes the one-pass kernel serves; others take block means + sa_select
    if (head_dim != 128 || g > 16 || (16 * g) > FU_THREADS || npl > 32 || R * nbp > FU_MAX_FLOATS)
        return fail(SA_ERR_UNSUPPORTED, "%s: %d heads per KV head, %d key blocks, head_dim %d (use sa_select)", name, g,
                    nb_total, head_dim);
    if (!q || (!km && nb_km > 0) || (q8 && !inv_scale)) return fail(SA_ERR_ARG, "%s: null pointer", name);
    if (!aligned16(q) || q_row_stride % 8 || q_head_stride % 8 || !aligned16(km) || km_block_stride % 4 ||
        km_head_stride % 4 || (q8 && ((reinterpret_cast<uintptr_t>(q8) & 7) || q8_row_stride % 8 || q8_head_stride % 8)))
        return fail(SA_ERR_ALIGN, "%s: q and km 16-byte aligned, strides of 8 elements (q8: 8 bytes)", name);
    const int per_row = 16 * g, RG = FU_THREADS / per_row;
    // logits region: also holds the pooling partials, (FU_THREADS / (16 gs) - 1) x 16 gs x 8 floats
    // (below 2048) for a CTA of gs query heads
    const size_t smem = (static_cast<size_t>((R + 7) & ~7) * 128 + std::max<size_t>(static_cast<size_t>(R) * nbp,
                         std::max<size_t>(static_cast<size_t>(RG - 1) * per_row * 8, 2048)) + static_cast<size_t>(R) * 32 +
                         static_cast<size_t>(FS_STAGES) * FS_STAGE_FLOATS) * 4 + 1024;   // + stage alignment
    FusedArgs fa{static_cast<const uint16_t*>(q), q_row_stride, q_head_stride, n, q_start, block, qblk0, MB, km,
                 km_head_stride, km_block_stride, nb_km, num_heads, num_kv_heads, nb_total, nbp, scale,
                 static_cast<float>(tau), counts, lists, list_stride, masks, q8, q8_row_stride, q8_head_stride,
                 inv_scale, inv_scale_stride, status, 0, 1};
    // key means [Hk][nb_km][128] fp32 as a 3D tensor map: boxes of FS_COLS columns x FS_BOX key
    // blocks, rows past nb_km read as zeros
    CUtensorMap km_map;
    memset(&km_map, 0, sizeof(km_map));
    if (nb_km > 0) {
        auto fn = encode_fn();
        if (!fn) return fail(SA_ERR_TMA, "%s: cuTensorMapEncodeTiled unavailable", name);
        const cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(nb_km), static_cast<cuuint64_t>(num_kv_heads)};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(km_block_stride) * 4,
                                       static_cast<cuuint64_t>(km_head_stride) * 4};
        const cuuint32_t box[3] = {FS_COLS, FS_BOX, 1}, estr[3] = {1, 1, 1};
        const CUresult r = fn(&km_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(km), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(SA_ERR_TMA, "%s: tensor map for the key means: error %d", name, (int)r);
    }
    void (*kern)(const FusedArgs, const CUtensorMap) = nullptr;
#define SA_FUSED_PICK(NPL_)                                                                            \
    kern = mode == SA_SELECT_PER_HEAD ? select_fused_kernel<NPL_, SA_SELECT_PER_HEAD>                 \
         : mode == SA_SELECT_KV_UNION ? select_fused_kernel<NPL_, SA_SELECT_KV_UNION>                 \
                                      : select_fused_kernel<NPL_, SA_SELECT_PAIR_UNION>;
    if (npl <= 4) { SA_FUSED_PICK(4) }
    else if (npl <= 8) { SA_FUSED_PICK(8) }
    else if (npl <= 16) { SA_FUSED_PICK(16) }
    else { SA_FUSED_PICK(32) }
#undef SA_FUSED_PICK
    if (smem > 48 * 1024) {                                       // before the occupancy query below
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
    }
    // launched as a programmatic dependent of the previous kernel in the stream: the pooling of q
    // (written by earlier kernels) may overlap that kernel, whose outputs (the key means) are read
    // only after grid_dependency_wait
    // Units (QB query blocks, KV head) in launch order; with per-head lists a partial last wave of
    // resident CTAs is cut into head subsets (largest divisor of g whose CTAs still fit one wave), so
    // that the units left over after the full waves do not run one CTA each on a few SMs.
    const int units = (MB / QB) * num_kv_heads;
    fa.n_whole = units;
    if (mode == SA_SELECT_PER_HEAD && g > 1 && select_split_enabled()) {
        int per_sm = 0;
        cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FU_THREADS, smem);
        if (oe != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(oe));
        const int slots = per_sm * num_sms();
        const int rem = slots > 0 ? units % slots : 0;
        for (int d = g; d > 1 && rem > 0; --d)
            if (g % d == 0 && static_cast<int64_t>(rem) * d <= slots) {
                fa.n_whole = units - rem;
                fa.split = d;
                break;
            }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(fa.n_whole + (units - fa.n_whole) * fa.split);
    cfg.blockDim = dim3(FU_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, fa, km_map);
    if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
    return check_launch(name);
}

// Same selection as sa_select, on the static scratch buffer above instead of a caller workspace.
// The buffer's device address is looked up once per device (cudaGetSymbolAddress, with the caller's
// current device) on the first call made with that device current.
extern "C" int sa_select_static(const float* qm, int64_t qm_block_stride, int64_t qm_head_stride, const float* km,
                                int64_t km_head_stride, int64_t km_block_stride, int nb_km, int num_heads,
                                int num_kv_heads, int head_dim, int MB, int nb_total, int qblk0, float scale, float tau,
                                int mode, int32_t* counts, int32_t* lists, int64_t list_stride, uint8_t* masks,
                                void* stream) {
    // device address of the scratch array, looked up once per device and context: a new context
    // (after cudaDeviceReset) loads the module again, possibly at another address
    static PerContext scratch;
    int dev = 0;
    void* ctx = nullptr;
    if (int rc = current_device_context("sa_select_static", &dev, &ctx)) return rc;
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(scratch.mu);
        if (scratch.ctx[dev] != ctx) {
            void* addr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&addr, g_select_scratch);
            if (e != cudaSuccess)
                return fail(SA_ERR_CUDA, "sa_select_static: scratch address on device %d: %s", dev,
                            cudaGetErrorString(e));
            scratch.value[dev] = addr;
            scratch.ctx[dev] = ctx;
        }
        ws = scratch.value[dev];
    }
    const size_t need = sa_select_workspace_bytes(num_heads, MB, nb_total);
    if (need > STATIC_SCRATCH_BYTES)
        return fail(SA_ERR_UNSUPPORTED,
                    "sa_select_static: %d heads x %d q blocks x %d key blocks need %zu bytes of scratch, more than "
                    "the %zu-byte static buffer; call sa_select with a workspace instead",
                    num_heads, MB, nb_total, need, STATIC_SCRATCH_BYTES);
    return sa_select(qm, qm_block_stride, qm_head_stride, km, km_head_stride, km_block_stride, nb_km, num_heads,
                     num_kv_heads, head_dim, MB, nb_total, qblk0, scale, tau, mode, counts, lists, list_stride, masks,
                     ws, STATIC_SCRATCH_BYTES, stream);
}
