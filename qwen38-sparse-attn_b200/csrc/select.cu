// Kernel (b): fused dynamic block selection.
//
// One CTA per (kv head, q block) - or per (kv head, pair of q blocks) in pair-union mode - scores
// every causal key block against the pooled queries of all g query heads of that kv head, so each
// cached key-block mean is read once per CTA.  Then one warp per query head:
//   softmax over the causal blocks (fp32, like the reference's torch.softmax);
//   tau selection without a sort: the kept set of the reference - the shortest prefix of the
//   probabilities sorted in descending order whose float64-accumulated sum, rounded to fp32,
//   reaches fp32(tau) (sparse_prefill.py:75-77) - is the set of blocks with p > v* plus the
//   first k ties of value v*, where v* is the largest probability whose "mass of all p >= v*"
//   reaches tau.  v* is found by bisection on the fp32 bit pattern (probabilities are >= 0, so
//   integer order is value order) with float64 warp sums; ties are taken in ascending block order.
// The diagonal and the sink block are forced and future blocks cleared per q block before any
// union (sparse_prefill.py:78-84, :223), then the row is emitted as counts / ascending lists /
// optional 0/1 mask.
#include <algorithm>

#include "sa_common.cuh"

namespace sa {
namespace {

constexpr int SEL_WARPS = 8;
constexpr int SEL_THREADS = SEL_WARPS * 32;

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

// Selects blocks of one (head, q block) row in place: L[0..nbc) holds logits on entry and the
// probabilities afterwards; the selection is OR-ed into bits[].
__device__ void select_row(float* L, int nbc, float tau_f, uint32_t* bits, int lane) {
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
    for (int j = lane; j < nbc; j += 32) {
        const float p = __fdiv_rn(L[j], s);
        L[j] = p;
        tot += static_cast<double>(p);
    }
    tot = warp_sum_d(tot);
    __syncwarp();
    if (!(static_cast<float>(tot) >= tau_f)) {          // tau never reached: keep every causal block
        for (int j = lane; j < nbc; j += 32) atomicOr(&bits[j >> 5], 1u << (j & 31));
        return;
    }
    // largest v (bit pattern) with fp32(sum_{p >= v} p) >= tau: pred(lo) true, pred(hi) false
    uint32_t lo = 0u, hi = 0x3F800001u;
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
    int kt = ties;                                        // ties needed to cross tau (ascending block order)
    double acc = above;
    for (int k = 1; k <= ties; ++k) {
        acc += static_cast<double>(vstar);
        if (static_cast<float>(acc) >= tau_f) { kt = k; break; }
    }
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

// Register-resident variant of select_row for rows of at most 32*NPL blocks: lane l holds blocks
// l, l+32, ...; identical arithmetic (fp32 softmax, float64 sums, bisection, tie order).
template <int NPL>
__device__ void select_row_regs(const float* L, int nbc, float tau_f, uint32_t* bits, int lane) {
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
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        p[c] = (lane + 32 * c < nbc) ? expf(p[c] - mx) : 0.f;
        s += p[c];
    }
    s = warp_sum_f(s);
    double tot = 0.0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        p[c] = (lane + 32 * c < nbc) ? __fdiv_rn(p[c], s) : -1.f;   // -1: not a block of this row
        tot += p[c] > 0.f ? static_cast<double>(p[c]) : 0.0;
    }
    tot = warp_sum_d(tot);
    if (!(static_cast<float>(tot) >= tau_f)) {
#pragma unroll
        for (int c = 0; c < NPL; ++c) {
            const uint32_t b = __ballot_sync(0xffffffffu, lane + 32 * c < nbc);
            if (lane == 0 && b) atomicOr(&bits[c], b);
        }
        return;
    }
    uint32_t lo = 0u, hi = 0x3F800001u;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        const float v = __uint_as_float(mid);
        double m = 0.0;
#pragma unroll
        for (int c = 0; c < NPL; ++c) m += p[c] >= v ? static_cast<double>(p[c]) : 0.0;
        m = warp_sum_d(m);
        if (static_cast<float>(m) >= tau_f) lo = mid; else hi = mid;
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
    int kt = ties;
    double acc = above;
    for (int k = 1; k <= ties; ++k) {
        acc += static_cast<double>(vstar);
        if (static_cast<float>(acc) >= tau_f) { kt = k; break; }
    }
    int seen = 0;
#pragma unroll
    for (int c = 0; c < NPL; ++c) {
        const bool tie = p[c] == vstar;
        const uint32_t tb = __ballot_sync(0xffffffffu, tie);
        const int rank = seen + __popc(tb & ((1u << lane) - 1u));
        const bool keep = p[c] > vstar || (tie && rank < kt);
        const uint32_t kb = __ballot_sync(0xffffffffu, keep);
        if (lane == 0 && kb) atomicOr(&bits[c], kb);
        seen += __popc(tb);
    }
}

__global__ void __launch_bounds__(SEL_THREADS) select_kernel(
    const float* __restrict__ qm, int64_t qbs, int64_t qhs, const float* __restrict__ km, int64_t khs, int64_t kbs,
    int nb_km, int H, int Hk, int D, int MB, int nb_total, int qblk0, float scale, float tau_f, int mode,
    int32_t* __restrict__ counts, int32_t* __restrict__ lists, int64_t list_stride, uint8_t* __restrict__ masks,
    int nbw) {
    extern __shared__ __align__(16) float sm[];
    const int g = H / Hk;
    const int hk = blockIdx.y, unit = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbp = nbw * 32;
    float* qv = sm;                                       // [g][D]
    float* logit = qv + g * D;                            // [g][nbp]
    uint32_t* bits = reinterpret_cast<uint32_t*>(logit + static_cast<size_t>(g) * nbp);   // [g][nbw]
    for (int i = threadIdx.x; i < g * nbw; i += SEL_THREADS) bits[i] = 0u;
    const int nsub = (mode == SA_SELECT_PAIR_UNION) ? 2 : 1;
    for (int sub = 0; sub < nsub; ++sub) {
        const int m = (mode == SA_SELECT_PAIR_UNION) ? 2 * unit + sub : unit;
        const int gi = qblk0 + m;
        const int nbc = min(gi + 1, nb_total);
        __syncthreads();
        for (int i = threadIdx.x; i < g * D; i += SEL_THREADS) {
            const int hh = i / D, d = i - hh * D;
            qv[i] = qm[static_cast<int64_t>(m) * qbs + static_cast<int64_t>(hk * g + hh) * qhs + d];
        }
        __syncthreads();
        // scores: one thread per key block, all g heads at once (km row read with 16-byte loads)
        for (int j = threadIdx.x; j < nbc; j += SEL_THREADS) {
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.f;
            if (j < nb_km) {
                const float* kr = km + static_cast<int64_t>(hk) * khs + static_cast<int64_t>(j) * kbs;
                for (int d = 0; d < D; d += 4) {
                    const float4 kv = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (i < g) {
                            const float* q = qv + i * D + d;
                            acc[i] = fmaf(q[0], kv.x, acc[i]);
                            acc[i] = fmaf(q[1], kv.y, acc[i]);
                            acc[i] = fmaf(q[2], kv.z, acc[i]);
                            acc[i] = fmaf(q[3], kv.w, acc[i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < g) logit[i * nbp + j] = acc[i] * scale;
        }
        __syncthreads();
        for (int i = warp; i < g; i += SEL_WARPS) {
            float* L = logit + static_cast<size_t>(i) * nbp;
            if (nbc <= 128) select_row_regs<4>(L, nbc, tau_f, bits + i * nbw, lane);
            else if (nbc <= 512) select_row_regs<16>(L, nbc, tau_f, bits + i * nbw, lane);
            else select_row(L, nbc, tau_f, bits + i * nbw, lane);
            __syncwarp();
            if (lane == 0) {
                if (gi < nb_total) atomicOr(&bits[i * nbw + (gi >> 5)], 1u << (gi & 31));   // diagonal
                atomicOr(&bits[i * nbw], 1u);                                                 // sink
            }
        }
    }
    __syncthreads();
    // emit rows
    const int nrows_here = (mode == SA_SELECT_KV_UNION) ? 1 : g;
    for (int i = warp; i < nrows_here; i += SEL_WARPS) {
        int64_t row;
        if (mode == SA_SELECT_PER_HEAD) row = static_cast<int64_t>(hk * g + i) * MB + unit;
        else if (mode == SA_SELECT_PAIR_UNION) row = static_cast<int64_t>(hk * g + i) * (MB / 2) + unit;
        else row = static_cast<int64_t>(hk) * MB + unit;
        int total = 0;
        for (int w = 0; w < nbw; ++w) {
            uint32_t word;
            if (mode == SA_SELECT_KV_UNION) {
                word = 0u;
                for (int hh = 0; hh < g; ++hh) word |= bits[hh * nbw + w];
            } else {
                word = bits[i * nbw + w];
            }
            const int j = w * 32 + lane;
            const bool on = (word >> lane) & 1u;
            if (lists && on) lists[row * list_stride + total + __popc(word & ((1u << lane) - 1u))] = j;
            if (masks && j < nb_total) masks[row * nb_total + j] = on ? 1 : 0;
            total += __popc(word);
        }
        if (counts && lane == 0) counts[row] = total;
    }
}

}  // namespace
}  // namespace sa

using namespace sa;

extern "C" int sa_select(const float* qm, int64_t qm_block_stride, int64_t qm_head_stride, const float* km,
                         int64_t km_head_stride, int64_t km_block_stride, int nb_km, int num_heads, int num_kv_heads,
                         int head_dim, int MB, int nb_total, int qblk0, float scale, float tau, int mode,
                         int32_t* counts, int32_t* lists, int64_t list_stride, uint8_t* masks, void* stream) {
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || MB <= 0 || nb_total <= 0 || qblk0 < 0 ||
        nb_km < 0)
        return fail(SA_ERR_ARG, "sa_select: bad sizes");
    const int g = num_heads / num_kv_heads;
    if (g > 16) return fail(SA_ERR_UNSUPPORTED, "sa_select: more than 16 query heads per kv head");
    if (head_dim % 4 || head_dim <= 0) return fail(SA_ERR_UNSUPPORTED, "sa_select: head_dim %% 4");
    if (!qm || (!km && nb_km > 0)) return fail(SA_ERR_ARG, "sa_select: null pointer");
    if ((reinterpret_cast<uintptr_t>(km) & 15) || km_block_stride % 4 || km_head_stride % 4)
        return fail(SA_ERR_ALIGN, "sa_select: km must be 16-byte aligned with strides %% 4 == 0");
    if (mode == SA_SELECT_PAIR_UNION && (MB % 2)) return fail(SA_ERR_ARG, "sa_select: pair union needs even MB");
    if (mode < 0 || mode > 2) return fail(SA_ERR_ARG, "sa_select: bad mode");
    if (lists && list_stride < nb_total) return fail(SA_ERR_ARG, "sa_select: list_stride < nb_total");
    const int nbw = (nb_total + 31) / 32;
    const size_t smem = (static_cast<size_t>(g) * head_dim + static_cast<size_t>(g) * nbw * 32) * sizeof(float) +
                        static_cast<size_t>(g) * nbw * sizeof(uint32_t);
    if (smem > 227 * 1024) return fail(SA_ERR_UNSUPPORTED, "sa_select: %d key blocks need %zu B of shared memory", nb_total, smem);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(SA_ERR_CUDA, "sa_select: %s", cudaGetErrorString(e));
    }
    const int units = (mode == SA_SELECT_PAIR_UNION) ? MB / 2 : MB;
    dim3 grid(units, num_kv_heads);
    select_kernel<<<grid, SEL_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
        qm, qm_block_stride, qm_head_stride, km, km_head_stride, km_block_stride, nb_km, num_heads, num_kv_heads,
        head_dim, MB, nb_total, qblk0, scale, static_cast<float>(tau), mode, counts, lists, list_stride, masks, nbw);
    return check_launch("select_kernel");
}
