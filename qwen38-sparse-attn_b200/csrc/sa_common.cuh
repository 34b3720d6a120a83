// Shared device helpers for the B200 (sm_100a) block-sparse prefill kernels.
//
// Thin inline-PTX wrappers for mbarriers, TMA tile loads, tcgen05 (tensor-memory MMA) and
// number-format conversions, plus the bounded wait every spin in these kernels uses: a wait
// gives up after SA_WAIT_TIMEOUT_NS of wall time (read from %globaltimer), records a status
// code in the caller's device status word and tells the rest of the CTA to stop through a
// shared-memory abort flag.  No kernel here traps or spins without a limit.
#pragma once

#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "../../include/sparse_attn_b200.h"

#ifndef SA_WAIT_TIMEOUT_NS
#define SA_WAIT_TIMEOUT_NS 2000000000ull   // 2 s: a legitimate wait here lasts microseconds
#endif

namespace sa {

// ------------------------------------------------------------------------------------------
// Host-side error text (thread-local) shared by every entry point.
// ------------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
int num_sms();                          // SM count of the current device (cached after the first call)
bool aligned16(const void* p);

// One-time per-device set-up (a kernel attribute, a symbol's device address), recorded together with
// the CUDA context it was made in.  After cudaDeviceReset (or any destruction of the primary
// context) the device gets a new context in which the module is loaded afresh, so a record made in
// another context is stale and the set-up is redone.  All members are guarded by `mu`.
constexpr int SA_MAX_DEVICES = 64;
struct PerContext {
    std::mutex mu;
    void* ctx[SA_MAX_DEVICES] = {};
    void* value[SA_MAX_DEVICES] = {};
};
// The calling thread's current device and context (the context is created if the runtime has not
// made it yet).  Returns SA_OK, or an SA_ERR_* code with the error text set.
int current_device_context(const char* who, int* dev, void** ctx);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda);
// nullptr when the driver does not provide it.
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// ------------------------------------------------------------------------------------------
// Small device utilities
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// One lane of a converged warp (elect.sync): tcgen05.mma / commit / TMA issue is predicated on it
// while the surrounding address and descriptor arithmetic stays warp-uniform.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// bf16 round-to-nearest-even of an fp32 value, returned as fp32.
__device__ __forceinline__ float bf16_round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// Two fp32 -> packed e4m3x2 (lo goes to bits 0..7), round to nearest even, saturating.
__device__ __forceinline__ uint16_t pack_e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two fp32 -> packed bf16x2 (lo goes to bits 0..15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe (Cody-Waite range reduction + minimax polynomial), so a share of the
// softmax exponentials can bypass the MUFU unit.  x = n + f with n = rint(x) taken from the low
// mantissa bits of x + 1.5*2^23, f in [-0.5, 0.5]; 2^f ~ c0 + f(c1 + f(c2 + f c3)) with
// coefficients from a Lawson (iteratively reweighted least squares) minimax fit of the relative
// error on [-0.5, 0.5] (max rel. error 7.5e-5); 2^n is added to the exponent field.  x is clamped
// at -120, below which the result (< 2^-119) is irrelevant next to the row maximum's term of ~1.
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -120.f);
    const float magic = 12582912.f;            // 1.5 * 2^23
    const float y = x + magic;
    const float f = x - (y - magic);
    float p = fmaf(0.0551716685f, f, 0.242611125f);
    p = fmaf(p, f, 0.693260968f);
    p = fmaf(p, f, 0.999928057f);
    return __int_as_float(__float_as_int(p) + __float_as_int(y) * 8388608);
}

// Packed fp32x2 arithmetic (one instruction for two lanes' worth of work on sm_100).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// exp2_poly on a pair of values with packed f32x2 arithmetic (same reduction and coefficients; two
// results for about the instruction count of one).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x = make_float2(fmaxf(x.x, -120.f), fmaxf(x.y, -120.f));
    const float2 magic = make_float2(12582912.f, 12582912.f), neg_magic = make_float2(-12582912.f, -12582912.f);
    const float2 y = fadd2(x, magic);
    const float2 f = ffma2(fadd2(y, neg_magic), make_float2(-1.f, -1.f), x);
    float2 p = ffma2(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.242611125f, 0.242611125f));
    p = ffma2(p, f, make_float2(0.693260968f, 0.693260968f));
    p = ffma2(p, f, make_float2(0.999928057f, 0.999928057f));
    return make_float2(__int_as_float(__float_as_int(p.x) + __float_as_int(y.x) * 8388608),
                       __int_as_float(__float_as_int(p.y) + __float_as_int(y.y) * 8388608));
}

// ------------------------------------------------------------------------------------------
// Streaming bf16 rows and their e4m3 quantisation (prep.cu, select.cu)
// ------------------------------------------------------------------------------------------
// 16-byte load that bypasses L1 (each row is read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Row addressing of a [rows, heads, head_dim] operand that is either contiguous (pages == nullptr:
// row r at r * row_stride) or held in fixed-size pages, like a vLLM KV cache [num_pages, page,
// heads, head_dim]: row r is logical row l = row0 + r, which sits in slot l % page of page
// pages[l / page] (page_stride elements between pages, row_stride between the slots of a page).
struct RowMap {
    const int32_t* pages;
    int64_t page_stride;
    int page, row0;
    __device__ __forceinline__ int64_t offset(int r, int64_t row_stride) const {
        if (!pages) return static_cast<int64_t>(r) * row_stride;
        const int l = row0 + r;
        const int pg = l / page;
        return static_cast<int64_t>(__ldg(pages + pg)) * page_stride + static_cast<int64_t>(l - pg * page) * row_stride;
    }
};
inline RowMap contiguous_rows() { return RowMap{nullptr, 0, 1, 0}; }

// Launch shape of a block-means reduction over nblk key blocks of `block` rows and `heads` heads of
// head_dim: heads per CTA (hpc, each with head_dim / 8 column threads) and row groups (rg).  The
// row groups fix the order in which a block's rows are added (group g sums rows lo+g, lo+g+rg, ...
// in order; the groups' sums are then added in group order), so kernels that produce block means
// for the same (nblk, heads, head_dim, block) through this shape produce the same bits.  Aims at
// >= 4 CTAs per SM and ~2048 threads per SM of independent 16-byte row streams: fewer heads per CTA
// first (more CTAs), then row groups (more loads in flight per block); hpc * head_dim / 8 * rg <= 512.
inline void block_means_shape(int nblk, int heads, int head_dim, int block, int* hpc_out, int* rg_out) {
    const int cols = head_dim / 8;
    int hpc = heads < 256 / cols ? heads : 256 / cols;
    if (hpc < 1) hpc = 1;
    while (hpc > 1 && static_cast<long long>(nblk) * ((heads + hpc - 1) / hpc) < 4ll * num_sms()) hpc = (hpc + 1) / 2;
    const int tx = hpc * cols;
    const long long ctas = static_cast<long long>(nblk) * ((heads + hpc - 1) / hpc);
    const long long target = 2048ll * num_sms();
    int rg = 1;
    while (rg < 16 && (ctas * tx * rg < target || tx * rg < 128) && tx * rg * 2 <= 512 && rg * 2 <= block / 4) rg *= 2;
    *hpc_out = hpc;
    *rg_out = rg;
}

// eight bf16 values -> fp32
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// value before the e4m3 cast under a quantisation mode (SA_QUANT_*)
__device__ __forceinline__ float scale_value(float x, float s, int mode) {
    if (mode == SA_QUANT_DIV) return __fdiv_rn(x, s);
    const float t = x * s;
    return mode == SA_QUANT_MUL_BF16 ? bf16_round(t) : t;
}

__device__ __forceinline__ uint2 quant8(const float (&f)[8], float s, int mode) {
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = scale_value(f[i], s, mode);
    uint2 r;
    r.x = static_cast<uint32_t>(pack_e4m3x2(y[0], y[1])) | (static_cast<uint32_t>(pack_e4m3x2(y[2], y[3])) << 16);
    r.y = static_cast<uint32_t>(pack_e4m3x2(y[4], y[5])) | (static_cast<uint32_t>(pack_e4m3x2(y[6], y[7])) << 16);
    return r;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// ------------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with the programmatic-serialization attribute
// may start once every CTA of the kernel before it in the stream has executed
// grid_dependents_launch (or exited); grid_dependency_wait then blocks until that kernel has
// completed and its memory writes are visible.  Both are no-ops for kernels launched normally.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}

#ifndef SA_WAIT_SUSPEND_NS
#define SA_WAIT_SUSPEND_NS 1000000u   // try_wait suspend-time hint: a waiting warp sleeps (up to 1 ms)
#endif                                // until the phase completes instead of re-issuing polls

// Non-blocking test of a phase (mbarrier.test_wait): returns at once whether the phase with this
// parity has completed.  (try_wait, below, may suspend the thread until the phase completes or a
// time limit passes, so it must not be used to poll several barriers in turn.)
__device__ __forceinline__ bool mbar_poll(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait without a suspend hint: the cheapest wait for a phase that has usually completed already.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(SA_WAIT_SUSPEND_NS) : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and raises the CTA abort
// flag, plus `code` in the device status word the first time) when limit_ns of wall time expire,
// or false at once when another thread of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait_limit(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                                int code, uint64_t limit_ns) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 7u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > limit_ns) {
                *abort_flag = 1;
                if (status) atomicOr(status, code);
                return false;
            }
        }
    }
}

// The same with the library's limit, SA_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int code) {
    return mbar_wait_limit(bar, parity, abort_flag, status, code, SA_WAIT_TIMEOUT_NS);
}

// Same bound, polling without the suspend hint: for a latency-critical waiter whose wake-up after a
// suspension would sit on the pipeline's critical path (the attention kernel's MMA issuer, its
// softmax warps waiting for S and O, its producer waiting for a free stage: measured 0.4-0.5%
// faster than suspending waits there).
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                               int* status, int code) {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 7u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > SA_WAIT_TIMEOUT_NS) {
                *abort_flag = 1;
                if (status) atomicOr(status, code);
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag: used while draining copies after an abort.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
    volatile int never = 0;
    mbar_wait(bar, parity, &never, nullptr, 0);
}

// ------------------------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads/stores
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (tensor cores,
// TMA) before the hand-off that lets them be read.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 inputs) or kind::f8f6f4 (e4m3).
template <bool FP8>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (FP8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
            :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
    }
}

// D(tmem) (+)= A(tmem) * B(smem desc)^T.
template <bool FP8>
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (FP8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}"
            :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
            :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
    }
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#define SA_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                 "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define SA_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), \
                 "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : SA_R8(0), SA_R8(8), SA_R8(16), SA_R8(24)
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        :: "r"(taddr), SA_W8(0), SA_W8(8), SA_W8(16), SA_W8(24)
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 :: "r"(taddr), SA_W8(0) : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        :: "r"(taddr), SA_W8(0), SA_W8(8) : "memory");
}

#undef SA_R8
#undef SA_W8

// ------------------------------------------------------------------------------------------
// UMMA descriptors (sm_100)
// ------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand tile stored as rows of `row_bytes`
// (64 or 128) bytes, written by TMA with the matching swizzle; 8-row groups are `8*row_bytes`
// apart.  Bits: [0,14) start>>4, [16,30) leading offset>>4 (unused for swizzled K-major),
// [32,46) stride offset>>4, [46,48) version 1, [61,64) layout (2 = 128B swizzle, 4 = 64B).
__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t saddr, int row_bytes) {
    const uint64_t layout = (row_bytes == 128) ? 2ull : 4ull;
    const uint64_t sbo = static_cast<uint64_t>(8 * row_bytes) >> 4;
    return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) | (1ull << 16) | (sbo << 32) | (1ull << 46) |
           (layout << 61);
}

// Shared-memory descriptor for an MN-major operand tile with 128B swizzle: rows of 128 bytes along
// the MN dimension, one row per K index; 8-row groups (1024 B) along K are the stride offset, and
// successive 128-byte MN column blocks are `mn_block_bytes` apart (leading offset).
__device__ __forceinline__ uint64_t smem_desc_mnmajor(uint32_t saddr, uint32_t mn_block_bytes) {
    return (static_cast<uint64_t>((saddr >> 4) & 0x3FFFu)) | (static_cast<uint64_t>((mn_block_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: fp32 accumulator, A/B K-major, A/B format (bf16 = 1, e4m3 = 0).
__host__ __device__ constexpr uint32_t instr_desc(int M, int N, uint32_t ab_format) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace sa
