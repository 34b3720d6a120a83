// Elementwise kernels of the end-to-end prefill harness (random-init dense GQA decoder, benchmark
// config 5): fused residual add + RMSNorm, rotary position embedding of q/k with the K/V cache write,
// and the SwiGLU activation.  The reference measures TTFT through vLLM's model code (its fused
// add RMSNorm, neox-style rotary embedding and SiluAndMul, vllm 0.22:
// model_executor/layers/layernorm.py, rotary_embedding/base.py, activation.py); these kernels
// compute the same functions.  All are HBM-streaming: 16-byte vector loads, grids sized to the SM
// count, fp32 arithmetic, bf16 in and out.
#include <algorithm>

#include "sa_common.cuh"

namespace sa {
namespace {

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
}

// One CTA of 128 threads per row (grid-stride over rows); thread i holds chunks i, i+128, ... of 8
// elements.  h <- bf16(h + delta); x <- bf16(s * rsqrt(mean(s^2) + eps) * w), s the fp32 sum.
template <int NV>
__global__ void __launch_bounds__(128) add_rmsnorm_kernel(const uint16_t* __restrict__ delta, int64_t d_stride,
                                                          uint16_t* __restrict__ h, int64_t h_stride,
                                                          const uint16_t* __restrict__ w, uint16_t* __restrict__ x,
                                                          int64_t x_stride, int rows, int hidden, float eps) {
    __shared__ float red[4];
    const int nch = hidden / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
        float v[NV][8];
        float ss = 0.f;
        uint4* hrow = reinterpret_cast<uint4*>(h + static_cast<int64_t>(row) * h_stride);
        const uint4* drow = delta ? reinterpret_cast<const uint4*>(delta + static_cast<int64_t>(row) * d_stride) : nullptr;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int j = threadIdx.x + 128 * i;
            if (j < nch) {
                bf16x8_to_f32(hrow[j], v[i]);
                if (drow) {
                    float d[8];
                    bf16x8_to_f32(drow[j], d);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[i][e] += d[e];
                    hrow[j] = f32_to_bf16x8(v[i]);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        const float total = (red[0] + red[1]) + (red[2] + red[3]);
        __syncthreads();                                          // red is rewritten by the next row
        const float rinv = rsqrtf(total / static_cast<float>(hidden) + eps);
        uint4* xrow = reinterpret_cast<uint4*>(x + static_cast<int64_t>(row) * x_stride);
        const uint4* wv = reinterpret_cast<const uint4*>(w);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int j = threadIdx.x + 128 * i;
            if (j < nch) {
                float wf[8], o[8];
                bf16x8_to_f32(__ldg(wv + j), wf);
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = v[i][e] * rinv * wf[e];
                xrow[j] = f32_to_bf16x8(o);
            }
        }
    }
}

// Neox-style rotary embedding of 8 pairs: elements 8j..8j+7 (a) pair with half+8j.. (b) at the
// angles of position row cs (cos_sin[pos] holds cos of the D/2 angles then their sin, fp32).
__device__ __forceinline__ void rope8(const uint4 a, const uint4 b, const float* __restrict__ cs, int j, int half,
                                      uint4& oa, uint4& ob) {
    const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + 8 * j));
    const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + 8 * j + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(cs + half + 8 * j));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(cs + half + 8 * j + 4));
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float x1[8], x2[8], y1[8], y2[8];
    bf16x8_to_f32(a, x1);
    bf16x8_to_f32(b, x2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        y1[e] = x1[e] * c[e] - x2[e] * s[e];
        y2[e] = x2[e] * c[e] + x1[e] * s[e];
    }
    oa = f32_to_bf16x8(y1);
    ob = f32_to_bf16x8(y2);
}

struct RopeArgs {
    const uint16_t* qkv;
    int64_t qkv_stride;
    int rows, hq, hk, D, pos0;
    const float* cos_sin;
    uint16_t* q_out;
    uint16_t* k_out;
    int64_t k_stride;
    uint16_t* v_out;
    int64_t v_stride;
    // key block means of the rotated k rows (kctas > 0): CTAs [0, kctas) = nblk key blocks x nhg
    // groups of hpc KV heads, rg row groups (block_means_shape); km[h, b - km_block0, :]
    int kctas, nhg, hpc, rg, block, b0;
    float* km;
    int64_t km_hs, km_bs;
    int km_block0;
};

// Rotary embedding of the k heads with their key block means (kctas > 0): CTA (b, head group) owns
// the rows of block b within [pos0, pos0 + rows); thread (head, pair group j, row group g) rotates
// rows lo+g, lo+g+rg, ... into the cache rows and sums the bf16 results in that order; the rg
// partial sums are then added in group order and divided by the row count.  That is
// block_means_kernel's order for the same launch shape, so the means equal sa_block_means_bf16's
// over the written k rows bit for bit.  A kernel of its own: its per-thread row batches need far more
// registers than the elementwise rotation, whose occupancy they would otherwise cap.
__global__ void __launch_bounds__(256) rope_k_means_kernel(const RopeArgs a) {
    const int D = a.D, half = D / 2, jn = D / 16;
    {
        extern __shared__ float partial[];                       // [rg - 1][threads in use][16]
        const int txp = a.hpc * jn;
        const int tid = threadIdx.x, tx = tid % txp, ty = tid / txp;
        const int used = txp * a.rg;
        const int hl = tx / jn, j = tx - hl * jn;
        const int b = a.b0 + static_cast<int>(blockIdx.x) / a.nhg;
        const int h = (static_cast<int>(blockIdx.x) % a.nhg) * a.hpc + hl;
        const bool active = tid < used && h < a.hk;
        const int lo = max(a.pos0, b * a.block) - a.pos0;
        const int hi = min(a.pos0 + a.rows, (b + 1) * a.block) - a.pos0;
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
        if (active) {
            const uint16_t* src = a.qkv + static_cast<int64_t>(a.hq + h) * D;
            uint16_t* dst = a.k_out + static_cast<int64_t>(h) * D;
            constexpr int BATCH = 4;
            for (int base = lo + ty; base < hi; base += BATCH * a.rg) {
                uint4 va[BATCH], vb[BATCH];
#pragma unroll
                for (int k = 0; k < BATCH; ++k) {
                    const int r = base + k * a.rg;
                    if (r < hi) {
                        const uint16_t* row = src + static_cast<int64_t>(r) * a.qkv_stride;
                        va[k] = *reinterpret_cast<const uint4*>(row + 8 * j);
                        vb[k] = *reinterpret_cast<const uint4*>(row + half + 8 * j);
                    }
                }
#pragma unroll
                for (int k = 0; k < BATCH; ++k) {
                    const int r = base + k * a.rg;
                    if (r >= hi) break;
                    uint4 oa, ob;
                    rope8(va[k], vb[k], a.cos_sin + static_cast<int64_t>(a.pos0 + r) * D, j, half, oa, ob);
                    uint16_t* drow = dst + static_cast<int64_t>(r) * a.k_stride;
                    *reinterpret_cast<uint4*>(drow + 8 * j) = oa;
                    *reinterpret_cast<uint4*>(drow + half + 8 * j) = ob;
                    float f[8];
                    bf16x8_to_f32(oa, f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] += f[i];
                    bf16x8_to_f32(ob, f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[8 + i] += f[i];
                }
            }
        }
        if (a.rg > 1) {
            if (active && ty > 0) {
#pragma unroll
                for (int i = 0; i < 16; ++i) partial[((ty - 1) * txp + tx) * 16 + i] = acc[i];
            }
            __syncthreads();
            if (ty != 0) return;
            for (int g = 1; g < a.rg; ++g) {
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[i] += partial[((g - 1) * txp + tx) * 16 + i];
            }
        }
        if (!active) return;
        const float cnt = static_cast<float>(max(hi - lo, 1));
        float* o = a.km + static_cast<int64_t>(h) * a.km_hs + static_cast<int64_t>(b - a.km_block0) * a.km_bs;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[8 * j + i] = __fdiv_rn(acc[i], cnt);
            o[half + 8 * j + i] = __fdiv_rn(acc[8 + i], cnt);
        }
    }
}

// Rotary embedding of the q heads of qkv rows (positions pos0 + row) into q_out [rows, Hq, D], of the
// k heads into the cache rows unless rope_k_means_kernel does them (kctas > 0), and the v heads
// copied to theirs: grid-strided, one thread per 8 pairs of one head of one row.
__global__ void __launch_bounds__(256) rope_qkv_kernel(const RopeArgs a) {
    const int D = a.D, half = D / 2, jn = D / 16;
    const int nk = a.kctas ? 0 : a.hk;                           // k heads rotated here
    const int heads = a.hq + nk + a.hk;
    const int64_t total = static_cast<int64_t>(a.rows) * heads * jn;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t idx = first; idx < total; idx += stride) {
        const int j = static_cast<int>(idx % jn);
        const int64_t rest = idx / jn;
        const int hh = static_cast<int>(rest % heads);
        const int row = static_cast<int>(rest / heads);
        uint16_t* dst;
        int src_head;
        if (hh < a.hq) {
            dst = a.q_out + (static_cast<int64_t>(row) * a.hq + hh) * D;
            src_head = hh;
        } else if (hh < a.hq + nk) {
            dst = a.k_out + static_cast<int64_t>(row) * a.k_stride + static_cast<int64_t>(hh - a.hq) * D;
            src_head = hh;
        } else {
            const int hv = hh - a.hq - nk;
            dst = a.v_out + static_cast<int64_t>(row) * a.v_stride + static_cast<int64_t>(hv) * D;
            src_head = a.hq + a.hk + hv;
        }
        const uint16_t* src = a.qkv + static_cast<int64_t>(row) * a.qkv_stride + static_cast<int64_t>(src_head) * D;
        const uint4 va = *reinterpret_cast<const uint4*>(src + 8 * j);
        const uint4 vb = *reinterpret_cast<const uint4*>(src + half + 8 * j);
        uint4 oa = va, ob = vb;
        if (hh < a.hq + nk) rope8(va, vb, a.cos_sin + static_cast<int64_t>(a.pos0 + row) * D, j, half, oa, ob);
        *reinterpret_cast<uint4*>(dst + 8 * j) = oa;
        *reinterpret_cast<uint4*>(dst + half + 8 * j) = ob;
    }
}

// out[r, j] = silu(g) * u with g = gate_up[r, j], u = gate_up[r, inter + j] (vLLM SiluAndMul).
__global__ void __launch_bounds__(256) silu_mul_kernel(const uint16_t* __restrict__ gu, int64_t gu_stride, int rows,
                                                       int inter, uint16_t* __restrict__ out, int64_t out_stride) {
    const int jn = inter / 8;
    const int64_t total = static_cast<int64_t>(rows) * jn;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(idx % jn);
        const int64_t row = idx / jn;
        const uint16_t* src = gu + row * gu_stride;
        float g[8], u[8], o[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(src + 8 * j), g);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(src + inter + 8 * j), u);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = g[e] / (1.f + __expf(-g[e])) * u[e];
        *reinterpret_cast<uint4*>(out + row * out_stride + 8 * j) = f32_to_bf16x8(o);
    }
}

int grid_for(int64_t work, int threads) {
    const int64_t want = (work + threads - 1) / threads;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 16ll * num_sms())));
}

}  // namespace
}  // namespace sa

using namespace sa;

extern "C" int sa_add_rmsnorm_bf16(const void* delta, int64_t delta_row_stride, void* h, int64_t h_row_stride,
                                   const void* weight, void* x, int64_t x_row_stride, int rows, int hidden, float eps,
                                   void* stream) {
    if (rows < 0 || hidden <= 0 || hidden % 8) return fail(SA_ERR_ARG, "sa_add_rmsnorm_bf16: bad sizes");
    if (hidden > 128 * 8 * 8) return fail(SA_ERR_UNSUPPORTED, "sa_add_rmsnorm_bf16: hidden %d > 8192", hidden);
    if (!h || !weight || !x) return fail(SA_ERR_ARG, "sa_add_rmsnorm_bf16: null pointer");
    if (!aligned16(h) || !aligned16(weight) || !aligned16(x) || (delta && !aligned16(delta)) || h_row_stride % 8 ||
        x_row_stride % 8 || (delta && delta_row_stride % 8))
        return fail(SA_ERR_ALIGN, "sa_add_rmsnorm_bf16: tensors must be 16-byte aligned with row strides %% 8 == 0");
    if (rows == 0) return SA_OK;
    const int nv = (hidden / 8 + 127) / 128;
    const dim3 grid(std::min(rows, 32 * num_sms()));             // up to 16 resident per SM, rows grid-strided
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto* d = static_cast<const uint16_t*>(delta);
    auto* hp = static_cast<uint16_t*>(h);
    auto* w = static_cast<const uint16_t*>(weight);
    auto* xp = static_cast<uint16_t*>(x);
    if (nv <= 1)
        add_rmsnorm_kernel<1><<<grid, 128, 0, s>>>(d, delta_row_stride, hp, h_row_stride, w, xp, x_row_stride, rows, hidden, eps);
    else if (nv <= 2)
        add_rmsnorm_kernel<2><<<grid, 128, 0, s>>>(d, delta_row_stride, hp, h_row_stride, w, xp, x_row_stride, rows, hidden, eps);
    else if (nv <= 4)
        add_rmsnorm_kernel<4><<<grid, 128, 0, s>>>(d, delta_row_stride, hp, h_row_stride, w, xp, x_row_stride, rows, hidden, eps);
    else if (nv <= 5)
        add_rmsnorm_kernel<5><<<grid, 128, 0, s>>>(d, delta_row_stride, hp, h_row_stride, w, xp, x_row_stride, rows, hidden, eps);
    else
        add_rmsnorm_kernel<8><<<grid, 128, 0, s>>>(d, delta_row_stride, hp, h_row_stride, w, xp, x_row_stride, rows, hidden, eps);
    return check_launch("add_rmsnorm_kernel");
}

namespace sa {
namespace {

int rope_qkv(const char* who, const void* qkv, int64_t qkv_row_stride, int rows, int num_heads, int num_kv_heads,
             int head_dim, const float* cos_sin, int pos0, int max_pos, void* q_out, void* k_out, int64_t k_row_stride,
             void* v_out, int64_t v_row_stride, int block, float* km, int64_t km_head_stride, int64_t km_block_stride,
             int km_block0, void* stream) {
    if (rows < 0 || num_heads <= 0 || num_kv_heads <= 0 || pos0 < 0) return fail(SA_ERR_ARG, "%s: bad sizes", who);
    if (head_dim % 16 || head_dim > 8 * 256)
        return fail(SA_ERR_UNSUPPORTED, "%s: head_dim %d not a multiple of 16 (<= 2048)", who, head_dim);
    if (pos0 + rows > max_pos) return fail(SA_ERR_ARG, "%s: positions %d.. beyond the table (%d)", who, pos0, max_pos);
    if (!qkv || !cos_sin || !q_out || !k_out || !v_out) return fail(SA_ERR_ARG, "%s: null pointer", who);
    if (!aligned16(qkv) || !aligned16(cos_sin) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out) ||
        qkv_row_stride % 8 || k_row_stride % 8 || v_row_stride % 8)
        return fail(SA_ERR_ALIGN, "%s: tensors must be 16-byte aligned with row strides %% 8 == 0", who);
    RopeArgs a{};
    a.qkv = static_cast<const uint16_t*>(qkv);
    a.qkv_stride = qkv_row_stride;
    a.rows = rows;
    a.hq = num_heads;
    a.hk = num_kv_heads;
    a.D = head_dim;
    a.pos0 = pos0;
    a.cos_sin = cos_sin;
    a.q_out = static_cast<uint16_t*>(q_out);
    a.k_out = static_cast<uint16_t*>(k_out);
    a.k_stride = k_row_stride;
    a.v_out = static_cast<uint16_t*>(v_out);
    a.v_stride = v_row_stride;
    size_t smem = 0;
    if (km) {
        if (block <= 0) return fail(SA_ERR_ARG, "%s: block %d", who, block);
        const int b0 = pos0 / block, b1 = (pos0 + rows + block - 1) / block;
        if (b0 < km_block0) return fail(SA_ERR_ARG, "%s: first block %d < km_block0 %d", who, b0, km_block0);
        if (rows > 0) {
            block_means_shape(b1 - b0, num_kv_heads, head_dim, block, &a.hpc, &a.rg);
            a.nhg = (num_kv_heads + a.hpc - 1) / a.hpc;
            a.kctas = (b1 - b0) * a.nhg;
            a.block = block;
            a.b0 = b0;
            a.km = km;
            a.km_hs = km_head_stride;
            a.km_bs = km_block_stride;
            a.km_block0 = km_block0;
            smem = static_cast<size_t>(a.rg - 1) * a.hpc * (head_dim / 16) * 16 * sizeof(float);   // <= 15.5 KB
        }
    }
    if (rows == 0) return SA_OK;
    const int64_t work = static_cast<int64_t>(rows) * (num_heads + (a.kctas ? 0 : num_kv_heads) + num_kv_heads) *
                         (head_dim / 16);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (a.kctas) {
        rope_k_means_kernel<<<a.kctas, 256, smem, st>>>(a);
        if (int rc = check_launch("rope_k_means_kernel")) return rc;
    }
    rope_qkv_kernel<<<grid_for(work, 256), 256, 0, st>>>(a);
    return check_launch("rope_qkv_kernel");
}

}  // namespace
}  // namespace sa

extern "C" int sa_rope_qkv_bf16(const void* qkv, int64_t qkv_row_stride, int rows, int num_heads, int num_kv_heads,
                                int head_dim, const float* cos_sin, int pos0, int max_pos, void* q_out, void* k_out,
                                int64_t k_row_stride, void* v_out, int64_t v_row_stride, void* stream) {
    return rope_qkv("sa_rope_qkv_bf16", qkv, qkv_row_stride, rows, num_heads, num_kv_heads, head_dim, cos_sin, pos0,
                    max_pos, q_out, k_out, k_row_stride, v_out, v_row_stride, 0, nullptr, 0, 0, 0, stream);
}

extern "C" int sa_rope_qkv_means_bf16(const void* qkv, int64_t qkv_row_stride, int rows, int num_heads,
                                      int num_kv_heads, int head_dim, const float* cos_sin, int pos0, int max_pos,
                                      void* q_out, void* k_out, int64_t k_row_stride, void* v_out,
                                      int64_t v_row_stride, int block, float* km, int64_t km_head_stride,
                                      int64_t km_block_stride, int km_block0, void* stream) {
    if (!km) return fail(SA_ERR_ARG, "sa_rope_qkv_means_bf16: null km");
    return rope_qkv("sa_rope_qkv_means_bf16", qkv, qkv_row_stride, rows, num_heads, num_kv_heads, head_dim, cos_sin,
                    pos0, max_pos, q_out, k_out, k_row_stride, v_out, v_row_stride, block, km, km_head_stride,
                    km_block_stride, km_block0, stream);
}

extern "C" int sa_silu_mul_bf16(const void* gate_up, int64_t gate_up_row_stride, int rows, int inter, void* out,
                                int64_t out_row_stride, void* stream) {
    if (rows < 0 || inter <= 0 || inter % 8) return fail(SA_ERR_ARG, "sa_silu_mul_bf16: bad sizes");
    if (!gate_up || !out) return fail(SA_ERR_ARG, "sa_silu_mul_bf16: null pointer");
    if (!aligned16(gate_up) || !aligned16(out) || gate_up_row_stride % 8 || out_row_stride % 8)
        return fail(SA_ERR_ALIGN, "sa_silu_mul_bf16: tensors must be 16-byte aligned with row strides %% 8 == 0");
    if (rows == 0) return SA_OK;
    const int64_t work = static_cast<int64_t>(rows) * (inter / 8);
    silu_mul_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(gate_up), gate_up_row_stride, rows, inter, static_cast<uint16_t*>(out),
        out_row_stride);
    return check_launch("silu_mul_kernel");
}
