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

// Neox-style rotary embedding: element i < D/2 pairs with i + D/2 at angle pos * theta^(-2i/D);
// cos_sin[pos] holds cos of the D/2 angles then their sin (fp32).  One thread per 8 pairs of one
// head of one row; q heads go to q_out [rows, Hq, D], k heads (rotated) and v heads (copied) to the
// cache rows.
__global__ void __launch_bounds__(256) rope_qkv_kernel(const uint16_t* __restrict__ qkv, int64_t qkv_stride, int rows,
                                                       int hq, int hk, int D, const float* __restrict__ cos_sin,
                                                       int pos0, uint16_t* __restrict__ q_out,
                                                       uint16_t* __restrict__ k_out, int64_t k_stride,
                                                       uint16_t* __restrict__ v_out, int64_t v_stride) {
    const int jn = D / 16;                                        // 8-pair groups per head
    const int heads = hq + 2 * hk;
    const int64_t total = static_cast<int64_t>(rows) * heads * jn;
    const int half = D / 2;
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(idx % jn);
        const int64_t rest = idx / jn;
        const int hh = static_cast<int>(rest % heads);
        const int row = static_cast<int>(rest / heads);
        const uint16_t* src = qkv + static_cast<int64_t>(row) * qkv_stride + static_cast<int64_t>(hh) * D;
        const uint4 a = *reinterpret_cast<const uint4*>(src + 8 * j);
        const uint4 b = *reinterpret_cast<const uint4*>(src + half + 8 * j);
        uint4 oa = a, ob = b;
        if (hh < hq + hk) {
            const float* cs = cos_sin + static_cast<int64_t>(pos0 + row) * D;
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
        uint16_t* dst;
        if (hh < hq)
            dst = q_out + (static_cast<int64_t>(row) * hq + hh) * D;
        else if (hh < hq + hk)
            dst = k_out + static_cast<int64_t>(row) * k_stride + static_cast<int64_t>(hh - hq) * D;
        else
            dst = v_out + static_cast<int64_t>(row) * v_stride + static_cast<int64_t>(hh - hq - hk) * D;
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

extern "C" int sa_rope_qkv_bf16(const void* qkv, int64_t qkv_row_stride, int rows, int num_heads, int num_kv_heads,
                                int head_dim, const float* cos_sin, int pos0, int max_pos, void* q_out, void* k_out,
                                int64_t k_row_stride, void* v_out, int64_t v_row_stride, void* stream) {
    if (rows < 0 || num_heads <= 0 || num_kv_heads <= 0 || pos0 < 0) return fail(SA_ERR_ARG, "sa_rope_qkv_bf16: bad sizes");
    if (head_dim % 16) return fail(SA_ERR_UNSUPPORTED, "sa_rope_qkv_bf16: head_dim %d not a multiple of 16", head_dim);
    if (pos0 + rows > max_pos) return fail(SA_ERR_ARG, "sa_rope_qkv_bf16: positions %d.. beyond the table (%d)", pos0, max_pos);
    if (!qkv || !cos_sin || !q_out || !k_out || !v_out) return fail(SA_ERR_ARG, "sa_rope_qkv_bf16: null pointer");
    if (!aligned16(qkv) || !aligned16(cos_sin) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out) ||
        qkv_row_stride % 8 || k_row_stride % 8 || v_row_stride % 8)
        return fail(SA_ERR_ALIGN, "sa_rope_qkv_bf16: tensors must be 16-byte aligned with row strides %% 8 == 0");
    if (rows == 0) return SA_OK;
    const int64_t work = static_cast<int64_t>(rows) * (num_heads + 2 * num_kv_heads) * (head_dim / 16);
    rope_qkv_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(qkv), qkv_row_stride, rows, num_heads, num_kv_heads, head_dim, cos_sin, pos0,
        static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_out), k_row_stride, static_cast<uint16_t*>(v_out),
        v_row_stride);
    return check_launch("rope_qkv_kernel");
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
