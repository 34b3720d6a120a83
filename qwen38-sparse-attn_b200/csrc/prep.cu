// Memory-bound preparation kernels: block means (kernel a), e4m3 quantisation (row-major, or
// transposed into the V^T layout of the reference's pre-quantised inputs) and absmax reductions.  All are HBM-streaming kernels: 16-byte vector loads along head_dim,
// coalesced across a warp, rows walked by each thread with several loads in flight.
#include <algorithm>

#include "sa_common.cuh"

namespace sa {
namespace {

// One CTA per (block b, group of heads).  threadIdx.x -> (head in group, 16-byte column chunk),
// threadIdx.y -> row group: rows lo+ty, lo+ty+RG, ... are summed in order by each thread and the
// RG partial sums are added in row-group order (RG = 1 gives a strictly sequential row sum).
// Row r of x is at rm.offset(r, xrs) (contiguous, or a paged cache with rm.row0 = pos0).
__global__ void __launch_bounds__(512, 2) block_means_kernel(const uint16_t* __restrict__ x, RowMap rm, int64_t xrs, int64_t xhs, int n, int heads,
                                   int D, int pos0, int block, int b0, int heads_per_cta, float* __restrict__ out,
                                   int64_t ohs, int64_t obs, int out_block0, uint8_t* __restrict__ q8,
                                   int64_t q8rs, int64_t q8hs, const float* __restrict__ inv_scale, int iss,
                                   int fixed_divisor) {
    // a one-pass selection launched next may start its query pooling now (it waits for this kernel's
    // block means before it reads them)
    grid_dependents_launch();
    extern __shared__ float partial[];          // [RG-1][blockDim.x][8]
    const int cols = D >> 3;
    const int tx = threadIdx.x, ty = threadIdx.y, RG = blockDim.y;
    const int hl = tx / cols, c = tx - hl * cols;
    const int h = blockIdx.y * heads_per_cta + hl;
    const int b = b0 + blockIdx.x;
    const bool active = hl < heads_per_cta && h < heads;
    const int lo = max(pos0, b * block) - pos0;
    const int hi = min(pos0 + n, (b + 1) * block) - pos0;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (active) {
        const uint16_t* src = x + static_cast<int64_t>(h) * xhs + c * 8;
        const float inv = q8 ? inv_scale[h * iss] : 0.f;
        uint8_t* dst = q8 ? q8 + static_cast<int64_t>(h) * q8hs + c * 8 : nullptr;
        // 8 rows per batch: all 8 loads are issued before the first is used (8 x 16 B in flight per
        // thread); the rows are still added in order
        constexpr int BATCH = 8;
        for (int base = lo + ty; base < hi; base += BATCH * RG) {
            uint4 v[BATCH];
#pragma unroll
            for (int k = 0; k < BATCH; ++k) {
                const int r = base + k * RG;
                v[k] = r < hi ? ld_stream(src + rm.offset(r, xrs)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < BATCH; ++k) {
                const int r = base + k * RG;
                if (r >= hi) break;
                float f[8];
                unpack8(v[k], f);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] += f[i];
                if (dst) *reinterpret_cast<uint2*>(dst + static_cast<int64_t>(r) * q8rs) = quant8(f, inv, SA_QUANT_MUL_BF16);
            }
        }
    }
    if (RG > 1) {
        if (ty > 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) partial[((ty - 1) * blockDim.x + tx) * 8 + i] = acc[i];
        }
        __syncthreads();
        if (ty != 0) return;
        for (int g = 1; g < RG; ++g) {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += partial[((g - 1) * blockDim.x + tx) * 8 + i];
        }
    }
    if (!active) return;
    const float cnt = static_cast<float>(fixed_divisor > 0 ? fixed_divisor : max(hi - lo, 1));
    float* o = out + static_cast<int64_t>(h) * ohs + static_cast<int64_t>(b - out_block0) * obs + c * 8;
    float4 m0 = make_float4(__fdiv_rn(acc[0], cnt), __fdiv_rn(acc[1], cnt), __fdiv_rn(acc[2], cnt), __fdiv_rn(acc[3], cnt));
    float4 m1 = make_float4(__fdiv_rn(acc[4], cnt), __fdiv_rn(acc[5], cnt), __fdiv_rn(acc[6], cnt), __fdiv_rn(acc[7], cnt));
    if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
        reinterpret_cast<float4*>(o)[0] = m0;
        reinterpret_cast<float4*>(o)[1] = m1;
    } else {
        o[0] = m0.x; o[1] = m0.y; o[2] = m0.z; o[3] = m0.w; o[4] = m1.x; o[5] = m1.y; o[6] = m1.z; o[7] = m1.w;
    }
}

// Elementwise e4m3 quantisation, row-major output.  threadIdx.x (with blockIdx.y) picks a 16-byte
// column chunk hc = (head, 8 elements) of the row, fixed for the thread; rows are walked in
// batches of 8 blockDim.y apart, all 8 loads issued before the first is used.  Row r of x is at
// rm.offset(r, xrs) (contiguous or paged).
__global__ void __launch_bounds__(256) quant_rows_kernel(const uint16_t* __restrict__ x, RowMap rm, int64_t xrs, int64_t xhs,
                                                         int rows, int heads, int D, const float* __restrict__ scale,
                                                         int iss, int mode, uint8_t* __restrict__ out, int64_t ors,
                                                         int64_t ohs) {
    constexpr int BATCH = 8;
    const int cols = D >> 3;
    const int HC = heads * cols;
    const int rstep = blockDim.y * BATCH;
    for (int hc = blockIdx.y * blockDim.x + threadIdx.x; hc < HC; hc += gridDim.y * blockDim.x) {
        const int h = hc / cols, c = hc - h * cols;
        const uint16_t* src = x + static_cast<int64_t>(h) * xhs + c * 8;
        uint8_t* dst = out + static_cast<int64_t>(h) * ohs + c * 8;
        const float sc = scale[h * iss];
        for (int r0 = blockIdx.x * rstep + threadIdx.y; r0 < rows; r0 += gridDim.x * rstep) {
            uint4 v[BATCH];
#pragma unroll
            for (int k = 0; k < BATCH; ++k) {
                const int r = r0 + k * static_cast<int>(blockDim.y);
                v[k] = r < rows ? ld_stream(src + rm.offset(r, xrs)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < BATCH; ++k) {
                const int r = r0 + k * static_cast<int>(blockDim.y);
                if (r >= rows) break;
                float f[8];
                unpack8(v[k], f);
                *reinterpret_cast<uint2*>(dst + static_cast<int64_t>(r) * ors) = quant8(f, sc, mode);
            }
        }
    }
}

// Tile transpose [64 rows x D] of one head -> out[h][d][r0..r0+63].  ELEM_OUT = 1 (e4m3).
template <int ELEM_OUT>
__global__ void transpose_kernel(const uint16_t* __restrict__ x, int64_t xrs, int64_t xhs, int rows, int D,
                                 const float* __restrict__ scale, int iss, int mode, uint8_t* __restrict__ out,
                                 int64_t ohs, int64_t ods, int rows_pad) {
    constexpr int TR = 64;
    extern __shared__ uint8_t tile[];           // [D][TR * ELEM_OUT + 16] bytes
    const int pitch = TR * ELEM_OUT + 16;
    const int h = blockIdx.y;
    const int r0 = blockIdx.x * TR;
    const int cols = D >> 3;
    const float sc = ELEM_OUT == 1 ? scale[h * iss] : 1.f;
    for (int i = threadIdx.x; i < TR * cols; i += blockDim.x) {
        const int rr = i / cols, c = i - rr * cols;
        const int r = r0 + rr;
        float f[8];
        if (r < rows) {
            unpack8(ld_stream(x + static_cast<int64_t>(r) * xrs + static_cast<int64_t>(h) * xhs + c * 8), f);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int d = c * 8 + j;
            if (ELEM_OUT == 1) {
                tile[d * pitch + rr] = static_cast<uint8_t>(pack_e4m3x2(scale_value(f[j], sc, mode), 0.f) & 0xFF);
            } else {
                reinterpret_cast<uint16_t*>(tile + d * pitch)[rr] = static_cast<uint16_t>(pack_bf16x2(f[j], 0.f) & 0xFFFF);
            }
        }
    }
    __syncthreads();
    constexpr int CHUNKS = TR * ELEM_OUT / 16;  // 16-byte chunks per output row
    for (int i = threadIdx.x; i < D * CHUNKS; i += blockDim.x) {
        const int d = i / CHUNKS, cc = i - d * CHUNKS;
        const int rbyte = cc * 16;
        if (r0 + rbyte / ELEM_OUT >= rows_pad) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(tile + d * pitch + rbyte);
        *reinterpret_cast<uint4*>(out + (static_cast<int64_t>(h) * ohs + static_cast<int64_t>(d) * ods +
                                         r0) * ELEM_OUT + rbyte) = v;
    }
}

__global__ void absmax_kernel(const uint16_t* __restrict__ x, RowMap rm, int64_t xrs, int64_t xhs, int rows, int heads,
                              int D, int per_head, float* __restrict__ out) {
    // grid.y = head; grid.x strides over rows
    const int h = blockIdx.y;
    const int cols = D >> 3;
    uint32_t m = 0;   // bit pattern of a non-negative float: integer order == float order
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < static_cast<int64_t>(rows) * cols;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        const int c = static_cast<int>(i - r * cols);
        const uint4 v = ld_stream(x + rm.offset(static_cast<int>(r), xrs) + static_cast<int64_t>(h) * xhs + c * 8);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            m = max(m, (w[j] << 16) & 0x7FFFFFFFu);
            m = max(m, w[j] & 0x7FFF0000u);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(out + (per_head ? h : 0)), m);
}

}  // namespace
}  // namespace sa

namespace sa {
namespace {

int check_pages(const char* who, const int32_t* pages, int page, int64_t page_stride) {
    if (!pages || page <= 0) return fail(SA_ERR_ARG, "%s: page table and page_size > 0 required", who);
    if (page_stride % 8) return fail(SA_ERR_ALIGN, "%s: page_stride %% 8 != 0", who);
    return SA_OK;
}

int block_means(const char* who, const void* x, RowMap rm, int64_t x_row_stride, int64_t x_head_stride, int n,
                int heads, int head_dim, int pos0, int block, float* out, int64_t out_head_stride,
                int64_t out_block_stride, int out_block0, uint8_t* q8, int64_t q8_row_stride, int64_t q8_head_stride,
                const float* inv_scale, int inv_scale_stride, int fixed_divisor, void* stream) {
    if (n < 0 || heads <= 0 || block <= 0 || pos0 < 0) return fail(SA_ERR_ARG, "%s: bad sizes", who);
    if (head_dim % 8 || head_dim > 8 * 256) return fail(SA_ERR_UNSUPPORTED, "%s: head_dim %d", who, head_dim);
    if (!x || !out) return fail(SA_ERR_ARG, "%s: null pointer", who);
    if (!aligned16(x) || x_row_stride % 8 || x_head_stride % 8)
        return fail(SA_ERR_ALIGN, "%s: x must be 16-byte aligned with strides %% 8 == 0", who);
    if (q8 && (!inv_scale || (reinterpret_cast<uintptr_t>(q8) & 7) || q8_row_stride % 8 || q8_head_stride % 8))
        return fail(SA_ERR_ALIGN, "%s: q8 needs inv_scale, 8-byte alignment, strides %% 8 == 0", who);
    if (n == 0) return SA_OK;
    const int b0 = pos0 / block;
    const int b1 = (pos0 + n + block - 1) / block;
    if (b0 < out_block0) return fail(SA_ERR_ARG, "%s: first block %d < out_block0 %d", who, b0, out_block0);
    const int nblk = b1 - b0;
    int hpc, rg;
    block_means_shape(nblk, heads, head_dim, block, &hpc, &rg);
    const int tx = hpc * (head_dim / 8);
    const int nhg = (heads + hpc - 1) / hpc;
    dim3 grid(nblk, nhg), blk(tx, rg);
    const size_t smem = rg > 1 ? static_cast<size_t>(rg - 1) * tx * 8 * sizeof(float) : 0;   // <= 15.5 KB
    block_means_kernel<<<grid, blk, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x), rm, x_row_stride, x_head_stride, n, heads, head_dim, pos0, block, b0, hpc,
        out, out_head_stride, out_block_stride, out_block0, q8, q8_row_stride, q8_head_stride, inv_scale,
        inv_scale_stride, fixed_divisor);
    return check_launch("block_means_kernel");
}

int quantize_rows(const char* who, const void* x, RowMap rm, int64_t x_row_stride, int64_t x_head_stride, int rows,
                  int heads, int head_dim, const float* scale, int scale_stride, int mode, uint8_t* out,
                  int64_t out_row_stride, int64_t out_head_stride, cudaStream_t s) {
    if ((reinterpret_cast<uintptr_t>(out) & 7) || out_row_stride % 8 || out_head_stride % 8)
        return fail(SA_ERR_ALIGN, "%s: out must be 8-byte aligned with strides %% 8 == 0", who);
    if (rows == 0) return SA_OK;
    const int HC = heads * (head_dim / 8);
    const int bx = std::min(HC, 128);
    const dim3 blk(bx, 256 / bx);
    const int gy = (HC + bx - 1) / bx;
    const int per_cta = static_cast<int>(blk.y) * 8;
    const int gx = std::max(1, std::min((rows + per_cta - 1) / per_cta, (8 * num_sms() + gy - 1) / gy));
    quant_rows_kernel<<<dim3(gx, gy), blk, 0, s>>>(static_cast<const uint16_t*>(x), rm, x_row_stride, x_head_stride,
                                                   rows, heads, head_dim, scale, scale_stride, mode, out,
                                                   out_row_stride, out_head_stride);
    return check_launch("quant_rows_kernel");
}

int absmax(const char* who, const void* x, RowMap rm, int64_t x_row_stride, int64_t x_head_stride, int rows, int heads,
           int head_dim, int per_head, float* out, void* stream) {
    if (rows < 0 || heads <= 0 || head_dim % 8) return fail(SA_ERR_ARG, "%s: bad sizes", who);
    if (!x || !out) return fail(SA_ERR_ARG, "%s: null pointer", who);
    if (!aligned16(x) || x_row_stride % 8 || x_head_stride % 8) return fail(SA_ERR_ALIGN, "%s: alignment", who);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float) * (per_head ? heads : 1), s);
    if (e != cudaSuccess) return fail(SA_ERR_CUDA, "%s: %s", who, cudaGetErrorString(e));
    if (rows == 0) return SA_OK;
    const int64_t per = static_cast<int64_t>(rows) * (head_dim / 8);
    const int bx = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((per + 255) / 256, (8ll * num_sms()) / heads + 1)));
    absmax_kernel<<<dim3(bx, heads), 256, 0, s>>>(static_cast<const uint16_t*>(x), rm, x_row_stride, x_head_stride,
                                                 rows, heads, head_dim, per_head, out);
    return check_launch("absmax_kernel");
}

}  // namespace
}  // namespace sa

using namespace sa;

extern "C" int sa_block_means_bf16(const void* x, int64_t x_row_stride, int64_t x_head_stride, int n, int heads,
                                   int head_dim, int pos0, int block, float* out, int64_t out_head_stride,
                                   int64_t out_block_stride, int out_block0, uint8_t* q8, int64_t q8_row_stride,
                                   int64_t q8_head_stride, const float* inv_scale, int inv_scale_stride,
                                   int fixed_divisor, void* stream) {
    return block_means("sa_block_means_bf16", x, contiguous_rows(), x_row_stride, x_head_stride, n, heads, head_dim,
                       pos0, block, out, out_head_stride, out_block_stride, out_block0, q8, q8_row_stride,
                       q8_head_stride, inv_scale, inv_scale_stride, fixed_divisor, stream);
}

extern "C" int sa_block_means_paged_bf16(const void* cache, int64_t page_stride, int64_t row_stride,
                                         int64_t head_stride, const int32_t* page_table, int page_size, int n,
                                         int heads, int head_dim, int pos0, int block, float* out,
                                         int64_t out_head_stride, int64_t out_block_stride, int out_block0,
                                         void* stream) {
    const char* who = "sa_block_means_paged_bf16";
    if (int rc = check_pages(who, page_table, page_size, page_stride)) return rc;
    const RowMap rm{page_table, page_stride, page_size, pos0};
    return block_means(who, cache, rm, row_stride, head_stride, n, heads, head_dim, pos0, block, out, out_head_stride,
                       out_block_stride, out_block0, nullptr, 0, 0, nullptr, 0, 0, stream);
}

extern "C" int sa_quantize_e4m3(const void* x, int64_t x_row_stride, int64_t x_head_stride, int rows, int heads,
                                int head_dim, const float* scale, int scale_stride, int mode, uint8_t* out,
                                int64_t out_row_stride, int64_t out_head_stride, int transpose, int rows_pad,
                                void* stream) {
    if (rows < 0 || heads <= 0 || head_dim % 8) return fail(SA_ERR_ARG, "sa_quantize_e4m3: bad sizes");
    if (!x || !out || !scale) return fail(SA_ERR_ARG, "sa_quantize_e4m3: null pointer");
    if (mode < SA_QUANT_MUL || mode > SA_QUANT_DIV) return fail(SA_ERR_ARG, "sa_quantize_e4m3: bad mode %d", mode);
    if (!aligned16(x) || x_row_stride % 8 || x_head_stride % 8)
        return fail(SA_ERR_ALIGN, "sa_quantize_e4m3: x must be 16-byte aligned with strides % 8 == 0");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!transpose)
        return quantize_rows("sa_quantize_e4m3", x, contiguous_rows(), x_row_stride, x_head_stride, rows, heads,
                             head_dim, scale, scale_stride, mode, out, out_row_stride, out_head_stride, s);
    if (rows_pad < rows || rows_pad % 64 || !aligned16(out) || out_row_stride % 16 || out_head_stride % 16)
        return fail(SA_ERR_ALIGN, "sa_quantize_e4m3: transposed output needs rows_pad %% 64 == 0, 16-byte alignment");
    if (rows_pad == 0) return SA_OK;
    const size_t smem = static_cast<size_t>(head_dim) * (64 + 16);
    dim3 grid(rows_pad / 64, heads);
    transpose_kernel<1><<<grid, 256, smem, s>>>(static_cast<const uint16_t*>(x), x_row_stride, x_head_stride, rows,
                                                head_dim, scale, scale_stride, mode, out, out_head_stride,
                                                out_row_stride, rows_pad);
    return check_launch("transpose_kernel<e4m3>");
}

extern "C" int sa_quantize_paged_e4m3(const void* cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                      const int32_t* page_table, int page_size, int row0, int rows, int heads,
                                      int head_dim, const float* scale, int scale_stride, int mode, uint8_t* out,
                                      int64_t out_row_stride, int64_t out_head_stride, void* stream) {
    const char* who = "sa_quantize_paged_e4m3";
    if (rows < 0 || row0 < 0 || heads <= 0 || head_dim % 8) return fail(SA_ERR_ARG, "%s: bad sizes", who);
    if (!cache || !out || !scale) return fail(SA_ERR_ARG, "%s: null pointer", who);
    if (mode < SA_QUANT_MUL || mode > SA_QUANT_DIV) return fail(SA_ERR_ARG, "%s: bad mode %d", who, mode);
    if (int rc = check_pages(who, page_table, page_size, page_stride)) return rc;
    if (!aligned16(cache) || row_stride % 8 || head_stride % 8)
        return fail(SA_ERR_ALIGN, "%s: cache must be 16-byte aligned with strides %% 8 == 0", who);
    const RowMap rm{page_table, page_stride, page_size, row0};
    return quantize_rows(who, cache, rm, row_stride, head_stride, rows, heads, head_dim, scale, scale_stride, mode, out,
                         out_row_stride, out_head_stride, static_cast<cudaStream_t>(stream));
}

extern "C" int sa_absmax_bf16(const void* x, int64_t x_row_stride, int64_t x_head_stride, int rows, int heads,
                              int head_dim, int per_head, float* out, void* stream) {
    return absmax("sa_absmax_bf16", x, contiguous_rows(), x_row_stride, x_head_stride, rows, heads, head_dim, per_head,
                  out, stream);
}

extern "C" int sa_absmax_paged_bf16(const void* cache, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                    const int32_t* page_table, int page_size, int row0, int rows, int heads,
                                    int head_dim, int per_head, float* out, void* stream) {
    const char* who = "sa_absmax_paged_bf16";
    if (row0 < 0) return fail(SA_ERR_ARG, "%s: row0 < 0", who);
    if (int rc = check_pages(who, page_table, page_size, page_stride)) return rc;
    const RowMap rm{page_table, page_stride, page_size, row0};
    return absmax(who, cache, rm, row_stride, head_stride, rows, heads, head_dim, per_head, out, stream);
}
