// Sparse 2x subdivide, channel-to-spatial gather and the standalone bias/activation pass.
//
// tb_subdivide replaces the host octant loop of sparse_c2s (src/sparse.cpp:205-222):
// parents in order, octants ascending, child (2x+(o&1), 2y+((o>>1)&1), 2z+((o>>2)&1)),
// gidx = o + 8i, mstart[i] = first child of parent i. The output order is fixed by a
// prefix sum over the per-parent child counts, so the result is identical to the
// sequential loop. Three kernels: per-block counts, a scan of the block totals, then each
// block rescans its parents and writes children.
#include "tb_common.cuh"
#include "tb_scan.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace {

constexpr int kSubThreads = 256;
constexpr int kPerThread = 4;
constexpr int kPerBlock = kSubThreads * kPerThread;   // parents per block

__device__ __forceinline__ uint32_t parent_bits(const uint8_t* __restrict__ mask, int64_t i) {
    const uint8_t* m = mask + 8 * i;
    uint32_t b = 0;
    if ((reinterpret_cast<uintptr_t>(m) & 7) == 0) {
        const uint2 v = *reinterpret_cast<const uint2*>(m);
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            b |= (((v.x >> (8 * o)) & 0xFF) != 0) << o;
            b |= (((v.y >> (8 * o)) & 0xFF) != 0) << (o + 4);
        }
    } else {
#pragma unroll
        for (int o = 0; o < 8; ++o) b |= (m[o] != 0) << o;
    }
    return b;
}

__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t* total) {
    return tb_scan::block_exclusive_scan<kSubThreads>(v, total);
}

__global__ void k_sub_count(const uint8_t* __restrict__ mask, int64_t n, int64_t* __restrict__ block_sums) {
    const int64_t base = (int64_t)blockIdx.x * kPerBlock + (int64_t)threadIdx.x * kPerThread;
    int64_t c = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j)
        if (base + j < n) c += __popc(parent_bits(mask, base + j));
    int64_t total;
    block_exclusive_scan(c, &total);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

__global__ void k_sub_emit(const int32_t* __restrict__ coords, int64_t n, int stride,
                           const uint8_t* __restrict__ mask, const int64_t* __restrict__ block_off,
                           int32_t* __restrict__ child, int32_t* __restrict__ gidx,
                           int32_t* __restrict__ mstart, int64_t max_children) {
    const int64_t base = (int64_t)blockIdx.x * kPerBlock + (int64_t)threadIdx.x * kPerThread;
    uint32_t bits[kPerThread];
    int64_t c = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        bits[j] = base + j < n ? parent_bits(mask, base + j) : 0u;
        c += __popc(bits[j]);
    }
    int64_t total;
    int64_t m = block_exclusive_scan(c, &total) + block_off[blockIdx.x];
    const int off = stride == 4 ? 1 : 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
        const int64_t i = base + j;
        if (i >= n) break;
        if (mstart) mstart[i] = (int32_t)m;
        const int32_t* pc = coords + i * stride;
        const int32_t b = stride == 4 ? pc[0] : 0;
        const int32_t x = pc[off], y = pc[off + 1], z = pc[off + 2];
        for (int o = 0; o < 8; ++o) {
            if (!((bits[j] >> o) & 1u)) continue;
            if (m < max_children) {
                int32_t* d = child + m * stride;
                if (stride == 4) d[0] = b;
                d[off] = 2 * x + (o & 1);
                d[off + 1] = 2 * y + ((o >> 1) & 1);
                d[off + 2] = 2 * z + ((o >> 2) & 1);
                if (gidx) gidx[m] = (int32_t)(o + 8 * i);
            }
            ++m;
        }
    }
}

__global__ void k_sub_finish(int32_t* __restrict__ mstart, int64_t n, const int64_t* __restrict__ grand) {
    if (mstart) mstart[n] = (int32_t)*grand;
}

template <typename V>
__global__ void k_row_gather(const V* __restrict__ src, const int32_t* __restrict__ gidx, int64_t m,
                             int64_t vec_per_row, V* __restrict__ out) {
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= m) return;
    const V* s = src + (int64_t)gidx[warp] * vec_per_row;
    V* d = out + warp * vec_per_row;
    for (int64_t k = lane; k < vec_per_row; k += 32) d[k] = s[k];
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__global__ void k_bias_act(T* __restrict__ x, int64_t total, int c, const float* __restrict__ bias, int epi) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (; i < total; i += stride) {
        float v = to_f<T>(x[i]) + (bias ? bias[i % c] : 0.f);
        if (epi == TB_EPI_SILU) v = tb_silu(v);
        x[i] = from_f<T>(v);
    }
}

}  // namespace

extern "C" tb_status tb_subdivide(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                                  const uint8_t* mask, int32_t* child_coords, int32_t* gidx,
                                  int32_t* mstart, int64_t max_children, int64_t* m_out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (!m_out || n < 0 || max_children < 0 || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_subdivide: bad arguments");
    *m_out = 0;
    if (n >= (int64_t)INT32_MAX / 8) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_subdivide: 8n must fit in int32 (gidx)");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (n == 0) {
        if (mstart) TB_CUDA_TRY(ctx, cudaMemsetAsync(mstart, 0, sizeof(int32_t), ctx->stream));
        TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        return TB_OK;
    }
    if (!coords || !mask || (max_children > 0 && !child_coords))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_subdivide: null pointer");
    const int64_t nb = (n + kPerBlock - 1) / kPerBlock;
    tb_status s = tb_ensure(ctx, &ctx->ws, &ctx->ws_bytes, sizeof(int64_t) * (size_t)(nb + 2), "subdivide scan");
    if (s != TB_OK) return s;
    int64_t* sums = reinterpret_cast<int64_t*>(ctx->ws);
    int64_t* grand = sums + nb;
    k_sub_count<<<(unsigned)nb, kSubThreads, 0, ctx->stream>>>(mask, n, sums);
    TB_LAUNCH_CHECK(ctx, "k_sub_count");
    tb_scan::k_scan_block_totals<kSubThreads, kPerThread><<<1, kSubThreads, 0, ctx->stream>>>(sums, nb, grand);
    TB_LAUNCH_CHECK(ctx, "k_scan_block_totals");
    k_sub_emit<<<(unsigned)nb, kSubThreads, 0, ctx->stream>>>(coords, n, coord_stride, mask, sums, child_coords,
                                                              gidx, mstart, max_children);
    TB_LAUNCH_CHECK(ctx, "k_sub_emit");
    k_sub_finish<<<1, 1, 0, ctx->stream>>>(mstart, n, grand);
    TB_LAUNCH_CHECK(ctx, "k_sub_finish");
    int64_t m = 0;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(&m, grand, sizeof(m), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    *m_out = m;
    if (m > max_children)
        return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_subdivide: more children than max_children (M written to m_out)");
    return TB_OK;
}

extern "C" tb_status tb_c2s_gather(tb_ctx* ctx, const void* src, const int32_t* gidx, int64_t m, int c,
                                   tb_dtype dtype, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (m < 0 || c <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_c2s_gather: m < 0 or c <= 0");
    if (m == 0) return TB_OK;
    if (!src || !gidx || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_c2s_gather: null pointer");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int64_t row_bytes = (int64_t)c * (int64_t)tb_dtype_size(dtype);
    const unsigned blocks = (unsigned)((m * 32 + 255) / 256);
    const bool al16 = tb_aligned16(src) && tb_aligned16(out);
    if (row_bytes % 16 == 0 && al16) {
        k_row_gather<uint4><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<const uint4*>(src), gidx, m,
                                                             row_bytes / 16, reinterpret_cast<uint4*>(out));
    } else if (row_bytes % 4 == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 3) == 0) {
        k_row_gather<uint32_t><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<const uint32_t*>(src), gidx, m,
                                                                row_bytes / 4, reinterpret_cast<uint32_t*>(out));
    } else {
        k_row_gather<uint16_t><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<const uint16_t*>(src), gidx, m,
                                                                row_bytes / 2, reinterpret_cast<uint16_t*>(out));
    }
    TB_LAUNCH_CHECK(ctx, "k_row_gather");
    return TB_OK;
}

extern "C" tb_status tb_bias_act(tb_ctx* ctx, void* x, int64_t n, int c, const float* bias, tb_dtype dtype,
                                 tb_epilogue epi) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || c <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_bias_act: n < 0 or c <= 0");
    if (n == 0) return TB_OK;
    if (!x) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_bias_act: null x");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int64_t total = n * c;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, (int64_t)ctx->num_sms * 32);
    if (dtype == TB_F32)
        k_bias_act<float><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<float*>(x), total, c, bias, epi);
    else if (dtype == TB_F16)
        k_bias_act<__half><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<__half*>(x), total, c, bias, epi);
    else
        k_bias_act<__nv_bfloat16><<<blocks, 256, 0, ctx->stream>>>(reinterpret_cast<__nv_bfloat16*>(x), total, c,
                                                                     bias, epi);
    TB_LAUNCH_CHECK(ctx, "k_bias_act");
    return TB_OK;
}
