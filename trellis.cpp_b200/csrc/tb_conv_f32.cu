// fp32-operand submanifold conv on CUDA cores (FFMA, fp32 accumulation).
//
// The precision mode of the reference's g_sparse_cast_f32 / --f32 switch
// (src/sparse.cpp:16-19, src/trellis_cli.cpp:63), where f16 weights are cast to f32 and
// multiplied with f32 activations. Same math as src/sparse.cpp:64-79: per output row,
// bias + sum over the 27 taps of W_t . x[nbr], absent taps reading zero.
//
// Tiling: a block computes 32 output rows x 64 output channels. For each tap it gathers
// the 32 neighbor rows, 32 channels at a time, into shared memory next to the matching
// 64x32 weight slice, and every thread accumulates 1 row x 8 channels in registers.
#include "tb_common.cuh"

namespace {

constexpr int BR = 32;   // rows per block
constexpr int BC = 64;   // output channels per block
constexpr int BK = 32;   // input channels per step

__global__ void __launch_bounds__(256)
k_submconv_f32(const int32_t* __restrict__ nbr, int64_t n, int64_t row0, int64_t row_end,
               const float* __restrict__ feats, int ci,
               const float* __restrict__ w, const float* __restrict__ bias, int co, int epi,
               float* __restrict__ out) {
    __shared__ float xs[BR][BK + 1];
    __shared__ float ws[BC][BK + 1];
    __shared__ int32_t rows[BR];
    const int tx = threadIdx.x & 7;          // channel group: o = o0 + tx + 8*j
    const int ty = threadIdx.x >> 3;         // row within block
    const int64_t r0 = row0 + (int64_t)blockIdx.x * BR;
    const int o0 = blockIdx.y * BC;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;

    for (int t = 0; t < 27; ++t) {
        __syncthreads();
        if (threadIdx.x < BR) {
            const int64_t r = r0 + threadIdx.x;
            rows[threadIdx.x] = r < n ? nbr[(int64_t)t * n + r] : (int32_t)n;
        }
        __syncthreads();
        for (int k0 = 0; k0 < ci; k0 += BK) {
            // gather 32 rows x 32 channels (zero for absent rows / channel tail)
            for (int idx = threadIdx.x; idx < BR * BK; idx += blockDim.x) {
                const int r = idx / BK, k = idx % BK;
                const int32_t src = rows[r];
                xs[r][k] = (src != (int32_t)n && k0 + k < ci) ? feats[(int64_t)src * ci + k0 + k] : 0.f;
            }
            for (int idx = threadIdx.x; idx < BC * BK; idx += blockDim.x) {
                const int o = idx / BK, k = idx % BK;
                ws[o][k] = (o0 + o < co && k0 + k < ci) ? w[((int64_t)(o0 + o) * 27 + t) * ci + k0 + k] : 0.f;
            }
            __syncthreads();
#pragma unroll 8
            for (int k = 0; k < BK; ++k) {
                const float xv = xs[ty][k];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(xv, ws[tx + 8 * j][k], acc[j]);
            }
            __syncthreads();
        }
    }
    const int64_t r = r0 + ty;
    if (r >= row_end) return;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int o = o0 + tx + 8 * j;
        if (o >= co) continue;
        float v = acc[j] + (bias ? bias[o] : 0.f);
        if (epi == TB_EPI_SILU) v = tb_silu(v);
        out[r * co + o] = v;
    }
}

}  // namespace

tb_status tb_conv_f32_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                             const float* feats, int ci, const float* weight, const float* bias, int co,
                             tb_epilogue epi, float* out) {
    dim3 grid((unsigned)((nrows + BR - 1) / BR), (unsigned)((co + BC - 1) / BC));
    k_submconv_f32<<<grid, 256, 0, ctx->stream>>>(nbr, n, row0, row0 + nrows, feats, ci, weight, bias, co, (int)epi, out);
    TB_LAUNCH_CHECK(ctx, "k_submconv_f32");
    return TB_OK;
}
