// fp32-operand submanifold conv on CUDA cores (FFMA, fp32 accumulation).
//
// The precision mode of the reference's g_sparse_cast_f32 / --f32 switch
// (src/sparse.cpp:16-19, src/trellis_cli.cpp:63), where f16 weights are cast to f32 and
// multiplied with f32 activations. Same math as src/sparse.cpp:64-79: per output row,
// bias + sum over the 27 taps of W_t . x[nbr], absent taps reading zero.
//
// Tiling: a block of 256 threads computes 64 output rows x 64 output channels; each thread
// holds a 4-row x 4-channel register tile. For each tap the block gathers its 64 neighbor rows,
// up to 32 input channels at a time, into shared memory transposed ([k][row]) next to the
// matching weight slice ([k][o]), so every k step is two 16-byte shared loads feeding 16 FMAs;
// the next step's gather is in flight while the current step computes.
// Each output element accumulates its taps in ascending order and, within a tap, its input
// channels in ascending order, whichever block or range computes it.
#include "tb_common.cuh"

namespace {

constexpr int BR = 64;   // rows per block
constexpr int BC = 64;   // output channels per block
constexpr int BK = 32;   // input channels per step
static_assert(BR == BC && BR * BK == 8 * 256, "eight staged elements per thread of each operand");

// Per step (tap t, input-channel block k0) every thread stages 8 gathered inputs and 8 weights;
// the next step's are loaded into registers while the current step's FMAs run, so the gathers'
// latency overlaps the arithmetic instead of adding up over the 27 * Ci/32 steps.
__global__ void __launch_bounds__(256)
k_submconv_f32(const int32_t* __restrict__ nbr, int64_t n, int64_t row0, int64_t row_end,
               const float* __restrict__ feats, int ci,
               const float* __restrict__ w, const float* __restrict__ bias, int co, int epi,
               float* __restrict__ out) {
    // rows padded by 4 floats: the transposing stores (consecutive threads, consecutive k) spread
    // over 8 banks instead of one, and every row stays 16-byte aligned for the float4 reads
    __shared__ __align__(16) float xs[BK][BR + 4];     // gathered inputs, transposed
    __shared__ __align__(16) float ws[BK][BC + 4];     // weight slice of one tap, [k][o]
    __shared__ int32_t rows[27][BR];
    const int tr = threadIdx.x >> 4;               // row group: rows 4 tr .. 4 tr + 3
    const int tc = threadIdx.x & 15;               // channel group: channels 4 tc .. 4 tc + 3
    const int64_t r0 = row0 + (int64_t)blockIdx.x * BR;
    const int o0 = blockIdx.y * BC;
    // all 27 taps' neighbor rows of the block's 64 rows, once
    for (int idx = threadIdx.x; idx < 27 * BR; idx += blockDim.x) {
        const int t = idx / BR, r = idx % BR;
        const int64_t rr = r0 + r;
        rows[t][r] = rr < row_end ? nbr[(int64_t)t * n + rr] : (int32_t)n;
    }
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    const int nkb = (ci + BK - 1) / BK;
    const int nsteps = 27 * nkb;
    // this thread's 8 staged elements of each operand: element e at flat index threadIdx.x + 256 e
    // of the [BR x BK] gather ([r][k]) and of the [BC x BK] weight slice ([o][k])
    float xr[8], wr[8];
    auto load_step = [&](int st) {
        const int t = st / nkb, k0 = (st % nkb) * BK;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int idx = threadIdx.x + 256 * e;
            const int r = idx / BK, k = idx % BK;
            const int32_t src = rows[t][r];
            xr[e] = (src != (int32_t)n && k0 + k < ci) ? __ldg(feats + (int64_t)src * ci + k0 + k) : 0.f;
            const int o = idx / BK;
            wr[e] = (o0 + o < co && k0 + k < ci) ? __ldg(w + ((int64_t)(o0 + o) * 27 + t) * ci + k0 + k) : 0.f;
        }
    };
    load_step(0);
    for (int st = 0; st < nsteps; ++st) {
        __syncthreads();                           // the previous step's FMAs are done with xs / ws
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int idx = threadIdx.x + 256 * e;
            const int r = idx / BK, k = idx % BK;
            xs[k][r] = xr[e];
            ws[k][r] = wr[e];                      // BR == BC: the weight slice's o is the same index
        }
        __syncthreads();
        if (st + 1 < nsteps) load_step(st + 1);    // in flight during this step's FMAs
#pragma unroll 8
        for (int k = 0; k < BK; ++k) {
            const float4 xv = *reinterpret_cast<const float4*>(&xs[k][4 * tr]);
            const float4 wv = *reinterpret_cast<const float4*>(&ws[k][4 * tc]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
            const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wa[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t r = r0 + 4 * tr + i;
        if (r >= row_end) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + 4 * tc + j;
            if (o >= co) continue;
            float v = acc[i][j] + (bias ? bias[o] : 0.f);
            if (epi == TB_EPI_SILU) v = tb_silu(v);
            out[r * co + o] = v;
        }
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
