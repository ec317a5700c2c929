// ConvNeXt tail of a sparse ConvNeXt block: out = x + Linear2(SiLU(Linear1(LN(h)))).
//
// Replaces the per-voxel part of trellis::sparse_convnext (src/sparse.cpp:124-133): after the
// submanifold conv h = conv(x), ggml_norm over the channels (eps 1e-6) with the affine
// norm.weight / norm.bias, mlp.0 (Linear C -> 4C, weight [4C][C], bias [4C]), SiLU, mlp.2
// (Linear 4C -> C, weight [C][4C], bias [C]) and the residual add of the block input x. The
// reference chunks this over voxels to bound its [4C, n] intermediates (src/sparse.cpp:94-118);
// here no intermediate leaves the SM.
//
// Tensor-core kernel (C in {64, 128, 256}, bf16 or f16 operands, fp32 accumulate): one CTA per
// SM walks 128-row tiles. Four row warps (thread = row) compute the LayerNorm in fp32 from h and
// write the normalised row, rounded to the operand type, into a 128-byte-swizzled shared-memory
// A tile. The hidden layer is processed 128 units at a time: the issuer thread streams the
// chunk's mlp.0 rows by TMA and runs tcgen05.mma into a 128-column TMEM accumulator; the row
// warps add the bias, apply SiLU, round and write the chunk into a second A tile; the issuer
// streams the matching mlp.2 columns and accumulates the 4C -> C product in a C-column TMEM
// accumulator. The row warps then add mlp.2's bias and the residual and write each row once.
//
// fp32 kernel (any C up to 1024, fp32 operands): one block per row on CUDA cores; it reads the
// weights once per row, so it is meant for the fp32 mode and small channel counts.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>

namespace {

using namespace tbtc;

constexpr int kRows = 128;           // rows per tile
constexpr int kHid = 128;            // hidden units per chunk
constexpr int kThreads = 5 * 32;     // row warps 0-3, issuer warp 4
// a1f w1f d1f w2f a2f g2d d2f d2e drain
constexpr int kNumBars = 9;

struct TailParams {
    const uint8_t* h;      // [N][C] conv output, h_kind
    const uint8_t* x;      // [N][C] block input, operand type
    const float* nw;       // [C]
    const float* nb;       // [C]
    const float* b1;       // [4C]
    const float* b2;       // [C]
    uint8_t* out;          // [N][C]
    int* err;
    int64_t n;
    int ntiles;
    int h_kind;            // 0 f32, 1 f16, 2 bf16
    int x_kind;            // 1 f16, 2 bf16
    int out_kind;          // 0 f32, 1 f16, 2 bf16
    uint32_t idesc1, idesc2;
    uint32_t tmem_cols;
};

__device__ __forceinline__ float load_val(const uint8_t* row, int j, int kind) {
    if (kind == 0) return reinterpret_cast<const float*>(row)[j];
    const uint16_t u = reinterpret_cast<const uint16_t*>(row)[j];
    if (kind == 2) return __uint_as_float((uint32_t)u << 16);
    return __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int kind) {
    if (kind == 2) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Eight consecutive values (16 bytes) of row r, K chunk kc (0..7 within a 64-wide K block) of a
// [128 rows][128 B] K-major block with the 128-byte swizzle: chunk kc sits at kc ^ (r & 7).
__device__ __forceinline__ void put16(uint8_t* blk, int r, int kc, uint4 v) {
    *reinterpret_cast<uint4*>(blk + r * 128 + ((kc ^ (r & 7)) << 4)) = v;
}

template <int C>
__global__ void __launch_bounds__(kThreads, 1)
k_convnext_tail(const __grid_constant__ CUtensorMap w1map, const __grid_constant__ CUtensorMap w2map,
                const TailParams p) {
    constexpr int KB1 = C / 64;                  // K blocks of the LN tile and of an mlp.0 chunk
    constexpr int NCH = 4 * C / kHid;            // hidden chunks
    constexpr uint32_t kBlk = kRows * 128;       // one [128 rows][128 B] block
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a1 = smem;                          // [KB1][128][128 B]
    uint8_t* a2 = a1 + KB1 * kBlk;               // [2][128][128 B]
    uint8_t* w1s = a2 + 2 * kBlk;                // [KB1][128 hidden][128 B]
    uint8_t* w2s = w1s + KB1 * kBlk;             // [2][C][128 B]
    uint64_t* bars = reinterpret_cast<uint64_t*>(w2s + 2 * C * 128);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kNumBars);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b0 = smem_u32(bars);
    const uint32_t a1f = b0, w1f = b0 + 8, d1f = b0 + 16, w2f = b0 + 24, a2f = b0 + 32, g2d = b0 + 40,
                   d2f = b0 + 48, d2e = b0 + 56, drain = b0 + 64;
    if (threadIdx.x == 0) {
        mbar_init(a1f, 4);
        mbar_init(w1f, 1);
        mbar_init(d1f, 1);
        mbar_init(w2f, 1);
        mbar_init(a2f, 4);
        mbar_init(g2d, 1);
        mbar_init(d2f, 1);
        mbar_init(d2e, 4);
        mbar_init(drain, 1);
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&w1map)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&w2map)) : "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_misc[0];

    if (warp == 4) {
        // ------------------------------------------------------------------ TMA + MMA issuer
        if (lane == 0) {
            bool ok = true;
            int t = 0, gc = 0;
            for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x, ++t) {
                for (int j = 0; j < NCH && ok; ++j, ++gc) {
                    // mlp.0 rows of this chunk (the previous GEMM1, the last reader, has completed:
                    // this thread waited for its commit before issuing GEMM2 below)
                    mbar_arrive_expect_tx(w1f, KB1 * kBlk);
                    for (int kb = 0; kb < KB1; ++kb)
                        tma_load_2d(smem_u32(w1s + kb * kBlk), &w1map, kb * 64, j * kHid, w1f);
                    if (j == 0 && !mbar_wait(a1f, (uint32_t)(t & 1), s_abort, p.err)) { ok = false; break; }
                    if (!mbar_wait(w1f, (uint32_t)(gc & 1), s_abort, p.err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kb = 0; kb < KB1; ++kb)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma(tmem, smem_desc<128>(smem_u32(a1 + kb * kBlk)) + 2 * k,
                                   smem_desc<128>(smem_u32(w1s + kb * kBlk)) + 2 * k, p.idesc1,
                                   (kb | k) ? 1u : 0u);
                    tc_commit(d1f);
                    // mlp.2 columns of this chunk, once the previous GEMM2 has read the old ones
                    if (gc > 0 && !mbar_wait(g2d, (uint32_t)((gc - 1) & 1), s_abort, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(w2f, 2u * C * 128u);
                    for (int kb = 0; kb < 2; ++kb)
                        tma_load_2d(smem_u32(w2s + kb * C * 128), &w2map, j * kHid + kb * 64, 0, w2f);
                    // the row warps have read D1 and written the chunk's activations
                    if (!mbar_wait(a2f, (uint32_t)(gc & 1), s_abort, p.err)) { ok = false; break; }
                    if (!mbar_wait(w2f, (uint32_t)(gc & 1), s_abort, p.err)) { ok = false; break; }
                    // the previous tile's output accumulator has been read
                    if (j == 0 && t > 0 && !mbar_wait(d2e, (uint32_t)((t - 1) & 1), s_abort, p.err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma(tmem + kHid, smem_desc<128>(smem_u32(a2 + kb * kBlk)) + 2 * k,
                                   smem_desc<128>(smem_u32(w2s + kb * C * 128)) + 2 * k, p.idesc2,
                                   (j | kb | k) ? 1u : 0u);
                    tc_commit(g2d);
                }
                if (ok) tc_commit(d2f);
            }
            // every MMA of this thread has finished before the TMEM is freed (also after an abort)
            tc_commit(drain);
            const long long t0 = clock64();
            while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) { }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ row warps
        const int r = warp * 32 + lane;                          // row in the tile = TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const size_t hsz = p.h_kind == 0 ? 4 : 2, osz = p.out_kind == 0 ? 4 : 2;
        int t = 0, gc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x, ++t) {
            const int64_t row = (int64_t)tile * kRows + r;
            const bool valid = row < p.n;
            // LayerNorm, warp-cooperative: the warp normalises its 32 rows eight at a time; lane l
            // holds channels 2l, 2l + 1 of each 64-channel block, so every load of a row is
            // coalesced, and writes them as one packed word into the swizzled A tile.
#pragma unroll 1
            for (int rb = 0; rb < 32; rb += 8) {
                float2 v[8][KB1];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int64_t rq = (int64_t)tile * kRows + warp * 32 + rb + q;
                    const bool vq = rq < p.n;
                    const uint8_t* hr = p.h + (size_t)(vq ? rq : 0) * C * hsz;
#pragma unroll
                    for (int k = 0; k < KB1; ++k) {
                        const int col = 64 * k + 2 * lane;
                        if (!vq) v[q][k] = make_float2(0.f, 0.f);
                        else if (p.h_kind == 0) v[q][k] = *reinterpret_cast<const float2*>(hr + (size_t)col * 4);
                        else {
                            const uint32_t u = *reinterpret_cast<const uint32_t*>(hr + (size_t)col * 2);
                            v[q][k] = make_float2(load_val(reinterpret_cast<const uint8_t*>(&u), 0, p.h_kind),
                                                  load_val(reinterpret_cast<const uint8_t*>(&u), 1, p.h_kind));
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    float s = 0.f;
#pragma unroll
                    for (int k = 0; k < KB1; ++k) s += v[q][k].x + v[q][k].y;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                    const float mean = s / C;
                    float s2 = 0.f;
#pragma unroll
                    for (int k = 0; k < KB1; ++k) {
                        const float dx = v[q][k].x - mean, dy = v[q][k].y - mean;
                        s2 = fmaf(dx, dx, fmaf(dy, dy, s2));
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
                    const float rstd = rsqrtf(s2 / C + 1e-6f);
                    const int rr = warp * 32 + rb + q;                     // row in the tile
                    const bool vq = (int64_t)tile * kRows + rr < p.n;
#pragma unroll
                    for (int k = 0; k < KB1; ++k) {
                        const int col = 64 * k + 2 * lane;
                        float y0 = 0.f, y1 = 0.f;
                        if (vq) {
                            y0 = (v[q][k].x - mean) * rstd * __ldg(p.nw + col) + __ldg(p.nb + col);
                            y1 = (v[q][k].y - mean) * rstd * __ldg(p.nw + col + 1) + __ldg(p.nb + col + 1);
                        }
                        // 4-byte word (lane & 3) of 16-byte chunk lane >> 2 of row rr in block k
                        uint8_t* blk = a1 + k * kBlk;
                        *reinterpret_cast<uint32_t*>(blk + rr * 128 + (((lane >> 2) ^ (rr & 7)) << 4) + (lane & 3) * 4) =
                            pack2(y0, y1, p.x_kind);
                    }
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(a1f);
            for (int j = 0; j < NCH; ++j, ++gc) {
                if (!mbar_wait(d1f, (uint32_t)(gc & 1), s_abort, p.err)) { ok = false; break; }
                tc_fence_after();
                // the previous GEMM2 has read the activation tile
                if (gc > 0 && !mbar_wait(g2d, (uint32_t)((gc - 1) & 1), s_abort, p.err)) { ok = false; break; }
#pragma unroll 1
                for (int c0 = 0; c0 < kHid; c0 += 16) {
                    uint32_t v[16];
                    TMEM_LD_X16(lane_base + (uint32_t)c0, v);
                    tmem_wait_ld();
                    float f[16], e[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q) f[q] = __uint_as_float(v[q]) + __ldg(p.b1 + j * kHid + c0 + q);
#pragma unroll
                    for (int q = 0; q < 16; ++q) e[q] = __expf(-f[q]);
#pragma unroll
                    for (int q = 0; q < 16; ++q) f[q] = __fdividef(f[q], 1.0f + e[q]);
                    uint32_t w[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) w[q] = pack2(f[2 * q], f[2 * q + 1], p.x_kind);
                    const int kc = c0 / 8;                       // 16-byte chunk index in the 128 units
                    put16(a2 + (kc >> 3) * kBlk, r, kc & 7, make_uint4(w[0], w[1], w[2], w[3]));
                    put16(a2 + ((kc + 1) >> 3) * kBlk, r, (kc + 1) & 7, make_uint4(w[4], w[5], w[6], w[7]));
                }
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a2f);
            }
            if (!ok) break;
            if (!mbar_wait(d2f, (uint32_t)(t & 1), s_abort, p.err)) { ok = false; break; }
            tc_fence_after();
            const uint8_t* xrow = p.x + (size_t)(valid ? row : 0) * C * 2;
            uint8_t* orow = p.out + (size_t)(valid ? row : 0) * C * osz;
#pragma unroll 1
            for (int c0 = 0; c0 < C; c0 += 32) {
                // the residual's 32 channels as four 16-byte loads, issued before the TMEM reads
                uint4 xv[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    xv[q] = valid ? *reinterpret_cast<const uint4*>(xrow + (size_t)(c0 + 8 * q) * 2) : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t v[16];
                    TMEM_LD_X16(lane_base + (uint32_t)(kHid + c0 + 16 * hh), v);
                    tmem_wait_ld();
                    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[2 * hh]);
                    float f[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q)
                        f[q] = __uint_as_float(v[q]) + __ldg(p.b2 + c0 + 16 * hh + q) +
                               load_val(reinterpret_cast<const uint8_t*>(xw), q, p.x_kind);
                    if (valid) store16(orow + (size_t)(c0 + 16 * hh) * osz, f, p.out_kind);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d2e);
        }
    }
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// fp32 tail, one block of 256 threads per row (any C <= 1024).
__global__ void __launch_bounds__(256)
k_convnext_tail_f32(const float* __restrict__ h, const float* __restrict__ x, const float* __restrict__ nw,
                    const float* __restrict__ nb, const float* __restrict__ w1, const float* __restrict__ b1,
                    const float* __restrict__ w2, const float* __restrict__ b2, float* __restrict__ out,
                    int64_t n, int c) {
    extern __shared__ float sh[];
    float* xl = sh;                 // [C]
    float* hid = sh + c;            // [4C]
    __shared__ float red[2][8];
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
    const float* hr = h + row * c;
    float s = 0.f;
    for (int k = tid; k < c; k += blockDim.x) s += hr[k];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[0][wid] = s;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += red[0][w];
    const float mean = tot / c;
    float s2 = 0.f;
    for (int k = tid; k < c; k += blockDim.x) { const float d = hr[k] - mean; s2 = fmaf(d, d, s2); }
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    if (lane == 0) red[1][wid] = s2;
    __syncthreads();
    float tot2 = 0.f;
    for (int w = 0; w < 8; ++w) tot2 += red[1][w];
    const float rstd = rsqrtf(tot2 / c + 1e-6f);
    for (int k = tid; k < c; k += blockDim.x) xl[k] = (hr[k] - mean) * rstd * nw[k] + nb[k];
    __syncthreads();
    for (int u = tid; u < 4 * c; u += blockDim.x) {
        const float* wr = w1 + (int64_t)u * c;
        float a = b1[u];
        for (int k = 0; k < c; ++k) a = fmaf(wr[k], xl[k], a);
        hid[u] = tb_silu(a);
    }
    __syncthreads();
    for (int o = tid; o < c; o += blockDim.x) {
        const float* wr = w2 + (int64_t)o * 4 * c;
        float a = b2[o];
        for (int k = 0; k < 4 * c; ++k) a = fmaf(wr[k], hid[k], a);
        out[row * c + o] = a + x[row * c + o];
    }
}

template <int C>
tb_status launch_tail_tc(tb_ctx* ctx, int64_t n, const void* h, tb_dtype h_dtype, const void* x, const float* nw,
                         const float* nb, const void* w1, const float* b1, const void* w2, const float* b2,
                         tb_dtype dtype, tb_dtype out_dtype, void* out) {
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    const auto kind = [](tb_dtype d) { return d == TB_F32 ? 0 : (d == TB_F16 ? 1 : 2); };
    TailParams p{};
    p.h = reinterpret_cast<const uint8_t*>(h);
    p.x = reinterpret_cast<const uint8_t*>(x);
    p.nw = nw;
    p.nb = nb;
    p.b1 = b1;
    p.b2 = b2;
    p.out = reinterpret_cast<uint8_t*>(out);
    p.err = ctx->d_err;
    p.n = n;
    p.ntiles = (int)((n + kRows - 1) / kRows);
    p.h_kind = kind(h_dtype);
    p.x_kind = kind(dtype);
    p.out_kind = kind(out_dtype);
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    // D f32, A/B format, K-major; M = 128; N = 128 (hidden chunk) and N = C
    p.idesc1 = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(kHid >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
    p.idesc2 = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(C >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
    p.tmem_cols = (kHid + C) <= 256 ? 256u : 512u;

    CUtensorMap w1map, w2map;
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)C, (cuuint64_t)(4 * C)};
        const cuuint64_t gstride[1] = {(cuuint64_t)C * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)kHid};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &w1map, dt, 2, const_cast<void*>(w1), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for mlp.0 weights");
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)(4 * C), (cuuint64_t)C};
        const cuuint64_t gstride[1] = {(cuuint64_t)(4 * C) * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)C};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &w2map, dt, 2, const_cast<void*>(w2), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for mlp.2 weights");
    }
    const size_t smem = (size_t)(C / 64) * kRows * 128 * 2 + 2 * kRows * 128 + 2 * (size_t)C * 128 +
                        8 * kNumBars + 16 + 1024;
    if (smem > (size_t)ctx->max_smem_optin) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: shared memory too small");
    static size_t smem_set[3] = {0, 0, 0};      // per C; the attribute only ever grows
    const int si = C == 64 ? 0 : (C == 128 ? 1 : 2);
    if (smem > smem_set[si]) {
        cudaError_t e = cudaFuncSetAttribute(k_convnext_tail<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_convnext_tail)");
        smem_set[si] = smem;
    }
    const int grid = std::max(1, std::min(p.ntiles, ctx->num_sms));
    k_convnext_tail<C><<<grid, kThreads, smem, ctx->stream>>>(w1map, w2map, p);
    TB_LAUNCH_CHECK(ctx, "k_convnext_tail");
    return TB_OK;
}

}  // namespace

bool tb_convnext_tc_supported(int c) { return c == 64 || c == 128 || c == 256; }

tb_status tb_convnext_tail_launch(tb_ctx* ctx, int64_t n, int c, const void* h, tb_dtype h_dtype, const void* x,
                                  const float* nw, const float* nb, const void* w1, const float* b1, const void* w2,
                                  const float* b2, tb_dtype dtype, tb_dtype out_dtype, void* out) {
    if (dtype == TB_F32) {
        if (h_dtype != TB_F32 || out_dtype != TB_F32)
            return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: fp32 operands need fp32 h and output");
        if (c > 1024) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: fp32 kernel takes C <= 1024");
        k_convnext_tail_f32<<<(unsigned)n, 256, (size_t)5 * c * sizeof(float), ctx->stream>>>(
            reinterpret_cast<const float*>(h), reinterpret_cast<const float*>(x), nw, nb,
            reinterpret_cast<const float*>(w1), b1, reinterpret_cast<const float*>(w2), b2,
            reinterpret_cast<float*>(out), n, c);
        TB_LAUNCH_CHECK(ctx, "k_convnext_tail_f32");
        return TB_OK;
    }
    switch (c) {
        case 64: return launch_tail_tc<64>(ctx, n, h, h_dtype, x, nw, nb, w1, b1, w2, b2, dtype, out_dtype, out);
        case 128: return launch_tail_tc<128>(ctx, n, h, h_dtype, x, nw, nb, w1, b1, w2, b2, dtype, out_dtype, out);
        case 256: return launch_tail_tc<256>(ctx, n, h, h_dtype, x, nw, nb, w1, b1, w2, b2, dtype, out_dtype, out);
        default:
            return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: 16-bit operands need C in {64, 128, 256}");
    }
}
