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
// SM walks 128-row tiles with a warp-specialised pipeline, so that the LayerNorm (bound by the
// latency of its row loads), the SiLU (bound by the MUFU unit) and the output stores of
// different tiles and hidden chunks run at the same time:
//  * 4 LayerNorm warps, 32 rows of a tile each, a lane per C/32 consecutive channels so that
//    every row load is coalesced: fp32 statistics, the normalised row rounded to the operand
//    type into a 128-byte-swizzled A tile; with two A tiles (C <= 128) the next tile is
//    normalised while this one is in the tensor pipe;
//  * 1 issuer warp: per hidden chunk of HC units, GEMM1 (A tile x the chunk's mlp.0 rows) into
//    one of two HC-column TMEM accumulators D1, then GEMM2 of the previous chunk (its SiLU
//    activations x the chunk's mlp.2 columns, accumulated over the chunks in a C-column TMEM
//    accumulator D2, two of them when TMEM has room); the weight chunks stream by TMA through
//    shared-memory stages, or stay resident when the stages hold all chunks (C = 64);
//  * 8 activation warps, two per TMEM lane quarter and each half of a chunk's columns: D1 +
//    mlp.0's bias, SiLU, rounded into one of two activation A tiles;
//  * 4 output warps: D2 + mlp.2's bias + the residual x, each row written once.
// SiLU is evaluated as u + u * tanh(u), u = v / 2 (v * sigmoid(v) with sigmoid(v) =
// (1 + tanh(v / 2)) / 2): one MUFU tanh.approx.f32 per value (relative error about 2^-11, below
// the rounding of the 16-bit activation it feeds) instead of an exponential and a reciprocal.
//
// fp32 kernel (any C up to 1024, fp32 operands): one block per row on CUDA cores; it reads the
// weights once per row, so it is meant for the fp32 mode and small channel counts.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>

#ifdef TB_TRACE
extern long long* g_trace_buffer;
#endif

namespace {

using namespace tbtc;

constexpr int kRows = 128;                                  // rows per tile = TMEM lanes
constexpr int kLnWarps = 4, kActWarps = 8, kOutWarps = 4;
constexpr int kActWarp0 = kLnWarps, kOutWarp0 = kActWarp0 + kActWarps, kIssuerWarp = kOutWarp0 + kOutWarps;
constexpr int kThreads = (kIssuerWarp + 1) * 32;
constexpr uint32_t kBlk = kRows * 128;                      // one [128 rows][128 B] swizzled block

// mbarriers: two slots per kind (stage s of a ring at 2 * kind + s), then the drain barrier.
enum { A1F, A1E, D1F, D1E, A2F, A2E, D2F, D2E, W1F, W1E, W2F, W2E, HF, HE, kKinds };
constexpr int kNumBars = 2 * kKinds + 1;

// Pipeline shape per width: hidden chunk HC, LayerNorm A tiles NA1, mlp.0 / mlp.2 weight stages
// NW1 / NW2, output accumulators NB2, staged h tiles NH, within one SM's 227 KB of shared memory
// and 512 TMEM columns (C = 256 keeps one A tile and one mlp.2 stage to leave room for the staged
// parameters). With NH = 2 (C = 64: two 32 KB fp32 tiles fill the last of the 227 KB) the
// LayerNorm warps read h from shared memory, bulk-copied two tiles ahead; wider tiles do not fit
// and are loaded by the LayerNorm warps themselves.
template <int C> struct TailCfg;
template <> struct TailCfg<64> { static constexpr int HC = 128, NA1 = 2, NW1 = 2, NW2 = 2, NB2 = 2, NH = 2; };
template <> struct TailCfg<128> { static constexpr int HC = 64, NA1 = 2, NW1 = 2, NW2 = 2, NB2 = 2, NH = 0; };
template <> struct TailCfg<256> { static constexpr int HC = 64, NA1 = 1, NW1 = 2, NW2 = 1, NB2 = 1, NH = 0; };

template <int C> struct TailLayout {
    using K = TailCfg<C>;
    static constexpr int HC = K::HC, NCH = 4 * C / HC, KB1 = C / 64, KB2 = HC / 64;
    // one A tile, one activation tile, one mlp.0 stage ([HC rows][C]), one mlp.2 stage ([C rows][HC])
    static constexpr uint32_t A1 = KB1 * kBlk, A2 = KB2 * kBlk, W1 = KB1 * HC * 128, W2 = KB2 * C * 128;
    static constexpr uint32_t H = kRows * C * 4;            // one staged h tile (fp32 at most)
    static constexpr uint32_t off_a2 = K::NA1 * A1, off_w1 = off_a2 + 2 * A2, off_w2 = off_w1 + K::NW1 * W1,
                              off_h = off_w2 + K::NW2 * W2, off_bar = off_h + K::NH * H;
    static constexpr bool resident = K::NW1 >= NCH && K::NW2 >= NCH;
    static constexpr uint32_t d2_col = 2 * HC;              // D1 slots at columns 0 and HC
    static constexpr uint32_t tmem_cols = (2 * HC + K::NB2 * C) <= 256 ? 256u : 512u;
    // fp32 parameters staged once per CTA: mlp.0 bias / 2 [4C], mlp.2 bias [C], norm weight, bias [C]
    static constexpr uint32_t off_par = off_bar + ((8 * kNumBars + 16 + 15) & ~15u);
    static constexpr size_t smem = off_par + 7 * C * 4 + 1024;
    static_assert(2 * HC + K::NB2 * C <= 512, "TMEM columns");
    static_assert(smem <= 232448, "shared memory");
};

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
    long long* trace;      // TB_TRACE builds only
};

// Pipeline tracing (compiled in with -DTB_TRACE): CTA 0 stamps clock64 into p.trace, laid out
// as [event][kTraceCap]: 0 LayerNorm warp 0 starts tile t, 1 ... has written it, 2 activation
// warp 0 starts waiting for chunk gc, 3 ... got its accumulator, 4 ... has written its
// activations, 5 output warp 0 got tile t's accumulator, 6 ... has stored tile t, 7 GEMM1 of
// chunk gc issued, 8 GEMM2 of chunk g issued.
[[maybe_unused]] constexpr int kTraceCap = 4096;
#ifdef TB_TRACE
#define TB_STAMP(ev, idx)                                                                         \
    do {                                                                                          \
        if (p.trace && blockIdx.x == 0 && lane == 0 && (idx) < kTraceCap) p.trace[(ev) * kTraceCap + (idx)] = clock64(); \
    } while (0)
#else
#define TB_STAMP(ev, idx) do { } while (0)
#endif

// Element kinds are template parameters (0 f32, 1 f16, 2 bf16), so that no per-element branch
// splits the unrolled loops.
template <int KIND>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (KIND == 2) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

// The two 16-bit values of a packed word (low half first).
template <int KIND>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
    if constexpr (KIND == 2) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    else return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// 16 consecutive output channels of one row.
template <int KIND>
__device__ __forceinline__ void store16k(uint8_t* dst, const float* v) {
    if constexpr (KIND == 0) {
        float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) w[q] = pack2<KIND>(v[2 * q], v[2 * q + 1]);
        uint4* d = reinterpret_cast<uint4*>(dst);
        d[0] = make_uint4(w[0], w[1], w[2], w[3]);
        d[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// SiLU of d + b given bh = b / 2: u = (d + b) / 2 in one FMA, then u + u tanh(u).
__device__ __forceinline__ float silu_half(float d, float bh) {
    const float u = fmaf(0.5f, d, bh);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return fmaf(u, t, u);
}
// Eight consecutive values (16 bytes) of row r, K chunk kc (0..7 within a 64-wide K block) of a
// [128 rows][128 B] K-major block with the 128-byte swizzle: chunk kc sits at kc ^ (r & 7).
__device__ __forceinline__ void put16(uint8_t* blk, int r, int kc, uint4 v) {
    *reinterpret_cast<uint4*>(blk + r * 128 + ((kc ^ (r & 7)) << 4)) = v;
}

// Wait on the clock alone (the exit drain: the abort flag may already be set).
__device__ __forceinline__ void wait_bounded(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity) && clock64() - t0 < kWaitCycles) { }
}

__device__ __forceinline__ uint32_t bar_at(uint32_t b0, int kind, int slot) { return b0 + 8u * (2 * kind + slot); }

// Bring rows [tile * 128, tile * 128 + 128) of a [N][row_bytes] array into L2 ahead of their
// loads (one bulk prefetch; rows are contiguous, row_bytes a multiple of 16).
__device__ __forceinline__ void prefetch_tile_l2(const uint8_t* base, int64_t n, int tile, int ntiles,
                                                 uint32_t row_bytes) {
    if (tile >= ntiles) return;
    const int64_t r0 = (int64_t)tile * kRows;
    const int64_t rows = n - r0 < kRows ? n - r0 : kRows;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 :: "l"(base + (size_t)r0 * row_bytes), "r"((uint32_t)(rows * row_bytes)) : "memory");
}

// Bounded wait with a warp-uniform result, so that a warp leaves its loop as a whole and its
// .sync.aligned instructions (TMEM loads, elect.sync, shuffles) stay converged.
__device__ __forceinline__ bool wait_all(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err));
}

// LayerNorm warp with staged h (C = 64): the CTA's h tiles arrive by TMA two tiles ahead in the
// 128-byte-swizzled layout (in each 128-byte box of a row, 16-byte chunk c of row r sits at
// c ^ (r & 7)), so a thread reads its own row without bank conflicts. Thread = row: the mean and
// variance (one shifted pass), then the normalised row, in two passes over shared memory, with no
// shuffles and one rsqrt per row (the shuffle reductions and their per-row-group rsqrt queued
// behind the activation warps' MUFU and shared-memory traffic).
template <int C, int HK, int XK>
__device__ __forceinline__ void ln_warp_staged(const TailParams& p, const CUtensorMap* hmap, uint8_t* a1, uint8_t* hst,
                                               uint32_t b0, const float* s_nw, const float* s_nb, int ntl, int w,
                                               int lane, volatile int* s_abort) {
    using L = TailLayout<C>;
    constexpr int ES = HK == 0 ? 4 : 2, NBOX = C * ES / 128, VPC = 16 / ES;   // values per 16-byte chunk
    constexpr uint32_t kBoxBytes = kRows * 128;
    const int r = w * 32 + lane;
    int issued = 0, consumed = 0;
    auto issue = [&](int u) {
        const int tile_u = blockIdx.x + u * gridDim.x;
        const uint32_t fb = bar_at(b0, HF, u & 1);
        mbar_arrive_expect_tx(fb, NBOX * kBoxBytes);
#pragma unroll
        for (int b = 0; b < NBOX; ++b)
            tma_load_2d(smem_u32(hst + (u & 1) * L::H + b * kBoxBytes), hmap, b * (128 / ES), tile_u * kRows, fb);
    };
    if (w == 0 && lane == 0)
        for (; issued < 2 && issued < ntl; ++issued) issue(issued);
    for (int t = 0; t < ntl; ++t) {
        const int s = t % L::K::NA1;
        if (!wait_all(bar_at(b0, HF, t & 1), (uint32_t)((t >> 1) & 1), s_abort, p.err)) break;
        consumed = t + 1;
        if (t >= L::K::NA1 && !wait_all(bar_at(b0, A1E, s), (uint32_t)(((t / L::K::NA1) - 1) & 1), s_abort, p.err))
            break;
        if (w == 0) TB_STAMP(0, t);
        const uint8_t* hrow = hst + (t & 1) * L::H + r * 128;
        // VPC values of chunk c (0..7) of box b of this thread's row
        auto chunk = [&](int b, int c, float* v) {
            const uint4 u = *reinterpret_cast<const uint4*>(hrow + b * kBoxBytes + ((c ^ (r & 7)) << 4));
            if constexpr (HK == 0) {
                v[0] = __uint_as_float(u.x), v[1] = __uint_as_float(u.y), v[2] = __uint_as_float(u.z),
                v[3] = __uint_as_float(u.w);
            } else {
                const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = unpack2<HK>(wd[q]);
                    v[2 * q] = f.x, v[2 * q + 1] = f.y;
                }
            }
        };
        // one pass for both statistics, shifted by the row's first value (x - x0 keeps the sums
        // small, so E[(x-x0)^2] - E[x-x0]^2 does not cancel for rows far from zero)
        float x0;
        {
            float v[VPC];
            chunk(0, 0, v);
            x0 = v[0];
        }
        float part[4] = {0.f, 0.f, 0.f, 0.f}, q2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int b = 0; b < NBOX; ++b)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float v[VPC];
                chunk(b, c, v);
#pragma unroll
                for (int e = 0; e < VPC; ++e) {
                    const float d = v[e] - x0;
                    part[e & 3] += d;
                    q2[e & 3] = fmaf(d, d, q2[e & 3]);
                }
            }
        const float dm = ((part[0] + part[1]) + (part[2] + part[3])) * (1.0f / C);
        const float mean = x0 + dm;
        const float var = fmaxf(((q2[0] + q2[1]) + (q2[2] + q2[3])) * (1.0f / C) - dm * dm, 0.f);
        const float rs = rsqrtf(var + 1e-6f);
        uint8_t* a1s = a1 + s * L::A1;
#pragma unroll 2
        for (int oc = 0; oc < C / 8; ++oc) {                  // 8 channels = one 16-byte chunk of A1
            float v[8];
            if constexpr (VPC == 4) {
                chunk((oc * 8) / 32, ((oc * 8) % 32) / 4, v);
                chunk((oc * 8) / 32, ((oc * 8) % 32) / 4 + 1, v + 4);
            } else {
                chunk((oc * 8) / 64, ((oc * 8) % 64) / 8, v);
            }
            const float4 w0 = *reinterpret_cast<const float4*>(s_nw + oc * 8);
            const float4 w1 = *reinterpret_cast<const float4*>(s_nw + oc * 8 + 4);
            const float4 n0 = *reinterpret_cast<const float4*>(s_nb + oc * 8);
            const float4 n1 = *reinterpret_cast<const float4*>(s_nb + oc * 8 + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            const float bv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                pk[e] = pack2<XK>((v[2 * e] - mean) * rs * wv[2 * e] + bv[2 * e],
                                  (v[2 * e + 1] - mean) * rs * wv[2 * e + 1] + bv[2 * e + 1]);
            put16(a1s + (oc >> 3) * kBlk, r, oc & 7, make_uint4(pk[0], pk[1], pk[2], pk[3]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(bar_at(b0, A1F, s));
            mbar_arrive(bar_at(b0, HE, t & 1));       // this warp is done with the staged tile
        }
        if (w == 0 && lane == 0 && t + 2 < ntl) {
            // the copy of tile t + 2 reuses this stage once all four LayerNorm warps have read it
            if (!mbar_wait(bar_at(b0, HE, t & 1), (uint32_t)((t >> 1) & 1), s_abort, p.err)) {
                __syncwarp(1u);
            } else {
                issue(t + 2);
                issued = t + 3;
            }
        }
        __syncwarp();
        if (w == 0) TB_STAMP(1, t);
    }
    // copies still in flight after an abort land before the CTA exits
    if (w == 0 && lane == 0)
        for (int u = consumed; u < issued; ++u) wait_bounded(bar_at(b0, HF, u & 1), (uint32_t)((u >> 1) & 1));
}

// LayerNorm warp: rows [32 w, 32 w + 32) of every tile of this CTA into the A tiles. Eight
// lanes share a row (lane group g = lane & 7 owns channels [g V, g V + V), V = C / 8), so a warp
// step covers four rows with coalesced 16-byte loads and the row statistics take three shuffle
// levels; S steps are loaded together (32 values per lane) and their reductions are interleaved
// level by level.
template <int C, int HK, int XK>
__device__ __forceinline__ void ln_warp(const TailParams& p, uint8_t* a1, uint32_t b0, const float* s_nw,
                                        const float* s_nb, int ntl, int w, int lane, volatile int* s_abort) {
    using L = TailLayout<C>;
    constexpr int V = C / 8, ES = HK == 0 ? 4 : 2, NWD = V * ES / 4;   // 32-bit words per lane per row
    constexpr int S = 32 / V;                                           // row steps per load batch
    const int g = lane & 7, rsub = lane >> 3, c0 = g * V;
    for (int t = 0; t < ntl; ++t) {
        const int tile = blockIdx.x + t * gridDim.x, s = t % L::K::NA1;
        if (w == 0 && lane == 0) {
            // this CTA's rows of h two tiles ahead (and one ahead at the start) into L2
            if (t == 0) prefetch_tile_l2(p.h, p.n, tile + gridDim.x, p.ntiles, C * ES);
            prefetch_tile_l2(p.h, p.n, tile + 2 * gridDim.x, p.ntiles, C * ES);
        }
        if (t >= L::K::NA1 && !wait_all(bar_at(b0, A1E, s), (uint32_t)(((t / L::K::NA1) - 1) & 1), s_abort, p.err))
            return;
        if (w == 0) TB_STAMP(0, t);
        uint8_t* a1s = a1 + s * L::A1;
#pragma unroll 1
        for (int bs = 0; bs < 8; bs += S) {
            uint32_t raw[S][NWD];
#pragma unroll
            for (int i = 0; i < S; ++i) {
                const int64_t row = (int64_t)tile * kRows + w * 32 + (bs + i) * 4 + rsub;
                const uint4* src = reinterpret_cast<const uint4*>(p.h + ((size_t)row * C + c0) * ES);
#pragma unroll
                for (int k = 0; k < NWD / 4; ++k) {
                    const uint4 u = row < p.n ? __ldcs(src + k) : make_uint4(0, 0, 0, 0);
                    raw[i][4 * k] = u.x, raw[i][4 * k + 1] = u.y, raw[i][4 * k + 2] = u.z, raw[i][4 * k + 3] = u.w;
                }
            }
            auto val = [&](int i, int e) -> float {
                if constexpr (HK == 0) {
                    return __uint_as_float(raw[i][e]);
                } else {
                    const float2 f = unpack2<HK>(raw[i][e >> 1]);
                    return (e & 1) ? f.y : f.x;
                }
            };
            float mean[S], rstd[S];
#pragma unroll
            for (int i = 0; i < S; ++i) {
                float sm = 0.f;
#pragma unroll
                for (int e = 0; e < V; ++e) sm += val(i, e);
                mean[i] = sm;
            }
            if (w == 0 && bs == 0) TB_STAMP(13, t);
#pragma unroll
            for (int o = 4; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < S; ++i) mean[i] += __shfl_xor_sync(0xffffffffu, mean[i], o);
#pragma unroll
            for (int i = 0; i < S; ++i) {
                mean[i] *= 1.0f / C;
                float s2 = 0.f;
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const float d = val(i, e) - mean[i];
                    s2 = fmaf(d, d, s2);
                }
                rstd[i] = s2;
            }
#pragma unroll
            for (int o = 4; o > 0; o >>= 1)
#pragma unroll
                for (int i = 0; i < S; ++i) rstd[i] += __shfl_xor_sync(0xffffffffu, rstd[i], o);
#pragma unroll
            for (int i = 0; i < S; ++i) {
                const float rs = rsqrtf(rstd[i] * (1.0f / C) + 1e-6f);
                const int rr = w * 32 + (bs + i) * 4 + rsub;                   // row in the tile
#pragma unroll
                for (int k = 0; k < V / 8; ++k) {
                    const int cb = c0 + 8 * k;                                  // 8 channels = 16 bytes
                    const float4 w0 = *reinterpret_cast<const float4*>(s_nw + cb);
                    const float4 w1 = *reinterpret_cast<const float4*>(s_nw + cb + 4);
                    const float4 n0 = *reinterpret_cast<const float4*>(s_nb + cb);
                    const float4 n1 = *reinterpret_cast<const float4*>(s_nb + cb + 4);
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    const float bv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        pk[e] = pack2<XK>((val(i, 8 * k + 2 * e) - mean[i]) * rs * wv[2 * e] + bv[2 * e],
                                          (val(i, 8 * k + 2 * e + 1) - mean[i]) * rs * wv[2 * e + 1] + bv[2 * e + 1]);
                    put16(a1s + (cb >> 6) * kBlk, rr, (cb & 63) >> 3, make_uint4(pk[0], pk[1], pk[2], pk[3]));
                }
            }
            if (w == 0) TB_STAMP(bs == 0 ? 14 : 15, t);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_at(b0, A1F, s));
        if (w == 0) TB_STAMP(1, t);
    }
}

// The LayerNorm role: staged h tiles where shared memory holds them (C = 64), else row loads.
template <int C, int HK, int XK>
__device__ __forceinline__ void ln_role(const TailParams& p, const CUtensorMap* hmap, uint8_t* a1, uint8_t* hst,
                                        uint32_t b0, const float* s_nw, const float* s_nb, int ntl, int w, int lane,
                                        volatile int* s_abort) {
    if constexpr (TailCfg<C>::NH > 0) ln_warp_staged<C, HK, XK>(p, hmap, a1, hst, b0, s_nw, s_nb, ntl, w, lane, s_abort);
    else ln_warp<C, HK, XK>(p, a1, b0, s_nw, s_nb, ntl, w, lane, s_abort);
}

// What every warp role of the tail kernel reads.
struct RoleCtx {
    const TailParams* p;
    uint8_t* a2;
    const float* s_b1h;
    const float* s_b2;
    uint32_t b0, tmem;
    int ntl, warp, lane;
    volatile int* s_abort;
};

// Activation warp: D1 of each hidden chunk + mlp.0's bias, SiLU, rounded into the chunk's A tile.
template <int C, int XK>
__device__ __forceinline__ void act_warp(const RoleCtx& x) {
    using L = TailLayout<C>;
    using K = typename L::K;
    constexpr int HC = L::HC, NCH = L::NCH;
    const TailParams& p = *x.p;
    const int warp = x.warp, lane = x.lane;
    const uint32_t b0 = x.b0, tmem = x.tmem;
    const int ntl = x.ntl;
    volatile int* s_abort = x.s_abort;
    uint8_t* a2 = x.a2;
    const float* s_b1h = x.s_b1h;
    constexpr int HW = HC / 2;                                 // columns per warp
    const int q = warp & 3, half = (warp - kActWarp0) >> 2, r = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int total = ntl * NCH;
    for (int gc = 0; gc < total; ++gc) {
        const int j = gc % NCH, b = gc & 1;
        if (warp == kActWarp0) TB_STAMP(2, gc);
        if (!wait_all(bar_at(b0, D1F, b), (uint32_t)((gc >> 1) & 1), s_abort, p.err)) break;
        if (gc >= 2 && !wait_all(bar_at(b0, A2E, b), (uint32_t)(((gc >> 1) - 1) & 1), s_abort, p.err)) break;
        if (warp == kActWarp0) TB_STAMP(3, gc);
        tc_fence_after();
        uint8_t* a2b = a2 + b * L::A2;
#pragma unroll
        for (int c = 0; c < HW; c += 32) {
            const int c0 = half * HW + c;                      // column within the chunk
            uint32_t v[32];
            uint32_t* vh = v + 16;
            TMEM_LD_X16(lane_base + (uint32_t)(b * HC + c0), v);
            TMEM_LD_X16(lane_base + (uint32_t)(b * HC + c0 + 16), vh);
            tmem_wait_ld();
            if (warp == kActWarp0) TB_STAMP(9 + 2 * (c / 32), gc);
            if (c + 32 == HW) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar_at(b0, D1E, b));
            }
            const float4* bias = reinterpret_cast<const float4*>(s_b1h + j * HC + c0);
            uint32_t wd[16];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 bh = bias[e];
                wd[2 * e] = pack2<XK>(silu_half(__uint_as_float(v[4 * e]), bh.x),
                                      silu_half(__uint_as_float(v[4 * e + 1]), bh.y));
                wd[2 * e + 1] = pack2<XK>(silu_half(__uint_as_float(v[4 * e + 2]), bh.z),
                                          silu_half(__uint_as_float(v[4 * e + 3]), bh.w));
            }
            uint8_t* blk = a2b + (c0 >> 6) * kBlk;
            const int kc = (c0 & 63) >> 3;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                put16(blk, r, kc + e, make_uint4(wd[4 * e], wd[4 * e + 1], wd[4 * e + 2], wd[4 * e + 3]));
            if (warp == kActWarp0) TB_STAMP(10 + 2 * (c / 32), gc);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_at(b0, A2F, b));
        if (warp == kActWarp0) TB_STAMP(4, gc);
    }
}

// Output warp: D2 of each tile + mlp.2's bias + the residual x, one row per thread.
template <int C, int XK, int OK>
__device__ __forceinline__ void out_warp(const RoleCtx& x) {
    using L = TailLayout<C>;
    using K = typename L::K;
    const TailParams& p = *x.p;
    const int warp = x.warp, lane = x.lane;
    const uint32_t b0 = x.b0, tmem = x.tmem;
    const int ntl = x.ntl;
    volatile int* s_abort = x.s_abort;
    const float* s_b2 = x.s_b2;
    const int q = warp & 3, r = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    constexpr size_t osz = OK == 0 ? 4 : 2;
    for (int t = 0; t < ntl; ++t) {
        const int tile = blockIdx.x + t * gridDim.x, b = t % K::NB2;
        if (warp == kOutWarp0 && lane == 0) prefetch_tile_l2(p.x, p.n, tile + gridDim.x, p.ntiles, C * 2);
        const int64_t row = (int64_t)tile * kRows + r;
        const bool valid = row < p.n;
        const uint4* xrow = reinterpret_cast<const uint4*>(p.x + (size_t)(valid ? row : 0) * C * 2);
        uint8_t* orow = p.out + (size_t)(valid ? row : 0) * C * osz;
        // the residual's first 32 channels, loaded while the accumulator completes
        uint4 xv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) xv[e] = valid ? __ldcs(xrow + e) : make_uint4(0, 0, 0, 0);
        if (!wait_all(bar_at(b0, D2F, b), (uint32_t)((t / K::NB2) & 1), s_abort, p.err)) break;
        if (warp == kOutWarp0) TB_STAMP(5, t);
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < C; c0 += 32) {
            uint4 xn[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                xn[e] = (valid && c0 + 32 < C) ? __ldcs(xrow + (c0 + 32) / 8 + e) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t v[16];
                TMEM_LD_X16(lane_base + (uint32_t)(L::d2_col + b * C + c0 + 16 * hh), v);
                tmem_wait_ld();
                if (hh == 1 && c0 + 32 == C) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar_at(b0, D2E, b));
                }
                const uint32_t* xw = reinterpret_cast<const uint32_t*>(xv + 2 * hh);
                const float4* bias = reinterpret_cast<const float4*>(s_b2 + c0 + 16 * hh);
                float f[16];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 bb = bias[e];
                    const float2 x0 = unpack2<XK>(xw[2 * e]), x1 = unpack2<XK>(xw[2 * e + 1]);
                    f[4 * e] = __uint_as_float(v[4 * e]) + bb.x + x0.x;
                    f[4 * e + 1] = __uint_as_float(v[4 * e + 1]) + bb.y + x0.y;
                    f[4 * e + 2] = __uint_as_float(v[4 * e + 2]) + bb.z + x1.x;
                    f[4 * e + 3] = __uint_as_float(v[4 * e + 3]) + bb.w + x1.y;
                }
                if (valid) store16k<OK>(orow + (size_t)(c0 + 16 * hh) * osz, f);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) xv[e] = xn[e];
        }
        if (warp == kOutWarp0) TB_STAMP(6, t);
    }
}

template <int C>
__global__ void __launch_bounds__(kThreads, 1)
k_convnext_tail(const __grid_constant__ CUtensorMap w1map, const __grid_constant__ CUtensorMap w2map,
                const __grid_constant__ CUtensorMap hmap, const TailParams p) {
    using L = TailLayout<C>;
    using K = typename L::K;
    constexpr int HC = L::HC, NCH = L::NCH, KB1 = L::KB1, KB2 = L::KB2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* a1 = smem;
    uint8_t* a2 = smem + L::off_a2;
    uint8_t* w1s = smem + L::off_w1;
    uint8_t* w2s = smem + L::off_w2;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kNumBars);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);
    float* s_b1h = reinterpret_cast<float*>(smem + L::off_par);     // [4C] mlp.0 bias / 2
    float* s_b2 = s_b1h + 4 * C;                                      // [C]
    float* s_nw = s_b2 + C;                                           // [C]
    float* s_nb = s_nw + C;                                           // [C]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b0 = smem_u32(bars);
    const int ntl = (int)blockIdx.x < p.ntiles ? (p.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar_at(b0, A1F, s), kLnWarps);
            mbar_init(bar_at(b0, A1E, s), 1);
            mbar_init(bar_at(b0, D1F, s), 1);
            mbar_init(bar_at(b0, D1E, s), kActWarps);
            mbar_init(bar_at(b0, A2F, s), kActWarps);
            mbar_init(bar_at(b0, A2E, s), 1);
            mbar_init(bar_at(b0, D2F, s), 1);
            mbar_init(bar_at(b0, D2E, s), kOutWarps);
            mbar_init(bar_at(b0, W1F, s), 1);
            mbar_init(bar_at(b0, W1E, s), 1);
            mbar_init(bar_at(b0, W2F, s), 1);
            mbar_init(bar_at(b0, W2E, s), 1);
            mbar_init(bar_at(b0, HF, s), 1);
            mbar_init(bar_at(b0, HE, s), kLnWarps);
        }
        mbar_init(b0 + 8u * (kNumBars - 1), 1);
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&w1map)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&w2map)) : "memory");
        if (K::NH > 0) asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&hmap)) : "memory");
    }
    for (int i = threadIdx.x; i < 4 * C; i += kThreads) s_b1h[i] = 0.5f * __ldg(p.b1 + i);
    for (int i = threadIdx.x; i < C; i += kThreads) {
        s_b2[i] = __ldg(p.b2 + i);
        s_nw[i] = __ldg(p.nw + i);
        s_nb[i] = __ldg(p.nb + i);
    }
    if (warp == kIssuerWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(L::tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_misc[0];
    const RoleCtx rc{&p, a2, s_b1h, s_b2, b0, tmem, ntl, warp, lane, s_abort};

    if (warp < kActWarp0) {
        // ------------------------------------------------------------------ LayerNorm warps
        if (p.x_kind == 2) {
            if (p.h_kind == 0) ln_role<C, 0, 2>(p, &hmap, a1, smem + L::off_h, b0, s_nw, s_nb, ntl, warp, lane, s_abort);
            else ln_role<C, 2, 2>(p, &hmap, a1, smem + L::off_h, b0, s_nw, s_nb, ntl, warp, lane, s_abort);
        } else {
            if (p.h_kind == 0) ln_role<C, 0, 1>(p, &hmap, a1, smem + L::off_h, b0, s_nw, s_nb, ntl, warp, lane, s_abort);
            else ln_role<C, 1, 1>(p, &hmap, a1, smem + L::off_h, b0, s_nw, s_nb, ntl, warp, lane, s_abort);
        }
    } else if (warp < kOutWarp0) {
        // ------------------------------------------------------------------ activation warps
        if (p.x_kind == 2) act_warp<C, 2>(rc);
        else act_warp<C, 1>(rc);
    } else if (warp < kIssuerWarp) {
        // ------------------------------------------------------------------ output warps
        if (p.x_kind == 2) {
            if (p.out_kind == 0) out_warp<C, 2, 0>(rc);
            else out_warp<C, 2, 2>(rc);
        } else {
            if (p.out_kind == 0) out_warp<C, 1, 0>(rc);
            else out_warp<C, 1, 1>(rc);
        }
    } else {
        // ------------------------------------------------------------------ TMA + MMA issuer warp
        // The whole warp runs the schedule (waits in every lane); one elected lane issues.
        const int total = ntl * NCH;
        auto load_w1 = [&](int u) {
            const int s = L::resident ? u : u % K::NW1, j = u % NCH;
            const uint32_t fb = bar_at(b0, W1F, s);
            if (elect_one()) {
                mbar_arrive_expect_tx(fb, L::W1);
#pragma unroll
                for (int kb = 0; kb < KB1; ++kb)
                    tma_load_2d(smem_u32(w1s + s * L::W1 + kb * HC * 128), &w1map, kb * 64, j * HC, fb);
            }
            __syncwarp();
        };
        auto load_w2 = [&](int u) {
            const int s = L::resident ? u : u % K::NW2, j = u % NCH;
            const uint32_t fb = bar_at(b0, W2F, s);
            if (elect_one()) {
                mbar_arrive_expect_tx(fb, L::W2);
#pragma unroll
                for (int kb = 0; kb < KB2; ++kb)
                    tma_load_2d(smem_u32(w2s + s * L::W2 + kb * C * 128), &w2map, j * HC + kb * 64, 0, fb);
            }
            __syncwarp();
        };
        int n1 = 0, n2 = 0;                  // weight uses whose loads were issued
        int c1 = 0, c2 = 0;                  // ... and waited on
        if (L::resident) {
            for (; n1 < NCH; ++n1) load_w1(n1);
            for (; n2 < NCH; ++n2) load_w2(n2);
        } else {
            for (; n1 < K::NW1 && n1 < total; ++n1) load_w1(n1);
            for (; n2 < K::NW2 && n2 < total; ++n2) load_w2(n2);
        }
        for (int gc = 0; gc <= total; ++gc) {
            if (gc < total) {
                // GEMM1 of chunk gc: D1[gc & 1] = A tile x mlp.0 rows of the chunk
                const int t = gc / NCH, j = gc % NCH, sa = t % K::NA1, b = gc & 1;
                if (j == 0 && !wait_all(bar_at(b0, A1F, sa), (uint32_t)((t / K::NA1) & 1), s_abort, p.err)) break;
                if (gc >= 2 && !wait_all(bar_at(b0, D1E, b), (uint32_t)(((gc >> 1) - 1) & 1), s_abort, p.err)) break;
                const int ws = L::resident ? j : gc % K::NW1;
                if (!wait_all(bar_at(b0, W1F, ws), L::resident ? 0u : (uint32_t)((gc / K::NW1) & 1), s_abort, p.err))
                    break;
                c1 = c1 > (L::resident ? j + 1 : gc + 1) ? c1 : (L::resident ? j + 1 : gc + 1);
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int kb = 0; kb < KB1; ++kb)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma(tmem + (uint32_t)(b * HC), smem_desc<128>(smem_u32(a1 + sa * L::A1 + kb * kBlk)) + 2 * k,
                                   smem_desc<128>(smem_u32(w1s + ws * L::W1 + kb * HC * 128)) + 2 * k, p.idesc1,
                                   (kb | k) ? 1u : 0u);
                    tc_commit(bar_at(b0, D1F, b));
                    TB_STAMP(7, gc);
                    if (j == NCH - 1) tc_commit(bar_at(b0, A1E, sa));
                    if (!L::resident) tc_commit(bar_at(b0, W1E, ws));
                }
                __syncwarp();
            }
            if (gc >= 1) {
                // GEMM2 of chunk g = gc - 1: D2[tile] += activations x mlp.2 columns of the chunk
                const int g = gc - 1, t = g / NCH, j = g % NCH, b = g & 1, sd = t % K::NB2;
                if (!wait_all(bar_at(b0, A2F, b), (uint32_t)((g >> 1) & 1), s_abort, p.err)) break;
                if (j == 0 && t >= K::NB2 &&
                    !wait_all(bar_at(b0, D2E, sd), (uint32_t)(((t / K::NB2) - 1) & 1), s_abort, p.err))
                    break;
                const int ws = L::resident ? j : g % K::NW2;
                if (!wait_all(bar_at(b0, W2F, ws), L::resident ? 0u : (uint32_t)((g / K::NW2) & 1), s_abort, p.err))
                    break;
                c2 = c2 > (L::resident ? j + 1 : g + 1) ? c2 : (L::resident ? j + 1 : g + 1);
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int kb = 0; kb < KB2; ++kb)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma(tmem + (uint32_t)(L::d2_col + sd * C),
                                   smem_desc<128>(smem_u32(a2 + b * L::A2 + kb * kBlk)) + 2 * k,
                                   smem_desc<128>(smem_u32(w2s + ws * L::W2 + kb * C * 128)) + 2 * k, p.idesc2,
                                   (j | kb | k) ? 1u : 0u);
                    tc_commit(bar_at(b0, A2E, b));
                    TB_STAMP(8, g);
                    if (j == NCH - 1) tc_commit(bar_at(b0, D2F, sd));
                    if (!L::resident) tc_commit(bar_at(b0, W2E, ws));
                }
                __syncwarp();
            }
            if (!L::resident) {
                // refill the stages the MMAs just issued read, once they have completed
                if (gc < total && gc + K::NW1 < total) {
                    if (!wait_all(bar_at(b0, W1E, gc % K::NW1), (uint32_t)((gc / K::NW1) & 1), s_abort, p.err)) break;
                    load_w1(gc + K::NW1);
                    n1 = gc + K::NW1 + 1;
                }
                if (gc >= 1 && gc - 1 + K::NW2 < total) {
                    if (!wait_all(bar_at(b0, W2E, (gc - 1) % K::NW2), (uint32_t)(((gc - 1) / K::NW2) & 1), s_abort,
                                   p.err))
                        break;
                    load_w2(gc - 1 + K::NW2);
                    n2 = gc - 1 + K::NW2 + 1;
                }
            }
        }
        // weight copies still in flight after an abort land before the CTA exits
        for (int u = c1; u < n1; ++u)
            wait_bounded(bar_at(b0, W1F, L::resident ? u : u % K::NW1), L::resident ? 0u : (uint32_t)((u / K::NW1) & 1));
        for (int u = c2; u < n2; ++u)
            wait_bounded(bar_at(b0, W2F, L::resident ? u : u % K::NW2), L::resident ? 0u : (uint32_t)((u / K::NW2) & 1));
        // every MMA of this CTA has finished before the TMEM is freed (also after an abort)
        const uint32_t drain = b0 + 8u * (kNumBars - 1);
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        wait_bounded(drain, 0);
    }
    __syncthreads();
    if (warp == kIssuerWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(L::tmem_cols) : "memory");
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
    using L = TailLayout<C>;
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
    // D f32, A/B format, K-major; M = 128; N = HC (hidden chunk) and N = C
    p.idesc1 = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(L::HC >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
    p.idesc2 = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(C >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
#ifdef TB_TRACE
    p.trace = g_trace_buffer;
#else
    p.trace = nullptr;
#endif

    CUtensorMap w1map, w2map, hmap;
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    {
        // mlp.0 weight [4C][C]: a box is 64 input channels of HC hidden rows
        const cuuint64_t gdim[2] = {(cuuint64_t)C, (cuuint64_t)(4 * C)};
        const cuuint64_t gstride[1] = {(cuuint64_t)C * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)L::HC};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &w1map, dt, 2, const_cast<void*>(w1), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for mlp.0 weights");
    }
    {
        // mlp.2 weight [C][4C]: a box is 64 hidden units of all C output rows
        const cuuint64_t gdim[2] = {(cuuint64_t)(4 * C), (cuuint64_t)C};
        const cuuint64_t gstride[1] = {(cuuint64_t)(4 * C) * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)C};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &w2map, dt, 2, const_cast<void*>(w2), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for mlp.2 weights");
    }
    hmap = w1map;                      // not read unless the h tiles are staged
    if (TailCfg<C>::NH > 0) {
        // h [n][C] in boxes of 128 bytes x 128 rows, 128-byte swizzle (rows past n read as zero)
        const int es = h_dtype == TB_F32 ? 4 : 2;
        const CUtensorMapDataType hdt = h_dtype == TB_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                        : (h_dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
        const cuuint64_t gdim[2] = {(cuuint64_t)C, (cuuint64_t)n};
        const cuuint64_t gstride[1] = {(cuuint64_t)C * es};
        const cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)kRows};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &hmap, hdt, 2, const_cast<void*>(h), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for h");
    }
    const size_t smem = L::smem;
    if (smem > (size_t)ctx->max_smem_optin) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: shared memory too small");
    static size_t smem_set[3] = {0, 0, 0};      // per C; the attribute only ever grows
    const int si = C == 64 ? 0 : (C == 128 ? 1 : 2);
    if (smem > smem_set[si]) {
        cudaError_t e = cudaFuncSetAttribute(k_convnext_tail<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_convnext_tail)");
        smem_set[si] = smem;
    }
    const int grid = std::max(1, std::min(p.ntiles, ctx->num_sms));
    k_convnext_tail<C><<<grid, kThreads, smem, ctx->stream>>>(w1map, w2map, hmap, p);
    TB_LAUNCH_CHECK(ctx, "k_convnext_tail");
    return TB_OK;
}

}  // namespace

bool tb_convnext_tc_supported(int c) { return c == 64 || c == 128 || c == 256; }
bool tb_convnext_two_pass_supported(int c) { return c == 16 || c == 32 || (c % 64 == 0 && c <= 2048); }

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
        default: break;
    }
    if (!tb_convnext_two_pass_supported(c))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "convnext tail: 16-bit operands need C in {16, 32} or a multiple of 64 up to 2048");
    // Widths whose LayerNorm tile does not fit the fused kernel's shared memory (C = 512, 1024 in
    // decode_unet's first stages) run as three passes with the same roundings: LayerNorm to the
    // operand type, mlp.0 + SiLU into a [n][4C] activation tile in HBM, mlp.2 + bias + residual.
    const size_t es = tb_dtype_size(dtype);
    const size_t y_b = ((size_t)n * c * es + 255) & ~size_t(255);
    tb_status s = tb_ensure(ctx, &ctx->tail_ws, &ctx->tail_ws_bytes, y_b + (size_t)n * 4 * c * es, "convnext tail passes");
    if (s != TB_OK) return s;
    uint8_t* y = reinterpret_cast<uint8_t*>(ctx->tail_ws);
    uint8_t* act = y + y_b;
    s = tb_row_norm_launch(ctx, h, h_dtype, nullptr, n, c, nw, nb, 0, dtype, y, 1e-6f);
    if (s != TB_OK) return s;
    s = tb_linear_launch(ctx, n, c, 4 * c, y, w1, b1, nullptr, dtype, 1, dtype, dtype, act);
    if (s != TB_OK) return s;
    return tb_linear_launch(ctx, n, 4 * c, c, act, w2, b2, x, dtype, 0, dtype, out_dtype, out);
}
