// Submanifold 3x3x3 sparse convolution as a warp-specialised implicit GEMM on sm_100a.
//
// Replaces the reference's per-tap graph chain (src/sparse.cpp:64-79): 27 x {get_rows,
// mul_mat, add} over materialised [Ci, nr] gathers plus a bias add, i.e. about 3x27 HBM
// passes of the features. Here one persistent kernel computes each 128-voxel output tile
// in TMEM and writes it once, with no intermediate tensors and no atomics:
//
//   D[128 x NB] (fp32, TMEM) = sum over present taps t and channel chunks k of
//        A_t,k [128 x KC]  (gathered feature rows, bf16/f16, smem)
//      x B_t,k [KC x NB]   (weight tap slice, smem)
//
// Roles (288 threads):
//   warps 0-3  epilogue: tcgen05.ld the accumulator (warp w owns TMEM lanes 32w..32w+31,
//              i.e. tile rows), add bias, optional SiLU, convert, store rows.
//   warps 4-7  producers: stage the tile's 27x128 neighbor indices in smem, OR their
//              presence bits into a tile tap mask, then for every present tap and channel
//              chunk gather A with cp.async (absent rows are zero-filled by a src-size-0
//              copy, the padded zero row of src/sparse.cpp:82-85) and issue one TMA load
//              of B from the [Co][27*Ci] weight view.
//   warp 8     MMA: one thread issues tcgen05.mma kind::f16 (M=128, N=NB, K=16) per
//              16-channel step and tcgen05.commit to release smem stages and hand the
//              accumulator to the epilogue. Two accumulator buffers let the epilogue of
//              tile i overlap the MMAs of tile i+1.
// Taps that no row of a tile has are skipped for the whole tile.
//
// Every mbarrier wait is bounded (about 2 s of clock). On timeout the kernel records
// TB_DEVERR_WAIT_TIMEOUT, raises a CTA abort flag that all waits observe, lets its own
// copies land, drains its MMAs, frees TMEM and returns.
#include "tb_common.cuh"

#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace {

constexpr int kTileM = 128;
constexpr int kThreads = 288;
constexpr int kMaxStages = 8;
constexpr int kNbrSmem = 27 * kTileM * 4;   // staged neighbor indices of one tile
constexpr long long kWaitCycles = 4000000000ll;   // ~2 s at 1.9 GHz

struct ConvParams {
    const int32_t* nbr;
    const uint8_t* feats;
    const float* bias;
    uint8_t* out;
    int* err;
    int64_t n;
    int ci, co;
    int out_kind;       // 0 f32, 1 f16, 2 bf16
    int epi;
    int ntiles, ncb, nkc;
    int kc;             // channels per chunk (16, 32 or 64)
    int nb;             // accumulator columns per work unit
    int stages;
    uint32_t a_bytes, b_bytes, stage_bytes;
    uint32_t idesc;
    uint32_t tmem_cols;
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: false when the CTA aborted or the clock limit ran out (then aborts it).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitCycles) {
            *abort_flag = 1;
            atomicCAS(err, 0, TB_DEVERR_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// K-major operand tile: rows of RB bytes, 8-row atoms, swizzle width = RB (32/64/128 B).
template <int RB>
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    constexpr uint64_t layout = RB == 128 ? 2 : (RB == 64 ? 4 : 6);
    constexpr uint64_t sbo = (8 * RB) >> 4;
    return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (sbo << 32) | (1ull << 46) | (layout << 61);
}
// Byte offset of 16-byte chunk c of row r inside a swizzled tile with RB-byte rows.
template <int RB>
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
    if (RB == 128) return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
    if (RB == 64) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
}

#define TMEM_LD_X16(taddr, v)                                                              \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "                                 \
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"          \
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),  \
                   "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),\
                   "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])                       \
                 : "r"(taddr))

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float apply_epi(float v, int epi) {
    return epi == TB_EPI_SILU ? v / (1.0f + __expf(-v)) : v;
}

// Store 16 consecutive output channels of one row.
__device__ __forceinline__ void store16(uint8_t* dst, const float* v, int kind) {
    if (kind == 0) {
        float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int q = 0; q < 4; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (kind == 2) {
                __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
                w[q] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __half2 h = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
                w[q] = *reinterpret_cast<uint32_t*>(&h);
            }
        }
        uint4* d = reinterpret_cast<uint4*>(dst);
        d[0] = make_uint4(w[0], w[1], w[2], w[3]);
        d[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

template <int RB>
__global__ void __launch_bounds__(kThreads, 1)
k_submconv_tc(const __grid_constant__ CUtensorMap wmap, const ConvParams p) {
    constexpr int CH = RB / 16;          // 16-byte chunks per gathered row
    constexpr int KSTEPS = RB / 32;      // K=16 MMAs per chunk
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    uint8_t* stage_base = smem;
    int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + (size_t)p.stages * p.stage_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_nbr) + kNbrSmem);
    // bars: full[kMaxStages] empty[kMaxStages] acc_full[2] acc_empty[2] prod_sync drain
    uint32_t* s_hdr = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 6);
    uint32_t* s_misc = s_hdr + kMaxStages;   // [0] tmem base, [1] tap mask, [2] abort
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
    auto accf_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + b); };
    auto acce_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + 2 + b); };
    const uint32_t prod_bar = bar0 + 8u * (2 * kMaxStages + 4);
    const uint32_t drain_bar = bar0 + 8u * (2 * kMaxStages + 5);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full_bar(s), 128 + 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accf_bar(b), 1);
            mbar_init(acce_bar(b), 128);
        }
        mbar_init(prod_bar, 128);
        mbar_init(drain_bar, 1);
        s_misc[1] = 0;
        s_misc[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_misc[0];

    const int nunits = p.ntiles * p.ncb;

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------------ producers
        const int pt = threadIdx.x - 128;
        int stage = 0;
        uint32_t phase = 0;
        uint32_t prod_phase = 0;
        bool ok = true;
        // TMA loads issued by thread 0 whose completion has not been observed.
        auto prod_sync = [&]() -> bool {
            mbar_arrive(prod_bar);
            const bool r = mbar_wait(prod_bar, prod_phase, s_abort, p.err);
            prod_phase ^= 1;
            return r;
        };
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
            const int tile = u / p.ncb, cb = u % p.ncb;
            const int64_t r0 = (int64_t)tile * kTileM;
            if (!prod_sync()) { ok = false; break; }            // previous unit done with s_nbr
            for (int idx = pt; idx < 27 * kTileM; idx += 128) {
                const int t = idx >> 7, r = idx & 127;
                const int64_t row = r0 + r;
                s_nbr[idx] = row < p.n ? __ldg(p.nbr + (int64_t)t * p.n + row) : (int32_t)p.n;
            }
            if (pt == 0) s_misc[1] = 0;
            if (!prod_sync()) { ok = false; break; }
            uint32_t bits = 0;
#pragma unroll
            for (int t = 0; t < 27; ++t) bits |= (uint32_t)(s_nbr[t * kTileM + pt] != (int32_t)p.n) << t;
            bits = __reduce_or_sync(0xffffffffu, bits);
            if (lane == 0) atomicOr(&s_misc[1], bits);
            if (!prod_sync()) { ok = false; break; }
            uint32_t taps = s_misc[1];
            const int nstages_unit = __popc(taps) * p.nkc;
            int si = 0;
            while (taps && ok) {
                const int t = __ffs(taps) - 1;
                taps &= taps - 1;
                for (int kc = 0; kc < p.nkc; ++kc, ++si) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, s_abort, p.err)) { ok = false; break; }
                    uint8_t* a_tile = stage_base + (size_t)stage * p.stage_bytes;
                    const uint32_t a_addr = smem_u32(a_tile);
                    const int c = pt % CH;
#pragma unroll
                    for (int j = 0; j < CH; ++j) {
                        const int r = pt / CH + j * (kTileM / CH);
                        const int32_t src_row = s_nbr[t * kTileM + r];
                        const bool present = src_row != (int32_t)p.n;
                        const uint8_t* src = present
                            ? p.feats + ((int64_t)src_row * p.ci + (int64_t)kc * p.kc) * 2 + c * 16
                            : p.feats;
                        cp_async_16(a_addr + swz_off<RB>(r, c), src, present ? 16u : 0u);
                    }
                    cp_async_mbar_arrive_noinc(full_bar(stage));
                    if (pt == 0) {
                        s_hdr[stage] = (si == 0 ? 1u : 0u) | (si == nstages_unit - 1 ? 2u : 0u);
                        mbar_arrive_expect_tx(full_bar(stage), p.b_bytes);
                        tma_load_2d(a_addr + p.a_bytes, &wmap, t * p.ci + kc * p.kc, cb * p.nb, full_bar(stage));
                    }
                    if (++stage == p.stages) { stage = 0; phase ^= 1; }
                }
            }
        }
        cp_async_wait_all();
        if (!ok && pt == 0) {
            // let this CTA's in-flight TMA loads land before the CTA can exit
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int it = 0;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
                const int ab = it & 1;
                const uint32_t aph = (it >> 1) & 1;
                if (!mbar_wait(acce_bar(ab), aph ^ 1, s_abort, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * p.nb);
                bool first = true;
                while (true) {
                    if (!mbar_wait(full_bar(stage), phase, s_abort, p.err)) { ok = false; break; }
                    fence_proxy_async();
                    tc_fence_after();
                    const uint32_t hdr = s_hdr[stage];
                    const uint32_t a_addr = smem_u32(stage_base + (size_t)stage * p.stage_bytes);
                    const uint32_t b_addr = a_addr + p.a_bytes;
#pragma unroll
                    for (int k = 0; k < KSTEPS; ++k) {
                        tc_mma(d_tmem, smem_desc<RB>(a_addr + 32 * k), smem_desc<RB>(b_addr + 32 * k),
                               p.idesc, (first && k == 0) ? 0u : 1u);
                    }
                    tc_commit(empty_bar(stage));
                    first = false;
                    if (++stage == p.stages) { stage = 0; phase ^= 1; }
                    if (hdr & 2u) break;
                }
                if (!ok) break;
                tc_commit(accf_bar(ab));
            }
            // drain: every MMA issued by this thread has completed once this arrives
            tc_commit(drain_bar);
            const long long t0 = clock64();
            while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < kWaitCycles) __nanosleep(64);
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp;          // TMEM lanes 32q..32q+31
        int it = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
            const int tile = u / p.ncb, cb = u % p.ncb;
            const int ab = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait(accf_bar(ab), aph, s_abort, p.err)) break;
            tc_fence_after();
            const int64_t row = (int64_t)tile * kTileM + q * 32 + lane;
            const size_t esize = p.out_kind == 0 ? 4 : 2;
            uint8_t* orow = p.out + ((size_t)row * p.co + (size_t)cb * p.nb) * esize;
            for (int c0 = 0; c0 < p.nb; c0 += 16) {
                uint32_t v[16];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * p.nb + c0);
                TMEM_LD_X16(taddr, v);
                tmem_wait_ld();
                float f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int o = cb * p.nb + c0 + j;
                    float x = __uint_as_float(v[j]) + (p.bias ? __ldg(p.bias + o) : 0.0f);
                    f[j] = apply_epi(x, p.epi);
                }
                if (row < p.n) store16(orow + (size_t)c0 * esize, f, p.out_kind);
            }
            tc_fence_before();
            mbar_arrive(acce_bar(ab));
        }
    }

    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(p.tmem_cols) : "memory");
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

bool tb_conv_tc_supported(int ci, int co) {
    const bool ci_ok = ci == 16 || ci == 32 || (ci > 0 && ci % 64 == 0);
    const bool co_ok = co > 0 && co % 16 == 0 && (co <= 256 || co % 256 == 0);
    return ci_ok && co_ok;
}

tb_status tb_conv_tc_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, const void* feats, int ci,
                            const void* weight, const float* bias, int co, tb_dtype dtype,
                            tb_dtype out_dtype, tb_epilogue epi, void* out) {
    if (!tb_conv_tc_supported(ci, co))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_submconv: tensor-core path needs ci in {16,32,64k} and co%16==0 (<=256 or 256k)");
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    const int kc = ci < 64 ? ci : 64;
    const int rb = kc * 2;
    const int nb = co <= 256 ? co : 256;
    ConvParams p{};
    p.nbr = nbr;
    p.feats = reinterpret_cast<const uint8_t*>(feats);
    p.bias = bias;
    p.out = reinterpret_cast<uint8_t*>(out);
    p.err = ctx->d_err;
    p.n = n;
    p.ci = ci;
    p.co = co;
    p.out_kind = out_dtype == TB_F32 ? 0 : (out_dtype == TB_F16 ? 1 : 2);
    p.epi = epi;
    p.ntiles = (int)((n + kTileM - 1) / kTileM);
    p.ncb = co / nb;
    p.nkc = ci / kc;
    p.kc = kc;
    p.nb = nb;
    p.a_bytes = kTileM * rb;
    p.b_bytes = (uint32_t)(nb * rb);
    const uint32_t b_alloc = (p.b_bytes + 1023u) & ~1023u;
    p.stage_bytes = p.a_bytes + b_alloc;
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * nb)) cols <<= 1;
    p.tmem_cols = cols;
    // instruction descriptor: D f32, A/B bf16 (1) or f16 (0), both K-major, N>>3, M>>4
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(nb >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);

    const size_t fixed = kNbrSmem + 8 * (2 * kMaxStages + 6) + 4 * (kMaxStages + 4) + 1024;
    const size_t budget = (size_t)ctx->max_smem_optin;
    int stages = (int)std::min<size_t>(kMaxStages, (budget - fixed) / p.stage_bytes);
    if (stages < 2) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_submconv: stage does not fit in shared memory");
    p.stages = stages;
    size_t smem = fixed + (size_t)stages * p.stage_bytes;
    // one CTA per SM: TMEM columns and the persistent schedule assume it
    smem = std::max<size_t>(smem, 120 * 1024);
    smem = std::min<size_t>(smem, budget);

    CUtensorMap map;
    const cuuint64_t gdim[2] = {(cuuint64_t)27 * ci, (cuuint64_t)co};
    const cuuint64_t gstride[1] = {(cuuint64_t)27 * ci * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kc, (cuuint32_t)nb};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle swz = rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : (rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
        &map, dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
        const_cast<void*>(weight), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight view");

    const int units = p.ntiles * p.ncb;
    const int grid = std::min(units, ctx->num_sms);
    cudaError_t e;
    if (rb == 128) {
        e = cudaFuncSetAttribute(k_submconv_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<128><<<grid, kThreads, smem, ctx->stream>>>(map, p);
    } else if (rb == 64) {
        e = cudaFuncSetAttribute(k_submconv_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<64><<<grid, kThreads, smem, ctx->stream>>>(map, p);
    } else {
        e = cudaFuncSetAttribute(k_submconv_tc<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<32><<<grid, kThreads, smem, ctx->stream>>>(map, p);
    }
    if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_tc)");
    TB_LAUNCH_CHECK(ctx, "k_submconv_tc");
    return TB_OK;
}
