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
// Roles (224 threads):
//   warps 0-3  epilogue: tcgen05.ld the accumulator (warp w owns TMEM lanes 32w..32w+31,
//              i.e. tile rows), add bias, optional SiLU, convert, store rows.
//   warp 4     neighbor loader: copies the tile's 27x128 neighbor indices into one of two
//              smem buffers and ORs their presence bits into the tile's tap mask, one or
//              two tiles ahead of the producer.
//   warp 5     producer: for every present tap and channel chunk, each lane issues one TMA
//              tile::gather4 (4 feature rows -> swizzled smem rows of A); absent rows use
//              the row index N, which is out of bounds and arrives zero-filled (the padded
//              zero row of src/sparse.cpp:82-85). Lane 0 adds one TMA load of B from the
//              [Co][27*Ci] weight view. All of it completes on the stage's mbarrier.
//   warp 6     MMA: one thread issues tcgen05.mma kind::f16 (M=128, N=NB, K=16) per
//              16-channel step and tcgen05.commit to release smem stages and hand the
//              accumulator to the epilogue. Two accumulator buffers let the epilogue of
//              tile i overlap the MMAs of tile i+1.
// Taps that no row of a tile has are skipped for the whole tile. TMA writes straight into
// shared memory, so the gather is not limited by the L1 left over after the smem carve-out.
//
// Every mbarrier wait is bounded (about 2 s of clock). On timeout the kernel records
// TB_DEVERR_WAIT_TIMEOUT, raises a CTA abort flag that all waits observe, lets its own
// copies land, drains its MMAs, frees TMEM and returns.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>

namespace {

using namespace tbtc;

constexpr int kTileM = 128;
constexpr int kThreads = 224;
constexpr int kMaxStages = 8;
constexpr int kNbrSmem = 27 * kTileM * 4;   // staged neighbor indices of one tile

struct ConvParams {
    const int32_t* nbr;
    const uint8_t* feats;
    const float* bias;
    uint8_t* out;
    int* err;
    const int32_t* perm;    // optional tile order: tile position -> output row
    int64_t n;
    int ci, co;
    int out_kind;       // 0 f32, 1 f16, 2 bf16
    int epi;
    int ntiles, ncb, nkc;  // ntiles: tiles of the range
    int tile0;             // first tile of the range
    int64_t row_begin;     // rows before it are computed (whole tiles) but not stored
    int64_t row_end;       // rows at or past it are not stored
    int kc;             // channels per chunk (16, 32 or 64)
    int nb;             // accumulator columns per work unit
    int stages;
    uint32_t a_bytes, b_bytes, stage_bytes;
    uint32_t idesc;
    uint32_t tmem_cols;
    long long* trace;   // TB_TRACE builds only: per-role event stamps of CTA 0, else null
};

// Pipeline tracing (compiled in with -DTB_TRACE): CTA 0 stamps clock64 at each hand-off into
// p.trace laid out as [role][kTraceCap]; role 0 producer issue, 1 MMA full-wait done,
// 2 epilogue accumulator ready, 3 epilogue done, 4 loader tile staged.
constexpr int kTraceCap = 4096;
#ifdef TB_TRACE
#define TB_STAMP(role, idx)                                                                      \
    do {                                                                                         \
        if (p.trace && blockIdx.x == 0 && (idx) < kTraceCap) p.trace[(role) * kTraceCap + (idx)] = clock64(); \
    } while (0)
#else
#define TB_STAMP(role, idx) do { } while (0)
#endif

template <int RB>
__global__ void __launch_bounds__(kThreads, 1)
k_submconv_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap fmap,
              const ConvParams p) {
    constexpr int KSTEPS = RB / 32;      // K=16 MMAs per chunk
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);

    uint8_t* stage_base = smem;
    int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + (size_t)p.stages * p.stage_bytes);   // [2][27*128]
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(s_nbr) + 2 * kNbrSmem);
    // bars: full[kMaxStages] empty[kMaxStages] acc_full[2] acc_empty[2] nbr_full[2] nbr_empty[2] drain
    uint32_t* s_hdr = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 9);
    uint32_t* s_misc = s_hdr + kMaxStages;   // [0] tmem base, [1..2] tap masks, [3] abort
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 3);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
    auto accf_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + b); };
    auto acce_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + 2 + b); };
    auto nbrf_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + 4 + b); };
    auto nbre_bar = [&](int b) { return bar0 + 8u * (2 * kMaxStages + 6 + b); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kMaxStages + 8);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accf_bar(b), 1);
            mbar_init(acce_bar(b), 128);
            mbar_init(nbrf_bar(b), 1);
            mbar_init(nbre_bar(b), 1);
        }
        mbar_init(drain_bar, 1);
        s_misc[3] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&fmap)) : "memory");
    }
    if (warp == 6) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_misc[0];

    const int nunits = p.ntiles * p.ncb;
    const int32_t sentinel = (int32_t)p.n;

    if (warp == 4) {
        // ------------------------------------------------------------------ neighbor loader
        int it = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
            const int tile = p.tile0 + u / p.ncb;
            const int buf = it & 1;
            const uint32_t ph = (it >> 1) & 1;
            if (!mbar_wait(nbre_bar(buf), ph ^ 1, s_abort, p.err)) break;
            const int64_t r0 = (int64_t)tile * kTileM;
            int32_t* dst = s_nbr + buf * (27 * kTileM);
            uint32_t bits = 0;
#pragma unroll 3
            for (int t = 0; t < 27; ++t) {
                const int32_t* src = p.nbr + (int64_t)t * p.n + r0;
                int32_t v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int64_t row = r0 + lane + 32 * q;
                    v[q] = row < p.n ? __ldg(src + lane + 32 * q) : sentinel;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    dst[t * kTileM + lane + 32 * q] = v[q];
                    bits |= (uint32_t)(v[q] != sentinel) << t;
                }
            }
            bits = __reduce_or_sync(0xffffffffu, bits);
            if (lane == 0) s_misc[1 + buf] = bits;
            __syncwarp();
            if (lane == 0) mbar_arrive(nbrf_bar(buf));
            if (lane == 0) TB_STAMP(4, it);
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ TMA producer
        int gsi = 0;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int it = 0;
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
            const int cb = u % p.ncb;
            const int buf = it & 1;
            const uint32_t ph = (it >> 1) & 1;
            if (!mbar_wait(nbrf_bar(buf), ph, s_abort, p.err)) { ok = false; break; }
            const int32_t* rows_s = s_nbr + buf * (27 * kTileM);
            uint32_t taps = s_misc[1 + buf];
            const int nstages_unit = __popc(taps) * p.nkc;
            int si = 0;
            while (taps && ok) {
                const int t = __ffs(taps) - 1;
                taps &= taps - 1;
                const int4 rows = *reinterpret_cast<const int4*>(rows_s + t * kTileM + 4 * lane);
                for (int kc = 0; kc < p.nkc; ++kc, ++si) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, s_abort, p.err)) { ok = false; break; }
                    const uint32_t a_addr = smem_u32(stage_base + (size_t)stage * p.stage_bytes);
                    if (lane == 0) TB_STAMP(0, gsi);
                    ++gsi;
                    if (lane == 0) {
                        s_hdr[stage] = (si == 0 ? 1u : 0u) | (si == nstages_unit - 1 ? 2u : 0u);
                        mbar_arrive_expect_tx(full_bar(stage), p.a_bytes + p.b_bytes);
                    }
                    __syncwarp();
                    tma_gather4(a_addr + (uint32_t)(4 * lane * RB), &fmap, kc * p.kc, rows, full_bar(stage));
                    if (lane == 0)
                        tma_load_2d(a_addr + p.a_bytes, &wmap, t * p.ci + kc * p.kc, cb * p.nb, full_bar(stage));
                    if (++stage == p.stages) { stage = 0; phase ^= 1; }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbre_bar(buf));   // row indices are in registers / issued
        }
        if (!ok && lane == 0) {
            // let this CTA's in-flight TMA loads land before the CTA can exit
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp == 6) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int gsi = 0;
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
                    TB_STAMP(1, gsi);
                    ++gsi;
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
        const size_t esize = p.out_kind == 0 ? 4 : 2;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
            const int tile = p.tile0 + u / p.ncb, cb = u % p.ncb;
            const int ab = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            if (!mbar_wait(accf_bar(ab), aph, s_abort, p.err)) break;
            if (threadIdx.x == 0) TB_STAMP(2, it);
            tc_fence_after();
            const int64_t pos = (int64_t)tile * kTileM + q * 32 + lane;
            const bool valid = pos >= p.row_begin && pos < p.row_end;
            const int64_t row = (valid && p.perm) ? (int64_t)__ldg(p.perm + pos) : pos;
            uint8_t* orow = p.out + ((size_t)row * p.co + (size_t)cb * p.nb) * esize;
            for (int c0 = 0; c0 < p.nb; c0 += 16) {
                uint32_t v[16];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * p.nb + c0);
                TMEM_LD_X16(taddr, v);
                tmem_wait_ld();
                float a[16], f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) a[j] = __uint_as_float(v[j]);
                epi16(a, p.bias ? p.bias + cb * p.nb + c0 : nullptr, p.epi, f);
                if (valid) store16(orow + (size_t)c0 * esize, f, p.out_kind);
            }
            tc_fence_before();
            mbar_arrive(acce_bar(ab));
            if (threadIdx.x == 0) TB_STAMP(3, it);
        }
    }

    __syncthreads();
    if (warp == 6) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(p.tmem_cols) : "memory");
    }
}

}  // namespace

#ifdef TB_TRACE
long long* g_trace_buffer = nullptr;
extern "C" void tb_debug_set_trace(long long* buf) { g_trace_buffer = buf; }
#endif

bool tb_conv_tc_supported(int ci, int co) {
    const bool ci_ok = ci == 16 || ci == 32 || (ci > 0 && ci % 64 == 0);
    const bool co_ok = co > 0 && co % 16 == 0 && (co <= 256 || co % 256 == 0);
    return ci_ok && co_ok;
}

tb_status tb_conv_tc_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                            const void* feats, int ci, const void* weight, const float* bias, int co,
                            tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
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
    p.perm = nullptr;
    p.trace = nullptr;
#ifdef TB_TRACE
    p.trace = g_trace_buffer;
#endif
    p.feats = reinterpret_cast<const uint8_t*>(feats);
    p.bias = bias;
    p.out = reinterpret_cast<uint8_t*>(out);
    p.err = ctx->d_err;
    p.n = n;
    p.ci = ci;
    p.co = co;
    p.out_kind = out_dtype == TB_F32 ? 0 : (out_dtype == TB_F16 ? 1 : 2);
    p.epi = epi;
    p.tile0 = (int)(row0 / kTileM);
    p.row_begin = row0;
    p.row_end = row0 + nrows;
    p.ntiles = (int)((row0 + nrows + kTileM - 1) / kTileM) - p.tile0;
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

    const size_t fixed = 2 * kNbrSmem + 8 * (2 * kMaxStages + 9) + 4 * (kMaxStages + 4) + 1024;
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
    // feature rows for tile::gather4: [n][ci], box = one row of kc channels; row index n is out
    // of bounds and reads as zeros
    CUtensorMap fmap;
    const cuuint64_t fdim[2] = {(cuuint64_t)ci, (cuuint64_t)n};
    const cuuint64_t fstride[1] = {(cuuint64_t)ci * 2};
    const cuuint32_t fbox[2] = {(cuuint32_t)kc, 1};
    cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
        &fmap, dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
        const_cast<void*>(feats), fdim, fstride, fbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the feature view");

    const int units = p.ntiles * p.ncb;
    const int grid = std::min(units, ctx->num_sms);
    cudaError_t e;
    if (rb == 128) {
        e = cudaFuncSetAttribute(k_submconv_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<128><<<grid, kThreads, smem, ctx->stream>>>(map, fmap, p);
    } else if (rb == 64) {
        e = cudaFuncSetAttribute(k_submconv_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<64><<<grid, kThreads, smem, ctx->stream>>>(map, fmap, p);
    } else {
        e = cudaFuncSetAttribute(k_submconv_tc<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) k_submconv_tc<32><<<grid, kThreads, smem, ctx->stream>>>(map, fmap, p);
    }
    if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_tc)");
    TB_LAUNCH_CHECK(ctx, "k_submconv_tc");
    return TB_OK;
}
