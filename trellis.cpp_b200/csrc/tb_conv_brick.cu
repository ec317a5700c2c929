// Submanifold conv for Ci a multiple of 64: implicit GEMM with a per-tile "brick" of
// neighbor rows staged on chip, A operands assembled in TMEM, tcgen05 MMA.
//
// Why: every tap of a 128-voxel output tile reads 128 feature rows at scattered addresses.
// Gathering those rows from L2 once per tap (27 times per tile) tops out far below the
// tensor-core rate on B200 (scattered 128-byte rows reach roughly 20 B/clk per SM). But in
// the reference's voxel order (x-major, argwhere of a dense grid; src/ss_decoder.cpp:114),
// the ~450 distinct neighbor rows of 128 consecutive voxels fall into three contiguous row
// ranges, one per x offset (tap group kd = 0, 1, 2; the tap order of src/sparse.cpp:30-33).
// So each tile's neighbors are fetched once with large TMA boxes, and the per-tap gathers
// become shared-memory reads.
//
// Per 64-channel chunk kc of a work unit (tile, output-column block cb):
//   loader warp   stages the tile's 27x128 neighbor indices in smem, reduces them to the
//                 three [min, max] row ranges, and loads those rows (channels kc*64..+63) as
//                 32-row SW128 TMA boxes into one of two brick buffers. Rows beyond the
//                 brick capacity stay in global memory.
//   builder warps for each tap t, thread i (TMEM lane i = tile row i) reads its neighbor
//   (4-7)         row from the brick (or global memory if it overflowed; zeros if absent,
//                 the padded zero row of src/sparse.cpp:82-85) and writes it to a TMEM A slot
//                 with tcgen05.st (row i in lane i, bf16 pairs per column).
//   weight warp   TMA-loads the [nb x 64] weight slice of (t, kc) into a smem stage.
//   MMA warp      tcgen05.mma kind::f16, A from TMEM, B from smem, D (fp32) in TMEM;
//                 commits release the A slot, the weight stage and finally the accumulator.
//   epilogue      warps 0-3: tcgen05.ld, bias, SiLU, convert, store each row once.
// All 27 taps are issued for every tile (absent neighbors are zero rows); in this voxel order
// the union of present taps over 128 rows is 27 for almost every tile.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>
#include <climits>

namespace {

using namespace tbtc;

constexpr int kTileM = 128;
constexpr int kThreads = 352;        // 11 warps
constexpr int kBox = 32;             // rows per brick TMA box
constexpr int kNbrInts = 27 * kTileM;
constexpr int kNA = 8;               // TMEM A slots (32 columns each)
constexpr int kMaxB = 4;             // weight smem stages
constexpr int kNumBars = 2 + 2 + 2 + 2 + kNA + kNA + kMaxB + kMaxB + 2 + 2 + 1;

struct BrickMeta {
    int32_t lo[3];     // first row of each tap group's range
    int32_t len[3];    // rows of the range held in the brick
    int32_t off[3];    // brick row where the range starts
    int32_t nbox;      // 32-row boxes issued per channel chunk
    int32_t pad[2];
};

struct BrickParams {
    const int32_t* nbr;
    const uint8_t* feats;
    const float* bias;
    uint8_t* out;
    int* err;
    int64_t n;
    int ci, co;
    int out_kind, epi;
    int ntiles, ncb, nkc, nb;
    int nbst;              // weight stages
    int brick_cap;         // rows per brick buffer (multiple of kBox)
    uint32_t b_bytes;      // nb * 128
    uint32_t b_alloc;      // b_bytes rounded up to 1024
    int nd;                // accumulator buffers
    uint32_t a_col0;       // first TMEM column of the A slots
    uint32_t idesc;
    uint32_t tmem_cols;
};

__global__ void __launch_bounds__(kThreads, 1)
k_submconv_brick(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap fmap,
                 const BrickParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const size_t brick_bytes = (size_t)p.brick_cap * 128;
    uint8_t* brick_base = smem;                                        // [2][brick_cap][128]
    uint8_t* wst_base = smem + 2 * brick_bytes;                        // [nbst][b_alloc]
    int32_t* s_nbr = reinterpret_cast<int32_t*>(wst_base + (size_t)p.nbst * p.b_alloc);   // [2][27*128]
    BrickMeta* s_meta = reinterpret_cast<BrickMeta*>(s_nbr + 2 * kNbrInts);               // [2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_meta + 2);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kNumBars);   // [0] tmem base, [1] abort
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(bars);
    // barrier table
    const uint32_t nbrf = bar0, nbre = bar0 + 16, brkf = bar0 + 32, brke = bar0 + 48;
    const uint32_t af = bar0 + 64, ae = af + 8 * kNA;
    const uint32_t bf = ae + 8 * kNA, be = bf + 8 * kMaxB;
    const uint32_t df = be + 8 * kMaxB, de = df + 16, drain = de + 16;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(nbrf + 8 * b, 1);
            mbar_init(nbre + 8 * b, 4);
            mbar_init(brkf + 8 * b, 1);
            mbar_init(brke + 8 * b, 4);
            mbar_init(df + 8 * b, 1);
            mbar_init(de + 8 * b, 128);
        }
        for (int a = 0; a < kNA; ++a) {
            mbar_init(af + 8 * a, 4);
            mbar_init(ae + 8 * a, 1);
        }
        for (int s = 0; s < kMaxB; ++s) {
            mbar_init(bf + 8 * s, 1);
            mbar_init(be + 8 * s, 1);
        }
        mbar_init(drain, 1);
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&fmap)) : "memory");
    }
    if (warp == 10) {
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

    if (warp == 8) {
        // ------------------------------------------------------------------ loader
        int it = 0, bseq = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
            const int tile = u / p.ncb;
            const int buf = it & 1;
            if (!mbar_wait(nbre + 8 * buf, ((it >> 1) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
            const int64_t r0 = (int64_t)tile * kTileM;
            int32_t* dst = s_nbr + buf * kNbrInts;
            int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
#pragma unroll
            for (int g = 0; g < 3; ++g) {
#pragma unroll 3
                for (int tt = 0; tt < 9; ++tt) {
                    const int t = 9 * g + tt;
                    const int32_t* src = p.nbr + (int64_t)t * p.n + r0;
                    int32_t v[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        v[q] = (r0 + lane + 32 * q) < p.n ? __ldg(src + lane + 32 * q) : sentinel;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        dst[t * kTileM + lane + 32 * q] = v[q];
                        if (v[q] != sentinel) { lo[g] = min(lo[g], v[q]); hi[g] = max(hi[g], v[q]); }
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                lo[g] = __reduce_min_sync(0xffffffffu, lo[g]);
                hi[g] = __reduce_max_sync(0xffffffffu, hi[g]);
            }
            // brick layout: group g at 32-row aligned offset, clipped to the capacity
            int off = 0, nbox = 0;
            int glo[3], glen[3], goff[3];
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                const int len = hi[g] >= 0 ? hi[g] - lo[g] + 1 : 0;
                const int room = p.brick_cap - off;
                const int held = len < room ? len : room;
                glo[g] = hi[g] >= 0 ? lo[g] : 0;
                glen[g] = held;
                goff[g] = off;
                const int boxes = (held + kBox - 1) / kBox;
                off += boxes * kBox;
                nbox += boxes;
            }
            if (lane == 0) {
                BrickMeta& m = s_meta[buf];
#pragma unroll
                for (int g = 0; g < 3; ++g) { m.lo[g] = glo[g]; m.len[g] = glen[g]; m.off[g] = goff[g]; }
                m.nbox = nbox;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbrf + 8 * buf);
            for (int kc = 0; kc < p.nkc; ++kc, ++bseq) {
                const int slot = bseq & 1;
                if (!mbar_wait(brke + 8 * slot, ((bseq >> 1) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                const uint32_t bdst = smem_u32(brick_base + (size_t)slot * brick_bytes);
                if (lane == 0) mbar_arrive_expect_tx(brkf + 8 * slot, (uint32_t)nbox * kBox * 128);
                __syncwarp();
                // box j -> (group, index): lanes issue in parallel (nbox <= brick_cap/32 <= 32)
                for (int j = lane; j < nbox; j += 32) {
                    int g = 0, k = j;
                    const int b0 = (glen[0] + kBox - 1) / kBox, b1 = (glen[1] + kBox - 1) / kBox;
                    if (k >= b0) { k -= b0; g = 1; if (k >= b1) { k -= b1; g = 2; } }
                    tma_load_2d(bdst + (uint32_t)(goff[g] + k * kBox) * 128, &fmap, kc * 64, glo[g] + k * kBox,
                                brkf + 8 * slot);
                }
            }
        }
        if (!ok && lane == 0) {
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------------ A builders
        const int q = warp - 4;
        const int i = q * 32 + lane;                    // tile row = TMEM lane
        int it = 0, bseq = 0, aseq = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
            const int buf = it & 1;
            if (!mbar_wait(nbrf + 8 * buf, (it >> 1) & 1, s_abort, p.err)) { ok = false; break; }
            const BrickMeta m = s_meta[buf];
            const int32_t* rows = s_nbr + buf * kNbrInts;
            for (int kc = 0; kc < p.nkc && ok; ++kc, ++bseq) {
                const int slot = bseq & 1;
                if (!mbar_wait(brkf + 8 * slot, (bseq >> 1) & 1, s_abort, p.err)) { ok = false; break; }
                const uint8_t* brick = brick_base + (size_t)slot * brick_bytes;
#pragma unroll
                for (int g = 0; g < 3; ++g) {
                    const int glo = m.lo[g], glen = m.len[g], goff = m.off[g];
#pragma unroll 1
                    for (int tt = 0; tt < 9 && ok; ++tt, ++aseq) {
                        const int t = 9 * g + tt;
                        const int a = aseq % kNA;
                        if (!mbar_wait(ae + 8 * a, ((aseq / kNA) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                        const int32_t v = rows[t * kTileM + i];
                        uint32_t r[32];
                        if (v == sentinel) {
#pragma unroll
                            for (int k = 0; k < 32; ++k) r[k] = 0u;
                        } else {
                            const int pos = v - glo;
                            if (pos < glen) {
                                const int b = goff + pos;
                                const uint8_t* rowp = brick + (size_t)b * 128;
#pragma unroll
                                for (int c = 0; c < 8; ++c) {
                                    const uint4 x = *reinterpret_cast<const uint4*>(rowp + ((c ^ (b & 7)) << 4));
                                    r[4 * c] = x.x; r[4 * c + 1] = x.y; r[4 * c + 2] = x.z; r[4 * c + 3] = x.w;
                                }
                            } else {
                                const uint4* gp = reinterpret_cast<const uint4*>(
                                    p.feats + ((size_t)v * p.ci + (size_t)kc * 64) * 2);
#pragma unroll
                                for (int c = 0; c < 8; ++c) {
                                    const uint4 x = __ldg(gp + c);
                                    r[4 * c] = x.x; r[4 * c + 1] = x.y; r[4 * c + 2] = x.z; r[4 * c + 3] = x.w;
                                }
                            }
                        }
                        tmem_st_x32(tmem_base + ((uint32_t)(q * 32) << 16) + p.a_col0 + 32u * a, r);
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(af + 8 * a);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(brke + 8 * slot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbre + 8 * buf);
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------ weight producer
        if (lane == 0) {
            int seq = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
                const int cb = u % p.ncb;
                for (int kc = 0; kc < p.nkc && ok; ++kc) {
                    for (int t = 0; t < 27; ++t, ++seq) {
                        const int st = seq % p.nbst;
                        if (!mbar_wait(be + 8 * st, ((seq / p.nbst) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                        mbar_arrive_expect_tx(bf + 8 * st, p.b_bytes);
                        tma_load_2d(smem_u32(wst_base + (size_t)st * p.b_alloc), &wmap, t * p.ci + kc * 64,
                                    cb * p.nb, bf + 8 * st);
                    }
                }
            }
            if (!ok) {
                const long long t0 = clock64();
                while (clock64() - t0 < 4000000ll) __nanosleep(256);
            }
        }
    } else if (warp == 10) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int seq = 0, it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
                const int d = it % p.nd;
                if (!mbar_wait(de + 8 * d, ((it / p.nd) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dt = tmem_base + (uint32_t)(d * p.nb);
                for (int kc = 0; kc < p.nkc && ok; ++kc) {
                    for (int t = 0; t < 27; ++t, ++seq) {
                        const int a = seq % kNA;
                        const int st = seq % p.nbst;
                        if (!mbar_wait(af + 8 * a, (seq / kNA) & 1, s_abort, p.err)) { ok = false; break; }
                        if (!mbar_wait(bf + 8 * st, (seq / p.nbst) & 1, s_abort, p.err)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t at = tmem_base + p.a_col0 + 32u * a;
                        const uint32_t baddr = smem_u32(wst_base + (size_t)st * p.b_alloc);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            tc_mma_ts(dt, at + 8u * k, smem_desc<128>(baddr + 32 * k), p.idesc,
                                      (kc | t | k) != 0 ? 1u : 0u);
                        tc_commit(ae + 8 * a);
                        tc_commit(be + 8 * st);
                    }
                }
                if (!ok) break;
                tc_commit(df + 8 * d);
            }
            tc_commit(drain);
            const long long t0 = clock64();
            while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) __nanosleep(64);
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int q = warp;
        int it = 0;
        const size_t esize = p.out_kind == 0 ? 4 : 2;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
            const int tile = u / p.ncb, cb = u % p.ncb;
            const int d = it % p.nd;
            if (!mbar_wait(df + 8 * d, (it / p.nd) & 1, s_abort, p.err)) break;
            tc_fence_after();
            const int64_t row = (int64_t)tile * kTileM + q * 32 + lane;
            const bool valid = row < p.n;
            uint8_t* orow = p.out + ((size_t)row * p.co + (size_t)cb * p.nb) * esize;
            for (int c0 = 0; c0 < p.nb; c0 += 16) {
                uint32_t v[16];
                const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(d * p.nb + c0);
                TMEM_LD_X16(taddr, v);
                tmem_wait_ld();
                float f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int o = cb * p.nb + c0 + j;
                    const float x = __uint_as_float(v[j]) + (p.bias ? __ldg(p.bias + o) : 0.0f);
                    f[j] = apply_epi(x, p.epi);
                }
                if (valid) store16(orow + (size_t)c0 * esize, f, p.out_kind);
            }
            tc_fence_before();
            mbar_arrive(de + 8 * d);
        }
    }

    __syncthreads();
    if (warp == 10) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(p.tmem_cols) : "memory");
    }
}

}  // namespace

bool tb_conv_brick_supported(int ci, int co) {
    return ci > 0 && ci % 64 == 0 && co > 0 && co % 16 == 0 && (co <= 256 || co % 256 == 0);
}

tb_status tb_conv_brick_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, const void* feats, int ci,
                               const void* weight, const float* bias, int co, tb_dtype dtype,
                               tb_dtype out_dtype, tb_epilogue epi, void* out) {
    if (!tb_conv_brick_supported(ci, co))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "brick conv needs ci%64==0 and co%16==0 (<=256 or 256k)");
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    const int nb = co <= 256 ? co : 256;
    BrickParams p{};
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
    p.nkc = ci / 64;
    p.nb = nb;
    p.b_bytes = (uint32_t)nb * 128;
    p.b_alloc = (p.b_bytes + 1023u) & ~1023u;
    p.nbst = nb <= 128 ? kMaxB : 2;
    p.nd = (2 * nb + 32 * kNA <= 512) ? 2 : 1;
    p.a_col0 = (uint32_t)(p.nd * nb);
    uint32_t cols = 32;
    while (cols < p.a_col0 + 32u * kNA) cols <<= 1;
    p.tmem_cols = cols;
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(nb >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);

    const size_t fixed = 2 * (size_t)kNbrInts * 4 + 2 * sizeof(BrickMeta) + 8 * kNumBars + 16 + 1024;
    const size_t budget = (size_t)ctx->max_smem_optin;
    const size_t wbytes = (size_t)p.nbst * p.b_alloc;
    if (budget < fixed + wbytes + 2 * 128 * 128)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "brick conv: shared memory too small");
    int cap = (int)((budget - fixed - wbytes) / (2 * 128));
    cap = (cap / kBox) * kBox;
    if (cap > 32 * kBox) cap = 32 * kBox;    // at most 32 boxes per brick (one per lane)
    p.brick_cap = cap;
    const size_t smem = fixed + wbytes + 2 * (size_t)cap * 128;

    CUtensorMap wmap, fmap;
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)27 * ci, (cuuint64_t)co};
        const cuuint64_t gstride[1] = {(cuuint64_t)27 * ci * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)nb};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &wmap, dt, 2, const_cast<void*>(weight), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight view");
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)ci, (cuuint64_t)n};
        const cuuint64_t gstride[1] = {(cuuint64_t)ci * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)kBox};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &fmap, dt, 2, const_cast<void*>(feats), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the feature view");
    }
    const int units = p.ntiles * p.ncb;
    const int grid = std::min(units, ctx->num_sms);
    cudaError_t e = cudaFuncSetAttribute(k_submconv_brick, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_brick)");
    k_submconv_brick<<<grid, kThreads, smem, ctx->stream>>>(wmap, fmap, p);
    TB_LAUNCH_CHECK(ctx, "k_submconv_brick");
    return TB_OK;
}
