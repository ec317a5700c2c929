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
// Per 64-channel chunk kc of a work unit (tile, output-column block cb) -- a "group" of 27
// stages, one per tap, numbered by a running stage sequence:
//   loader warp     stages the tile's 27x128 neighbor indices in smem, reduces them to the
//                   three [min, max] row ranges, and loads those rows (channels kc*64..+63) as
//                   32-row SW128 TMA boxes into one of two brick buffers. Rows beyond the
//                   brick capacity stay in global memory.
//   builder warps   two warpgroups take alternate stages. Thread i (TMEM lane i = tile row i)
//   (4-11)          reads its neighbor row from the brick (or global memory if it overflowed;
//                   zeros if absent, the padded zero row of src/sparse.cpp:82-85) and writes
//                   it to a TMEM A slot with tcgen05.st (row i in lane i, bf16 pairs per
//                   column). Each warp keeps two stages' rows in flight.
//   weight warps    up to four warps, each owning every fourth stage, TMA-load the [nb x 64]
//   (13-16)         weight slice of (tap, kc) into a smem stage (one thread's TMA issues
//                   serialise, so several threads issue).
//   MMA warps       tcgen05.mma kind::f16, A from TMEM, B from smem, D (fp32) in TMEM. For
//   (17-18)         nb <= 64 two warps issue alternate stages into two accumulators, because
//                   one issuing thread sustains one MMA per ~64 cycles, twice the math time of
//                   a 128x64x16 MMA; the epilogue adds the two. Commits release the A slot,
//                   the weight stage and finally the accumulator.
//   epilogue        warps 0-3: tcgen05.ld, bias, SiLU, convert, store each row once.
// All 27 taps are issued for every tile (absent neighbors are zero rows); in this voxel order
// the union of present taps over 128 rows is 27 for almost every tile. Each unit starts its
// tap sequence at tap (unit mod 27); the fp32 accumulation order therefore differs between
// tiles but is fixed for a given launch shape.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>
#include <climits>

namespace {

using namespace tbtc;

constexpr int kTileM = 128;
constexpr int kWarpBuild0 = 4;       // builders: warps 4-11
constexpr int kWarpLoader = 12;
constexpr int kWarpWeight0 = 13;     // weight producers: warps 13-16
constexpr int kWeightWarps = 4;
constexpr int kWarpMma0 = 17;        // MMA issuers: warps 17-18
constexpr int kThreads = 19 * 32;
constexpr int kBox = 32;             // rows per brick TMA box
constexpr int kNbrInts = 27 * kTileM;
constexpr int kNA = 8;               // TMEM A slots (32 columns each); a power of two
constexpr int kMaxB = 8;             // weight smem stages (nbst is 2, 4 or 8)
// nbrf[2] nbre[2] brkf[2] brke[2] af[8] ae[8] bf[8] be[8] df[2][2] de[2][2] drain
constexpr int kNumBars = 2 + 2 + 2 + 2 + kNA + kNA + kMaxB + kMaxB + 4 + 4 + 1;

// Pipeline tracing (compiled in with -DTB_TRACE): CTA 0 stamps clock64 into p.trace laid out
// as [role][kTraceCap]: 0 loader brick issued, 1 builder A slot written, 2 MMA stage inputs
// ready, 3 weight stage issued, 4 epilogue accumulator ready.
constexpr int kTraceCap = 4096;
#ifdef TB_TRACE
#define TB_STAMP(role, idx)                                                                       \
    do {                                                                                          \
        if (p.trace && blockIdx.x == 0 && (idx) < kTraceCap) p.trace[(role) * kTraceCap + (idx)] = clock64(); \
    } while (0)
#define TB_PROGRESS(slot, v)                                                                      \
    do {                                                                                          \
        if (p.trace) *(volatile long long*)&p.trace[5 * kTraceCap + blockIdx.x * 8 + (slot)] = (v);  \
    } while (0)
#else
#define TB_STAMP(role, idx) do { } while (0)
#define TB_PROGRESS(slot, v) do { } while (0)
#endif

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
    int ntiles, ncb, nkc, nb;  // ntiles: tiles of the range
    int tile0;                 // first tile of the range
    int64_t row_begin;         // rows before it are computed (whole tiles) but not stored
    int64_t row_end;           // rows at or past it are not stored
    int nbst, nbst_log2;   // weight stages (2, 4 or 8)
    int brick_cap;         // rows per brick buffer (multiple of kBox)
    uint32_t b_bytes;      // nb * 128
    uint32_t b_alloc;      // b_bytes rounded up to 1024
    int nd;                // accumulator buffers per issuer (1 or 2)
    int niss;              // MMA issuer warps (1 or 2)
    uint32_t a_col0;       // first TMEM column of the A slots
    uint32_t idesc;
    uint32_t tmem_cols;
    long long* trace;      // TB_TRACE builds only
};

// Tap order within a stage group starts at tap `rot` (the unit index mod 27), so CTAs that
// run at the same time fetch different weight slices instead of all hitting the same L2 lines.
__device__ __forceinline__ int rot_tap(int rot, int j) {
    const int t = rot + j;
    return t >= 27 ? t - 27 : t;
}

// Row of the tap-t neighbor for this thread, from the brick or global memory (zeros if absent).
__device__ __forceinline__ void load_nbr_row(const BrickParams& p, const BrickMeta& m, const uint8_t* brick,
                                             int32_t v, int t, int kc, uint32_t* r) {
    if (v == (int32_t)p.n) {
#pragma unroll
        for (int k = 0; k < 32; ++k) r[k] = 0u;
        return;
    }
    const int glo = t < 9 ? m.lo[0] : (t < 18 ? m.lo[1] : m.lo[2]);
    const int glen = t < 9 ? m.len[0] : (t < 18 ? m.len[1] : m.len[2]);
    const int goff = t < 9 ? m.off[0] : (t < 18 ? m.off[1] : m.off[2]);
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
        const uint4* gp = reinterpret_cast<const uint4*>(p.feats + ((size_t)v * p.ci + (size_t)kc * 64) * 2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 x = __ldg(gp + c);
            r[4 * c] = x.x; r[4 * c + 1] = x.y; r[4 * c + 2] = x.z; r[4 * c + 3] = x.w;
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
k_submconv_brick(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap fmap,
                 const BrickParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
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
    const uint32_t nbrf = bar0, nbre = bar0 + 16, brkf = bar0 + 32, brke = bar0 + 48;
    const uint32_t af = bar0 + 64, ae = af + 8 * kNA;
    const uint32_t bf = ae + 8 * kNA, be = bf + 8 * kMaxB;
    const uint32_t df = be + 8 * kMaxB, de = df + 32, drain = de + 32;   // df/de: [issuer][buffer]

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(nbrf + 8 * b, 1);
            mbar_init(nbre + 8 * b, 8);
            mbar_init(brkf + 8 * b, 1);
            mbar_init(brke + 8 * b, 8);
        }
        for (int k = 0; k < 4; ++k) {
            mbar_init(df + 8 * k, 1);
            mbar_init(de + 8 * k, 128);
        }
        for (int a = 0; a < kNA; ++a) {
            mbar_init(af + 8 * a, 4);
            mbar_init(ae + 8 * a, 1);
        }
        for (int s = 0; s < kMaxB; ++s) {
            mbar_init(bf + 8 * s, 1);
            mbar_init(be + 8 * s, 1);
        }
        mbar_init(drain, (uint32_t)p.niss);   // one commit from each issuer completes phase 0
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&fmap)) : "memory");
    }
    if (warp == kWarpMma0) {
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

    if (warp == kWarpLoader) {
        // ------------------------------------------------------------------ loader
        int it = 0, bseq = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
            const int tile = p.tile0 + u / p.ncb;
            const int buf = it & 1;
            if (!mbar_wait(nbre + 8 * buf, ((it >> 1) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
            const int64_t r0 = (int64_t)tile * kTileM;
            int32_t* dst = s_nbr + buf * kNbrInts;
            // all 108 indices of this lane in flight at once (the map is usually not L2-resident)
            for (int t = 0; t < 27; ++t) {
                const int32_t* src = p.nbr + (int64_t)t * p.n + r0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int r = lane + 32 * q;
                    if (r0 + r < p.n) cp_async_4(smem_u32(dst + t * kTileM + r), src + r);
                    else dst[t * kTileM + r] = sentinel;
                }
            }
            cp_async_wait_all();
            __syncwarp();
            int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                for (int tt = 0; tt < 9; ++tt) {
                    const int t = 9 * g + tt;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int32_t v = dst[t * kTileM + lane + 32 * q];
                        if (v != sentinel) { lo[g] = min(lo[g], v); hi[g] = max(hi[g], v); }
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                lo[g] = __reduce_min_sync(0xffffffffu, lo[g]);
                hi[g] = __reduce_max_sync(0xffffffffu, hi[g]);
            }
            // brick layout: group g at a 32-row aligned offset, clipped to the capacity
            int off = 0, nbox = 0;
            int glo[3], glen[3], goff[3], gbox[3];
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                const int len = hi[g] >= 0 ? hi[g] - lo[g] + 1 : 0;
                const int room = p.brick_cap - off;
                const int held = len < room ? len : room;
                glo[g] = hi[g] >= 0 ? lo[g] : 0;
                glen[g] = held;
                goff[g] = off;
                gbox[g] = (held + kBox - 1) / kBox;
                off += gbox[g] * kBox;
                nbox += gbox[g];
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
                // box j -> (group, index); lanes issue in parallel (nbox <= brick_cap/32 <= 32)
                for (int j = lane; j < nbox; j += 32) {
                    int g = 0, k = j;
                    if (k >= gbox[0]) { k -= gbox[0]; g = 1; if (k >= gbox[1]) { k -= gbox[1]; g = 2; } }
                    const int go = g == 0 ? goff[0] : (g == 1 ? goff[1] : goff[2]);
                    const int gl = g == 0 ? glo[0] : (g == 1 ? glo[1] : glo[2]);
                    tma_load_2d(bdst + (uint32_t)(go + k * kBox) * 128, &fmap, kc * 64, gl + k * kBox, brkf + 8 * slot);
                }
                if (lane == 0) { TB_STAMP(0, bseq); TB_PROGRESS(0, bseq + 1); }
            }
        }
        if (!ok && lane == 0) {
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp >= kWarpBuild0 && warp < kWarpBuild0 + 8) {
        // ------------------------------------------------------------------ A builders
        const int q = warp & 3;                         // TMEM subpartition (warp id % 4)
        const int half = (warp - kWarpBuild0) >> 2;     // builds stages with seq % 2 == half
        const int i = q * 32 + lane;                    // tile row = TMEM lane
        const uint32_t a_lane = tmem_base + ((uint32_t)(q * 32) << 16) + p.a_col0;
        int it = 0, bseq = 0, seq0 = 0;                 // seq0: stage sequence of tap 0 of the group
        bool ok = true;
        for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
            const int buf = it & 1;
            if (!mbar_wait(nbrf + 8 * buf, (it >> 1) & 1, s_abort, p.err)) { ok = false; break; }
            const BrickMeta m = s_meta[buf];
            const int32_t* rows = s_nbr + buf * kNbrInts;
            const int rot = u % 27;
            for (int kc = 0; kc < p.nkc && ok; ++kc, ++bseq, seq0 += 27) {
                const int slot = bseq & 1;
                if (!mbar_wait(brkf + 8 * slot, (bseq >> 1) & 1, s_abort, p.err)) { ok = false; break; }
                const uint8_t* brick = brick_base + (size_t)slot * brick_bytes;
                // this half's stages: position j with (seq0 + j) % 2 == half, two at a time; the
                // tap of position j is (rot + j) % 27
                for (int j = (half ^ seq0) & 1; j < 27 && ok; j += 4) {
                    const int j2 = j + 2;
                    const bool has2 = j2 < 27;
                    const int t = rot_tap(rot, j), t2 = rot_tap(rot, j2);
                    uint32_t r0[32], r1[32];
                    load_nbr_row(p, m, brick, rows[t * kTileM + i], t, kc, r0);
                    if (has2) load_nbr_row(p, m, brick, rows[t2 * kTileM + i], t2, kc, r1);
                    const int s1 = seq0 + j, s2 = seq0 + j2;
                    const int a1 = s1 & (kNA - 1), a2 = s2 & (kNA - 1);
                    if (!mbar_wait(ae + 8 * a1, ((s1 >> 3) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                    tmem_st_x32(a_lane + 32u * a1, r0);
                    if (has2) {
                        if (!mbar_wait(ae + 8 * a2, ((s2 >> 3) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                        tmem_st_x32(a_lane + 32u * a2, r1);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(af + 8 * a1);
                        if (has2) mbar_arrive(af + 8 * a2);
                        if (q == 0) { TB_STAMP(1, s1); TB_PROGRESS(1 + half, s1 + 1); }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(brke + 8 * slot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbre + 8 * buf);
        }
    } else if (warp >= kWarpWeight0 && warp < kWarpWeight0 + kWeightWarps) {
        // ------------------------------------------------------------------ weight producers
        // stage st is always loaded by warp st % nw (nbst is a multiple of nw), so each stage's
        // loads stay in order; a stage shared by two warps could be refilled a phase early
        const int wk = warp - kWarpWeight0;
        const int nw = p.nbst < kWeightWarps ? p.nbst : kWeightWarps;
        if (lane == 0 && wk < nw) {
            int seq = wk;
            bool ok = true;
            const int stages_per_unit = 27 * p.nkc;
            int it = 0;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
                const int cb = u % p.ncb;
                const int unit_end = (it + 1) * stages_per_unit;
                for (; seq < unit_end; seq += nw) {
                    const int local = seq - it * stages_per_unit;
                    const int kc = local / 27, t = rot_tap(u % 27, local - kc * 27);
                    const int st = seq & (p.nbst - 1);
                    if (!mbar_wait(be + 8 * st, ((seq >> p.nbst_log2) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(bf + 8 * st, p.b_bytes);
                    tma_load_2d(smem_u32(wst_base + (size_t)st * p.b_alloc), &wmap, t * p.ci + kc * 64, cb * p.nb,
                                bf + 8 * st);
                    TB_STAMP(3, seq);
                    TB_PROGRESS(3, seq + 1);
                }
            }
            if (!ok) {
                const long long t0 = clock64();
                while (clock64() - t0 < 4000000ll) __nanosleep(256);
            }
        }
    } else if (warp >= kWarpMma0 && warp < kWarpMma0 + 2) {
        // ------------------------------------------------------------------ MMA issuers
        const int mi = warp - kWarpMma0;
        if (lane == 0 && mi < p.niss) {
            const uint64_t bdesc0 = smem_desc<128>(smem_u32(wst_base));
            const uint32_t bstep = p.b_alloc >> 4;              // descriptor address units per stage
            const uint32_t a0 = tmem_base + p.a_col0;
            const int stages_per_unit = 27 * p.nkc;
            int seq = mi, it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++it) {
                const int d = p.nd == 2 ? (it & 1) : 0;
                const uint32_t dph = p.nd == 2 ? ((it >> 1) & 1) : (it & 1);
                const int dk = mi * 2 + d;
                if (!mbar_wait(de + 8 * dk, dph ^ 1, s_abort, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dt = tmem_base + (uint32_t)((mi * p.nd + d) * p.nb);
                const int unit_end = (it + 1) * stages_per_unit;
                uint32_t acc = 0;
                for (; seq < unit_end; seq += p.niss) {
                    const int a = seq & (kNA - 1);
                    const int st = seq & (p.nbst - 1);
                    if (!mbar_wait(af + 8 * a, (seq >> 3) & 1, s_abort, p.err)) { ok = false; break; }
                    if (!mbar_wait(bf + 8 * st, (seq >> p.nbst_log2) & 1, s_abort, p.err)) { ok = false; break; }
                    TB_STAMP(2, seq);
                    TB_PROGRESS(4 + mi, seq + 1);
                    tc_fence_after();
                    const uint32_t at = a0 + 32u * (uint32_t)a;
                    const uint64_t bd = bdesc0 + (uint64_t)(bstep * (uint32_t)st);
                    tc_mma_ts(dt, at, bd, p.idesc, acc);
                    tc_mma_ts(dt, at + 8, bd + 2, p.idesc, 1u);
                    tc_mma_ts(dt, at + 16, bd + 4, p.idesc, 1u);
                    tc_mma_ts(dt, at + 24, bd + 6, p.idesc, 1u);
                    acc = 1u;
                    tc_commit(ae + 8 * a);
                    tc_commit(be + 8 * st);
                }
                if (!ok) break;
                tc_commit(df + 8 * dk);
            }
            tc_commit(drain);
            const long long t0 = clock64();
            while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) __nanosleep(64);
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------------ epilogue
        const int q = warp;
        int it = 0;
        const size_t esize = p.out_kind == 0 ? 4 : 2;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
            const int tile = p.tile0 + u / p.ncb, cb = u % p.ncb;
            const int d = p.nd == 2 ? (it & 1) : 0;
            const uint32_t dph = p.nd == 2 ? ((it >> 1) & 1) : (it & 1);
            bool ok = mbar_wait(df + 8 * d, dph, s_abort, p.err);
            if (ok && p.niss == 2) ok = mbar_wait(df + 8 * (2 + d), dph, s_abort, p.err);
            if (!ok) break;
            if (threadIdx.x == 0) { TB_STAMP(4, it); TB_PROGRESS(6, it + 1); }
            tc_fence_after();
            const int64_t row = (int64_t)tile * kTileM + q * 32 + lane;
            const bool valid = row >= p.row_begin && row < p.row_end;
            uint8_t* orow = p.out + ((size_t)row * p.co + (size_t)cb * p.nb) * esize;
            const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
            const uint32_t d0 = lane_base + (uint32_t)(d * p.nb);
            const uint32_t d1 = lane_base + (uint32_t)((p.nd + d) * p.nb);
            for (int c0 = 0; c0 < p.nb; c0 += 16) {
                uint32_t v[16], w[16];
                TMEM_LD_X16(d0 + c0, v);
                if (p.niss == 2) {
                    TMEM_LD_X16(d1 + c0, w);
                }
                tmem_wait_ld();
                float a[16], f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) a[j] = __uint_as_float(v[j]) + (p.niss == 2 ? __uint_as_float(w[j]) : 0.0f);
                epi16(a, p.bias ? p.bias + cb * p.nb + c0 : nullptr, p.epi, f);
                if (valid) store16(orow + (size_t)c0 * esize, f, p.out_kind);
            }
            tc_fence_before();
            mbar_arrive(de + 8 * d);
            if (p.niss == 2) mbar_arrive(de + 8 * (2 + d));
        }
    }

    __syncthreads();
    if (warp == kWarpMma0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(p.tmem_cols) : "memory");
    }
}

// ---- CTA-pair form ---------------------------------------------------------------------------
// The same pipeline on two CTAs of a cluster (neighbouring SMs) sharing each MMA, for output
// column blocks of 128 or more: each CTA loads its own tile's indices and brick and builds its
// own 128 rows of A in its TMEM, but streams only half of every weight slice (nb / 2 output
// columns); the even CTA issues tcgen05.mma.cta_group::2 with M = 256, whose B operand is the two
// halves and whose D rows land in each CTA's TMEM. Per output row that halves the weight bytes
// streamed from L2 and doubles the work each stage hand-off covers.
// Cross-CTA hand-offs: one barrier of the even CTA per stage collects both CTAs' builder warps,
// the even CTA's weight TMA and the odd CTA's weight half, which the odd CTA's first MMA warp
// passes on once its TMA has landed, so the issuer waits once per stage; epilogue warps arrive on
// the even CTA's barriers; MMA commits multicast to both CTAs. The cross-CTA arrives and waits
// are relaxed at cluster scope: with release / acquire the hand-offs took more than twice as long
// (C2: 1.17 ms against 0.75 ms per conv). Every wait is bounded and aborts the CTA cleanly.
constexpr int kNumBarsPair = kNumBars;
constexpr int kPairMinNb = 128;                 // output column blocks at least this wide use the pair

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
k_submconv_brick_pair(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap fmap,
                      const BrickParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    const size_t brick_bytes = (size_t)p.brick_cap * 128;
    uint8_t* brick_base = smem;                                        // [2][brick_cap][128]
    uint8_t* wst_base = smem + 2 * brick_bytes;                        // [nbst][b_alloc]
    int32_t* s_nbr = reinterpret_cast<int32_t*>(wst_base + (size_t)p.nbst * p.b_alloc);   // [2][27*128]
    BrickMeta* s_meta = reinterpret_cast<BrickMeta*>(s_nbr + 2 * kNbrInts);               // [2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_meta + 2);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kNumBarsPair);   // [0] tmem base, [1] abort
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t bar0 = smem_u32(bars);
    const uint32_t nbrf = bar0, nbre = bar0 + 16, brkf = bar0 + 32, brke = bar0 + 48;
    const uint32_t af = bar0 + 64, ae = af + 8 * kNA;
    const uint32_t bf = ae + 8 * kNA, be = bf + 8 * kMaxB;
    const uint32_t df = be + 8 * kMaxB, de = df + 32, drain = de + 32;   // df/de: [issuer][buffer]

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(nbrf + 8 * b, 1);
            mbar_init(nbre + 8 * b, 8);
            mbar_init(brkf + 8 * b, 1);
            mbar_init(brke + 8 * b, 8);
        }
        for (int k = 0; k < 4; ++k) {
            mbar_init(df + 8 * k, 1);
            mbar_init(de + 8 * k, 8);        // four epilogue warps in each CTA (even CTA's copy used)
        }
        for (int a = 0; a < kNA; ++a) {
            // stage seq is ready when af[seq % kNA] of the even CTA has: four builder warps of each
            // CTA, the odd CTA's weight half (forwarded) and the even CTA's own weight TMA
            mbar_init(af + 8 * a, 10);
            mbar_init(ae + 8 * a, 1);
        }
        for (int s = 0; s < kMaxB; ++s) {
            mbar_init(bf + 8 * s, 1);
            mbar_init(be + 8 * s, 1);
        }
        mbar_init(drain, (uint32_t)p.niss);
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&fmap)) : "memory");
    }
    if (warp == kWarpMma0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync_all();                       // both CTAs' barriers and TMEM exist before any cross-CTA use
    tc_fence_after();
    const uint32_t tmem_base = s_misc[0];
    const int npairs = (p.ntiles + 1) / 2;
    const int nunits = npairs * p.ncb;
    const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();
    const int32_t sentinel = (int32_t)p.n;

    if (warp == kWarpLoader) {
        // ------------------------------------------------------------------ loader (per CTA)
        int it = 0, bseq = 0;
        bool ok = true;
        for (int u = cid; u < nunits && ok; u += ncl, ++it) {
            const int tile = p.tile0 + 2 * (u / p.ncb) + (int)rank;
            const int buf = it & 1;
            if (!mbar_wait(nbre + 8 * buf, ((it >> 1) & 1) ^ 1, s_abort, p.err)) { ok = false; break; }
            const int64_t r0 = (int64_t)tile * kTileM;
            int32_t* dst = s_nbr + buf * kNbrInts;
            for (int t = 0; t < 27; ++t) {
                const int32_t* src = p.nbr + (int64_t)t * p.n + r0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int r = lane + 32 * q;
                    if (r0 + r < p.n) cp_async_4(smem_u32(dst + t * kTileM + r), src + r);
                    else dst[t * kTileM + r] = sentinel;
                }
            }
            cp_async_wait_all();
            __syncwarp();
            int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                for (int tt = 0; tt < 9; ++tt) {
                    const int t = 9 * g + tt;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int32_t v = dst[t * kTileM + lane + 32 * q];
                        if (v != sentinel) { lo[g] = min(lo[g], v); hi[g] = max(hi[g], v); }
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                lo[g] = __reduce_min_sync(0xffffffffu, lo[g]);
                hi[g] = __reduce_max_sync(0xffffffffu, hi[g]);
            }
            int off = 0, nbox = 0;
            int glo[3], glen[3], goff[3], gbox[3];
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                const int len = hi[g] >= 0 ? hi[g] - lo[g] + 1 : 0;
                const int room = p.brick_cap - off;
                const int held = len < room ? len : room;
                glo[g] = hi[g] >= 0 ? lo[g] : 0;
                glen[g] = held;
                goff[g] = off;
                gbox[g] = (held + kBox - 1) / kBox;
                off += gbox[g] * kBox;
                nbox += gbox[g];
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
                for (int j = lane; j < nbox; j += 32) {
                    int g = 0, k = j;
                    if (k >= gbox[0]) { k -= gbox[0]; g = 1; if (k >= gbox[1]) { k -= gbox[1]; g = 2; } }
                    const int go = g == 0 ? goff[0] : (g == 1 ? goff[1] : goff[2]);
                    const int gl = g == 0 ? glo[0] : (g == 1 ? glo[1] : glo[2]);
                    tma_load_2d(bdst + (uint32_t)(go + k * kBox) * 128, &fmap, kc * 64, gl + k * kBox, brkf + 8 * slot);
                }
            }
        }
        if (!ok && lane == 0) {
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp >= kWarpBuild0 && warp < kWarpBuild0 + 8) {
        // ------------------------------------------------------------------ A builders (per CTA)
        const int q = warp & 3;
        const int half = (warp - kWarpBuild0) >> 2;
        const int i = q * 32 + lane;
        const uint32_t a_lane = tmem_base + ((uint32_t)(q * 32) << 16) + p.a_col0;
        int it = 0, bseq = 0, seq0 = 0;
        bool ok = true;
        for (int u = cid; u < nunits && ok; u += ncl, ++it) {
            const int buf = it & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(nbrf + 8 * buf, (it >> 1) & 1, s_abort, p.err))) { ok = false; break; }
            const BrickMeta m = s_meta[buf];
            const int32_t* rows = s_nbr + buf * kNbrInts;
            const int rot = u % 27;
            for (int kc = 0; kc < p.nkc && ok; ++kc, ++bseq, seq0 += 27) {
                const int slot = bseq & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(brkf + 8 * slot, (bseq >> 1) & 1, s_abort, p.err))) {
                    ok = false;
                    break;
                }
                const uint8_t* brick = brick_base + (size_t)slot * brick_bytes;
                for (int j = (half ^ seq0) & 1; j < 27 && ok; j += 4) {
                    const int j2 = j + 2;
                    const bool has2 = j2 < 27;
                    const int t = rot_tap(rot, j), t2 = rot_tap(rot, j2);
                    uint32_t r0[32], r1[32];
                    load_nbr_row(p, m, brick, rows[t * kTileM + i], t, kc, r0);
                    if (has2) load_nbr_row(p, m, brick, rows[t2 * kTileM + i], t2, kc, r1);
                    const int s1 = seq0 + j, s2 = seq0 + j2;
                    const int a1 = s1 & (kNA - 1), a2 = s2 & (kNA - 1);
                    // the slots' previous stages have been multiplied (commits reach both CTAs)
                    if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(ae + 8 * a1, ((s1 >> 3) & 1) ^ 1, s_abort,
                                                                           p.err))) { ok = false; break; }
                    if (has2 && !__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(ae + 8 * a2, ((s2 >> 3) & 1) ^ 1,
                                                                                   s_abort, p.err))) { ok = false; break; }
                    tc_fence_after();
                    tmem_st_x32(a_lane + 32u * a1, r0);
                    if (has2) tmem_st_x32(a_lane + 32u * a2, r1);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive_cluster_relaxed(af + 8 * a1, 0);
                        if (has2) mbar_arrive_cluster_relaxed(af + 8 * a2, 0);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(brke + 8 * slot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbre + 8 * buf);
        }
    } else if (warp >= kWarpWeight0 && warp < kWarpWeight0 + kWeightWarps) {
        // ------------------------------------------------------------------ weight producers (per CTA)
        // this CTA's half of each [nb x 64] slice: output columns cb*nb + rank*nb/2 .. + nb/2
        const int wk = warp - kWarpWeight0;
        const int nw = p.nbst < kWeightWarps ? p.nbst : kWeightWarps;
        if (lane == 0 && wk < nw) {
            int seq = wk;
            bool ok = true;
            const int stages_per_unit = 27 * p.nkc;
            int it = 0;
            for (int u = cid; u < nunits && ok; u += ncl, ++it) {
                const int cb = u % p.ncb;
                const int unit_end = (it + 1) * stages_per_unit;
                for (; seq < unit_end; seq += nw) {
                    const int local = seq - it * stages_per_unit;
                    const int kc = local / 27, t = rot_tap(u % 27, local - kc * 27);
                    const int st = seq & (p.nbst - 1);
                    // the stage's previous slice has been multiplied (the commit reaches both CTAs)
                    if (!mbar_wait_cluster_relaxed(be + 8 * st, ((seq >> p.nbst_log2) & 1) ^ 1, s_abort, p.err)) {
                        ok = false;
                        break;
                    }
                    // the even CTA's half completes on the stage's ready barrier directly; the odd
                    // CTA's on its own barrier, which the forwarder passes on
                    const uint32_t done = leader ? af + 8 * (seq & (kNA - 1)) : bf + 8 * st;
                    mbar_arrive_expect_tx(done, p.b_bytes);
                    tma_load_2d(smem_u32(wst_base + (size_t)st * p.b_alloc), &wmap, t * p.ci + kc * 64,
                                cb * p.nb + (int)rank * (p.nb / 2), done);
                }
            }
            if (!ok) {
                const long long t0 = clock64();
                while (clock64() - t0 < 4000000ll) __nanosleep(256);
            }
        }
    } else if (warp == kWarpMma0 && !leader) {
        // ------------------------------------------------------------------ odd CTA: stage forwarder
        // each of this CTA's weight stages, once its TMA has landed, is passed on to the even CTA
        if (lane == 0) {
            const int total = ((nunits - cid + ncl - 1) / ncl) * 27 * p.nkc;   // stages of this cluster's units
            for (int seq = 0; seq < total; ++seq) {
                const int st = seq & (p.nbst - 1);
                if (!mbar_wait(bf + 8 * st, (seq >> p.nbst_log2) & 1, s_abort, p.err)) break;
                mbar_arrive_cluster_relaxed(af + 8 * (seq & (kNA - 1)), 0);
            }
        }
    } else if (warp >= kWarpMma0 && warp < kWarpMma0 + 2) {
        // ------------------------------------------------------------------ MMA issuers (even CTA)
        // The whole warp runs the loop and waits (warp-uniform results); one elected lane issues.
        // From a converged warp an MMA issues in about 40 cycles with the commits hidden, against
        // about 55 plus about 80 per commit from a lone active lane.
        const int mi = warp - kWarpMma0;
        if (leader && mi < p.niss) {
            const uint64_t bdesc0 = smem_desc<128>(smem_u32(wst_base));
            const uint32_t bstep = p.b_alloc >> 4;
            const uint32_t a0 = tmem_base + p.a_col0;
            const int stages_per_unit = 27 * p.nkc;
            int seq = mi, it = 0;
            bool ok = true;
            for (int u = cid; u < nunits && ok; u += ncl, ++it) {
                const int d = p.nd == 2 ? (it & 1) : 0;
                const uint32_t dph = p.nd == 2 ? ((it >> 1) & 1) : (it & 1);
                const int dk = mi * 2 + d;
                // both CTAs' epilogues have read this accumulator
                if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(de + 8 * dk, dph ^ 1, s_abort, p.err))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t dt = tmem_base + (uint32_t)((mi * p.nd + d) * p.nb);
                const int unit_end = (it + 1) * stages_per_unit;
                uint32_t acc = 0;
                for (; seq < unit_end; seq += p.niss) {
                    const int a = seq & (kNA - 1);
                    const int st = seq & (p.nbst - 1);
                    // both CTAs' A rows and weight halves of the stage (one barrier)
                    if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(af + 8 * a, (seq >> 3) & 1, s_abort, p.err))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t at = a0 + 32u * (uint32_t)a;
                        const uint64_t bd = bdesc0 + (uint64_t)(bstep * (uint32_t)st);
                        tc_mma_ts_pair(dt, at, bd, p.idesc, acc);
                        tc_mma_ts_pair(dt, at + 8, bd + 2, p.idesc, 1u);
                        tc_mma_ts_pair(dt, at + 16, bd + 4, p.idesc, 1u);
                        tc_mma_ts_pair(dt, at + 24, bd + 6, p.idesc, 1u);
                        tc_commit_pair(ae + 8 * a, 0x3);
                        tc_commit_pair(be + 8 * st, 0x3);
                    }
                    __syncwarp();
                    acc = 1u;
                }
                if (!ok) break;
                if (elect_one()) tc_commit_pair(df + 8 * dk, 0x3);
                __syncwarp();
            }
            if (elect_one()) tc_commit_pair(drain, 0x1);
            __syncwarp();
            if (lane == 0) {
                const long long t0 = clock64();
                while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) __nanosleep(64);
            }
            __syncwarp();
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------------ epilogue (per CTA)
        const int q = warp;
        int it = 0;
        const size_t esize = p.out_kind == 0 ? 4 : 2;
        for (int u = cid; u < nunits; u += ncl, ++it) {
            const int tile = p.tile0 + 2 * (u / p.ncb) + (int)rank, cb = u % p.ncb;
            const int d = p.nd == 2 ? (it & 1) : 0;
            const uint32_t dph = p.nd == 2 ? ((it >> 1) & 1) : (it & 1);
            bool ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(df + 8 * d, dph, s_abort, p.err));
            if (ok && p.niss == 2) ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(df + 8 * (2 + d), dph, s_abort, p.err));
            if (!ok) break;
            tc_fence_after();
            const int64_t row = (int64_t)tile * kTileM + q * 32 + lane;
            const bool valid = row >= p.row_begin && row < p.row_end;
            uint8_t* orow = p.out + ((size_t)row * p.co + (size_t)cb * p.nb) * esize;
            const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
            const uint32_t d0 = lane_base + (uint32_t)(d * p.nb);
            const uint32_t d1 = lane_base + (uint32_t)((p.nd + d) * p.nb);
            for (int c0 = 0; c0 < p.nb; c0 += 16) {
                uint32_t v[16], w[16];
                TMEM_LD_X16(d0 + c0, v);
                if (p.niss == 2) {
                    TMEM_LD_X16(d1 + c0, w);
                }
                tmem_wait_ld();
                float a[16], f[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) a[j] = __uint_as_float(v[j]) + (p.niss == 2 ? __uint_as_float(w[j]) : 0.0f);
                epi16(a, p.bias ? p.bias + cb * p.nb + c0 : nullptr, p.epi, f);
                if (valid) store16(orow + (size_t)c0 * esize, f, p.out_kind);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_cluster_relaxed(de + 8 * d, 0);
                if (p.niss == 2) mbar_arrive_cluster_relaxed(de + 8 * (2 + d), 0);
            }
        }
    }

    __syncthreads();
    cluster_sync_all();                       // the peer's MMAs and reads are finished
    if (warp == kWarpMma0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(p.tmem_cols) : "memory");
    }
}

}  // namespace

#ifdef TB_TRACE
extern long long* g_trace_buffer;
#endif

bool tb_conv_brick_supported(int ci, int co) {
    return ci > 0 && ci % 64 == 0 && co > 0 && co % 16 == 0 && (co <= 256 || co % 256 == 0);
}

tb_status tb_conv_brick_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                               const void* feats, int ci, const void* weight, const float* bias, int co,
                               tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
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
    // output column blocks of kPairMinNb or more run on CTA pairs (each CTA streams half the weights)
    const bool pair = nb >= kPairMinNb;
    BrickParams p{};
    p.trace = nullptr;
#ifdef TB_TRACE
    p.trace = g_trace_buffer;
#endif
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
    p.tile0 = (int)(row0 / kTileM);
    p.row_begin = row0;
    p.row_end = row0 + nrows;
    p.ntiles = (int)((row0 + nrows + kTileM - 1) / kTileM) - p.tile0;
    p.ncb = co / nb;
    p.nkc = ci / 64;
    p.nb = nb;
    const int nb_cta = pair ? nb / 2 : nb;      // weight rows each CTA streams per stage
    p.b_bytes = (uint32_t)nb_cta * 128;
    p.b_alloc = (p.b_bytes + 1023u) & ~1023u;
    // 64 KB of weight stages; each stage is owned by weight warp (seq % 4)
    p.nbst = nb_cta <= 64 ? kMaxB : (nb_cta <= 128 ? 4 : 2);
    p.nbst_log2 = p.nbst == 8 ? 3 : (p.nbst == 4 ? 2 : 1);
    // two issuers alternate stages into two accumulators where one stage's MMAs are shorter than
    // the hand-offs around them: 64-column blocks, and 128-column blocks on CTA pairs
    p.niss = (nb <= 64 || (pair && nb <= 128)) ? 2 : 1;
    p.nd = (p.niss * 2 * nb + 32 * kNA <= 512) ? 2 : 1;
    p.a_col0 = (uint32_t)(p.niss * p.nd * nb);
    uint32_t cols = 32;
    while (cols < p.a_col0 + 32u * kNA) cols <<= 1;
    p.tmem_cols = cols;
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    // D f32, A/B format, K-major, N = nb, M = 128 (one CTA) or 256 (the pair)
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(nb >> 3) << 17) |
              ((uint32_t)((pair ? 2 : 1) * kTileM >> 4) << 24);

    const size_t fixed = 2 * (size_t)kNbrInts * 4 + 2 * sizeof(BrickMeta) + 8 * (pair ? kNumBarsPair : kNumBars) + 16 +
                         1024;
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
        const cuuint32_t box[2] = {64, (cuuint32_t)nb_cta};
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
    cudaError_t e = cudaSuccess;
    if (pair) {
        const int units = (p.ntiles + 1) / 2 * p.ncb;
        const int nclusters = std::max(1, std::min(units, ctx->num_sms / 2));
        if (smem > ctx->brick_pair_smem_set) {
            e = cudaFuncSetAttribute(k_submconv_brick_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_brick_pair)");
            ctx->brick_pair_smem_set = smem;
        }
        k_submconv_brick_pair<<<2 * nclusters, kThreads, smem, ctx->stream>>>(wmap, fmap, p);
        TB_LAUNCH_CHECK(ctx, "k_submconv_brick_pair");
        return TB_OK;
    }
    const int units = p.ntiles * p.ncb;
    const int grid = std::min(units, ctx->num_sms);
    if (smem > ctx->brick_smem_set) {
        e = cudaFuncSetAttribute(k_submconv_brick, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_brick)");
        ctx->brick_smem_set = smem;
    }
    k_submconv_brick<<<grid, kThreads, smem, ctx->stream>>>(wmap, fmap, p);
    TB_LAUNCH_CHECK(ctx, "k_submconv_brick");
    return TB_OK;
}
