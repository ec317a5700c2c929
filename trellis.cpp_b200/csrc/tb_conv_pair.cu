// Submanifold conv for Ci in {32, 64} and Co in {32, 64} on CTA pairs, with the weights resident.
//
// Same neighbor handling as the brick kernel (tb_conv_brick.cu): in the reference's x-major
// voxel order the neighbor rows of a 128-voxel tile form three contiguous row ranges, one per
// x offset (tap groups kd = 0, 1, 2 of src/sparse.cpp:30-33), loaded once per tile with TMA
// boxes, and builder warps assemble each tap's A operand in TMEM. What differs:
//
// * Two CTAs on neighbouring SMs form a cluster and share each MMA: the even CTA issues
//   tcgen05.mma.cta_group::2 with M = 256 (128 rows of its own tile + 128 rows of the odd CTA's
//   tile). Each CTA holds N/2 output columns of the weights, so the 27 tap slices of
//   W[Co][27][64] fit in shared memory for the whole kernel (27 x 32 x 128 B = 108 KB at
//   Co = 64) and no weight bytes move per tile. Streaming weights per tap was the limit of
//   the single-CTA kernel.
// * Row ranges go into a ring of shared-memory rows. Ranges are consumed in order
//   (tile, group 0, 1, 2), so a range is released as soon as its nine taps are built and the
//   loader can prefetch the next ranges into the freed rows; no fixed per-tile brick capacity.
// * Two issuer threads in the even CTA alternate stages into two accumulators (one thread
//   sustains about one MMA per 64 cycles, twice the math time of a 128x64x16 step per SM).
//
// Warps per CTA: 0-3 epilogue, 4-11 builders (two groups, alternate stages), 12 loader,
// 13-14 MMA issuers (even CTA only). Cross-CTA hand-offs: the odd CTA's builders and epilogue
// arrive on the even CTA's barriers (mapa + release.cluster); MMA commits multicast to both.
// Every wait is bounded (about 2 s) and aborts the CTA cleanly.
//
// Ci is a template parameter: a voxel row is 2 Ci bytes (128 B with the 128-byte TMA swizzle at
// Ci = 64, 64 B with the 64-byte swizzle at Ci = 32), a tap of A takes Ci / 2 TMEM columns, and
// at Ci = 32 twice as many two-tap units fit in the same TMEM columns, so the A pipeline is twice
// as deep. Ci = 32 is the bandwidth-bound regime (BASELINE config 5 at C = 32).
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>
#include <climits>

namespace {

using namespace tbtc;

constexpr int kTileM = 128;
constexpr int kNBuild = 8;           // builder warps: 4 lane quarters x 2 issuers
constexpr int kWarpBuild0 = 4;       // builders: warps 4-11
constexpr int kWarpLoader = kWarpBuild0 + kNBuild;
constexpr int kWarpMma0 = kWarpLoader + 1;   // issuers: two warps (even CTA)
constexpr int kThreads = (kWarpMma0 + 2) * 32;
constexpr int kBox = 32;             // rows per TMA box
constexpr int kNbrRow = kTileM + 4;     // one tap's indices, copied from a 16-byte aligned start
constexpr int kNbrInts = 27 * kNbrRow;
constexpr int kNB = 3;                  // neighbor-index buffers (two tiles fetched ahead)
constexpr int kNR = 8;               // range descriptor ring
constexpr uint32_t kACol0 = 128;     // first A column; issuer k accumulates in columns 64k..64k+co-1
constexpr int kPairTPU64 = 2;         // taps per A unit at Ci = 64
constexpr int kPairTPU32 = 4;         // taps per A unit at Ci = 32
constexpr int kNUMax = 6;            // A unit slots per issuer (192 TMEM columns / unit width)
// nbrf[kNB] nbre[kNB] rngf[8] rnge[8] af[2][kNU] ae[2][kNU] df[2] de[2] wbar drain (sized for kNUMax)
constexpr int kNumBars = kNB + kNB + kNR + kNR + 2 * kNUMax + 2 * kNUMax + 2 + 2 + 1 + 1;

// Per-Ci geometry: row bytes, 16-byte chunks per row, TMEM columns per tap, K steps per tap, A
// unit slots per issuer (384 A columns split over two issuers, two taps per unit).
template <int CI, int TPU>
struct PairGeom {
    static_assert(CI == 32 || CI == 64, "pair kernel: Ci 32 or 64");
    static_assert(TPU >= 2 && TPU <= 5 && TPU * (CI / 2) <= 96, "pair kernel: taps per A unit");
    static constexpr int kTPU = TPU;                   // taps per A unit (one wait, one commit)
    static constexpr int kRB = 2 * CI;
    static constexpr int kChunks = kRB / 16;
    static constexpr int kTapCols = CI / 2;
    static constexpr int kKSteps = CI / 16;
    static constexpr int kUnitCols = TPU * kTapCols;
    static constexpr int kNU = 192 / kUnitCols;
    // 16-byte chunk c of ring row b after the TMA swizzle (128 B: bits 4-6 ^= bits 7-9; 64 B:
    // bits 4-5 ^= bits 7-8 of the byte offset)
    static __device__ __forceinline__ int slot(int c, int b) { return CI == 64 ? (c ^ (b & 7)) : (c ^ ((b >> 1) & 3)); }
};

// Pipeline tracing (compiled in with -DTB_TRACE): the first cluster stamps clock64 into p.trace
// laid out as [role][kTraceCap] (clock64 is per SM, so compare stamps of one CTA only):
// 0 even loader issued range k, 1 even builder wrote A seq s, 2 MMA seq s inputs ready,
// 3 odd builder wrote A seq s, 4 even epilogue accumulator ready (it), 5 even builder got
// range k, 6 even builder's gathered rows arrived (seq s), 7 issuer accumulator free (2 * it + issuer), 8 even
// builder starts seq s, 9 even builder's A slot free for seq s, 11 first tcgen05.st issued,
// 12 tcgen05.wait::st done, 13 before the arrive, 10 even loader starts tile it's neighbor
// indices ([it]) and their arrival ([2048 + it]), 14 even loader: ranges computed [it], waits for
// the index buffer of tile it - 1 [1024 + it], got it [2048 + it]; counters at [15][0..2]: rows gathered from
// the ring, from global memory, missing (traced CTAs only).
[[maybe_unused]] constexpr int kTraceCap = 4096;
#ifdef TB_TRACE
#define TB_STAMP(role, idx)                                                                       \
    do {                                                                                          \
        if (p.trace && blockIdx.x < 2 && (idx) < kTraceCap) p.trace[(role) * kTraceCap + (idx)] = clock64(); \
    } while (0)
#define TB_COUNT(which, v)                                                                        \
    do {                                                                                          \
        if (p.trace && blockIdx.x < 2) atomicAdd(reinterpret_cast<unsigned long long*>(p.trace + 15 * kTraceCap + (which)), (unsigned long long)(v)); \
    } while (0)
#else
#define TB_STAMP(role, idx) do { } while (0)
#define TB_COUNT(which, v) do { } while (0)
#endif

struct Range {
    int32_t lo;        // first global row of the range
    int32_t len;       // rows held in the ring
    int32_t off;       // ring row where the range starts
    int32_t pad;
};

struct PairParams {
    const int32_t* nbr;
    const uint8_t* feats;
    const float* bias;
    uint8_t* out;
    int* err;
    int64_t n;
    int co;
    int out_kind, epi;
    int ntiles;
    // Pairs of tiles to compute: pair pr0 + v for v < npa, then prb0 + (v - npa) for v < nv (a
    // second, disjoint range, or none). Whole pairs are computed; only rows inside
    // [row_begin, row_end) or [row_begin_b, row_end_b) are stored.
    int pr0, npa, prb0, nv;
    int64_t row_begin, row_end, row_begin_b, row_end_b;
    int ring_rows;               // multiple of kBox
    int nbr_bulk;                // map pointer 16-byte aligned: tiles fetch indices with bulk copies
    uint32_t w_tap_bytes;        // (co/2) rows x 128 B, rounded up to 1024
    uint32_t idesc;
    long long* trace;            // TB_TRACE builds only
    long long wait_limit;        // clock cycles a bounded wait may take (about 2 s)
    int withhold;                // test hook: the even CTA's first epilogue warp withholds one arrive
};

// the pair of tiles of work item v
__device__ __forceinline__ int pair_at(const PairParams& p, int v) { return v < p.npa ? p.pr0 + v : p.prb0 + (v - p.npa); }

template <int CI, int TPU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
k_submconv_pair(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap fmap,
                const PairParams p) {
    using G = PairGeom<CI, TPU>;
    constexpr int kNU = G::kNU;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* w_base = smem;                                                   // [27][w_tap_bytes]
    uint8_t* ring = w_base + 27 * (size_t)p.w_tap_bytes;                      // [ring_rows][128]
    int32_t* s_nbr = reinterpret_cast<int32_t*>(ring + (size_t)p.ring_rows * G::kRB);   // [kNB][27][kNbrRow]
    Range* s_rng = reinterpret_cast<Range*>(s_nbr + kNB * kNbrInts);          // [kNR]
    int32_t* s_alloc = reinterpret_cast<int32_t*>(s_rng + kNR);               // [kNR] loader-private
    uint64_t* bars = reinterpret_cast<uint64_t*>(s_alloc + kNR);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kNumBars);          // [0] tmem base, [1] abort
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t bar0 = smem_u32(bars);
    const uint32_t nbrf = bar0, nbre = bar0 + 8 * kNB;
    const uint32_t rngf = bar0 + 16 * kNB, rnge = rngf + 8 * kNR;
    const uint32_t af = rnge + 8 * kNR, ae = af + 16 * kNU;  // [issuer][unit slot]
    const uint32_t df = ae + 16 * kNU, de = df + 16;          // [issuer]
    const uint32_t wbar = de + 16, drain = wbar + 8;

    if (threadIdx.x == 0) {
        for (int b = 0; b < kNB; ++b) {
            mbar_init(nbrf + 8 * b, 1);
            mbar_init(nbre + 8 * b, kNBuild);
        }
        for (int r = 0; r < kNR; ++r) {
            mbar_init(rngf + 8 * r, 1);
            mbar_init(rnge + 8 * r, kNBuild);
        }
        for (int a = 0; a < 2 * kNU; ++a) {
            mbar_init(af + 8 * a, 8);        // four builder warps in each CTA (even CTA's copy used)
            mbar_init(ae + 8 * a, 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(df + 8 * k, 1);
            mbar_init(de + 8 * k, 8);        // four epilogue warps in each CTA (even CTA's copy used)
        }
        mbar_init(wbar, 1);
        mbar_init(drain, 2);
        s_misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&fmap)) : "memory");
    }
    if (warp == kWarpMma0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;"
                     :: "r"(smem_u32(s_misc)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync_all();                       // both CTAs' barriers and TMEM exist before any cross-CTA use
    tc_fence_after();
    const uint32_t tmem_base = s_misc[0];
    const int32_t sentinel = (int32_t)p.n;
    const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();
    const int nhalf = p.co / 2;
    // tap t's indices of a tile start at word (t * n) & 3 of its kNbrRow-word row: the bulk copy
    // starts at the 16-byte boundary at or below t * n + r0 (r0 is a multiple of 128)
    const int n4 = (int)(p.n & 3);

    if (warp == kWarpLoader) {
        // ------------------------------------------------------------------ weights + loader
        if (lane == 0) mbar_arrive_expect_tx(wbar, 27u * (uint32_t)nhalf * (uint32_t)G::kRB);
        __syncwarp();
        if (lane < 27)
            tma_load_2d(smem_u32(w_base + (size_t)lane * p.w_tap_bytes), &wmap, lane * CI, (int)rank * nhalf, wbar);
        // Neighbor indices of tile j go to buffer j % kNB. Tiles whose 27 copies stay inside the
        // map (and a 16-byte aligned map) use one bulk copy per tap; the last tiles copy
        // element by element with bounds checks. Either way nbrf completes when they landed.
        auto fetch_nbr = [&](int pr_j, int buf_j) {
            const int64_t rj = (int64_t)(2 * pr_j + (int)rank) * kTileM;
            int32_t* dst = s_nbr + buf_j * kNbrInts;
            if (p.nbr_bulk && rj + kNbrRow <= p.n) {
                if (lane == 0) mbar_arrive_expect_tx(nbrf + 8 * buf_j, 27u * kNbrRow * 4u);
                __syncwarp();
                if (lane < 27) {
                    const int o = (lane * n4) & 3;
                    bulk_load(smem_u32(dst + lane * kNbrRow), p.nbr + (int64_t)lane * p.n + rj - o, kNbrRow * 4u,
                              nbrf + 8 * buf_j);
                }
            } else {
                for (int t = 0; t < 27; ++t) {
                    const int o = (t * n4) & 3;
                    const int32_t* src = p.nbr + (int64_t)t * p.n + rj;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int r = lane + 32 * q;
                        if (rj + r < p.n) cp_async_4(smem_u32(dst + t * kNbrRow + o + r), src + r);
                        else dst[t * kNbrRow + o + r] = sentinel;
                    }
                }
                cp_async_wait_all();
                __syncwarp();
                if (lane == 0) mbar_arrive(nbrf + 8 * buf_j);
            }
            __syncwarp();
        };
        // the first kNB - 1 tiles' indices
        {
            int j = 0;
            for (int vj = cid; vj < p.nv && j < kNB - 1; vj += ncl, ++j) fetch_nbr(pair_at(p, vj), j);
        }
        int it = 0, k = 0, koldest = 0, head = 0, used = 0;
        int buf = 0, ph = 0;                     // consumer side of the index buffers
        int fbuf = kNB - 1, fph = 0;             // next fetch: tile it + kNB - 1
        bool ok = true;
        for (int v = cid; v < p.nv && ok; v += ncl, ++it) {
            const int pr = pair_at(p, v);
            const int64_t r0 = (int64_t)(2 * pr + (int)rank) * kTileM;
            const int nvalid = p.n - r0 < kTileM ? (int)(p.n - r0) : kTileM;
            if (leader && lane == 0) TB_STAMP(10, it);
            if (!mbar_wait(nbrf + 8 * buf, (uint32_t)ph, s_abort, p.err, p.wait_limit)) { ok = false; break; }
            if (leader && lane == 0) TB_STAMP(10, it + 2048);
            const int32_t* rows = s_nbr + buf * kNbrInts;
            // per tap group: min and max present neighbor row over the tile's valid rows (lane
            // reads rows lane + 32q; a group's 36 loads are issued before any is used)
            int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                int32_t v[9][4];
#pragma unroll
                for (int tt = 0; tt < 9; ++tt) {
                    const int t = 9 * g + tt;
                    const int32_t* rt = rows + t * kNbrRow + ((t * n4) & 3) + lane;
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[tt][q] = rt[32 * q];
                }
#pragma unroll
                for (int tt = 0; tt < 9; ++tt) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (lane + 32 * q < nvalid && v[tt][q] != sentinel) {
                            lo[g] = min(lo[g], v[tt][q]);
                            hi[g] = max(hi[g], v[tt][q]);
                        }
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < 3; ++g) {
                lo[g] = __reduce_min_sync(0xffffffffu, lo[g]);
                hi[g] = __reduce_max_sync(0xffffffffu, hi[g]);
            }
            if (++buf == kNB) { buf = 0; ph ^= 1; }
            if (leader && lane == 0) TB_STAMP(14, it);
#pragma unroll 1
            for (int g = 0; g < 3 && ok; ++g, ++k) {
                const int glo = g == 0 ? lo[0] : (g == 1 ? lo[1] : lo[2]);
                const int ghi = g == 0 ? hi[0] : (g == 1 ? hi[1] : hi[2]);
                const int len = ghi >= 0 ? ghi - glo + 1 : 0;
                const int held = len < p.ring_rows ? len : p.ring_rows;
                const int need = (held + kBox - 1) / kBox * kBox;
                const int slot = k & (kNR - 1);
                // descriptor slot free (range k-8 built), then enough ring rows free
                if (!mbar_wait(rnge + 8 * slot, ((k >> 3) & 1) ^ 1, s_abort, p.err, p.wait_limit)) { ok = false; break; }
                // ranges at least kNR behind are built (that is what the wait above saw): reclaim
                // them without waiting, so the loop below only waits on the last kNR - 1 ranges,
                // whose barriers cannot have moved a phase further yet
                while (koldest <= k - kNR) {
                    used -= s_alloc[koldest & (kNR - 1)];
                    ++koldest;
                }
                while (used + need > p.ring_rows && ok) {
                    if (!mbar_wait(rnge + 8 * (koldest & (kNR - 1)), (koldest >> 3) & 1, s_abort, p.err, p.wait_limit)) { ok = false; break; }
                    used -= s_alloc[koldest & (kNR - 1)];
                    ++koldest;
                }
                if (!ok) break;
                const int off = head;
                head += need;
                if (head >= p.ring_rows) head -= p.ring_rows;
                used += need;
                __syncwarp();
                if (lane == 0) {
                    s_alloc[slot] = need;
                    s_rng[slot].lo = ghi >= 0 ? glo : 0;
                    s_rng[slot].len = held;
                    s_rng[slot].off = off;
                    mbar_arrive_expect_tx(rngf + 8 * slot, (uint32_t)need * (uint32_t)G::kRB);
                    if (leader) TB_STAMP(0, k);
                }
                __syncwarp();
                const int nbox = need / kBox;
                for (int j = lane; j < nbox; j += 32) {
                    int row = off + j * kBox;
                    if (row >= p.ring_rows) row -= p.ring_rows;
                    tma_load_2d(smem_u32(ring + (size_t)row * G::kRB), &fmap, 0, glo + j * kBox, rngf + 8 * slot);
                }
            }
            if (!ok) break;
            // indices of tile it + kNB - 1 into the buffer of tile it - 1, once its builders are done
            const int vf = v + (kNB - 1) * ncl;
            if (vf < p.nv) {
                if (leader && lane == 0) TB_STAMP(14, 1024 + it);
                if (!mbar_wait(nbre + 8 * fbuf, (uint32_t)(fph ^ 1), s_abort, p.err, p.wait_limit)) { ok = false; break; }
                if (leader && lane == 0) TB_STAMP(14, 2048 + it);
                fetch_nbr(pair_at(p, vf), fbuf);
                if (++fbuf == kNB) { fbuf = 0; fph ^= 1; }
            }
        }
        if (!ok && lane == 0) {
            const long long t0 = clock64();
            while (clock64() - t0 < 4000000ll) __nanosleep(256);
        }
    } else if (warp >= kWarpBuild0 && warp < kWarpBuild0 + kNBuild) {
        // ------------------------------------------------------------------ A builders
        // warp w writes TMEM lane quarter w % 4 of the units of issuer half
        const int q = warp & 3;
        const int half = (warp - kWarpBuild0) >> 2;
        const int i = q * 32 + lane;
        // this half's unit slots: columns kACol0 + kUnitCols * (kNU * half + u), kTapCols per tap
        const uint32_t a_lane = tmem_base + ((uint32_t)(q * 32) << 16) + kACol0 + (uint32_t)G::kUnitCols * kNU * (uint32_t)half;
        const uint32_t afh = af + 8 * kNU * half, aeh = ae + 8 * kNU * half;
        int u = 0, uph = 0;                 // unit slot and its phase
        // every wait's result is made warp-uniform: the TMEM stores that follow are warp-collective,
        // and a lane that timed out must not leave the others to run them alone
        bool ok = __all_sync(0xffffffffu, mbar_wait(wbar, 0, s_abort, p.err, p.wait_limit));   // weights landed
        int it = 0, k = 0, buf = 0, ph = 0;
        for (int v = cid; v < p.nv && ok; v += ncl, ++it) {
            const int pr = pair_at(p, v);
            if (!__all_sync(0xffffffffu, mbar_wait(nbrf + 8 * buf, (uint32_t)ph, s_abort, p.err, p.wait_limit))) {
                ok = false;
                break;
            }
            const int32_t* rows = s_nbr + buf * kNbrInts;
            const int64_t r0 = (int64_t)(2 * pr + (int)rank) * kTileM;
            const bool row_valid = r0 + i < p.n;     // rows past the map end are never stored
            const int seq0 = 27 * it;
#pragma unroll 1
            for (int g = 0; g < 3 && ok; ++g, ++k) {
                const int slot = k & (kNR - 1);
                if (!__all_sync(0xffffffffu, mbar_wait(rngf + 8 * slot, (k >> 3) & 1, s_abort, p.err, p.wait_limit))) {
                    ok = false;
                    break;
                }
                if (leader && half == 0 && q == 0 && lane == 0) TB_STAMP(5, k);
                const int rlo = s_rng[slot].lo, rlen = s_rng[slot].len, roff = s_rng[slot].off;
                // this group's taps with stage parity == half (t0, t0 + 2, ..., t0 + 8, those inside
                // the group), TPU of them per unit. The lane's neighbor rows of all of them are read
                // first, so each unit's row loads wait on one load latency only.
                const int t0 = 9 * g + ((half ^ (seq0 + 9 * g)) & 1);
                const int tend = 9 * g + 9;
                int32_t vrow[5];
#pragma unroll
                for (int e = 0; e < 5; ++e) {
                    const int tt = t0 + 2 * e;
                    vrow[e] = (tt < tend && row_valid) ? rows[tt * kNbrRow + ((tt * n4) & 3) + i] : sentinel;
                }
#pragma unroll
                for (int j = 0; j < (5 + TPU - 1) / TPU; ++j) {
                    const int t = t0 + 2 * TPU * j;
                    if (t >= tend || !ok) break;
                    const bool tr0 = leader && half == 0 && q == 0 && lane == 0;
                    if (tr0) TB_STAMP(8, seq0 + t);
                    // the unit's rows of A in registers before the slot wait: ring row, missing
                    // (zero) or, for a row outside the held range, global memory
                    uint32_t rv[TPU][G::kTapCols];
#pragma unroll
                    for (int e = 0; e < TPU; ++e) {
                        if (TPU * j + e >= 5 || t + 2 * e >= tend) break;
                        const int32_t v = vrow[TPU * j + e];
                        if (v == sentinel) {
#pragma unroll
                            for (int c = 0; c < G::kTapCols; ++c) rv[e][c] = 0u;
                        } else if ((uint32_t)(v - rlo) < (uint32_t)rlen) {
                            int b = roff + (v - rlo);
                            if (b >= p.ring_rows) b -= p.ring_rows;
                            const uint8_t* rowp = ring + (size_t)b * G::kRB;
#pragma unroll
                            for (int c = 0; c < G::kChunks; ++c) {
                                const uint4 x = *reinterpret_cast<const uint4*>(rowp + (G::slot(c, b) << 4));
                                rv[e][4 * c] = x.x; rv[e][4 * c + 1] = x.y; rv[e][4 * c + 2] = x.z; rv[e][4 * c + 3] = x.w;
                            }
                        } else {
                            const uint4* gp = reinterpret_cast<const uint4*>(p.feats + (size_t)v * G::kRB);
#pragma unroll
                            for (int c = 0; c < G::kChunks; ++c) {
                                const uint4 x = __ldg(gp + c);
                                rv[e][4 * c] = x.x; rv[e][4 * c + 1] = x.y; rv[e][4 * c + 2] = x.z; rv[e][4 * c + 3] = x.w;
                            }
                        }
                    }
#ifdef TB_TRACE
                    if (p.trace) {
                        int nring = 0, nglob = 0, nmiss = 0;
#pragma unroll
                        for (int e = 0; e < TPU; ++e) {
                            if (TPU * j + e >= 5 || t + 2 * e >= tend) break;
                            const int tv = t + 2 * e;
                            const int32_t v = row_valid ? rows[tv * kNbrRow + ((tv * n4) & 3) + i] : sentinel;
                            const unsigned m1 = __ballot_sync(0xffffffffu, v == sentinel);
                            const unsigned m2 = __ballot_sync(0xffffffffu, v != sentinel && (uint32_t)(v - rlo) < (uint32_t)rlen);
                            nmiss += __popc(m1); nring += __popc(m2); nglob += 32 - __popc(m1) - __popc(m2);
                        }
                        if (lane == 0) { TB_COUNT(0, nring); TB_COUNT(1, nglob); TB_COUNT(2, nmiss); }
                    }
                    if (tr0) {
                        asm volatile("" :: "r"(rv[0][G::kTapCols - 1]));   // rows arrived
                        TB_STAMP(6, seq0 + t);
                    }
#endif
                    // the unit slot's previous taps have been multiplied
                    if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(aeh + 8 * u, (uint32_t)(uph ^ 1), s_abort, p.err,
                                                                           p.wait_limit))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (tr0) TB_STAMP(9, seq0 + t);
                    const uint32_t ua = a_lane + (uint32_t)G::kUnitCols * (uint32_t)u;
#pragma unroll
                    for (int e = 0; e < TPU; ++e) {
                        if (TPU * j + e >= 5 || t + 2 * e >= tend) break;
                        if constexpr (CI == 64) tmem_st_x32(ua + (uint32_t)(e * G::kTapCols), rv[e]);
                        else tmem_st_x16(ua + (uint32_t)(e * G::kTapCols), rv[e]);
                        if (tr0 && e == 0) TB_STAMP(11, seq0 + t);
                    }
                    tmem_wait_st();
                    if (tr0) TB_STAMP(12, seq0 + t);
                    tc_fence_before();
                    __syncwarp();
                    if (tr0) TB_STAMP(13, seq0 + t);
                    if (lane == 0) {
                        mbar_arrive_cluster_relaxed(afh + 8 * u, 0);
                        if (q == 0) {
#pragma unroll
                            for (int e = 0; e < TPU; ++e)
                                if (t + 2 * e < tend) TB_STAMP(leader ? 1 : 3, seq0 + t + 2 * e);
                        }
                    }
                    if (++u == kNU) { u = 0; uph ^= 1; }
                }
                // The range's ring rows go back to the loader, whose TMA may refill them next. No
                // proxy fence: every load from them has returned its value (the tcgen05.wait::st
                // above waited for the stores of that data), so a later async-proxy write cannot
                // reach a read still in flight. (A fence here cost 3% of the conv.)
                __syncwarp();
                if (lane == 0) mbar_arrive(rnge + 8 * slot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(nbre + 8 * buf);
            if (++buf == kNB) { buf = 0; ph ^= 1; }
        }
    } else if (warp >= kWarpMma0 && warp < kWarpMma0 + 2) {
        // ------------------------------------------------------------------ MMA issuers (even CTA)
        // The whole warp runs the loop and waits; one elected lane issues. Issuing from a
        // converged warp costs about 40 cycles per MMA with the commit hidden, against about 55
        // per MMA plus about 80 per commit from a lone active lane.
        const int mi = warp - kWarpMma0;
        if (leader) {
            const uint64_t wdesc0 = smem_desc<G::kRB>(smem_u32(w_base));
            const uint32_t wstep = p.w_tap_bytes >> 4;
            // issuer mi takes the taps whose sequence number (27 * tile + tap) has parity mi, in
            // the units its builder half writes them: per tap group, taps t0, t0 + 2, ..., t0 + 8
            // (those inside the group), TPU per unit; one wait and one commit per unit
            int it = 0, u = 0, uph = 0;
            bool ok = true;
            const uint32_t dt = tmem_base + 64u * (uint32_t)mi;
            const uint32_t a_base = tmem_base + kACol0 + (uint32_t)G::kUnitCols * kNU * (uint32_t)mi;
            const uint32_t afh = af + 8 * kNU * mi, aeh = ae + 8 * kNU * mi;
            for (int v = cid; v < p.nv && ok; v += ncl, ++it) {
            const int pr = pair_at(p, v);
                // the epilogue has read this issuer's accumulator for the previous tile
                ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(de + 8 * mi, (uint32_t)((it & 1) ^ 1), s_abort, p.err, p.wait_limit));
                if (!ok) break;
                if (lane == 0) TB_STAMP(7, 2 * it + mi);
                const int seq0 = 27 * it;
                uint32_t acc = 0;
                for (int g = 0; g < 3 && ok; ++g) {
                    for (int t = 9 * g + ((mi ^ (seq0 + 9 * g)) & 1); t < 9 * g + 9; t += 2 * TPU) {
                        ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(afh + 8 * u, (uint32_t)uph, s_abort, p.err, p.wait_limit));
                        if (!ok) break;
                        if (lane == 0) TB_STAMP(2, seq0 + t);
                        tc_fence_after();
                        if (elect_one()) {
                            // K = 16 per MMA: 8 TMEM columns of A, 32 bytes (2 descriptor units) of B;
                            // the unit's taps t, t + 2, ... sit kTapCols columns apart
                            const uint32_t at = a_base + (uint32_t)G::kUnitCols * (uint32_t)u;
                            const uint64_t bd = wdesc0 + (uint64_t)(wstep * (uint32_t)t);
#pragma unroll
                            for (int e = 0; e < TPU; ++e) {
                                if (t + 2 * e >= 9 * g + 9) break;
#pragma unroll
                                for (int ks = 0; ks < G::kKSteps; ++ks)
                                    tc_mma_ts_pair(dt, at + (uint32_t)(e * G::kTapCols) + 8u * ks,
                                                   bd + (uint64_t)(2u * (uint32_t)e * wstep) + 2u * ks, p.idesc,
                                                   (e == 0 && ks == 0) ? acc : 1u);
                            }
                            tc_commit_pair(aeh + 8 * u, 0x3);
                        }
                        __syncwarp();
                        acc = 1u;
                        if (++u == kNU) { u = 0; uph ^= 1; }
                    }
                }
                if (!ok) break;
                if (elect_one()) tc_commit_pair(df + 8 * mi, 0x3);
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
        // ------------------------------------------------------------------ epilogue
        const int q = warp;
        int it = 0;
        const size_t esize = p.out_kind == 0 ? 4 : 2;
        for (int v = cid; v < p.nv; v += ncl, ++it) {
            const int pr = pair_at(p, v);
            const uint32_t dph = (uint32_t)(it & 1);
            bool ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(df, dph, s_abort, p.err, p.wait_limit));
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait_cluster_relaxed(df + 8, dph, s_abort, p.err, p.wait_limit));
            if (!ok) break;
            if (leader && q == 0 && lane == 0) TB_STAMP(4, it);
            tc_fence_after();
            // sum the two issuers' accumulators into registers, then hand the TMEM back before
            // the bias, activation and stores
            const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
            float accv[64];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if (16 * c < p.co) {
                    uint32_t v[16], w[16];
                    TMEM_LD_X16(lane_base + 16u * c, v);
                    TMEM_LD_X16(lane_base + 64u + 16u * c, w);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) accv[16 * c + j] = __uint_as_float(v[j]) + __uint_as_float(w[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            // (the test hook leaves the first tile's accumulator-free barrier one arrive short, so
            // the issuers' next waits run out and every role leaves through the abort path)
            if (lane == 0 && !(p.withhold && it == 0 && leader && q == 0)) {
                mbar_arrive_cluster_relaxed(de, 0);
                mbar_arrive_cluster_relaxed(de + 8, 0);
            }
            const int64_t row = (int64_t)(2 * pr + (int)rank) * kTileM + q * 32 + lane;
            if ((row >= p.row_begin && row < p.row_end) || (row >= p.row_begin_b && row < p.row_end_b)) {
                uint8_t* orow = p.out + (size_t)row * p.co * esize;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (16 * c < p.co) {
                        epi16(accv + 16 * c, p.bias ? p.bias + 16 * c : nullptr, p.epi, accv + 16 * c);
                        store16(orow + (size_t)(16 * c) * esize, accv + 16 * c, p.out_kind);
                    }
                }
            }
        }
    }

    __syncthreads();
    cluster_sync_all();                       // the peer's MMAs and reads are finished
    if (warp == kWarpMma0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" :: "r"(tmem_base) : "memory");
    }
}

}  // namespace

#ifdef TB_TRACE
extern long long* g_trace_buffer;
#endif

// Test hook (not declared in the public header): make the next pair-kernel launches withhold one
// epilogue arrive and give up waiting after `limit_cycles` (about 1 ms at 2e6), so a test can
// run the bounded-wait abort path without hanging anything; on = 0 restores the defaults.
static long long g_pair_wait_limit = kWaitCycles;
static int g_pair_withhold = 0;
extern "C" void tb_debug_pair_withhold_arrive(int on, long long limit_cycles) {
    g_pair_withhold = on ? 1 : 0;
    g_pair_wait_limit = on && limit_cycles > 0 ? limit_cycles : kWaitCycles;
}

bool tb_conv_pair_supported(int ci, int co) { return (ci == 64 || ci == 32) && (co == 64 || co == 32); }

tb_status tb_conv_pair_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                              const void* feats, int ci, const void* weight, const float* bias, int co,
                              tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
    return tb_conv_pair_launch2(ctx, nbr, n, row0, nrows, 0, 0, feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
}

tb_status tb_conv_pair_launch2(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows, int64_t row0b,
                               int64_t nrowsb, const void* feats, int ci, const void* weight, const float* bias, int co,
                               tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
    if (!tb_conv_pair_supported(ci, co))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "pair conv needs ci and co in {32, 64}");
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    PairParams p{};
    p.trace = nullptr;
#ifdef TB_TRACE
    p.trace = g_trace_buffer;
#endif
    p.wait_limit = g_pair_wait_limit;
    p.withhold = g_pair_withhold;
    p.nbr = nbr;
    p.feats = reinterpret_cast<const uint8_t*>(feats);
    p.bias = bias;
    p.out = reinterpret_cast<uint8_t*>(out);
    p.err = ctx->d_err;
    p.n = n;
    p.co = co;
    p.out_kind = out_dtype == TB_F32 ? 0 : (out_dtype == TB_F16 ? 1 : 2);
    p.epi = epi;
    p.ntiles = (int)((n + kTileM - 1) / kTileM);
    // output rows [row0, row0 + nrows) (and [row0b, row0b + nrowsb)): whole pairs of tiles from the
    // one holding the first row; two ranges whose pairs meet become one run of pairs
    auto pairs_of = [](int64_t r0, int64_t nr, int& a, int& b) {
        a = (int)(r0 / (2 * kTileM));
        b = (int)((r0 + nr + 2 * kTileM - 1) / (2 * kTileM));
    };
    int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
    pairs_of(row0, nrows, a0, a1);
    if (nrows <= 0) a1 = a0;
    if (nrowsb > 0) pairs_of(row0b, nrowsb, b0, b1);
    if (nrowsb > 0 && b0 < a0) { std::swap(a0, b0); std::swap(a1, b1); }
    if (nrowsb > 0 && b0 <= a1) { a1 = std::max(a1, b1); b0 = b1 = 0; }
    p.pr0 = a0;
    p.npa = a1 - a0;
    p.prb0 = b0;
    p.nv = p.npa + (b1 - b0);
    p.row_begin = row0;
    p.row_end = row0 + std::max<int64_t>(nrows, 0);
    p.row_begin_b = nrowsb > 0 ? row0b : 0;
    p.row_end_b = nrowsb > 0 ? row0b + nrowsb : 0;
    const int nhalf = co / 2;
    const uint32_t rb = 2u * (uint32_t)ci;      // bytes per voxel row
    p.w_tap_bytes = ((uint32_t)nhalf * rb + 1023u) & ~1023u;
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    // D f32, A/B format, K-major, N = co, M = 256 (the pair)
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(co >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

    p.nbr_bulk = (reinterpret_cast<uintptr_t>(nbr) & 15) == 0;
    const size_t fixed = 27 * (size_t)p.w_tap_bytes + kNB * (size_t)kNbrInts * 4 + kNR * sizeof(Range) + kNR * 4 +
                         8 * kNumBars + 16 + 1024;
    const size_t budget = (size_t)ctx->max_smem_optin;
    if (budget < fixed + 256 * (size_t)rb) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "pair conv: shared memory too small");
    int ring = (int)((budget - fixed) / rb);
    ring = ring / kBox * kBox;
    p.ring_rows = ring;
    const size_t smem = fixed + (size_t)ring * rb;

    CUtensorMap wmap, fmap;
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUtensorMapSwizzle swz = ci == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)27 * ci, (cuuint64_t)co};
        const cuuint64_t gstride[1] = {(cuuint64_t)27 * ci * 2};
        const cuuint32_t box[2] = {(cuuint32_t)ci, (cuuint32_t)nhalf};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &wmap, dt, 2, const_cast<void*>(weight), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the weight view");
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)ci, (cuuint64_t)n};
        const cuuint64_t gstride[1] = {(cuuint64_t)ci * 2};
        const cuuint32_t box[2] = {(cuuint32_t)ci, (cuuint32_t)kBox};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &fmap, dt, 2, const_cast<void*>(feats), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the feature view");
    }
    if (p.nv <= 0) return TB_OK;
    const int nclusters = std::max(1, std::min(p.nv, ctx->num_sms / 2));
    cudaError_t e = cudaSuccess;
    // taps per A unit: at Ci = 32 a tap is half as wide, and four-tap units halve the per-unit
    // hand-offs (waits, fences, commits) that bound the kernel at that width
    auto kern = ci == 64 ? k_submconv_pair<64, kPairTPU64> : k_submconv_pair<32, kPairTPU32>;
    size_t& smem_set = ctx->pair_smem_set[ci == 64 ? 0 : 1];
    if (smem > smem_set) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_submconv_pair)");
        smem_set = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * nclusters);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    e = cudaLaunchKernelEx(&cfg, kern, wmap, fmap, p);
    if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaLaunchKernelEx(k_submconv_pair)");
    TB_LAUNCH_CHECK(ctx, "k_submconv_pair");
    return TB_OK;
}
