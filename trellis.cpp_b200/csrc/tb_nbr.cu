// Coordinate hash table and 27-tap neighbor map on the GPU.
//
// Replaces trellis::build_neighbor_table (src/sparse.cpp:21-39), which inserts every voxel
// into a std::unordered_map keyed by the packed coordinate (src/sparse.cpp:25-26, a later
// duplicate overwrites) and then does 27 lookups per voxel into a tap-major [27*N] table
// whose absent entries hold N.
//
// Sorted layout (rows already in ascending (batch, x, y, z) order, as every caller in this
// library and the reference's generators give them): a dense table of the row range of each
// (batch, x, y) column of the bounding box, and per voxel a search of its 9 neighbouring columns
// for z - 1, z, z + 1. Built with plain stores; no hashing. Details at the kernels below.
//
// Block layout (any row order): voxels are grouped in 4x4x4 coordinate blocks. A hash table maps
// each block to a 64-entry bucket of rows indexed by the voxel's position in the block, so a
// voxel's 27 lookups need at most 8 block probes (mostly its own block) and read buckets that
// neighbouring voxels read too; in the usual x-major voxel order the table and buckets stay in
// L1/L2 instead of every probe going to DRAM. It applies when every coordinate is in
// [0, 2^20 - 2] and every batch index in [0, 15]: there the reference's packed key (20 bits per
// coordinate, batch in the top 4 bits) is injective, and the keys of the out-of-grid neighbours
// (a coordinate of -1) cannot equal a voxel's key, so "same key" is "same coordinates" and
// absent neighbours stay absent. The block table has twice as many slots as there are buckets,
// min(N/4 + 64, 2^25 - 64). Otherwise, or when there are more blocks than buckets (very sparse
// voxels) or a block insert probes 64 slots without a place, a device flag routes the build to
// the voxel hash below, which clears and uses its own full-size table; no host round trip.
//
// Voxel hash (fallback, and the allocation-free entry point): open addressing with linear
// probing over 16-byte slots {key, row}. The
// capacity is the next power of two >= 2N (load factor <= 1/2), so one 16-byte load per
// probe. Insert: atomicCAS claims the slot for the key, then atomicMax on the row makes the
// largest row index win, which is exactly "last writer wins" of the sequential reference.
// The all-ones key is reachable (coords (-1,-1,-1)) and is the empty marker, so that one
// key lives in a separate cell. Lookups run one thread per voxel, 27 probes each, and write
// nbr[t*N + i] coalesced across the warp for every tap.
#include "tb_common.cuh"

#include <algorithm>
#include <climits>
#include <mutex>

namespace {

constexpr unsigned long long kEmpty = ~0ull;

struct __align__(16) Slot {
    unsigned long long key;
    int row;
    int pad;
};

__device__ __forceinline__ uint64_t key_of(const int32_t* c, int stride, int dx, int dy, int dz) {
    if (stride == 4)
        return tb_key3(c[1] + dx, c[2] + dy, c[3] + dz) ^ ((uint64_t)(uint32_t)c[0] << 60);
    return tb_key3(c[0] + dx, c[1] + dy, c[2] + dz);
}

// Grid-stride bodies of the voxel hash's three steps; kernels of their own for the
// allocation-free entry point, and the fallback branch of the layout kernels below.
__device__ __forceinline__ void hash_clear_body(Slot* __restrict__ t, uint64_t cap, int* __restrict__ special) {
    uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (; i < cap; i += stride) {
        ulonglong2 v; v.x = kEmpty; v.y = 0xFFFFFFFFull;   // row = -1
        reinterpret_cast<ulonglong2*>(t)[i] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *special = -1;
}

__global__ void k_hash_clear(Slot* __restrict__ t, uint64_t cap, int* __restrict__ special) {
    hash_clear_body(t, cap, special);
}

__device__ __forceinline__ void hash_insert_body(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                 Slot* __restrict__ t, uint64_t mask, int* __restrict__ special,
                                                 int* __restrict__ err) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t k = key_of(coords + i * stride, stride, 0, 0, 0);
        if (k == kEmpty) { atomicMax(special, (int)i); continue; }
        uint64_t h = tb_mix64(k) & mask;
        bool done = false;
        for (uint64_t probe = 0; probe <= mask; ++probe) {
            const unsigned long long prev = atomicCAS(&t[h].key, kEmpty, (unsigned long long)k);
            if (prev == kEmpty || prev == k) { atomicMax(&t[h].row, (int)i); done = true; break; }
            h = (h + 1) & mask;
        }
        if (!done && err) atomicCAS(err, 0, TB_DEVERR_HASH_PROBE);
    }
}

__global__ void k_hash_insert(const int32_t* __restrict__ coords, int64_t n, int stride, Slot* __restrict__ t,
                              uint64_t mask, int* __restrict__ special, int* __restrict__ err) {
    hash_insert_body(coords, n, stride, t, mask, special, err);
}

__device__ __forceinline__ int lookup(const Slot* __restrict__ t, uint64_t mask, int special,
                                      uint64_t k, int absent, int* __restrict__ err) {
    if (k == kEmpty) return special >= 0 ? special : absent;
    uint64_t h = tb_mix64(k) & mask;
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        const ulonglong2 s = __ldg(reinterpret_cast<const ulonglong2*>(t) + h);
        if (s.x == k) return (int)(uint32_t)s.y;
        if (s.x == kEmpty) return absent;
        h = (h + 1) & mask;
    }
    if (err) atomicCAS(err, 0, TB_DEVERR_HASH_PROBE);
    return absent;
}

// The taps a lookup writes: all 27 (NT = 27, out[tap * N + i]) or the seven quad-corner taps of
// the dual-grid mesh (NT = 7, out[j * N + i] for tap tb_quad_tap(j)). Both lists are known at
// compile time, so the per-tap index arithmetic folds into constants.
template <int NT>
__device__ __forceinline__ constexpr int tap_at(int j) {
    static_assert(NT == 27 || NT == 7, "tap set");
    if constexpr (NT == 27) return j;
    else return tb_quad_tap(j);
}

template <int NT>
__device__ __forceinline__ void nbr_lookup_body(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                const Slot* __restrict__ t, uint64_t mask,
                                                const int* __restrict__ special_p, int32_t* __restrict__ nbr,
                                                int* __restrict__ err) {
    const int special = *special_p;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int32_t c[4];
        for (int d = 0; d < stride; ++d) c[d] = coords[i * stride + d];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int tap = tap_at<NT>(j);
            const int kd = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
            const uint64_t k = key_of(c, stride, kd - 1, kh - 1, kw - 1);
            nbr[(int64_t)j * n + i] = lookup(t, mask, special, k, (int)n, err);
        }
    }
}

template <int NT>
__global__ void k_nbr_lookup(const int32_t* __restrict__ coords, int64_t n, int stride, const Slot* __restrict__ t,
                             uint64_t mask, const int* __restrict__ special_p, int32_t* __restrict__ nbr,
                             int* __restrict__ err) {
    nbr_lookup_body<NT>(coords, n, stride, t, mask, special_p, nbr, err);
}

// ---- block layout ---------------------------------------------------------------------------
constexpr int32_t kMaxCoord = (1 << 20) - 2;

struct BlockCtl {
    unsigned int nblocks;   // buckets handed out
    int fallback;           // 1: build with the voxel hash instead
    int unsorted;           // 1: rows out of (batch, x, y, z) order, or a coordinate outside the block range
    int sorted;             // 1: the sorted layout builds the map (decided by k_srt_clear)
    int block_on;           // 1 - sorted: the gate of the block table's clear
    int lo_inv[3];          // kMaxCoord - minimum of batch, x, y (atomicMax from zero)
    int hi[3];              // maximum of batch, x, y
    int pad;
};
static_assert(sizeof(BlockCtl) % 16 == 0, "the bucket pool after BlockCtl takes 16-byte stores");

__device__ __forceinline__ uint64_t block_key(int32_t b, int32_t bx, int32_t by, int32_t bz) {
    return tb_key3(bx, by, bz) ^ ((uint64_t)(uint32_t)b << 60);
}

// Slot index of a block: the coordinates, each below 2^18, mixed in 32-bit arithmetic (the
// comparison is on the full 64-bit key, so the mix only spreads the blocks over the table).
__device__ __forceinline__ uint64_t block_slot(int32_t b, int32_t bx, int32_t by, int32_t bz, uint64_t mask) {
    uint32_t h = (uint32_t)bx * 0x9E3779B1u ^ (uint32_t)by * 0x85EBCA77u ^ (uint32_t)bz * 0xC2B2AE3Du ^
                 (uint32_t)b * 0x27D4EB2Fu;
    h ^= h >> 15;
    h *= 0x2C1B3C6Du;
    h ^= h >> 13;
    return (uint64_t)h & mask;
}

// Bucket of the block (b, bx, by, bz), or -1 when the block holds no voxel.
__device__ __forceinline__ ulonglong2 slot_at(const Slot* __restrict__ t, uint64_t h) {
    return __ldg(reinterpret_cast<const ulonglong2*>(t) + h);
}

// Bucket of key k given its home slot h and that slot's contents s (loaded by the caller, so
// that several first probes can be in flight together), or -1 when the block holds no voxel.
__device__ __forceinline__ int block_resolve(const Slot* __restrict__ t, uint64_t mask, uint64_t k, uint64_t h,
                                             ulonglong2 s) {
    for (uint64_t probe = 0; probe <= mask; ++probe) {
        if (s.x == k) return (int)(uint32_t)s.y;
        if (s.x == kEmpty) return -1;
        h = (h + 1) & mask;
        s = slot_at(t, h);
    }
    return -1;
}

__device__ __forceinline__ void read_coords(const int32_t* c, int stride, int32_t& b, int32_t& x, int32_t& y, int32_t& z) {
    if (stride == 4) { b = c[0]; x = c[1]; y = c[2]; z = c[3]; }
    else { b = 0; x = c[0]; y = c[1]; z = c[2]; }
}

constexpr int kInsPer = 4;      // voxels per thread in the insert kernels
constexpr int kTpb = 256;       // threads per block of every map kernel

// Coordinates of row i: one 16-byte load when the rows are [b, x, y, z] and 16-byte aligned.
__device__ __forceinline__ void load_row(const int32_t* __restrict__ coords, int64_t i, int stride, bool vec,
                                         int32_t& b, int32_t& x, int32_t& y, int32_t& z) {
    if (vec) {
        const int4 v = __ldg(reinterpret_cast<const int4*>(coords) + i);
        b = v.x; x = v.y; y = v.z; z = v.w;
    } else {
        read_coords(coords + i * stride, stride, b, x, y, z);
    }
}

// Claims each voxel's block and hands the block a bucket; flags coordinates outside the range
// where block lookup equals the reference's key lookup, and bucket overflow. A warp takes
// 32 * kInsPer consecutive voxels (group j = voxels j*32 .. j*32+31 of its range) and issues the
// first claim attempt of every group before it waits on any: the work is bound by the latency
// of these dependent round trips, not by bandwidth.
__device__ __forceinline__ void blk_insert_body(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                Slot* __restrict__ t, uint64_t mask, BlockCtl* __restrict__ ctl,
                                                unsigned int pool_blocks) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) * kInsPer;
    uint64_t k[kInsPer], h[kInsPer];
    bool lead[kInsPer];
#pragma unroll
    for (int j = 0; j < kInsPer; ++j) {
        const int64_t i = warp0 + j * 32 + lane;
        int32_t b = 0, x = 0, y = 0, z = 0;
        bool valid = i < n;
        if (valid) {
            read_coords(coords + i * stride, stride, b, x, y, z);
            if ((uint32_t)x > (uint32_t)kMaxCoord || (uint32_t)y > (uint32_t)kMaxCoord ||
                (uint32_t)z > (uint32_t)kMaxCoord || (uint32_t)b > 15u) {
                ctl->fallback = 1;
                valid = false;
            }
        }
        // consecutive voxels mostly share a block: one lane per distinct block of the group claims it
        k[j] = valid ? block_key(b, x >> 2, y >> 2, z >> 2) : (kEmpty - (uint64_t)lane);
        const unsigned same = __match_any_sync(0xffffffffu, k[j]);
        lead[j] = valid && (same & ((1u << lane) - 1u)) == 0;
        h[j] = valid ? block_slot(b, x >> 2, y >> 2, z >> 2, mask) : 0;
    }
    unsigned long long prev[kInsPer];
#pragma unroll
    for (int j = 0; j < kInsPer; ++j)
        prev[j] = lead[j] ? atomicCAS(&t[h[j]].key, kEmpty, (unsigned long long)k[j]) : 0ull;
    bool claimed[kInsPer];
#pragma unroll
    for (int j = 0; j < kInsPer; ++j) {
        claimed[j] = false;
        if (!lead[j]) continue;
        // the table holds twice the buckets; a probe run this long means far more blocks than
        // buckets (the table filling up), so the voxel hash builds the map
        int probe = 0;
        for (; probe < 64; ++probe) {
            if (prev[j] == kEmpty) {
                claimed[j] = true;
                break;
            }
            if (prev[j] == k[j]) break;
            h[j] = (h[j] + 1) & mask;
            if (probe + 1 < 64) prev[j] = atomicCAS(&t[h[j]].key, kEmpty, (unsigned long long)k[j]);
        }
        if (probe == 64) ctl->fallback = 1;
    }
    // bucket ids for the blocks this warp claimed: one counter update per warp
    unsigned cm[kInsPer];
    unsigned total = 0;
#pragma unroll
    for (int j = 0; j < kInsPer; ++j) {
        cm[j] = __ballot_sync(0xffffffffu, claimed[j]);
        total += (unsigned)__popc(cm[j]);
    }
    if (total == 0) return;
    unsigned int base = 0;
    if (lane == 0) base = atomicAdd(&ctl->nblocks, total);
    base = __shfl_sync(0xffffffffu, base, 0);
#pragma unroll
    for (int j = 0; j < kInsPer; ++j) {
        if (claimed[j]) {
            const unsigned int id = base + (unsigned int)__popc(cm[j] & ((1u << lane) - 1u));
            if (id >= pool_blocks) ctl->fallback = 1;
            t[h[j]].row = (int)id;
        }
        base += (unsigned)__popc(cm[j]);
    }
}

// The largest row index of each coordinate wins, as the reference's later insert overwrites.
// Grid-stride over chunks of kTpb * kInsPer voxels: four voxels per thread (kTpb apart, so each
// load of a warp is coalesced) whose first table probes are in flight together.
__device__ __forceinline__ void vox_insert_body(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                const Slot* __restrict__ t, uint64_t mask, int32_t* __restrict__ pool) {
    const int64_t nchunks = (n + (int64_t)kTpb * kInsPer - 1) / ((int64_t)kTpb * kInsPer);
    for (int64_t ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
        const int64_t i0 = ch * kTpb * kInsPer + threadIdx.x;
        uint64_t k[kInsPer], h[kInsPer];
        int loc[kInsPer];
        ulonglong2 s[kInsPer];
#pragma unroll
        for (int j = 0; j < kInsPer; ++j) {
            const int64_t i = i0 + (int64_t)j * kTpb;
            if (i < n) {
                int32_t b, x, y, z;
                read_coords(coords + i * stride, stride, b, x, y, z);
                k[j] = block_key(b, x >> 2, y >> 2, z >> 2);
                h[j] = block_slot(b, x >> 2, y >> 2, z >> 2, mask);
                loc[j] = ((x & 3) << 4) | ((y & 3) << 2) | (z & 3);
                s[j] = slot_at(t, h[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < kInsPer; ++j) {
            const int64_t i = i0 + (int64_t)j * kTpb;
            if (i >= n) break;
            const int bucket = block_resolve(t, mask, k[j], h[j], s[j]);
            if (bucket < 0) continue;                                    // cannot happen after the block claims
            atomicMax(&pool[(int64_t)bucket * 64 + loc[j]], (int32_t)i);
        }
    }
}

// 27 lookups per voxel (grid-stride). Per axis the taps reach at most one block besides the
// voxel's own (the one below at position 0, above at position 3), so the up to 8 blocks are
// looked up once. Their bucket bases go to shared memory (a column per thread, so reads never
// conflict), and each tap reads the one its three "leaves the block" bits select instead of a
// select tree over eight registers.
template <int NT>
__device__ __forceinline__ void blk_lookup_body(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                const Slot* __restrict__ t, uint64_t mask,
                                                const int32_t* __restrict__ pool, int32_t* __restrict__ nbr,
                                                int (*s_base)[kTpb]) {
    for (int64_t i = blockIdx.x * (int64_t)kTpb + threadIdx.x; i < n; i += (int64_t)gridDim.x * kTpb) {
        int32_t b, x, y, z;
        read_coords(coords + i * stride, stride, b, x, y, z);
        const int32_t bx = x >> 2, by = y >> 2, bz = z >> 2;
        const int lx = x & 3, ly = y & 3, lz = z & 3;
        const int ox = lx == 0 ? -1 : (lx == 3 ? 1 : 0);
        const int oy = ly == 0 ? -1 : (ly == 3 ? 1 : 0);
        const int oz = lz == 0 ? -1 : (lz == 3 ? 1 : 0);
        // s_base[m] = bucket base (bucket * 64) of block own + (ax ? ox : 0, ay ? oy : 0, az ? oz : 0), or -1
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int ax = (m >> 2) & 1, ay = (m >> 1) & 1, az = m & 1;
            const bool need = (!ax || ox) && (!ay || oy) && (!az || oz);
            const int32_t cx = bx + (ax ? ox : 0), cy = by + (ay ? oy : 0), cz = bz + (az ? oz : 0);
            int bucket = -1;
            if (need && cx >= 0 && cy >= 0 && cz >= 0) {
                const uint64_t h = block_slot(b, cx, cy, cz, mask);
                bucket = block_resolve(t, mask, block_key(b, cx, cy, cz), h, slot_at(t, h));
            }
            s_base[m][threadIdx.x] = bucket >= 0 ? bucket * 64 : -1;
        }
        // per axis and offset d in {-1, 0, +1}: the block-select bit (x + d leaves the block) and the
        // position in the block, pre-shifted into the bucket index
        const int mx[3] = {lx == 0 ? 4 : 0, 0, lx == 3 ? 4 : 0};
        const int my[3] = {ly == 0 ? 2 : 0, 0, ly == 3 ? 2 : 0};
        const int mz[3] = {lz == 0 ? 1 : 0, 0, lz == 3 ? 1 : 0};
        const int px[3] = {((lx - 1) & 3) << 4, lx << 4, ((lx + 1) & 3) << 4};
        const int py[3] = {((ly - 1) & 3) << 2, ly << 2, ((ly + 1) & 3) << 2};
        const int pz[3] = {(lz - 1) & 3, lz, (lz + 1) & 3};
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int tap = tap_at<NT>(j);
            const int kd = tap / 9, kh = (tap / 3) % 3, kw = tap % 3;
            const int bb = s_base[mx[kd] | my[kh] | mz[kw]][threadIdx.x];
            int32_t r = -1;
            if (bb >= 0) r = __ldg(pool + bb + (px[kd] | py[kh] | pz[kw]));
            nbr[(int64_t)j * n + i] = r >= 0 ? r : (int32_t)n;
        }
    }
}

// ---- sorted layout ---------------------------------------------------------------------------
// When the rows are in strictly ascending (batch, x, y, z) order (no repeated coordinate), every
// (batch, x, y) column of voxels is a contiguous run of rows with z ascending. A dense table over
// the columns of the bounding box holds each column's row range, built with plain stores from
// the column boundaries of the row order (no hashing, no atomics), and a lookup finds z - 1, z
// and z + 1 in the 9 columns (x + dx, y + dy). It applies when the block layout's coordinate
// range holds (so no two coordinates share a key and out-of-grid neighbours are absent), the rows
// are in that order, and the box has at most col_cap columns; the rows' z values are copied to a
// compact array so that a column's rows sit in one or two sectors. All three conditions are
// decided on the device; when one fails, the block layout builds the map.

constexpr int kSrtPer = 4;      // rows per thread per grid-stride step of the check

__device__ __forceinline__ uint64_t srt_key(int32_t b, int32_t x, int32_t y, int32_t z) {
    return ((uint64_t)(uint32_t)b << 60) | ((uint64_t)(uint32_t)x << 40) | ((uint64_t)(uint32_t)y << 20) |
           (uint64_t)(uint32_t)z;
}

struct SrtBox {
    int32_t b0, x0, y0, x1, y1;
    int64_t nx, ny;
};

__device__ __forceinline__ SrtBox srt_box(const BlockCtl* ctl) {
    SrtBox bx;
    bx.b0 = kMaxCoord - ctl->lo_inv[0];
    bx.x0 = kMaxCoord - ctl->lo_inv[1];
    bx.y0 = kMaxCoord - ctl->lo_inv[2];
    bx.x1 = ctl->hi[1];
    bx.y1 = ctl->hi[2];
    bx.nx = (int64_t)bx.x1 - bx.x0 + 1;
    bx.ny = (int64_t)bx.y1 - bx.y0 + 1;
    return bx;
}

// Column index of (b, x, y) inside the box; below col_cap < 2^31 wherever the layout applies.
__device__ __forceinline__ int srt_col(const SrtBox& bx, int32_t b, int32_t x, int32_t y) {
    return ((b - bx.b0) * (int)bx.nx + (x - bx.x0)) * (int)bx.ny + (y - bx.y0);
}

__device__ __forceinline__ int warp_min(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_max(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// First kernel of a build: range and order check, the (batch, x, y) bounding box and the compact
// z array. Grid-stride over steps of kSrtPer rows per thread (kTpb apart, coalesced, loaded
// together; row i - 1 from the neighbouring lane); a small grid, since each block ends with one
// set of atomics on the same few words.
__global__ void __launch_bounds__(kTpb) k_srt_check(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                    bool vec, BlockCtl* __restrict__ ctl, int32_t* __restrict__ zc) {
    __shared__ int s_red[kTpb / 32][7];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int bad = 0;
    int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {INT_MIN, INT_MIN, INT_MIN};
    const int64_t step = (int64_t)gridDim.x * kTpb * kSrtPer;
    for (int64_t base = (int64_t)blockIdx.x * kTpb * kSrtPer; base < n; base += step) {
        int32_t b[kSrtPer], x[kSrtPer], y[kSrtPer], z[kSrtPer];
#pragma unroll
        for (int j = 0; j < kSrtPer; ++j) {
            const int64_t i = base + (int64_t)j * kTpb + threadIdx.x;
            b[j] = x[j] = y[j] = z[j] = 0;
            if (i < n) load_row(coords, i, stride, vec, b[j], x[j], y[j], z[j]);
        }
#pragma unroll
        for (int j = 0; j < kSrtPer; ++j) {
            const int64_t i = base + (int64_t)j * kTpb + threadIdx.x;
            const uint64_t key = srt_key(b[j], x[j], y[j], z[j]);
            uint64_t prev = __shfl_up_sync(0xffffffffu, key, 1);
            if (i >= n) continue;
            if ((uint32_t)x[j] > (uint32_t)kMaxCoord || (uint32_t)y[j] > (uint32_t)kMaxCoord ||
                (uint32_t)z[j] > (uint32_t)kMaxCoord || (uint32_t)b[j] > 15u)
                bad = 1;
            zc[i] = z[j];
            if (lane == 0 && i > 0) {
                int32_t pb, px, py, pz;
                load_row(coords, i - 1, stride, vec, pb, px, py, pz);
                prev = srt_key(pb, px, py, pz);
            }
            if (i > 0 && prev >= key) bad = 1;       // out of order, or a repeated coordinate
            lo[0] = min(lo[0], b[j]); lo[1] = min(lo[1], x[j]); lo[2] = min(lo[2], y[j]);
            hi[0] = max(hi[0], b[j]); hi[1] = max(hi[1], x[j]); hi[2] = max(hi[2], y[j]);
        }
    }
    bad = __any_sync(0xffffffffu, bad);
#pragma unroll
    for (int k = 0; k < 3; ++k) { lo[k] = warp_min(lo[k]); hi[k] = warp_max(hi[k]); }
    if (lane == 0) {
        s_red[warp][0] = bad;
#pragma unroll
        for (int k = 0; k < 3; ++k) { s_red[warp][1 + k] = lo[k]; s_red[warp][4 + k] = hi[k]; }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kTpb / 32; ++w) {
            bad |= s_red[w][0];
#pragma unroll
            for (int k = 0; k < 3; ++k) { lo[k] = min(lo[k], s_red[w][1 + k]); hi[k] = max(hi[k], s_red[w][4 + k]); }
        }
        if (bad) ctl->unsorted = 1;
        if (lo[0] <= hi[0]) {          // the block saw at least one row; with bad unset they are in range
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                atomicMax(&ctl->lo_inv[k], kMaxCoord - max(0, min(lo[k], kMaxCoord)));
                atomicMax(&ctl->hi[k], max(0, min(hi[k], kMaxCoord)));
            }
        }
    }
}

// cols[column] = {first row, last row + 1} from the column boundaries of the row order
// (grid-stride, one row at a time, its neighbours' coordinates read again).
__device__ __forceinline__ void srt_fill_body(const int32_t* __restrict__ coords, int64_t n, int stride, bool vec,
                                              const BlockCtl* __restrict__ ctl, int2* __restrict__ cols) {
    const SrtBox bx = srt_box(ctl);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int32_t b, x, y, z;
        load_row(coords, i, stride, vec, b, x, y, z);
        const int c = srt_col(bx, b, x, y);
        bool first = i == 0, last = i == n - 1;
        if (!first) {
            load_row(coords, i - 1, stride, vec, b, x, y, z);
            first = srt_col(bx, b, x, y) != c;
        }
        if (!last) {
            load_row(coords, i + 1, stride, vec, b, x, y, z);
            last = srt_col(bx, b, x, y) != c;
        }
        if (first) cols[c].x = (int)i;
        if (last) cols[c].y = (int)(i + 1);
    }
}

// Slot of a tap in the tap list (-1 when the list does not hold it).
template <int NT>
__device__ __forceinline__ constexpr int slot_of_tap(int tap) {
    for (int j = 0; j < NT; ++j)
        if (tap_at<NT>(j) == tap) return j;
    return -1;
}

// Column c = kd * 3 + kh (x + kd - 1, y + kh - 1) holds a tap of the list.
template <int NT>
__device__ __forceinline__ constexpr bool srt_col_needed(int c) {
    return slot_of_tap<NT>(c * 3) >= 0 || slot_of_tap<NT>(c * 3 + 1) >= 0 || slot_of_tap<NT>(c * 3 + 2) >= 0;
}

// The rows of z - 1, z and z + 1 (-1 where absent) among the column rows [s, e), whose z values
// strictly ascend: a binary search for the first row with z' >= z - 1, then at most three rows.
__device__ __forceinline__ void srt_col_find(const int32_t* __restrict__ zc, int s, int e, int z, int& rm, int& r0,
                                             int& rp) {
    rm = r0 = rp = -1;
    int lo = s, hi = e;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(zc + mid) < z - 1) lo = mid + 1; else hi = mid;
    }
    for (int k = lo; k < e && k < lo + 3; ++k) {
        const int d = __ldg(zc + k) - z;
        if (d > 1) return;
        if (d < 0) rm = k; else if (d == 0) r0 = k; else rp = k;
    }
}

// One row per thread: per neighbouring column (x + dx, y + dy) its row range from the table, then
// srt_col_find; in the voxel's own column row i itself, and z -/+ 1 can only be rows i -/+ 1.
template <int NT>
__device__ __forceinline__ void srt_lookup_body(const int32_t* __restrict__ coords, int64_t n, int stride, bool vec,
                                                const BlockCtl* __restrict__ ctl, const int2* __restrict__ cols,
                                                const int32_t* __restrict__ zc, int32_t* __restrict__ nbr) {
    const int64_t i = blockIdx.x * (int64_t)kTpb + threadIdx.x;
    if (i >= n) return;
    const SrtBox bx = srt_box(ctl);
    int32_t b, x, y, z;
    load_row(coords, i, stride, vec, b, x, y, z);
#pragma unroll
    for (int c = 0; c < 9; ++c) {
        if (!srt_col_needed<NT>(c)) continue;
        const int32_t xx = x + c / 3 - 1, yy = y + c % 3 - 1;
        int rm = -1, r0 = -1, rp = -1;
        if (c == 4) {
            const int2 se = __ldg(cols + srt_col(bx, b, x, y));
            r0 = (int)i;
            if (i > se.x && __ldg(zc + i - 1) == z - 1) rm = (int)i - 1;
            if (i + 1 < se.y && __ldg(zc + i + 1) == z + 1) rp = (int)i + 1;
        } else if (xx >= bx.x0 && xx <= bx.x1 && yy >= bx.y0 && yy <= bx.y1) {
            const int2 se = __ldg(cols + srt_col(bx, b, xx, yy));
            if (se.y > se.x) srt_col_find(zc, se.x, se.y, z, rm, r0, rp);
        }
        const int jm = slot_of_tap<NT>(c * 3), j0 = slot_of_tap<NT>(c * 3 + 1), jp = slot_of_tap<NT>(c * 3 + 2);
        if (jm >= 0) nbr[(int64_t)jm * n + i] = rm >= 0 ? rm : (int32_t)n;
        if (j0 >= 0) nbr[(int64_t)j0 * n + i] = r0 >= 0 ? r0 : (int32_t)n;
        if (jp >= 0) nbr[(int64_t)jp * n + i] = rp >= 0 ? rp : (int32_t)n;
    }
}

// ---- the build: six kernels, whichever layout applies ----------------------------------------
// 1 k_srt_check (above). 2-6 below: each branches on the layout decided on the device, so the
// layouts share launches and a build that takes the sorted layout ends with two that return at
// once. The block and voxel-hash tables share memory (the block table is a prefix of the voxel
// hash's), the sorted layout's column table takes the bucket pool's memory and its z array the
// table's: only one layout writes them in a build.

// 2: the layout, then the sorted layout's column table or the block layout's table cleared.
__global__ void __launch_bounds__(kTpb) k_map_decide_clear(BlockCtl* __restrict__ ctl, int2* __restrict__ cols,
                                                           uint64_t col_cap, Slot* __restrict__ t, uint64_t cap_b) {
    const SrtBox bx = srt_box(ctl);
    const int64_t nb = (int64_t)ctl->hi[0] - bx.b0 + 1;
    const bool applies = !ctl->unsorted && nb > 0 && bx.nx > 0 && bx.ny > 0 &&
                         (uint64_t)nb * (uint64_t)bx.nx * (uint64_t)bx.ny <= col_cap;
    if (blockIdx.x == 0 && threadIdx.x == 0) ctl->sorted = applies ? 1 : 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (applies) {
        const uint64_t cells = (uint64_t)nb * (uint64_t)bx.nx * (uint64_t)bx.ny;
        for (; c < cells; c += stride) cols[c] = make_int2(0, 0);
    } else {
        for (; c < cap_b; c += stride) {
            ulonglong2 v; v.x = kEmpty; v.y = 0xFFFFFFFFull;   // row = -1
            reinterpret_cast<ulonglong2*>(t)[c] = v;
        }
    }
}

// 3: the sorted layout's column table, or the block layout's block claims.
__global__ void k_map_fill_claim(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                         bool vec, BlockCtl* __restrict__ ctl, int2* __restrict__ cols,
                                                         Slot* __restrict__ t, uint64_t mask_b,
                                                         unsigned int pool_blocks) {
    if (ctl->sorted) srt_fill_body(coords, n, stride, vec, ctl, cols);
    else blk_insert_body(coords, n, stride, t, mask_b, ctl, pool_blocks);
}

// 4: the sorted layout's lookups; otherwise the block layout's bucket pool cleared, or the voxel
// hash's table when the block layout did not apply either.
template <int NT>
__global__ void __launch_bounds__(kTpb) k_map_lookup_clear(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                           bool vec, const BlockCtl* __restrict__ ctl,
                                                           const int2* __restrict__ cols, const int32_t* __restrict__ zc,
                                                           int32_t* __restrict__ nbr, int32_t* __restrict__ pool,
                                                           Slot* __restrict__ t, uint64_t cap, int* __restrict__ special) {
    if (ctl->sorted) {
        srt_lookup_body<NT>(coords, n, stride, vec, ctl, cols, zc, nbr);
    } else if (ctl->fallback) {
        hash_clear_body(t, cap, special);
    } else {
        const uint64_t total = (uint64_t)ctl->nblocks * 16;            // int4 words
        const uint64_t stride_w = (uint64_t)gridDim.x * blockDim.x;
        for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < total; j += stride_w)
            reinterpret_cast<int4*>(pool)[j] = make_int4(-1, -1, -1, -1);
    }
}

// 5: the block layout's voxel inserts, or the voxel hash's inserts (nothing for the sorted layout).
__global__ void __launch_bounds__(kTpb) k_map_insert(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                     const BlockCtl* __restrict__ ctl, Slot* __restrict__ t,
                                                     uint64_t mask_b, int32_t* __restrict__ pool, uint64_t cap,
                                                     int* __restrict__ special, int* __restrict__ err) {
    if (ctl->sorted) return;
    if (ctl->fallback) hash_insert_body(coords, n, stride, t, cap - 1, special, err);
    else vox_insert_body(coords, n, stride, t, mask_b, pool);
}

// 6: the block layout's lookups, or the voxel hash's (nothing for the sorted layout).
template <int NT>
__global__ void __launch_bounds__(kTpb) k_map_lookup(const int32_t* __restrict__ coords, int64_t n, int stride,
                                                     const BlockCtl* __restrict__ ctl, const Slot* __restrict__ t,
                                                     uint64_t mask_b, const int32_t* __restrict__ pool, uint64_t cap,
                                                     const int* __restrict__ special, int32_t* __restrict__ nbr,
                                                     int* __restrict__ err) {
    __shared__ int s_base[8][kTpb];
    if (ctl->sorted) return;
    if (ctl->fallback) nbr_lookup_body<NT>(coords, n, stride, t, cap - 1, special, nbr, err);
    else blk_lookup_body<NT>(coords, n, stride, t, mask_b, pool, nbr, s_base);
}

__global__ void k_count_valid(const int32_t* __restrict__ nbr, int64_t total, int32_t n,
                              unsigned long long* __restrict__ out) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    unsigned long long local = 0;
    for (; i < total; i += stride) local += (nbr[i] != n);
    for (int o = 16; o > 0; o >>= 1) local += __shfl_down_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, local);
}

__global__ void k_zslab_counts(const int32_t* __restrict__ coords, int64_t n, int stride,
                               int32_t z_min, int32_t nz, unsigned long long* __restrict__ counts) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t z = coords[i * stride + (stride - 1)];
    const int64_t b = (int64_t)z - z_min;
    if (b >= 0 && b < nz) atomicAdd(&counts[b], 1ull);
}

__global__ void k_gather_rows(const uint32_t* __restrict__ src, const int32_t* __restrict__ rows,
                              int64_t m, int64_t words, uint32_t* __restrict__ out) {
    // one warp per row, 4-byte words (16-byte vectors when the row allows it)
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= m) return;
    const int64_t r = rows[warp];
    const uint32_t* s = src + r * words;
    uint32_t* d = out + warp * words;
    if ((words & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
        const int64_t v = words >> 2;
        for (int64_t k = lane; k < v; k += 32)
            reinterpret_cast<uint4*>(d)[k] = reinterpret_cast<const uint4*>(s)[k];
    } else {
        for (int64_t k = lane; k < words; k += 32) d[k] = s[k];
    }
}

// out[rows[k]] = src[k]: the inverse of k_gather_rows (halo rows received into a contiguous
// buffer land at their positions in the local row order).
__global__ void k_scatter_rows(const uint32_t* __restrict__ src, const int32_t* __restrict__ rows,
                               int64_t m, int64_t words, uint32_t* __restrict__ out) {
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= m) return;
    const int64_t r = rows[warp];
    const uint32_t* s = src + warp * words;
    uint32_t* d = out + r * words;
    if ((words & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
        const int64_t v = words >> 2;
        for (int64_t k = lane; k < v; k += 32)
            reinterpret_cast<uint4*>(d)[k] = reinterpret_cast<const uint4*>(s)[k];
    } else {
        for (int64_t k = lane; k < words; k += 32) d[k] = s[k];
    }
}

}  // namespace

uint64_t tb_hash_capacity(int64_t n) {
    uint64_t cap = 1024;
    while (cap < (uint64_t)(2 * n)) cap <<= 1;
    return cap;
}

// Buckets for at most N/4 + 64 blocks, and fewer than 2^25 so a bucket's first entry index
// (bucket * 64) fits an int; more blocks than that send the build to the voxel hash.
static uint64_t tb_nbr_pool_blocks(int64_t n) {
    return std::min<uint64_t>((uint64_t)n / 4 + 64, (1ull << 25) - 64);
}

// The voxel-hash table (cap Slots, then one int: the all-ones key cell, padded to 16 bytes),
// BlockCtl, and the block layout's bucket pool.
size_t tb_nbr_workspace_bytes(int64_t n) {
    const uint64_t cap = tb_hash_capacity(n);
    return cap * sizeof(Slot) + 16 + sizeof(BlockCtl) + tb_nbr_pool_blocks(n) * 64 * sizeof(int32_t);
}

namespace {

template <int NT>
tb_status nbr_build_blocks(tb_ctx* ctx, const int32_t* coords, int64_t n, int stride, int32_t* nbr, void* ws) {
    const uint64_t cap = tb_hash_capacity(n);                   // voxel-hash table
    const uint64_t pool_blocks = tb_nbr_pool_blocks(n);
    const uint64_t cap_b = tb_hash_capacity((int64_t)pool_blocks);   // block table, a prefix of it
    const uint64_t mask_b = cap_b - 1;
    Slot* t = reinterpret_cast<Slot*>(ws);
    int* special = reinterpret_cast<int*>(t + cap);
    unsigned char* after = reinterpret_cast<unsigned char*>(t + cap) + 16;
    BlockCtl* ctl = reinterpret_cast<BlockCtl*>(after);
    int32_t* pool = reinterpret_cast<int32_t*>(after + sizeof(BlockCtl));
    int2* cols = reinterpret_cast<int2*>(pool);                 // sorted layout: column table
    int32_t* zc = reinterpret_cast<int32_t*>(t);                // sorted layout: z of every row
    const uint64_t col_cap = pool_blocks * 64 * sizeof(int32_t) / sizeof(int2);
    const bool vec = stride == 4 && (reinterpret_cast<uintptr_t>(coords) & 15) == 0;
    const int64_t sms = ctx->num_sms;
    const int64_t blocks = (n + kTpb - 1) / kTpb;
    const int64_t ins_blocks = (n + (int64_t)kTpb * kInsPer - 1) / ((int64_t)kTpb * kInsPer);
    TB_CUDA_TRY(ctx, cudaMemsetAsync(ctl, 0, sizeof(BlockCtl), ctx->stream));
    k_srt_check<<<(unsigned)std::min<int64_t>((n + kTpb * kSrtPer - 1) / (kTpb * kSrtPer), sms * 4), kTpb, 0,
                  ctx->stream>>>(coords, n, stride, vec, ctl, zc);
    TB_LAUNCH_CHECK(ctx, "k_srt_check");
    k_map_decide_clear<<<(unsigned)(sms * 8), kTpb, 0, ctx->stream>>>(ctl, cols, col_cap, t, cap_b);
    TB_LAUNCH_CHECK(ctx, "k_map_decide_clear");
    k_map_fill_claim<<<(unsigned)ins_blocks, kTpb, 0, ctx->stream>>>(coords, n, stride, vec, ctl, cols, t, mask_b,
                                                                     (unsigned)pool_blocks);
    TB_LAUNCH_CHECK(ctx, "k_map_fill_claim");
    k_map_lookup_clear<NT><<<(unsigned)blocks, kTpb, 0, ctx->stream>>>(coords, n, stride, vec, ctl, cols, zc, nbr, pool,
                                                                       t, cap, special);
    TB_LAUNCH_CHECK(ctx, "k_map_lookup_clear");
    // grid-stride kernels: when the sorted layout applied they return at once, so a small grid
    k_map_insert<<<(unsigned)std::min<int64_t>(ins_blocks, sms * 8), kTpb, 0, ctx->stream>>>(
        coords, n, stride, ctl, t, mask_b, pool, cap, special, ctx->d_err);
    TB_LAUNCH_CHECK(ctx, "k_map_insert");
    k_map_lookup<NT><<<(unsigned)std::min<int64_t>(blocks, sms * 8), kTpb, 0, ctx->stream>>>(
        coords, n, stride, ctl, t, mask_b, pool, cap, special, nbr, ctx->d_err);
    TB_LAUNCH_CHECK(ctx, "k_map_lookup");
    return TB_OK;
}

}  // namespace

tb_status tb_nbr_build_blocks(tb_ctx* ctx, const int32_t* coords, int64_t n, int stride, int32_t* nbr, void* ws) {
    return nbr_build_blocks<27>(ctx, coords, n, stride, nbr, ws);
}

tb_status tb_nbr_build_quad_taps(tb_ctx* ctx, const int32_t* coords, int64_t n, int stride, int32_t* out, void* ws) {
    return nbr_build_blocks<7>(ctx, coords, n, stride, out, ws);
}

extern "C" tb_status tb_build_neighbor_map(tb_ctx* ctx, const int32_t* coords, int64_t n,
                                           int coord_stride, int32_t* nbr_out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_build_neighbor_map: n < 0 or coord_stride not 3/4");
    if (n == 0) return TB_OK;
    if (!coords || !nbr_out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_build_neighbor_map: null pointer");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_build_neighbor_map: n must be < 2^31-1");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    tb_status s = tb_ensure(ctx, &ctx->ws, &ctx->ws_bytes, tb_nbr_workspace_bytes(n), "neighbor-map workspace");
    if (s != TB_OK) return s;
    return tb_nbr_build_blocks(ctx, coords, n, coord_stride, nbr_out, ctx->ws);
}

extern "C" tb_status tb_count_valid_pairs(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t* pairs) {
    if (!ctx || !pairs || n < 0) return TB_ERR_INVALID_ARG;
    *pairs = 0;
    if (n == 0) return TB_OK;
    if (!nbr) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_count_valid_pairs: null nbr");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    tb_status s = tb_ensure(ctx, &ctx->ws, &ctx->ws_bytes, 16, "counter");
    if (s != TB_OK) return s;
    unsigned long long* d = reinterpret_cast<unsigned long long*>(ctx->ws);
    TB_CUDA_TRY(ctx, cudaMemsetAsync(d, 0, sizeof(unsigned long long), ctx->stream));
    k_count_valid<<<ctx->num_sms * 8, 256, 0, ctx->stream>>>(nbr, 27 * n, (int32_t)n, d);
    TB_LAUNCH_CHECK(ctx, "k_count_valid");
    unsigned long long h = 0;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    *pairs = (int64_t)h;
    return TB_OK;
}

extern "C" tb_status tb_zslab_counts(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                                     int32_t z_min, int32_t nz, int64_t* counts) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || nz <= 0 || (coord_stride != 3 && coord_stride != 4) || !counts)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_zslab_counts: bad arguments");
    if (n > 0 && !coords) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_zslab_counts: null coords");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    TB_CUDA_TRY(ctx, cudaMemsetAsync(counts, 0, sizeof(int64_t) * (size_t)nz, ctx->stream));
    if (n == 0) return TB_OK;
    k_zslab_counts<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
        coords, n, coord_stride, z_min, nz, reinterpret_cast<unsigned long long*>(counts));
    TB_LAUNCH_CHECK(ctx, "k_zslab_counts");
    return TB_OK;
}

extern "C" tb_status tb_gather_rows(tb_ctx* ctx, const void* src, const int32_t* rows, int64_t m,
                                    int64_t row_bytes, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (m < 0 || row_bytes <= 0 || (row_bytes & 3))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_gather_rows: m < 0 or row_bytes not a positive multiple of 4");
    if (m == 0) return TB_OK;
    if (!src || !rows || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_gather_rows: null pointer");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int64_t threads = m * 32;
    k_gather_rows<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const uint32_t*>(src), rows, m, row_bytes / 4, reinterpret_cast<uint32_t*>(out));
    TB_LAUNCH_CHECK(ctx, "k_gather_rows");
    return TB_OK;
}

extern "C" tb_status tb_scatter_rows(tb_ctx* ctx, const void* src, const int32_t* rows, int64_t m,
                                     int64_t row_bytes, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (m < 0 || row_bytes <= 0 || (row_bytes & 3))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_scatter_rows: m < 0 or row_bytes not a positive multiple of 4");
    if (m == 0) return TB_OK;
    if (!src || !rows || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_scatter_rows: null pointer");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int64_t threads = m * 32;
    k_scatter_rows<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const uint32_t*>(src), rows, m, row_bytes / 4, reinterpret_cast<uint32_t*>(out));
    TB_LAUNCH_CHECK(ctx, "k_scatter_rows");
    return TB_OK;
}

// ---- neighbor map without any device allocation ---------------------------------------------
// Some callers cannot allocate device memory at the point where they need a neighbor map:
// for example a host framework that hands out all device memory from its own pool and treats
// any other allocation as an accounting error, or code that must not call cudaMalloc because
// that call can synchronise the whole device and stall unrelated work. For them this entry
// point builds the same map as tb_build_neighbor_map using a hash table that is part of the
// library image: a static device array that every GPU loading the library holds until the
// process exits. No context is needed and nothing is allocated or freed.
namespace {

constexpr int64_t kNoAllocMaxVoxels = TB_NOALLOC_MAX_VOXELS;
constexpr uint64_t kNoAllocSlots = 2 * (uint64_t)kNoAllocMaxVoxels;      // load factor <= 1/2
constexpr size_t kNoAllocBytes = kNoAllocSlots * sizeof(Slot) + 256;    // slots + the all-ones-key cell
static_assert(kNoAllocBytes == TB_NOALLOC_SCRATCH, "the header states the array's size");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
void* g_noalloc_addr[kMaxDevices];          // device address of g_noalloc_scratch, per device
int g_noalloc_sms[kMaxDevices];
std::once_flag g_noalloc_once[kMaxDevices];
cudaError_t g_noalloc_setup_err[kMaxDevices];

// True when p is device (or managed) memory that device `dev` can use as a kernel argument.
bool noalloc_on_device(const void* p, int dev) {
    cudaPointerAttributes a;
    const cudaError_t pending = cudaPeekAtLastError();
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        // clear the error this query left, but only when no earlier error was pending: that one
        // belongs to the caller's own work
        if (pending == cudaSuccess) cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeDevice && a.device == dev;
}

}  // namespace

extern "C" tb_status tb_build_neighbor_map_noalloc(void* stream, const int32_t* coords, int64_t n,
                                                   int coord_stride, int32_t* nbr_out) {
    if (n < 0 || (coord_stride != 3 && coord_stride != 4)) return TB_ERR_INVALID_ARG;
    if (n > kNoAllocMaxVoxels) return TB_ERR_TOO_LARGE;       // nothing enqueued
    if (n == 0) return TB_OK;
    if (!coords || !nbr_out) return TB_ERR_INVALID_ARG;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TB_ERR_CUDA;
    // both arrays must live on the current device: the kernels run there
    if (!noalloc_on_device(coords, dev) || !noalloc_on_device(nbr_out, dev)) return TB_ERR_INVALID_ARG;
    // one-time set-up per device, with that device current: the host-side name of the array is
    // only a stand-in, so its device address has to be looked up before a kernel may use it
    std::call_once(g_noalloc_once[dev], [dev]() {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        int sms = 0;
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_noalloc_setup_err[dev] = e;
        if (e == cudaSuccess) {
            g_noalloc_addr[dev] = ptr;
            g_noalloc_sms[dev] = sms;
        }
    });
    if (g_noalloc_setup_err[dev] != cudaSuccess || !g_noalloc_addr[dev]) return TB_ERR_CUDA;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint64_t cap = tb_hash_capacity(n);                   // <= kNoAllocSlots for n <= the maximum
    Slot* t = reinterpret_cast<Slot*>(g_noalloc_addr[dev]);
    int* special = reinterpret_cast<int*>(t + cap);
    // No error word: the table has at least 2n slots for at most n keys, and the probe loops may
    // scan the whole table, so an insert always finds a free or matching slot and a lookup always
    // reaches one; the probe bound of the hash kernels can never be hit here.
    int* const no_err = nullptr;
    const int tpb = 256;
    const int64_t blocks = (n + tpb - 1) / tpb;
    // every call rebuilds the table from scratch: the previous call's contents are cleared here.
    // Each launch's own status is checked (cudaLaunchKernelEx returns it), so an error left
    // pending by unrelated earlier work is neither reported as this call's nor cleared.
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(tpb);
    cfg.stream = st;
    cfg.gridDim = dim3((unsigned)std::min<uint64_t>((cap + tpb - 1) / tpb, (uint64_t)g_noalloc_sms[dev] * 16));
    if (cudaLaunchKernelEx(&cfg, k_hash_clear, t, cap, special) != cudaSuccess) return TB_ERR_CUDA;
    cfg.gridDim = dim3((unsigned)blocks);
    if (cudaLaunchKernelEx(&cfg, k_hash_insert, coords, n, coord_stride, t, cap - 1, special, no_err) != cudaSuccess)
        return TB_ERR_CUDA;
    if (cudaLaunchKernelEx(&cfg, k_nbr_lookup<27>, coords, n, coord_stride, (const Slot*)t, cap - 1,
                           (const int*)special, nbr_out, no_err) != cudaSuccess)
        return TB_ERR_CUDA;
    return TB_OK;
}
