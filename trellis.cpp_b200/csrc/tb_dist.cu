// Multi-GPU z-slabs: a voxel set split across ranks along z, one process per GPU, with the
// one-plane halo of every conv exchanged over NCCL send/recv.
//
// The reference runs on one device and only chunks output rows within it (src/sparse.cpp:94-118);
// its per-stage caller (src/shape_decoder.cpp:91-113) builds one neighbor table and runs the
// stage's convs on it. On N GPUs each rank does the same on its slab:
//
// * Partition (tb_dist_partition_zslab, once per voxel set): every rank passes the same global
//   coordinates. A z histogram on the device (one small read-back) gives the cut at voxel-count
//   quantiles on whole planes (tb_zslab_cuts, shared with the host-side tests). Rank r owns
//   z in [z_lo, z_hi) and also holds the halo planes z_lo - 1 and z_hi of its neighbours: a 3^3
//   submanifold conv at an owned voxel reads only voxels within one plane.
// * Local order: the slab's rows sorted stably by z (one radix-sort pass over plane indices), so
//   the local rows are [halo plane z_lo-1 | plane z_lo | interior planes | plane z_hi-1 | halo
//   plane z_hi], each a contiguous range, and within a plane the input's (x-major) order. The
//   halo planes are received in place and the edge planes sent in place (no pack or unpack
//   kernels), and the interior rows -- whose neighbours are all owned -- are one range that a
//   conv can run while the halo is in flight.
// * Axis relabelling: the local coordinates are stored as (z, x, y) (batch kept first), so the
//   local map's tap groups (kd, the leading axis) are the z offsets, and in the z-major local order
//   each group's neighbour rows again form one contiguous range per 128-row tile, which is what
//   the tensor-core kernels stream. A local tap t' = kd'*9 + kh'*3 + kw' is the global tap
//   kh'*9 + kw'*3 + kd' (offsets (kh'-1, kw'-1, kd'-1) on x, y, z); the convs take the weight with
//   its taps permuted to match, so the result is the reference's conv. Only the order in which an
//   output row's 27 products are accumulated differs from the single-GPU launch (fp32 rounding).
// * A conv (tb_dist_submconv): the weight permutation, then the halo exchange of the input's edge
//   planes on a communication stream (ncclGroupStart; ncclSend / ncclRecv with each neighbour;
//   ncclGroupEnd) while the interior rows run on the caller's stream, then the two edge planes.
//   Only owned rows are computed and written.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, the copy already in the process when
// there is one), so the library loads and runs its single-GPU calls where NCCL is absent.
#include "tb_common.cuh"

#include <nccl.h>   // types and constants only; the functions are looked up with dlsym
#include <dlfcn.h>

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);   // the process's own copy, if any
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW);
        if (!h) {
            const char* e = dlerror();
            api.why = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "");
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv &&
                 api.group_start && api.group_end && api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks a needed symbol";
    });
    return api;
}

// global tap of local tap t' (local coordinates are (z, x, y) of the global (x, y, z))
__host__ __device__ __forceinline__ int global_tap(int tl) { return ((tl / 3) % 3) * 9 + (tl % 3) * 3 + tl / 9; }

__global__ void k_z_minmax(const int32_t* __restrict__ coords, int64_t n, int stride, int* __restrict__ mm) {
    int lo = INT_MAX, hi = INT_MIN;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int z = coords[i * stride + stride - 1];
        lo = min(lo, z);
        hi = max(hi, z);
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if ((threadIdx.x & 31) == 0) {
        atomicMin(mm, lo);
        atomicMax(mm + 1, hi);
    }
}

__global__ void k_z_hist(const int32_t* __restrict__ coords, int64_t n, int stride, int32_t z_min, int32_t nz,
                         unsigned long long* __restrict__ counts) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = (int64_t)coords[i * stride + stride - 1] - z_min;
        if (b >= 0 && b < nz) atomicAdd(&counts[b], 1ull);
    }
}

// key = plane index within [plane0, plane0 + nplanes), or nplanes for rows outside the slab;
// val = the global row
__global__ void k_slab_keys(const int32_t* __restrict__ coords, int64_t n, int stride, int32_t plane0,
                            uint32_t nplanes, uint32_t* __restrict__ keys, int32_t* __restrict__ vals) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = (int64_t)coords[i * stride + stride - 1] - plane0;
        keys[i] = (p >= 0 && p < (int64_t)nplanes) ? (uint32_t)p : nplanes;
        vals[i] = (int32_t)i;
    }
}

// local coordinates: row k takes coords[rows[k]] (coords[k] when rows is null) with (x, y, z)
// stored as (z, x, y); a batch column stays first
__global__ void k_slab_coords(const int32_t* __restrict__ coords, int stride, const int32_t* __restrict__ rows,
                              int64_t m, int32_t* __restrict__ out) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < m; k += (int64_t)gridDim.x * blockDim.x) {
        const int32_t* c = coords + (rows ? (int64_t)rows[k] : k) * stride;
        int32_t* o = out + k * stride;
        const int b = stride - 3;
        if (b) o[0] = c[0];
        o[b] = c[b + 2];
        o[b + 1] = c[b];
        o[b + 2] = c[b + 1];
    }
}

// w_local[o][t'][c] = w[o][global_tap(t')][c]
template <typename T>
__global__ void k_permute_taps(const T* __restrict__ w, int64_t co, int ci, T* __restrict__ out) {
    const int64_t total = co * 27 * ci;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e % ci);
        const int tl = (int)((e / ci) % 27);
        const int64_t o = e / (27 * (int64_t)ci);
        out[e] = w[(o * 27 + global_tap(tl)) * ci + c];
    }
}

__global__ void k_count_range(const int32_t* __restrict__ nbr, int64_t n, int64_t r0, int64_t nr,
                              unsigned long long* __restrict__ out) {
    unsigned long long local = 0;
    const int64_t total = 27 * nr;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / nr, i = r0 + e % nr;
        local += (nbr[t * n + i] != (int32_t)n);
    }
    for (int o = 16; o > 0; o >>= 1) local += __shfl_down_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, local);
}

int grid_for(int64_t items, int sms) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)sms * 8));
}

}  // namespace

struct tb_dist {
    tb_ctx* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // the plan
    bool planned = false, mapped = false;
    int stride = 3;
    int halo = 1;                 // planes held per side (tb_dist_set_halo_planes)
    int64_t halo_rows_lo[TB_DIST_MAX_HALO] = {};   // rows of plane z_lo - 1 - k
    int64_t halo_rows_hi[TB_DIST_MAX_HALO] = {};   // rows of plane z_hi + k
    int64_t plane_rows_lo = 0, plane_rows_hi = 0;  // rows of the owned planes z_lo and z_hi - 1
    bool exchange_pending = false;                 // ev_join marks an exchange the next conv waits for
    tb_zslab slab{};
    void* rows = nullptr;         // int32 [n_local]: the global row of each local row
    void* coords = nullptr;       // int32 [n_local][stride]: local coordinates, (z, x, y) order
    void* nbr = nullptr;          // int32 [27][n_local]: the local map
    size_t rows_bytes = 0, coords_bytes = 0, nbr_bytes = 0;
    void* wperm = nullptr;        // the weight with its taps in local order
    size_t wperm_bytes = 0;
    void* scratch = nullptr;      // partition scratch: histogram, sort keys and values, CUB temp
    size_t scratch_bytes = 0;
    std::string last_error;
};

namespace {

tb_status dfail(tb_dist* d, tb_status s, const std::string& msg) {
    if (d) {
        d->last_error = msg;
        if (d->ctx) d->ctx->last_error = msg;
    }
    return s;
}

tb_status dcuda(tb_dist* d, cudaError_t e, const char* what) {
    return dfail(d, e == cudaErrorMemoryAllocation ? TB_ERR_OUT_OF_MEMORY : TB_ERR_CUDA,
                 std::string(what) + ": " + cudaGetErrorString(e));
}

#define TB_DCUDA(d, call)                                    \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return dcuda((d), e_, #call); \
    } while (0)

tb_status dnccl(tb_dist* d, ncclResult_t r, const char* what) {
    return dfail(d, TB_ERR_CUDA, std::string(what) + ": " + nccl().error_string(r));
}

// Grow a dist-owned device buffer (never shrinks); the stream is drained first, since queued
// work may still read the old buffer.
tb_status dgrow(tb_dist* d, void** buf, size_t* cap, size_t bytes) {
    if (*buf && *cap >= bytes) return TB_OK;
    if (*buf) {
        TB_DCUDA(d, cudaStreamSynchronize(d->ctx->stream));
        cudaFree(*buf);
        *buf = nullptr;
        *cap = 0;
    }
    const size_t want = std::max<size_t>(bytes, 256);
    cudaError_t e = cudaMalloc(buf, want);
    if (e != cudaSuccess) {
        *buf = nullptr;
        return dcuda(d, e, "cudaMalloc (tb_dist workspace)");
    }
    *cap = want;
    return TB_OK;
}

}  // namespace

extern "C" {

tb_status tb_zslab_cuts(const int64_t* counts, int32_t nz, int32_t z_min, int world, int32_t* cuts) {
    if (!counts || !cuts || nz < 0 || world < 1) return TB_ERR_INVALID_ARG;
    int64_t total = 0;
    for (int32_t i = 0; i < nz; ++i) {
        if (counts[i] < 0) return TB_ERR_INVALID_ARG;
        total += counts[i];
    }
    if (total == 0) {
        for (int r = 0; r <= world; ++r) cuts[r] = z_min + r;
        return TB_OK;
    }
    // the occupied planes, from the first to the last
    int32_t first = 0, last = nz - 1;
    while (counts[first] == 0) ++first;
    while (counts[last] == 0) --last;
    const int32_t zmin = z_min + first, zmax = z_min + last;
    if ((int64_t)zmax - zmin + 1 < world) return TB_ERR_INVALID_ARG;   // fewer planes than slabs
    cuts[0] = zmin;
    cuts[world] = zmax + 1;
    // cumulative counts from zmin; cut r goes after the first plane whose cumulative count reaches
    // total * r / world (compared as real numbers), kept so that every slab has at least one plane
    std::vector<int64_t> csum((size_t)(zmax - zmin + 1));
    int64_t acc = 0;
    for (int32_t z = zmin; z <= zmax; ++z) {
        acc += counts[z - z_min];
        csum[(size_t)(z - zmin)] = acc;
    }
    for (int r = 1; r < world; ++r) {
        const double q = (double)(total * (int64_t)r) / (double)world;
        const size_t k = (size_t)(std::lower_bound(csum.begin(), csum.end(), q,
                                                   [](int64_t a, double b) { return (double)a < b; }) -
                                  csum.begin());
        const int64_t lo = (int64_t)cuts[r - 1] + 1;
        const int64_t hi = (int64_t)zmax + 1 - (world - r);
        cuts[r] = (int32_t)std::min<int64_t>(std::max<int64_t>((int64_t)zmin + (int64_t)k + 1, lo), hi);
    }
    return TB_OK;
}

tb_status tb_nccl_unique_id(uint8_t* id) {
    if (!id) return TB_ERR_INVALID_ARG;
    NcclApi& api = nccl();
    if (!api.ok) return TB_ERR_UNSUPPORTED;
    ncclUniqueId u;
    if (api.get_unique_id(&u) != ncclSuccess) return TB_ERR_CUDA;
    memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return TB_OK;
}

tb_status tb_nccl_comm_create(const uint8_t* id, int rank, int world, int device, void** comm) {
    if (!id || !comm || world < 1 || rank < 0 || rank >= world) return TB_ERR_INVALID_ARG;
    *comm = nullptr;
    NcclApi& api = nccl();
    if (!api.ok) return TB_ERR_UNSUPPORTED;
    if (cudaSetDevice(device) != cudaSuccess) return TB_ERR_CUDA;
    ncclUniqueId u;
    memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t c = nullptr;
    if (api.comm_init_rank(&c, world, u, rank) != ncclSuccess) return TB_ERR_CUDA;
    *comm = c;
    return TB_OK;
}

tb_status tb_nccl_comm_destroy(void* comm) {
    if (!comm) return TB_OK;
    NcclApi& api = nccl();
    if (!api.ok) return TB_ERR_UNSUPPORTED;
    return api.comm_destroy(reinterpret_cast<ncclComm_t>(comm)) == ncclSuccess ? TB_OK : TB_ERR_CUDA;
}

tb_status tb_dist_create(tb_ctx* ctx, void* nccl_comm, int rank, int world, tb_dist** out) {
    if (!ctx || !out || world < 1 || rank < 0 || rank >= world) return TB_ERR_INVALID_ARG;
    *out = nullptr;
    if (nccl_comm && !nccl().ok) return tb_fail(ctx, TB_ERR_UNSUPPORTED, nccl().why);
    tb_dist* d = new (std::nothrow) tb_dist();
    if (!d) return TB_ERR_OUT_OF_MEMORY;
    d->ctx = ctx;
    d->comm = reinterpret_cast<ncclComm_t>(nccl_comm);
    d->rank = rank;
    d->world = world;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&d->comm_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->ev_join, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        tb_status s = tb_cuda_fail(ctx, e, "tb_dist_create");
        tb_dist_destroy(d);
        return s;
    }
    *out = d;
    return TB_OK;
}

tb_status tb_dist_destroy(tb_dist* d) {
    if (!d) return TB_OK;
    if (d->ctx) {
        cudaSetDevice(d->ctx->device);
        cudaStreamSynchronize(d->ctx->stream);
    }
    if (d->comm_stream) {
        cudaStreamSynchronize(d->comm_stream);
        cudaStreamDestroy(d->comm_stream);
    }
    if (d->ev_fork) cudaEventDestroy(d->ev_fork);
    if (d->ev_join) cudaEventDestroy(d->ev_join);
    for (void* p : {d->rows, d->coords, d->nbr, d->wperm, d->scratch})
        if (p) cudaFree(p);
    delete d;
    return TB_OK;
}

const char* tb_dist_last_error(const tb_dist* d) { return d ? d->last_error.c_str() : "null tb_dist"; }

tb_status tb_dist_partition_zslab(tb_dist* d, const int32_t* coords, int64_t n, int coord_stride, tb_zslab* slab) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!coords || !slab || n <= 0 || (coord_stride != 3 && coord_stride != 4))
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_partition_zslab: null pointer, n <= 0 or bad stride");
    if (n >= (int64_t)INT32_MAX) return dfail(d, TB_ERR_TOO_LARGE, "tb_dist_partition_zslab: n must be < 2^31-1");
    tb_ctx* ctx = d->ctx;
    cudaStream_t st = ctx->stream;
    TB_DCUDA(d, cudaSetDevice(ctx->device));
    d->planned = d->mapped = false;
    const int sms = ctx->num_sms;
    // 1. the z range (one read-back)
    tb_status s = dgrow(d, &d->scratch, &d->scratch_bytes, 256);
    if (s != TB_OK) return s;
    int* mm = reinterpret_cast<int*>(d->scratch);
    static const int init[2] = {INT_MAX, INT_MIN};
    TB_DCUDA(d, cudaMemcpyAsync(mm, init, sizeof(init), cudaMemcpyHostToDevice, st));
    k_z_minmax<<<grid_for(n, sms), 256, 0, st>>>(coords, n, coord_stride, mm);
    TB_DCUDA(d, cudaGetLastError());
    int zr[2];
    TB_DCUDA(d, cudaMemcpyAsync(zr, mm, sizeof(zr), cudaMemcpyDeviceToHost, st));
    TB_DCUDA(d, cudaStreamSynchronize(st));
    const int64_t nz = (int64_t)zr[1] - zr[0] + 1;
    if (nz > ((int64_t)1 << 24))
        return dfail(d, TB_ERR_TOO_LARGE, "tb_dist_partition_zslab: z spans more than 2^24 planes");
    // 2. the z histogram (one read-back) and the cut on the host
    const size_t key_bytes = ((size_t)n * 4 + 255) & ~(size_t)255;
    size_t cub_bytes = 0;
    TB_DCUDA(d, cub::DeviceRadixSort::SortPairs(nullptr, cub_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                                (const int32_t*)nullptr, (int32_t*)nullptr, (int)n, 0, 32, st));
    const size_t hist_bytes = ((size_t)nz * 8 + 255) & ~(size_t)255;
    s = dgrow(d, &d->scratch, &d->scratch_bytes, hist_bytes + 4 * key_bytes + cub_bytes + 256);
    if (s != TB_OK) return s;
    uint8_t* sb = reinterpret_cast<uint8_t*>(d->scratch);
    unsigned long long* hist = reinterpret_cast<unsigned long long*>(sb);
    uint32_t* keys_in = reinterpret_cast<uint32_t*>(sb + hist_bytes);
    uint32_t* keys_out = reinterpret_cast<uint32_t*>(sb + hist_bytes + key_bytes);
    int32_t* vals_in = reinterpret_cast<int32_t*>(sb + hist_bytes + 2 * key_bytes);
    int32_t* vals_out = reinterpret_cast<int32_t*>(sb + hist_bytes + 3 * key_bytes);
    void* cub_tmp = sb + hist_bytes + 4 * key_bytes;
    TB_DCUDA(d, cudaMemsetAsync(hist, 0, (size_t)nz * 8, st));
    k_z_hist<<<grid_for(n, sms), 256, 0, st>>>(coords, n, coord_stride, zr[0], (int32_t)nz, hist);
    TB_DCUDA(d, cudaGetLastError());
    std::vector<int64_t> counts((size_t)nz);
    TB_DCUDA(d, cudaMemcpyAsync(counts.data(), hist, (size_t)nz * 8, cudaMemcpyDeviceToHost, st));
    TB_DCUDA(d, cudaStreamSynchronize(st));
    std::vector<int32_t> cuts((size_t)d->world + 1);
    if (tb_zslab_cuts(counts.data(), (int32_t)nz, zr[0], d->world, cuts.data()) != TB_OK)
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_partition_zslab: fewer occupied z planes than ranks");
    const int H = d->halo;
    if (H > 1 && d->world > 1)          // every rank checks every slab, so all ranks fail alike
        for (int r = 0; r < d->world; ++r)
            if (cuts[(size_t)r + 1] - cuts[(size_t)r] < H)
                return dfail(d, TB_ERR_UNSUPPORTED, "tb_dist_partition_zslab: a slab holds fewer planes than the halo");
    auto plane = [&](int64_t z) -> int64_t { return (z >= zr[0] && z <= zr[1]) ? counts[(size_t)(z - zr[0])] : 0; };
    tb_zslab sl{};
    sl.z_lo = cuts[(size_t)d->rank];
    sl.z_hi = cuts[(size_t)d->rank + 1];
    const bool has_lo = d->rank > 0, has_hi = d->rank < d->world - 1;
    for (int k = 0; k < TB_DIST_MAX_HALO; ++k) {
        d->halo_rows_lo[k] = has_lo && k < H ? plane((int64_t)sl.z_lo - 1 - k) : 0;
        d->halo_rows_hi[k] = has_hi && k < H ? plane((int64_t)sl.z_hi + k) : 0;
    }
    const int he = std::min<int>(H, sl.z_hi - sl.z_lo);    // edge planes (a one-rank slab may be thin)
    for (int k = 0; k < H; ++k) {
        sl.n_halo_lo += d->halo_rows_lo[k];
        sl.n_halo_hi += d->halo_rows_hi[k];
    }
    for (int k = 0; k < he; ++k) {
        sl.n_edge_lo += plane((int64_t)sl.z_lo + k);
        sl.n_edge_hi += plane((int64_t)sl.z_hi - 1 - k);
    }
    d->plane_rows_lo = plane(sl.z_lo);
    d->plane_rows_hi = plane((int64_t)sl.z_hi - 1);
    sl.n_owned = 0;
    for (int64_t z = sl.z_lo; z < sl.z_hi; ++z) sl.n_owned += plane(z);
    sl.owned_begin = sl.n_halo_lo;
    sl.n_local = sl.n_halo_lo + sl.n_owned + sl.n_halo_hi;
    // 3. the local rows: every row sorted stably by its plane index (rows outside the slab last)
    const int32_t plane0 = sl.z_lo - (has_lo ? H : 0);
    const uint32_t nplanes = (uint32_t)((int64_t)sl.z_hi + (has_hi ? H : 0) - plane0);
    int end_bit = 1;
    while (end_bit < 32 && (1u << end_bit) <= nplanes) ++end_bit;
    k_slab_keys<<<grid_for(n, sms), 256, 0, st>>>(coords, n, coord_stride, plane0, nplanes, keys_in, vals_in);
    TB_DCUDA(d, cudaGetLastError());
    size_t tmp = cub_bytes;
    TB_DCUDA(d, cub::DeviceRadixSort::SortPairs(cub_tmp, tmp, keys_in, keys_out, vals_in, vals_out, (int)n, 0, end_bit,
                                                st));
    const size_t lrows = (size_t)std::max<int64_t>(sl.n_local, 1);
    s = dgrow(d, &d->rows, &d->rows_bytes, lrows * 4);
    if (s == TB_OK) s = dgrow(d, &d->coords, &d->coords_bytes, lrows * 4 * (size_t)coord_stride);
    if (s == TB_OK) s = dgrow(d, &d->nbr, &d->nbr_bytes, lrows * 108);
    if (s != TB_OK) return s;
    if (sl.n_local > 0) {
        TB_DCUDA(d, cudaMemcpyAsync(d->rows, vals_out, (size_t)sl.n_local * 4, cudaMemcpyDeviceToDevice, st));
        k_slab_coords<<<grid_for(sl.n_local, sms), 256, 0, st>>>(coords, coord_stride, (const int32_t*)d->rows,
                                                                   sl.n_local, (int32_t*)d->coords);
        TB_DCUDA(d, cudaGetLastError());
    }
    d->stride = coord_stride;
    d->slab = sl;
    d->planned = true;
    *slab = sl;
    return TB_OK;
}

tb_status tb_dist_local_rows(tb_dist* d, int32_t* rows) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!d->planned) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_local_rows: no partition yet");
    if (!rows) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_local_rows: null pointer");
    if (d->slab.n_local == 0) return TB_OK;
    TB_DCUDA(d, cudaSetDevice(d->ctx->device));
    TB_DCUDA(d, cudaMemcpyAsync(rows, d->rows, (size_t)d->slab.n_local * 4, cudaMemcpyDeviceToDevice, d->ctx->stream));
    return TB_OK;
}

tb_status tb_dist_load_coords(tb_dist* d, const int32_t* coords_local) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!d->planned) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_load_coords: no partition yet");
    if (!coords_local) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_load_coords: null pointer");
    if (d->slab.n_local == 0) return TB_OK;
    TB_DCUDA(d, cudaSetDevice(d->ctx->device));
    // the partition's relabelling, over rows already in local order
    const int64_t m = d->slab.n_local;
    k_slab_coords<<<grid_for(m, d->ctx->num_sms), 256, 0, d->ctx->stream>>>(coords_local, d->stride, nullptr, m,
                                                                             (int32_t*)d->coords);
    TB_DCUDA(d, cudaGetLastError());
    d->mapped = false;
    return TB_OK;
}

tb_status tb_dist_build_map(tb_dist* d) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!d->planned) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_build_map: no partition yet");
    if (d->slab.n_local == 0) {
        d->mapped = true;
        return TB_OK;
    }
    tb_status s = tb_build_neighbor_map(d->ctx, (const int32_t*)d->coords, d->slab.n_local, d->stride,
                                        (int32_t*)d->nbr);
    if (s != TB_OK) return dfail(d, s, std::string("tb_dist_build_map: ") + d->ctx->last_error);
    d->mapped = true;
    return TB_OK;
}

tb_status tb_dist_local_map(const tb_dist* d, const int32_t** nbr) {
    if (!d || !nbr) return TB_ERR_INVALID_ARG;
    *nbr = d->mapped ? (const int32_t*)d->nbr : nullptr;
    return d->mapped ? TB_OK : TB_ERR_INVALID_ARG;
}

tb_status tb_dist_count_valid_pairs(tb_dist* d, int64_t* pairs) {
    if (!d || !pairs) return TB_ERR_INVALID_ARG;
    if (!d->mapped) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_count_valid_pairs: no local map yet");
    *pairs = 0;
    if (d->slab.n_owned == 0) return TB_OK;
    cudaStream_t st = d->ctx->stream;
    TB_DCUDA(d, cudaSetDevice(d->ctx->device));
    tb_status s = dgrow(d, &d->scratch, &d->scratch_bytes, 256);
    if (s != TB_OK) return s;
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(d->scratch);
    TB_DCUDA(d, cudaMemsetAsync(acc, 0, 8, st));
    k_count_range<<<grid_for(27 * d->slab.n_owned, d->ctx->num_sms), 256, 0, st>>>(
        (const int32_t*)d->nbr, d->slab.n_local, d->slab.owned_begin, d->slab.n_owned, acc);
    TB_DCUDA(d, cudaGetLastError());
    unsigned long long h = 0;
    TB_DCUDA(d, cudaMemcpyAsync(&h, acc, 8, cudaMemcpyDeviceToHost, st));
    TB_DCUDA(d, cudaStreamSynchronize(st));
    *pairs = (int64_t)h;
    return TB_OK;
}

}  // extern "C"

namespace {

// The arguments of a dist conv, checked alike by tb_dist_submconv and tb_dist_submconv_grow.
tb_status dist_conv_args(tb_dist* d, const char* who, const void* feats, int ci, const void* weight,
                         const float* bias, int co, tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi,
                         const void* out) {
    const std::string w(who);
    if (!d->mapped) return dfail(d, TB_ERR_INVALID_ARG, w + ": build the local map first");
    if (!feats || !weight || !out || ci <= 0 || co <= 0)
        return dfail(d, TB_ERR_INVALID_ARG, w + ": null pointer or channels <= 0");
    if (dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16) return dfail(d, TB_ERR_INVALID_ARG, w + ": bad dtype");
    if (out_dtype != TB_F32 && out_dtype != dtype)
        return dfail(d, TB_ERR_UNSUPPORTED, w + ": out_dtype must be TB_F32 or the operand dtype");
    if (epi != TB_EPI_NONE && epi != TB_EPI_SILU) return dfail(d, TB_ERR_INVALID_ARG, w + ": bad epilogue");
    if (!tb_aligned16(feats) || !tb_aligned16(weight) || !tb_aligned16(out) || (bias && !tb_aligned16(bias)))
        return dfail(d, TB_ERR_INVALID_ARG, w + ": feats/weight/bias/out must be 16-byte aligned");
    if (feats == out) return dfail(d, TB_ERR_INVALID_ARG, w + ": out must not alias feats");
    return TB_OK;
}

// w_local = the weight with its taps in local order
tb_status dist_permute(tb_dist* d, const void* weight, int ci, int co, tb_dtype dtype, void* w_local) {
    const int64_t welems = (int64_t)co * 27 * ci;
    tb_ctx* ctx = d->ctx;
    if (tb_dtype_size(dtype) == 4)
        k_permute_taps<uint32_t><<<grid_for(welems, ctx->num_sms), 256, 0, ctx->stream>>>(
            reinterpret_cast<const uint32_t*>(weight), co, ci, reinterpret_cast<uint32_t*>(w_local));
    else
        k_permute_taps<uint16_t><<<grid_for(welems, ctx->num_sms), 256, 0, ctx->stream>>>(
            reinterpret_cast<const uint16_t*>(weight), co, ci, reinterpret_cast<uint16_t*>(w_local));
    TB_DCUDA(d, cudaGetLastError());
    return TB_OK;
}

// The halo exchange of the edge planes of f (rows of row_bytes) on the communication stream, after
// the work already on ctx's stream; ev_join marks its end and the next conv waits for it. Nothing
// moves without a communicator (the caller has filled the halo rows).
tb_status dist_exchange(tb_dist* d, uint8_t* f, size_t row_bytes) {
    const tb_zslab& sl = d->slab;
    const int64_t ob = sl.owned_begin, oe = sl.owned_begin + sl.n_owned;
    const bool lo = d->rank > 0, hi = d->rank < d->world - 1;
    const bool any = d->comm && ((lo && (sl.n_edge_lo || sl.n_halo_lo)) || (hi && (sl.n_edge_hi || sl.n_halo_hi)));
    if (!any) return TB_OK;
    NcclApi& api = nccl();
    TB_DCUDA(d, cudaEventRecord(d->ev_fork, d->ctx->stream));
    TB_DCUDA(d, cudaStreamWaitEvent(d->comm_stream, d->ev_fork, 0));
    ncclResult_t r = api.group_start();
    if (r != ncclSuccess) return dnccl(d, r, "ncclGroupStart");
    // a plane that is empty on one side is empty on the other (it is the same plane), so both
    // ranks skip the same transfers
    if (lo && sl.n_edge_lo && r == ncclSuccess)
        r = api.send(f + (size_t)ob * row_bytes, (size_t)sl.n_edge_lo * row_bytes, ncclUint8, d->rank - 1, d->comm,
                     d->comm_stream);
    if (lo && sl.n_halo_lo && r == ncclSuccess)
        r = api.recv(f, (size_t)sl.n_halo_lo * row_bytes, ncclUint8, d->rank - 1, d->comm, d->comm_stream);
    if (hi && sl.n_edge_hi && r == ncclSuccess)
        r = api.send(f + (size_t)(oe - sl.n_edge_hi) * row_bytes, (size_t)sl.n_edge_hi * row_bytes, ncclUint8,
                     d->rank + 1, d->comm, d->comm_stream);
    if (hi && sl.n_halo_hi && r == ncclSuccess)
        r = api.recv(f + (size_t)oe * row_bytes, (size_t)sl.n_halo_hi * row_bytes, ncclUint8, d->rank + 1, d->comm,
                     d->comm_stream);
    const ncclResult_t r2 = api.group_end();
    if (r != ncclSuccess) return dnccl(d, r, "ncclSend/ncclRecv");
    if (r2 != ncclSuccess) return dnccl(d, r2, "ncclGroupEnd");
    TB_DCUDA(d, cudaEventRecord(d->ev_join, d->comm_stream));
    d->exchange_pending = true;
    return TB_OK;
}

// ctx's stream waits for the exchange in flight, if any
tb_status dist_join(tb_dist* d) {
    if (!d->exchange_pending) return TB_OK;
    TB_DCUDA(d, cudaStreamWaitEvent(d->ctx->stream, d->ev_join, 0));
    d->exchange_pending = false;
    return TB_OK;
}

}  // namespace

extern "C" {

tb_status tb_dist_submconv(tb_dist* d, void* feats, int ci, const void* weight, const float* bias, int co,
                           tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
    if (!d) return TB_ERR_INVALID_ARG;
    tb_status s = dist_conv_args(d, "tb_dist_submconv", feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
    if (s != TB_OK) return s;
    const tb_zslab& sl = d->slab;
    if (sl.n_local == 0) return TB_OK;
    tb_ctx* ctx = d->ctx;
    TB_DCUDA(d, cudaSetDevice(ctx->device));
    // the weight with its taps in local order
    const size_t esz = tb_dtype_size(dtype);
    s = dgrow(d, &d->wperm, &d->wperm_bytes, (size_t)co * 27 * ci * esz);
    if (s != TB_OK) return s;
    s = dist_permute(d, weight, ci, co, dtype, d->wperm);
    if (s != TB_OK) return s;
    s = dist_join(d);                 // an earlier tb_dist_exchange may still write these rows
    if (s != TB_OK) return s;
    s = dist_exchange(d, reinterpret_cast<uint8_t*>(feats), (size_t)ci * esz);
    if (s != TB_OK) return s;
    const int64_t ob = sl.owned_begin, oe = sl.owned_begin + sl.n_owned;
    const int64_t e_lo = d->plane_rows_lo, e_hi = d->plane_rows_hi;   // the planes that read the halo
    auto conv = [&](int64_t r0, int64_t nr) -> tb_status {
        if (nr <= 0) return TB_OK;
        tb_status cs = tb_submconv_range(ctx, (const int32_t*)d->nbr, sl.n_local, r0, nr, feats, ci, d->wperm, bias,
                                         co, dtype, out_dtype, epi, out);
        return cs == TB_OK ? TB_OK : dfail(d, cs, std::string("tb_dist_submconv: ") + ctx->last_error);
    };
    // the interior planes (z_lo + 1 .. z_hi - 2) read only owned rows: they run while the halo moves
    const bool one_plane = sl.z_hi - sl.z_lo == 1;
    if (!one_plane) {
        s = conv(ob + e_lo, sl.n_owned - e_lo - e_hi);
        if (s != TB_OK) return s;
    }
    s = dist_join(d);
    if (s != TB_OK) return s;
    if (one_plane) return conv(ob, sl.n_owned);
    // the two edge planes: one launch of the pair kernel where it serves the shape
    const bool pair = dtype != TB_F32 && tb_conv_pair_supported(ci, co) &&
                      (ctx->conv_path == TB_CONV_AUTO || ctx->conv_path == TB_CONV_PAIR);
    if (pair && e_lo > 0 && e_hi > 0) {
        tb_status cs = tb_conv_pair_launch2(ctx, (const int32_t*)d->nbr, sl.n_local, ob, e_lo, oe - e_hi, e_hi, feats,
                                            ci, d->wperm, bias, co, dtype, out_dtype, epi, out);
        return cs == TB_OK ? TB_OK : dfail(d, cs, std::string("tb_dist_submconv: ") + ctx->last_error);
    }
    s = conv(ob, e_lo);
    if (s != TB_OK) return s;
    return conv(oe - e_hi, e_hi);
}

tb_status tb_dist_set_halo_planes(tb_dist* d, int planes) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (planes < 1 || planes > TB_DIST_MAX_HALO)
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_set_halo_planes: planes must be in [1, TB_DIST_MAX_HALO]");
    d->halo = planes;
    d->planned = d->mapped = false;
    return TB_OK;
}

tb_status tb_dist_exchange(tb_dist* d, void* feats, int64_t row_bytes) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!d->planned) return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_exchange: no partition yet");
    if (!feats || row_bytes <= 0 || (row_bytes & 15) || !tb_aligned16(feats))
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_exchange: null or unaligned feats, or row_bytes not a multiple of 16");
    if (d->slab.n_local == 0) return TB_OK;
    TB_DCUDA(d, cudaSetDevice(d->ctx->device));
    tb_status s = dist_join(d);
    if (s != TB_OK) return s;
    return dist_exchange(d, reinterpret_cast<uint8_t*>(feats), (size_t)row_bytes);
}

tb_status tb_dist_local_weight(tb_dist* d, const void* weight, int ci, int co, tb_dtype dtype, void* weight_local) {
    if (!d) return TB_ERR_INVALID_ARG;
    if (!weight || !weight_local || ci <= 0 || co <= 0 || weight == weight_local)
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_local_weight: null or aliasing pointers, or channels <= 0");
    if (dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16)
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_local_weight: bad dtype");
    TB_DCUDA(d, cudaSetDevice(d->ctx->device));
    return dist_permute(d, weight, ci, co, dtype, weight_local);
}

tb_status tb_dist_submconv_grow(tb_dist* d, int grow, const void* feats, int ci, const void* weight_local,
                                const float* bias, int co, tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi,
                                void* out) {
    if (!d) return TB_ERR_INVALID_ARG;
    tb_status s = dist_conv_args(d, "tb_dist_submconv_grow", feats, ci, weight_local, bias, co, dtype, out_dtype,
                                 epi, out);
    if (s != TB_OK) return s;
    if (grow < 0 || grow >= d->halo)
        return dfail(d, TB_ERR_INVALID_ARG, "tb_dist_submconv_grow: grow must be in [0, halo planes)");
    const tb_zslab& sl = d->slab;
    if (sl.n_local == 0) return TB_OK;
    tb_ctx* ctx = d->ctx;
    TB_DCUDA(d, cudaSetDevice(ctx->device));
    s = dist_join(d);
    if (s != TB_OK) return s;
    // owned rows and the `grow` nearest halo planes on each side: one contiguous local range
    int64_t r0 = sl.owned_begin, r1 = sl.owned_begin + sl.n_owned;
    for (int k = 0; k < grow; ++k) {
        r0 -= d->halo_rows_lo[k];
        r1 += d->halo_rows_hi[k];
    }
    if (r1 <= r0) return TB_OK;
    tb_status cs = tb_submconv_range(ctx, (const int32_t*)d->nbr, sl.n_local, r0, r1 - r0, feats, ci, weight_local,
                                     bias, co, dtype, out_dtype, epi, out);
    return cs == TB_OK ? TB_OK : dfail(d, cs, std::string("tb_dist_submconv_grow: ") + ctx->last_error);
}

}  // extern "C"
