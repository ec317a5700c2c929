// Dual-grid mesh extraction on the device: trellis::dual_grid_to_mesh (src/dual_grid.cpp:16-56).
//
// The reference runs on the host: a sigmoid per vertex coordinate, a std::unordered_map of
// every voxel's packed key (a later duplicate overwrites), then per voxel and edge axis whose
// intersected logit is not <= 0, four key lookups (the voxel and three neighbours at offsets in
// {0,1}^3) and a split of the quad by the products of its corners' softplus weights.
//
// Here the neighbor-map table (block layout, voxel-hash fallback: the same keys, the same
// "largest row wins") answers the seven distinct offsets the quads use as seven taps of the
// map, int32 [7][n]. Then three kernels, 256 threads and 1024 voxels per block:
//   k_mesh_count  vertices, softplus weight per voxel, each voxel's quad bits (axis a set when
//                 its logit passes and all four corners exist), per-block quad counts;
//   (scan of the block counts)
//   k_mesh_emit   each block rescans its voxels' quad counts and writes every quad's two
//                 triangles at its place in the reference's order (voxel ascending, axis x, y, z).
// The floating-point steps follow the reference's expression order with explicitly rounded
// operations (no contraction into FMAs): 1 / (1 + exp(-x)), (c + (2 s - 0.5)) * (1 / res) - 0.5,
// x > 20 ? x : log1p(exp(x)). exp and log1p are CUDA's, within 2 ulp of the host library's,
// so a vertex can differ from the reference's in the last bits and a quad whose two
// diagonal weights are within rounding of each other can take the other split.
#include "tb_common.cuh"
#include "tb_scan.cuh"

namespace {

constexpr int kMeshThreads = 256;
constexpr int kMeshPer = 4;
constexpr int kMeshPerBlock = kMeshThreads * kMeshPer;

// Corner k of the quad around the edge along axis a, as a slot of the seven-tap map
// (tb_quad_tap: 0 (0,0,0) 1 (0,0,1) 2 (0,1,0) 3 (0,1,1) 4 (1,0,0) 5 (1,0,1) 6 (1,1,0)), from the
// reference's offset table (src/dual_grid.cpp:8-12; o_voxel's edge_neighbor_voxel_offset):
//   x {000, 001, 011, 010}, y {000, 100, 101, 001}, z {000, 010, 110, 100}.
__device__ __forceinline__ int corner_slot(int a, int k) {
    constexpr int8_t t[3][4] = {{0, 1, 3, 2}, {0, 4, 5, 1}, {0, 2, 6, 4}};
    return t[a][k];
}

__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ float softplus_ref(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

struct MeshArgs {
    const int32_t* coords;
    int64_t n;
    int stride;
    const float* f7;       // [n][7]
    float inv_res;         // 1.0f / res, rounded as the reference's float division
    const int32_t* t7;     // [7][n] rows of the seven offsets, n when absent
    float* verts;          // [n][3]
    float* sp;             // [n] softplus of channel 6
    uint8_t* bits;         // [n] quad bits
    int64_t* block_sums;   // [blocks] quad counts, then their exclusive scan
    int32_t* faces;        // [max_faces][3]
    int64_t max_faces;
};

// Voxel j * kMeshThreads + t of the block is thread t's j-th voxel, so every load and store of a
// warp covers consecutive voxels.
__global__ void __launch_bounds__(kMeshThreads) k_mesh_count(const MeshArgs a) {
    const int64_t base = (int64_t)blockIdx.x * kMeshPerBlock + threadIdx.x;
    const int32_t n32 = (int32_t)a.n;
    const int off = a.stride == 4 ? 1 : 0;
    int64_t c = 0;
#pragma unroll
    for (int j = 0; j < kMeshPer; ++j) {
        const int64_t i = base + (int64_t)j * kMeshThreads;
        if (i >= a.n) break;
        float f[7];
#pragma unroll
        for (int ch = 0; ch < 7; ++ch) f[ch] = a.f7[7 * i + ch];
        const int32_t* pc = a.coords + i * a.stride + off;
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) {
            const float dv = __fsub_rn(__fmul_rn(2.0f, sigmoid_ref(f[ax])), 0.5f);
            a.verts[3 * i + ax] = __fadd_rn(__fmul_rn(__fadd_rn((float)pc[ax], dv), a.inv_res), -0.5f);
        }
        a.sp[i] = softplus_ref(f[6]);
        uint32_t b = 0;
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) {
            if (f[3 + ax] <= 0.0f) continue;                 // a NaN logit passes, as in the reference
            bool ok = true;
#pragma unroll
            for (int k = 0; k < 4; ++k) ok = ok && a.t7[(int64_t)corner_slot(ax, k) * a.n + i] != n32;
            if (ok) b |= 1u << ax;
        }
        a.bits[i] = (uint8_t)b;
        c += __popc(b);
    }
    int64_t total;
    tb_scan::block_exclusive_scan<kMeshThreads>(c, &total);
    if (threadIdx.x == 0) a.block_sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kMeshThreads) k_mesh_emit(const MeshArgs a) {
    const int64_t base = (int64_t)blockIdx.x * kMeshPerBlock + threadIdx.x;
    int64_t carry = a.block_sums[blockIdx.x];
#pragma unroll 1
    for (int j = 0; j < kMeshPer; ++j) {
        // the block's voxels in order: row j of the block after rows 0..j-1
        const int64_t i = base + (int64_t)j * kMeshThreads;
        const uint32_t bits = i < a.n ? a.bits[i] : 0u;
        int64_t total;
        int64_t quad = tb_scan::block_exclusive_scan<kMeshThreads>(__popc(bits), &total) + carry;
        carry += total;
#pragma unroll
        for (int ax = 0; ax < 3; ++ax) {
            if (!((bits >> ax) & 1u)) continue;
            if (2 * quad + 2 <= a.max_faces) {
                int32_t q[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) q[k] = a.t7[(int64_t)corner_slot(ax, k) * a.n + i];
                const float w02 = __fmul_rn(a.sp[q[0]], a.sp[q[2]]);
                const float w13 = __fmul_rn(a.sp[q[1]], a.sp[q[3]]);
                int2* d = reinterpret_cast<int2*>(a.faces + 6 * quad);
                if (w02 > w13) {        // {q0,q1,q2, q0,q2,q3}
                    d[0] = make_int2(q[0], q[1]);
                    d[1] = make_int2(q[2], q[0]);
                    d[2] = make_int2(q[2], q[3]);
                } else {                // {q0,q1,q3, q3,q1,q2}
                    d[0] = make_int2(q[0], q[1]);
                    d[1] = make_int2(q[3], q[3]);
                    d[2] = make_int2(q[1], q[2]);
                }
            }
            ++quad;
        }
    }
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

extern "C" tb_status tb_dual_grid_mesh(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                                       const float* feats7, int res, float* verts, int32_t* faces,
                                       int64_t max_faces, int64_t* f_out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (!f_out || n < 0 || max_faces < 0 || res <= 0 || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_dual_grid_mesh: bad arguments");
    *f_out = 0;
    if (n == 0) return TB_OK;
    if (!coords || !feats7 || !verts || (max_faces > 0 && !faces))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_dual_grid_mesh: null pointer");
    if ((reinterpret_cast<uintptr_t>(faces) & 7) != 0)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_dual_grid_mesh: faces must be 8-byte aligned");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_dual_grid_mesh: n must be < 2^31-1");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int64_t nb = (n + kMeshPerBlock - 1) / kMeshPerBlock;
    const size_t nbr_b = align256(tb_nbr_workspace_bytes(n)), t7_b = align256((size_t)n * 7 * sizeof(int32_t));
    const size_t sp_b = align256((size_t)n * sizeof(float)), bits_b = align256((size_t)n);
    const size_t sums_b = sizeof(int64_t) * (size_t)(nb + 2);
    tb_status s = tb_ensure(ctx, &ctx->ws, &ctx->ws_bytes, nbr_b + t7_b + sp_b + bits_b + sums_b, "mesh workspace");
    if (s != TB_OK) return s;
    uint8_t* w = reinterpret_cast<uint8_t*>(ctx->ws);
    int32_t* t7 = reinterpret_cast<int32_t*>(w + nbr_b);
    MeshArgs a{};
    a.coords = coords;
    a.n = n;
    a.stride = coord_stride;
    a.f7 = feats7;
    a.inv_res = 1.0f / (float)res;
    a.t7 = t7;
    a.verts = verts;
    a.sp = reinterpret_cast<float*>(w + nbr_b + t7_b);
    a.bits = w + nbr_b + t7_b + sp_b;
    a.block_sums = reinterpret_cast<int64_t*>(w + nbr_b + t7_b + sp_b + bits_b);
    int64_t* grand = a.block_sums + nb;
    a.faces = faces;
    a.max_faces = max_faces;
    s = tb_nbr_build_quad_taps(ctx, coords, n, coord_stride, t7, w);
    if (s != TB_OK) return s;
    k_mesh_count<<<(unsigned)nb, kMeshThreads, 0, ctx->stream>>>(a);
    TB_LAUNCH_CHECK(ctx, "k_mesh_count");
    tb_scan::k_scan_block_totals<kMeshThreads, kMeshPer><<<1, kMeshThreads, 0, ctx->stream>>>(a.block_sums, nb, grand);
    TB_LAUNCH_CHECK(ctx, "k_scan_block_totals");
    k_mesh_emit<<<(unsigned)nb, kMeshThreads, 0, ctx->stream>>>(a);
    TB_LAUNCH_CHECK(ctx, "k_mesh_emit");
    int64_t quads = 0;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(&quads, grand, sizeof(quads), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    *f_out = 2 * quads;
    if (2 * quads > max_faces)
        return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_dual_grid_mesh: more triangles than max_faces (F written to f_out)");
    return TB_OK;
}
