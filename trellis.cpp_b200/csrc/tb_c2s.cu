// SparseResBlockC2S3d on the device: trellis::sparse_c2s (src/sparse.cpp:172-336) as one call.
//
// The reference runs the to_subdiv logits as a graph, the octant loop and both neighbor tables on
// the host, then a second graph for norm1 / conv1 / channel-to-spatial / norm2 / conv2 + skip,
// with host<->device copies around each. Here every step runs on the device in one stream; the
// host reads back only the child count M (to size the second half):
//   1. mask = (to_subdiv(x) > 0), [8N] (src/sparse.cpp:184-190,215), or the caller's mask;
//   2. children, gidx = o + 8i in the reference's order (tb_subdivide, src/sparse.cpp:205-222);
//   3. h = SiLU(LayerNorm(x) * norm1.weight + norm1.bias), eps 1e-6 (src/sparse.cpp:259-261);
//   4. h1 = conv1(h) at 8 * Cout output channels, fp32 (src/sparse.cpp:279-286);
//   5. hn[m] = SiLU(LayerNorm(h1 viewed [8N][Cout], row gidx[m])), no affine: the
//      channel-to-spatial gather fused with norm2 (src/sparse.cpp:288,293);
//   6. o = conv2(hn) on the children's neighbor map, fp32 (src/sparse.cpp:224,316-319);
//   7. out[m][k R + r] = o[m][k R + r] + x viewed [8N][K], row gidx[m], element k, with
//      K = Cin / 8 and R = Cout / K: the skip's gather and repeat_interleave (src/sparse.cpp:307,
//      322-323).
// The reference chunks conv1 and conv2 over voxels to bound its host-side graph memory
// (src/sparse.cpp:234-246,309-314); one device pass over each needs no chunking.
#include "tb_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <climits>

namespace {

// element kinds: 0 f32, 1 f16, 2 bf16
template <int KIND>
__device__ __forceinline__ void load8(const void* base, int64_t elem, float* v) {
    if constexpr (KIND == 0) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + elem);
        const float4 a = p[0], b = p[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + elem);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (KIND == 2) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            } else {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                v[2 * i] = f.x, v[2 * i + 1] = f.y;
            }
        }
    }
}

template <int KIND>
__device__ __forceinline__ void store8(void* base, int64_t elem, const float* v) {
    if constexpr (KIND == 0) {
        float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + elem);
        p[0] = make_float4(v[0], v[1], v[2], v[3]);
        p[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (KIND == 2) {
                __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + elem) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

template <int KIND>
__device__ __forceinline__ float load1(const void* base, int64_t elem) {
    if constexpr (KIND == 0) return reinterpret_cast<const float*>(base)[elem];
    const uint16_t u = reinterpret_cast<const uint16_t*>(base)[elem];
    if constexpr (KIND == 2) return __uint_as_float((uint32_t)u << 16);
    else return __half2float(__ushort_as_half(u));
}

constexpr int kWarpsPerBlock = 8;

// to_subdiv: logits[i][o] = b[o] + sum_c W[o][c] x[i][c] in fp32 (a fixed order: lane-strided
// 8-channel chunks, then a butterfly over the lanes), mask[8 i + o] = logits > 0. One warp per
// voxel, W staged in shared memory ([8][cin] floats).
template <int XK>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_to_subdiv(const void* __restrict__ x, int64_t n, int cin, const float* __restrict__ w,
            const float* __restrict__ b, uint8_t* __restrict__ mask) {
    extern __shared__ float s_w[];                 // [8][cin]
    for (int i = threadIdx.x; i < 8 * cin; i += blockDim.x) s_w[i] = w[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int nchunk = cin / 8;
    for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < n;
         row += (int64_t)gridDim.x * kWarpsPerBlock) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = lane; k < nchunk; k += 32) {
            float v[8];
            load8<XK>(x, row * cin + 8 * k, v);
#pragma unroll
            for (int o = 0; o < 8; ++o) {
                const float* wr = s_w + o * cin + 8 * k;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[o] = fmaf(wr[e], v[e], acc[o]);
            }
        }
#pragma unroll
        for (int o = 0; o < 8; ++o)
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) acc[o] += __shfl_xor_sync(0xffffffffu, acc[o], s);
        if (lane == 0) {
            uint64_t bits = 0;
#pragma unroll
            for (int o = 0; o < 8; ++o) bits |= (uint64_t)((acc[o] + (b ? b[o] : 0.f)) > 0.f) << (8 * o);
            reinterpret_cast<uint64_t*>(mask)[row] = bits;
        }
    }
}

// Row LayerNorm (eps given: 1e-6 in the blocks, 1e-5 before decode_unet's output layer) over c channels, optional affine, optional SiLU; one warp per output
// row. Output row r reads source row rows[r] (rows == nullptr: row r). Lane l owns the 8-channel
// chunks l, l + 32, ... (NCH of them at most, c <= 256 NCH).
template <int IK, int OK, int NCH>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_row_norm(const void* __restrict__ src, const int32_t* __restrict__ rows, int64_t n, int c,
           const float* __restrict__ w, const float* __restrict__ b, int silu, float eps, void* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int nchunk = c / 8;
    for (int64_t r = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); r < n;
         r += (int64_t)gridDim.x * kWarpsPerBlock) {
        const int64_t sr = rows ? (int64_t)rows[r] : r;
        float v[NCH][8];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const int k = lane + 32 * j;
            if (k < nchunk) {
                load8<IK>(src, sr * c + 8 * k, v[j]);
#pragma unroll
                for (int e = 0; e < 8; ++e) sum += v[j][e];
            }
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
        const float mean = sum / (float)c;
        float s2 = 0.f;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            if (lane + 32 * j < nchunk) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float d = v[j][e] - mean;
                    s2 = fmaf(d, d, s2);
                }
            }
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, s);
        const float rstd = rsqrtf(s2 / (float)c + eps);
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
            const int k = lane + 32 * j;
            if (k < nchunk) {
                float y[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float t = (v[j][e] - mean) * rstd;
                    if (w) t = t * w[8 * k + e] + b[8 * k + e];
                    y[e] = silu ? tb_silu(t) : t;
                }
                store8<OK>(out, r * c + 8 * k, y);
            }
        }
    }
}

// out[m][ch] = o[m][ch] + x_flat[gidx[m] * K + ch / R]: the skip of src/sparse.cpp:307,322-323
// (x viewed [8N][K], gathered by gidx, each of its K values repeated R times). One thread per 8
// output channels.
// With `orow` (a permutation), row m of o is stored as output row orow[m].
template <int XK, int OK>
__global__ void __launch_bounds__(256)
k_c2s_skip(const float* __restrict__ o, const void* __restrict__ x, const int32_t* __restrict__ gidx,
           const int32_t* __restrict__ orow, int64_t m, int cout, int k, int r, void* __restrict__ out) {
    const int per_row = cout / 8;
    const int64_t total = m * per_row;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / per_row;
        const int c0 = (int)(t - row * per_row) * 8;
        const int64_t xb = (int64_t)gidx[row] * k;
        float v[8];
        load8<0>(o, row * cout + c0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += load1<XK>(x, xb + (c0 + e) / r);
        store8<OK>(out, (orow ? (int64_t)orow[row] : row) * cout + c0, v);
    }
}

// Bounds of the children's coordinates: mm = {min b, min x, min y, min z, max b, max x, max y, max z}
// (b = 0 for stride 3), for the compact sort key.
__global__ void k_coord_bounds(const int32_t* __restrict__ c, int64_t m, int stride, int* __restrict__ mm) {
    int lo[4] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX}, hi[4] = {INT_MIN, INT_MIN, INT_MIN, INT_MIN};
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int v = a < 4 - stride ? 0 : c[i * stride + a - (4 - stride)];
            lo[a] = min(lo[a], v);
            hi[a] = max(hi[a], v);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        lo[a] = __reduce_min_sync(0xffffffffu, lo[a]);
        hi[a] = __reduce_max_sync(0xffffffffu, hi[a]);
    }
    if ((threadIdx.x & 31) == 0)
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            atomicMin(mm + a, lo[a]);
            atomicMax(mm + 4 + a, hi[a]);
        }
}

// key of child i = (b, x, y, z) relative to the minima, packed in sh[a]-shifted fields (the
// reference's key order, src/sparse.cpp:25); val = i
__global__ void k_child_keys(const int32_t* __restrict__ c, int64_t m, int stride, const int* __restrict__ mm,
                             int sb, int sx, int sy, unsigned long long* __restrict__ keys, int32_t* __restrict__ vals) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t* p = c + i * stride;
        const int o = stride - 3;
        const unsigned long long b = o ? (unsigned long long)(uint32_t)(p[0] - mm[0]) : 0ull;
        keys[i] = (b << sb) | ((unsigned long long)(uint32_t)(p[o] - mm[1]) << sx) |
                  ((unsigned long long)(uint32_t)(p[o + 1] - mm[2]) << sy) | (unsigned long long)(uint32_t)(p[o + 2] - mm[3]);
        vals[i] = (int32_t)i;
    }
}

__global__ void k_iota(int32_t* __restrict__ v, int64_t m) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        v[i] = (int32_t)i;
}

int kind_of(tb_dtype d) { return d == TB_F32 ? 0 : (d == TB_F16 ? 1 : 2); }

int grid_for(tb_ctx* ctx, int64_t work, int per_block) {
    const int64_t want = (work + per_block - 1) / per_block;
    return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)ctx->num_sms * 16));
}

template <int IK, int OK>
tb_status launch_row_norm_k(tb_ctx* ctx, const void* src, const int32_t* rows, int64_t n, int c, const float* w,
                            const float* b, int silu, float eps, void* out) {
    const int grid = grid_for(ctx, n, kWarpsPerBlock);
    const int nch = (c / 8 + 31) / 32;
    const dim3 blk(kWarpsPerBlock * 32);
    if (nch <= 1) k_row_norm<IK, OK, 1><<<grid, blk, 0, ctx->stream>>>(src, rows, n, c, w, b, silu, eps, out);
    else if (nch <= 2) k_row_norm<IK, OK, 2><<<grid, blk, 0, ctx->stream>>>(src, rows, n, c, w, b, silu, eps, out);
    else if (nch <= 4) k_row_norm<IK, OK, 4><<<grid, blk, 0, ctx->stream>>>(src, rows, n, c, w, b, silu, eps, out);
    else k_row_norm<IK, OK, 8><<<grid, blk, 0, ctx->stream>>>(src, rows, n, c, w, b, silu, eps, out);
    TB_LAUNCH_CHECK(ctx, "k_row_norm");
    return TB_OK;
}

}  // namespace

// Row LayerNorm + optional affine + optional SiLU (c % 8 == 0, c <= 2048): the ggml_norm /
// ggml_mul / ggml_add / ggml_silu chains of src/sparse.cpp:259-261,293. in_dtype is the source's
// element type; out has `out_dtype`.
tb_status tb_row_norm_launch(tb_ctx* ctx, const void* src, tb_dtype in_dtype, const int32_t* rows, int64_t n, int c,
                             const float* w, const float* b, int silu, tb_dtype out_dtype, void* out, float eps) {
    if (n == 0) return TB_OK;
    const int ik = kind_of(in_dtype), ok = kind_of(out_dtype);
    if (ik == 0 && ok == 0) return launch_row_norm_k<0, 0>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 0 && ok == 1) return launch_row_norm_k<0, 1>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 0 && ok == 2) return launch_row_norm_k<0, 2>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 1 && ok == 1) return launch_row_norm_k<1, 1>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 2 && ok == 2) return launch_row_norm_k<2, 2>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 1 && ok == 0) return launch_row_norm_k<1, 0>(ctx, src, rows, n, c, w, b, silu, eps, out);
    if (ik == 2 && ok == 0) return launch_row_norm_k<2, 0>(ctx, src, rows, n, c, w, b, silu, eps, out);
    return tb_fail(ctx, TB_ERR_UNSUPPORTED, "row norm: unsupported dtype pair");
}

tb_status tb_to_subdiv_launch(tb_ctx* ctx, const void* x, tb_dtype dtype, int64_t n, int cin, const float* w,
                              const float* b, uint8_t* mask) {
    if (n == 0) return TB_OK;
    const size_t smem = (size_t)8 * cin * sizeof(float);
    if (smem > (size_t)ctx->max_smem_optin) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "to_subdiv: cin too large");
    const int grid = grid_for(ctx, n, kWarpsPerBlock);
    const int k = kind_of(dtype);
    cudaError_t e = cudaSuccess;
    if (smem > 48 * 1024) {
        if (k == 0) e = cudaFuncSetAttribute(k_to_subdiv<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        else if (k == 1) e = cudaFuncSetAttribute(k_to_subdiv<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        else e = cudaFuncSetAttribute(k_to_subdiv<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_to_subdiv)");
    }
    if (k == 0) k_to_subdiv<0><<<grid, kWarpsPerBlock * 32, smem, ctx->stream>>>(x, n, cin, w, b, mask);
    else if (k == 1) k_to_subdiv<1><<<grid, kWarpsPerBlock * 32, smem, ctx->stream>>>(x, n, cin, w, b, mask);
    else k_to_subdiv<2><<<grid, kWarpsPerBlock * 32, smem, ctx->stream>>>(x, n, cin, w, b, mask);
    TB_LAUNCH_CHECK(ctx, "k_to_subdiv");
    return TB_OK;
}

tb_status tb_c2s_skip_launch(tb_ctx* ctx, const float* o, const void* x, tb_dtype x_dtype, const int32_t* gidx,
                             const int32_t* orow, int64_t m, int cin, int cout, tb_dtype out_dtype, void* out) {
    if (m == 0) return TB_OK;
    const int k = cin / 8, r = cout / k;
    const int grid = grid_for(ctx, m * (cout / 8), 256);
    const int xk = kind_of(x_dtype), ok = kind_of(out_dtype);
    if (xk == 0 && ok == 0) k_c2s_skip<0, 0><<<grid, 256, 0, ctx->stream>>>(o, x, gidx, orow, m, cout, k, r, out);
    else if (xk == 1 && ok == 0) k_c2s_skip<1, 0><<<grid, 256, 0, ctx->stream>>>(o, x, gidx, orow, m, cout, k, r, out);
    else if (xk == 2 && ok == 0) k_c2s_skip<2, 0><<<grid, 256, 0, ctx->stream>>>(o, x, gidx, orow, m, cout, k, r, out);
    else if (xk == 1 && ok == 1) k_c2s_skip<1, 1><<<grid, 256, 0, ctx->stream>>>(o, x, gidx, orow, m, cout, k, r, out);
    else if (xk == 2 && ok == 2) k_c2s_skip<2, 2><<<grid, 256, 0, ctx->stream>>>(o, x, gidx, orow, m, cout, k, r, out);
    else return tb_fail(ctx, TB_ERR_UNSUPPORTED, "c2s skip: unsupported dtype pair");
    TB_LAUNCH_CHECK(ctx, "k_c2s_skip");
    return TB_OK;
}

extern "C" tb_status tb_sparse_c2s(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                                   const void* feats, int cin, int cout, const tb_c2s_params* prm,
                                   const uint8_t* ext_mask, tb_dtype dtype, tb_dtype out_dtype,
                                   int64_t max_children, int32_t* child_coords, void* out, uint8_t* mask_out,
                                   int64_t* m_out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (!m_out || !prm) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: null m_out or params");
    *m_out = 0;
    if (n < 0 || cin <= 0 || cout <= 0 || max_children < 0 || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: bad sizes or coord_stride");
    if (cin % 8 != 0 || cout % (cin / 8) != 0 || cout % 8 != 0 || cin > 2048 || cout > 2048)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                       "tb_sparse_c2s: needs cin % 8 == 0, cout a multiple of cin/8 and of 8, cin, cout <= 2048");
    if (dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: bad dtype");
    if (out_dtype != TB_F32 && out_dtype != dtype)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_sparse_c2s: out_dtype must be TB_F32 or the operand dtype");
    if (!ext_mask && (!prm->to_subdiv_w))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: to_subdiv weight needed without an external mask");
    if (!prm->norm1_w || !prm->norm1_b || !prm->conv1_w || !prm->conv2_w)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: null parameter");
    if (n == 0) return TB_OK;
    if (!coords || !feats || !child_coords || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: null pointer");
    if (!tb_aligned16(feats) || !tb_aligned16(out) || !tb_aligned16(prm->conv1_w) || !tb_aligned16(prm->conv2_w))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_c2s: feats/out/conv weights must be 16-byte aligned");
    if (n >= (int64_t)INT32_MAX / 8) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_sparse_c2s: 8n must be < 2^31-1");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const size_t es = tb_dtype_size(dtype);
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    // ---- first half: everything sized by n
    const size_t nbr_b = al((size_t)n * 27 * 4), mask_b = al((size_t)n * 8), h_b = al((size_t)n * cin * es),
                 h1_b = al((size_t)n * 8 * cout * 4), gidx_b = al((size_t)std::max<int64_t>(max_children, 1) * 4);
    tb_status s = tb_ensure(ctx, &ctx->c2s_ws1, &ctx->c2s_ws1_bytes, nbr_b + mask_b + h_b + h1_b + gidx_b, "c2s workspace");
    if (s != TB_OK) return s;
    uint8_t* base = reinterpret_cast<uint8_t*>(ctx->c2s_ws1);
    int32_t* nbr = reinterpret_cast<int32_t*>(base);
    uint8_t* mask = base + nbr_b;
    void* h = base + nbr_b + mask_b;
    float* h1 = reinterpret_cast<float*>(base + nbr_b + mask_b + h_b);
    int32_t* gidx = reinterpret_cast<int32_t*>(base + nbr_b + mask_b + h_b + h1_b);

    const uint8_t* use_mask = ext_mask;
    if (!ext_mask) {
        s = tb_to_subdiv_launch(ctx, feats, dtype, n, cin, prm->to_subdiv_w, prm->to_subdiv_b, mask);
        if (s != TB_OK) return s;
        use_mask = mask;
    }
    if (mask_out && mask_out != use_mask)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(mask_out, use_mask, (size_t)n * 8, cudaMemcpyDeviceToDevice, ctx->stream));
    // conv1 on the parents (independent of the mask), queued before the subdivide's read-back
    s = tb_build_neighbor_map(ctx, coords, n, coord_stride, nbr);
    if (s != TB_OK) return s;
    s = tb_row_norm_launch(ctx, feats, dtype, nullptr, n, cin, prm->norm1_w, prm->norm1_b, 1, dtype, h);
    if (s != TB_OK) return s;
    s = tb_submconv(ctx, nbr, n, h, cin, prm->conv1_w, prm->conv1_b, 8 * cout, dtype, TB_F32, TB_EPI_NONE, h1);
    if (s != TB_OK) return s;
    int64_t m = 0;
    s = tb_subdivide(ctx, coords, n, coord_stride, use_mask, child_coords, gidx, nullptr, max_children, &m);
    *m_out = m;
    if (s != TB_OK) return s;
    if (m == 0) return TB_OK;
    // ---- second half: sized by m
    // The children come parent-major (the reference's order, which the outputs keep), so a
    // 128-row tile's neighbours are spread over distant rows and the range-staged conv kernels
    // run about 2x slower on them. The child half therefore works on the children sorted by the
    // reference's key (a stable device radix sort on a compact key; one small read-back of the
    // coordinate bounds): the map and conv2 see sorted rows, norm2 reads gidx in that order, and
    // the skip kernel writes each row back to its place in the reference's order.
    const size_t nbr2_b = al((size_t)m * 27 * 4), hn_b = al((size_t)m * cout * es), o_b = al((size_t)m * cout * 4);
    const size_t key_b = al((size_t)m * 8), val_b = al((size_t)m * 4), cs_b = al((size_t)m * coord_stride * 4);
    size_t cub_b = 0;
    TB_CUDA_TRY(ctx, cub::DeviceRadixSort::SortPairs(nullptr, cub_b, (const unsigned long long*)nullptr,
                                                     (unsigned long long*)nullptr, (const int32_t*)nullptr,
                                                     (int32_t*)nullptr, (int)m, 0, 64, ctx->stream));
    cub_b = al(cub_b);
    s = tb_ensure(ctx, &ctx->c2s_ws2, &ctx->c2s_ws2_bytes,
                  nbr2_b + hn_b + o_b + 2 * key_b + 3 * val_b + cs_b + cub_b + 256, "c2s child workspace");
    if (s != TB_OK) return s;
    uint8_t* b2 = reinterpret_cast<uint8_t*>(ctx->c2s_ws2);
    int32_t* nbr2 = reinterpret_cast<int32_t*>(b2);
    void* hn = b2 + nbr2_b;
    float* o = reinterpret_cast<float*>(b2 + nbr2_b + hn_b);
    uint8_t* p2 = b2 + nbr2_b + hn_b + o_b;
    auto* keys_in = reinterpret_cast<unsigned long long*>(p2);
    auto* keys_out = reinterpret_cast<unsigned long long*>(p2 + key_b);
    int32_t* iota = reinterpret_cast<int32_t*>(p2 + 2 * key_b);
    int32_t* perm = reinterpret_cast<int32_t*>(p2 + 2 * key_b + val_b);
    int32_t* gidx_s = reinterpret_cast<int32_t*>(p2 + 2 * key_b + 2 * val_b);
    int32_t* child_s = reinterpret_cast<int32_t*>(p2 + 2 * key_b + 3 * val_b);
    void* cub_tmp = p2 + 2 * key_b + 3 * val_b + cs_b;
    int* mm = reinterpret_cast<int*>(p2 + 2 * key_b + 3 * val_b + cs_b + cub_b);
    static const int mm0[8] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX, INT_MIN, INT_MIN, INT_MIN, INT_MIN};
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(mm, mm0, sizeof(mm0), cudaMemcpyHostToDevice, ctx->stream));
    k_coord_bounds<<<grid_for(ctx, m, 256), 256, 0, ctx->stream>>>(child_coords, m, coord_stride, mm);
    TB_LAUNCH_CHECK(ctx, "k_coord_bounds");
    int bh[8];
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(bh, mm, sizeof(bh), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    auto bits = [](int lo, int hi) {
        const uint64_t span = (uint64_t)((int64_t)hi - lo);
        int k = 0;
        while (k < 33 && (span >> k) != 0) ++k;
        return k;
    };
    const int bz = bits(bh[3], bh[7]), by = bits(bh[2], bh[6]), bx = bits(bh[1], bh[5]), bb = bits(bh[0], bh[4]);
    const int total_bits = bb + bx + by + bz;
    const bool sorted_path = total_bits <= 64;
    const int32_t* cmap_coords = child_coords;
    const int32_t* gsel = gidx;
    const int32_t* orow = nullptr;
    if (sorted_path) {
        k_child_keys<<<grid_for(ctx, m, 256), 256, 0, ctx->stream>>>(child_coords, m, coord_stride, mm, bx + by + bz,
                                                                    by + bz, bz, keys_in, iota);
        TB_LAUNCH_CHECK(ctx, "k_child_keys");
        size_t tmp = cub_b;
        TB_CUDA_TRY(ctx, cub::DeviceRadixSort::SortPairs(cub_tmp, tmp, keys_in, keys_out, iota, perm, (int)m, 0,
                                                         std::max(1, total_bits), ctx->stream));
        s = tb_gather_rows(ctx, child_coords, perm, m, (int64_t)coord_stride * 4, child_s);
        if (s != TB_OK) return s;
        s = tb_gather_rows(ctx, gidx, perm, m, 4, gidx_s);
        if (s != TB_OK) return s;
        cmap_coords = child_s;
        gsel = gidx_s;
        orow = perm;
    }
    s = tb_row_norm_launch(ctx, h1, TB_F32, gsel, m, cout, nullptr, nullptr, 1, dtype, hn);
    if (s != TB_OK) return s;
    s = tb_build_neighbor_map(ctx, cmap_coords, m, coord_stride, nbr2);
    if (s != TB_OK) return s;
    s = tb_submconv(ctx, nbr2, m, hn, cout, prm->conv2_w, prm->conv2_b, cout, dtype, TB_F32, TB_EPI_NONE, o);
    if (s != TB_OK) return s;
    return tb_c2s_skip_launch(ctx, o, feats, dtype, gsel, orow, m, cin, cout, out_dtype, out);
}

// Stable order of rows by their signed (b, x, y, z) coordinates (for non-negative ones the
// reference's key order, src/sparse.cpp:25): the coordinate
// bounds (one small read-back), a compact key of the rows' offsets from the minima, and a stable
// device radix sort of (key, row). Rows whose key span needs more than 63 bits keep their order.
extern "C" tb_status tb_sort_rows(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride, int32_t* perm) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sort_rows: bad n or coord_stride");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_sort_rows: n must be < 2^31-1");
    if (n == 0) return TB_OK;
    if (!coords || !perm) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sort_rows: null pointer");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    size_t cub_b = 0;
    TB_CUDA_TRY(ctx, cub::DeviceRadixSort::SortPairs(nullptr, cub_b, (const unsigned long long*)nullptr,
                                                     (unsigned long long*)nullptr, (const int32_t*)nullptr,
                                                     (int32_t*)nullptr, (int)n, 0, 64, ctx->stream));
    const size_t key_b = al((size_t)n * 8), val_b = al((size_t)n * 4);
    cub_b = al(cub_b);
    tb_status s = tb_ensure(ctx, &ctx->sort_ws, &ctx->sort_ws_bytes, 2 * key_b + val_b + cub_b + 256, "sort workspace");
    if (s != TB_OK) return s;
    uint8_t* b = reinterpret_cast<uint8_t*>(ctx->sort_ws);
    auto* keys_in = reinterpret_cast<unsigned long long*>(b);
    auto* keys_out = reinterpret_cast<unsigned long long*>(b + key_b);
    int32_t* rows = reinterpret_cast<int32_t*>(b + 2 * key_b);
    void* cub_tmp = b + 2 * key_b + val_b;
    int* mm = reinterpret_cast<int*>(b + 2 * key_b + val_b + cub_b);
    static const int mm0[8] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX, INT_MIN, INT_MIN, INT_MIN, INT_MIN};
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(mm, mm0, sizeof(mm0), cudaMemcpyHostToDevice, ctx->stream));
    k_coord_bounds<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(coords, n, coord_stride, mm);
    TB_LAUNCH_CHECK(ctx, "k_coord_bounds");
    int bh[8];
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(bh, mm, sizeof(bh), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    auto bits = [](int lo, int hi) {
        const uint64_t span = (uint64_t)((int64_t)hi - lo);
        int k = 0;
        while (k < 33 && (span >> k) != 0) ++k;
        return k;
    };
    const int bz = bits(bh[3], bh[7]), by = bits(bh[2], bh[6]), bx = bits(bh[1], bh[5]), bb = bits(bh[0], bh[4]);
    const int total_bits = bb + bx + by + bz;
    if (total_bits > 63) {
        k_iota<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(perm, n);
        TB_LAUNCH_CHECK(ctx, "k_iota");
        return TB_OK;
    }
    k_child_keys<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(coords, n, coord_stride, mm, bx + by + bz, by + bz, bz,
                                                                 keys_in, rows);
    TB_LAUNCH_CHECK(ctx, "k_child_keys");
    size_t tmp = cub_b;
    TB_CUDA_TRY(ctx, cub::DeviceRadixSort::SortPairs(cub_tmp, tmp, keys_in, keys_out, rows, perm, (int)n, 0,
                                                     std::max(1, total_bits), ctx->stream));
    return TB_OK;
}
