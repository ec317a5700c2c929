// Shared host/device helpers of the sparse-conv library: the context, status plumbing,
// workspace growth and the 64-bit coordinate key of the reference (src/sparse.cpp:25).
#pragma once

#include <cuda_runtime.h>
#include <cuda.h>
#include <stdint.h>
#include <string>

#include "tb_sparse.h"

// Device-side error codes written to tb_ctx::d_err (first failure wins).
enum tb_device_error : int {
    TB_DEVERR_NONE = 0,
    TB_DEVERR_HASH_PROBE = 1,     // hash insert/lookup exceeded its probe bound
    TB_DEVERR_WAIT_TIMEOUT = 2,   // a bounded mbarrier wait in the conv kernel ran out
    TB_DEVERR_TMEM_ALLOC = 3,     // TMEM allocation returned an unusable address
};

struct tb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    int max_smem_optin = 0;
    int* d_err = nullptr;          // one int on the device
    void* ws = nullptr;            // hash table / scratch
    size_t ws_bytes = 0;
    void* host_stage = nullptr;    // device buffers of the *_host calls
    size_t host_stage_bytes = 0;
    std::string last_error;
    void* encode_tiled = nullptr;  // cuTensorMapEncodeTiled, fetched once
    int conv_path = 0;             // tb_conv_path
    // dynamic shared memory already allowed per conv kernel on this device: the attribute is set
    // only when a launch needs more, so repeated launches (and launches recorded into a CUDA
    // graph) make no function-attribute call
    size_t pair_smem_set[2] = {0, 0};   // the pair kernel's Ci = 64 and Ci = 32 instances
    size_t brick_smem_set = 0;
    size_t brick_pair_smem_set = 0;
    void* block_h = nullptr;       // fp32 conv output of tb_sparse_convnext
    size_t block_h_bytes = 0;
    void* c2s_ws1 = nullptr;       // tb_sparse_c2s: parent map, mask, norm1 output, conv1 output, gidx
    size_t c2s_ws1_bytes = 0;
    void* c2s_ws2 = nullptr;       // tb_sparse_c2s: child map, norm2 output, conv2 output
    size_t c2s_ws2_bytes = 0;
    // tb_submconv_stack_host's pipeline: copy streams, chunk events, pinned chunk bounds
    cudaStream_t copy_in = nullptr;
    cudaStream_t copy_out = nullptr;
    cudaEvent_t stage_ev[2 + 2 * 32] = {};
    bool stage_ev_made = false;
    int32_t* chunk_hi_host = nullptr;
    void* tail_ws = nullptr;       // ConvNeXt tail passes at wide C: LayerNorm output, activations
    size_t tail_ws_bytes = 0;
    void* sort_ws = nullptr;       // tb_sort_rows: keys, values, radix-sort scratch, coordinate bounds
    size_t sort_ws_bytes = 0;
};

// Record a failure on the context and return the status.
tb_status tb_fail(tb_ctx* ctx, tb_status s, const std::string& msg);
tb_status tb_cuda_fail(tb_ctx* ctx, cudaError_t e, const char* what);
// Grow a context-owned device buffer to at least `bytes` (never shrinks).
tb_status tb_ensure(tb_ctx* ctx, void** buf, size_t* cap, size_t bytes, const char* what);

#define TB_CUDA_TRY(ctx, call)                                          \
    do {                                                                \
        cudaError_t e_ = (call);                                        \
        if (e_ != cudaSuccess) return tb_cuda_fail((ctx), e_, #call);   \
    } while (0)

#define TB_LAUNCH_CHECK(ctx, what)                                      \
    do {                                                                \
        cudaError_t e_ = cudaGetLastError();                            \
        if (e_ != cudaSuccess) return tb_cuda_fail((ctx), e_, what);    \
    } while (0)

// ---- the packed key (src/sparse.cpp:25), with the batch folded into bits 60..63 ----------
__host__ __device__ __forceinline__ uint64_t tb_key3(int32_t x, int32_t y, int32_t z) {
    return ((uint64_t)(uint32_t)x << 40) | ((uint64_t)(uint32_t)y << 20) | (uint64_t)(uint32_t)z;
}

__host__ __device__ __forceinline__ uint64_t tb_mix64(uint64_t k) {   // murmur3 fmix64
    k ^= k >> 33; k *= 0xff51afd7ed558ccdULL; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ULL; k ^= k >> 33;
    return k;
}

inline size_t tb_dtype_size(tb_dtype d) { return d == TB_F32 ? 4 : 2; }

// SiLU v / (1 + e^-v) with the fast exponential and divide (a few ulp); for large negative v the
// denominator exceeds 2^126 and the result is 0 (the exact value is below 2^-100 in magnitude).
__device__ __forceinline__ float tb_silu(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

inline bool tb_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch helpers implemented in the individual .cu files (all enqueue on ctx->stream).
tb_status tb_nbr_build_blocks(tb_ctx* ctx, const int32_t* coords, int64_t n, int stride, int32_t* nbr, void* ws);
size_t tb_nbr_workspace_bytes(int64_t n);
// The seven neighbor offsets in {0,1}^3 other than (1,1,1), the corners of the dual-grid quads,
// as taps of the map (tap = kd*9 + kh*3 + kw): slot j = (dx,dy,dz)
//   0 (0,0,0)  1 (0,0,1)  2 (0,1,0)  3 (0,1,1)  4 (1,0,0)  5 (1,0,1)  6 (1,1,0)
__host__ __device__ constexpr int tb_quad_tap(int j) {
    return j == 0 ? 13 : j == 1 ? 14 : j == 2 ? 16 : j == 3 ? 17 : j == 4 ? 22 : j == 5 ? 23 : 25;
}
// Those seven taps of the map: out[j*n + i] = row of coords[i] + slot j's offset, or n when
// absent; the same table and lookups as the 27-tap map. ws: tb_nbr_workspace_bytes(n).
tb_status tb_nbr_build_quad_taps(tb_ctx* ctx, const int32_t* coords, int64_t n, int stride, int32_t* out, void* ws);
tb_status tb_conv_tc_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                            const void* feats, int ci, const void* weight, const float* bias, int co,
                            tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);
// The conv kernels compute output rows [row0, row0 + nrows) of an n-row map (tap stride and
// sentinel n); the tensor-core kernels run whole tiles from the one holding row0 and store only
// the range's rows.
tb_status tb_conv_f32_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                             const float* feats, int ci, const float* weight, const float* bias, int co,
                             tb_epilogue epi, float* out);
bool tb_conv_tc_supported(int ci, int co);
tb_status tb_conv_brick_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                               const void* feats, int ci, const void* weight, const float* bias, int co,
                               tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);
bool tb_conv_brick_supported(int ci, int co);
tb_status tb_conv_pair_launch(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                              const void* feats, int ci, const void* weight, const float* bias, int co,
                              tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);
bool tb_conv_pair_supported(int ci, int co);
// The pair kernel over two row ranges in one launch ([row0, row0 + nrows) and
// [row0b, row0b + nrowsb); nrowsb may be 0): the two edge planes of a slab.
tb_status tb_conv_pair_launch2(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows, int64_t row0b,
                               int64_t nrowsb, const void* feats, int ci, const void* weight, const float* bias, int co,
                               tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);
tb_status tb_convnext_tail_launch(tb_ctx* ctx, int64_t n, int c, const void* h, tb_dtype h_dtype, const void* x,
                                  const float* nw, const float* nb, const void* w1, const float* b1, const void* w2,
                                  const float* b2, tb_dtype dtype, tb_dtype out_dtype, void* out);
bool tb_convnext_tc_supported(int c);
bool tb_convnext_two_pass_supported(int c);
// Row LayerNorm over c channels (c % 8 == 0, c <= 2048): out row r = act(LN(src row rows[r] or r)
// * w + b) with eps; w/b may be NULL (no affine).
tb_status tb_row_norm_launch(tb_ctx* ctx, const void* src, tb_dtype in_dtype, const int32_t* rows, int64_t n, int c,
                             const float* w, const float* b, int silu, tb_dtype out_dtype, void* out,
                             float eps = 1e-6f);
// Per-voxel linear on tcgen05 (16-bit operands): out[m][n] = act(a[m] . w[n] + bias[n]) + res[m][n].
tb_status tb_linear_launch(tb_ctx* ctx, int64_t m, int k, int n, const void* a, const void* w, const float* bias,
                           const void* res, tb_dtype res_dtype, int act, tb_dtype dtype, tb_dtype out_dtype,
                           void* out);
uint64_t tb_hash_capacity(int64_t n);
