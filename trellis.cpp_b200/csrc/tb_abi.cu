// C-ABI glue: contexts, status reporting, workspace, conv dispatch and the host-buffer
// stack call. The kernels live in tb_nbr.cu, tb_conv_tc.cu, tb_conv_f32.cu, tb_subdiv.cu.
#include "tb_common.cuh"

#include <algorithm>
#include <cstring>
#include <new>

tb_status tb_fail(tb_ctx* ctx, tb_status s, const std::string& msg) {
    if (ctx) ctx->last_error = msg;
    return s;
}

tb_status tb_cuda_fail(tb_ctx* ctx, cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return tb_fail(ctx, TB_ERR_OUT_OF_MEMORY, m);
    return tb_fail(ctx, TB_ERR_CUDA, m);
}

tb_status tb_ensure(tb_ctx* ctx, void** buf, size_t* cap, size_t bytes, const char* what) {
    if (*cap >= bytes && *buf) return TB_OK;
    if (*buf) {
        // the old buffer may still be read by queued work on this stream
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaStreamSynchronize before workspace growth");
        cudaFree(*buf);
        *buf = nullptr;
        *cap = 0;
    }
    size_t want = std::max<size_t>(bytes, 1 << 20);
    cudaError_t e = cudaMalloc(buf, want);
    if (e != cudaSuccess) {
        *buf = nullptr;
        return tb_fail(ctx, TB_ERR_OUT_OF_MEMORY, std::string("workspace allocation failed (") + what + ")");
    }
    *cap = want;
    return TB_OK;
}

extern "C" {

const char* tb_status_string(tb_status s) {
    switch (s) {
        case TB_OK: return "ok";
        case TB_ERR_INVALID_ARG: return "invalid argument";
        case TB_ERR_UNSUPPORTED: return "unsupported configuration";
        case TB_ERR_CUDA: return "CUDA error";
        case TB_ERR_OUT_OF_MEMORY: return "out of device memory";
        case TB_ERR_DEVICE: return "device-side check failed";
        case TB_ERR_TOO_LARGE: return "size above the supported maximum";
    }
    return "unknown status";
}

const char* tb_version(void) { return "tb_sparse 0.1.0 (sm_100a)"; }

tb_status tb_ctx_create(int device, void* stream, tb_ctx** out) {
    if (!out) return TB_ERR_INVALID_ARG;
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return TB_ERR_INVALID_ARG;
    tb_ctx* ctx = new (std::nothrow) tb_ctx();
    if (!ctx) return TB_ERR_OUT_OF_MEMORY;
    ctx->device = device;
    ctx->stream = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSetDevice(device);
    cudaDeviceProp prop;
    if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, device);
    if (e == cudaSuccess && prop.major != 10) {
        delete ctx;
        return TB_ERR_UNSUPPORTED;   // sm_100a kernels only
    }
    if (e == cudaSuccess) {
        ctx->num_sms = prop.multiProcessorCount;
        ctx->max_smem_optin = (int)prop.sharedMemPerBlockOptin;
        e = cudaMalloc(&ctx->d_err, sizeof(int));
    }
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        if (ctx->d_err) cudaFree(ctx->d_err);
        delete ctx;
        return e == cudaErrorMemoryAllocation ? TB_ERR_OUT_OF_MEMORY : TB_ERR_CUDA;
    }
    *out = ctx;
    return TB_OK;
}

tb_status tb_ctx_destroy(tb_ctx* ctx) {
    if (!ctx) return TB_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->host_stage) cudaFree(ctx->host_stage);
    if (ctx->block_h) cudaFree(ctx->block_h);
    if (ctx->c2s_ws1) cudaFree(ctx->c2s_ws1);
    if (ctx->c2s_ws2) cudaFree(ctx->c2s_ws2);
    if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
    if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
    if (ctx->stage_ev_made)
        for (cudaEvent_t e : ctx->stage_ev) cudaEventDestroy(e);
    if (ctx->chunk_hi_host) cudaFreeHost(ctx->chunk_hi_host);
    if (ctx->tail_ws) cudaFree(ctx->tail_ws);
    if (ctx->sort_ws) cudaFree(ctx->sort_ws);
    if (ctx->d_err) cudaFree(ctx->d_err);
    delete ctx;
    return TB_OK;
}

tb_status tb_ctx_set_stream(tb_ctx* ctx, void* stream) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    ctx->stream = reinterpret_cast<cudaStream_t>(stream);
    return TB_OK;
}

const char* tb_ctx_last_error(const tb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

tb_status tb_ctx_check_device(tb_ctx* ctx) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    int h = 0;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (h != TB_DEVERR_NONE) {
        TB_CUDA_TRY(ctx, cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream));
        TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        const char* what = h == TB_DEVERR_HASH_PROBE ? "hash probe bound exceeded"
                         : h == TB_DEVERR_WAIT_TIMEOUT ? "bounded mbarrier wait timed out in the conv kernel"
                         : h == TB_DEVERR_TMEM_ALLOC ? "TMEM allocation failed" : "unknown device error";
        return tb_fail(ctx, TB_ERR_DEVICE, what);
    }
    return TB_OK;
}

tb_status tb_submconv_range(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                            const void* feats, int ci, const void* weight, const float* bias, int co,
                            tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || ci <= 0 || co <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: n < 0 or channels <= 0");
    if (row0 < 0 || nrows < 0 || row0 + nrows > n)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv_range: need 0 <= row0 and row0 + nrows <= n");
    if (epi != TB_EPI_NONE && epi != TB_EPI_SILU) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: bad epilogue");
    if (dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: bad dtype");
    if (out_dtype != TB_F32 && out_dtype != dtype)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_submconv: out_dtype must be TB_F32 or the operand dtype");
    if (nrows == 0) return TB_OK;
    if (!nbr || !feats || !weight || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: null pointer");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_submconv: n must be < 2^31-1");
    if (!tb_aligned16(feats) || !tb_aligned16(weight) || !tb_aligned16(out) || (bias && !tb_aligned16(bias)))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: feats/weight/bias/out must be 16-byte aligned");
    if (feats == out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv: out must not alias feats");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (dtype == TB_F32)
        return tb_conv_f32_launch(ctx, nbr, n, row0, nrows, reinterpret_cast<const float*>(feats), ci,
                                  reinterpret_cast<const float*>(weight), bias, co, epi, reinterpret_cast<float*>(out));
    const bool pair = ctx->conv_path == TB_CONV_PAIR ||
                      (ctx->conv_path == TB_CONV_AUTO && tb_conv_pair_supported(ci, co));
    if (pair)
        return tb_conv_pair_launch(ctx, nbr, n, row0, nrows, feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
    const bool brick = ctx->conv_path == TB_CONV_BRICK ||
                       (ctx->conv_path == TB_CONV_AUTO && tb_conv_brick_supported(ci, co));
    if (brick)
        return tb_conv_brick_launch(ctx, nbr, n, row0, nrows, feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
    return tb_conv_tc_launch(ctx, nbr, n, row0, nrows, feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
}

tb_status tb_submconv(tb_ctx* ctx, const int32_t* nbr, int64_t n, const void* feats, int ci,
                      const void* weight, const float* bias, int co, tb_dtype dtype, tb_dtype out_dtype,
                      tb_epilogue epi, void* out) {
    return tb_submconv_range(ctx, nbr, n, 0, n, feats, ci, weight, bias, co, dtype, out_dtype, epi, out);
}

tb_status tb_convnext_tail(tb_ctx* ctx, int64_t n, int c, const void* h, tb_dtype h_dtype, const void* x,
                           const float* norm_w, const float* norm_b, const void* w1, const float* b1,
                           const void* w2, const float* b2, tb_dtype dtype, tb_dtype out_dtype, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || c <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_convnext_tail: n < 0 or c <= 0");
    if ((dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16) || (h_dtype != TB_F32 && h_dtype != dtype))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_convnext_tail: bad dtype (h must be TB_F32 or the operand dtype)");
    if (out_dtype != TB_F32 && out_dtype != dtype)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_convnext_tail: out_dtype must be TB_F32 or the operand dtype");
    if (n == 0) return TB_OK;
    if (!h || !x || !norm_w || !norm_b || !w1 || !b1 || !w2 || !b2 || !out)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_convnext_tail: null pointer");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_convnext_tail: n must be < 2^31-1");
    if (!tb_aligned16(h) || !tb_aligned16(x) || !tb_aligned16(w1) || !tb_aligned16(w2) || !tb_aligned16(out))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_convnext_tail: h/x/w1/w2/out must be 16-byte aligned");
    if (out == h || out == x) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_convnext_tail: out must not alias h or x");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    return tb_convnext_tail_launch(ctx, n, c, h, h_dtype, x, norm_w, norm_b, w1, b1, w2, b2, dtype, out_dtype, out);
}

tb_status tb_sparse_convnext(tb_ctx* ctx, const int32_t* nbr, int64_t n, const void* feats, int c,
                             const void* conv_w, const float* conv_b, const float* norm_w, const float* norm_b,
                             const void* w1, const float* b1, const void* w2, const float* b2, tb_dtype dtype,
                             tb_dtype out_dtype, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || c <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_sparse_convnext: n < 0 or c <= 0");
    if (n == 0) return TB_OK;
    if (dtype != TB_F32 && !tb_convnext_tc_supported(c) && !tb_convnext_two_pass_supported(c))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                       "tb_sparse_convnext: 16-bit operands need c in {16, 32} or a multiple of 64 up to 2048");
    tb_status s = tb_ensure(ctx, &ctx->block_h, &ctx->block_h_bytes, (size_t)n * c * sizeof(float), "convnext conv output");
    if (s != TB_OK) return s;
    s = tb_submconv(ctx, nbr, n, feats, c, conv_w, conv_b, c, dtype, TB_F32, TB_EPI_NONE, ctx->block_h);
    if (s != TB_OK) return s;
    return tb_convnext_tail(ctx, n, c, ctx->block_h, TB_F32, feats, norm_w, norm_b, w1, b1, w2, b2, dtype, out_dtype,
                            out);
}

tb_status tb_ctx_set_conv_path(tb_ctx* ctx, tb_conv_path path) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (path != TB_CONV_AUTO && path != TB_CONV_GATHER && path != TB_CONV_BRICK && path != TB_CONV_PAIR)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_ctx_set_conv_path: unknown path");
    ctx->conv_path = path;
    return TB_OK;
}

}  // extern "C"
