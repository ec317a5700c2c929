// tb_submconv_stack_host: one decoder stage run from host buffers (the shape of run1 /
// GraphRun::run, src/shape_decoder.cpp:34-51 and src/sparse.cpp:145-169: upload, map, stacked
// convs, read back), pipelined over row chunks so that the PCIe transfers in both directions
// and the convs overlap.
//
// The map needs every coordinate, so the coordinates go up first and the map is built. The
// features then stream up in K chunks of rows on a copy stream. A small kernel finds, for each
// output chunk k, the largest neighbor row hi[k] that any of its rows reads; the conv of chunk k
// of the first layer waits only for the upload of the chunk holding hi[k], and the conv of
// chunk k of layer l only for layer l-1's chunks up to that one (they are issued in that order
// on the compute stream). Each layer writes its own buffer, so no conv overwrites rows that a
// later-issued conv still reads. As soon as the last layer has computed chunk k, a second copy
// stream sends it down while later chunks upload and compute.
#include "tb_common.cuh"

#include <algorithm>

namespace {

// Chunks of at least 131,072 rows keep a conv launch (about 45 us at C=64) well above its fixed
// cost; up to 32 of them keep the tail after the last upload (the last chunks' convs and
// downloads) near 1 ms at 4.9M voxels.
constexpr int kMaxChunks = 32;
constexpr int64_t kChunkAlign = 256;        // tb_submconv_range's row0 granularity
constexpr int64_t kMinChunkRows = 131072;

// hi[k] = max over the rows i of chunk k of max(i, every present neighbor row of i).
__global__ void k_chunk_hi(const int32_t* __restrict__ nbr, int64_t n, int64_t chunk, int32_t* __restrict__ hi) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int32_t m = (int32_t)i;
#pragma unroll 9
        for (int t = 0; t < 27; ++t) {
            const int32_t v = nbr[(int64_t)t * n + i];
            if (v != (int32_t)n && v > m) m = v;
        }
        const int k = (int)(i / chunk);
        const unsigned same = __match_any_sync(__activemask(), k);
        const int32_t mx = __reduce_max_sync(same, m);
        if ((int)(threadIdx.x & 31) == __ffs(same) - 1) atomicMax(hi + k, mx);
    }
}

tb_status ensure_pipeline(tb_ctx* ctx) {
    if (!ctx->copy_in) TB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking));
    if (!ctx->copy_out) TB_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking));
    if (!ctx->stage_ev_made) {
        for (cudaEvent_t& e : ctx->stage_ev) TB_CUDA_TRY(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        ctx->stage_ev_made = true;
    }
    if (!ctx->chunk_hi_host)
        TB_CUDA_TRY(ctx, cudaHostAlloc(reinterpret_cast<void**>(&ctx->chunk_hi_host), kMaxChunks * sizeof(int32_t),
                                       cudaHostAllocDefault));
    return TB_OK;
}

}  // namespace

extern "C" tb_status tb_submconv_stack_host(tb_ctx* ctx, const int32_t* coords_host, int64_t n, int coord_stride,
                                            const void* feats_host, const tb_conv_layer* layers, int nlayers,
                                            tb_dtype dtype, tb_dtype out_dtype, void* out_host) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || nlayers <= 0 || !layers || (coord_stride != 3 && coord_stride != 4))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv_stack_host: bad arguments");
    for (int l = 0; l < nlayers; ++l) {
        if (layers[l].ci <= 0 || layers[l].co <= 0 || !layers[l].weight)
            return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv_stack_host: bad layer");
        if (l > 0 && layers[l].ci != layers[l - 1].co)
            return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv_stack_host: layer ci != previous co");
    }
    if (n == 0) return TB_OK;
    if (!coords_host || !feats_host || !out_host)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_submconv_stack_host: null pointer");
    if (n >= (int64_t)INT32_MAX) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_submconv_stack_host: n must be < 2^31-1");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    tb_status s = ensure_pipeline(ctx);
    if (s != TB_OK) return s;

    // buffers: coords, map, chunk bounds, then one feature buffer per layer boundary
    const size_t es = tb_dtype_size(dtype), oes = tb_dtype_size(out_dtype);
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t coords_b = al((size_t)n * coord_stride * 4), nbr_b = al((size_t)n * 27 * 4), hi_b = al(kMaxChunks * 4);
    size_t total = coords_b + nbr_b + hi_b;
    size_t buf_off[64 + 1];
    if (nlayers > 64) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_submconv_stack_host: at most 64 layers");
    for (int l = 0; l <= nlayers; ++l) {
        const int c = l == 0 ? layers[0].ci : layers[l - 1].co;
        buf_off[l] = total;
        total += al((size_t)n * c * (l == nlayers ? oes : es));
    }
    s = tb_ensure(ctx, &ctx->host_stage, &ctx->host_stage_bytes, total, "host-call staging");
    if (s != TB_OK) return s;
    uint8_t* base = reinterpret_cast<uint8_t*>(ctx->host_stage);
    int32_t* d_coords = reinterpret_cast<int32_t*>(base);
    int32_t* d_nbr = reinterpret_cast<int32_t*>(base + coords_b);
    int32_t* d_hi = reinterpret_cast<int32_t*>(base + coords_b + nbr_b);

    // row chunks: multiples of kChunkAlign, at least kMinChunkRows, at most kMaxChunks
    int64_t nk = std::max<int64_t>(1, std::min<int64_t>(kMaxChunks, n / kMinChunkRows));
    int64_t chunk = ((n + nk - 1) / nk + kChunkAlign - 1) / kChunkAlign * kChunkAlign;
    const int K = (int)((n + chunk - 1) / chunk);
    auto rows_of = [&](int k) { return std::min<int64_t>(chunk, n - (int64_t)k * chunk); };
    cudaEvent_t ev_coords = ctx->stage_ev[0], ev_hi = ctx->stage_ev[1];
    cudaEvent_t* ev_in = ctx->stage_ev + 2;
    cudaEvent_t* ev_out = ctx->stage_ev + 2 + kMaxChunks;
    cudaStream_t sc = ctx->stream;

    // once copies are queued, an error return first lets them finish (the caller's host buffers)
    auto drain = [&](tb_status st) {
        cudaStreamSynchronize(ctx->copy_in);
        cudaStreamSynchronize(ctx->copy_out);
        return st;
    };
    // 1. coordinates, then every feature chunk, on the upload stream
    const int c0 = layers[0].ci;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(d_coords, coords_host, (size_t)n * coord_stride * 4, cudaMemcpyHostToDevice,
                                     ctx->copy_in));
    TB_CUDA_TRY(ctx, cudaEventRecord(ev_coords, ctx->copy_in));
    for (int k = 0; k < K; ++k) {
        const size_t off = (size_t)k * chunk * c0 * es;
        cudaError_t e = cudaMemcpyAsync(base + buf_off[0] + off, reinterpret_cast<const uint8_t*>(feats_host) + off,
                                        (size_t)rows_of(k) * c0 * es, cudaMemcpyHostToDevice, ctx->copy_in);
        if (e == cudaSuccess) e = cudaEventRecord(ev_in[k], ctx->copy_in);
        if (e != cudaSuccess) return drain(tb_cuda_fail(ctx, e, "feature chunk upload"));
    }
    // 2. the map, and each chunk's highest input row
    cudaError_t e = cudaStreamWaitEvent(sc, ev_coords, 0);
    if (e != cudaSuccess) return drain(tb_cuda_fail(ctx, e, "cudaStreamWaitEvent(coords)"));
    s = tb_build_neighbor_map(ctx, d_coords, n, coord_stride, d_nbr);
    if (s != TB_OK) return drain(s);
    int need[kMaxChunks];
    for (int k = 0; k < K; ++k) need[k] = k;
    if (K > 1) {
        e = cudaMemsetAsync(d_hi, 0, K * sizeof(int32_t), sc);
        if (e == cudaSuccess) {
            const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->num_sms * 8);
            k_chunk_hi<<<grid, 256, 0, sc>>>(d_nbr, n, chunk, d_hi);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->chunk_hi_host, d_hi, K * sizeof(int32_t), cudaMemcpyDeviceToHost, sc);
        if (e == cudaSuccess) e = cudaEventRecord(ev_hi, sc);
        if (e == cudaSuccess) e = cudaEventSynchronize(ev_hi);
        if (e != cudaSuccess) return drain(tb_cuda_fail(ctx, e, "chunk bounds"));
        for (int k = 0; k < K; ++k)
            need[k] = std::min(K - 1, std::max(k, (int)(ctx->chunk_hi_host[k] / chunk)));
        for (int k = 1; k < K; ++k) need[k] = std::max(need[k], need[k - 1]);
    }
    // 3. convs, deepest ready layer first; each finished last-layer chunk goes down at once
    int next[64] = {0};
    int waited = -1;
    const int L = nlayers;
    while (next[L - 1] < K) {
        int l = L - 1;
        while (l > 0 && !(next[l] < K && next[l - 1] > need[next[l]])) --l;
        const int k = next[l];
        if (l == 0 && need[k] > waited) {
            e = cudaStreamWaitEvent(sc, ev_in[need[k]], 0);
            if (e != cudaSuccess) return drain(tb_cuda_fail(ctx, e, "cudaStreamWaitEvent(features)"));
            waited = need[k];
        }
        const tb_dtype od = l == L - 1 ? out_dtype : dtype;
        s = tb_submconv_range(ctx, d_nbr, n, (int64_t)k * chunk, rows_of(k), base + buf_off[l], layers[l].ci,
                              layers[l].weight, layers[l].bias, layers[l].co, dtype, od, layers[l].epi,
                              base + buf_off[l + 1]);
        if (s != TB_OK) return drain(s);
        ++next[l];
        if (l == L - 1) {
            const int co = layers[L - 1].co;
            const size_t off = (size_t)k * chunk * co * oes;
            e = cudaEventRecord(ev_out[k], sc);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->copy_out, ev_out[k], 0);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(reinterpret_cast<uint8_t*>(out_host) + off, base + buf_off[L] + off,
                                    (size_t)rows_of(k) * co * oes, cudaMemcpyDeviceToHost, ctx->copy_out);
            if (e != cudaSuccess) return drain(tb_cuda_fail(ctx, e, "output chunk download"));
        }
    }
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->copy_out));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->copy_in));
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(sc));
    return tb_ctx_check_device(ctx);
}
