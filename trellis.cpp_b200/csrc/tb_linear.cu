// Per-voxel linear layers on tcgen05: out[m][n] = act(bias[n] + sum_k a[m][k] w[n][k]) + res[m][n].
//
// The dense layers of the decoder path: from_latent (32 -> 1024) and output_layer (64 -> out_ch)
// of decode_unet (src/shape_decoder.cpp:62-77,84-86,114), and the two MLP layers of a ConvNeXt
// block tail (src/sparse.cpp:127-131) at widths whose LayerNorm tile does not fit the fused
// tail kernel's shared memory (C = 512, 1024). The reference runs them as ggml_mul_mat with a
// separate ggml_add / ggml_silu.
//
// Persistent kernel, one CTA per SM over 128 x BN output tiles (BN <= 256, N-tiles of one row
// block adjacent so A stays in L2): a producer warp streams 128 x KB blocks of A and BN x KB
// blocks of W by TMA (KB = 64 with the 128-byte swizzle when K % 64 == 0, else K = 32 or 16 with
// the 64 / 32-byte swizzle) through a 4-stage ring; an issuer warp runs tcgen05.mma (M = 128,
// N = BN, K = 16) into one of two BN-column TMEM accumulators, so the epilogue of one tile
// overlaps the MMAs of the next; four epilogue warps (one per TMEM lane quarter, a thread per
// output row) add the bias, apply SiLU, add the residual row, convert and store. Rows past m and
// weight rows past n are zero-filled by TMA and never stored.
#include "tb_common.cuh"
#include "tb_tc_ptx.cuh"

#include <algorithm>

namespace {

using namespace tbtc;

constexpr int kStages = 4;
constexpr int kLinThreads = 6 * 32;   // warp 0 producer, warp 1 issuer, warps 2-5 epilogue
constexpr int kLinBars = 2 * kStages + 2 * 2 + 1;

struct LinParams {
    int64_t m;
    int k, n, kb, nkb, bn, ntn;
    int64_t ntiles;
    const float* bias;
    const uint8_t* res;
    int res_kind;          // 0 f32, 1 f16, 2 bf16
    uint8_t* out;
    int out_kind;
    int act;               // 0 none, 1 SiLU
    int vec_ok;            // bias and residual rows 16-byte aligned: the epilogue reads them by 16 bytes
    uint32_t idesc, tmem_cols, a_bytes, b_bytes;   // b_bytes: the W block's slot, rounded to 1024
    uint32_t tx_bytes;                             // bytes one stage's two TMA boxes deliver
    int* err;
};

__device__ __forceinline__ float ld_kind(const uint8_t* p, int64_t i, int kind) {
    if (kind == 0) return reinterpret_cast<const float*>(p)[i];
    const uint16_t u = reinterpret_cast<const uint16_t*>(p)[i];
    if (kind == 2) return __uint_as_float((uint32_t)u << 16);
    return __half2float(__ushort_as_half(u));
}

// 16 consecutive elements from element index i of a 16-byte aligned row (i a multiple of 8, of 4
// for fp32): one thread's columns of an output row in the epilogue, read with 16-byte loads.
__device__ __forceinline__ void ld16_kind(const uint8_t* p, int64_t i, int kind, float* v) {
    if (kind == 0) {
        const float4* s = reinterpret_cast<const float4*>(p) + i / 4;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 x = s[q];
            v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
        }
        return;
    }
    const uint4* s = reinterpret_cast<const uint4*>(p) + i / 8;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint4 x = s[q];            // plain loads: the residual may be the output buffer itself
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = w[j] & 0xFFFFu, hi = w[j] >> 16;
            if (kind == 2) {
                v[8 * q + 2 * j] = __uint_as_float(lo << 16);
                v[8 * q + 2 * j + 1] = __uint_as_float(hi << 16);
            } else {
                v[8 * q + 2 * j] = __half2float(__ushort_as_half((unsigned short)lo));
                v[8 * q + 2 * j + 1] = __half2float(__ushort_as_half((unsigned short)hi));
            }
        }
    }
}

__device__ __forceinline__ void st_kind(uint8_t* p, int64_t i, float v, int kind) {
    if (kind == 0) reinterpret_cast<float*>(p)[i] = v;
    else if (kind == 2) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, volatile int* ab, int* err) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, ab, err));
}

template <int RB>
__global__ void __launch_bounds__(kLinThreads, 1)
k_linear(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap, const LinParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    const uint32_t stage_bytes = p.a_bytes + p.b_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * stage_bytes);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kLinBars);   // [0] tmem, [1] abort, [2] consumed
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);
    const uint32_t b0 = smem_u32(bars);
    auto full = [&](int s) { return b0 + 8u * s; };
    auto empty = [&](int s) { return b0 + 8u * (kStages + s); };
    auto accf = [&](int s) { return b0 + 8u * (2 * kStages + s); };
    auto acce = [&](int s) { return b0 + 8u * (2 * kStages + 2 + s); };
    const uint32_t drain = b0 + 8u * (2 * kStages + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(accf(s), 1);
            mbar_init(acce(s), 4);
        }
        mbar_init(drain, 1);
        s_misc[1] = 0;
        s_misc[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_misc[0];
    int issued = 0;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        int it = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x) {
            const int tm = (int)(t / p.ntn), tn = (int)(t % p.ntn);
            for (int kb = 0; kb < p.nkb; ++kb, ++it) {
                const int s = it % kStages;
                if (it >= kStages && !wait_warp(empty(s), (uint32_t)(((it / kStages) - 1) & 1), s_abort, p.err)) {
                    ok = false;
                    break;
                }
                if (elect_one()) {
                    const uint32_t dst = smem_u32(smem + s * stage_bytes);
                    mbar_arrive_expect_tx(full(s), p.tx_bytes);
                    tma_load_2d(dst, &amap, kb * p.kb, tm * 128, full(s));
                    tma_load_2d(dst + p.a_bytes, &wmap, kb * p.kb, tn * p.bn, full(s));
                }
                __syncwarp();
                issued = it + 1;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        int it = 0, i = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < p.ntiles && ok; t += gridDim.x, ++i) {
            const int acc = i & 1;
            if (i >= 2 && !wait_warp(acce(acc), (uint32_t)(((i >> 1) - 1) & 1), s_abort, p.err)) { ok = false; break; }
            tc_fence_after();
            for (int kb = 0; kb < p.nkb; ++kb, ++it) {
                const int s = it % kStages;
                if (!wait_warp(full(s), (uint32_t)((it / kStages) & 1), s_abort, p.err)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t a_addr = smem_u32(smem + s * stage_bytes), b_addr = a_addr + p.a_bytes;
                    for (int k = 0; k < p.kb / 16; ++k)
                        tc_mma(tmem + (uint32_t)(acc * p.bn), smem_desc<RB>(a_addr + 32 * k),
                               smem_desc<RB>(b_addr + 32 * k), p.idesc, (kb | k) ? 1u : 0u);
                    tc_commit(empty(s));
                    if (kb == p.nkb - 1) tc_commit(accf(acc));
                }
                __syncwarp();
                if (lane == 0) s_misc[2] = (uint32_t)(it + 1);
            }
        }
        // every MMA has completed before the TMEM is freed (also after an abort)
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) { }
    } else {
        // ------------------------------------------------------------------ epilogue warps
        const int q = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const int osz = p.out_kind == 0 ? 4 : 2;
        int i = 0;
        for (int64_t t = blockIdx.x; t < p.ntiles; t += gridDim.x, ++i) {
            const int acc = i & 1;
            const int tm = (int)(t / p.ntn), tn = (int)(t % p.ntn);
            if (!wait_warp(accf(acc), (uint32_t)((i >> 1) & 1), s_abort, p.err)) break;
            tc_fence_after();
            const int64_t row = (int64_t)tm * 128 + q * 32 + lane;
            const bool rvalid = row < p.m;
            for (int c0 = 0; c0 < p.bn; c0 += 16) {
                uint32_t v[16];
                __syncwarp();
                TMEM_LD_X16(lane_base + (uint32_t)(acc * p.bn + c0), v);
                tmem_wait_ld();
                if (c0 + 16 >= p.bn) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acce(acc));
                }
                const int col0 = tn * p.bn + c0;
                if (!rvalid || col0 >= p.n) continue;
                float f[16];
                if (col0 + 16 <= p.n && p.vec_ok) {
                    // whole chunk, 16-byte aligned bias and residual rows: vector loads
                    float bb[16], rr[16];
                    if (p.bias) ld16_kind(reinterpret_cast<const uint8_t*>(p.bias), col0, 0, bb);
                    if (p.res) ld16_kind(p.res, row * p.n + col0, p.res_kind, rr);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float x = __uint_as_float(v[j]);
                        if (p.bias) x += bb[j];
                        if (p.act) x = tb_silu(x);
                        if (p.res) x += rr[j];
                        f[j] = x;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = col0 + j;
                        float x = __uint_as_float(v[j]);
                        if (col < p.n) {
                            if (p.bias) x += __ldg(p.bias + col);
                            if (p.act) x = tb_silu(x);
                            if (p.res) x += ld_kind(p.res, row * p.n + col, p.res_kind);
                        }
                        f[j] = x;
                    }
                }
                uint8_t* orow = p.out + (size_t)row * p.n * osz;
                if (col0 + 16 <= p.n && (p.n % (osz == 4 ? 4 : 8)) == 0) {
                    store16(orow + (size_t)col0 * osz, f, p.out_kind);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (col0 + j < p.n) st_kind(orow, col0 + j, f[j], p.out_kind);
                }
            }
        }
    }
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // TMA loads still in flight after an abort land before the CTA exits
        for (int it = (int)s_misc[2]; it < issued; ++it) {
            const long long t0 = clock64();
            while (!mbar_try_wait(full(it % kStages), (uint32_t)((it / kStages) & 1)) && clock64() - t0 < kWaitCycles) { }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// ---- CTA-pair form (K a multiple of 64, 256-column tiles, at least two row blocks) -----------
// Two CTAs of a cluster (neighbouring SMs) share each MMA: each loads its own 128-row block of A
// and half of the tile's 256 weight rows, and the even CTA issues tcgen05.mma.cta_group::2
// (M = 256) over both. Per output row that halves the weight bytes streamed from L2. The even
// CTA's stage barrier also waits for the odd CTA's stage, which the odd CTA's MMA warp passes on
// once its TMA has landed; MMA commits multicast to both CTAs; the epilogue warps of both arrive
// on the even CTA's accumulator-free barrier. Cross-CTA hand-offs are relaxed at cluster scope.
constexpr int kLinPairStages = 6;
constexpr int kLinPairBars = 2 * kLinPairStages + 2 * 2 + 1;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kLinThreads, 1)
k_linear_pair(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap, const LinParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    const uint32_t stage_bytes = p.a_bytes + p.b_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kLinPairStages * stage_bytes);
    uint32_t* s_misc = reinterpret_cast<uint32_t*>(bars + kLinPairBars);   // [0] tmem, [1] abort, [2] consumed
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_misc + 1);
    const uint32_t b0 = smem_u32(bars);
    auto full = [&](int s) { return b0 + 8u * s; };
    auto empty = [&](int s) { return b0 + 8u * (kLinPairStages + s); };
    auto accf = [&](int s) { return b0 + 8u * (2 * kLinPairStages + s); };
    auto acce = [&](int s) { return b0 + 8u * (2 * kLinPairStages + 2 + s); };
    const uint32_t drain = b0 + 8u * (2 * kLinPairStages + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kLinPairStages; ++s) {
            mbar_init(full(s), leader ? 2 : 1);     // even CTA: its own TMA and the odd CTA's, passed on
            mbar_init(empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(accf(s), 1);
            mbar_init(acce(s), 8);                  // four epilogue warps in each CTA (even CTA's copy used)
        }
        mbar_init(drain, 1);
        s_misc[1] = 0;
        s_misc[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(s_misc)), "r"(p.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = s_misc[0];
    const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();
    int issued = 0;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer (per CTA)
        int it = 0;
        bool ok = true;
        for (int64_t t = cid; t < p.ntiles && ok; t += ncl) {
            const int tm = 2 * (int)(t / p.ntn) + (int)rank, tn = (int)(t % p.ntn);
            for (int kb = 0; kb < p.nkb; ++kb, ++it) {
                const int s = it % kLinPairStages;
                if (it >= kLinPairStages &&
                    !__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(empty(s), (uint32_t)(((it / kLinPairStages) - 1) & 1),
                                                                      s_abort, p.err))) {
                    ok = false;
                    break;
                }
                if (elect_one()) {
                    const uint32_t dst = smem_u32(smem + s * stage_bytes);
                    mbar_arrive_expect_tx(full(s), p.tx_bytes);
                    tma_load_2d(dst, &amap, kb * p.kb, tm * 128, full(s));
                    tma_load_2d(dst + p.a_bytes, &wmap, kb * p.kb, tn * p.bn + (int)rank * (p.bn / 2), full(s));
                }
                __syncwarp();
                issued = it + 1;
            }
        }
    } else if (warp == 1 && !leader) {
        // ------------------------------------------------------------------ odd CTA: stage forwarder
        if (lane == 0) {
            const int64_t ntl = (p.ntiles - cid + ncl - 1) / ncl;       // this cluster's tiles
            const int64_t total = ntl * p.nkb;
            for (int64_t it = 0; it < total; ++it) {
                const int s = (int)(it % kLinPairStages);
                if (!mbar_wait(full(s), (uint32_t)((it / kLinPairStages) & 1), s_abort, p.err)) break;
                mbar_arrive_cluster_relaxed(full(s), 0);
                s_misc[2] = (uint32_t)(it + 1);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer (even CTA)
        int it = 0, i = 0;
        bool ok = true;
        for (int64_t t = cid; t < p.ntiles && ok; t += ncl, ++i) {
            const int acc = i & 1;
            if (i >= 2 && !__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(acce(acc), (uint32_t)(((i >> 1) - 1) & 1),
                                                                            s_abort, p.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int kb = 0; kb < p.nkb; ++kb, ++it) {
                const int s = it % kLinPairStages;
                if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(full(s), (uint32_t)((it / kLinPairStages) & 1),
                                                                      s_abort, p.err))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t a_addr = smem_u32(smem + s * stage_bytes), b_addr = a_addr + p.a_bytes;
                    for (int k = 0; k < p.kb / 16; ++k)
                        tc_mma_ss_pair(tmem + (uint32_t)(acc * p.bn), smem_desc<128>(a_addr + 32 * k),
                                       smem_desc<128>(b_addr + 32 * k), p.idesc, (kb | k) ? 1u : 0u);
                    tc_commit_pair(empty(s), 0x3);
                    if (kb == p.nkb - 1) tc_commit_pair(accf(acc), 0x3);
                }
                __syncwarp();
                if (lane == 0) s_misc[2] = (uint32_t)(it + 1);
            }
        }
        if (elect_one()) tc_commit_pair(drain, 0x1);
        __syncwarp();
        const long long t0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitCycles) { }
    } else if (warp >= 2) {
        // ------------------------------------------------------------------ epilogue warps (per CTA)
        const int q = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const int osz = p.out_kind == 0 ? 4 : 2;
        int i = 0;
        for (int64_t t = cid; t < p.ntiles; t += ncl, ++i) {
            const int acc = i & 1;
            const int tm = 2 * (int)(t / p.ntn) + (int)rank, tn = (int)(t % p.ntn);
            if (!__all_sync(0xffffffffu, mbar_wait_cluster_relaxed(accf(acc), (uint32_t)((i >> 1) & 1), s_abort, p.err)))
                break;
            tc_fence_after();
            const int64_t row = (int64_t)tm * 128 + q * 32 + lane;
            const bool rvalid = row < p.m;
            for (int c0 = 0; c0 < p.bn; c0 += 16) {
                uint32_t v[16];
                __syncwarp();
                TMEM_LD_X16(lane_base + (uint32_t)(acc * p.bn + c0), v);
                tmem_wait_ld();
                if (c0 + 16 >= p.bn) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster_relaxed(acce(acc), 0);
                }
                const int col0 = tn * p.bn + c0;
                if (!rvalid || col0 >= p.n) continue;
                float f[16];
                if (col0 + 16 <= p.n && p.vec_ok) {
                    // whole chunk, 16-byte aligned bias and residual rows: vector loads
                    float bb[16], rr[16];
                    if (p.bias) ld16_kind(reinterpret_cast<const uint8_t*>(p.bias), col0, 0, bb);
                    if (p.res) ld16_kind(p.res, row * p.n + col0, p.res_kind, rr);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float x = __uint_as_float(v[j]);
                        if (p.bias) x += bb[j];
                        if (p.act) x = tb_silu(x);
                        if (p.res) x += rr[j];
                        f[j] = x;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = col0 + j;
                        float x = __uint_as_float(v[j]);
                        if (col < p.n) {
                            if (p.bias) x += __ldg(p.bias + col);
                            if (p.act) x = tb_silu(x);
                            if (p.res) x += ld_kind(p.res, row * p.n + col, p.res_kind);
                        }
                        f[j] = x;
                    }
                }
                uint8_t* orow = p.out + (size_t)row * p.n * osz;
                if (col0 + 16 <= p.n && (p.n % (osz == 4 ? 4 : 8)) == 0) {
                    store16(orow + (size_t)col0 * osz, f, p.out_kind);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (col0 + j < p.n) st_kind(orow, col0 + j, f[j], p.out_kind);
                }
            }
        }
    }
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // TMA loads still in flight after an abort land before the CTA exits (the odd CTA's own
        // barrier completes with its TMA alone; the even CTA's also needs the passed-on stage)
        for (int it = (int)s_misc[2]; it < issued; ++it) {
            const long long t0 = clock64();
            while (!mbar_try_wait(full(it % kLinPairStages), (uint32_t)((it / kLinPairStages) & 1)) &&
                   clock64() - t0 < kWaitCycles) { }
        }
    }
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

template <int RB>
tb_status launch_linear(tb_ctx* ctx, const LinParams& p0, const void* a, const void* w, tb_dtype dtype) {
    LinParams p = p0;
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUtensorMapSwizzle swz = RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                             : (RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap amap, wmap;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)p.k, (cuuint64_t)p.m};
        const cuuint64_t gstride[1] = {(cuuint64_t)p.k * 2};
        const cuuint32_t box[2] = {(cuuint32_t)p.kb, 128};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &amap, dt, 2, const_cast<void*>(a), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the linear input");
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)p.k, (cuuint64_t)p.n};
        const cuuint64_t gstride[1] = {(cuuint64_t)p.k * 2};
        const cuuint32_t box[2] = {(cuuint32_t)p.kb, (cuuint32_t)p.bn};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &wmap, dt, 2, const_cast<void*>(w), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the linear weight");
    }
    const size_t smem = (size_t)kStages * (p.a_bytes + p.b_bytes) + 8 * kLinBars + 16 + 1024;
    if (smem > (size_t)ctx->max_smem_optin) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "linear: shared memory too small");
    static size_t smem_set[3] = {0, 0, 0};
    const int si = RB == 128 ? 0 : (RB == 64 ? 1 : 2);
    if (smem > smem_set[si]) {
        cudaError_t e = cudaFuncSetAttribute(k_linear<RB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_linear)");
        smem_set[si] = smem;
    }
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(p.ntiles, ctx->num_sms));
    k_linear<RB><<<grid, kLinThreads, smem, ctx->stream>>>(amap, wmap, p);
    TB_LAUNCH_CHECK(ctx, "k_linear");
    return TB_OK;
}

tb_status launch_linear_pair(tb_ctx* ctx, const LinParams& p0, const void* a, const void* w, tb_dtype dtype) {
    LinParams p = p0;
    if (!ctx->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        TB_CUDA_TRY(ctx, cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess)
            return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
        ctx->encode_tiled = fn;
    }
    const CUtensorMapDataType dt = dtype == TB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap amap, wmap;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)p.k, (cuuint64_t)p.m};
        const cuuint64_t gstride[1] = {(cuuint64_t)p.k * 2};
        const cuuint32_t box[2] = {64, 128};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &amap, dt, 2, const_cast<void*>(a), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the linear input");
    }
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)p.k, (cuuint64_t)p.n};
        const cuuint64_t gstride[1] = {(cuuint64_t)p.k * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)(p.bn / 2)};
        CUresult cr = reinterpret_cast<EncodeTiledFn>(ctx->encode_tiled)(
            &wmap, dt, 2, const_cast<void*>(w), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the linear weight");
    }
    const size_t smem = (size_t)kLinPairStages * (p.a_bytes + p.b_bytes) + 8 * kLinPairBars + 16 + 1024;
    if (smem > (size_t)ctx->max_smem_optin) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "linear: shared memory too small");
    static size_t smem_set = 0;
    if (smem > smem_set) {
        cudaError_t e = cudaFuncSetAttribute(k_linear_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return tb_cuda_fail(ctx, e, "cudaFuncSetAttribute(k_linear_pair)");
        smem_set = smem;
    }
    const int nclusters = (int)std::max<int64_t>(1, std::min<int64_t>(p.ntiles, ctx->num_sms / 2));
    k_linear_pair<<<2 * nclusters, kLinThreads, smem, ctx->stream>>>(amap, wmap, p);
    TB_LAUNCH_CHECK(ctx, "k_linear_pair");
    return TB_OK;
}

}  // namespace

tb_status tb_linear_launch(tb_ctx* ctx, int64_t m, int k, int n, const void* a, const void* w, const float* bias,
                           const void* res, tb_dtype res_dtype, int act, tb_dtype dtype, tb_dtype out_dtype,
                           void* out) {
    if (m == 0) return TB_OK;
    const auto kind = [](tb_dtype d) { return d == TB_F32 ? 0 : (d == TB_F16 ? 1 : 2); };
    LinParams p{};
    p.m = m;
    p.k = k;
    p.n = n;
    p.kb = k % 64 == 0 ? 64 : k;
    p.nkb = k / p.kb;
    p.bn = std::min(256, (n + 15) / 16 * 16);
    p.ntn = (n + p.bn - 1) / p.bn;
    p.ntiles = ((m + 127) / 128) * p.ntn;
    p.bias = bias;
    p.res = reinterpret_cast<const uint8_t*>(res);
    p.res_kind = kind(res_dtype);
    p.out = reinterpret_cast<uint8_t*>(out);
    p.out_kind = kind(out_dtype);
    p.act = act;
    p.err = ctx->d_err;
    {
        // a residual row starts 16-byte aligned when the base is and n elements fill whole 16 bytes
        const int rsz = res ? (p.res_kind == 0 ? 4 : 2) : 4;
        const bool bias_ok = !bias || (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
        const bool res_ok = !res || ((reinterpret_cast<uintptr_t>(res) & 15) == 0 && ((int64_t)n * rsz) % 16 == 0);
        p.vec_ok = bias_ok && res_ok ? 1 : 0;
    }
    const uint32_t fmt = dtype == TB_BF16 ? 1u : 0u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * p.bn)) cols *= 2;
    p.tmem_cols = cols;
    p.a_bytes = 128u * (uint32_t)p.kb * 2u;
    p.b_bytes = ((uint32_t)p.bn * (uint32_t)p.kb * 2u + 1023u) & ~1023u;
    p.tx_bytes = p.a_bytes + (uint32_t)p.bn * (uint32_t)p.kb * 2u;
    if (p.kb == 64 && p.bn == 256 && m > 128) {
        // CTA pairs over two row blocks: each CTA loads half of the 256 weight rows of a tile
        p.ntiles = ((m + 255) / 256) * p.ntn;
        p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
        p.b_bytes = 128u * 64u * 2u;
        p.tx_bytes = p.a_bytes + p.b_bytes;
        return launch_linear_pair(ctx, p, a, w, dtype);
    }
    if (p.kb == 64) return launch_linear<128>(ctx, p, a, w, dtype);
    if (p.kb == 32) return launch_linear<64>(ctx, p, a, w, dtype);
    return launch_linear<32>(ctx, p, a, w, dtype);
}

// ---- fp32 operands (the precision mode): CUDA-core tiles of 32 rows x 64 outputs ---------------
namespace {

constexpr int kFR = 32, kFC = 64, kFK = 32;

__global__ void __launch_bounds__(256)
k_linear_f32(const float* __restrict__ a, const float* __restrict__ w, const float* __restrict__ bias,
             const float* __restrict__ res, int64_t m, int k, int n, int act, float* __restrict__ out) {
    __shared__ float as[kFR][kFK + 1];
    __shared__ float ws[kFC][kFK + 1];
    const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
    const int64_t r0 = (int64_t)blockIdx.x * kFR;
    const int c0 = blockIdx.y * kFC;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < k; k0 += kFK) {
        for (int i = threadIdx.x; i < kFR * kFK; i += 256) {
            const int r = i / kFK, kk = i % kFK;
            as[r][kk] = (r0 + r < m && k0 + kk < k) ? a[(r0 + r) * k + k0 + kk] : 0.f;
        }
        for (int i = threadIdx.x; i < kFC * kFK; i += 256) {
            const int c = i / kFK, kk = i % kFK;
            ws[c][kk] = (c0 + c < n && k0 + kk < k) ? w[(int64_t)(c0 + c) * k + k0 + kk] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kFK; ++kk) {
            const float x = as[ty][kk];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(x, ws[tx + 8 * j][kk], acc[j]);
        }
        __syncthreads();
    }
    const int64_t r = r0 + ty;
    if (r >= m) return;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = c0 + tx + 8 * j;
        if (c >= n) continue;
        float v = acc[j] + (bias ? bias[c] : 0.f);
        if (act) v = tb_silu(v);
        if (res) v += res[r * n + c];
        out[r * n + c] = v;
    }
}

}  // namespace

extern "C" tb_status tb_linear(tb_ctx* ctx, int64_t m, int k, int n, const void* a, const void* w, const float* bias,
                               const void* res, tb_dtype res_dtype, tb_epilogue act, tb_dtype dtype,
                               tb_dtype out_dtype, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (m < 0 || k <= 0 || n <= 0) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: m < 0 or k, n <= 0");
    if (act != TB_EPI_NONE && act != TB_EPI_SILU) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: bad activation");
    if (dtype != TB_F32 && dtype != TB_F16 && dtype != TB_BF16) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: bad dtype");
    if ((out_dtype != TB_F32 && out_dtype != dtype) || (res && res_dtype != TB_F32 && res_dtype != dtype))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_linear: out / residual dtype must be TB_F32 or the operand dtype");
    if (m == 0) return TB_OK;
    if (!a || !w || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: null pointer");
    if (!tb_aligned16(a) || !tb_aligned16(w) || !tb_aligned16(out) || (res && !tb_aligned16(res)))
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: a / w / res / out must be 16-byte aligned");
    if (out == a || out == w) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_linear: out must not alias a or w");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    if (dtype == TB_F32) {
        if (res && res_dtype != TB_F32) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_linear: fp32 mode needs an fp32 residual");
        const dim3 grid((unsigned)((m + kFR - 1) / kFR), (unsigned)((n + kFC - 1) / kFC));
        k_linear_f32<<<grid, 256, 0, ctx->stream>>>(reinterpret_cast<const float*>(a), reinterpret_cast<const float*>(w),
                                                    bias, reinterpret_cast<const float*>(res), m, k, n,
                                                    act == TB_EPI_SILU, reinterpret_cast<float*>(out));
        TB_LAUNCH_CHECK(ctx, "k_linear_f32");
        return TB_OK;
    }
    if (!(k % 64 == 0 || k == 16 || k == 32))
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_linear: 16-bit operands need k a multiple of 64, or 16 or 32");
    if (m >= ((int64_t)1 << 31)) return tb_fail(ctx, TB_ERR_TOO_LARGE, "tb_linear: m must be < 2^31");
    return tb_linear_launch(ctx, m, k, n, a, w, bias, res, res_dtype, act == TB_EPI_SILU ? 1 : 0, dtype, out_dtype, out);
}

extern "C" tb_status tb_layer_norm(tb_ctx* ctx, const void* x, tb_dtype x_dtype, int64_t n, int c, const float* w,
                                   const float* b, float eps, tb_epilogue act, tb_dtype out_dtype, void* out) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (n < 0 || c <= 0 || c % 8 != 0 || c > 2048)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_layer_norm: needs n >= 0 and c a multiple of 8 up to 2048");
    if ((w == nullptr) != (b == nullptr)) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_layer_norm: give both w and b or neither");
    if (act != TB_EPI_NONE && act != TB_EPI_SILU) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_layer_norm: bad activation");
    if (n == 0) return TB_OK;
    if (!x || !out) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_layer_norm: null pointer");
    if (!tb_aligned16(x) || !tb_aligned16(out)) return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_layer_norm: x / out must be 16-byte aligned");
    if (x_dtype != TB_F32 && out_dtype != TB_F32 && x_dtype != out_dtype)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_layer_norm: f16 <-> bf16 is not supported");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    return tb_row_norm_launch(ctx, x, x_dtype, nullptr, n, c, w, b, act == TB_EPI_SILU ? 1 : 0, out_dtype, out, eps);
}
