/*
 * tb_oracle.c -- CPU restatement of pwilkin/trellis.cpp's sparse submanifold-conv path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker and the timed CPU
 * baseline. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg
 * and its `--impl reference` arm) load it. The product library never links it and has
 * no CPU fallback to it.
 *
 * What it restates (paths are inside the reference project):
 *   orc_key                    src/sparse.cpp:25        20-bit-per-axis packed key
 *   orc_build_neighbor_table   src/sparse.cpp:21-39     hash insert (last writer wins),
 *                                                        27 lookups, tap-major [27*N],
 *                                                        sentinel N
 *   orc_submconv_f64           src/sparse.cpp:64-92     per-tap gather -> GEMM -> accumulate
 *                                                        + bias; absent taps read a zero row
 *   orc_submconv_rows_f64      same, for a subset of output rows
 *   orc_submconv_f32_mt        same, fp32, threads over voxel blocks (the CPU baseline)
 *   orc_subdivide              src/sparse.cpp:205-222   octant loop, child coords, gidx
 *   orc_c2s_gather             src/sparse.cpp:263-266,288  child takes channel block o
 *   orc_dual_grid_mesh         src/dual_grid.cpp:16-56  dual vertices, quad lookup, split
 *
 * Parity pin: tests/golden/make_golden.py runs the reference's own torch restatements
 * (tools/ref_sparse_conv.py:47-67, tools/ref_c2s.py:38-79) on seeded inputs and commits
 * their outputs; tests/test_oracle_golden.py checks this file against them.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <pthread.h>

/* ---- key packing: src/sparse.cpp:25 ------------------------------------------------
 * key = (u64)(u32)x << 40 | (u64)(u32)y << 20 | (u32)z, computed in 64 bits, so fields
 * overlap for coords outside [0, 2^20); the oracle keeps that aliasing on purpose.
 * With 4 columns (b,x,y,z) the batch is folded into bits 60..63 (XOR), which leaves the
 * key of batch 0 identical to the reference's. */
static inline uint64_t orc_key3(int32_t x, int32_t y, int32_t z) {
    return ((uint64_t)(uint32_t)x << 40) | ((uint64_t)(uint32_t)y << 20) | (uint64_t)(uint32_t)z;
}
static inline uint64_t orc_key_row(const int32_t* c, int stride, int dx, int dy, int dz) {
    if (stride == 4)
        return orc_key3(c[1] + dx, c[2] + dy, c[3] + dz) ^ ((uint64_t)(uint32_t)c[0] << 60);
    return orc_key3(c[0] + dx, c[1] + dy, c[2] + dz);
}

uint64_t orc_key(int32_t b, int32_t x, int32_t y, int32_t z) {
    return orc_key3(x, y, z) ^ ((uint64_t)(uint32_t)b << 60);
}

/* ---- a plain open-addressing map from key to row: stands in for std::unordered_map --- */
typedef struct { uint64_t* keys; int32_t* vals; uint8_t* used; uint64_t mask; } orc_map;

static uint64_t orc_mix(uint64_t k) {   /* murmur3 fmix64 */
    k ^= k >> 33; k *= 0xff51afd7ed558ccdULL; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ULL; k ^= k >> 33;
    return k;
}
static int orc_map_init(orc_map* m, int64_t n) {
    uint64_t cap = 16; while (cap < (uint64_t)(2 * n + 2)) cap <<= 1;
    m->keys = (uint64_t*)malloc(cap * sizeof(uint64_t));
    m->vals = (int32_t*)malloc(cap * sizeof(int32_t));
    m->used = (uint8_t*)calloc(cap, 1);
    m->mask = cap - 1;
    return (m->keys && m->vals && m->used) ? 0 : -1;
}
static void orc_map_free(orc_map* m) { free(m->keys); free(m->vals); free(m->used); }
/* cmap[key] = i  (src/sparse.cpp:26): a later row with the same key overwrites. */
static void orc_map_put(orc_map* m, uint64_t k, int32_t v) {
    uint64_t h = orc_mix(k) & m->mask;
    while (m->used[h] && m->keys[h] != k) h = (h + 1) & m->mask;
    m->used[h] = 1; m->keys[h] = k; m->vals[h] = v;
}
static int32_t orc_map_get(const orc_map* m, uint64_t k, int32_t absent) {
    uint64_t h = orc_mix(k) & m->mask;
    while (m->used[h]) { if (m->keys[h] == k) return m->vals[h]; h = (h + 1) & m->mask; }
    return absent;
}

/* ---- build_neighbor_table: src/sparse.cpp:21-39 ----------------------------------------
 * nbr[t*N + i] = row of coords[i] + (kd-1, kh-1, kw-1) on (x,y,z), t = kd*9 + kh*3 + kw,
 * or N when that voxel is absent. Single-threaded like the reference. Returns 0 or -1. */
int orc_build_neighbor_table(const int32_t* coords, int64_t n, int stride, int32_t* nbr) {
    if (n < 0 || (stride != 3 && stride != 4)) return -1;
    if (n == 0) return 0;
    orc_map m;
    if (orc_map_init(&m, n)) { orc_map_free(&m); return -1; }
    for (int64_t i = 0; i < n; ++i) orc_map_put(&m, orc_key_row(coords + i * stride, stride, 0, 0, 0), (int32_t)i);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* c = coords + i * stride;
        for (int kd = 0; kd < 3; ++kd)
            for (int kh = 0; kh < 3; ++kh)
                for (int kw = 0; kw < 3; ++kw) {
                    int t = kd * 9 + kh * 3 + kw;
                    nbr[(int64_t)t * n + i] = orc_map_get(&m, orc_key_row(c, stride, kd - 1, kh - 1, kw - 1), (int32_t)n);
                }
    }
    orc_map_free(&m);
    return 0;
}

/* ---- submconv_range + sparse_submconv: src/sparse.cpp:64-92 -----------------------------
 * out[i][o] = bias[o] + sum_t sum_c W[o][t][c] * feats[nbr[t*N+i]][c]; sentinel N reads the
 * zero row (submconv_pad, src/sparse.cpp:82-85). feats [N][Ci], W [Co][27][Ci]
 * (tools/convert.py:141-146 layout), out [N][Co]. Accumulates in fp64 on the exact operand
 * values it is given. epi = 1 applies SiLU after the bias. */
int orc_submconv_f64(const int32_t* nbr, int64_t n, const float* feats, int ci,
                     const float* w, const float* bias, int co, int epi, double* out) {
    if (n < 0 || ci <= 0 || co <= 0) return -1;
    double* acc = (double*)malloc(sizeof(double) * (size_t)co);
    if (!acc) return -1;
    for (int64_t i = 0; i < n; ++i) {
        for (int o = 0; o < co; ++o) acc[o] = bias ? (double)bias[o] : 0.0;
        for (int t = 0; t < 27; ++t) {
            int64_t j = nbr[(int64_t)t * n + i];
            if (j < 0 || j >= n) continue;                 /* zero row */
            const float* x = feats + j * ci;
            for (int o = 0; o < co; ++o) {
                const float* wr = w + ((int64_t)o * 27 + t) * ci;
                double s = 0.0;
                for (int c = 0; c < ci; ++c) s += (double)wr[c] * (double)x[c];
                acc[o] += s;
            }
        }
        for (int o = 0; o < co; ++o) {
            double v = acc[o];
            if (epi == 1) v = v / (1.0 + exp(-v));
            out[i * co + o] = v;
        }
    }
    free(acc);
    return 0;
}

/* The same as orc_submconv_f64 for a subset of output rows (rows[k] < n); out is
 * [nrows][Co]. Lets the tests check sampled rows of full-size configurations. */
int orc_submconv_rows_f64(const int32_t* nbr, int64_t n, const int64_t* rows, int64_t nrows,
                          const float* feats, int ci, const float* w, const float* bias, int co,
                          int epi, double* out) {
    if (n < 0 || ci <= 0 || co <= 0) return -1;
    for (int64_t k = 0; k < nrows; ++k) {
        const int64_t i = rows[k];
        if (i < 0 || i >= n) return -1;
        double* acc = out + k * co;
        for (int o = 0; o < co; ++o) acc[o] = bias ? (double)bias[o] : 0.0;
        for (int t = 0; t < 27; ++t) {
            int64_t j = nbr[(int64_t)t * n + i];
            if (j < 0 || j >= n) continue;
            const float* x = feats + j * ci;
            for (int o = 0; o < co; ++o) {
                const float* wr = w + ((int64_t)o * 27 + t) * ci;
                double sum = 0.0;
                for (int c = 0; c < ci; ++c) sum += (double)wr[c] * (double)x[c];
                acc[o] += sum;
            }
        }
        if (epi == 1)
            for (int o = 0; o < co; ++o) acc[o] = acc[o] / (1.0 + exp(-acc[o]));
    }
    return 0;
}

/* ---- the timed CPU baseline: the same loop in fp32 with a blocked GEMM per tap ----------
 * wt is the weight re-laid as [27][Ci][Co] (orc_weight_tap_major) so the inner loop runs
 * over contiguous output channels; the caller picks the thread count. */
void orc_weight_tap_major(const float* w, int ci, int co, float* wt) {
    for (int o = 0; o < co; ++o)
        for (int t = 0; t < 27; ++t)
            for (int c = 0; c < ci; ++c)
                wt[((int64_t)t * ci + c) * co + o] = w[((int64_t)o * 27 + t) * ci + c];
}

typedef struct {
    const int32_t* nbr; int64_t n; const float* feats; int ci; const float* wt;
    const float* bias; int co; int epi; float* out; int64_t i_begin, i_end;
} orc_mt_job;

/* Output rows [i_begin, i_end) in blocks of 32; out row k of the job's range is written to
 * out[(i - row0) * co] where row0 is the first row of the whole call (the caller offsets out). */
static void* orc_mt_worker(void* arg) {
    enum { B = 32 };
    const orc_mt_job* J = (const orc_mt_job*)arg;
    const int64_t n = J->n; const int ci = J->ci, co = J->co;
    float* acc = (float*)malloc(sizeof(float) * (size_t)B * co);
    if (!acc) return (void*)1;
    for (int64_t i0 = J->i_begin; i0 < J->i_end; i0 += B) {
        const int64_t nb = (J->i_end - i0 < B) ? (J->i_end - i0) : B;
        for (int64_t r = 0; r < nb; ++r)
            for (int o = 0; o < co; ++o) acc[r * co + o] = J->bias ? J->bias[o] : 0.f;
        for (int t = 0; t < 27; ++t) {
            const float* wtt = J->wt + (int64_t)t * ci * co;
            for (int64_t r = 0; r < nb; ++r) {
                int64_t j = J->nbr[(int64_t)t * n + i0 + r];
                if (j < 0 || j >= n) continue;
                const float* x = J->feats + j * ci;
                float* a = acc + r * co;
                for (int c = 0; c < ci; ++c) {
                    const float xv = x[c];
                    const float* wr = wtt + (int64_t)c * co;
                    for (int o = 0; o < co; ++o) a[o] += xv * wr[o];
                }
            }
        }
        for (int64_t r = 0; r < nb; ++r)
            for (int o = 0; o < co; ++o) {
                float v = acc[r * co + o];
                if (J->epi == 1) v = v / (1.f + expf(-v));
                J->out[(i0 + r) * co + o] = v;
            }
    }
    free(acc);
    return NULL;
}

/* Rows [row0, row0 + nrows) of the conv over all n voxels (nbr is the full tap-major map,
 * sentinel n), on nthreads pthreads. out points at row 0 of a [n][Co] buffer. */
int orc_submconv_f32_mt_range(const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                              const float* feats, int ci, const float* wt, const float* bias, int co,
                              int epi, float* out, int nthreads) {
    if (n < 0 || ci <= 0 || co <= 0 || row0 < 0 || nrows < 0 || row0 + nrows > n) return -1;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    const int64_t nblk = (nrows + 31) / 32;
    orc_mt_job jobs[256];
    pthread_t th[256];
    int rc = 0;
    for (int k = 0; k < nthreads; ++k) {
        int64_t b0 = nblk * k / nthreads, b1 = nblk * (k + 1) / nthreads;
        int64_t e = row0 + b1 * 32;
        orc_mt_job j = { nbr, n, feats, ci, wt, bias, co, epi, out, row0 + b0 * 32, e < row0 + nrows ? e : row0 + nrows };
        jobs[k] = j;
    }
    for (int k = 1; k < nthreads; ++k)
        if (pthread_create(&th[k], NULL, orc_mt_worker, &jobs[k])) { rc = -1; nthreads = k; break; }
    if (orc_mt_worker(&jobs[0])) rc = -1;
    for (int k = 1; k < nthreads; ++k) { void* r = NULL; pthread_join(th[k], &r); if (r) rc = -1; }
    return rc;
}

int orc_submconv_f32_mt(const int32_t* nbr, int64_t n, const float* feats, int ci,
                        const float* wt, const float* bias, int co, int epi, float* out,
                        int nthreads) {
    return orc_submconv_f32_mt_range(nbr, n, 0, n, feats, ci, wt, bias, co, epi, out, nthreads);
}

/* ---- subdivide: src/sparse.cpp:205-222 ------------------------------------------------
 * for i ascending, octant o ascending, if mask[o + 8i]: emit child
 * (2x + (o&1), 2y + ((o>>1)&1), 2z + ((o>>2)&1)) and gidx = o + 8i; mstart[i] = first child
 * of parent i, mstart[N] = M. With 4 columns the batch column is copied. Returns M. */
int64_t orc_subdivide(const int32_t* coords, int64_t n, int stride, const uint8_t* mask,
                      int32_t* child, int32_t* gidx, int32_t* mstart) {
    int64_t m = 0;
    const int off = (stride == 4) ? 1 : 0;
    for (int64_t i = 0; i < n; ++i) {
        if (mstart) mstart[i] = (int32_t)m;
        const int32_t* c = coords + i * stride;
        for (int o = 0; o < 8; ++o) {
            if (!mask[(int64_t)o + 8 * i]) continue;
            int32_t* d = child + m * stride;
            if (stride == 4) d[0] = c[0];
            d[off + 0] = 2 * c[off + 0] + (o & 1);
            d[off + 1] = 2 * c[off + 1] + ((o >> 1) & 1);
            d[off + 2] = 2 * c[off + 2] + ((o >> 2) & 1);
            if (gidx) gidx[m] = (int32_t)(o + 8 * i);
            ++m;
        }
    }
    if (mstart) mstart[n] = (int32_t)m;
    return m;
}

/* ---- SparseChannel2Spatial gather: src/sparse.cpp:263-266,288 --------------------------
 * src is [N][8*C] (conv1's output, octant o in channels o*C .. o*C+C-1); the free reshape to
 * [8N][C] makes child m take row gidx[m]. */
void orc_c2s_gather(const float* src, const int32_t* gidx, int64_t m, int c, float* out) {
    for (int64_t k = 0; k < m; ++k) memcpy(out + k * c, src + (int64_t)gidx[k] * c, sizeof(float) * (size_t)c);
}

/* Count of (voxel, tap) pairs whose neighbor is present -- the algorithmic work unit. */
int64_t orc_count_valid(const int32_t* nbr, int64_t n) {
    int64_t p = 0;
    for (int64_t k = 0; k < 27 * n; ++k) p += (nbr[k] != (int32_t)n);
    return p;
}

/* ---- dual_grid_to_mesh: src/dual_grid.cpp:16-56 ------------------------------------------
 * f7 [N][7] fp32 per voxel (ggml's [7, N]): channels 0-2 vertex-offset logits, 3-5 the
 * intersected logits of the x, y, z edges, 6 the split-weight logit.
 *   verts[i][a] = ((float)coord[i][a] + (2 sigmoid(f7[i][a]) - 0.5)) * (1 / res) - 0.5
 * For voxel i ascending and axis a ascending, when f7[i][3+a] is not <= 0 and the four voxels
 * coord[i] + ORC_EDGE_OFF[a][k] are all present (rows q0..q3; a later duplicate wins), two
 * triangles: {q0,q1,q2, q0,q2,q3} when softplus(f7[q0][6]) softplus(f7[q2][6]) >
 * softplus(f7[q1][6]) softplus(f7[q3][6]), else {q0,q1,q3, q3,q1,q2}.
 * coords [N][3]; verts [N][3]; faces: room for 6N triangles (18N int32). gap (may be NULL):
 * per emitted quad, |w02 - w13| / max(w02, w13), the margin of its split decision. Returns
 * the triangle count F, or -1 on a failed allocation. */
static const int ORC_EDGE_OFF[3][4][3] = {   /* the quad around each edge axis (o_voxel's table) */
    {{0, 0, 0}, {0, 0, 1}, {0, 1, 1}, {0, 1, 0}},
    {{0, 0, 0}, {1, 0, 0}, {1, 0, 1}, {0, 0, 1}},
    {{0, 0, 0}, {0, 1, 0}, {1, 1, 0}, {1, 0, 0}},
};

static float orc_sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }
static float orc_softplusf(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

int64_t orc_dual_grid_mesh(const int32_t* coords, int64_t n, const float* f7, int res, float* verts,
                           int32_t* faces, float* gap) {
    const float vs = 1.0f / (float)res, org = -0.5f;
    for (int64_t i = 0; i < n; ++i)
        for (int a = 0; a < 3; ++a) {
            const float dv = 2.0f * orc_sigmoidf(f7[7 * i + a]) - 0.5f;
            verts[3 * i + a] = ((float)coords[3 * i + a] + dv) * vs + org;
        }
    if (n == 0) return 0;
    orc_map m;
    if (orc_map_init(&m, n)) { orc_map_free(&m); return -1; }
    for (int64_t i = 0; i < n; ++i) orc_map_put(&m, orc_key_row(coords + 3 * i, 3, 0, 0, 0), (int32_t)i);
    int64_t f = 0, quad = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* c = coords + 3 * i;
        for (int a = 0; a < 3; ++a) {
            if (f7[7 * i + 3 + a] <= 0.0f) continue;
            int32_t q[4];
            int ok = 1;
            for (int k = 0; k < 4 && ok; ++k) {
                q[k] = orc_map_get(&m, orc_key_row(c, 3, ORC_EDGE_OFF[a][k][0], ORC_EDGE_OFF[a][k][1],
                                                   ORC_EDGE_OFF[a][k][2]), -1);
                ok = q[k] >= 0;
            }
            if (!ok) continue;
            const float w02 = orc_softplusf(f7[7 * (int64_t)q[0] + 6]) * orc_softplusf(f7[7 * (int64_t)q[2] + 6]);
            const float w13 = orc_softplusf(f7[7 * (int64_t)q[1] + 6]) * orc_softplusf(f7[7 * (int64_t)q[3] + 6]);
            int32_t* t = faces + 3 * f;
            if (w02 > w13) {
                t[0] = q[0]; t[1] = q[1]; t[2] = q[2]; t[3] = q[0]; t[4] = q[2]; t[5] = q[3];
            } else {
                t[0] = q[0]; t[1] = q[1]; t[2] = q[3]; t[3] = q[3]; t[4] = q[1]; t[5] = q[2];
            }
            if (gap) {
                const float hi = w02 > w13 ? w02 : w13;
                gap[quad] = hi > 0.0f ? fabsf(w02 - w13) / hi : 0.0f;
            }
            f += 2;
            ++quad;
        }
    }
    orc_map_free(&m);
    return f;
}
