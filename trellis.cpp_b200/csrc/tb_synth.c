/*
 * tb_synth.c -- seeded synthetic voxel sets for the benchmark configurations (host code).
 *
 * The reference publishes no dataset for this path; its own stress test builds a synthetic
 * dense cube (src/test_bigop.cpp:96-106). These generators produce the occupancy patterns
 * the benchmark configurations describe: noisy sphere shells and random boxes. Every
 * decision is a pure function of (coordinate, seed), so the output does not depend on the
 * thread count. Coordinates come out x-major lexicographic (x, then y, then z), the order
 * an argwhere over a dense occupancy grid gives (the sparse-structure decoder's output,
 * src/ss_decoder.cpp:114).
 *
 * Value noise: lattice values v(i) = 2u - 1, with u uniform in [0,1) from splitmix64 of the
 * seeded lattice point. Trilinear interpolation. Three octaves with spacings S, S/2, S/4 and
 * amplitudes 1, 1/2, 1/4, divided by 1.75 so the result lies in [-1, 1].
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint64_t sm64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

static inline uint64_t hash3(int64_t x, int64_t y, int64_t z, uint64_t seed) {
    uint64_t h = sm64(seed);
    h = sm64(h ^ (uint64_t)x);
    h = sm64(h ^ (uint64_t)y);
    return sm64(h ^ (uint64_t)z);
}

static inline double unit(uint64_t h) { return (double)(h >> 11) * (1.0 / 9007199254740992.0); }

static double lattice(int64_t x, int64_t y, int64_t z, uint64_t seed) {
    return 2.0 * unit(hash3(x, y, z, seed)) - 1.0;
}

static double value_noise1(double px, double py, double pz, double spacing, uint64_t seed) {
    const double qx = px / spacing, qy = py / spacing, qz = pz / spacing;
    const double fx0 = floor(qx), fy0 = floor(qy), fz0 = floor(qz);
    const int64_t ix = (int64_t)fx0, iy = (int64_t)fy0, iz = (int64_t)fz0;
    const double fx = qx - fx0, fy = qy - fy0, fz = qz - fz0;
    double c[2][2][2];
    for (int a = 0; a < 2; ++a)
        for (int b = 0; b < 2; ++b)
            for (int d = 0; d < 2; ++d) c[a][b][d] = lattice(ix + a, iy + b, iz + d, seed);
    const double x00 = c[0][0][0] + (c[1][0][0] - c[0][0][0]) * fx;
    const double x01 = c[0][0][1] + (c[1][0][1] - c[0][0][1]) * fx;
    const double x10 = c[0][1][0] + (c[1][1][0] - c[0][1][0]) * fx;
    const double x11 = c[0][1][1] + (c[1][1][1] - c[0][1][1]) * fx;
    const double y0 = x00 + (x10 - x00) * fy;
    const double y1 = x01 + (x11 - x01) * fy;
    return y0 + (y1 - y0) * fz;
}

double tbs_noise(double px, double py, double pz, double spacing0, uint64_t seed) {
    double s = value_noise1(px, py, pz, spacing0, seed)
             + 0.5 * value_noise1(px, py, pz, spacing0 / 2, seed + 1)
             + 0.25 * value_noise1(px, py, pz, spacing0 / 4, seed + 2);
    return s / 1.75;
}

double tbs_keep_u(int64_t x, int64_t y, int64_t z, uint64_t seed) { return unit(hash3(x, y, z, seed ^ 0xA5A5A5A5ULL)); }

/* ---- growable per-thread buffers ------------------------------------------------------ */
typedef struct { int32_t* v; int64_t n, cap; } vec3;
static int vpush(vec3* b, int32_t x, int32_t y, int32_t z) {
    if (b->n == b->cap) {
        int64_t nc = b->cap ? 2 * b->cap : 4096;
        int32_t* nv = (int32_t*)realloc(b->v, (size_t)nc * 3 * sizeof(int32_t));
        if (!nv) return -1;
        b->v = nv; b->cap = nc;
    }
    b->v[3 * b->n] = x; b->v[3 * b->n + 1] = y; b->v[3 * b->n + 2] = z; b->n++;
    return 0;
}

typedef struct {
    int kind;            /* 0 shell, 1 shell band (C1), 2 boxes */
    int res; double R, A, spacing0, thick, rmin, rmax, keep_p; uint64_t seed;
    const uint8_t* occ;  /* boxes: occupancy bitmap res^3 bits */
    int x0, x1; vec3 out; int err;
} job_t;

static void* worker(void* arg) {
    job_t* J = (job_t*)arg;
    const double c = J->res / 2.0;
    for (int x = J->x0; x < J->x1 && !J->err; ++x) {
        const double dx = x - c;
        for (int y = 0; y < J->res && !J->err; ++y) {
            const double dy = y - c;
            if (J->kind == 2) {
                const uint64_t base = ((uint64_t)x * J->res + y) * J->res;
                for (int z = 0; z < J->res; ++z) {
                    const uint64_t b = base + z;
                    if ((J->occ[b >> 3] >> (b & 7)) & 1)
                        if (tbs_keep_u(x, y, z, J->seed) < J->keep_p && vpush(&J->out, x, y, z)) J->err = 1;
                }
                continue;
            }
            const double s = dx * dx + dy * dy;
            const double hi = J->rmax * J->rmax - s;
            if (hi < 0) continue;
            const double lo = J->rmin > 0 ? J->rmin * J->rmin - s : -1.0;
            const double zh = sqrt(hi), zl = lo > 0 ? sqrt(lo) : 0.0;
            /* two z intervals: [c - zh, c - zl] and [c + zl, c + zh] */
            int za = (int)floor(c - zh) - 1, zb = (int)ceil(c - zl) + 1;
            int zc = (int)floor(c + zl) - 1, zd = (int)ceil(c + zh) + 1;
            if (zb >= zc) { zb = zd; zc = zd + 1; }   /* merged interval */
            for (int seg = 0; seg < 2; ++seg) {
                int z0 = seg == 0 ? za : zc, z1 = seg == 0 ? zb : zd;
                if (z0 < 0) z0 = 0;
                if (z1 > J->res - 1) z1 = J->res - 1;
                for (int z = z0; z <= z1; ++z) {
                    const double dz = z - c;
                    const double d = sqrt(s + dz * dz);
                    int keep;
                    if (J->kind == 1) {
                        keep = d >= J->rmin && d < J->rmax && tbs_keep_u(x, y, z, J->seed) < J->keep_p;
                    } else {
                        if (d < J->rmin || d > J->rmax) continue;
                        const double r = J->R + J->A * tbs_noise(x, y, z, J->spacing0, J->seed);
                        keep = fabs(d - r) < J->thick / 2;
                    }
                    if (keep && vpush(&J->out, x, y, z)) J->err = 1;
                }
            }
        }
    }
    return NULL;
}

static int64_t run_jobs(job_t* proto, int nthreads, int32_t** out) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 128) nthreads = 128;
    job_t jobs[128];
    pthread_t th[128];
    for (int k = 0; k < nthreads; ++k) {
        jobs[k] = *proto;
        jobs[k].x0 = (int)((int64_t)proto->res * k / nthreads);
        jobs[k].x1 = (int)((int64_t)proto->res * (k + 1) / nthreads);
        memset(&jobs[k].out, 0, sizeof(vec3));
        jobs[k].err = 0;
    }
    for (int k = 1; k < nthreads; ++k) pthread_create(&th[k], NULL, worker, &jobs[k]);
    worker(&jobs[0]);
    for (int k = 1; k < nthreads; ++k) pthread_join(th[k], NULL);
    int64_t total = 0;
    int err = 0;
    for (int k = 0; k < nthreads; ++k) { total += jobs[k].out.n; err |= jobs[k].err; }
    int32_t* r = err ? NULL : (int32_t*)malloc((size_t)(total > 0 ? total : 1) * 3 * sizeof(int32_t));
    int64_t off = 0;
    for (int k = 0; k < nthreads; ++k) {
        if (r) memcpy(r + 3 * off, jobs[k].out.v, (size_t)jobs[k].out.n * 3 * sizeof(int32_t));
        off += jobs[k].out.n;
        free(jobs[k].out.v);
    }
    *out = r;
    return r ? total : -1;
}

/* Noisy shell: voxels p in [0,res)^3 with | |p - c| - (R + A*noise(p)) | < thick/2,
 * c = (res/2, res/2, res/2). Returns N (or -1) and a malloc'd [N][3] buffer. */
int64_t tbs_shell(int res, double R, double A, double spacing0, uint64_t seed, double thick,
                  int nthreads, int32_t** out) {
    job_t j; memset(&j, 0, sizeof(j));
    j.kind = 0; j.res = res; j.R = R; j.A = A; j.spacing0 = spacing0; j.seed = seed; j.thick = thick;
    j.rmin = R - fabs(A) - thick; j.rmax = R + fabs(A) + thick;
    return run_jobs(&j, nthreads, out);
}

/* Band rmin <= |p - c| < rmax, each voxel kept with probability keep_p. */
int64_t tbs_band(int res, double rmin, double rmax, double keep_p, uint64_t seed, int nthreads, int32_t** out) {
    job_t j; memset(&j, 0, sizeof(j));
    j.kind = 1; j.res = res; j.rmin = rmin; j.rmax = rmax; j.keep_p = keep_p; j.seed = seed;
    return run_jobs(&j, nthreads, out);
}

/* nbox random axis-aligned boxes (edges uniform integers in [emin, emax] per axis, corner
 * uniform so the box fits in the grid), union of their voxels each kept with keep_p. */
int64_t tbs_boxes(int res, int nbox, int emin, int emax, double keep_p, uint64_t seed, int nthreads,
                  int32_t** out) {
    const uint64_t nvox = (uint64_t)res * res * res;
    uint8_t* occ = (uint8_t*)calloc((size_t)((nvox + 7) / 8), 1);
    if (!occ) return -1;
    for (int k = 0; k < nbox; ++k) {
        int e[3], c0[3];
        for (int a = 0; a < 3; ++a) {
            e[a] = emin + (int)(unit(hash3(k, a, 0, seed)) * (emax - emin + 1));
            c0[a] = (int)(unit(hash3(k, a, 1, seed)) * (res - e[a] + 1));
        }
        for (int x = c0[0]; x < c0[0] + e[0]; ++x)
            for (int y = c0[1]; y < c0[1] + e[1]; ++y)
                for (int z = c0[2]; z < c0[2] + e[2]; ++z) {
                    const uint64_t b = ((uint64_t)x * res + y) * res + z;
                    occ[b >> 3] |= (uint8_t)(1u << (b & 7));
                }
    }
    job_t j; memset(&j, 0, sizeof(j));
    j.kind = 2; j.res = res; j.keep_p = keep_p; j.seed = seed; j.occ = occ;
    int64_t n = run_jobs(&j, nthreads, out);
    free(occ);
    return n;
}

/* C3 child mask: for each parent p and octant o, the child q = 2p + bits(o) is kept when its
 * centre, in parent units (q + 0.5) / 2, lies within `half` of the noisy surface
 * R + A*noise. mask is uint8 [n][8]. */
void tbs_child_mask(const int32_t* coords, int64_t n, int stride, int res, double R, double A,
                    double spacing0, uint64_t seed, double half, uint8_t* mask) {
    const double c = res / 2.0;
    const int off = stride == 4 ? 1 : 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t* p = coords + i * stride;
        for (int o = 0; o < 8; ++o) {
            const double qx = (2.0 * p[off] + (o & 1) + 0.5) / 2.0;
            const double qy = (2.0 * p[off + 1] + ((o >> 1) & 1) + 0.5) / 2.0;
            const double qz = (2.0 * p[off + 2] + ((o >> 2) & 1) + 0.5) / 2.0;
            const double d = sqrt((qx - c) * (qx - c) + (qy - c) * (qy - c) + (qz - c) * (qz - c));
            const double r = R + A * tbs_noise(qx, qy, qz, spacing0, seed);
            mask[i * 8 + o] = fabs(d - r) < half ? 1 : 0;
        }
    }
}

void tbs_free(void* p) { free(p); }
