/*
 * tb_sparse.h -- C ABI of the B200 (sm_100a) sparse submanifold-convolution path.
 *
 * This is the drop-in boundary for the operator layer of pwilkin/trellis.cpp,
 * `include/sparse.h` + `src/sparse.cpp`. Every entry point names the reference symbol it
 * replaces (paths inside that project).
 *
 * Conventions (shared by every call):
 *   - Pointers are DEVICE pointers unless the name ends in `_host`. The caller owns all
 *     memory it passes in. A context may hold device workspace of its own (hash tables,
 *     staging for the `_host` calls), grown on demand and freed by tb_ctx_destroy.
 *   - Layouts follow the reference:
 *       coords   int32 [N][3] = (x,y,z) or [N][4] = (b,x,y,z)     coord_stride 3 or 4
 *       feats    [N][Ci], a voxel's channels contiguous (ggml ne [Ci,N], src/sparse.cpp:66)
 *       weight   [Co][27][Ci] (torch [Co,3,3,3,Ci], tools/convert.py:141-146)
 *       bias     float32 [Co] or NULL
 *       nbr      int32 tap-major [27][N]; nbr[t*N+i] is the row of coords[i] + offset(t),
 *                or N when that voxel is absent. t = kd*9 + kh*3 + kw and
 *                offset = (kd-1, kh-1, kw-1) on (x,y,z)       (include/sparse.h:14-17)
 *   - All calls return tb_status and never throw. A call enqueues work on the context's
 *     stream and returns without synchronising, unless its comment says otherwise.
 *   - One tb_ctx per device and stream. A context is not thread-safe; separate contexts
 *     are.
 */
#ifndef TB_SPARSE_H
#define TB_SPARSE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tb_status {
    TB_OK = 0,
    TB_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad stride, misaligned pointer */
    TB_ERR_UNSUPPORTED = 2,   /* channel count or dtype combination without a kernel */
    TB_ERR_CUDA = 3,          /* a CUDA runtime/driver call failed (see tb_ctx_last_error) */
    TB_ERR_OUT_OF_MEMORY = 4, /* workspace allocation failed */
    TB_ERR_DEVICE = 5,        /* a kernel reported a failed check (bounded wait ran out,
                                 hash probe limit); see tb_ctx_check_device */
    TB_ERR_TOO_LARGE = 6      /* size above a documented maximum */
} tb_status;

typedef enum tb_dtype { TB_F32 = 0, TB_F16 = 1, TB_BF16 = 2 } tb_dtype;

/* Epilogue fused after bias. SILU = x * sigmoid(x) (the ggml_silu that follows the norms in
 * src/sparse.cpp:127,261,293). */
typedef enum tb_epilogue { TB_EPI_NONE = 0, TB_EPI_SILU = 1 } tb_epilogue;

typedef struct tb_ctx tb_ctx;

const char* tb_status_string(tb_status s);
const char* tb_version(void);

/* Create a context on `device`, enqueuing on `stream` (a cudaStream_t; NULL = legacy
 * default stream). No reference counterpart: ggml's backend object plays this role
 * (src/trellis_model.cpp:36-94). */
tb_status tb_ctx_create(int device, void* stream, tb_ctx** out);
tb_status tb_ctx_destroy(tb_ctx* ctx);
tb_status tb_ctx_set_stream(tb_ctx* ctx, void* stream);
/* Human-readable detail of the last failure on this context ("" if none). */
const char* tb_ctx_last_error(const tb_ctx* ctx);
/* Synchronise the stream and report device-side check failures since the last call
 * (TB_OK or TB_ERR_DEVICE; the flag is cleared). */
tb_status tb_ctx_check_device(tb_ctx* ctx);

/* ---- neighbor map -------------------------------------------------------------------
 * Replaces trellis::build_neighbor_table (include/sparse.h:14-17, src/sparse.cpp:21-39).
 * Output is bit-exact with the reference: the same 64-bit key packing (src/sparse.cpp:25),
 * a later duplicate row wins (src/sparse.cpp:26), sentinel N. With coord_stride 4 the
 * batch b is XOR-ed into key bits 60..63, so batch 0 keys equal the reference's.
 * nbr_out: int32 [27*n]. Uses a context-owned hash table of 16*next_pow2(2n) bytes. */
tb_status tb_build_neighbor_map(tb_ctx* ctx, const int32_t* coords, int64_t n,
                                int coord_stride, int32_t* nbr_out);

/* ---- neighbor map without device allocation --------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device memory when they
 * need a map -- a host framework that serves every device buffer from its own pool, or code
 * that must not call cudaMalloc because it can synchronise the device -- this builds exactly
 * the map of tb_build_neighbor_map without a context and without allocating or freeing
 * anything. Its hash table is a static device array inside the library, TB_NOALLOC_SCRATCH
 * bytes, which every GPU that loads the library holds until the process exits.
 *   - n may be at most TB_NOALLOC_MAX_VOXELS; a larger n returns TB_ERR_TOO_LARGE and enqueues
 *     nothing.
 *   - Runs on the calling thread's current device and enqueues on `stream` (a cudaStream_t,
 *     NULL = legacy default stream); returns without synchronising. coords and nbr_out must
 *     be device (or managed) memory of that device, else TB_ERR_INVALID_ARG.
 *   - The first call on a device looks up the array's device address (with that device
 *     current); make that first call before any stream capture. With lazy module loading
 *     (CUDA_MODULE_LOADING=LAZY, the CUDA 12 default) that first lookup also loads the
 *     library's device code on that device, which backs the 16 MiB array and may synchronise
 *     the device: make the first call at start-up, or set CUDA_MODULE_LOADING=EAGER.
 *   - TB_ERR_CUDA reports a failed launch of this call's own kernels only; an error that
 *     earlier, unrelated work left pending is neither reported nor cleared.
 *   - All calls on one device share the single table, and each call clears it before use:
 *     calls that overlap on the GPU (for example on two streams) race and corrupt each
 *     other's maps. Serialise them on one stream. */
#define TB_NOALLOC_MAX_VOXELS 524288
#define TB_NOALLOC_SCRATCH (2 * TB_NOALLOC_MAX_VOXELS * 16 + 256)
tb_status tb_build_neighbor_map_noalloc(void* stream, const int32_t* coords, int64_t n,
                                        int coord_stride, int32_t* nbr_out);

/* Number of (voxel, tap) pairs with a present neighbor in `nbr` (the algorithmic work of
 * one conv). Synchronises the stream. No reference counterpart (instrumentation). */
tb_status tb_count_valid_pairs(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t* pairs);

/* ---- submanifold conv -----------------------------------------------------------------
 * Replaces sparse_submconv (include/sparse.h:19-22, src/sparse.cpp:87-92) and its
 * submconv_range (src/sparse.cpp:64-79):
 *   out[i][o] = epi( bias[o] + sum_t sum_c weight[o][t][c] * feats[nbr[t*n+i]][c] )
 * with absent taps (nbr == n) contributing zero (the padded zero row, src/sparse.cpp:82-85).
 *   dtype TB_BF16 / TB_F16: feats and weight in that type, fp32 accumulation on tcgen05
 *        tensor cores. Needs ci in {16, 32} or a multiple of 64, co a multiple of 16 up
 *        to 256 or a multiple of 256.
 *   dtype TB_F32: fp32 operands and fp32 FFMA accumulation (the precision mode of
 *        g_sparse_cast_f32 / --f32, src/sparse.cpp:16-19). Any ci, co >= 1.
 *   out_dtype: TB_F32 or the operand dtype. Pointers must be 16-byte aligned.
 * `out` must not alias `feats`. */
tb_status tb_submconv(tb_ctx* ctx, const int32_t* nbr, int64_t n,
                      const void* feats, int ci, const void* weight, const float* bias,
                      int co, tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);

/* tb_submconv_range: the output rows [row0, row0 + nrows) of tb_submconv, the reference's
 * submconv_range(r0, nr) (src/sparse.cpp:64-79) used to chunk a conv over voxels. nbr, feats
 * and out are the whole n-row arrays (out [n][co]); only the range's rows of out are written,
 * and its inputs may be any rows of feats. row0 may be any row: the tensor-core kernels run the
 * whole tiles that hold the range and store only its rows. */
tb_status tb_submconv_range(tb_ctx* ctx, const int32_t* nbr, int64_t n, int64_t row0, int64_t nrows,
                            const void* feats, int ci, const void* weight, const float* bias,
                            int co, tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);

/* ---- ConvNeXt block --------------------------------------------------------------------
 * Replaces the per-voxel tail of sparse_convnext (include/sparse.h:23-25,
 * src/sparse.cpp:124-133) after its conv:
 *   out[i] = x[i] + W2 . silu( W1 . LN(h[i]) + b1 ) + b2
 * LN = LayerNorm over the c channels, eps 1e-6, scaled by norm_w and shifted by norm_b
 * (ggml_norm + affine); W1 = mlp.0.weight [4c][c], b1 [4c]; W2 = mlp.2.weight [c][4c], b2 [c].
 * h is the block's conv output [n][c] in TB_F32 or the operand dtype; x is the block input
 * [n][c] in the operand dtype; norm_w, norm_b, b1, b2 are float32.
 *   dtype TB_BF16 / TB_F16: x, W1, W2 in that type, tcgen05 tensor cores with fp32
 *        accumulation; the normalised row and the SiLU activations are rounded to the operand
 *        type before their products (ggml rounds activations to the weight type likewise).
 *        c in {64, 128, 256}: one fused kernel, nothing but x, h and out leaves the SM. Other
 *        c in {16, 32} or a multiple of 64 up to 2048 (the 512 and 1024 of decode_unet): the
 *        same arithmetic as three passes (LayerNorm, mlp.0 + SiLU, mlp.2 + bias + residual; see
 *        tb_layer_norm and tb_linear) with a [n][4c] activation buffer in context workspace.
 *   dtype TB_F32: fp32 throughout on CUDA cores (h and out fp32), any c <= 1024; one block per
 *        row, meant for the precision mode and small n.
 *   out_dtype: TB_F32 or the operand dtype. `out` must not alias h or x. */
tb_status tb_convnext_tail(tb_ctx* ctx, int64_t n, int c, const void* h, tb_dtype h_dtype, const void* x,
                           const float* norm_w, const float* norm_b, const void* w1, const float* b1,
                           const void* w2, const float* b2, tb_dtype dtype, tb_dtype out_dtype, void* out);

/* The whole block, replacing sparse_convnext (include/sparse.h:23-25, src/sparse.cpp:101-137):
 * h = tb_submconv(feats; conv_w, conv_b) into context workspace (fp32), then
 * tb_convnext_tail(h, x = feats). Same dtype rules as the two calls; `out` must not alias feats. */
tb_status tb_sparse_convnext(tb_ctx* ctx, const int32_t* nbr, int64_t n, const void* feats, int c,
                             const void* conv_w, const float* conv_b, const float* norm_w, const float* norm_b,
                             const void* w1, const float* b1, const void* w2, const float* b2, tb_dtype dtype,
                             tb_dtype out_dtype, void* out);

/* Which tensor-core kernel tb_submconv uses for bf16/f16 operands. AUTO picks PAIR when
 * ci == 64 and co is 32 or 64 (CTA pairs with the weights resident in shared memory), BRICK
 * when ci is another multiple of 64 (neighbor rows staged per tile in shared memory, A
 * operands built in TMEM) and GATHER otherwise (per-tap row gathers). Forcing a path that
 * does not support the shape makes tb_submconv return TB_ERR_UNSUPPORTED. No reference
 * counterpart (tuning and testing knob). */
typedef enum tb_conv_path {
    TB_CONV_AUTO = 0, TB_CONV_GATHER = 1, TB_CONV_BRICK = 2, TB_CONV_PAIR = 3
} tb_conv_path;
tb_status tb_ctx_set_conv_path(tb_ctx* ctx, tb_conv_path path);

/* ---- dual-grid mesh extraction (trellis::dual_grid_to_mesh, src/dual_grid.cpp:16-56) ------
 * The decoder head's 7 fields per voxel become a triangle mesh. coords: int32
 * [n][coord_stride] (x,y,z), or (b,x,y,z) with the batch folded into the key as in the
 * neighbor map; feats7: float32 [n][7] (ggml's [7, n]): vertex-offset logits (0-2), the
 * intersected logits of the x, y, z edges (3-5), the split-weight logit (6). All device.
 * verts: float32 [n][3] = (coord + 2 sigmoid(f) - 0.5) * (1 / res) - 0.5 per axis.
 * faces: int32 [max_faces][3] (8-byte aligned): for voxel i ascending and axis x, y, z, when
 * the logit is not <= 0 and the voxel and its three edge neighbours all exist (a later
 * duplicate coordinate wins), the quad's two triangles, split along the diagonal whose
 * corners have the larger product of softplus weights (the 1-3 diagonal on ties).
 * *f_out (host) = F, the triangle count; the call synchronises. TB_ERR_TOO_LARGE (F
 * written, faces incomplete) when F > max_faces; 6n always suffices. res > 0. */
tb_status tb_dual_grid_mesh(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                            const float* feats7, int res, float* verts, int32_t* faces,
                            int64_t max_faces, int64_t* f_out);

/* ---- subdivide and channel-to-spatial gather (sparse_c2s, src/sparse.cpp:172-336) -------
 * tb_subdivide replaces the host octant loop of src/sparse.cpp:205-222: for parent i
 * ascending and octant o ascending with mask[o + 8i] != 0, emit the child
 * (2x + (o&1), 2y + ((o>>1)&1), 2z + ((o>>2)&1)) (batch column copied when stride is 4),
 * gidx = o + 8i, and mstart[i] = index of parent i's first child, mstart[n] = M.
 * mask: uint8 [8n]. child_coords: int32 [max_children][coord_stride], gidx: int32
 * [max_children], mstart: int32 [n+1] (may be NULL). Writes M to *m_out (host) and
 * synchronises. Returns TB_ERR_TOO_LARGE (and writes M) when M > max_children; the
 * outputs are then incomplete. */
tb_status tb_subdivide(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                       const uint8_t* mask, int32_t* child_coords, int32_t* gidx,
                       int32_t* mstart, int64_t max_children, int64_t* m_out);

/* Child m takes row gidx[m] of src viewed as [8n][c]: the SparseChannel2Spatial gather
 * of src/sparse.cpp:263-266,288 (octant o of parent i is channels o*c..o*c+c-1 of conv1's
 * [n][8c] output), and the skip gather of src/sparse.cpp:307 with c = Cin/8.
 * out: [m][c] of `dtype`. */
tb_status tb_c2s_gather(tb_ctx* ctx, const void* src, const int32_t* gidx, int64_t m,
                        int c, tb_dtype dtype, void* out);

/* In-place bias + activation over x [n][c] (the bias add of src/sparse.cpp:78 and the
 * SiLU of src/sparse.cpp:127 as a standalone pass). bias may be NULL. */
tb_status tb_bias_act(tb_ctx* ctx, void* x, int64_t n, int c, const float* bias,
                      tb_dtype dtype, tb_epilogue epi);

/* ---- per-voxel dense layers ---------------------------------------------------------------
 * tb_linear: out[i][j] = act(bias[j] + sum_k a[i][k] * w[j][k]) + res[i][j] for i < m, j < n:
 * the ggml_mul_mat + ggml_add (+ ggml_silu) of decode_unet's from_latent / output_layer
 * (src/shape_decoder.cpp:62-77,84-86,114) and of the ConvNeXt MLP (src/sparse.cpp:127-131).
 * a [m][k] and w [n][k] (torch Linear weight) of dtype; bias float32 [n] or NULL; res [m][n]
 * of res_dtype (TB_F32 or dtype) or NULL, may equal out; act TB_EPI_NONE or TB_EPI_SILU;
 * out [m][n] of out_dtype (TB_F32 or dtype). 16-bit dtypes run on tcgen05 tensor cores (fp32
 * accumulate) and need k a multiple of 64, or 16 or 32; TB_F32 runs on CUDA cores, any k.
 * tb_layer_norm: out = act(LN(x) * w + b), LayerNorm over c channels (c % 8 == 0, <= 2048)
 * with the given eps (1e-6 in the blocks, 1e-5 before decode_unet's output layer,
 * src/shape_decoder.cpp:70); w, b float32 [c], both NULL for no affine. x of x_dtype, out of
 * out_dtype (TB_F32 or x_dtype). */
tb_status tb_linear(tb_ctx* ctx, int64_t m, int k, int n, const void* a, const void* w, const float* bias,
                    const void* res, tb_dtype res_dtype, tb_epilogue act, tb_dtype dtype,
                    tb_dtype out_dtype, void* out);
tb_status tb_layer_norm(tb_ctx* ctx, const void* x, tb_dtype x_dtype, int64_t n, int c, const float* w,
                        const float* b, float eps, tb_epilogue act, tb_dtype out_dtype, void* out);

/* ---- SparseResBlockC2S3d ------------------------------------------------------------------
 * Parameters of one C2S up-block, device pointers named after the reference's tensors under
 * the block prefix (src/sparse.cpp:186-187,259-261,279,316). */
typedef struct tb_c2s_params {
    const float* to_subdiv_w;   /* [8][cin] float32; NULL when an external mask is given */
    const float* to_subdiv_b;   /* [8] float32 or NULL */
    const float* norm1_w;       /* [cin] float32 */
    const float* norm1_b;       /* [cin] float32 */
    const void* conv1_w;        /* [8*cout][27][cin] of dtype */
    const float* conv1_b;       /* [8*cout] float32 or NULL */
    const void* conv2_w;        /* [cout][27][cout] of dtype */
    const float* conv2_b;       /* [cout] float32 or NULL */
} tb_c2s_params;

/* tb_sparse_c2s replaces trellis::sparse_c2s (include/sparse.h:27-35, src/sparse.cpp:172-336)
 * with every step on the device: the to_subdiv logits and their > 0 mask (or ext_mask, uint8
 * [8n], the texture decoder's external mask), the octant subdivide, norm1 (LayerNorm eps 1e-6,
 * affine) + SiLU, conv1 to 8*cout channels (fp32), the channel-to-spatial gather fused with
 * norm2 (no affine) + SiLU, conv2 on the children's neighbor map (fp32), and the skip (x viewed
 * [8n][cin/8], gathered per child and each value repeated cout/(cin/8) times) added in fp32.
 * feats: [n][cin] of dtype (device). Outputs (device): child_coords [max_children][coord_stride]
 * in the reference's order, out [max_children][cout] of out_dtype, mask_out [8n] (may be NULL);
 * *m_out (host) = M, the child count. The call reads M back from the device (one
 * synchronisation between conv1 and the child half). M > max_children returns
 * TB_ERR_TOO_LARGE with *m_out = M (outputs incomplete; 8n always suffices).
 * Needs cin % 8 == 0, cout a multiple of cin/8 and of 8, cin, cout <= 2048, and both convs
 * supported by tb_submconv for dtype. */
tb_status tb_sparse_c2s(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                        const void* feats, int cin, int cout, const tb_c2s_params* params,
                        const uint8_t* ext_mask, tb_dtype dtype, tb_dtype out_dtype,
                        int64_t max_children, int32_t* child_coords, void* out, uint8_t* mask_out,
                        int64_t* m_out);

/* tb_sort_rows: perm (device int32 [n]) lists the rows in ascending lexicographic order of their
 * (b, x, y, z) coordinates (signed; for non-negative coordinates the order of the reference's
 * voxel key, src/sparse.cpp:25), stably (equal coordinates keep their input order).
 * No reference counterpart: the reference's decoder keeps the subdivide's parent-major row order
 * (src/sparse.cpp:205-222). The conv kernels read each 128-row tile's neighbours as three
 * contiguous row ranges only in this order, so a caller that holds rows in another order can
 * gather them into it (tb_gather_rows) for a stage's map and convs and scatter the results back
 * (tb_scatter_rows). One small read-back of the coordinate bounds (synchronises the context's
 * stream). When the key span needs more than 63 bits the rows keep their order (perm = 0..n-1). */
tb_status tb_sort_rows(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride, int32_t* perm);

/* ---- host-buffer end-to-end call --------------------------------------------------------
 * Mirrors one decoder stage graph run (run1 / GraphRun::run: upload inputs, compute, read
 * back; src/shape_decoder.cpp:34-51, src/sparse.cpp:145-169), without the LayerNorm/MLP
 * tail. It copies coords_host and feats_host to the device, builds the neighbor map, runs
 * `nlayers` stacked submanifold convs (layer l reads layer l-1's output) and copies the
 * last output to out_host. Weights and biases are DEVICE pointers: they are resident
 * model parameters, as in the reference's backend buffer. Intermediate outputs use
 * `dtype`; the last layer writes `out_dtype`. Synchronises before returning. Host
 * buffers may be pageable; pinned buffers copy faster, and with pinned buffers the call
 * overlaps its transfers with the convs: after the coordinates and the map, the features go
 * up in row chunks on a copy stream, each chunk's conv of each layer starts once the input
 * rows it reads (found from the map) are on the device, and each finished chunk of the last
 * layer goes down on a second copy stream while later chunks still compute or upload. */
typedef struct tb_conv_layer {
    const void* weight;   /* [co][27][ci] of dtype, device */
    const float* bias;    /* [co] float32, device, or NULL */
    int ci;
    int co;
    tb_epilogue epi;
} tb_conv_layer;

tb_status tb_submconv_stack_host(tb_ctx* ctx, const int32_t* coords_host, int64_t n,
                                 int coord_stride, const void* feats_host,
                                 const tb_conv_layer* layers, int nlayers, tb_dtype dtype,
                                 tb_dtype out_dtype, void* out_host);

/* ---- multi-GPU z-slab sharding (no reference counterpart: the reference is single-GPU,
 * it only chunks output ranges on one device, src/sparse.cpp:94-118) -----------------------
 * tb_zslab_counts: histogram of voxels per z plane, counts[z - z_min] for z in
 * [z_min, z_min + nz); voxels outside the range are ignored. counts is int64 [nz], zeroed by
 * the call.
 * tb_gather_rows: out[k] = src[rows[k]] for k < m, row_bytes per row (halo packing and
 * owned-row extraction). tb_scatter_rows: out[rows[k]] = src[k] (received halo rows into
 * their local positions). row_bytes must be a multiple of 4. */
tb_status tb_zslab_counts(tb_ctx* ctx, const int32_t* coords, int64_t n, int coord_stride,
                          int32_t z_min, int32_t nz, int64_t* counts);
tb_status tb_gather_rows(tb_ctx* ctx, const void* src, const int32_t* rows, int64_t m,
                         int64_t row_bytes, void* out);
tb_status tb_scatter_rows(tb_ctx* ctx, const void* src, const int32_t* rows, int64_t m,
                          int64_t row_bytes, void* out);

/* ---- multi-GPU sharded convs: z-slabs with an NCCL halo -----------------------------------
 * No reference counterpart: the reference is single-GPU (src/sparse.cpp:94-118 only chunks
 * output rows on one device). These calls let its per-stage caller (src/shape_decoder.cpp:91-113:
 * build_neighbor_table, then the stage's sparse_submconv calls) run one process per GPU: each rank
 * partitions the stage's voxels, builds the map of its slab and runs each conv on its owned rows,
 * with the halo exchanged inside the conv call. Callable from C/C++ without torch.
 *
 * tb_nccl_unique_id / tb_nccl_comm_create / tb_nccl_comm_destroy: a communicator for callers
 *   that have none (rank 0 makes the 128-byte id, every rank receives it out of band, e.g. over
 *   torch.distributed or MPI). NCCL is loaded at run time (libnccl.so.2, the copy already in the
 *   process when there is one); TB_ERR_UNSUPPORTED where it cannot be loaded. A communicator
 *   passed to tb_dist_create must come from that same library.
 * tb_dist_create: a sharding handle on ctx's device for `rank` of `world` (nccl_comm: an
 *   ncclComm_t of `world` ranks). The dist enqueues on ctx's stream and on a communication
 *   stream of its own; it owns neither ctx nor the communicator. With nccl_comm NULL nothing is
 *   exchanged: the caller puts the halo rows into feats before each tb_dist_submconv (one process
 *   driving several slabs, or world == 1).
 * tb_dist_set_halo_planes: H, the planes of each neighbour a rank holds (1 by default, at most
 *   TB_DIST_MAX_HALO); set before tb_dist_partition_zslab. A conv at an owned voxel reads one
 *   plane beyond the slab; a stack of L convs whose intermediate results are not exchanged
 *   (tb_dist_submconv_grow) reads L planes beyond it.
 * tb_dist_partition_zslab: every rank passes the same voxel set (device coords [n][stride]). The
 *   z axis is cut into `world` slabs of whole planes at voxel-count quantiles (tb_zslab_cuts);
 *   this rank owns z_lo <= z < z_hi and holds the neighbours' planes z_lo-H .. z_lo-1 and
 *   z_hi .. z_hi+H-1 as a halo. Its local rows are [lower halo planes | owned planes | upper halo
 *   planes], in z order and within a plane in the input's order, so the owned rows are local rows
 *   [owned_begin, owned_begin + n_owned). Synchronises (two small read-backs). Fails when the
 *   voxels span fewer z planes than ranks, and with TB_ERR_UNSUPPORTED when H > 1 and a slab
 *   holds fewer than H planes (its neighbours' halos would reach past it).
 * tb_dist_local_rows: the global row of every local row (device int32 [n_local]), to gather a
 *   stage's features into local order (tb_gather_rows) and scatter owned outputs back.
 * tb_dist_load_coords: replace the local coordinates with coords_local (device [n_local][stride],
 *   the local rows' coordinates in local order, e.g. uploaded from a host copy); the next
 *   tb_dist_build_map uses them.
 * tb_dist_build_map: the neighbor map of the local rows (dist-owned), tb_build_neighbor_map's map
 *   of those rows up to a relabelling of taps (it is built on (z, x, y); tb_dist_submconv
 *   permutes the weight's taps to match).
 * tb_dist_submconv: one conv of tb_submconv's semantics on the local rows: feats [n_local][ci]
 *   holds the input's owned rows; the call fills its halo rows from the neighbours (NCCL send/recv
 *   of the edge planes, on the communication stream) while the interior planes are computed, then
 *   computes the edge planes. out [n_local][co]: owned rows written, halo rows untouched;
 *   feats's halo rows are overwritten. Same dtype and shape rules as tb_submconv. Rows match the
 *   single-GPU conv up to fp32 accumulation order.
 * tb_dist_exchange: the halo exchange alone: feats [n_local] rows of row_bytes (a multiple of
 *   16) get the neighbours' edge planes in their halo rows. Enqueued on the communication stream
 *   after the work already on ctx's stream, so work enqueued next on ctx's stream (the map build)
 *   overlaps it; the next conv on the dist waits for it.
 * tb_dist_local_weight: the weight [co][27][ci] with its taps in the local map's order (the
 *   permutation tb_dist_submconv applies on every call), for tb_dist_submconv_grow.
 * tb_dist_submconv_grow: a conv with no exchange over the owned rows and the `grow` halo planes
 *   nearest the slab on each side (0 <= grow < H); feats's rows those outputs read -- up to grow + 1
 *   halo planes -- must hold the neighbours' rows (tb_dist_exchange, or an earlier
 *   tb_dist_submconv_grow with a larger grow). weight_local from tb_dist_local_weight. Other rows
 *   of out are untouched. A stack of L convs then needs one exchange of L planes: conv l runs with
 *   grow = L - 1 - l, recomputing the halo rows the next conv reads instead of exchanging them.
 * tb_dist_count_valid_pairs: present (voxel, tap) pairs over the owned rows; synchronises.
 * tb_dist_local_map: the dist-owned local map (device int32 [27][n_local]) after build_map. */
typedef struct tb_dist tb_dist;
typedef struct tb_zslab {
    int32_t z_lo, z_hi;             /* owned planes: z_lo <= z < z_hi */
    int64_t n_local;                /* local rows: lower halo planes, owned planes, upper halo planes */
    int64_t n_owned;
    int64_t owned_begin;            /* owned rows are local rows [owned_begin, owned_begin + n_owned) */
    int64_t n_halo_lo, n_halo_hi;   /* rows of planes z_lo-H .. z_lo-1 and z_hi .. z_hi+H-1 (received) */
    int64_t n_edge_lo, n_edge_hi;   /* rows of planes z_lo .. z_lo+H-1 and z_hi-H .. z_hi-1 (sent) */
} tb_zslab;
#define TB_DIST_MAX_HALO 8

tb_status tb_nccl_unique_id(uint8_t* id /* [128] */);
tb_status tb_nccl_comm_create(const uint8_t* id /* [128] */, int rank, int world, int device, void** comm);
tb_status tb_nccl_comm_destroy(void* comm);
tb_status tb_dist_create(tb_ctx* ctx, void* nccl_comm, int rank, int world, tb_dist** out);
tb_status tb_dist_destroy(tb_dist* d);
const char* tb_dist_last_error(const tb_dist* d);
tb_status tb_dist_set_halo_planes(tb_dist* d, int planes);
tb_status tb_dist_partition_zslab(tb_dist* d, const int32_t* coords, int64_t n, int coord_stride, tb_zslab* slab);
tb_status tb_dist_local_rows(tb_dist* d, int32_t* rows);
tb_status tb_dist_load_coords(tb_dist* d, const int32_t* coords_local);
tb_status tb_dist_build_map(tb_dist* d);
tb_status tb_dist_local_map(const tb_dist* d, const int32_t** nbr);
tb_status tb_dist_submconv(tb_dist* d, void* feats, int ci, const void* weight, const float* bias, int co,
                           tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi, void* out);
tb_status tb_dist_exchange(tb_dist* d, void* feats, int64_t row_bytes);
tb_status tb_dist_local_weight(tb_dist* d, const void* weight, int ci, int co, tb_dtype dtype, void* weight_local);
tb_status tb_dist_submconv_grow(tb_dist* d, int grow, const void* feats, int ci, const void* weight_local,
                                const float* bias, int co, tb_dtype dtype, tb_dtype out_dtype, tb_epilogue epi,
                                void* out);
tb_status tb_dist_count_valid_pairs(tb_dist* d, int64_t* pairs);
/* The slab cut on the host (what tb_dist_partition_zslab computes from its histogram): counts
 * [nz] = voxels of plane z_min + i; cuts [world + 1]: cuts[0] the first occupied plane,
 * cuts[world] one past the last, slab r = [cuts[r], cuts[r+1]) with at least one plane each.
 * TB_ERR_INVALID_ARG when the occupied range has fewer planes than ranks. */
tb_status tb_zslab_cuts(const int64_t* counts, int32_t nz, int32_t z_min, int world, int32_t* cuts);

/* ---- model and input files, read without ggml --------------------------------------------
 * GGUF checkpoints as the reference's tools/convert.py writes them and src/trellis_model.cpp:96-137
 * loads them (conv / linear weights F16, 1-D parameters F32, names kept verbatim; a sparse conv
 * weight has ne = (Ci, 27, Co), the bytes of the [Co][27][Ci] layout tb_submconv takes), and the
 * hr_slat.bin decode input of src/decode_replay.cpp:19-28. Host-only calls report failures
 * through tb_io_last_error() (per thread); tb_gguf_upload_tensor reports on its context.
 *   tb_gguf_open / tb_gguf_close: parse the header, metadata and tensor infos (GGUF v2/v3).
 *   tb_gguf_find_tensor: index of a tensor by name, or -1.
 *   tb_gguf_tensor_info: name, ggml type (0 F32, 1 F16, 30 BF16, others listed but not read),
 *     n_dims, ne[4] (innermost first, unused dims 1) and byte size (0 for unreadable types).
 *   tb_gguf_get_string: a string metadata value (e.g. "general.architecture",
 *     "trellis.config_json"), or NULL.
 *   tb_gguf_read_tensor: the raw bytes into a host buffer of exactly `nbytes`.
 *   tb_gguf_upload_tensor: into device memory as `dtype` (F32/F16/BF16 converted on the device,
 *     rounding to nearest even). Synchronises.
 *   tb_slat_read: N and res, then (when the pointers are non-NULL) coords int32 [N][3] and
 *     feats float32 [N][32]; call once with NULL buffers to learn N. */
typedef struct tb_gguf tb_gguf;
tb_status tb_gguf_open(const char* path, tb_gguf** out);
void tb_gguf_close(tb_gguf* g);
int64_t tb_gguf_n_tensors(const tb_gguf* g);
int64_t tb_gguf_find_tensor(const tb_gguf* g, const char* name);
tb_status tb_gguf_tensor_info(const tb_gguf* g, int64_t i, const char** name, int32_t* ggml_type,
                              int32_t* n_dims, int64_t* ne, uint64_t* nbytes);
const char* tb_gguf_get_string(const tb_gguf* g, const char* key);
tb_status tb_gguf_read_tensor(const tb_gguf* g, int64_t i, void* dst, uint64_t nbytes);
tb_status tb_gguf_upload_tensor(tb_ctx* ctx, const tb_gguf* g, int64_t i, tb_dtype dtype, void* dst);
tb_status tb_slat_read(const char* path, int64_t* n, int32_t* res, int32_t* coords, float* feats);
const char* tb_io_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* TB_SPARSE_H */
