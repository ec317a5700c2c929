// trellis_sparse.hpp -- C++ host mirror of pwilkin/trellis.cpp's include/sparse.h, built on
// the C ABI in tb_sparse.h. A decoder that called the reference's host functions can call
// these with the same arguments. Like the reference, failures throw std::runtime_error.
//
//   build_neighbor_table   include/sparse.h:14-17   (src/sparse.cpp:21-39)
//   sparse_submconv        include/sparse.h:19-22   (src/sparse.cpp:64-92), on host vectors:
//                          the ggml graph builder takes a Model + name prefix, this one takes
//                          the conv's device weights (ConvWeights)
//   sparse_convnext        include/sparse.h:23-25 (src/sparse.cpp:94-137), on host vectors,
//                          with the block's device weights (ConvNeXtWeights)
//   subdivide              the octant loop of sparse_c2s (src/sparse.cpp:205-222)
//   GgufModel              the Model of src/trellis_model.cpp:96-137: a GGUF checkpoint's
//                          tensors on the device, looked up by the reference's names; its
//                          conv(), convnext() and c2s() give the weights of a block prefix
//   read_slat              the hr_slat.bin decode input of src/decode_replay.cpp:19-28
//   dual_grid_to_mesh      src/dual_grid.cpp:16-56, the decoder head's fields to a mesh
//   shape_decode, shape_upsample, tex_decode
//                          include/shape_decoder.h: decode_unet (src/shape_decoder.cpp:79-138),
//                          every stage on the device
//   sparse_c2s             include/sparse.h:27-35 (src/sparse.cpp:172-336), the whole
//                          SparseResBlockC2S3d; the block's device weights (C2SWeights) take
//                          the place of Model + prefix
//
// All calls run on device `trellis::set_device()` (default 0) and the legacy stream, and
// return after the result is back on the host.
#pragma once

#include <array>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "tb_sparse.h"

namespace trellis {

void set_device(int device);

// Tap-major int32 [27*N]; nbr[t*N+i] = row of coords[i] + (kd-1,kh-1,kw-1), or N if absent.
std::vector<int32_t> build_neighbor_table(const std::vector<std::array<int, 3>>& coords);

// One conv's parameters, resident on the device (the reference keeps them in the model's
// backend buffer): weight [co][27][ci] of `dtype`, bias float32 [co] or nullptr.
struct ConvWeights {
    const void* weight = nullptr;
    const float* bias = nullptr;
    int ci = 0;
    int co = 0;
    tb_dtype dtype = TB_BF16;
};

// feats: [N][Ci] float32 (ggml's channel-major [Ci, N]); nbr from build_neighbor_table.
// Returns [N][Co] float32. With a bf16/f16 `w.dtype` the features are rounded to that type
// (round to nearest even) before the tensor-core conv, as ggml rounds activations to the
// weight's type.
std::vector<float> sparse_submconv(const ConvWeights& w, const std::vector<float>& feats,
                                   const std::vector<int32_t>& nbr, int N,
                                   tb_epilogue epi = TB_EPI_NONE);

// One ConvNeXt block's parameters on the device: the conv, norm (LayerNorm affine, float32
// [C]), mlp.0 ([4C][C] of conv.dtype, bias float32 [4C]) and mlp.2 ([C][4C], bias [C]).
struct ConvNeXtWeights {
    ConvWeights conv;
    const float* norm_w = nullptr;
    const float* norm_b = nullptr;
    const void* mlp0_w = nullptr;
    const float* mlp0_b = nullptr;
    const void* mlp2_w = nullptr;
    const float* mlp2_b = nullptr;
};

// feats: [N][C] float32 (rounded to conv.dtype when that is bf16/f16); returns [N][C] float32:
// conv -> LayerNorm (eps 1e-6) -> Linear C->4C -> SiLU -> Linear 4C->C -> + feats.
std::vector<float> sparse_convnext(const ConvNeXtWeights& w, const std::vector<float>& feats,
                                   const std::vector<int32_t>& nbr, int N);

struct SubdivideResult {
    std::vector<std::array<int, 3>> coords;   // children, parent-major, octant ascending
    std::vector<int32_t> gidx;                // o + 8*i: row of the [8N, C] view of conv1
    std::vector<int32_t> mstart;              // [N+1], first child of each parent
};
// mask: uint8 [8*N], mask[o + 8*i] != 0 keeps octant o of parent i.
SubdivideResult subdivide(const std::vector<std::array<int, 3>>& coords, const std::vector<uint8_t>& mask);

// The reference's C2SResult (include/sparse.h:31): feats [M][C] float32 (ggml's [C, M]),
// the children's coordinates, C, and the [8N] mask actually used.
struct C2SResult {
    std::vector<float> feats;
    std::vector<std::array<int, 3>> coords;
    int C = 0;
    std::vector<uint8_t> subdiv;
};

// One C2S block's parameters, resident on the device (tb_c2s_params: to_subdiv, norm1, conv1,
// conv2 under the block prefix); conv weights of `dtype`.
struct C2SWeights {
    tb_c2s_params p{};
    tb_dtype dtype = TB_BF16;
};

// feats_in: [N][Cin] float32. ext_subdiv: a [8N] mask (the texture decoder's guide), or
// nullptr to predict it with to_subdiv. With a bf16/f16 `w.dtype` the input is rounded to that
// type first. Output features are float32.
C2SResult sparse_c2s(const C2SWeights& w, const std::vector<float>& feats_in, int Cin,
                     const std::vector<std::array<int, 3>>& coords, int Cout,
                     const std::vector<uint8_t>* ext_subdiv = nullptr);

// A GGUF checkpoint (tools/convert.py's output) on device `device`. Every F32/F16/BF16 tensor is
// uploaded: tensors of two or more dims (conv and linear weights) as `weight_dtype`, 1-D tensors
// and the C2S `to_subdiv.weight` as float32, the types the kernels take. Move-only; frees its
// device memory when destroyed.
class GgufModel {
public:
    static GgufModel load(const std::string& path, int device = 0, tb_dtype weight_dtype = TB_BF16);
    GgufModel() = default;
    GgufModel(GgufModel&& o) noexcept;
    GgufModel& operator=(GgufModel&& o) noexcept;
    GgufModel(const GgufModel&) = delete;
    GgufModel& operator=(const GgufModel&) = delete;
    ~GgufModel();

    bool has(const std::string& name) const { return t_.count(name) != 0; }
    const void* get(const std::string& name) const;                 // throws if absent
    std::vector<int64_t> shape(const std::string& name) const;      // torch order
    // prefix.weight [Co,27,Ci] + prefix.bias (src/sparse.cpp:87-92)
    ConvWeights conv(const std::string& prefix) const;
    // prefix.conv, prefix.norm, prefix.mlp.0, prefix.mlp.2 (src/sparse.cpp:104-133)
    ConvNeXtWeights convnext(const std::string& prefix) const;
    // prefix.to_subdiv (absent in the texture decoder), norm1, conv1, conv2 (src/sparse.cpp:186-316)
    C2SWeights c2s(const std::string& prefix) const;

    std::string arch;           // general.architecture
    std::string config_json;    // trellis.config_json
    tb_dtype weight_dtype = TB_BF16;

private:
    struct Tensor {
        void* dev = nullptr;
        tb_dtype dtype = TB_F32;
        std::vector<int64_t> shape;
    };
    std::unordered_map<std::string, Tensor> t_;
    int device_ = 0;
};

// The hr_slat.bin dump (src/decode_replay.cpp:19-28): coords, feats [N][32] and the resolution.
struct SlatInput {
    std::vector<std::array<int, 3>> coords;
    std::vector<float> feats;
    int res = 0;
};
SlatInput read_slat(const std::string& path);

// The reference's ShapeOut (include/shape_decoder.h): per-voxel output fields [M][7] (ggml's
// [7, M]), the final coordinates, the resolution and the per-stage subdivision masks.
struct ShapeOut {
    std::vector<float> feats7;
    std::vector<std::array<int, 3>> coords;
    int res = 512;
    std::vector<std::vector<uint8_t>> subs;
};

// decode_unet (src/shape_decoder.cpp:79-117) on the device: from_latent, then per stage the
// neighbor map, the stage's ConvNeXt blocks and its C2S up-block, then LayerNorm (eps 1e-5, no
// affine) and output_layer. The stage layout (widths, block counts) is read from the
// checkpoint's tensor names and shapes: blocks.<s>.<j>.conv.* are the ConvNeXt blocks of stage
// s and blocks.<s>.<nblk>.* its C2S block, as in the reference's stage table
// (src/shape_decoder.cpp:88). latent: [N0][32] float32.
ShapeOut shape_decode(const GgufModel& m, const std::vector<float>& latent,
                      const std::vector<std::array<int, 3>>& coords0, int resolution = 512);
std::vector<std::array<int, 3>> shape_upsample(const GgufModel& m, const std::vector<float>& latent,
                                               const std::vector<std::array<int, 3>>& coords0);
std::vector<float> tex_decode(const GgufModel& m, const std::vector<float>& tex_latent,
                              const std::vector<std::array<int, 3>>& coords0,
                              const std::vector<std::vector<uint8_t>>& subs);

// The reference's Mesh (include/dual_grid.h): verts [V*3] float32, faces [F*3] int32.
struct Mesh {
    std::vector<float> verts;
    std::vector<int32_t> faces;
    int V() const { return (int)verts.size() / 3; }
    int F() const { return (int)faces.size() / 3; }
};

// dual_grid_to_mesh (src/dual_grid.cpp:16-56) on the device: one dual vertex per voxel in the
// world cube [-0.5, 0.5]^3 and two triangles per intersected edge whose four voxels exist, in
// the reference's order (tb_dual_grid_mesh).
Mesh dual_grid_to_mesh(const ShapeOut& so);

}  // namespace trellis
