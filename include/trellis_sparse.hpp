// trellis_sparse.hpp -- C++ host mirror of pwilkin/trellis.cpp's include/sparse.h, built on
// the C ABI in tb_sparse.h. A decoder that called the reference's host functions can call
// these with the same arguments. Like the reference, failures throw std::runtime_error.
//
//   build_neighbor_table   include/sparse.h:14-17   (src/sparse.cpp:21-39)
//   sparse_submconv        include/sparse.h:19-22   (src/sparse.cpp:64-92), on host vectors:
//                          the ggml graph builder takes a Model + name prefix, this one takes
//                          the conv's device weights (ConvWeights)
//   subdivide              the octant loop of sparse_c2s (src/sparse.cpp:205-222)
//
// All calls run on device `trellis::set_device()` (default 0) and the legacy stream, and
// return after the result is back on the host.
#pragma once

#include <array>
#include <cstdint>
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

struct SubdivideResult {
    std::vector<std::array<int, 3>> coords;   // children, parent-major, octant ascending
    std::vector<int32_t> gidx;                // o + 8*i: row of the [8N, C] view of conv1
    std::vector<int32_t> mstart;              // [N+1], first child of each parent
};
// mask: uint8 [8*N], mask[o + 8*i] != 0 keeps octant o of parent i.
SubdivideResult subdivide(const std::vector<std::array<int, 3>>& coords, const std::vector<uint8_t>& mask);

}  // namespace trellis
