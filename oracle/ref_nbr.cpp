// C entry point around the reference's own trellis::build_neighbor_table (src/sparse.cpp:21-39
// of the reference project). The function is taken from that file at build time by
// oracle/extract_ref_function.py (the rest of the file needs ggml, which is absent) and compiled
// with this wrapper by `make -C oracle ref REF=<reference>` into oracle/_ref/, not committed.
//
// TEST INFRASTRUCTURE ONLY: tests pin the oracle's and the GPU's maps to it, and bench.py's CPU
// baseline times it (single-threaded, as the reference runs it). Nothing in the product library
// links or calls it.
#include <array>
#include <cstdint>
#include <cstring>
#include <vector>

namespace trellis {
std::vector<int32_t> build_neighbor_table(const std::vector<std::array<int, 3>>& coords);
}

// coords: int32 [n][stride] with (x, y, z) in the last three columns; nbr: int32 [27 n].
extern "C" int ref_build_neighbor_table(const int32_t* coords, int64_t n, int stride, int32_t* nbr) {
    if (n < 0 || (stride != 3 && stride != 4)) return 1;
    std::vector<std::array<int, 3>> c((size_t)n);
    const int o = stride - 3;
    for (int64_t i = 0; i < n; ++i) c[(size_t)i] = {coords[i * stride + o], coords[i * stride + o + 1], coords[i * stride + o + 2]};
    const std::vector<int32_t> t = trellis::build_neighbor_table(c);
    std::memcpy(nbr, t.data(), t.size() * sizeof(int32_t));
    return 0;
}
