// C entry point around the reference's own trellis::dual_grid_to_mesh (src/dual_grid.cpp of
// the reference project, compiled from its sources by `make -C oracle ref REF=<reference>`
// into oracle/_ref/, which is not committed).
//
// TEST INFRASTRUCTURE ONLY: tests/golden/make_mesh_golden.py calls it to write the mesh
// fixtures that pin orc_dual_grid_mesh, and bench.py --op mesh may time it as the CPU
// baseline. Nothing in the product library links or calls it.
#include "dual_grid.h"

#include <cstdint>
#include <cstring>

extern "C" int64_t ref_dual_grid_mesh(const int32_t* coords, int64_t n, const float* f7, int res, float* verts,
                                      int32_t* faces, int64_t max_faces) {
    trellis::ShapeOut so;
    so.res = res;
    so.coords.resize((size_t)n);
    for (int64_t i = 0; i < n; ++i) so.coords[i] = {coords[3 * i], coords[3 * i + 1], coords[3 * i + 2]};
    so.feats7.assign(f7, f7 + 7 * n);
    const trellis::Mesh m = trellis::dual_grid_to_mesh(so);
    std::memcpy(verts, m.verts.data(), m.verts.size() * sizeof(float));
    const int64_t f = m.F();
    if (f <= max_faces) std::memcpy(faces, m.faces.data(), m.faces.size() * sizeof(int32_t));
    return f;
}
