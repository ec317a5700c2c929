// C++ host mirror of the reference's sparse.h host functions, over the C ABI (see
// include/trellis_sparse.hpp). Uploads host inputs, runs the device path, reads back.
#include "trellis_sparse.hpp"

#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

namespace trellis {
namespace {

int g_device = 0;

struct Ctx {
    tb_ctx* ctx = nullptr;
    explicit Ctx(int dev) {
        if (tb_ctx_create(dev, nullptr, &ctx) != TB_OK) throw std::runtime_error("trellis: tb_ctx_create failed");
    }
    ~Ctx() { tb_ctx_destroy(ctx); }
};

tb_ctx* ctx() {
    thread_local std::unique_ptr<Ctx> c;
    thread_local int dev = -1;
    if (!c || dev != g_device) {
        c.reset();
        c.reset(new Ctx(g_device));
        dev = g_device;
    }
    return c->ctx;
}

void ok(tb_status s, const char* what) {
    if (s != TB_OK)
        throw std::runtime_error(std::string("trellis: ") + what + ": " + tb_status_string(s) + " (" +
                                 tb_ctx_last_error(ctx()) + ")");
}

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("trellis: ") + what + ": " + cudaGetErrorString(e));
}

// Device buffer owned by the caller's scope.
struct DBuf {
    void* p = nullptr;
    explicit DBuf(size_t bytes) { cuda_ok(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc"); }
    ~DBuf() { cudaFree(p); }
    template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);   // NaN
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// IEEE binary32 -> binary16, round to nearest even (subnormals and overflow included).
uint16_t f32_to_f16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t absu = u & 0x7FFFFFFFu;
    if (absu >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (absu > 0x7F800000u ? 0x200u : 0u));
    if (absu >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);   // rounds to >= 65520: inf
    const int exp = (int)(absu >> 23) - 127;
    if (exp >= -14) {   // normal half
        uint32_t mant = absu & 0x7FFFFFu;
        uint32_t h = ((uint32_t)(exp + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    if (exp < -25) return (uint16_t)sign;   // below half the smallest subnormal
    // subnormal: value = mant_full * 2^(exp-23), half subnormal unit = 2^-24
    const uint32_t mant_full = (absu & 0x7FFFFFu) | 0x800000u;
    const int drop = -exp - 1;              // right shift that lands on 2^-24 units (14..24)
    uint32_t h = mant_full >> drop;
    const uint32_t rem = mant_full & ((1u << drop) - 1u);
    const uint32_t halfway = 1u << (drop - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

}  // namespace

void set_device(int device) { g_device = device; }

std::vector<int32_t> build_neighbor_table(const std::vector<std::array<int, 3>>& coords) {
    const int64_t n = (int64_t)coords.size();
    std::vector<int32_t> nbr((size_t)27 * n);
    if (n == 0) return nbr;
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    DBuf dc((size_t)n * 12), dn((size_t)n * 27 * 4);
    cuda_ok(cudaMemcpy(dc.p, coords.data(), (size_t)n * 12, cudaMemcpyHostToDevice), "upload coords");
    ok(tb_build_neighbor_map(ctx(), dc.as<int32_t>(), n, 3, dn.as<int32_t>()), "tb_build_neighbor_map");
    cuda_ok(cudaMemcpy(nbr.data(), dn.p, nbr.size() * 4, cudaMemcpyDeviceToHost), "download nbr");
    ok(tb_ctx_check_device(ctx()), "neighbor map device check");
    return nbr;
}

std::vector<float> sparse_submconv(const ConvWeights& w, const std::vector<float>& feats,
                                   const std::vector<int32_t>& nbr, int N, tb_epilogue epi) {
    if ((int64_t)feats.size() != (int64_t)N * w.ci || (int64_t)nbr.size() != (int64_t)27 * N)
        throw std::runtime_error("trellis: sparse_submconv: feats/nbr size mismatch");
    std::vector<float> out((size_t)N * w.co);
    if (N == 0) return out;
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    const size_t es = w.dtype == TB_F32 ? 4 : 2;
    DBuf df((size_t)N * w.ci * es), dn((size_t)N * 27 * 4), dout((size_t)N * w.co * 4);
    if (w.dtype == TB_F32) {
        cuda_ok(cudaMemcpy(df.p, feats.data(), feats.size() * 4, cudaMemcpyHostToDevice), "upload feats");
    } else {
        std::vector<uint16_t> h(feats.size());
        for (size_t k = 0; k < feats.size(); ++k)
            h[k] = w.dtype == TB_BF16 ? f32_to_bf16_rne(feats[k]) : f32_to_f16_rne(feats[k]);
        cuda_ok(cudaMemcpy(df.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "upload feats");
    }
    cuda_ok(cudaMemcpy(dn.p, nbr.data(), nbr.size() * 4, cudaMemcpyHostToDevice), "upload nbr");
    ok(tb_submconv(ctx(), dn.as<int32_t>(), N, df.p, w.ci, w.weight, w.bias, w.co, w.dtype, TB_F32, epi, dout.p),
       "tb_submconv");
    cuda_ok(cudaMemcpy(out.data(), dout.p, out.size() * 4, cudaMemcpyDeviceToHost), "download out");
    ok(tb_ctx_check_device(ctx()), "conv device check");
    return out;
}

std::vector<float> sparse_convnext(const ConvNeXtWeights& w, const std::vector<float>& feats,
                                   const std::vector<int32_t>& nbr, int N) {
    const int c = w.conv.ci;
    if (w.conv.co != c) throw std::runtime_error("trellis: sparse_convnext: the conv must keep the width");
    if ((int64_t)feats.size() != (int64_t)N * c || (int64_t)nbr.size() != (int64_t)27 * N)
        throw std::runtime_error("trellis: sparse_convnext: feats/nbr size mismatch");
    std::vector<float> out((size_t)N * c);
    if (N == 0) return out;
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    const size_t es = w.conv.dtype == TB_F32 ? 4 : 2;
    DBuf df((size_t)N * c * es), dn((size_t)N * 27 * 4), dout((size_t)N * c * 4);
    if (w.conv.dtype == TB_F32) {
        cuda_ok(cudaMemcpy(df.p, feats.data(), feats.size() * 4, cudaMemcpyHostToDevice), "upload feats");
    } else {
        std::vector<uint16_t> h(feats.size());
        for (size_t k = 0; k < feats.size(); ++k)
            h[k] = w.conv.dtype == TB_BF16 ? f32_to_bf16_rne(feats[k]) : f32_to_f16_rne(feats[k]);
        cuda_ok(cudaMemcpy(df.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "upload feats");
    }
    cuda_ok(cudaMemcpy(dn.p, nbr.data(), nbr.size() * 4, cudaMemcpyHostToDevice), "upload nbr");
    ok(tb_sparse_convnext(ctx(), dn.as<int32_t>(), N, df.p, c, w.conv.weight, w.conv.bias, w.norm_w, w.norm_b,
                          w.mlp0_w, w.mlp0_b, w.mlp2_w, w.mlp2_b, w.conv.dtype, TB_F32, dout.p),
       "tb_sparse_convnext");
    cuda_ok(cudaMemcpy(out.data(), dout.p, out.size() * 4, cudaMemcpyDeviceToHost), "download out");
    ok(tb_ctx_check_device(ctx()), "convnext device check");
    return out;
}

SubdivideResult subdivide(const std::vector<std::array<int, 3>>& coords, const std::vector<uint8_t>& mask) {
    const int64_t n = (int64_t)coords.size();
    if ((int64_t)mask.size() != 8 * n) throw std::runtime_error("trellis: subdivide: mask must have 8*N entries");
    SubdivideResult r;
    r.mstart.assign((size_t)n + 1, 0);
    if (n == 0) return r;
    int64_t mmax = 0;
    for (uint8_t v : mask) mmax += v != 0;
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    DBuf dc((size_t)n * 12), dm((size_t)n * 8), dch((size_t)mmax * 12), dg((size_t)mmax * 4), ds((size_t)(n + 1) * 4);
    cuda_ok(cudaMemcpy(dc.p, coords.data(), (size_t)n * 12, cudaMemcpyHostToDevice), "upload coords");
    cuda_ok(cudaMemcpy(dm.p, mask.data(), (size_t)n * 8, cudaMemcpyHostToDevice), "upload mask");
    int64_t m = 0;
    ok(tb_subdivide(ctx(), dc.as<int32_t>(), n, 3, dm.as<uint8_t>(), dch.as<int32_t>(), dg.as<int32_t>(),
                    ds.as<int32_t>(), mmax, &m), "tb_subdivide");
    r.coords.resize((size_t)m);
    r.gidx.resize((size_t)m);
    cuda_ok(cudaMemcpy(r.coords.data(), dch.p, (size_t)m * 12, cudaMemcpyDeviceToHost), "download children");
    cuda_ok(cudaMemcpy(r.gidx.data(), dg.p, (size_t)m * 4, cudaMemcpyDeviceToHost), "download gidx");
    cuda_ok(cudaMemcpy(r.mstart.data(), ds.p, (size_t)(n + 1) * 4, cudaMemcpyDeviceToHost), "download mstart");
    return r;
}

Mesh dual_grid_to_mesh(const ShapeOut& so) {
    const int64_t n = (int64_t)so.coords.size();
    if ((int64_t)so.feats7.size() != 7 * n) throw std::runtime_error("trellis: dual_grid_to_mesh: feats7 must have 7*M entries");
    Mesh mesh;
    if (n == 0) return mesh;
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    DBuf dc((size_t)n * 12), df((size_t)n * 28), dv((size_t)n * 12), dfa((size_t)n * 72);
    cuda_ok(cudaMemcpy(dc.p, so.coords.data(), (size_t)n * 12, cudaMemcpyHostToDevice), "upload coords");
    cuda_ok(cudaMemcpy(df.p, so.feats7.data(), (size_t)n * 28, cudaMemcpyHostToDevice), "upload feats7");
    int64_t f = 0;
    ok(tb_dual_grid_mesh(ctx(), dc.as<int32_t>(), n, 3, df.as<float>(), so.res, dv.as<float>(), dfa.as<int32_t>(),
                         6 * n, &f), "tb_dual_grid_mesh");
    mesh.verts.resize((size_t)n * 3);
    mesh.faces.resize((size_t)f * 3);
    cuda_ok(cudaMemcpy(mesh.verts.data(), dv.p, (size_t)n * 12, cudaMemcpyDeviceToHost), "download verts");
    if (f > 0) cuda_ok(cudaMemcpy(mesh.faces.data(), dfa.p, (size_t)f * 12, cudaMemcpyDeviceToHost), "download faces");
    return mesh;
}

C2SResult sparse_c2s(const C2SWeights& w, const std::vector<float>& feats_in, int Cin,
                     const std::vector<std::array<int, 3>>& coords, int Cout,
                     const std::vector<uint8_t>* ext_subdiv) {
    const int64_t n = (int64_t)coords.size();
    if ((int64_t)feats_in.size() != n * Cin) throw std::runtime_error("trellis: sparse_c2s: feats_in size mismatch");
    if (ext_subdiv && (int64_t)ext_subdiv->size() != 8 * n)
        throw std::runtime_error("trellis: sparse_c2s: ext_subdiv must have 8*N entries");
    C2SResult r;
    r.C = Cout;
    r.subdiv.assign((size_t)(8 * n), 0);
    if (n == 0) return r;
    int64_t cap = 8 * n;
    if (ext_subdiv) {
        cap = 0;
        for (uint8_t v : *ext_subdiv) cap += v != 0;
    }
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    const size_t es = w.dtype == TB_F32 ? 4 : 2;
    DBuf dc((size_t)n * 12), df((size_t)n * Cin * es), dm((size_t)n * 8), dch((size_t)cap * 12),
        dout((size_t)cap * Cout * 4), dmo((size_t)n * 8);
    cuda_ok(cudaMemcpy(dc.p, coords.data(), (size_t)n * 12, cudaMemcpyHostToDevice), "upload coords");
    if (w.dtype == TB_F32) {
        cuda_ok(cudaMemcpy(df.p, feats_in.data(), feats_in.size() * 4, cudaMemcpyHostToDevice), "upload feats");
    } else {
        std::vector<uint16_t> h(feats_in.size());
        for (size_t k = 0; k < feats_in.size(); ++k)
            h[k] = w.dtype == TB_BF16 ? f32_to_bf16_rne(feats_in[k]) : f32_to_f16_rne(feats_in[k]);
        cuda_ok(cudaMemcpy(df.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "upload feats");
    }
    if (ext_subdiv)
        cuda_ok(cudaMemcpy(dm.p, ext_subdiv->data(), (size_t)n * 8, cudaMemcpyHostToDevice), "upload mask");
    int64_t m = 0;
    ok(tb_sparse_c2s(ctx(), dc.as<int32_t>(), n, 3, df.p, Cin, Cout, &w.p, ext_subdiv ? dm.as<uint8_t>() : nullptr,
                     w.dtype, TB_F32, cap, dch.as<int32_t>(), dout.p, dmo.as<uint8_t>(), &m),
       "tb_sparse_c2s");
    r.coords.resize((size_t)m);
    r.feats.resize((size_t)m * Cout);
    cuda_ok(cudaMemcpy(r.coords.data(), dch.p, (size_t)m * 12, cudaMemcpyDeviceToHost), "download children");
    cuda_ok(cudaMemcpy(r.feats.data(), dout.p, r.feats.size() * 4, cudaMemcpyDeviceToHost), "download feats");
    cuda_ok(cudaMemcpy(r.subdiv.data(), dmo.p, (size_t)n * 8, cudaMemcpyDeviceToHost), "download mask");
    ok(tb_ctx_check_device(ctx()), "c2s device check");
    return r;
}

// ---- GGUF checkpoints and the slat dump ---------------------------------------------------------
GgufModel GgufModel::load(const std::string& path, int device, tb_dtype weight_dtype) {
    tb_gguf* g = nullptr;
    if (tb_gguf_open(path.c_str(), &g) != TB_OK) throw std::runtime_error(std::string("trellis: ") + tb_io_last_error());
    struct Closer {
        tb_gguf* g;
        ~Closer() { tb_gguf_close(g); }
    } closer{g};
    set_device(device);
    cuda_ok(cudaSetDevice(device), "cudaSetDevice");
    GgufModel m;
    m.device_ = device;
    m.weight_dtype = weight_dtype;
    if (const char* a = tb_gguf_get_string(g, "general.architecture")) m.arch = a;
    if (const char* c = tb_gguf_get_string(g, "trellis.config_json")) m.config_json = c;
    const int64_t n = tb_gguf_n_tensors(g);
    for (int64_t i = 0; i < n; ++i) {
        const char* name = nullptr;
        int32_t type = 0, nd = 0;
        int64_t ne[4];
        uint64_t nbytes = 0;
        ok(tb_gguf_tensor_info(g, i, &name, &type, &nd, ne, &nbytes), "tb_gguf_tensor_info");
        if (!nbytes) continue;                      // quantised types are not used on this path
        const std::string nm = name;
        static const std::string kSubdiv = ".to_subdiv.weight";    // read by tb_sparse_c2s as float32
        const bool subdiv = nm.size() >= kSubdiv.size() &&
                            nm.compare(nm.size() - kSubdiv.size(), kSubdiv.size(), kSubdiv) == 0;
        Tensor t;
        t.dtype = nd >= 2 && !subdiv ? weight_dtype : TB_F32;
        int64_t elems = 1;
        for (int d = nd - 1; d >= 0; --d) {
            t.shape.push_back(ne[d]);
            elems *= ne[d];
        }
        cuda_ok(cudaMalloc(&t.dev, (size_t)elems * (t.dtype == TB_F32 ? 4 : 2) + 16), "cudaMalloc");
        m.t_[nm] = t;   // owned by m from here on (freed by its destructor on an error below)
        ok(tb_gguf_upload_tensor(ctx(), g, i, t.dtype, t.dev), "tb_gguf_upload_tensor");
    }
    return m;
}

GgufModel::GgufModel(GgufModel&& o) noexcept
    : arch(std::move(o.arch)), config_json(std::move(o.config_json)), weight_dtype(o.weight_dtype),
      t_(std::move(o.t_)), device_(o.device_) {
    o.t_.clear();
}

GgufModel& GgufModel::operator=(GgufModel&& o) noexcept {
    if (this != &o) {
        for (auto& kv : t_) cudaFree(kv.second.dev);
        t_ = std::move(o.t_);
        o.t_.clear();
        arch = std::move(o.arch);
        config_json = std::move(o.config_json);
        weight_dtype = o.weight_dtype;
        device_ = o.device_;
    }
    return *this;
}

GgufModel::~GgufModel() {
    if (t_.empty()) return;
    cudaSetDevice(device_);
    for (auto& kv : t_) cudaFree(kv.second.dev);
}

const void* GgufModel::get(const std::string& name) const {
    auto it = t_.find(name);
    if (it == t_.end()) throw std::runtime_error("trellis: missing tensor " + name);
    return it->second.dev;
}

std::vector<int64_t> GgufModel::shape(const std::string& name) const {
    auto it = t_.find(name);
    if (it == t_.end()) throw std::runtime_error("trellis: missing tensor " + name);
    return it->second.shape;
}

ConvWeights GgufModel::conv(const std::string& prefix) const {
    const auto s = shape(prefix + ".weight");
    if (s.size() != 3 || s[1] != 27) throw std::runtime_error("trellis: " + prefix + ".weight is not [Co,27,Ci]");
    ConvWeights w;
    w.weight = get(prefix + ".weight");
    w.bias = has(prefix + ".bias") ? static_cast<const float*>(get(prefix + ".bias")) : nullptr;
    w.co = (int)s[0];
    w.ci = (int)s[2];
    w.dtype = weight_dtype;
    return w;
}

ConvNeXtWeights GgufModel::convnext(const std::string& prefix) const {
    ConvNeXtWeights w;
    w.conv = conv(prefix + ".conv");
    w.norm_w = static_cast<const float*>(get(prefix + ".norm.weight"));
    w.norm_b = static_cast<const float*>(get(prefix + ".norm.bias"));
    w.mlp0_w = get(prefix + ".mlp.0.weight");
    w.mlp0_b = static_cast<const float*>(get(prefix + ".mlp.0.bias"));
    w.mlp2_w = get(prefix + ".mlp.2.weight");
    w.mlp2_b = static_cast<const float*>(get(prefix + ".mlp.2.bias"));
    return w;
}

C2SWeights GgufModel::c2s(const std::string& prefix) const {
    C2SWeights w;
    w.dtype = weight_dtype;
    if (has(prefix + ".to_subdiv.weight")) {
        w.p.to_subdiv_w = static_cast<const float*>(get(prefix + ".to_subdiv.weight"));
        w.p.to_subdiv_b = has(prefix + ".to_subdiv.bias") ? static_cast<const float*>(get(prefix + ".to_subdiv.bias"))
                                                          : nullptr;
    }
    w.p.norm1_w = static_cast<const float*>(get(prefix + ".norm1.weight"));
    w.p.norm1_b = static_cast<const float*>(get(prefix + ".norm1.bias"));
    w.p.conv1_w = get(prefix + ".conv1.weight");
    w.p.conv1_b = has(prefix + ".conv1.bias") ? static_cast<const float*>(get(prefix + ".conv1.bias")) : nullptr;
    w.p.conv2_w = get(prefix + ".conv2.weight");
    w.p.conv2_b = has(prefix + ".conv2.bias") ? static_cast<const float*>(get(prefix + ".conv2.bias")) : nullptr;
    return w;
}

// ---- decode_unet on the device ----------------------------------------------------------------
namespace {

struct Stage {
    std::string prefix;      // "blocks.<s>."
    int c = 0, nblk = 0, cout = 0;
};

std::vector<Stage> stages_of(const GgufModel& m) {
    std::vector<Stage> st;
    for (int s = 0;; ++s) {
        Stage g;
        g.prefix = "blocks." + std::to_string(s) + ".";
        while (m.has(g.prefix + std::to_string(g.nblk) + ".conv.weight")) ++g.nblk;
        const std::string c2s = g.prefix + std::to_string(g.nblk);
        if (!m.has(c2s + ".conv1.weight")) {
            if (g.nblk) throw std::runtime_error("trellis: stage " + g.prefix + " has no C2S block");
            break;
        }
        g.c = (int)m.shape(c2s + ".norm1.weight")[0];
        g.cout = (int)m.shape(c2s + ".conv2.weight")[0];
        st.push_back(g);
    }
    if (st.empty()) throw std::runtime_error("trellis: no decoder stages (blocks.0.*) in the model");
    return st;
}

size_t esize(tb_dtype d) { return d == TB_F32 ? 4 : 2; }

std::vector<float> decode_unet(const GgufModel& m, const std::vector<float>& latent, int out_ch,
                               std::vector<std::array<int, 3>>& coords,
                               const std::vector<std::vector<uint8_t>>* guide,
                               std::vector<std::vector<uint8_t>>* subs_out, bool coords_only) {
    const std::vector<Stage> st = stages_of(m);
    const tb_dtype dt = m.weight_dtype;
    const size_t es = esize(dt);
    int64_t n = (int64_t)coords.size();
    if ((int64_t)latent.size() != n * 32) throw std::runtime_error("trellis: decode: latent must be [N][32]");
    if (guide && guide->size() < st.size()) throw std::runtime_error("trellis: decode: one guide mask per stage needed");
    const int c0 = (int)m.shape("from_latent.weight")[0];
    cuda_ok(cudaSetDevice(g_device), "cudaSetDevice");
    tb_ctx* c = ctx();
    // inputs: coordinates and the latent (rounded to the operand type like the features)
    auto d_coords = std::make_unique<DBuf>((size_t)n * 12);
    cuda_ok(cudaMemcpy(d_coords->p, coords.data(), (size_t)n * 12, cudaMemcpyHostToDevice), "upload coords");
    DBuf d_lat((size_t)n * 32 * es);
    if (dt == TB_F32) {
        cuda_ok(cudaMemcpy(d_lat.p, latent.data(), latent.size() * 4, cudaMemcpyHostToDevice), "upload latent");
    } else {
        std::vector<uint16_t> hl(latent.size());
        for (size_t k = 0; k < latent.size(); ++k)
            hl[k] = dt == TB_BF16 ? f32_to_bf16_rne(latent[k]) : f32_to_f16_rne(latent[k]);
        cuda_ok(cudaMemcpy(d_lat.p, hl.data(), hl.size() * 2, cudaMemcpyHostToDevice), "upload latent");
    }
    auto h = std::make_unique<DBuf>((size_t)n * c0 * es);
    ok(tb_linear(c, n, 32, c0, d_lat.p, m.get("from_latent.weight"),
                 static_cast<const float*>(m.get("from_latent.bias")), nullptr, dt, TB_EPI_NONE, dt, dt, h->p),
       "from_latent");
    int ch = c0;
    for (size_t s = 0; s < st.size(); ++s) {
        const Stage& g = st[s];
        if (g.c != ch) throw std::runtime_error("trellis: decode: stage width does not match the previous stage");
        // The stage's map and ConvNeXt blocks run on its rows in key order (the C2S block's
        // children come parent-major, and the conv kernels read a tile's neighbours as contiguous
        // row ranges only in key order); the blocks' output goes back to the reference's order.
        DBuf perm((size_t)n * 4), sc((size_t)n * 12), nbr((size_t)n * 27 * 4);
        auto h2 = std::make_unique<DBuf>((size_t)n * ch * es);
        ok(tb_sort_rows(c, d_coords->as<int32_t>(), n, 3, perm.as<int32_t>()), "stage row order");
        ok(tb_gather_rows(c, d_coords->p, perm.as<int32_t>(), n, 12, sc.p), "stage coords in key order");
        ok(tb_gather_rows(c, h->p, perm.as<int32_t>(), n, (int64_t)ch * (int64_t)es, h2->p), "stage rows in key order");
        std::swap(h, h2);
        ok(tb_build_neighbor_map(c, sc.as<int32_t>(), n, 3, nbr.as<int32_t>()), "stage map");
        for (int j = 0; j < g.nblk; ++j) {
            const ConvNeXtWeights w = m.convnext(g.prefix + std::to_string(j));
            ok(tb_sparse_convnext(c, nbr.as<int32_t>(), n, h->p, ch, w.conv.weight, w.conv.bias, w.norm_w, w.norm_b,
                                  w.mlp0_w, w.mlp0_b, w.mlp2_w, w.mlp2_b, dt, dt, h2->p),
               "ConvNeXt block");
            std::swap(h, h2);
        }
        ok(tb_scatter_rows(c, h->p, perm.as<int32_t>(), n, (int64_t)ch * (int64_t)es, h2->p), "stage rows back");
        std::swap(h, h2);
        const C2SWeights w = m.c2s(g.prefix + std::to_string(g.nblk));
        std::unique_ptr<DBuf> d_guide;
        if (guide) {
            if ((int64_t)(*guide)[s].size() != 8 * n) throw std::runtime_error("trellis: decode: guide mask size");
            d_guide = std::make_unique<DBuf>((size_t)n * 8);
            cuda_ok(cudaMemcpy(d_guide->p, (*guide)[s].data(), (size_t)n * 8, cudaMemcpyHostToDevice), "upload guide");
        }
        const int64_t cap = 8 * n;
        auto child = std::make_unique<DBuf>((size_t)cap * 12);
        auto out = std::make_unique<DBuf>((size_t)cap * g.cout * es);
        DBuf mask((size_t)n * 8);
        int64_t mc = 0;
        ok(tb_sparse_c2s(c, d_coords->as<int32_t>(), n, 3, h->p, ch, g.cout, &w.p,
                         d_guide ? d_guide->as<uint8_t>() : nullptr, dt, dt, cap, child->as<int32_t>(), out->p,
                         mask.as<uint8_t>(), &mc),
           "C2S block");
        if (subs_out) {
            std::vector<uint8_t> hm((size_t)n * 8);
            cuda_ok(cudaMemcpy(hm.data(), mask.p, hm.size(), cudaMemcpyDeviceToHost), "download mask");
            subs_out->push_back(std::move(hm));
        }
        d_coords = std::move(child);
        h = std::move(out);
        n = mc;
        ch = g.cout;
    }
    coords.resize((size_t)n);
    cuda_ok(cudaMemcpy(coords.data(), d_coords->p, (size_t)n * 12, cudaMemcpyDeviceToHost), "download coords");
    if (coords_only) return {};
    // LayerNorm (no affine, eps 1e-5) and output_layer (src/shape_decoder.cpp:62-77,114)
    DBuf y((size_t)n * ch * es), o((size_t)n * out_ch * 4);
    ok(tb_layer_norm(c, h->p, dt, n, ch, nullptr, nullptr, 1e-5f, TB_EPI_NONE, dt, y.p), "final LayerNorm");
    ok(tb_linear(c, n, ch, out_ch, y.p, m.get("output_layer.weight"),
                 static_cast<const float*>(m.get("output_layer.bias")), nullptr, dt, TB_EPI_NONE, dt, TB_F32, o.p),
       "output_layer");
    std::vector<float> res((size_t)n * out_ch);
    cuda_ok(cudaMemcpy(res.data(), o.p, res.size() * 4, cudaMemcpyDeviceToHost), "download output");
    ok(tb_ctx_check_device(c), "decode device check");
    return res;
}

}  // namespace

ShapeOut shape_decode(const GgufModel& m, const std::vector<float>& latent,
                      const std::vector<std::array<int, 3>>& coords0, int resolution) {
    ShapeOut so;
    so.coords = coords0;
    so.res = resolution;
    so.feats7 = decode_unet(m, latent, (int)m.shape("output_layer.weight")[0], so.coords, nullptr, &so.subs, false);
    return so;
}

std::vector<std::array<int, 3>> shape_upsample(const GgufModel& m, const std::vector<float>& latent,
                                               const std::vector<std::array<int, 3>>& coords0) {
    std::vector<std::array<int, 3>> coords = coords0;
    decode_unet(m, latent, 0, coords, nullptr, nullptr, true);
    return coords;
}

std::vector<float> tex_decode(const GgufModel& m, const std::vector<float>& tex_latent,
                              const std::vector<std::array<int, 3>>& coords0,
                              const std::vector<std::vector<uint8_t>>& subs) {
    std::vector<std::array<int, 3>> coords = coords0;
    return decode_unet(m, tex_latent, (int)m.shape("output_layer.weight")[0], coords, &subs, nullptr, false);
}

SlatInput read_slat(const std::string& path) {
    int64_t n = 0;
    int32_t res = 0;
    if (tb_slat_read(path.c_str(), &n, &res, nullptr, nullptr) != TB_OK)
        throw std::runtime_error(std::string("trellis: ") + tb_io_last_error());
    SlatInput s;
    s.res = res;
    s.coords.resize((size_t)n);
    s.feats.resize((size_t)n * 32);
    if (tb_slat_read(path.c_str(), &n, &res, reinterpret_cast<int32_t*>(s.coords.data()), s.feats.data()) != TB_OK)
        throw std::runtime_error(std::string("trellis: ") + tb_io_last_error());
    return s;
}

}  // namespace trellis
