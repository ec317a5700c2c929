// Model and input files of the decoder path, read without ggml:
//
// * GGUF checkpoints as the reference's tools/convert.py writes them (gguf-py's GGUFWriter:
//   conv and linear weights F16, 1-D parameters F32, tensor names kept verbatim, the model
//   config as the `trellis.config_json` string) and as src/trellis_model.cpp:96-137 loads them
//   through ggml's gguf reader. The file layout parsed here is the published GGUF v2/v3 one:
//   magic "GGUF", u32 version, u64 tensor count, u64 key/value count, the key/value pairs, the
//   tensor infos (name, u32 n_dims, u64 ne[n_dims] innermost first, u32 ggml type, u64 offset),
//   then the data section at the next multiple of `general.alignment` (32 by default).
//   A sparse conv weight [Co,27,Ci] is stored with ne = (Ci, 27, Co): the bytes of the
//   [Co][27][Ci] layout the conv kernels take (tools/convert.py:141-146).
// * the hr_slat.bin dump of src/decode_replay.cpp:19-28: i32 N, i32 res, N x (i32 x, y, z),
//   then N x 32 float32 features, voxel-major.
#include "tb_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

constexpr uint32_t kGgufF32 = 0, kGgufF16 = 1, kGgufBF16 = 30;

thread_local std::string g_io_error;

tb_status io_fail(tb_status s, const std::string& msg) {
    g_io_error = msg;
    return s;
}

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    uint32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;     // from the data section
    uint64_t nbytes = 0;
};

size_t type_size(uint32_t t) { return t == kGgufF32 ? 4 : (t == kGgufF16 || t == kGgufBF16) ? 2 : 0; }

struct Reader {
    FILE* f;
    uint64_t size;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (ok && fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > (1ull << 30) || len > size) { ok = false; return {}; }
        std::string s(len, '\0');
        if (len && fread(&s[0], 1, len, f) != len) ok = false;
        return s;
    }
    void skip(uint64_t bytes) {
        if (ok && fseek(f, (long)bytes, SEEK_CUR) != 0) ok = false;
    }
};

// size in bytes of one scalar value type (GGUF metadata types), 0 for string/array
uint64_t scalar_size(uint32_t vt) {
    switch (vt) {
        case 0: case 1: case 7: return 1;       // u8 i8 bool
        case 2: case 3: return 2;               // u16 i16
        case 4: case 5: case 6: return 4;       // u32 i32 f32
        case 10: case 11: case 12: return 8;    // u64 i64 f64
        default: return 0;
    }
}

template <int SK, int DK>
__global__ void k_convert(const uint16_t* __restrict__ src16, const float* __restrict__ src32, int64_t n,
                          void* __restrict__ dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v;
        if constexpr (SK == 0) v = src32[i];
        else if constexpr (SK == 1) v = __half2float(__ushort_as_half(src16[i]));
        else v = __uint_as_float((uint32_t)src16[i] << 16);
        if constexpr (DK == 0) reinterpret_cast<float*>(dst)[i] = v;
        else if constexpr (DK == 1) reinterpret_cast<__half*>(dst)[i] = __float2half_rn(v);
        else reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
    }
}

}  // namespace

struct tb_gguf {
    std::string path;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_off = 0;
    std::vector<GgufTensor> tensors;
    std::unordered_map<std::string, int64_t> index;
    std::unordered_map<std::string, std::string> strings;
};

extern "C" {

const char* tb_io_last_error(void) { return g_io_error.c_str(); }

tb_status tb_gguf_open(const char* path, tb_gguf** out) {
    if (!path || !out) return io_fail(TB_ERR_INVALID_ARG, "tb_gguf_open: null argument");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return io_fail(TB_ERR_INVALID_ARG, std::string("tb_gguf_open: cannot open ") + path);
    fseek(f, 0, SEEK_END);
    const uint64_t fsize = (uint64_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    Reader r{f, fsize};
    auto bad = [&](const std::string& why) {
        fclose(f);
        return io_fail(TB_ERR_INVALID_ARG, std::string("tb_gguf_open: ") + path + ": " + why);
    };
    char magic[4];
    if (fread(magic, 1, 4, f) != 4 || std::memcmp(magic, "GGUF", 4) != 0) return bad("not a GGUF file");
    auto* g = new tb_gguf();
    g->path = path;
    g->version = r.get<uint32_t>();
    if (g->version != 2 && g->version != 3) {
        delete g;
        return bad("unsupported GGUF version " + std::to_string(g->version));
    }
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        delete g;
        return bad("bad header counts");
    }
    for (uint64_t k = 0; k < n_kv && r.ok; ++k) {
        const std::string key = r.str();
        const uint32_t vt = r.get<uint32_t>();
        if (vt == 8) {
            std::string v = r.str();
            if (r.ok) g->strings[key] = std::move(v);
        } else if (vt == 9) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t cnt = r.get<uint64_t>();
            if (!r.ok || cnt > fsize) { r.ok = false; break; }
            if (et == 8) {
                for (uint64_t j = 0; j < cnt && r.ok; ++j) r.str();
            } else if (scalar_size(et)) {
                r.skip(cnt * scalar_size(et));
            } else {
                r.ok = false;     // nested arrays are not written by the reference's converter
            }
        } else if (scalar_size(vt)) {
            if (key == "general.alignment" && vt == 4) {
                g->alignment = r.get<uint32_t>();
            } else {
                r.skip(scalar_size(vt));
            }
        } else {
            r.ok = false;
        }
    }
    if (!r.ok || g->alignment == 0 || (g->alignment & (g->alignment - 1))) {
        delete g;
        return bad("bad metadata");
    }
    g->tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        GgufTensor& t = g->tensors[i];
        t.name = r.str();
        t.n_dims = r.get<uint32_t>();
        if (!r.ok || t.n_dims < 1 || t.n_dims > 4) { r.ok = false; break; }
        // the element count and the byte size must not wrap: a wrapped product would report a
        // shape whose bytes differ from nbytes, and callers size buffers from ne[]
        uint64_t elems = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            const uint64_t e = r.get<uint64_t>();
            if (e > (1ull << 40) || (e != 0 && elems > UINT64_MAX / e)) r.ok = false;
            t.ne[d] = (int64_t)e;
            if (r.ok) elems *= e;
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        const uint64_t esz = type_size(t.type);
        if (esz != 0 && elems > UINT64_MAX / esz) r.ok = false;
        if (!r.ok) break;
        t.nbytes = elems * esz;   // 0 for types this reader does not convert
        g->index[t.name] = (int64_t)i;
    }
    if (!r.ok) {
        delete g;
        return bad("bad tensor infos");
    }
    const uint64_t pos = (uint64_t)ftell(f);
    g->data_off = (pos + g->alignment - 1) / g->alignment * g->alignment;
    fclose(f);
    for (const GgufTensor& t : g->tensors)
        // compared without sums that can wrap: data_off <= fsize here, then offset and nbytes in turn
        if (t.nbytes && (g->data_off > fsize || t.offset > fsize - g->data_off ||
                         t.nbytes > fsize - g->data_off - t.offset)) {
            const std::string name = t.name;
            delete g;
            return io_fail(TB_ERR_INVALID_ARG, std::string("tb_gguf_open: ") + path + ": tensor " + name +
                                                   " extends past the end of the file");
        }
    *out = g;
    return TB_OK;
}

void tb_gguf_close(tb_gguf* g) { delete g; }

int64_t tb_gguf_n_tensors(const tb_gguf* g) { return g ? (int64_t)g->tensors.size() : 0; }

int64_t tb_gguf_find_tensor(const tb_gguf* g, const char* name) {
    if (!g || !name) return -1;
    auto it = g->index.find(name);
    return it == g->index.end() ? -1 : it->second;
}

tb_status tb_gguf_tensor_info(const tb_gguf* g, int64_t i, const char** name, int32_t* ggml_type, int32_t* n_dims,
                              int64_t* ne, uint64_t* nbytes) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return io_fail(TB_ERR_INVALID_ARG, "tb_gguf_tensor_info: bad index");
    const GgufTensor& t = g->tensors[i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = (int32_t)t.type;
    if (n_dims) *n_dims = (int32_t)t.n_dims;
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
    if (nbytes) *nbytes = t.nbytes;
    return TB_OK;
}

const char* tb_gguf_get_string(const tb_gguf* g, const char* key) {
    if (!g || !key) return nullptr;
    auto it = g->strings.find(key);
    return it == g->strings.end() ? nullptr : it->second.c_str();
}

tb_status tb_gguf_read_tensor(const tb_gguf* g, int64_t i, void* dst, uint64_t nbytes) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size() || !dst)
        return io_fail(TB_ERR_INVALID_ARG, "tb_gguf_read_tensor: bad arguments");
    const GgufTensor& t = g->tensors[i];
    if (!t.nbytes) return io_fail(TB_ERR_UNSUPPORTED, "tb_gguf_read_tensor: " + t.name + " is not F32/F16/BF16");
    if (nbytes != t.nbytes) return io_fail(TB_ERR_INVALID_ARG, "tb_gguf_read_tensor: " + t.name + ": size mismatch");
    FILE* f = fopen(g->path.c_str(), "rb");
    if (!f) return io_fail(TB_ERR_INVALID_ARG, "tb_gguf_read_tensor: cannot reopen " + g->path);
    const bool ok = fseek(f, (long)(g->data_off + t.offset), SEEK_SET) == 0 && fread(dst, 1, nbytes, f) == nbytes;
    fclose(f);
    return ok ? TB_OK : io_fail(TB_ERR_INVALID_ARG, "tb_gguf_read_tensor: short read for " + t.name);
}

tb_status tb_gguf_upload_tensor(tb_ctx* ctx, const tb_gguf* g, int64_t i, tb_dtype dtype, void* dst) {
    if (!ctx) return TB_ERR_INVALID_ARG;
    if (!g || i < 0 || i >= (int64_t)g->tensors.size() || !dst)
        return tb_fail(ctx, TB_ERR_INVALID_ARG, "tb_gguf_upload_tensor: bad arguments");
    const GgufTensor& t = g->tensors[i];
    if (!t.nbytes) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "tb_gguf_upload_tensor: " + t.name + " is not F32/F16/BF16");
    std::vector<uint8_t> host(t.nbytes);
    tb_status s = tb_gguf_read_tensor(g, i, host.data(), t.nbytes);
    if (s != TB_OK) return tb_fail(ctx, s, g_io_error);
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    const int sk = t.type == kGgufF32 ? 0 : (t.type == kGgufF16 ? 1 : 2);
    const int dk = dtype == TB_F32 ? 0 : (dtype == TB_F16 ? 1 : 2);
    if (sk == dk) {
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(dst, host.data(), t.nbytes, cudaMemcpyHostToDevice, ctx->stream));
        TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        return TB_OK;
    }
    s = tb_ensure(ctx, &ctx->ws, &ctx->ws_bytes, t.nbytes, "gguf staging");
    if (s != TB_OK) return s;
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->ws, host.data(), t.nbytes, cudaMemcpyHostToDevice, ctx->stream));
    const int64_t n = (int64_t)(t.nbytes / type_size(t.type));
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->num_sms * 16);
    const uint16_t* s16 = reinterpret_cast<const uint16_t*>(ctx->ws);
    const float* s32 = reinterpret_cast<const float*>(ctx->ws);
#define TB_CONVERT(S, D) k_convert<S, D><<<grid, 256, 0, ctx->stream>>>(s16, s32, n, dst)
    if (sk == 0 && dk == 1) TB_CONVERT(0, 1);
    else if (sk == 0 && dk == 2) TB_CONVERT(0, 2);
    else if (sk == 1 && dk == 0) TB_CONVERT(1, 0);
    else if (sk == 1 && dk == 2) TB_CONVERT(1, 2);
    else if (sk == 2 && dk == 0) TB_CONVERT(2, 0);
    else TB_CONVERT(2, 1);
#undef TB_CONVERT
    TB_LAUNCH_CHECK(ctx, "k_convert");
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return TB_OK;
}

tb_status tb_slat_read(const char* path, int64_t* n, int32_t* res, int32_t* coords, float* feats) {
    if (!path || !n) return io_fail(TB_ERR_INVALID_ARG, "tb_slat_read: null argument");
    FILE* f = fopen(path, "rb");
    if (!f) return io_fail(TB_ERR_INVALID_ARG, std::string("tb_slat_read: cannot open ") + path);
    fseek(f, 0, SEEK_END);
    const int64_t fsize = (int64_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    int32_t hdr[2] = {0, 0};
    if (fread(hdr, 4, 2, f) != 2 || hdr[0] < 0) {
        fclose(f);
        return io_fail(TB_ERR_INVALID_ARG, std::string("tb_slat_read: bad header in ") + path);
    }
    const int64_t count = hdr[0];
    if (fsize != 8 + count * 12 + count * 32 * 4) {
        fclose(f);
        return io_fail(TB_ERR_INVALID_ARG, std::string("tb_slat_read: ") + path + ": size does not match N=" +
                                               std::to_string(count) + " (12 + 128 bytes per voxel)");
    }
    *n = count;
    if (res) *res = hdr[1];
    bool ok = true;
    if (coords) ok = fread(coords, 4, (size_t)count * 3, f) == (size_t)count * 3;
    else ok = fseek(f, (long)(count * 12), SEEK_CUR) == 0;
    if (ok && feats) ok = fread(feats, 4, (size_t)count * 32, f) == (size_t)count * 32;
    fclose(f);
    return ok ? TB_OK : io_fail(TB_ERR_INVALID_ARG, std::string("tb_slat_read: short read in ") + path);
}

}  // extern "C"
