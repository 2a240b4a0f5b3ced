// gguf.cu -- GGUF expert binding (host code): a model file's MoE block as a layer description.
//
// Follows the reference's loader, restated here:
//   * the header parse, src/gguf.rs:307-392: "GGUF" magic, version 2 or 3, tensor and KV counts
//     (u32 in version 2, u64 in 3), typed KV metadata (13 kinds, arrays nested), then the
//     tensor-info table (name, up to 8 dims, GGML type code, byte offset); errors carry the
//     byte offset ("gguf parse error at N: ...", src/gguf.rs:174-178);
//   * general.alignment (u32 or u64, default 32) and the aligned data start,
//     src/gguf.rs:146-162 / src/loader.rs:33-39;
//   * MmapModel::tensor_bytes, src/loader.rs:97-102: [data_start + offset, + nbytes), bounds-
//     checked against the mapping; nbytes = bytes_for_numel(type, numel), src/quant.rs:92-101;
//   * the MoE tensors of block N, src/model.rs:366-391: blk.N.ffn_gate_inp [H, E],
//     ffn_{gate,up}_exps [H, I, E], ffn_down_exps [I, H, E], optional ffn_*_shexp, checked
//     with the reference's messages ("missing required tensor", "dims [..] != expected [..]");
//   * expert_count / expert_used_count read as {arch}.{key}, then general.{key}
//     (src/model.rs:131-147, 239-240).
// The file is mapped read-only and the description points into the mapping (no copy); a
// router stored as F16 / BF16 is widened to f32 into memory the rmoe_gguf handle owns.
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "layer_impl.h"

using namespace rmoe;

namespace {

enum Kind : uint32_t {
    K_U8 = 0, K_I8, K_U16, K_I16, K_U32, K_I32, K_F32, K_BOOL, K_STR, K_ARR, K_U64, K_I64, K_F64,
};

struct Meta {
    uint32_t kind = 0;
    bool integer = false;  // an integer kind (the value is in u; i64 / i32 sign-extended)
    uint64_t u = 0;
    std::string s;
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
};

bool valid_utf8(const uint8_t* p, size_t n) {
    for (size_t i = 0; i < n;) {
        const uint8_t c = p[i];
        int len = c < 0x80 ? 1 : (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xe ? 3 : (c >> 3) == 0x1e ? 4 : 0;
        if (!len || i + len > n) return false;
        for (int j = 1; j < len; j++)
            if ((p[i + j] & 0xc0) != 0x80) return false;
        i += len;
    }
    return true;
}

struct Reader {
    const uint8_t* b;
    size_t n, pos = 0;
    std::string err;
    size_t err_at = 0;

    bool error(const std::string& m, size_t at) {
        if (err.empty()) {
            err = m;
            err_at = at;
        }
        return false;
    }
    bool need(uint64_t k) {
        if (k > n - pos) return error("unexpected EOF, need " + std::to_string(k) + " bytes", pos);
        return true;
    }
    template <class T>
    bool get(T& v) {
        if (!need(sizeof(T))) return false;
        memcpy(&v, b + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool str(std::string& s) {
        uint64_t len;
        if (!get(len) || !need(len)) return false;
        if (!valid_utf8(b + pos, len)) return error("invalid utf-8 string", pos);
        s.assign(reinterpret_cast<const char*>(b) + pos, len);
        pos += len;
        return true;
    }
    // One value of `kind` (arrays: element kind, count, elements; nested arrays allowed).
    bool value(uint32_t kind, Meta& m, int depth) {
        m.kind = kind;
        switch (kind) {
            case K_U8: case K_BOOL: { uint8_t v; if (!get(v)) return false; m.u = v; m.integer = kind == K_U8; return true; }
            case K_I8: { int8_t v; if (!get(v)) return false; m.u = (uint64_t)(int64_t)v; m.integer = true; return true; }
            case K_U16: { uint16_t v; if (!get(v)) return false; m.u = v; m.integer = true; return true; }
            case K_I16: { int16_t v; if (!get(v)) return false; m.u = (uint64_t)(int64_t)v; m.integer = true; return true; }
            case K_U32: { uint32_t v; if (!get(v)) return false; m.u = v; m.integer = true; return true; }
            case K_I32: { int32_t v; if (!get(v)) return false; m.u = (uint64_t)(int64_t)v; m.integer = true; return true; }
            case K_F32: { uint32_t v; return get(v); }
            case K_U64: case K_I64: { uint64_t v; if (!get(v)) return false; m.u = v; m.integer = true; return true; }
            case K_F64: { uint64_t v; return get(v); }
            case K_STR: return str(m.s);
            case K_ARR: {
                uint32_t ek;
                uint64_t count;
                if (!get(ek)) return false;
                if (ek > K_F64) return error("unknown array element kind " + std::to_string(ek), pos);
                if (!get(count)) return false;
                if (count > n - pos) return error("array count " + std::to_string(count) + " exceeds remaining bytes", pos);
                if (depth > 8) return error("arrays nested deeper than 8", pos);
                Meta e;
                for (uint64_t i = 0; i < count; i++)
                    if (!value(ek, e, depth + 1)) return false;
                m.u = count;
                return true;
            }
            default: return error("unknown value kind " + std::to_string(kind), pos);
        }
    }
};

}  // namespace

struct rmoe_gguf {
    void* map = nullptr;
    size_t len = 0;
    uint32_t version = 0;
    std::unordered_map<std::string, Meta> meta;
    std::vector<TensorInfo> tensors;
    std::unordered_map<std::string, size_t> by_name;
    uint64_t data_start = 0;
    std::string arch;
    std::vector<std::unique_ptr<std::vector<float>>> widened;  // routers widened to f32
    ~rmoe_gguf() {
        if (map) munmap(map, len);
    }
};

namespace {

rmoe_status parse_header(rmoe_gguf& g) {
    const uint8_t* b = static_cast<const uint8_t*>(g.map);
    if (g.len < 4 || memcmp(b, "GGUF", 4) != 0) return fail(RMOE_ERR_INVALID, "gguf parse error at 0: missing GGUF magic");
    Reader r{b, g.len};
    r.pos = 4;
    auto perr = [&]() { return fail(RMOE_ERR_INVALID, "gguf parse error at %zu: %s", r.err_at, r.err.c_str()); };
    if (!r.get(g.version)) return perr();
    if (g.version < 2 || g.version > 3)
        return fail(RMOE_ERR_INVALID, "gguf parse error at 4: unsupported GGUF version %u (need 2 or 3)", g.version);
    uint64_t n_tensors = 0, n_kv = 0;
    if (g.version >= 3) {
        if (!r.get(n_tensors) || !r.get(n_kv)) return perr();
    } else {
        uint32_t a, c;
        if (!r.get(a) || !r.get(c)) return perr();
        n_tensors = a;
        n_kv = c;
    }
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key;
        uint32_t kind;
        if (!r.str(key) || !r.get(kind)) return perr();
        if (kind > K_F64) {
            r.error("unknown value kind " + std::to_string(kind) + " for key " + key, r.pos);
            return perr();
        }
        Meta m;
        if (!r.value(kind, m, 0)) return perr();
        g.meta.emplace(key, m);  // the first value of a repeated key wins, as in the reference
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        TensorInfo t;
        uint32_t nd;
        if (!r.str(t.name) || !r.get(nd)) return perr();
        if (nd > 8) {
            r.error("tensor " + t.name + " declares " + std::to_string(nd) + " dims (max 8)", r.pos);
            return perr();
        }
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; d++)
            if (!r.get(t.dims[d])) return perr();
        if (!r.get(t.type) || !r.get(t.offset)) return perr();
        g.by_name.emplace(t.name, g.tensors.size());
        g.tensors.push_back(std::move(t));
    }
    uint64_t align = 32;
    auto a = g.meta.find("general.alignment");
    if (a != g.meta.end() && (a->second.kind == K_U32 || a->second.kind == K_U64)) align = a->second.u;
    if (align == 0) align = 1;
    g.data_start = (r.pos + align - 1) / align * align;
    auto ar = g.meta.find("general.architecture");
    if (ar != g.meta.end() && ar->second.kind == K_STR) g.arch = ar->second.s;
    return RMOE_OK;
}

// The named tensor's info and its bytes inside the mapping (MmapModel::tensor_bytes).
rmoe_status find_tensor(const rmoe_gguf& g, const std::string& name, const TensorInfo*& t, const uint8_t*& data,
                        uint64_t& nbytes) {
    auto it = g.by_name.find(name);
    if (it == g.by_name.end()) return fail(RMOE_ERR_INVALID, "missing required tensor '%s'", name.c_str());
    t = &g.tensors[it->second];
    uint64_t numel = 1;
    for (uint64_t d : t->dims) numel *= d;
    uint32_t el, by;
    if (!block_geom(t->type, el, by) || numel % el)
        return fail(RMOE_ERR_UNSUPPORTED, "tensor '%s' bytes out of bounds or type unsized (type %u)", name.c_str(), t->type);
    nbytes = numel / el * by;
    const uint64_t start = g.data_start + t->offset;
    if (start < g.data_start || start > g.len || nbytes > g.len - start)
        return fail(RMOE_ERR_INVALID, "tensor '%s' bytes out of bounds or type unsized", name.c_str());
    data = static_cast<const uint8_t*>(g.map) + start;
    return RMOE_OK;
}

std::string dims_str(const std::vector<uint64_t>& d) {
    std::string s = "[";
    for (size_t i = 0; i < d.size(); i++) s += (i ? ", " : "") + std::to_string(d[i]);
    return s + "]";
}

rmoe_status check_dims(const std::string& name, const TensorInfo& t, const std::vector<uint64_t>& want) {
    if (t.dims == want) return RMOE_OK;
    return fail(RMOE_ERR_INVALID, "%s: dims %s != expected %s", name.c_str(), dims_str(t.dims).c_str(),
                dims_str(want).c_str());
}

// {arch}.{key}, then general.{key}, as an unsigned integer
bool meta_uint(const rmoe_gguf& g, const std::string& key, uint64_t& v) {
    for (const std::string& k : {g.arch + "." + key, std::string("general.") + key}) {
        auto it = g.meta.find(k);
        if (it != g.meta.end() && it->second.integer) {
            v = it->second.u;
            return true;
        }
    }
    return false;
}

rmoe_status fill_tensor(const rmoe_gguf& g, const std::string& name, rmoe_tensor& out, const TensorInfo** info) {
    const TensorInfo* t;
    const uint8_t* data;
    uint64_t nbytes;
    rmoe_status s = find_tensor(g, name, t, data, nbytes);
    if (s) return s;
    if (t->dims.size() > 3)
        return fail(RMOE_ERR_UNSUPPORTED, "tensor '%s' has %zu dims (at most 3 here)", name.c_str(), t->dims.size());
    out.ggml_type = t->type;
    out.data = data;
    out.nbytes = nbytes;
    for (int i = 0; i < 3; i++) out.dims[i] = i < (int)t->dims.size() ? t->dims[i] : 1;
    if (info) *info = t;
    return RMOE_OK;
}

float bf16_to_f32(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// IEEE binary16 -> binary32, exact for every pattern (src/quant.rs:25-45)
float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ffu, u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {  // subnormal: normalise
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while (!(man & 0x400u));
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

}  // namespace

extern "C" {

RMOE_API rmoe_status rmoe_gguf_open(const char* path, rmoe_gguf** out) {
    if (!out) return fail(RMOE_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (!path) return fail(RMOE_ERR_INVALID, "null path");
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return fail(RMOE_ERR_INVALID, "%s: %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        const int e = errno;
        close(fd);
        return fail(RMOE_ERR_INVALID, "%s: %s", path, strerror(e));
    }
    std::unique_ptr<rmoe_gguf> g(new rmoe_gguf());
    g->len = (size_t)st.st_size;
    if (g->len) {
        void* m = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) {
            const int e = errno;
            close(fd);
            return fail(RMOE_ERR_INVALID, "%s: mmap: %s", path, strerror(e));
        }
        g->map = m;
    }
    close(fd);  // the mapping stays valid
    rmoe_status s = parse_header(*g);
    if (s) return s;
    *out = g.release();
    return RMOE_OK;
}

RMOE_API void rmoe_gguf_close(rmoe_gguf* g) { delete g; }

RMOE_API rmoe_status rmoe_gguf_tensor(const rmoe_gguf* g, const char* name, rmoe_tensor* out) {
    if (!g || !name || !out) return fail(RMOE_ERR_INVALID, "null argument");
    return fill_tensor(*g, name, *out, nullptr);
}

RMOE_API rmoe_status rmoe_gguf_meta_uint(const rmoe_gguf* g, const char* key, uint64_t* out) {
    if (!g || !key || !out) return fail(RMOE_ERR_INVALID, "null argument");
    auto it = g->meta.find(key);
    if (it == g->meta.end() || !it->second.integer) return fail(RMOE_ERR_INVALID, "missing required key '%s'", key);
    *out = it->second.u;
    return RMOE_OK;
}

RMOE_API rmoe_status rmoe_gguf_moe_layer_desc(rmoe_gguf* g, uint32_t block, rmoe_layer_desc* out) {
    if (!g || !out) return fail(RMOE_ERR_INVALID, "null argument");
    if (g->arch.empty()) return fail(RMOE_ERR_INVALID, "missing general.architecture");
    const std::string p = "blk." + std::to_string(block) + ".";
    rmoe_layer_desc d;
    memset(&d, 0, sizeof d);
    const TensorInfo *tg, *tu, *td, *tr;
    rmoe_tensor router;
    rmoe_status s;
    if ((s = fill_tensor(*g, p + "ffn_gate_exps.weight", d.gate_exps, &tg))) return s;
    if (tg->dims.size() != 3)
        return fail(RMOE_ERR_INVALID, "%sffn_gate_exps.weight: dims %s != expected [H, I, E]", p.c_str(),
                    dims_str(tg->dims).c_str());
    const uint64_t H = tg->dims[0], I = tg->dims[1], E = tg->dims[2];
    if ((s = fill_tensor(*g, p + "ffn_up_exps.weight", d.up_exps, &tu)) ||
        (s = check_dims(p + "ffn_up_exps.weight", *tu, {H, I, E})) ||
        (s = fill_tensor(*g, p + "ffn_down_exps.weight", d.down_exps, &td)) ||
        (s = check_dims(p + "ffn_down_exps.weight", *td, {I, H, E})) ||
        (s = fill_tensor(*g, p + "ffn_gate_inp.weight", router, &tr)) ||
        (s = check_dims(p + "ffn_gate_inp.weight", *tr, {H, E})))
        return s;
    uint64_t n_exp;
    if (meta_uint(*g, "expert_count", n_exp) && n_exp != E)
        return fail(RMOE_ERR_INVALID, "%sffn_gate_exps.weight holds %llu experts, %s.expert_count is %llu", p.c_str(),
                    (unsigned long long)E, g->arch.c_str(), (unsigned long long)n_exp);
    uint64_t used;
    if (!meta_uint(*g, "expert_used_count", used))
        return fail(RMOE_ERR_INVALID, "missing required key '%s.expert_used_count'", g->arch.c_str());
    uint64_t gating = 1;
    meta_uint(*g, "expert_gating_func", gating);  // 1 softmax (the default), 2 sigmoid
    if (gating != 1 && gating != 2)
        return fail(RMOE_ERR_UNSUPPORTED, "%s.expert_gating_func %llu (softmax 1 and sigmoid 2 only)", g->arch.c_str(),
                    (unsigned long long)gating);
    // router: E rows x H f32 (widened from F16 / BF16 into memory the handle owns)
    if (tr->type == T_F32) {
        d.router_w = static_cast<const float*>(router.data);
    } else if (tr->type == T_F16 || tr->type == T_BF16) {
        std::unique_ptr<std::vector<float>> w(new std::vector<float>(H * E));
        const uint8_t* src = static_cast<const uint8_t*>(router.data);
        for (uint64_t i = 0; i < H * E; i++) {
            uint16_t h;
            memcpy(&h, src + 2 * i, 2);
            (*w)[i] = tr->type == T_F16 ? f16_to_f32(h) : bf16_to_f32(h);
        }
        d.router_w = w->data();
        g->widened.push_back(std::move(w));
    } else {
        return fail(RMOE_ERR_UNSUPPORTED, "%sffn_gate_inp.weight: router type %u (F32, F16 or BF16 only)", p.c_str(),
                    tr->type);
    }
    // shared expert: all three tensors or none (an ffn_gate_inp_shexp gate, where a file has
    // one, is not applied: the reference adds the shared expert at weight 1, src/moe.rs:381-386)
    const char* sh[3] = {"ffn_gate_shexp.weight", "ffn_up_shexp.weight", "ffn_down_shexp.weight"};
    int n_sh = 0;
    for (const char* n : sh) n_sh += g->by_name.count(p + n) ? 1 : 0;
    if (n_sh == 3) {
        const TensorInfo *sg, *su, *sd;
        if ((s = fill_tensor(*g, p + sh[0], d.gate_shexp, &sg)) || (s = fill_tensor(*g, p + sh[1], d.up_shexp, &su)) ||
            (s = fill_tensor(*g, p + sh[2], d.down_shexp, &sd)))
            return s;
        if (sg->dims.size() != 2 || sg->dims[0] != H)
            return fail(RMOE_ERR_INVALID, "%s%s: dims %s != expected [%llu, I]", p.c_str(), sh[0],
                        dims_str(sg->dims).c_str(), (unsigned long long)H);
        if (sg->dims[1] != I)
            return fail(RMOE_ERR_UNSUPPORTED, "%s%s: shared expert width %llu differs from the experts' %llu", p.c_str(),
                        sh[0], (unsigned long long)sg->dims[1], (unsigned long long)I);
        if ((s = check_dims(p + sh[1], *su, {H, I})) || (s = check_dims(p + sh[2], *sd, {I, H}))) return s;
        d.has_shared = 1;
    } else if (n_sh) {
        return fail(RMOE_ERR_INVALID, "%s: %d of the 3 shared-expert tensors present", p.c_str(), n_sh);
    }
    if (H > 0xffffffffull || I > 0xffffffffull || E > 0xffffffffull)
        return fail(RMOE_ERR_INVALID, "%s: dims beyond 32 bits", p.c_str());
    d.hidden = (uint32_t)H;
    d.inter = (uint32_t)I;
    d.n_experts = (uint32_t)E;
    d.top_k = (uint32_t)used;
    d.gate = gating == 2 ? RMOE_GATE_SIGMOID : RMOE_GATE_SOFTMAX;
    d.device = 0;
    *out = d;
    return RMOE_OK;
}

}  // extern "C"
