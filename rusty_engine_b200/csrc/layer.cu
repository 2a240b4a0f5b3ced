// layer.cu -- C ABI (include/rmoe.h): layer handles, host-side validation, load-time
// re-striding of GGUF expert tensors into the device planes, and the forward pipeline
//   route+dispatch -> grouped gate/up (+SwiGLU) -> grouped down (+combine)
// all stream-ordered on the caller's stream.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "../../include/rmoe.h"
#include "kernels.h"
#include "layer_impl.h"

namespace rmoe {

static thread_local std::string g_err;

rmoe_status fail(rmoe_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return s;
}

rmoe_status cuda_fail(cudaError_t e, const char* what) {
    return fail(RMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// (elements, bytes) per block, src/quant.rs:75-88
bool block_geom(uint32_t t, uint32_t& el, uint32_t& by) {
    switch (t) {
        case T_F32: el = 1; by = 4; return true;
        case T_F16: case T_BF16: el = 1; by = 2; return true;
        case T_Q4_0: el = 32; by = 18; return true;
        case T_Q5_0: el = 32; by = 22; return true;
        case T_Q8_0: el = 32; by = 34; return true;
        case T_Q4_K: el = 256; by = 144; return true;
        case T_Q5_K: el = 256; by = 176; return true;
        case T_Q6_K: el = 256; by = 210; return true;
        default: return false;
    }
}

static const char* type_name(uint32_t t) {
    switch (t) {
        case T_F32: return "F32"; case T_F16: return "F16"; case T_BF16: return "BF16";
        case T_Q4_0: return "Q4_0"; case T_Q5_0: return "Q5_0"; case T_Q8_0: return "Q8_0";
        case T_Q4_K: return "Q4_K"; case T_Q5_K: return "Q5_K"; case T_Q6_K: return "Q6_K";
        default: return "?";
    }
}

// f32 -> binary16, round to nearest even; returns false when |f| is beyond the fp16 range.
static bool f32_to_f16_rne(float f, uint16_t& out) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a >= 0x477ff000u) {  // >= 65520 rounds to inf (or inf/NaN itself)
        out = (uint16_t)(sign | 0x7c00u);
        return false;
    }
    if (a < 0x33000000u) { out = (uint16_t)sign; return true; }  // < 2^-25 rounds to zero
    int e = (int)(a >> 23) - 127;
    uint32_t mant = (a & 0x7fffffu) | 0x800000u;
    if (e < -14) {  // subnormal half: value = mant * 2^(e-23), unit 2^-24
        int shift = 13 + (-14 - e);  // bits of the 24-bit significand below the 2^-24 unit
        uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        out = (uint16_t)(sign | q);
        return true;
    }
    uint32_t q = ((uint32_t)(e + 15) << 10) | ((mant >> 13) & 0x3ffu);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;  // carry may round up into the exponent
    out = (uint16_t)(sign | q);
    return (q & 0x7c00u) != 0x7c00u;
}

static float f16_to_f32_host(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, frac = h & 0x3FFu, bits;
    if (exp == 0 && frac == 0) bits = sign;
    else if (exp == 0) {
        uint32_t e = 113, f = frac;
        while (!(f & 0x400u)) { f <<= 1; e--; }
        bits = sign | (e << 23) | ((f & 0x3FFu) << 13);
    } else if (exp == 0x1F) bits = sign | 0x7F800000u | (frac << 13);
    else bits = sign | ((exp + 112) << 23) | (frac << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

DeviceGuard::DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (dev != prev) cudaSetDevice(dev);
    cur = dev;
}
DeviceGuard::~DeviceGuard() {
    if (cur != prev) cudaSetDevice(prev);
}

void* Owned::alloc(size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, n ? n : 16) != cudaSuccess) return nullptr;
    ptrs.push_back(p);
    return p;
}
Owned::~Owned() {
    for (void* p : ptrs) cudaFree(p);
}

// Re-stride `experts` matrices of `rows` x `K` GGUF rows into the device planes and upload.
rmoe_status upload_mat(const rmoe_tensor& t, uint32_t rows, uint32_t K, uint32_t experts, const char* name,
                       Owned& own, DevMat& out) {
    uint32_t el, by;
    if (!block_geom(t.ggml_type, el, by)) return fail(RMOE_ERR_UNSUPPORTED, "%s: ggml type %u has no kernel", name, t.ggml_type);
    if (K % 256 != 0)
        return fail(RMOE_ERR_UNSUPPORTED, "%s: row width %u is not a multiple of 256 (GPU tile constraint)", name, K);
    if (!t.data) return fail(RMOE_ERR_INVALID, "%s: null data", name);
    const uint64_t total_rows = (uint64_t)rows * experts;
    const uint64_t rb = (uint64_t)K / el * by;
    if (t.nbytes != rb * total_rows)
        return fail(RMOE_ERR_INVALID, "%s: %llu bytes, expected %llu for %s [%u x %u x %u]", name,
                    (unsigned long long)t.nbytes, (unsigned long long)(rb * total_rows), type_name(t.ggml_type), K,
                    rows, experts);
    const uint8_t* src = static_cast<const uint8_t*>(t.data);
    const uint64_t nblk = (uint64_t)K / el;
    std::vector<uint8_t> mainp;
    std::vector<uint16_t> dpl;
    std::vector<uint32_t> aux;
    out = DevMat{};
    out.rows = rows;
    out.K = K;
    out.dstride = (uint32_t)nblk;
    out.trows = total_rows;
    // fp16 operand range: bound |w| per block from its scales (d * 63 * 15 + dmin * 63 for
    // the K-quants, d * 32 / 16 / 128 for the others) and refuse layers that could overflow.
    double wmax = 0.0;
    if (t.ggml_type != T_F32 && t.ggml_type != T_F16 && t.ggml_type != T_BF16) {
        const uint64_t nb_all = total_rows * nblk;
        for (uint64_t b = 0; b < nb_all; b++) {
            const uint8_t* s = src + b * by;
            double bound;
            switch (t.ggml_type) {
                case T_Q4_K: case T_Q5_K:
                    bound = fabs(f16_to_f32_host((uint16_t)(s[0] | (s[1] << 8)))) * 63.0 * 31.0 +
                            fabs(f16_to_f32_host((uint16_t)(s[2] | (s[3] << 8)))) * 63.0;
                    break;
                case T_Q6_K: bound = fabs(f16_to_f32_host((uint16_t)(s[208] | (s[209] << 8)))) * 128.0 * 32.0; break;
                case T_Q8_0: bound = fabs(f16_to_f32_host((uint16_t)(s[0] | (s[1] << 8)))) * 128.0; break;
                default: bound = fabs(f16_to_f32_host((uint16_t)(s[0] | (s[1] << 8)))) * 16.0; break;
            }
            if (!(bound <= wmax)) wmax = bound;  // also catches NaN scales
        }
        if (!(wmax < 65504.0))
            return fail(RMOE_ERR_UNSUPPORTED, "%s: block scales allow |w| up to %g, beyond the fp16 operand range", name,
                        wmax);
    }
    switch (t.ggml_type) {
        case T_Q4_K: {
            // half-superblocks of 80 B: the four sub-blocks' fp16 scale d*sc and negated min
            // -(dmin*m) (the products exact in f32, rounded once, as the kernels used them),
            // then the 64 quant bytes of those 128 elements
            out.type = T_Q4_K;
            out.main_stride = nblk * 160;
            mainp.resize(total_rows * nblk * 160);
            for (uint64_t r = 0; r < total_rows; r++)
                for (uint64_t b = 0; b < nblk; b++) {
                    const uint8_t* sb = src + r * rb + b * 144;
                    const float d = f16_to_f32_host((uint16_t)(sb[0] | (sb[1] << 8)));
                    const float dmin = f16_to_f32_host((uint16_t)(sb[2] | (sb[3] << 8)));
                    for (int h = 0; h < 2; h++) {
                        uint8_t* o = &mainp[(r * nblk + b) * 160 + h * 80];
                        for (int i = 0; i < 4; i++) {
                            const int j = 4 * h + i;
                            const uint8_t* q = sb + 4;
                            int sc, mn;
                            if (j < 4) {
                                sc = q[j] & 63;
                                mn = q[j + 4] & 63;
                            } else {
                                sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
                                mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
                            }
                            uint16_t hd, hm;
                            f32_to_f16_rne(d * (float)sc, hd);
                            f32_to_f16_rne(-(dmin * (float)mn), hm);
                            memcpy(o + 4 * i, &hd, 2);
                            memcpy(o + 4 * i + 2, &hm, 2);
                        }
                        memcpy(o + 16, sb + 16 + 64 * h, 64);
                    }
                }
            break;
        }
        case T_Q5_K:
            out.type = (int)t.ggml_type;
            out.main_stride = rb;
            mainp.assign(src, src + t.nbytes);
            break;
        case T_Q6_K:
            out.type = T_Q6_K;
            out.main_stride = nblk * 208;
            mainp.resize(total_rows * nblk * 208);
            dpl.resize(total_rows * nblk);
            for (uint64_t r = 0; r < total_rows; r++)
                for (uint64_t b = 0; b < nblk; b++) {
                    const uint8_t* s = src + r * rb + b * 210;
                    memcpy(&mainp[(r * nblk + b) * 208], s, 208);
                    dpl[b * total_rows + r] = (uint16_t)(s[208] | (s[209] << 8));
                }
            break;
        case T_Q4_0: case T_Q8_0: {
            const uint32_t qb = t.ggml_type == T_Q4_0 ? 16 : 32;
            out.type = (int)t.ggml_type;
            out.main_stride = nblk * qb;
            mainp.resize(total_rows * nblk * qb);
            dpl.resize(total_rows * nblk);
            for (uint64_t r = 0; r < total_rows; r++)
                for (uint64_t b = 0; b < nblk; b++) {
                    const uint8_t* s = src + r * rb + b * by;
                    memcpy(&mainp[(r * nblk + b) * qb], s + 2, qb);
                    dpl[b * total_rows + r] = (uint16_t)(s[0] | (s[1] << 8));
                }
            break;
        }
        case T_Q5_0:
            out.type = T_Q5_0;
            out.main_stride = nblk * 16;
            mainp.resize(total_rows * nblk * 16);
            dpl.resize(total_rows * nblk);
            aux.resize(total_rows * nblk);
            for (uint64_t r = 0; r < total_rows; r++)
                for (uint64_t b = 0; b < nblk; b++) {
                    const uint8_t* s = src + r * rb + b * 22;
                    memcpy(&mainp[(r * nblk + b) * 16], s + 6, 16);
                    dpl[b * total_rows + r] = (uint16_t)(s[0] | (s[1] << 8));
                    aux[b * total_rows + r] = (uint32_t)s[2] | ((uint32_t)s[3] << 8) | ((uint32_t)s[4] << 16) | ((uint32_t)s[5] << 24);
                }
            break;
        case T_F32: case T_F16: case T_BF16: {
            out.type = T_DENSE;
            out.main_stride = (uint64_t)K * 2;
            mainp.resize(total_rows * K * 2);
            uint16_t* d = reinterpret_cast<uint16_t*>(mainp.data());
            const uint64_t n = total_rows * K;
            bool range_ok = true;
            for (uint64_t i = 0; i < n; i++) {
                float f;
                if (t.ggml_type == T_BF16) {
                    uint32_t b = (uint32_t)(src[2 * i] | (src[2 * i + 1] << 8)) << 16;
                    memcpy(&f, &b, 4);
                } else if (t.ggml_type == T_F16) {
                    f = f16_to_f32_host((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8)));
                } else {
                    memcpy(&f, src + 4 * i, 4);
                }
                range_ok &= f32_to_f16_rne(f, d[i]);
            }
            if (!range_ok) return fail(RMOE_ERR_UNSUPPORTED, "%s: a weight exceeds the fp16 operand range", name);
            break;
        }
        default:
            return fail(RMOE_ERR_UNSUPPORTED, "%s: ggml type %u has no kernel", name, t.ggml_type);
    }
    void* dm = own.alloc(mainp.size());
    if (!dm) return fail(RMOE_ERR_OOM, "%s: cudaMalloc(%zu) failed", name, mainp.size());
    cudaError_t e = cudaMemcpy(dm, mainp.data(), mainp.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, name);
    out.main = static_cast<const uint8_t*>(dm);
    if (!dpl.empty()) {
        void* dd = own.alloc(dpl.size() * 2);
        if (!dd) return fail(RMOE_ERR_OOM, "%s: cudaMalloc failed", name);
        if ((e = cudaMemcpy(dd, dpl.data(), dpl.size() * 2, cudaMemcpyHostToDevice)) != cudaSuccess) return cuda_fail(e, name);
        out.dpl = static_cast<const __half*>(dd);
    }
    if (!aux.empty()) {
        void* da = own.alloc(aux.size() * 4);
        if (!da) return fail(RMOE_ERR_OOM, "%s: cudaMalloc failed", name);
        if ((e = cudaMemcpy(da, aux.data(), aux.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return cuda_fail(e, name);
        out.aux = static_cast<const uint32_t*>(da);
    }
    return RMOE_OK;
}

static rmoe_status check_dims(const rmoe_tensor& t, uint64_t d0, uint64_t d1, uint64_t d2, const char* name) {
    uint64_t e2 = t.dims[2] ? t.dims[2] : 1;
    if (t.dims[0] != d0 || t.dims[1] != d1 || e2 != d2)
        return fail(RMOE_ERR_INVALID, "%s: dims [%llu, %llu, %llu], expected [%llu, %llu, %llu]", name,
                    (unsigned long long)t.dims[0], (unsigned long long)t.dims[1], (unsigned long long)t.dims[2],
                    (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2);
    return RMOE_OK;
}

// Device type a GGUF type is held as (unquantized experts become one fp16 plane).
int canon_type(uint32_t t) { return (t == T_F32 || t == T_F16 || t == T_BF16) ? T_DENSE : (int)t; }

rmoe_status validate_desc(const rmoe_layer_desc* d) {
    if (!d) return fail(RMOE_ERR_INVALID, "null layer description");
    if (d->hidden == 0 || d->inter == 0 || d->n_experts == 0)
        return fail(RMOE_ERR_INVALID, "hidden, inter and n_experts must be non-zero");
    if (d->n_experts > (uint32_t)MAX_E) return fail(RMOE_ERR_UNSUPPORTED, "n_experts %u > %d", d->n_experts, MAX_E);
    if (d->top_k == 0) return fail(RMOE_ERR_INVALID, "top_k must be >= 1");
    if (d->top_k > (uint32_t)MAX_K) return fail(RMOE_ERR_UNSUPPORTED, "top_k %u > %d", d->top_k, MAX_K);
    if (d->gate > 1) return fail(RMOE_ERR_INVALID, "gate %u is not softmax (0) or sigmoid (1)", d->gate);
    if (!d->router_w) return fail(RMOE_ERR_INVALID, "null router weights");
    if (d->hidden % 256 || d->inter % 256)
        return fail(RMOE_ERR_UNSUPPORTED, "hidden %u / inter %u must be multiples of 256", d->hidden, d->inter);
    rmoe_status s;
    if ((s = check_dims(d->gate_exps, d->hidden, d->inter, d->n_experts, "ffn_gate_exps"))) return s;
    if ((s = check_dims(d->up_exps, d->hidden, d->inter, d->n_experts, "ffn_up_exps"))) return s;
    if ((s = check_dims(d->down_exps, d->inter, d->hidden, d->n_experts, "ffn_down_exps"))) return s;
    if (d->has_shared) {
        // the grouped kernels decode a launch's tiles with one type per projection
        if (canon_type(d->gate_shexp.ggml_type) != canon_type(d->gate_exps.ggml_type) ||
            canon_type(d->up_shexp.ggml_type) != canon_type(d->up_exps.ggml_type) ||
            canon_type(d->down_shexp.ggml_type) != canon_type(d->down_exps.ggml_type))
            return fail(RMOE_ERR_UNSUPPORTED, "shared expert tensors must have the routed experts' ggml types");
        if ((s = check_dims(d->gate_shexp, d->hidden, d->inter, 1, "ffn_gate_shexp"))) return s;
        if ((s = check_dims(d->up_shexp, d->hidden, d->inter, 1, "ffn_up_shexp"))) return s;
        if ((s = check_dims(d->down_shexp, d->inter, d->hidden, 1, "ffn_down_shexp"))) return s;
    }
    return RMOE_OK;
}


rmoe_status layer_upload(const rmoe_layer_desc* d, const uint32_t* ids, uint32_t e_count, rmoe_layer* L) {
    const uint32_t H = d->hidden, I = d->inter;
    if (canon_type(d->gate_exps.ggml_type) != canon_type(d->up_exps.ggml_type))
        return fail(RMOE_ERR_UNSUPPORTED, "gate (%s) and up (%s) expert types differ", type_name(d->gate_exps.ggml_type),
                    type_name(d->up_exps.ggml_type));
    uint32_t el, by;
    rmoe_status s;
    // experts ids[j], j < e_count (gathered on the host), or 0 .. e_count - 1 when ids is null
    std::vector<uint8_t> gathered;
    auto slice = [&](const rmoe_tensor& t, uint32_t rows, uint32_t K) {
        rmoe_tensor u = t;
        block_geom(t.ggml_type, el, by);
        uint64_t per = (uint64_t)rows * (K / el) * by;
        if (t.nbytes == per * d->n_experts && t.data) {
            const uint8_t* src = static_cast<const uint8_t*>(t.data);
            if (!ids) {
                u.data = src;
            } else {
                gathered.resize(per * e_count);
                for (uint32_t j = 0; j < e_count; j++) memcpy(gathered.data() + per * j, src + per * ids[j], per);
                u.data = gathered.data();
            }
            u.nbytes = per * e_count;
        }
        return u;
    };
    if ((s = upload_mat(slice(d->gate_exps, I, H), I, H, e_count, "ffn_gate_exps", L->own, L->wg))) return s;
    if ((s = upload_mat(slice(d->up_exps, I, H), I, H, e_count, "ffn_up_exps", L->own, L->wu))) return s;
    if ((s = upload_mat(slice(d->down_exps, H, I), H, I, e_count, "ffn_down_exps", L->own, L->wd))) return s;
    L->swg.type = L->swu.type = L->swd.type = -1;
    if (d->has_shared) {
        if (canon_type(d->gate_shexp.ggml_type) != L->wg.type || canon_type(d->up_shexp.ggml_type) != L->wu.type ||
            canon_type(d->down_shexp.ggml_type) != L->wd.type)
            return fail(RMOE_ERR_UNSUPPORTED, "shared-expert tensor types must match the routed experts' types");
        if ((s = upload_mat(d->gate_shexp, I, H, 1, "ffn_gate_shexp", L->own, L->swg))) return s;
        if ((s = upload_mat(d->up_shexp, I, H, 1, "ffn_up_shexp", L->own, L->swu))) return s;
        if ((s = upload_mat(d->down_shexp, H, I, 1, "ffn_down_shexp", L->own, L->swd))) return s;
    }
    // TMA descriptors of every stack, for the tensor-core kernels
    bool maps_ok = make_weight_maps(L->wg, L->mg) && make_weight_maps(L->wu, L->mu) && make_weight_maps(L->wd, L->md);
    if (d->has_shared)
        maps_ok = maps_ok && make_weight_maps(L->swg, L->smg) && make_weight_maps(L->swu, L->smu) &&
                  make_weight_maps(L->swd, L->smd);
    if (!maps_ok) return fail(RMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for an expert stack");
    // 64-row boxes of gate/up for the decode kernels' finer row blocks
    L->maps64 = make_weight_maps(L->wg, L->mg64, 64) && make_weight_maps(L->wu, L->mu64, 64) &&
                (!d->has_shared || (make_weight_maps(L->swg, L->smg64, 64) && make_weight_maps(L->swu, L->smu64, 64)));
    void* rw = L->own.alloc((size_t)d->n_experts * H * 4);
    if (!rw) return fail(RMOE_ERR_OOM, "router cudaMalloc failed");
    cudaError_t e = cudaMemcpy(rw, d->router_w, (size_t)d->n_experts * H * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "router upload");
    L->router_w = static_cast<float*>(rw);
    // the router split for the tensor-core logits: hi = w with its 13 low mantissa bits
    // cleared (a tf32 value), lo = w - hi (exact)
    const size_t nw = (size_t)d->n_experts * H;
    std::vector<float> hl(2 * nw);
    for (size_t i = 0; i < nw; i++) {
        uint32_t u;
        memcpy(&u, d->router_w + i, 4);
        u &= 0xffffe000u;
        float h;
        memcpy(&h, &u, 4);
        hl[i] = h;
        hl[nw + i] = d->router_w[i] - h;
    }
    void* rs = L->own.alloc(2 * nw * 4);
    if (!rs) return fail(RMOE_ERR_OOM, "router split cudaMalloc failed");
    if ((e = cudaMemcpy(rs, hl.data(), 2 * nw * 4, cudaMemcpyHostToDevice)) != cudaSuccess)
        return cuda_fail(e, "router split upload");
    L->router_wh = static_cast<float*>(rs);
    L->router_wl = L->router_wh + nw;
    double wmax = 0.0;
    for (uint32_t e2 = 0; e2 < d->n_experts; e2++) {
        double ss = 0.0;
        for (uint32_t i = 0; i < H; i++) ss += (double)d->router_w[(size_t)e2 * H + i] * d->router_w[(size_t)e2 * H + i];
        wmax = std::max(wmax, std::sqrt(ss));
    }
    // rounded up a little so the window never undershoots the f32 sums it bounds
    L->router_wmax = (float)(wmax * (1.0 + 1e-6));
    return RMOE_OK;
}

// Workspace for T tokens (grows; a grow synchronises the device).
rmoe_status ensure_workspace(rmoe_layer* L, uint32_t T, bool need_y) {
    if (T <= L->ws_T && (!need_y || L->ws.y)) return RMOE_OK;
    uint32_t cap = T > L->ws_T ? (T + 255) / 256 * 256 : L->ws_T;
    cudaDeviceSynchronize();
    L->ws_own.~Owned();
    new (&L->ws_own) Owned();
    L->ws = Workspace{};
    Owned& o = L->ws_own;
    const uint32_t H = L->H, I = L->I, E = L->E, k = L->k;
    const uint64_t rows = (uint64_t)cap * k + (L->has_shared ? cap : 0);
    const int NT = small_tile_rows_min();
    L->max_tiles = (int)(rows / NT + E + 2);
    Workspace& w = L->ws;
    bool ok = true;
    auto A = [&](size_t n) { void* p = o.alloc(n); ok = ok && p; return p; };
    w.xin = (float*)A((size_t)cap * H * 4);
    w.xout = (float*)A((size_t)cap * H * 4);
    w.xb = (__half*)A((size_t)cap * H * 2);
    w.topk_id = (int*)A((size_t)cap * k * 4);
    w.topk_w = (float*)A((size_t)cap * k * 4);
    w.local_rank = (int*)A((size_t)cap * k * 4);
    w.cta_cnt = (int*)A((size_t)route_cnt_stride(route_grid((int)cap)) * E * 4);
    w.ticket = (unsigned*)A(64);  // dispatch tickets: one per launch, plus one per 8-token group
    w.status = (unsigned*)A(16);
    w.expert_off = (int*)A((size_t)(E + 2) * 4);
    w.row_tok = (int*)A(rows * 4);
    w.row_slot = (int*)A(rows * 4);
    w.slot_row = (int*)A((size_t)cap * k * 4);
    w.n_rows = (int*)A(16);
    w.n_tiles = (int*)A(16);
    w.tiles = (int4*)A((size_t)L->max_tiles * 16);
    w.h = (__half*)A(rows * I * 2);
    w.xs = (__half*)A(rows * H * 2);
    w.hexp = (int8_t*)A(rows * (I / GV_EBLK));
    w.rowexp = (int*)A(rows * 4);
    w.logits = (float*)A((size_t)cap * E * 4);
    w.logits_part = (float*)A((size_t)LOGIT_SPLITS * cap * E * 4);
    if (need_y || L->ws_had_y) w.y = (float*)A(rows * H * 4);
    if (!ok) return fail(RMOE_ERR_OOM, "workspace cudaMalloc failed for %u tokens", cap);
    if (!make_rows_map(w.h, rows, I, L->hmap) || !make_rows_map(w.xs, rows, H, L->xsmap))
        return fail(RMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the token operands");
    cudaMemset(w.ticket, 0, 64);
    cudaMemset(w.status, 0, 16);
    L->ws_T = cap;
    L->ws_had_y = w.y != nullptr;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "workspace init");
    return RMOE_OK;
}

rmoe_status layer_forward_device(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s,
                                 uint32_t flags, bool given, uint32_t shared_t0, int64_t shared_n) {
    if (shared_n < 0) shared_n = T;
    const bool det = flags & RMOE_FLAG_DETERMINISTIC;
    if (given) {
        if (T > L->ws_T || (det && !L->ws.y)) return fail(RMOE_ERR_INVALID, "given routing without its workspace");
    } else {
        rmoe_status st = ensure_workspace(L, T, det);
        if (st) return st;
    }
    Workspace& w = L->ws;
    RouteParams rp{};
    rp.x = given ? nullptr : x;
    rp.router_w = L->router_w; rp.router_wh = L->router_wh; rp.router_wl = L->router_wl;
    rp.T = (int)T; rp.H = (int)L->H; rp.E = (int)L->E; rp.k = (int)L->k; rp.gate = (int)L->gate_kind;
    rp.has_shared = L->has_shared;
    rp.shared_t0 = (int)shared_t0; rp.shared_n = (int)shared_n;
    rp.given = given ? 1 : 0;
    rp.exact = (flags & RMOE_FLAG_EXACT_ROUTER) ? 1 : 0;
    rp.router_wmax = L->router_wmax;
    rp.refined = w.status + 1;
    rp.xb = w.xb;
    rp.rowexp = w.rowexp;
    rp.logits = given ? nullptr : w.logits;
    rp.logits_part = (given || (flags & RMOE_FLAG_EXACT_ROUTER)) ? nullptr : w.logits_part;
    rp.out_zero = det ? nullptr : out;
    rp.topk_id = w.topk_id; rp.topk_w = w.topk_w; rp.local_rank = w.local_rank; rp.cta_cnt = w.cta_cnt;
    rp.ticket = w.ticket; rp.expert_off = w.expert_off; rp.row_tok = w.row_tok; rp.row_slot = w.row_slot;
    rp.slot_row = w.slot_row; rp.n_rows = w.n_rows; rp.tiles = w.tiles; rp.n_tiles = w.n_tiles;
    // Large batches (>= 32 routed rows per expert on average) run the tcgen05 kernels, small
    // ones the bandwidth-bound mma.sync kernels; the flags force either path.
    bool use_tc = (uint64_t)T * L->k >= 32ull * L->E;
    if (flags & RMOE_FLAG_FORCE_SMALL) use_tc = false;
    if (flags & RMOE_FLAG_FORCE_LARGE) use_tc = true;
    rp.xs = use_tc ? w.xs : nullptr;
    // decode GEMV kernels where both expert types have register-fragment decoders
    const bool gv = !use_tc && gv_supported(L->wg.type, L->wd.type);
    const int tile_rows = use_tc ? tc_tile_rows() : gv ? gv_tile_rows((int)T) : small_tile_rows((int)T);
    const uint64_t rows_T = (uint64_t)T * L->k + (L->has_shared ? (uint64_t)shared_n : 0);
    // an expert with c rows takes at most c / tile_rows + 1 tiles, and at most rows_T experts
    // are touched: the grids launch no more tile slots than that
    const int max_tiles = (int)std::min<uint64_t>((uint64_t)L->max_tiles,
                                                  rows_T / tile_rows + std::min<uint64_t>(L->E + 2, rows_T));
    rp.max_tiles = max_tiles; rp.tile_rows = tile_rows; rp.status = w.status;
    const bool timing = flags & RMOE_FLAG_STAGE_TIMING;
    // decode batches of Q4_K / Q6_K experts: the whole layer in one launch where the flags allow
    // (fast router, atomic combine, no stage events)
    // RMOE_SMALL_LAYER=1 (read at every call) runs such decode batches as one cooperative launch;
    // off by default: on the B200 the routing + two decode kernels with programmatic dependent
    // launch measured faster (C3 b = 1: 0.046 against 0.070 ms; b = 8: 0.126 against 0.151 ms)
    const char* small_env = getenv("RMOE_SMALL_LAYER");
    const bool small_on = small_env && small_env[0] == '1';
    if (small_on && gv && !given && !det && !timing && !rp.exact &&
        layer_small_supported(L->wg.type, L->wd.type, (int)T, (int)L->E, (int)L->k)) {
        GroupedParams gp{};
        gp.gate = L->wg; gp.up = L->wu; gp.down = L->wd;
        gp.sgate = L->swg; gp.sup = L->swu; gp.sdown = L->swd;
        gp.H = (int)L->H; gp.I = (int)L->I; gp.E = (int)L->E; gp.k = (int)L->k;
        gp.xb = w.xb; gp.h = w.h; gp.hexp = w.hexp; gp.rowexp = w.rowexp; gp.y = nullptr; gp.out = out;
        gp.status = w.status;
        cudaError_t e = launch_layer_small(rp, gp, w.ticket + 14, L->small_grid, s);
        if (e == cudaSuccess) {
            L->last_tc = false;
            L->ev_valid = false;
            L->ev_combine = false;
            L->last_T = T;
            return RMOE_OK;
        }
        if (e != cudaErrorNotSupported && e != cudaErrorCooperativeLaunchTooLarge) return cuda_fail(e, "small layer launch");
        cudaGetLastError();  // not for this shape or device: the multi-launch path below
    }
    if (timing && !L->ev[0])
        for (auto& ev : L->ev) cudaEventCreate(&ev);
    auto mark = [&](int i) {
        if (timing) cudaEventRecord(L->ev[i], s);
    };
    mark(0);
    cudaError_t e = launch_route_dispatch(rp, s);
    if (e != cudaSuccess) return cuda_fail(e, "route_dispatch launch");
    mark(1);

    GroupedParams gp{};
    gp.gate = L->wg; gp.up = L->wu; gp.down = L->wd;
    gp.sgate = L->swg; gp.sup = L->swu; gp.sdown = L->swd;
    gp.H = (int)L->H; gp.I = (int)L->I; gp.E = (int)L->E; gp.k = (int)L->k;
    gp.xb = w.xb; gp.row_tok = w.row_tok; gp.row_slot = w.row_slot; gp.tiles = w.tiles; gp.n_tiles = w.n_tiles;
    gp.n_rows = w.n_rows;
    gp.topk_w = w.topk_w; gp.h = w.h; gp.hexp = w.hexp; gp.rowexp = w.rowexp; gp.y = det ? w.y : nullptr; gp.out = out; gp.status = w.status;
    TcMaps maps;
    if (use_tc) {
        memset(&maps, 0, sizeof maps);
        maps.w[0][0] = L->mg;
        maps.w[0][1] = L->mu;
        maps.w[1][0] = L->smg;
        maps.w[1][1] = L->smu;
        maps.b = L->xsmap;
    }
    // decode batches of several tokens stream the weights with TMA (gemv_tma.cu); single tokens
    // (a few tiles) keep the per-lane copies of gv_kernel, whose K-split CTAs fill the GPU
    const bool gvt = gv && T >= GVT_MIN_T;
    TcMaps gmaps;
    if (gvt) {
        memset(&gmaps, 0, sizeof gmaps);
        gmaps.w[0][0] = L->mg;
        gmaps.w[0][1] = L->mu;
        gmaps.w[1][0] = L->smg;
        gmaps.w[1][1] = L->smu;
    }
    TcMaps gmaps64;
    if (gvt && L->maps64) {
        memset(&gmaps64, 0, sizeof gmaps64);
        gmaps64.w[0][0] = L->mg64;
        gmaps64.w[0][1] = L->mu64;
        gmaps64.w[1][0] = L->smg64;
        gmaps64.w[1][1] = L->smu64;
    }
    e = use_tc ? launch_tc_gateup(gp, maps, max_tiles, s) : cudaErrorNotSupported;
    // 64-row gate/up blocks for batches of up to GVT64_MAX_T tokens (few tiles: the finer items
    // shorten the last wave); larger batches keep the 128-row blocks, which measured faster there
    const bool use64 = L->maps64 && T <= GVT64_MAX_T;
    if (!use_tc && gvt) e = launch_gvt_gateup(gp, gmaps, use64 ? &gmaps64 : nullptr, max_tiles, tile_rows, s);
    if (!use_tc && e == cudaErrorNotSupported)
        e = gv ? launch_gv_gateup(gp, max_tiles, tile_rows, (int)T, s) : launch_small_gateup(gp, max_tiles, tile_rows, s);
    if (e != cudaSuccess) return cuda_fail(e, "gate/up launch");
    mark(2);
    if (use_tc && (e = launch_rescale_h(gp, (int)rows_T, s)) != cudaSuccess) return cuda_fail(e, "h rescale launch");
    if (use_tc) {
        maps.w[0][0] = L->md;
        maps.w[1][0] = L->smd;
        maps.b = L->hmap;
    }
    if (gvt) {
        gmaps.w[0][0] = L->md;
        gmaps.w[1][0] = L->smd;
    }
    e = use_tc ? launch_tc_down(gp, maps, max_tiles, s) : cudaErrorNotSupported;
    if (!use_tc && gvt) e = launch_gvt_down(gp, gmaps, max_tiles, tile_rows, s);
    if (!use_tc && e == cudaErrorNotSupported)
        e = gv ? launch_gv_down(gp, max_tiles, tile_rows, (int)T, s) : launch_small_down(gp, max_tiles, tile_rows, s);
    if (e != cudaSuccess) return cuda_fail(e, "down launch");
    L->last_tc = use_tc;
    mark(3);
    if (det) {
        CombineParams cp{};
        cp.y = w.y; cp.slot_row = w.slot_row; cp.topk_w = w.topk_w;
        cp.T = (int)T; cp.H = (int)L->H; cp.k = (int)L->k; cp.has_shared = L->has_shared;
        cp.shared_t0 = rp.shared_t0; cp.shared_n = rp.shared_n; cp.expert_off = w.expert_off; cp.E = (int)L->E;
        cp.out = out;
        if ((e = launch_combine(cp, s)) != cudaSuccess) return cuda_fail(e, "combine launch");
    }
    mark(4);
    L->ev_valid = timing;
    L->ev_combine = det;
    L->last_T = T;
    return RMOE_OK;
}

}  // namespace rmoe

using namespace rmoe;

extern "C" {

const char* rmoe_last_error(void) { return g_err.c_str(); }

const char* rmoe_build_info(void) { return "rmoe sm_100a: route_dispatch, small_gateup/down (mma.sync fp16), combine"; }

rmoe_status rmoe_layer_create(const rmoe_layer_desc* d, rmoe_layer** out) {
    if (!out) return fail(RMOE_ERR_INVALID, "null output handle pointer");
    *out = nullptr;
    rmoe_status s = validate_desc(d);
    if (s) return s;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(RMOE_ERR_CUDA, "no CUDA device");
    if (d->device < 0 || d->device >= ndev) return fail(RMOE_ERR_INVALID, "device %d out of range", d->device);
    DeviceGuard g(d->device);
    rmoe_layer* L = new rmoe_layer();
    L->device = d->device;
    L->H = d->hidden; L->I = d->inter; L->E = d->n_experts;
    L->k = d->top_k < d->n_experts ? d->top_k : d->n_experts;  // top_k clamps to E (src/moe.rs:79)
    L->gate_kind = d->gate;
    L->has_shared = d->has_shared ? 1 : 0;
    L->E_local = L->E;
    L->E_router = L->E;
    if ((s = layer_upload(d, nullptr, d->n_experts, L))) { delete L; return s; }
    *out = L;
    return RMOE_OK;
}

// Host buffers in and out.  Large batches are split into token chunks so that the copies
// overlap the compute: chunk i's upload (copy-in stream), chunk i - 1's forward (the caller's
// stream) and chunk i - 2's download (copy-out stream) run at once; the forwards of the chunks
// run one after another on the caller's stream (they share the workspace).  A chunk keeps at
// least HOSTIO_ROWS_PER_EXPERT routed rows per expert on average, so the tensor-core tiles stay
// full; smaller batches, and calls that ask for routing or stage times, run as one chunk.
static constexpr uint64_t HOSTIO_ROWS_PER_EXPERT = 128;
static constexpr int HOSTIO_MAX_CHUNKS = 8;

static rmoe_status forward_host_io(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s,
                                   uint32_t flags) {
    rmoe_status st = ensure_workspace(L, T, flags & RMOE_FLAG_DETERMINISTIC);
    if (st) return st;
    const size_t H = L->H;
    uint64_t nc = (uint64_t)T * L->k / (HOSTIO_ROWS_PER_EXPERT * L->E);
    if (flags & (RMOE_FLAG_ROUTING_OUT | RMOE_FLAG_STAGE_TIMING)) nc = 1;
    nc = std::max<uint64_t>(1, std::min<uint64_t>(nc, HOSTIO_MAX_CHUNKS));
    cudaError_t e = cudaSuccess;
    if (nc == 1) {
        e = cudaMemcpyAsync(L->ws.xin, x, (size_t)T * H * 4, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "x upload");
        st = layer_forward_device(L, L->ws.xin, T, L->ws.xout, s, flags);
        if (st) return st;
        e = cudaMemcpyAsync(out, L->ws.xout, (size_t)T * H * 4, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_fail(e, "out download");
    } else {
        if (!L->io_stream[0]) {
            for (auto& q : L->io_stream)
                if ((e = cudaStreamCreateWithFlags(&q, cudaStreamNonBlocking)) != cudaSuccess)
                    return cuda_fail(e, "host-IO copy stream");
            for (auto& ev : L->io_ev)
                if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
                    return cuda_fail(e, "host-IO event");
        }
        cudaStream_t cin = L->io_stream[0], cout = L->io_stream[1];
        cudaEvent_t* up = L->io_ev;            // chunk i uploaded
        cudaEvent_t* done = L->io_ev + 8;      // chunk i computed
        cudaEvent_t entry = L->io_ev[16];      // work queued on s before this call
        // the staging buffers may still be read by work queued earlier on s
        if ((e = cudaEventRecord(entry, s)) != cudaSuccess || (e = cudaStreamWaitEvent(cin, entry, 0)) != cudaSuccess)
            return cuda_fail(e, "host-IO ordering");
        const uint32_t per = (uint32_t)((T + nc - 1) / nc);
        for (uint64_t i = 0; i < nc; i++) {
            const uint32_t t0 = (uint32_t)i * per, n = std::min<uint32_t>(per, T - t0);
            e = cudaMemcpyAsync(L->ws.xin + t0 * H, x + t0 * H, (size_t)n * H * 4, cudaMemcpyHostToDevice, cin);
            if (e == cudaSuccess) e = cudaEventRecord(up[i], cin);
            if (e != cudaSuccess) return cuda_fail(e, "x upload");
        }
        for (uint64_t i = 0; i < nc; i++) {
            const uint32_t t0 = (uint32_t)i * per, n = std::min<uint32_t>(per, T - t0);
            if ((e = cudaStreamWaitEvent(s, up[i], 0)) != cudaSuccess) return cuda_fail(e, "host-IO ordering");
            if ((st = layer_forward_device(L, L->ws.xin + t0 * H, n, L->ws.xout + t0 * H, s, flags))) return st;
            if ((e = cudaEventRecord(done[i], s)) != cudaSuccess || (e = cudaStreamWaitEvent(cout, done[i], 0)) != cudaSuccess)
                return cuda_fail(e, "host-IO ordering");
            e = cudaMemcpyAsync(out + t0 * H, L->ws.xout + t0 * H, (size_t)n * H * 4, cudaMemcpyDeviceToHost, cout);
            if (e != cudaSuccess) return cuda_fail(e, "out download");
        }
        if ((e = cudaStreamSynchronize(cout)) != cudaSuccess) return cuda_fail(e, "out download");
    }
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(e, "forward");
    unsigned status = 0;
    cudaMemcpy(&status, L->ws.status, 4, cudaMemcpyDeviceToHost);
    if (status) return fail(RMOE_ERR_DEVICE, "device status 0x%x", status);
    return RMOE_OK;
}

rmoe_status rmoe_layer_forward(rmoe_layer* L, const float* x, uint32_t T, float* out, void* stream, uint32_t flags) {
    if (!L) return fail(RMOE_ERR_INVALID, "null layer");
    if (T == 0) return RMOE_OK;
    if (!x || !out) return fail(RMOE_ERR_INVALID, "null x / out");
    DeviceGuard g(L->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (L->ep && (flags & RMOE_FLAG_HOST_IO)) return ep_forward_host(L, x, T, out, s, flags);
    if (L->ep) {
        if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
            return fail(RMOE_ERR_INVALID, "device x / out must be 16-byte aligned");
        return ep_forward(L, x, T, out, s, flags);
    }
    if (flags & RMOE_FLAG_HOST_IO) return forward_host_io(L, x, T, out, s, flags);
    // the router streams x and the combine writes out with 16-B vector accesses
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(RMOE_ERR_INVALID, "device x / out must be 16-byte aligned");
    return layer_forward_device(L, x, T, out, s, flags);
}

rmoe_status rmoe_layer_routing(rmoe_layer* L, uint32_t T, uint32_t* ids, float* weights) {
    if (!L) return fail(RMOE_ERR_INVALID, "null layer");
    if (L->ep) {
        DeviceGuard g(L->device);
        return ep_routing(L, T, ids, weights, nullptr);
    }
    if (T > L->last_T) return fail(RMOE_ERR_INVALID, "routing of %u tokens requested, last forward had %u", T, L->last_T);
    DeviceGuard g(L->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "sync");
    if (ids && (e = cudaMemcpy(ids, L->ws.topk_id, (size_t)T * L->k * 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "routing ids");
    if (weights && (e = cudaMemcpy(weights, L->ws.topk_w, (size_t)T * L->k * 4, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "routing weights");
    return RMOE_OK;
}

rmoe_status rmoe_layer_logits(rmoe_layer* L, uint32_t T, float* logits) {
    if (!L || !logits) return fail(RMOE_ERR_INVALID, "null layer / buffer");
    if (L->ep) {
        DeviceGuard g(L->device);
        return ep_routing(L, T, nullptr, nullptr, logits);
    }
    if (T > L->last_T) return fail(RMOE_ERR_INVALID, "logits of %u tokens requested, last forward had %u", T, L->last_T);
    DeviceGuard g(L->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(logits, L->ws.logits, (size_t)T * L->E * 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "logits");
}

rmoe_status rmoe_layer_router_refined(rmoe_layer* L, uint32_t* count) {
    if (!L || !count) return fail(RMOE_ERR_INVALID, "null layer / count");
    *count = 0;
    DeviceGuard g(L->device);
    unsigned* st = L->ep ? ep_status(L) : L->ws.status;
    if (!st) return RMOE_OK;  // no forward yet
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(count, st + 1, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(st + 1, 0, 4);
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "router refinement count");
}

rmoe_status rmoe_layer_stage_ms(rmoe_layer* L, float ms[4]) {
    if (!L || !ms) return fail(RMOE_ERR_INVALID, "null layer / buffer");
    if (!L->ev_valid) return fail(RMOE_ERR_INVALID, "last forward did not set RMOE_FLAG_STAGE_TIMING");
    DeviceGuard g(L->device);
    cudaError_t e = cudaEventSynchronize(L->ev[4]);
    if (e != cudaSuccess) return cuda_fail(e, "stage events");
    for (int i = 0; i < 4; i++) {
        ms[i] = 0.0f;
        cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]);
    }
    if (!L->ev_combine) ms[3] = 0.0f;
    return RMOE_OK;
}

void rmoe_layer_destroy(rmoe_layer* L) {
    if (!L) return;
    DeviceGuard g(L->device);
    cudaDeviceSynchronize();
    delete L;
}

}  // extern "C"

rmoe_layer::~rmoe_layer() {
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    for (auto& e : io_ev)
        if (e) cudaEventDestroy(e);
    for (auto& q : io_stream)
        if (q) cudaStreamDestroy(q);
    if (ep) rmoe::ep_free(this);
}

extern "C" {

rmoe_status rmoe_dequant(uint32_t t, const void* src, uint64_t nbytes, float* dst, void* stream) {
    uint32_t el, by;
    if (!block_geom(t, el, by)) return fail(RMOE_ERR_UNSUPPORTED, "no scalar dequant for ggml type %u", t);
    if (nbytes % by) return fail(RMOE_ERR_INVALID, "%s data len %llu not a multiple of %u", type_name(t), (unsigned long long)nbytes, by);
    if (nbytes && (!src || !dst)) return fail(RMOE_ERR_INVALID, "null src / dst");
    cudaError_t e = launch_dequant_raw((int)t, src, nbytes / by, dst, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "dequant launch");
}

rmoe_status rmoe_route(const float* logits, uint32_t T, uint32_t E, uint32_t k, uint32_t gate, uint32_t* ids,
                       float* weights, void* stream) {
    if (E == 0 || T == 0) return RMOE_OK;
    if (E > (uint32_t)MAX_E) return fail(RMOE_ERR_UNSUPPORTED, "E %u > %d", E, MAX_E);
    if (k > E) k = E;
    if (k == 0 || k > (uint32_t)MAX_K) return fail(RMOE_ERR_UNSUPPORTED, "k %u unsupported", k);
    if (gate > 1) return fail(RMOE_ERR_INVALID, "gate %u", gate);
    cudaError_t e = launch_route_only(logits, (int)T, (int)E, (int)k, (int)gate, reinterpret_cast<int*>(ids), weights,
                                      static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "route launch");
}

rmoe_status rmoe_route_grouped(const float* logits, const float* bias, uint32_t nbias, uint32_t T, uint32_t E,
                               uint32_t k, uint32_t n_groups, int32_t top_k_group, int32_t noaux, uint32_t* ids,
                               float* weights, void* stream) {
    if (E == 0 || T == 0) return RMOE_OK;
    if (!logits || !ids || !weights || (nbias && !bias)) return fail(RMOE_ERR_INVALID, "null pointer");
    if (E > (uint32_t)MAX_E) return fail(RMOE_ERR_UNSUPPORTED, "E %u > %d", E, MAX_E);
    if (k == 0 || k > (uint32_t)MAX_K) return fail(RMOE_ERR_UNSUPPORTED, "k %u unsupported (1..%d)", k, MAX_K);
    uint32_t ng = n_groups < 1 ? 1 : n_groups;  // n_groups.max(1).min(n), src/moe.rs:211
    if (ng > E) ng = E;
    if (ng > (uint32_t)RG_MAX_G) return fail(RMOE_ERR_UNSUPPORTED, "%u expert groups (at most %d)", ng, RG_MAX_G);
    const int tkg = top_k_group < 0 ? -1 : (int)std::min<uint32_t>((uint32_t)top_k_group, ng);
    cudaError_t e = launch_route_grouped(logits, bias, (int)std::min<uint32_t>(nbias, E), (int)T, (int)E, (int)k, (int)ng,
                                         tkg, noaux ? 1 : 0, ids, weights, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "grouped route launch");
}

}  // extern "C"
