/*
 * rmoe_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C restatement of rusty-engine's CPU algorithm for the MoE-layer hot path, used
 * by tests/ (parity), __graft_entry__.smoke() (self-check) and bench.py's cpu_baseline /
 * --impl reference arm (timed CPU baseline).  Nothing in the shipped library links or
 * calls this file.
 *
 * Two modes, both restated from the Rust sources (paths relative to the rusty-engine crate):
 *
 *   1. EXACT f32 (parity oracle).  quant::dequant (src/quant.rs:25-45, 106-357, 363-453)
 *      feeding the moe_layer_forward arithmetic (src/moe.rs:44-93, 97-117, 271-300,
 *      360-388): sequential f32 sums with no FMA contraction (Rust never contracts a*b+c),
 *      stable descending argsort, softmax over the chosen k, accumulation in chosen order.
 *      Compiled with -ffp-contract=off so every a*b+c rounds twice, as in Rust.
 *
 *   2. POOLED fused (timed CPU baseline).  QMat::matmul split rules (src/qmat.rs:13-26,
 *      185-272) over kernel::matmul_reuse (src/kernel.rs:1328-1477: tile 96, group 4,
 *      w_rows 2, r_block 1024) with the per-block dequantizers (src/kernel.rs:206-279,
 *      965-993) and the AVX2 f32 dots (src/kernel.rs:1002-1235, hsum order :367-372),
 *      a persistent worker pool with parallel_for semantics (src/pool.rs:93-163), pooled
 *      SwiGLU (src/forward.rs:152-182) and the weighted accumulate (src/moe.rs:373-380).
 *
 * Parity pins: the reference's own known-answer tests (f16 widening over all 65536
 * patterns, per-format dequant KATs, router and layer KATs) are restated in
 * tests/test_oracle_pins.py and must pass against this file before it is trusted.
 */
#define _GNU_SOURCE
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------ */
/* f16 widening: src/quant.rs:25-45 (exact IEEE binary16 -> binary32, bit manipulation)  */
/* ------------------------------------------------------------------------------------ */
static inline float bits_to_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

EXPORT float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t frac = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0 && frac == 0) {
        bits = sign;
    } else if (exp == 0) {
        uint32_t e = 113, f = frac; /* subnormal: shift until the implicit bit appears */
        while ((f & 0x400u) == 0) {
            f <<= 1;
            e -= 1;
        }
        bits = sign | (e << 23) | ((f & 0x3FFu) << 13);
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (frac << 13);
    }
    return bits_to_f32(bits);
}

static inline float rd_f16(const uint8_t* p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------------------------ */
/* Block geometry: src/quant.rs:75-101                                                   */
/* ------------------------------------------------------------------------------------ */
EXPORT int orc_block_info(uint32_t t, uint64_t* elements, uint64_t* bytes) {
    uint64_t e, b;
    switch (t) {
        case 0: e = 1; b = 4; break;
        case 1: case 30: e = 1; b = 2; break;
        case 2: e = 32; b = 18; break;
        case 6: e = 32; b = 22; break;
        case 8: e = 32; b = 34; break;
        case 12: e = 256; b = 144; break;
        case 13: e = 256; b = 176; break;
        case 14: e = 256; b = 210; break;
        default: return 0;
    }
    *elements = e;
    *bytes = b;
    return 1;
}

/* bytes_for_numel (src/quant.rs:92-101); returns 0 when not a whole number of blocks. */
EXPORT uint64_t orc_bytes_for_numel(uint32_t t, uint64_t numel, int* ok) {
    uint64_t e, b;
    *ok = 0;
    if (!orc_block_info(t, &e, &b)) return 0;
    if (e == 1) { *ok = 1; return numel * b; }
    if (numel % e) return 0;
    *ok = 1;
    return numel / e * b;
}

/* ------------------------------------------------------------------------------------ */
/* Per-block dequantizers.  Each follows the Rust scalar reference element for element:  */
/* Q4_0 src/quant.rs:106-119, Q5_0 :126-144, Q8_0 :147-158, get_scale_min_k4 :250-258,  */
/* Q4_K :263-289, Q5_K :294-323, Q6_K :328-357.  Output order is the GGUF element order. */
/* ------------------------------------------------------------------------------------ */
static void dq_q4_0(const uint8_t* b, float* out) {
    float d = rd_f16(b);
    for (int j = 0; j < 16; j++) {
        uint8_t q = b[2 + j];
        out[j] = (float)((int)(q & 0x0F) - 8) * d;
        out[j + 16] = (float)((int)(q >> 4) - 8) * d;
    }
}

static void dq_q5_0(const uint8_t* b, float* out) {
    float d = rd_f16(b);
    uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    const uint8_t* qs = b + 6;
    for (int j = 0; j < 16; j++) {
        uint32_t bit0 = ((qh >> j) & 1u) << 4;
        uint32_t bit1 = ((qh >> (j + 16)) & 1u) << 4;
        int x0 = (int)(((uint32_t)(qs[j] & 0x0F)) | bit0) - 16;
        int x1 = (int)(((uint32_t)(qs[j] >> 4)) | bit1) - 16;
        out[j] = (float)x0 * d;
        out[j + 16] = (float)x1 * d;
    }
}

static void dq_q8_0(const uint8_t* b, float* out) {
    float d = rd_f16(b);
    for (int j = 0; j < 32; j++) out[j] = (float)(int8_t)b[2 + j] * d;
}

static void scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static void dq_q4_k(const uint8_t* b, float* out) {
    float d = rd_f16(b), mn = rd_f16(b + 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    for (int grp = 0; grp < 4; grp++) {
        uint8_t sc0, m0, sc1, m1;
        scale_min_k4(grp * 2, scales, &sc0, &m0);
        scale_min_k4(grp * 2 + 1, scales, &sc1, &m1);
        float d1 = d * (float)sc0, dm1 = mn * (float)m0;
        float d2 = d * (float)sc1, dm2 = mn * (float)m1;
        for (int l = 0; l < 32; l++) {
            uint8_t q = qs[grp * 32 + l];
            out[grp * 64 + l] = d1 * (float)(q & 0xF) - dm1;
            out[grp * 64 + 32 + l] = d2 * (float)(q >> 4) - dm2;
        }
    }
}

static void dq_q5_k(const uint8_t* b, float* out) {
    float d = rd_f16(b), mn = rd_f16(b + 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int grp = 0; grp < 4; grp++) {
        uint8_t sc0, m0, sc1, m1;
        scale_min_k4(grp * 2, scales, &sc0, &m0);
        scale_min_k4(grp * 2 + 1, scales, &sc1, &m1);
        float d1 = d * (float)sc0, dm1 = mn * (float)m0;
        float d2 = d * (float)sc1, dm2 = mn * (float)m1;
        uint8_t u1 = (uint8_t)(1u << (2 * grp)), u2 = (uint8_t)(2u << (2 * grp));
        for (int l = 0; l < 32; l++) {
            int lo = (qs[grp * 32 + l] & 0xF) + ((qh[l] & u1) ? 16 : 0);
            int hi = (qs[grp * 32 + l] >> 4) + ((qh[l] & u2) ? 16 : 0);
            out[grp * 64 + l] = d1 * (float)lo - dm1;
            out[grp * 64 + 32 + l] = d2 * (float)hi - dm2;
        }
    }
}

static void dq_q6_k(const uint8_t* b, float* out) {
    float d = rd_f16(b + 208);
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    for (int half = 0; half < 2; half++) {
        const uint8_t* qlh = ql + half * 64;
        const uint8_t* qhh = qh + half * 32;
        const int8_t* sch = sc + half * 8;
        float* o = out + half * 128;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = ((qlh[l] & 0xF) | ((qhh[l] & 3) << 4)) - 32;
            int q2 = ((qlh[l + 32] & 0xF) | (((qhh[l] >> 2) & 3) << 4)) - 32;
            int q3 = ((qlh[l] >> 4) | (((qhh[l] >> 4) & 3) << 4)) - 32;
            int q4 = ((qlh[l + 32] >> 4) | (((qhh[l] >> 6) & 3) << 4)) - 32;
            o[l] = d * (float)sch[is] * (float)q1;
            o[l + 32] = d * (float)sch[is + 2] * (float)q2;
            o[l + 64] = d * (float)sch[is + 4] * (float)q3;
            o[l + 96] = d * (float)sch[is + 6] * (float)q4;
        }
    }
}

typedef void (*dq_fn)(const uint8_t*, float*);

static int quant_geom(uint32_t t, int* bvals, int* bbytes, dq_fn* fn) {
    switch (t) {
        case 2: *bvals = 32; *bbytes = 18; *fn = dq_q4_0; return 1;
        case 6: *bvals = 32; *bbytes = 22; *fn = dq_q5_0; return 1;
        case 8: *bvals = 32; *bbytes = 34; *fn = dq_q8_0; return 1;
        case 12: *bvals = 256; *bbytes = 144; *fn = dq_q4_k; return 1;
        case 13: *bvals = 256; *bbytes = 176; *fn = dq_q5_k; return 1;
        case 14: *bvals = 256; *bbytes = 210; *fn = dq_q6_k; return 1;
        default: return 0;
    }
}

static __thread char g_err[256];
EXPORT const char* orc_last_error(void) { return g_err; }

/*
 * quant::dequant dispatch (src/quant.rs:363-453).  Returns the element count, or -1 with
 * orc_last_error() holding the reference's message for a ragged length / unknown type.
 */
EXPORT int64_t orc_dequant(uint32_t t, const uint8_t* data, uint64_t len, float* out) {
    if (t == 0) {
        if (len % 4) { snprintf(g_err, sizeof g_err, "F32 data len %lu not a multiple of 4", (unsigned long)len); return -1; }
        memcpy(out, data, len);
        return (int64_t)(len / 4);
    }
    if (t == 1) {
        if (len % 2) { snprintf(g_err, sizeof g_err, "F16 data len %lu not a multiple of 2", (unsigned long)len); return -1; }
        for (uint64_t i = 0; i < len / 2; i++) out[i] = rd_f16(data + 2 * i);
        return (int64_t)(len / 2);
    }
    if (t == 30) {
        if (len % 2) { snprintf(g_err, sizeof g_err, "BF16 data len %lu not a multiple of 2", (unsigned long)len); return -1; }
        for (uint64_t i = 0; i < len / 2; i++) out[i] = bits_to_f32((uint32_t)(data[2 * i] | (data[2 * i + 1] << 8)) << 16);
        return (int64_t)(len / 2);
    }
    int bv, bb;
    dq_fn fn;
    if (!quant_geom(t, &bv, &bb, &fn)) {
        snprintf(g_err, sizeof g_err, "no scalar dequant for ggml type %u", t);
        return -1;
    }
    if (len % (uint64_t)bb) {
        static const char* names[15] = {0, 0, "Q4_0", 0, 0, 0, "Q5_0", 0, "Q8_0", 0, 0, 0, "Q4_K", "Q5_K", "Q6_K"};
        snprintf(g_err, sizeof g_err, "%s data len %lu not a multiple of %d", names[t], (unsigned long)len, bb);
        return -1;
    }
    uint64_t nb = len / (uint64_t)bb;
    for (uint64_t i = 0; i < nb; i++) fn(data + i * bb, out + i * bv);
    return (int64_t)(nb * bv);
}

/* ------------------------------------------------------------------------------------ */
/* Router and FFN arithmetic: src/moe.rs                                                 */
/* ------------------------------------------------------------------------------------ */
EXPORT float orc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); } /* moe.rs:44-46 */
EXPORT float orc_silu(float x) { return x * orc_sigmoid(x); }           /* moe.rs:49-51 */

/* softmax_in_place (moe.rs:61-72): max fold, exp(v - max), sequential sum, divide. */
EXPORT void orc_softmax_in_place(float* x, uint64_t n) {
    float mx = -INFINITY;
    for (uint64_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
    for (uint64_t i = 0; i < n; i++) x[i] = expf(x[i] - mx);
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; i++) sum += x[i];
    if (sum != 0.0f)
        for (uint64_t i = 0; i < n; i++) x[i] /= sum;
}

/*
 * Stable descending argsort of `s` (Rust `sort_by(|a,b| s[b].partial_cmp(&s[a]))` is a
 * stable merge sort: equal keys keep ascending index order).  Insertion sort is stable
 * and gives the same permutation for non-NaN keys.
 */
static void argsort_desc_stable(const float* s, uint32_t* idx, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) idx[i] = (uint32_t)i;
    for (uint64_t i = 1; i < n; i++) {
        uint32_t v = idx[i];
        uint64_t j = i;
        while (j > 0 && s[idx[j - 1]] < s[v]) {
            idx[j] = idx[j - 1];
            j--;
        }
        idx[j] = v;
    }
}

/* top_k (moe.rs:75-93): stable argsort desc, softmax over the k chosen logits. */
EXPORT uint64_t orc_top_k(const float* scores, uint64_t n, uint64_t k, uint32_t* ids, float* w) {
    if (n == 0) return 0;
    if (k > n) k = n;
    uint32_t* idx = malloc(n * sizeof(uint32_t));
    argsort_desc_stable(scores, idx, n);
    for (uint64_t i = 0; i < k; i++) { ids[i] = idx[i]; w[i] = scores[idx[i]]; }
    orc_softmax_in_place(w, k);
    free(idx);
    return k;
}

/* top_k_sigmoid (moe.rs:97-117): sort by sigmoid, weight = sig / sum(sig of chosen). */
EXPORT uint64_t orc_top_k_sigmoid(const float* scores, uint64_t n, uint64_t k, uint32_t* ids, float* w) {
    if (n == 0) return 0;
    float* sig = malloc(n * sizeof(float));
    uint32_t* idx = malloc(n * sizeof(uint32_t));
    for (uint64_t i = 0; i < n; i++) sig[i] = orc_sigmoid(scores[i]);
    if (k > n) k = n;
    argsort_desc_stable(sig, idx, n);
    float wsum = 0.0f;
    for (uint64_t i = 0; i < k; i++) wsum += sig[idx[i]];
    for (uint64_t i = 0; i < k; i++) {
        ids[i] = idx[i];
        w[i] = wsum == 0.0f ? 0.0f : sig[idx[i]] / wsum;
    }
    free(sig);
    free(idx);
    return k;
}

/* route (moe.rs:120-125): gate 0 = Softmax, 1 = Sigmoid. */
EXPORT uint64_t orc_route(const float* logits, uint64_t n, int gate, uint64_t k, uint32_t* ids, float* w) {
    return gate == 1 ? orc_top_k_sigmoid(logits, n, k, ids, w) : orc_top_k(logits, n, k, ids, w);
}

/*
 * Group routing (moe.rs:133-268).  noaux != 0 selects route_noaux_tc (group score = sum of
 * the top-2 members), else route_group (group score = sum of all members).  top_k_group < 0
 * means "None" (every group allowed).
 */
EXPORT uint64_t orc_route_grouped(const float* logits, const float* bias, uint64_t nbias, uint64_t n,
                                  uint64_t n_groups, uint64_t top_k, int64_t top_k_group, int noaux,
                                  uint32_t* ids, float* w) {
    if (n == 0) return 0;
    float* e = malloc(n * sizeof(float));
    for (uint64_t i = 0; i < n; i++) e[i] = orc_sigmoid(logits[i] + (i < nbias ? bias[i] : 0.0f));
    uint64_t ng = n_groups < 1 ? 1 : n_groups;
    if (ng > n) ng = n;
    float* gs = calloc(ng, sizeof(float));
    if (noaux) {
        float* t1 = malloc(ng * sizeof(float));
        float* t2 = malloc(ng * sizeof(float));
        for (uint64_t g = 0; g < ng; g++) t1[g] = t2[g] = -3.40282347e38f; /* f32::MIN */
        for (uint64_t i = 0; i < n; i++) {
            uint64_t g = i * ng / n;
            if (e[i] >= t1[g]) { t2[g] = t1[g]; t1[g] = e[i]; }
            else if (e[i] > t2[g]) t2[g] = e[i];
        }
        for (uint64_t g = 0; g < ng; g++) gs[g] = t1[g] + (t2[g] == -3.40282347e38f ? 0.0f : t2[g]);
        free(t1);
        free(t2);
    } else {
        for (uint64_t i = 0; i < n; i++) gs[i * ng / n] += e[i];
    }
    char* allowed = malloc(ng);
    if (top_k_group < 0) {
        memset(allowed, 1, ng);
    } else {
        uint32_t* ord = malloc(ng * sizeof(uint32_t));
        argsort_desc_stable(gs, ord, ng);
        memset(allowed, 0, ng);
        uint64_t tkg = (uint64_t)top_k_group < ng ? (uint64_t)top_k_group : ng;
        for (uint64_t i = 0; i < tkg; i++) allowed[ord[i]] = 1;
        free(ord);
    }
    /* candidates in ascending index order, then stable sort by score */
    uint64_t nc = 0;
    float* cs = malloc(n * sizeof(float));
    uint32_t* cid = malloc(n * sizeof(uint32_t));
    for (uint64_t i = 0; i < n; i++)
        if (allowed[i * ng / n]) { cid[nc] = (uint32_t)i; cs[nc] = e[i]; nc++; }
    uint32_t* ord = malloc((nc ? nc : 1) * sizeof(uint32_t));
    argsort_desc_stable(cs, ord, nc);
    uint64_t k = top_k < nc ? top_k : nc;
    float wsum = 0.0f;
    for (uint64_t i = 0; i < k; i++) wsum += cs[ord[i]];
    for (uint64_t i = 0; i < k; i++) {
        ids[i] = cid[ord[i]];
        w[i] = wsum == 0.0f ? 0.0f : cs[ord[i]] / wsum;
    }
    free(e); free(gs); free(allowed); free(cs); free(cid); free(ord);
    return k;
}

/* matvec (moe.rs:271-277): each row a sequential f32 sum of products, starting at 0. */
EXPORT void orc_matvec(const float* w, uint64_t m, uint64_t n, const float* x, float* out) {
    for (uint64_t r = 0; r < m; r++) {
        const float* row = w + r * n;
        float s = 0.0f;
        for (uint64_t i = 0; i < n; i++) s += row[i] * x[i];
        out[r] = s;
    }
}

/* expert_ffn (moe.rs:288-300): down(swiglu(gate x, up x)). */
EXPORT void orc_expert_ffn(const float* x, const float* gw, const float* uw, const float* dw,
                           uint64_t hidden, uint64_t inter, float* out) {
    float* g = malloc(inter * sizeof(float));
    float* u = malloc(inter * sizeof(float));
    orc_matvec(gw, inter, hidden, x, g);
    orc_matvec(uw, inter, hidden, x, u);
    for (uint64_t i = 0; i < inter; i++) g[i] = orc_silu(g[i]) * u[i]; /* swiglu moe.rs:280-283 */
    orc_matvec(dw, hidden, inter, g, out);
    free(g);
    free(u);
}

/*
 * combine (moe.rs:306-345): out = sum_k w_k * routed_k (+ shared), in order.  Returns -1 on
 * the reference's error cases (count mismatch is checked by the caller's arguments here).
 */
EXPORT void orc_combine(const float* routed, const float* weights, uint64_t k, uint64_t dim,
                        const float* shared, float* out) {
    for (uint64_t i = 0; i < dim; i++) out[i] = 0.0f;
    for (uint64_t j = 0; j < k; j++)
        for (uint64_t i = 0; i < dim; i++) out[i] += routed[j * dim + i] * weights[j];
    if (shared)
        for (uint64_t i = 0; i < dim; i++) out[i] += shared[i];
}

/*
 * moe_layer_forward (moe.rs:360-388) for f32 ExpertWeights, one token.  gate_w/up_w/down_w
 * are arrays of n_experts pointers (NULL = expert missing, silently skipped like
 * experts.get(e.id) at moe.rs:374).  ids/wts (optional) receive the routing.
 */
EXPORT void orc_moe_layer_forward(const float* hidden, uint64_t dmodel, const float* router_w, uint64_t n_experts,
                                  const float* const* gate_w, const float* const* up_w, const float* const* down_w,
                                  const float* sh_gate, const float* sh_up, const float* sh_down, uint64_t inter,
                                  int gate, uint64_t top_k, float* out, uint32_t* ids_out, float* w_out) {
    float* logits = malloc(n_experts * sizeof(float));
    orc_matvec(router_w, n_experts, dmodel, hidden, logits);
    uint32_t* ids = malloc((n_experts ? n_experts : 1) * sizeof(uint32_t));
    float* wts = malloc((n_experts ? n_experts : 1) * sizeof(float));
    uint64_t k = orc_route(logits, n_experts, gate, top_k, ids, wts);
    float* eo = malloc(dmodel * sizeof(float));
    for (uint64_t i = 0; i < dmodel; i++) out[i] = 0.0f;
    for (uint64_t j = 0; j < k; j++) {
        uint32_t e = ids[j];
        if (ids_out) ids_out[j] = e;
        if (w_out) w_out[j] = wts[j];
        if (!gate_w[e]) continue;
        orc_expert_ffn(hidden, gate_w[e], up_w[e], down_w[e], dmodel, inter, eo);
        for (uint64_t i = 0; i < dmodel; i++) out[i] += wts[j] * eo[i];
    }
    if (sh_gate) {
        orc_expert_ffn(hidden, sh_gate, sh_up, sh_down, dmodel, inter, eo);
        for (uint64_t i = 0; i < dmodel; i++) out[i] += eo[i];
    }
    free(logits); free(ids); free(wts); free(eo);
}

/* ------------------------------------------------------------------------------------ */
/* Quantized MoE layer, exact mode: quant::dequant composed with moe_layer_forward.       */
/* GGUF expert layout (src/model.rs:366-391, src/qmat.rs:310-311): ffn_{gate,up}_exps    */
/* [H, I, E] = E experts of I rows x row_bytes(H); ffn_down_exps [I, H, E] = E experts    */
/* of H rows x row_bytes(I).  One token per "call", tokens spread over threads.           */
/* ------------------------------------------------------------------------------------ */
typedef struct {
    uint32_t type;
    const uint8_t* data;
} orc_qtensor;

static uint64_t row_bytes_of(uint32_t t, uint64_t n) {
    uint64_t e, b;
    if (!orc_block_info(t, &e, &b)) return 0;
    return n / e * b;
}

/* Dot of one stored row (dequantized exactly like quant::dequant) with x, sequential sum. */
static float qrow_dot_exact(uint32_t t, const uint8_t* row, uint64_t n, const float* x, float* scratch) {
    orc_dequant(t, row, row_bytes_of(t, n), scratch);
    float s = 0.0f;
    for (uint64_t i = 0; i < n; i++) s += scratch[i] * x[i];
    return s;
}

static void qmatvec_exact(uint32_t t, const uint8_t* w, uint64_t m, uint64_t n, const float* x, float* out,
                          float* scratch) {
    uint64_t rb = row_bytes_of(t, n);
    for (uint64_t r = 0; r < m; r++) out[r] = qrow_dot_exact(t, w + r * rb, n, x, scratch);
}

typedef struct {
    const float* x;
    uint64_t T, H, I, E, k;
    const float* router_w;
    orc_qtensor g, u, d;
    int has_shared;
    orc_qtensor sg, su, sd;
    int gate;
    float* out;
    uint32_t* ids;
    float* wts;
    float* logits;
    atomic_ulong next;
} layer_job;

static void layer_one_token(layer_job* J, uint64_t t, float* scratch, float* gbuf, float* ubuf, float* eo) {
    const float* x = J->x + t * J->H;
    float* out = J->out + t * J->H;
    float* logits = J->logits + t * J->E;
    orc_matvec(J->router_w, J->E, J->H, x, logits);
    uint32_t ids[256];
    float wts[256];
    uint64_t k = orc_route(logits, J->E, J->gate, J->k, ids, wts);
    uint64_t rbg = row_bytes_of(J->g.type, J->H), rbu = row_bytes_of(J->u.type, J->H),
             rbd = row_bytes_of(J->d.type, J->I);
    for (uint64_t i = 0; i < J->H; i++) out[i] = 0.0f;
    for (uint64_t j = 0; j < k; j++) {
        uint64_t e = ids[j];
        J->ids[t * J->k + j] = (uint32_t)e;
        J->wts[t * J->k + j] = wts[j];
        qmatvec_exact(J->g.type, J->g.data + e * J->I * rbg, J->I, J->H, x, gbuf, scratch);
        qmatvec_exact(J->u.type, J->u.data + e * J->I * rbu, J->I, J->H, x, ubuf, scratch);
        for (uint64_t i = 0; i < J->I; i++) gbuf[i] = orc_silu(gbuf[i]) * ubuf[i];
        qmatvec_exact(J->d.type, J->d.data + e * J->H * rbd, J->H, J->I, gbuf, eo, scratch);
        for (uint64_t i = 0; i < J->H; i++) out[i] += wts[j] * eo[i];
    }
    if (J->has_shared) {
        qmatvec_exact(J->sg.type, J->sg.data, J->I, J->H, x, gbuf, scratch);
        qmatvec_exact(J->su.type, J->su.data, J->I, J->H, x, ubuf, scratch);
        for (uint64_t i = 0; i < J->I; i++) gbuf[i] = orc_silu(gbuf[i]) * ubuf[i];
        qmatvec_exact(J->sd.type, J->sd.data, J->H, J->I, gbuf, eo, scratch);
        for (uint64_t i = 0; i < J->H; i++) out[i] += eo[i];
    }
}

static void* layer_worker(void* arg) {
    layer_job* J = arg;
    uint64_t big = J->H > J->I ? J->H : J->I;
    float* scratch = malloc(big * sizeof(float));
    float* gbuf = malloc(J->I * sizeof(float));
    float* ubuf = malloc(J->I * sizeof(float));
    float* eo = malloc(J->H * sizeof(float));
    for (;;) {
        uint64_t t = atomic_fetch_add(&J->next, 1);
        if (t >= J->T) break;
        layer_one_token(J, t, scratch, gbuf, ubuf, eo);
    }
    free(scratch); free(gbuf); free(ubuf); free(eo);
    return NULL;
}

/*
 * Exact-mode quantized layer over T tokens (each token = one moe_layer_forward call).
 * Outputs out[T*H], ids/wts[T*k] (routing in chosen order), logits[T*E] (f32 router logits).
 * Shared-expert tensors are used when sg_data != NULL.  Work is spread over `threads`.
 */
EXPORT void orc_moe_layer_q_exact(const float* x, uint64_t T, uint64_t H, uint64_t I, uint64_t E, uint64_t k,
                                  int gate, const float* router_w, uint32_t gt, const uint8_t* gd, uint32_t ut,
                                  const uint8_t* ud, uint32_t dt, const uint8_t* dd, uint32_t sgt,
                                  const uint8_t* sgd, uint32_t sut, const uint8_t* sud, uint32_t sdt,
                                  const uint8_t* sdd, float* out, uint32_t* ids, float* wts, float* logits,
                                  int threads) {
    layer_job J = {.x = x, .T = T, .H = H, .I = I, .E = E, .k = k, .router_w = router_w,
                   .g = {gt, gd}, .u = {ut, ud}, .d = {dt, dd}, .has_shared = sgd != NULL,
                   .sg = {sgt, sgd}, .su = {sut, sud}, .sd = {sdt, sdd}, .gate = gate,
                   .out = out, .ids = ids, .wts = wts, .logits = logits};
    atomic_init(&J.next, 0);
    if (threads < 1) threads = 1;
    pthread_t* th = malloc(sizeof(pthread_t) * (size_t)threads);
    for (int i = 0; i < threads; i++) pthread_create(&th[i], NULL, layer_worker, &J);
    for (int i = 0; i < threads; i++) pthread_join(th[i], NULL);
    free(th);
}

/* Router logits exactly as moe::matvec computes them, for T tokens, tokens over threads. */
typedef struct {
    const float* x;
    const float* w;
    uint64_t T, H, E;
    float* out;
    atomic_ulong next;
} lg_job;

static void* lg_worker(void* arg) {
    lg_job* J = arg;
    for (;;) {
        uint64_t t = atomic_fetch_add(&J->next, 1);
        if (t >= J->T) break;
        orc_matvec(J->w, J->E, J->H, J->x + t * J->H, J->out + t * J->E);
    }
    return NULL;
}

EXPORT void orc_router_logits(const float* x, uint64_t T, uint64_t H, const float* router_w, uint64_t E, float* out,
                              int threads) {
    lg_job J = {x, router_w, T, H, E, out};
    atomic_init(&J.next, 0);
    if (threads < 1) threads = 1;
    pthread_t* th = malloc(sizeof(pthread_t) * (size_t)threads);
    for (int i = 0; i < threads; i++) pthread_create(&th[i], NULL, lg_worker, &J);
    for (int i = 0; i < threads; i++) pthread_join(th[i], NULL);
    free(th);
}

/* Route T rows of logits (ids/w are T x k). */
EXPORT void orc_route_batch(const float* logits, uint64_t T, uint64_t E, int gate, uint64_t k, uint32_t* ids, float* w) {
    for (uint64_t t = 0; t < T; t++) orc_route(logits + t * E, E, gate, k, ids + t * k, w + t * k);
}

/* Router logits in f64 (for classifying near-ties when comparing index sets). */
EXPORT void orc_router_logits_f64(const float* x, uint64_t T, uint64_t H, const float* router_w, uint64_t E,
                                  double* out) {
    for (uint64_t t = 0; t < T; t++)
        for (uint64_t e = 0; e < E; e++) {
            double s = 0.0;
            for (uint64_t i = 0; i < H; i++) s += (double)router_w[e * H + i] * (double)x[t * H + i];
            out[t * E + e] = s;
        }
}

/* ------------------------------------------------------------------------------------ */
/* Pooled fused path (timed CPU baseline).                                                */
/* ------------------------------------------------------------------------------------ */

/* Persistent worker pool with parallel_for semantics (src/pool.rs:93-163): N detached
 * workers take job indices; the caller blocks until every job of its call has finished.
 * parallel_for must not nest (the reference has the same rule, src/pool.rs:10-11). */
typedef void (*job_fn)(void* ctx, uint64_t i);
static struct {
    pthread_mutex_t mu;
    pthread_cond_t work, done;
    int nworkers;
    job_fn fn;
    void* ctx;
    uint64_t njobs, next, pending;
    uint64_t gen;
} P = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER, 0, 0, 0, 0, 0, 0, 0};

static void* pool_worker(void* arg) {
    (void)arg;
    pthread_mutex_lock(&P.mu);
    for (;;) {
        while (P.next >= P.njobs) pthread_cond_wait(&P.work, &P.mu);
        uint64_t i = P.next++;
        job_fn fn = P.fn;
        void* ctx = P.ctx;
        pthread_mutex_unlock(&P.mu);
        fn(ctx, i);
        pthread_mutex_lock(&P.mu);
        if (--P.pending == 0) pthread_cond_broadcast(&P.done);
    }
    return NULL;
}

/* RUSTY_THREADS analogue: start `n` workers once (later calls only report the count). */
EXPORT int orc_pool_init(int n) {
    pthread_mutex_lock(&P.mu);
    if (P.nworkers == 0) {
        if (n < 1) n = 1;
        if (n > 256) n = 256;
        for (int i = 0; i < n; i++) {
            pthread_t t;
            pthread_attr_t a;
            pthread_attr_init(&a);
            pthread_attr_setdetachstate(&a, PTHREAD_CREATE_DETACHED);
            pthread_create(&t, &a, pool_worker, NULL);
            pthread_attr_destroy(&a);
        }
        P.nworkers = n;
    }
    int r = P.nworkers;
    pthread_mutex_unlock(&P.mu);
    return r;
}

static int requested_threads(void) { return P.nworkers > 0 ? P.nworkers : 1; }

static void parallel_for(uint64_t jobs, job_fn fn, void* ctx) {
    if (jobs <= 1 || P.nworkers == 0) {
        for (uint64_t i = 0; i < jobs; i++) fn(ctx, i);
        return;
    }
    pthread_mutex_lock(&P.mu);
    P.fn = fn;
    P.ctx = ctx;
    P.pending = jobs;
    P.next = 0;
    P.njobs = jobs;
    pthread_cond_broadcast(&P.work);
    while (P.pending > 0) pthread_cond_wait(&P.done, &P.mu);
    P.njobs = 0;
    P.next = 0;
    pthread_mutex_unlock(&P.mu);
}

/* hsum_ps_sse2 (src/kernel.rs:367-372) applied to lo128 + hi128 of an 8-lane accumulator. */
static inline float hsum8(__m256 acc) {
    __m128 v = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    __m128 t = _mm_add_ps(v, _mm_movehl_ps(v, v));
    t = _mm_add_ss(t, _mm_shuffle_ps(t, t, 0x55));
    return _mm_cvtss_f32(t);
}

/* dot_f32_avx2 (src/kernel.rs:1002-1027): one 8-lane FMA chain, hsum, scalar tail. */
static float dot_f32(const float* a, const float* b, uint64_t n) {
    __m256 acc = _mm256_setzero_ps();
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
    float s = hsum8(acc);
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

/* dot_f32_avx2_x4 (src/kernel.rs:1048-1085): four dots sharing the weight load. */
static void dot_f32_x4(const float* a, const float* const* b, uint64_t n, float* out) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 av = _mm256_loadu_ps(a + i);
        for (int k = 0; k < 4; k++) acc[k] = _mm256_fmadd_ps(av, _mm256_loadu_ps(b[k] + i), acc[k]);
    }
    for (int k = 0; k < 4; k++) {
        out[k] = hsum8(acc[k]);
        for (uint64_t j = i; j < n; j++) out[k] += a[j] * b[k][j];
    }
}

/* dot_f32_avx2_x4x2 (src/kernel.rs:1160-1202): two weight rows x four activation rows. */
static void dot_f32_x4x2(const float* a0, const float* a1, const float* const* b, uint64_t n, float* o0,
                         float* o1) {
    __m256 c0[4], c1[4];
    for (int k = 0; k < 4; k++) c0[k] = c1[k] = _mm256_setzero_ps();
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 av0 = _mm256_loadu_ps(a0 + i), av1 = _mm256_loadu_ps(a1 + i);
        for (int k = 0; k < 4; k++) {
            __m256 bv = _mm256_loadu_ps(b[k] + i);
            c0[k] = _mm256_fmadd_ps(av0, bv, c0[k]);
            c1[k] = _mm256_fmadd_ps(av1, bv, c1[k]);
        }
    }
    for (int k = 0; k < 4; k++) {
        o0[k] = hsum8(c0[k]);
        o1[k] = hsum8(c1[k]);
        for (uint64_t j = i; j < n; j++) o0[k] += a0[j] * b[k][j];
        for (uint64_t j = i; j < n; j++) o1[k] += a1[j] * b[k][j];
    }
}

enum { ROW_TILE = 96, ROW_GROUP = 4, W_ROWS = 2, R_BLOCK = 1024 }; /* src/kernel.rs:1328-1369 */

static void dequant_row(const uint8_t* raw, float* out, uint64_t n, int bbytes, int bvals, dq_fn fn) {
    for (uint64_t b = 0; b < n / (uint64_t)bvals; b++) fn(raw + b * bbytes, out + b * bvals);
}

/*
 * matmul_reuse (src/kernel.rs:1383-1477) with w_rows = 2, group = 4: per weight-row block,
 * per 96-row activation tile, dequantize two weight rows once and dot them against the
 * tile four activation rows at a time; single-row tails use the plain dot.
 */
static void matmul_reuse(const uint8_t* w, uint64_t m, uint64_t n, const float* x, uint64_t rows, uint32_t t,
                         float* out) {
    int bv, bb;
    dq_fn fn;
    quant_geom(t, &bv, &bb, &fn);
    uint64_t rbytes = n / (uint64_t)bv * (uint64_t)bb;
    float* rb0buf = aligned_alloc(64, ((n * 4 + 63) / 64) * 64);
    float* rb1buf = aligned_alloc(64, ((n * 4 + 63) / 64) * 64);
    for (uint64_t rb0 = 0; rb0 < m; rb0 += R_BLOCK) {
        uint64_t rb1 = rb0 + R_BLOCK < m ? rb0 + R_BLOCK : m;
        for (uint64_t r0 = 0; r0 < rows; r0 += ROW_TILE) {
            uint64_t r1 = r0 + ROW_TILE < rows ? r0 + ROW_TILE : rows;
            uint64_t r = rb0;
            while (r < rb1) {
                if (r + 1 < rb1) {
                    dequant_row(w + r * rbytes, rb0buf, n, bb, bv, fn);
                    dequant_row(w + (r + 1) * rbytes, rb1buf, n, bb, bv, fn);
                    uint64_t row = r0;
                    for (; row + 4 <= r1; row += 4) {
                        const float* b[4] = {x + row * n, x + (row + 1) * n, x + (row + 2) * n, x + (row + 3) * n};
                        float g0[4], g1[4];
                        dot_f32_x4x2(rb0buf, rb1buf, b, n, g0, g1);
                        for (int k = 0; k < 4; k++) {
                            out[(row + k) * m + r] = g0[k];
                            out[(row + k) * m + r + 1] = g1[k];
                        }
                    }
                    for (; row < r1; row++) {
                        out[row * m + r] = dot_f32(rb0buf, x + row * n, n);
                        out[row * m + r + 1] = dot_f32(rb1buf, x + row * n, n);
                    }
                    r += 2;
                } else {
                    dequant_row(w + r * rbytes, rb0buf, n, bb, bv, fn);
                    uint64_t row = r0;
                    for (; row + 4 <= r1; row += 4) {
                        const float* b[4] = {x + row * n, x + (row + 1) * n, x + (row + 2) * n, x + (row + 3) * n};
                        float g[4];
                        dot_f32_x4(rb0buf, b, n, g);
                        for (int k = 0; k < 4; k++) out[(row + k) * m + r] = g[k];
                    }
                    for (; row < r1; row++) out[row * m + r] = dot_f32(rb0buf, x + row * n, n);
                    r += 1;
                }
            }
        }
    }
    free(rb0buf);
    free(rb1buf);
}

/* QMat::matmul (src/qmat.rs:169-272): split by input rows while X fits the 6 MiB budget,
 * else by output rows; below PAR_MAC_MIN (2^18 MACs) or with < 2 rows it runs serially. */
enum { PAR_MAC_MIN = 1 << 18 };
#define MATMUL_X_L3_BUDGET (6u * 1024u * 1024u)

static uint64_t workers_for(uint64_t work, uint64_t rows) {
    if (work < PAR_MAC_MIN || rows < 2) return 1;
    uint64_t t = (uint64_t)requested_threads();
    return t < rows ? t : rows;
}

typedef struct {
    uint32_t t;
    const uint8_t* w;
    uint64_t m, n, rows, chunk, rbytes;
    const float* x;
    float* out;
} mm_ctx;

static void job_in_rows(void* p, uint64_t ji) {
    mm_ctx* c = p;
    uint64_t row0 = ji * c->chunk;
    uint64_t rc = c->chunk < c->rows - row0 ? c->chunk : c->rows - row0;
    matmul_reuse(c->w, c->m, c->n, c->x + row0 * c->n, rc, c->t, c->out + row0 * c->m);
}

static void job_out_rows(void* p, uint64_t ci) {
    mm_ctx* c = p;
    uint64_t col0 = ci * c->chunk;
    uint64_t mc = c->chunk < c->m - col0 ? c->chunk : c->m - col0;
    float* part = malloc(c->rows * mc * sizeof(float));
    matmul_reuse(c->w + col0 * c->rbytes, mc, c->n, c->x, c->rows, c->t, part);
    for (uint64_t r = 0; r < c->rows; r++) memcpy(c->out + r * c->m + col0, part + r * mc, mc * sizeof(float));
    free(part);
}

EXPORT void orc_qmat_matmul(uint32_t t, const uint8_t* w, uint64_t m, uint64_t n, const float* x, uint64_t rows,
                            float* out) {
    mm_ctx c = {.t = t, .w = w, .m = m, .n = n, .rows = rows, .x = x, .out = out};
    int bv, bb;
    dq_fn fn;
    quant_geom(t, &bv, &bb, &fn);
    c.rbytes = n / (uint64_t)bv * (uint64_t)bb;
    if (rows * n * 4 > MATMUL_X_L3_BUDGET) {
        uint64_t th = workers_for(rows * m * n, m);
        if (th <= 1) { matmul_reuse(w, m, n, x, rows, t, out); return; }
        c.chunk = (m + th - 1) / th;
        parallel_for((m + c.chunk - 1) / c.chunk, job_out_rows, &c);
        return;
    }
    uint64_t th = workers_for(rows * m * n, rows);
    if (th <= 1) { matmul_reuse(w, m, n, x, rows, t, out); return; }
    c.chunk = (rows + th - 1) / th;
    parallel_for((rows + c.chunk - 1) / c.chunk, job_in_rows, &c);
}

/* swiglu_batch (src/forward.rs:152-182): chunked over the pool above 2<<14 elements. */
typedef struct {
    const float* g;
    const float* u;
    float* o;
    uint64_t n, chunk;
} sw_ctx;

static void job_swiglu(void* p, uint64_t j) {
    sw_ctx* c = p;
    uint64_t lo = j * c->chunk, hi = (j + 1) * c->chunk;
    if (lo > c->n) lo = c->n;
    if (hi > c->n) hi = c->n;
    for (uint64_t i = lo; i < hi; i++) c->o[i] = orc_silu(c->g[i]) * c->u[i];
}

static void swiglu_batch(const float* g, const float* u, float* o, uint64_t n) {
    uint64_t th4 = (uint64_t)requested_threads() * 4;
    uint64_t chunk = (n + th4 - 1) / th4;
    if (chunk < 1) chunk = 1;
    uint64_t jobs = (n + chunk - 1) / chunk;
    if (jobs <= 1 || n < (2u << 14)) {
        for (uint64_t i = 0; i < n; i++) o[i] = orc_silu(g[i]) * u[i];
        return;
    }
    sw_ctx c = {g, u, o, n, chunk};
    parallel_for(jobs, job_swiglu, &c);
}

typedef struct {
    const float* x;
    const float* rw;
    uint64_t H, E, k;
    int gate;
    uint32_t* ids;
    float* wts;
    uint64_t chunk, T;
} rt_ctx;

static void job_route(void* p, uint64_t j) {
    rt_ctx* c = p;
    float* logits = malloc(c->E * sizeof(float));
    uint64_t t1 = (j + 1) * c->chunk < c->T ? (j + 1) * c->chunk : c->T;
    for (uint64_t t = j * c->chunk; t < t1; t++) {
        orc_matvec(c->rw, c->E, c->H, c->x + t * c->H, logits);
        orc_route(logits, c->E, c->gate, c->k, c->ids + t * c->k, c->wts + t * c->k);
    }
    free(logits);
}

/*
 * The pooled baseline for one MoE layer over T tokens: router matvec + route per token
 * (tokens split over the pool), then for every expert with >= 1 routed row: gather its rows,
 * QMat::matmul gate and up, pooled SwiGLU, QMat::matmul down, and the weighted accumulate
 * out[t] += w * y in each token's chosen order (moe.rs:373-380).  Requires k <= 64.
 */
EXPORT void orc_moe_layer_pooled(const float* x, uint64_t T, uint64_t H, uint64_t I, uint64_t E, uint64_t k,
                                 int gate, const float* router_w, uint32_t gt, const uint8_t* gd, uint32_t ut,
                                 const uint8_t* ud, uint32_t dt, const uint8_t* dd, float* out) {
    uint32_t* ids = malloc(T * k * sizeof(uint32_t));
    float* wts = malloc(T * k * sizeof(float));
    rt_ctx rc = {x, router_w, H, E, k, gate, ids, wts, 0, T};
    uint64_t th = (uint64_t)requested_threads();
    rc.chunk = (T + th - 1) / th;
    if (rc.chunk < 1) rc.chunk = 1;
    parallel_for((T + rc.chunk - 1) / rc.chunk, job_route, &rc);

    uint64_t* cnt = calloc(E + 1, sizeof(uint64_t));
    for (uint64_t i = 0; i < T * k; i++) cnt[ids[i] + 1]++;
    for (uint64_t e = 0; e < E; e++) cnt[e + 1] += cnt[e];
    uint64_t* pos = malloc(T * k * sizeof(uint64_t)); /* (token*k + slot) per expert-sorted row */
    uint64_t* fill = calloc(E, sizeof(uint64_t));
    for (uint64_t i = 0; i < T * k; i++) pos[cnt[ids[i]] + fill[ids[i]]++] = i;

    uint64_t maxr = 0;
    for (uint64_t e = 0; e < E; e++) if (cnt[e + 1] - cnt[e] > maxr) maxr = cnt[e + 1] - cnt[e];
    float* xe = malloc((maxr ? maxr : 1) * H * sizeof(float));
    float* ge = malloc((maxr ? maxr : 1) * I * sizeof(float));
    float* ue = malloc((maxr ? maxr : 1) * I * sizeof(float));
    float* he = malloc((maxr ? maxr : 1) * I * sizeof(float));
    float* ye = malloc((maxr ? maxr : 1) * H * sizeof(float));
    float* yall = malloc(T * k * H * sizeof(float));
    uint64_t rbg = row_bytes_of(gt, H), rbu = row_bytes_of(ut, H), rbd = row_bytes_of(dt, I);
    for (uint64_t e = 0; e < E; e++) {
        uint64_t r0 = cnt[e], nr = cnt[e + 1] - cnt[e];
        if (!nr) continue;
        for (uint64_t r = 0; r < nr; r++) memcpy(xe + r * H, x + (pos[r0 + r] / k) * H, H * sizeof(float));
        orc_qmat_matmul(gt, gd + e * I * rbg, I, H, xe, nr, ge);
        orc_qmat_matmul(ut, ud + e * I * rbu, I, H, xe, nr, ue);
        swiglu_batch(ge, ue, he, nr * I);
        orc_qmat_matmul(dt, dd + e * H * rbd, H, I, he, nr, ye);
        for (uint64_t r = 0; r < nr; r++) memcpy(yall + pos[r0 + r] * H, ye + r * H, H * sizeof(float));
    }
    for (uint64_t t = 0; t < T; t++) {
        float* o = out + t * H;
        for (uint64_t i = 0; i < H; i++) o[i] = 0.0f;
        for (uint64_t j = 0; j < k; j++) {
            const float* y = yall + (t * k + j) * H;
            float w = wts[t * k + j];
            for (uint64_t i = 0; i < H; i++) o[i] += w * y[i];
        }
    }
    free(ids); free(wts); free(cnt); free(pos); free(fill);
    free(xe); free(ge); free(ue); free(he); free(ye); free(yall);
}
