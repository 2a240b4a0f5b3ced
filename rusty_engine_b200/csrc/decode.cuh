// decode.cuh -- raw GGUF weight stages in shared memory and their decoders to fp16 operands,
// shared by the tensor-core (grouped_tc.cu) and small-batch (grouped_small.cu) kernels.
#pragma once
#include "common.cuh"

namespace rmoe {

// Raw-stage geometry per type: RK K-elements per stage; PITCH = bytes per row of the main-plane
// box (what each row needs, plus 16 B where that keeps the pitch an odd number of 16-B units so
// 16-B loads of 8 consecutive rows hit distinct banks); DBLK = block scales per row per stage
// ([block][row] plane); AUX = Q5_0 high-bit words ([block][row] plane).
template <int TYPE> struct Raw;
template <> struct Raw<T_Q4_K> { static constexpr int RK = 128, PITCH = 80, MB = 80, DBLK = 0, AUX = 0; };
template <> struct Raw<T_Q5_K> { static constexpr int RK = 256, PITCH = 176, MB = 176, DBLK = 0, AUX = 0; };
template <> struct Raw<T_Q6_K> { static constexpr int RK = 256, PITCH = 208, MB = 208, DBLK = 1, AUX = 0; };
template <> struct Raw<T_Q4_0> { static constexpr int RK = 256, PITCH = 144, MB = 128, DBLK = 8, AUX = 0; };
template <> struct Raw<T_Q5_0> { static constexpr int RK = 256, PITCH = 144, MB = 128, DBLK = 8, AUX = 8; };
template <> struct Raw<T_Q8_0> { static constexpr int RK = 256, PITCH = 272, MB = 256, DBLK = 8, AUX = 0; };
template <> struct Raw<T_DENSE> { static constexpr int RK = 128, PITCH = 272, MB = 256, DBLK = 0, AUX = 0; };

// One raw stage of ROWS weight rows of one matrix in shared memory: [ROWS][PITCH] main bytes,
// then the [DBLK][ROWS] block scales, then the [AUX][ROWS] high-bit words.
template <int TYPE, int ROWS>
struct RawStage {
    using R = Raw<TYPE>;
    static constexpr int MAIN = ROWS * R::PITCH;
    static constexpr int DOFF = MAIN, DBYTES = R::DBLK * ROWS * 2;
    static constexpr int AOFF = DOFF + DBYTES, ABYTES = R::AUX * ROWS * 4;
    static constexpr int BYTES = AOFF + ABYTES;   // per matrix; every region 128-B aligned
    static_assert(MAIN % 128 == 0 && DBYTES % 128 == 0 && ABYTES % 128 == 0, "regions must be 128-B aligned");
};


// Decode K-elements [64*sub + 32*half, +32) of one weight row into 16 packed fp16 pairs (k, k+1).
// p = the row's main-plane bytes for the stage; dq / aq = its block-scale / high-bit entries
// (block b of the stage at dq + 2 ROWS b / aq + 4 ROWS b, ROWS = rows of the stage).
template <int TYPE, int ROWS>
struct Slice;
template <int TYPE, int ROWS>
__device__ __forceinline__ void slice32(const uint8_t* p, const uint8_t* dq, const uint8_t* aq, int sub, int half,
                                        uint32_t* v) {
    Slice<TYPE, ROWS>::run(p, dq, aq, sub, half, v);
}

// Packed-half helpers: a 4- or 6-bit code c placed in the low mantissa bits of 0x6400 is the
// exact fp16 value 1024 + c, so code -> fp16 costs one byte permute and one logic op per pair.
__device__ __forceinline__ __half2 as_h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }
__device__ __forceinline__ uint32_t as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t lop_or3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xFE;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));  // a | b | c
    return r;
}

// Q4_K, device layout: a stage row is one half-superblock (128 elements): four (fp16 d*sc,
// fp16 -(dmin*m)) pairs, then 64 quant bytes (the low nibbles of bytes 32 g .. 32 g + 31 are
// sub-block 2 g, the high nibbles 2 g + 1).  y = d*sc*q - dmin*m for sub-block 2*sub + half:
// the two codes of a pair land in 1024 + q (exact), 1024 is subtracted exactly and one fused
// multiply-add by the fp16 scale and min gives the value (scale, min and result each round once
// to fp16; the f32 path rounds the result only, well inside the layer tolerance).
template <int ROWS>
struct Slice<T_Q4_K, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
                                               uint32_t* v) {
        const uint32_t dm = *reinterpret_cast<const uint32_t*>(p + 4 * (2 * sub + half));
        const __half2 D = as_h2(__byte_perm(dm, 0, 0x1010)), M = as_h2(__byte_perm(dm, 0, 0x3232));
        const __half2 K = __float2half2_rn(1024.0f);
        const uint4* q = reinterpret_cast<const uint4*>(p + 16 + sub * 32);
        const uint4 a = q[0], b = q[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const int sh = 4 * half;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t p01 = __byte_perm(w[i], 0, 0x4140), p23 = __byte_perm(w[i], 0, 0x4342);
            v[2 * i] = as_u32(__hfma2(__hsub2(as_h2(((p01 >> sh) & 0x000F000Fu) | 0x64006400u), K), D, M));
            v[2 * i + 1] = as_u32(__hfma2(__hsub2(as_h2(((p23 >> sh) & 0x000F000Fu) | 0x64006400u), K), D, M));
        }
    }
};

template <int ROWS>
struct Slice<T_Q5_K, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(p);
        const float d = h2f((uint16_t)(dd & 0xFFFF)), dmin = h2f((uint16_t)(dd >> 16));
        int sc, mn;
        scale_min_k4(2 * sub + half, p + 4, sc, mn);
        const float d1 = __fmul_rn(d, (float)sc), dm1 = __fmul_rn(dmin, (float)mn);
        const uint4* q = reinterpret_cast<const uint4*>(p + 48 + sub * 32);
        const uint4* hq = reinterpret_cast<const uint4*>(p + 16);
        const uint4 a = q[0], b = q[1], ha = hq[0], hb = hq[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
        const int sh = 4 * half, ub = 2 * sub + half;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            auto val = [&](int byte) {
                float qv = (float)(((w[i] >> (8 * byte + sh)) & 0xFu) + (((hw[i] >> (8 * byte + ub)) & 1u) << 4));
                return __fsub_rn(__fmul_rn(d1, qv), dm1);
            };
            v[2 * i] = pack_f16x2(val(0), val(1));
            v[2 * i + 1] = pack_f16x2(val(2), val(3));
        }
    }
};

// Q6_K main plane row: ql[128] | qh[64] | scales[16]; d from the block-scale plane.  Slice
// `sub` covers quadrants 2*(sub&1) and 2*(sub&1)+1 of the 128-element half sub>>1; `half`
// picks one: its low bits are the low (sub even) or high (sub odd) nibbles of ql[0..31]
// (half 0) or ql[32..63] (half 1) of that half, its two high bits sit at bits 2*quadrant of qh.
template <int ROWS>
struct Slice<T_Q6_K, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
        const float q6d = h2f(*reinterpret_cast<const uint16_t*>(dq));
        const int h = sub >> 1, odd = sub & 1, qd = 2 * odd + half;
        const uint4* ql = reinterpret_cast<const uint4*>(p + h * 64 + half * 32);
        const uint4* qh = reinterpret_cast<const uint4*>(p + 128 + h * 32);
        const uint4 l0 = ql[0], l1 = ql[1], h0 = qh[0], h1 = qh[1];
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192 + h * 8);
        const int nsh = 4 * odd;
        // scales rounded once to fp16; (q6 - 32) is exact in fp16 (1024 + q6 - 1056)
        const __half2 s0 = __float2half2_rn(__fmul_rn(q6d, (float)sc[qd * 2]));
        const __half2 s1 = __float2half2_rn(__fmul_rn(q6d, (float)sc[qd * 2 + 1]));
        const __half2 K = __float2half2_rn(1056.0f);
#pragma unroll
        for (int i = 0; i < 8; i++) {  // l = 4i .. 4i+3
            const __half2 s = (i < 4) ? s0 : s1;
#pragma unroll
            for (int pr = 0; pr < 2; pr++) {  // byte pairs (0,1) and (2,3)
                const uint32_t sel = pr ? 0x4342 : 0x4140;
                const uint32_t pl = __byte_perm(lw[i], 0, sel), ph = __byte_perm(hw[i], 0, sel);
                // the quadrant's two high bits (2*qd, 2*qd+1) moved to bits 4..5
                const uint32_t hb = qd <= 2 ? (ph << (4 - 2 * qd)) : (ph >> 2);
                const uint32_t c = lop_or3((pl >> nsh) & 0x000F000Fu, hb & 0x00300030u, 0x64006400u);
                v[2 * i + pr] = as_u32(__hmul2(__hsub2(as_h2(c), K), s));
            }
        }
    }
};

// Q6_K for the tensor-core down product, in the K-permuted operand order: inside every group of
// four K positions the stored order is (k, k+2, k+1, k+3) (kperm_pos), so a packed pair is bytes
// 0 and 2 (or 1 and 3) of one quant word and needs no byte permute (about 2.8 instructions per
// weight against 4 for slice32).  The other operand (h, or QMat's x) is stored in the same order,
// so the products are unchanged, and the decoded fp16 values are slice32's: q6 - 32 is formed
// exactly, either as (1024 + q6) - 1056 or as (1024 + 16 q6) / 16 - 96, then rounded once by the
// scale product.
template <int ROWS>
__device__ __forceinline__ void slice32_q6k_kperm(const uint8_t* p, const uint8_t* dq, int sub, int half,
                                                  uint32_t* v) {
    const float q6d = h2f(*reinterpret_cast<const uint16_t*>(dq));
    const int h = sub >> 1, odd = sub & 1, qd = 2 * odd + half;
    const uint4* ql = reinterpret_cast<const uint4*>(p + h * 64 + half * 32);
    const uint4* qh = reinterpret_cast<const uint4*>(p + 128 + h * 32);
    const uint4 l0 = ql[0], l1 = ql[1], h0 = qh[0], h1 = qh[1];
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192 + h * 8);
    const __half2 s0 = __float2half2_rn(__fmul_rn(q6d, (float)sc[qd * 2]));
    const __half2 s1 = __float2half2_rn(__fmul_rn(q6d, (float)sc[qd * 2 + 1]));
    const __half2 K1056 = __float2half2_rn(1056.0f), S16 = __float2half2_rn(0.0625f),
                  M96 = __float2half2_rn(-96.0f);
    const uint32_t C = 0x64006400u;
    // the quadrant's two high bits (at 2 qd of each qh byte) go to mantissa bit 4 (pair 0, 2 of a
    // low-nibble quadrant) or 8 (every other pair): a left shift by 4 - 2 half for pair (0, 2),
    // a right shift by 2 qd for pair (1, 3)
    const int hl = 4 - 2 * half, hr = 2 * qd;
    const int lsh = odd ? 8 : 4;  // pair (1, 3): the byte's nibble to mantissa bits 4..7
#pragma unroll
    for (int i = 0; i < 8; i++) {  // l = 4i .. 4i+3
        const __half2 s = (i < 4) ? s0 : s1;
        const uint32_t L = lw[i], Hh = hw[i];
        __half2 y02;
        if (!odd) {
            const uint32_t c = lop_or3(L & 0x000F000Fu, (Hh << hl) & 0x00300030u, C);
            y02 = __hsub2(as_h2(c), K1056);
        } else {
            const uint32_t c = lop_or3(L & 0x00F000F0u, (Hh << hl) & 0x03000300u, C);
            y02 = __hfma2(as_h2(c), S16, M96);
        }
        const uint32_t c13 = lop_or3((L >> lsh) & 0x00F000F0u, (Hh >> hr) & 0x03000300u, C);
        const __half2 y13 = __hfma2(as_h2(c13), S16, M96);
        v[2 * i] = as_u32(__hmul2(y02, s));
        v[2 * i + 1] = as_u32(__hmul2(y13, s));
    }
}

// Q4_0 main plane row: qs[8 x 16]; half = block 2*sub + half (low nibbles -> elements 0..15,
// high nibbles -> 16..31).
template <int ROWS>
struct Slice<T_Q4_0, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
        const int b = 2 * sub + half;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 2 * ROWS * b));
        const uint4 q = *reinterpret_cast<const uint4*>(p + 16 * b);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            auto lo = [&](int byte) { return __fmul_rn((float)((int)((w[i] >> (8 * byte)) & 0xFu) - 8), d); };
            auto hi = [&](int byte) { return __fmul_rn((float)((int)((w[i] >> (8 * byte + 4)) & 0xFu) - 8), d); };
            v[2 * i] = pack_f16x2(lo(0), lo(1));
            v[2 * i + 1] = pack_f16x2(lo(2), lo(3));
            v[8 + 2 * i] = pack_f16x2(hi(0), hi(1));
            v[8 + 2 * i + 1] = pack_f16x2(hi(2), hi(3));
        }
    }
};

// Q5_0 main plane row: qs[8 x 16]; high bits and scales from their planes.
template <int ROWS>
struct Slice<T_Q5_0, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t* dq, const uint8_t* aq, int sub,
                                                int half, uint32_t* v) {
        const int b = 2 * sub + half;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 2 * ROWS * b));
        const uint32_t qh = *reinterpret_cast<const uint32_t*>(aq + 4 * ROWS * b);
        const uint4 q = *reinterpret_cast<const uint4*>(p + 16 * b);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            auto lo = [&](int byte) {
                int j = 4 * i + byte;
                int x = (int)(((w[i] >> (8 * byte)) & 0xFu) | (((qh >> j) & 1u) << 4)) - 16;
                return __fmul_rn((float)x, d);
            };
            auto hi = [&](int byte) {
                int j = 4 * i + byte;
                int x = (int)(((w[i] >> (8 * byte + 4)) & 0xFu) | (((qh >> (j + 16)) & 1u) << 4)) - 16;
                return __fmul_rn((float)x, d);
            };
            v[2 * i] = pack_f16x2(lo(0), lo(1));
            v[2 * i + 1] = pack_f16x2(lo(2), lo(3));
            v[8 + 2 * i] = pack_f16x2(hi(0), hi(1));
            v[8 + 2 * i + 1] = pack_f16x2(hi(2), hi(3));
        }
    }
};

// Q8_0 main plane row: qs[8 x 32]; half = block 2*sub + half.
template <int ROWS>
struct Slice<T_Q8_0, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
        const int b = 2 * sub + half;
        const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 2 * ROWS * b));
        const uint4* q = reinterpret_cast<const uint4*>(p + 32 * b);
        const uint4 a = q[0], c = q[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {  // word i holds elements 4i..4i+3 of the block
            auto val = [&](int byte) { return __fmul_rn((float)(int8_t)((w[i] >> (8 * byte)) & 0xFFu), d); };
            v[2 * i] = pack_f16x2(val(0), val(1));
            v[2 * i + 1] = pack_f16x2(val(2), val(3));
        }
    }
};

template <int ROWS>
struct Slice<T_DENSE, ROWS> {
    static __device__ __forceinline__ void run(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
                                                 uint32_t* v) {
        const uint4* q = reinterpret_cast<const uint4*>(p + 128 * sub + 64 * half);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 a = q[i];
            v[4 * i] = a.x;
            v[4 * i + 1] = a.y;
            v[4 * i + 2] = a.z;
            v[4 * i + 3] = a.w;
        }
    }
};


}  // namespace rmoe
