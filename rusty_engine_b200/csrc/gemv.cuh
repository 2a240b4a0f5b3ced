// gemv.cuh -- the decode-size grouped expert products (Q4_K / Q6_K, dequantisation in the
// registers that feed mma.sync): fragment geometry per GGUF type and the per-tile body
// gv_tile, shared by the kernels of grouped_gemv.cu and the one-launch small-batch layer.
//
// At decode batch sizes a layer streams every touched expert's weights once, and what stands
// between the kernel and HBM speed is the issue budget for unpacking them (Q4_K arrives at
// about 40 weights per SM clock), not the tensor cores.  So no decoded weight tile is written
// anywhere:
//   * the K axis of every mma.m16n8k16 is permuted per GGUF type so that a thread's A-fragment
//     registers are exactly the fp16 pairs its own quant bytes give under the 0x6400
//     magic-number unpack, with no byte shuffles: pairs (k, k+2) and (k+1, k+3) of a 4-aligned
//     group of one sub-block.  The B operand (the tile's token rows) is staged once per CTA in
//     the same permuted order, so every product is unchanged and only the order of the f32
//     sums differs;
//   * each thread streams only its own quant bytes, through a private cp.async ring in shared
//     memory, so the K loop has no CTA barrier;
//   * a CTA is 8 warps = RG row groups (16 weight rows each; gate/up take the same 16 rows of
//     both matrices) x KS K-slices (interleaved 128-element units), the slices summed through
//     shared memory in a fixed order.
// Decoded weights are bit-identical to the other kernels' (the same fp16 roundings).
//
//   gate/up: h[row, f] = silu(gate_f . x) * (up_f . x)      (src/moe.rs:280-299), stored as fp16
//            x 2^e with e per (row, 16-feature block); the row's largest e goes to rowexp[row]
//   down:    y = down . h[row], every h block brought to the row's exponent while it is staged;
//            out[tok] += w_slot * y * 2^rowexp                  (src/moe.rs:373-380)
#pragma once
#include "common.cuh"
#include "decode.cuh"
#include "kernels.h"

namespace rmoe {

static constexpr int GV_THREADS = 256;          // 8 warps
static constexpr int GV_UK = 128;               // K elements per unit (32 per quad lane)
static constexpr int GV_SMEM_TWO = 113 * 1024;  // shared memory that keeps two CTAs per SM

__device__ __forceinline__ void gv_cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void gv_cp8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void gv_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void gv_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// wait until at most n (1..3) of this thread's groups are still in flight
__device__ __forceinline__ void gv_wait_dyn(int n) {
    if (n >= 3) gv_wait<3>();
    else if (n == 2) gv_wait<2>();
    else gv_wait<1>();
}

// ---------------------------------------------------------------------------------------------
// Per-type fragment geometry.  A unit is 128 consecutive K elements of one weight row; the lane
// at quad position c (lane & 3) owns 32 of them, eight k16 steps of two pairs.  k0(c, s) is the
// first K element (inside the unit) of step s for that lane: its A pairs are (k0, k0+2) and
// (k0+1, k0+3).  N16 / N8: 16-B / 8-B ring pieces per (matrix, row) per unit.
// ---------------------------------------------------------------------------------------------
template <int TYPE>
struct Gv;

// Q4_K half-superblock (80 B: four (fp16 d*sc, fp16 -dmin*m) pairs, 64 quant bytes whose low
// nibbles at 32 g + b are element 64 g + b and high nibbles element 64 g + 32 + b).  Lane c
// takes quant bytes 16 c .. 16 c + 15 (group g = c >> 1, bytes b = 16 (c & 1) ..) and the two
// scale pairs of sub-blocks 2 g, 2 g + 1.  Word i gives step 2 i (low nibbles) and step 2 i + 1
// (high nibbles).
template <>
struct Gv<T_Q4_K> {
    static constexpr int N16 = 1, N8 = 1;
    static constexpr bool DPL = false;
    __device__ static int k0(int c, int s) { return 32 * (2 * (c >> 1) + (s & 1)) + 16 * (c & 1) + 4 * (s >> 1); }
    // inverse: the (lane c, step s) whose group starts at kk (4-aligned, inside the unit)
    __device__ static void inv(int kk, int& c, int& s) {
        c = ((kk >> 6) << 1) | ((kk >> 4) & 1);
        s = (((kk >> 2) & 3) << 1) | ((kk >> 5) & 1);
    }
    // byte offset of unit u in a main-plane row, and of lane c's pieces inside the unit
    __device__ static int unit_base(int u) { return u * 80; }
    __device__ static int off16(int, int c, int) { return 16 + 16 * c; }
    __device__ static int off8(int, int c, int) { return 8 * (c >> 1); }
    // y = d*sc*q - dmin*m: q lands in 1024 + q (low nibble) or 1024 + 16 q (high nibble), both
    // exact; 1024 is taken off / the 16 divided out exactly, then one fma with the fp16 pair.
    template <int R>
    __device__ static void decode(const uint4* q16, const uint2* q8, int, uint16_t, uint32_t (&a)[8][4]) {
        const uint4 q = q16[0];
        const uint2 dm = q8[0];
        // the scale pairs splatted as half2: half selections the fma takes as operand forms (no
        // separate byte permutes; one ALU instruction per MMA fewer at 64 tokens)
        const __half2 Dl = __low2half2(as_h2(dm.x)), Ml = __high2half2(as_h2(dm.x));
        const __half2 Dh = __low2half2(as_h2(dm.y)), Mh = __high2half2(as_h2(dm.y));
        const __half2 K1024 = __float2half2_rn(1024.0f), S16 = __float2half2_rn(0.0625f),
                      M64 = __float2half2_rn(-64.0f);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t v = w[i], v8 = v >> 8;
            const __half2 l02 = __hsub2(as_h2((v & 0x000F000Fu) | 0x64006400u), K1024);
            const __half2 l13 = __hsub2(as_h2((v8 & 0x000F000Fu) | 0x64006400u), K1024);
            const __half2 h02 = __hfma2(as_h2((v & 0x00F000F0u) | 0x64006400u), S16, M64);
            const __half2 h13 = __hfma2(as_h2((v8 & 0x00F000F0u) | 0x64006400u), S16, M64);
            a[2 * i][R] = as_u32(__hfma2(l02, Dl, Ml));
            a[2 * i][2 + R] = as_u32(__hfma2(l13, Dl, Ml));
            a[2 * i + 1][R] = as_u32(__hfma2(h02, Dh, Mh));
            a[2 * i + 1][2 + R] = as_u32(__hfma2(h13, Dh, Mh));
        }
    }
};

// Q6_K, unit = one 128-element half n of a superblock (ql[64 n ..] | qh[32 n ..] | scales[8 n ..]
// in the 208-B main-plane entry, d from the d plane).  Element l + 32 q of the half (quadrant q)
// has its low four bits in ql[64 n + l] (q = 0, 2: low / high nibble) or ql[64 n + 32 + l] (q = 1,
// 3) and its two high bits at bits 2 q of qh[32 n + l]; its scale is scales[8 n + l / 16 + 2 q].
// Lane c takes l = 8 c .. 8 c + 7 of every quadrant; step s = 4 w + q covers l = 8 c + 4 w ...
template <>
struct Gv<T_Q6_K> {
    static constexpr int N16 = 0, N8 = 4;
    static constexpr bool DPL = true;
    __device__ static int k0(int c, int s) { return 32 * (s & 3) + 8 * c + 4 * (s >> 2); }
    __device__ static void inv(int kk, int& c, int& s) {
        c = (kk >> 3) & 3;
        s = (kk >> 5) | (((kk >> 2) & 1) << 2);
    }
    __device__ static int unit_base(int u) { return (u >> 1) * 208; }
    __device__ static int off16(int, int, int) { return 0; }
    __device__ static int off8(int u, int c, int j) {
        const int n = u & 1;
        return j == 0 ? 64 * n + 8 * c : j == 1 ? 64 * n + 32 + 8 * c : j == 2 ? 128 + 32 * n + 8 * c : 192 + 8 * n;
    }
    // q6 lands in 1024 + q6 (low bits at mantissa 0..3, high at 4..5) or 1024 + 16 q6 (4..7 and
    // 8..9), whichever needs fewer shifts for that quadrant and byte pair; q6 - 32 is recovered
    // exactly and multiplied by the scale d * sc (rounded once to fp16, as the other kernels).
    template <int R>
    __device__ static void decode(const uint4*, const uint2* q8, int c, uint16_t dbits, uint32_t (&a)[8][4]) {
        const uint2 A8 = q8[0], B8 = q8[1], H8 = q8[2], S8 = q8[3];
        const __half2 d2 = __half2half2(__ushort_as_half(dbits));
        const int sh = 8 * (c >> 1);
        // bytes 0 and 2 of sx: the int8 scales of quadrants 0, 1; of sy: quadrants 2, 3
        const uint32_t sx = S8.x >> sh, sy = S8.y >> sh;
        const __half2 K1152 = __float2half2_rn(1152.0f);
        const __half2 s01 = __hmul2(__hsub2(as_h2(((sx ^ 0x00800080u) & 0x00FF00FFu) | 0x64006400u), K1152), d2);
        const __half2 s23 = __hmul2(__hsub2(as_h2(((sy ^ 0x00800080u) & 0x00FF00FFu) | 0x64006400u), K1152), d2);
        const __half2 sq[4] = {__low2half2(s01), __high2half2(s01), __low2half2(s23), __high2half2(s23)};
        const __half2 K1056 = __float2half2_rn(1056.0f), S16 = __float2half2_rn(0.0625f),
                      M96 = __float2half2_rn(-96.0f);
        const uint32_t C = 0x64006400u;
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t A = w ? A8.y : A8.x, B = w ? B8.y : B8.x, H = w ? H8.y : H8.x;
            // byte pair (0, 2): quadrants 0, 1 at mantissa 0..5, quadrants 2, 3 at 4..9
            const __half2 q0a = __hsub2(as_h2((A & 0x000F000Fu) | ((H << 4) & 0x00300030u) | C), K1056);
            const __half2 q1a = __hsub2(as_h2((B & 0x000F000Fu) | ((H << 2) & 0x00300030u) | C), K1056);
            const __half2 q2a = __hfma2(as_h2((A & 0x00F000F0u) | ((H << 4) & 0x03000300u) | C), S16, M96);
            const __half2 q3a = __hfma2(as_h2((B & 0x00F000F0u) | ((H << 2) & 0x03000300u) | C), S16, M96);
            // byte pair (1, 3): every quadrant at mantissa 4..9
            const __half2 q0b = __hfma2(as_h2(((A >> 4) & 0x00F000F0u) | (H & 0x03000300u) | C), S16, M96);
            const __half2 q1b = __hfma2(as_h2(((B >> 4) & 0x00F000F0u) | ((H >> 2) & 0x03000300u) | C), S16, M96);
            const __half2 q2b = __hfma2(as_h2(((A >> 8) & 0x00F000F0u) | ((H >> 4) & 0x03000300u) | C), S16, M96);
            const __half2 q3b = __hfma2(as_h2(((B >> 8) & 0x00F000F0u) | ((H >> 6) & 0x03000300u) | C), S16, M96);
            a[4 * w + 0][R] = as_u32(__hmul2(q0a, sq[0]));
            a[4 * w + 0][2 + R] = as_u32(__hmul2(q0b, sq[0]));
            a[4 * w + 1][R] = as_u32(__hmul2(q1a, sq[1]));
            a[4 * w + 1][2 + R] = as_u32(__hmul2(q1b, sq[1]));
            a[4 * w + 2][R] = as_u32(__hmul2(q2a, sq[2]));
            a[4 * w + 2][2 + R] = as_u32(__hmul2(q2b, sq[2]));
            a[4 * w + 3][R] = as_u32(__hmul2(q3a, sq[3]));
            a[4 * w + 3][2 + R] = as_u32(__hmul2(q3b, sq[3]));
        }
    }
};

template <int TYPE, int NT, int NMAT, int KS>
struct GvGeom {
    using D = Gv<TYPE>;
    static constexpr int RG = 8 / KS, RB = 16 * RG, NTT = NT / 8;
    static constexpr int P16 = NMAT * 2 * D::N16, P8 = NMAT * 2 * D::N8;  // ring pieces per lane per unit
    static constexpr int OFF8 = GV_THREADS * 16 * P16;
    static constexpr int SLOT = OFF8 + GV_THREADS * 8 * P8;  // bytes per ring slot
    static constexpr int PER = NMAT * NTT * 4;                // accumulators per lane
    static_assert(KS == 1 || KS == 2 || KS == 4 || KS == 8, "K slices");
    static_assert((KS - 1) * RG * 32 * PER * 4 <= 2 * SLOT, "slice reduction fits in two ring slots");
};

// four fp16 values times 2^d (d <= 0), in f32, rounded back to fp16
__device__ __forceinline__ uint2 gv_scale4(uint2 v, int d) {
    if (d == 0) return v;
    if (d < -40) return make_uint2(0, 0);
    const float s = exp2i(d);
    const float2 a = __half22float2(as_h2(v.x)), b = __half22float2(as_h2(v.y));
    return make_uint2(pack_f16x2(__fmul_rn(a.x, s), __fmul_rn(a.y, s)), pack_f16x2(__fmul_rn(b.x, s), __fmul_rn(b.y, s)));
}

// One (tile, RB-row block) of the decode products: expert e's rows row0 .. row0 + nrows - 1 of
// the expert-sorted order against weight rows rblk * RB .. of its stack.  The body of
// gv_kernel, also run item by item by the one-launch small-batch layer (layer_small.cu), where
// the dispatch tables (p.row_tok, p.row_slot, p.topk_w) are in shared memory and h, hexp,
// rowexp and xb were written earlier in the same kernel: those are read through L2 (ld.cg),
// the tables with generic loads.  PDL: gv_kernel's launch-order waits.
template <int TYPE, int NT, int NMAT, int KS, bool PDL>
__device__ __forceinline__ void gv_tile(const GroupedParams& p, int e, int row0, int nrows, int rblk, int depth,
                                        int ring_off, uint8_t* smem) {
    using D = Gv<TYPE>;
    using G = GvGeom<TYPE, NT, NMAT, KS>;
    constexpr int RG = G::RG, RB = G::RB, NTT = G::NTT;
    __shared__ int s_tok[NT], s_rexp[NT];
    __shared__ float s_w[NT];
    const bool sh = e >= p.E;
    const DevMat& M0 = NMAT == 2 ? (sh ? p.sgate : p.gate) : (sh ? p.sdown : p.down);
    const DevMat& M1 = NMAT == 2 ? (sh ? p.sup : p.up) : M0;
    const int K = NMAT == 2 ? p.H : p.I;
    const int NU = K / GV_UK;
    const uint64_t grow0 = (uint64_t)(sh ? 0 : e) * M0.rows + (uint64_t)rblk * RB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rg = warp % RG, kq = warp / RG;
    const int g = lane >> 2, c = lane & 3;

    for (int n = tid; n < NT; n += GV_THREADS) {
        int tok = 0;
        float w = 0.0f;
        if (n < nrows) {
            const int r = row0 + n;
            tok = p.row_tok[r];
            if (NMAT == 1) {
                const int slot = p.row_slot[r];
                w = slot < p.k ? p.topk_w[(size_t)tok * p.k + slot] : 1.0f;
            }
        }
        s_tok[n] = tok;
        s_w[n] = w;
    }

    const uint32_t ring = smem_u32(smem) + ring_off;
    const int nmine = (NU - kq + KS - 1) / KS;
    // this lane's weight rows (matrix m, row g + 8 r of its group) and ring slot addresses
    const uint8_t* rowp[NMAT][2];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const DevMat& M = m ? M1 : M0;
            rowp[m][r] = M.main + (grow0 + 16 * rg + g + 8 * r) * M.main_stride;
        }
    int slot_in = 0;  // ring slot the next issued unit goes to
    auto issue = [&](int i) {
        if (i < nmine) {
            const int u = kq + i * KS;
            const uint32_t sl = ring + (uint32_t)(slot_in * G::SLOT) + tid * 16;
            const uint32_t sl8 = ring + (uint32_t)(slot_in * G::SLOT + G::OFF8) + tid * 8;
            const int ub = D::unit_base(u);
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const uint8_t* b = rowp[m][r] + ub;
#pragma unroll
                    for (int j = 0; j < D::N16; j++)
                        gv_cp16(sl + ((m * 2 + r) * D::N16 + j) * (GV_THREADS * 16), b + D::off16(u, c, j));
#pragma unroll
                    for (int j = 0; j < D::N8; j++)
                        gv_cp8(sl8 + ((m * 2 + r) * D::N8 + j) * (GV_THREADS * 8), b + D::off8(u, c, j));
                }
        }
        gv_commit();  // one group per unit (possibly empty), so the wait count stays fixed
        if (++slot_in == depth) slot_in = 0;
    };
    // the down kernel streams its first units while gate/up finishes; gate/up first sends the
    // token-row loads of its operand (below), so they do not queue behind the weight stream
    if (NMAT == 1) {
        for (int i = 0; i < depth - 1; i++) issue(i);
        if (PDL) pdl_wait();
        for (int n = tid; n < NT; n += GV_THREADS) s_rexp[n] = n < nrows ? __ldcg(p.rowexp + row0 + n) : 0;
    }
    __syncthreads();

    // token operand in fragment order: entry ((u * 8 + s) * NTT + t) * 32 + lane holds lane's
    // (b0, b1) of step s, n-tile t of unit u.  Only live token rows are staged: a dead row only
    // feeds MMA columns that are never read.
    uint2* bsm = reinterpret_cast<uint2*>(smem);
    {
        const int cpr = K / 8;  // 16-B chunks per row
        const int hstride = p.I / GV_EBLK;
        const int total = nrows * cpr;
        constexpr int SB = 4;  // loads in flight per thread
        for (int i0 = 0; i0 < total || (NMAT == 2 && i0 == 0); i0 += SB * GV_THREADS) {
            uint4 v[SB];
            int d[SB];
#pragma unroll
            for (int u = 0; u < SB; u++) {
                const int i = i0 + u * GV_THREADS + tid;
                d[u] = 0;
                if (i < total) {
                    const int n = i / cpr, j = i - n * cpr;
                    if (NMAT == 2) {
                        v[u] = __ldcg(reinterpret_cast<const uint4*>(p.xb + (size_t)s_tok[n] * K + 8 * j));
                    } else {
                        const size_t r = (size_t)(row0 + n);
                        v[u] = __ldcg(reinterpret_cast<const uint4*>(p.h + r * p.I + 8 * j));
                        d[u] = (int)__ldcg(p.hexp + r * hstride + (8 * j) / GV_EBLK);
                    }
                }
            }
            if (NMAT == 2 && i0 == 0)
                for (int i = 0; i < depth - 1; i++) issue(i);
#pragma unroll
            for (int u = 0; u < SB; u++) {
                const int i = i0 + u * GV_THREADS + tid;
                if (i >= total) continue;
                const int n = i / cpr, j = i - n * cpr;
                uint4 w = v[u];
                if (NMAT == 1) {
                    const int dd = d[u] - s_rexp[n];
                    const uint2 lo = gv_scale4(make_uint2(w.x, w.y), dd), hi = gv_scale4(make_uint2(w.z, w.w), dd);
                    w = make_uint4(lo.x, lo.y, hi.x, hi.y);
                }
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int kk = 8 * j + 4 * hf;
                    int cc, st;
                    D::inv(kk & (GV_UK - 1), cc, st);
                    const uint32_t x01 = hf ? w.z : w.x, x23 = hf ? w.w : w.y;
                    bsm[(((kk / GV_UK) * 8 + st) * NTT + (n >> 3)) * 32 + (n & 7) * 4 + cc] =
                        make_uint2(__byte_perm(x01, x23, 0x5410), __byte_perm(x01, x23, 0x7632));
                }
            }
        }
    }
    // d plane entries of the CTA's rows (Q6_K): [matrix][superblock][row]
    const uint16_t* dsm = reinterpret_cast<const uint16_t*>(smem + (size_t)NU * 8 * NTT * 32 * 8);
    if (D::DPL) {
        uint16_t* dw = const_cast<uint16_t*>(dsm);
        const int nsb = K / 256;
        for (int i = tid; i < NMAT * nsb * RB; i += GV_THREADS) {
            const int r = i % RB, rest = i / RB, sb = rest % nsb, m = rest / nsb;
            const DevMat& M = m ? M1 : M0;
            dw[i] = __ldg(reinterpret_cast<const uint16_t*>(M.dpl) + (size_t)sb * M.trows + grow0 + r);
        }
    }
    __syncthreads();

    float acc[NMAT][NTT][4];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int t = 0; t < NTT; t++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[m][t][q] = 0.0f;

    const int nsb = K / 256;
    const int ntl = (nrows + 7) >> 3;  // n-tiles holding live token rows
    int slot_out = 0;  // ring slot of unit i
    for (int i = 0; i < nmine; i++) {
        issue(i + depth - 1);
        gv_wait_dyn(depth - 1);  // this lane's unit i has landed (only this lane reads it)
        const int u = kq + i * KS;
        const uint8_t* sl = smem + ring_off + slot_out * G::SLOT;
        if (++slot_out == depth) slot_out = 0;
        const uint2* bu = bsm + (size_t)u * 8 * NTT * 32 + lane;
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            // A fragments in the register order mma.sync takes them: (row g, k pair 0), (row g + 8,
            // pair 0), (row g, pair 1), (row g + 8, pair 1) -- each decoder writes its row's two
            uint32_t afr[8][4];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                uint4 q16[D::N16 > 0 ? D::N16 : 1];
                uint2 q8[D::N8 > 0 ? D::N8 : 1];
#pragma unroll
                for (int j = 0; j < D::N16; j++)
                    q16[j] = *reinterpret_cast<const uint4*>(sl + ((m * 2 + r) * D::N16 + j) * (GV_THREADS * 16) + tid * 16);
#pragma unroll
                for (int j = 0; j < D::N8; j++)
                    q8[j] = *reinterpret_cast<const uint2*>(sl + G::OFF8 + ((m * 2 + r) * D::N8 + j) * (GV_THREADS * 8) +
                                                            tid * 8);
                const uint16_t db = D::DPL ? dsm[(m * nsb + (u >> 1)) * RB + 16 * rg + g + 8 * r] : 0;
                if (r == 0) D::template decode<0>(q16, q8, c, db, afr);
                else D::template decode<1>(q16, q8, c, db, afr);
            }
#pragma unroll
            for (int s = 0; s < 8; s++) {
                const uint32_t* a = afr[s];
#pragma unroll
                for (int t = 0; t < NTT; t++) {
                    if (NTT == 1 || t < ntl) {  // a tile always has a live first n-tile
                        const uint2 b = bu[(s * NTT + t) * 32];
                        mma_f16_16816(acc[m][t], a, b.x, b.y);
                    }
                }
            }
        }
    }

    // K slices 1.. hand their sums to slice 0 through the drained ring (added in slice order)
    gv_wait<0>();
    constexpr int PER = G::PER;
    if (KS > 1) {
        __syncthreads();
        float* red = reinterpret_cast<float*>(smem + ring_off);
        if (kq > 0)
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int t = 0; t < NTT; t++)
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        red[(((kq - 1) * RG + rg) * 32 + lane) * PER + (m * NTT + t) * 4 + q] = acc[m][t][q];
        __syncthreads();
        if (kq > 0) return;  // no CTA barrier below
        for (int j = 1; j < KS; j++)
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int t = 0; t < NTT; t++)
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        acc[m][t][q] =
                            __fadd_rn(acc[m][t][q], red[(((j - 1) * RG + rg) * 32 + lane) * PER + (m * NTT + t) * 4 + q]);
    }

    // accumulator (m, t, q): weight row 16 rg + g + 8 (q >> 1) of the CTA, token row 8 t + 2 c + (q & 1)
    const int fb = rblk * RG + rg;  // 16-row block of the output features
    const int f = fb * 16 + g;
    if (NMAT == 2) {
        const int hstride = p.I / GV_EBLK;
#pragma unroll
        for (int t = 0; t < NTT; t++) {
            float hv[4];
#pragma unroll
            for (int q = 0; q < 4; q++) hv[q] = silu_ref(acc[0][t][q]) * acc[NMAT - 1][t][q];  // src/moe.rs:280-283
            float m0 = fmaxf(fabsf(hv[0]), fabsf(hv[2])), m1 = fmaxf(fabsf(hv[1]), fabsf(hv[3]));
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
                m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int n = 8 * t + 2 * c + j;
                if (n < nrows) {
                    const int ex = block_exp(j ? m1 : m0);
                    const float sc = exp2i(-ex);
                    const size_t r = (size_t)(row0 + n);
                    p.h[r * p.I + f] = __float2half_rn(__fmul_rn(hv[j], sc));
                    p.h[r * p.I + f + 8] = __float2half_rn(__fmul_rn(hv[j + 2], sc));
                    if (g == 0) {
                        p.hexp[r * hstride + fb] = (int8_t)ex;
                        atomicMax(p.rowexp + r, ex);
                    }
                }
            }
        }
    } else {
#pragma unroll
        for (int t = 0; t < NTT; t++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int n = 8 * t + 2 * c + (q & 1);
                if (n < nrows) {
                    const int fo = f + 8 * (q >> 1);
                    const float yv = __fmul_rn(acc[0][t][q], exp2i(s_rexp[n]));
                    if (p.y) p.y[(size_t)(row0 + n) * p.H + fo] = yv;
                    else atomicAdd(p.out + (size_t)s_tok[n] * p.H + fo, __fmul_rn(s_w[n], yv));
                }
            }
    }
}


}  // namespace rmoe
