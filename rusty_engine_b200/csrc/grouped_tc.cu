// grouped_tc.cu -- tensor-core (tcgen05) grouped expert products for large batches (prefill).
//
// One CTA computes a 128-feature block of one expert for a tile of <= 128 expert-sorted rows:
//   gate/up: h[row, f] = silu(gate_f . x_row) * (up_f . x_row)   (src/moe.rs:280-299)
//   down:    out[tok] += w_slot * (down . h_row)                  (src/moe.rs:373-380)
//
// Warp roles (gate/up runs one CTA per SM, down two; everything is ordered through mbarriers):
//   warp 0      TMA producer: one 2-D tensor copy per matrix and plane brings the raw GGUF
//               bytes of the CTA's 128 weight rows for one 256-element superblock (or 8 blocks
//               of 32) into a shared ring;
//   warp 1      allocates tensor memory and issues tcgen05.mma (one elected thread): A is the
//               dequantized weight tile held in TMEM, B the token tile in shared memory;
//   warps 2-3   token tiles: one thread loads each 64-column tile of the expert-sorted x rows
//               (gate/up) or of the SwiGLU activations h (down) with a 128-B-swizzled 2-D TMA;
//               for down, warp 3 then brings each h row of the tile to its row's common scale;
//   warps 4..   one thread per weight row decodes 64 K-elements of its row per stage from the
//               raw ring (bit-identical f32 values to quant::dequant, rounded to fp16) and
//               stores them into its TMEM lane with tcgen05.st; after the last stage the same
//               warps drain the f32 accumulators from TMEM and run the epilogue.
// The fp16 weights never touch shared memory; shared memory carries the raw bytes and the
// token tiles only.  Every wait is bounded: on a timeout the kernel records DERR_TIMEOUT in the
// status word, skips the remaining work, waits for its own MMAs and frees its tensor memory.
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rmoe {
using namespace tc;

static constexpr int TC_M = 128;   // weight rows per matrix per CTA (= TMEM lanes, = TMA box rows)
static constexpr int TC_BN = 128;  // expert-sorted rows per tile (MMA N, rounded to 16 per tile)
static constexpr int TC_KS = 64;   // K elements per MMA stage (one 128-B swizzle row of fp16)
static constexpr int TC_NST = 4;   // MMA stages in flight
static constexpr int TC_RST = 2;   // raw weight stages in flight

int tc_tile_rows() { return TC_BN; }

// Raw-stage geometry per type: RK K-elements per stage; PITCH = bytes per row of the main-plane
// box (what each row needs, plus 16 B where that keeps the pitch an odd number of 16-B units so
// 16-B loads of 8 consecutive rows hit distinct banks); DBLK = block scales per row per stage
// ([block][row] plane); AUX = Q5_0 high-bit words ([block][row] plane).
template <int TYPE> struct Raw;
template <> struct Raw<T_Q4_K> { static constexpr int RK = 256, PITCH = 144, MB = 144, DBLK = 0, AUX = 0; };
template <> struct Raw<T_Q5_K> { static constexpr int RK = 256, PITCH = 176, MB = 176, DBLK = 0, AUX = 0; };
template <> struct Raw<T_Q6_K> { static constexpr int RK = 256, PITCH = 208, MB = 208, DBLK = 1, AUX = 0; };
template <> struct Raw<T_Q4_0> { static constexpr int RK = 256, PITCH = 144, MB = 128, DBLK = 8, AUX = 0; };
template <> struct Raw<T_Q5_0> { static constexpr int RK = 256, PITCH = 144, MB = 128, DBLK = 8, AUX = 8; };
template <> struct Raw<T_Q8_0> { static constexpr int RK = 256, PITCH = 272, MB = 256, DBLK = 8, AUX = 0; };
template <> struct Raw<T_DENSE> { static constexpr int RK = 128, PITCH = 272, MB = 256, DBLK = 0, AUX = 0; };

template <int TYPE>
struct RawStage {
    using R = Raw<TYPE>;
    static constexpr int MAIN = TC_M * R::PITCH;  // bytes per matrix: main box
    static constexpr int DOFF = MAIN, DBYTES = R::DBLK * TC_M * 2;
    static constexpr int AOFF = DOFF + DBYTES, ABYTES = R::AUX * TC_M * 4;
    static constexpr int BYTES = AOFF + ABYTES;   // per matrix; every region 128-B aligned
    static_assert(MAIN % 128 == 0 && DBYTES % 128 == 0 && ABYTES % 128 == 0, "TMA regions must be 128-B aligned");
};

// ---------------------------------------------------------------------------------------------
// host: tensor maps
// ---------------------------------------------------------------------------------------------
// The driver's tensor-map encoder, resolved through the runtime so the library does not link
// libcuda itself (it loads on hosts without a driver; only this call needs one).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static bool encode2d(CUtensorMap& m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                     uint64_t stride1_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {d0, d1};
    cuuint64_t strides[1] = {stride1_bytes};
    cuuint32_t box[2] = {b0, b1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int TYPE>
static bool maps_for(const DevMat& M, WMaps& o) {
    using R = Raw<TYPE>;
    // main plane as u16 [trows][main_stride / 2]; box = PITCH bytes x 128 rows (past the row end
    // the box reads zeros)
    bool ok = encode2d(o.main, CU_TENSOR_MAP_DATA_TYPE_UINT16, M.main, M.main_stride / 2, M.trows, M.main_stride,
                       R::PITCH / 2, TC_M, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (R::DBLK)
        ok = ok && encode2d(o.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, M.dpl, M.trows, M.dstride, M.trows * 2, TC_M, R::DBLK,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    if (R::AUX)
        ok = ok && encode2d(o.aux, CU_TENSOR_MAP_DATA_TYPE_UINT32, M.aux, M.trows, M.dstride, M.trows * 4, TC_M, R::AUX,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    return ok;
}

bool make_weight_maps(const DevMat& M, WMaps& out) {
    memset(&out, 0, sizeof out);
    switch (M.type) {
        case T_Q4_K: return maps_for<T_Q4_K>(M, out);
        case T_Q5_K: return maps_for<T_Q5_K>(M, out);
        case T_Q6_K: return maps_for<T_Q6_K>(M, out);
        case T_Q4_0: return maps_for<T_Q4_0>(M, out);
        case T_Q5_0: return maps_for<T_Q5_0>(M, out);
        case T_Q8_0: return maps_for<T_Q8_0>(M, out);
        case T_DENSE: return maps_for<T_DENSE>(M, out);
        default: return false;
    }
}

bool make_rows_map(const __half* base, uint64_t rows, uint32_t width, CUtensorMap& out) {
    return encode2d(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, width, rows, (uint64_t)width * 2, TC_KS, TC_BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---------------------------------------------------------------------------------------------
// device: TMA 2-D tile load (no multicast)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Decode K-elements [64*sub + 32*half, +32) of one weight row into 16 packed fp16 pairs (k, k+1).
// p = the row's main-plane bytes for the stage; dq / aq = its block-scale / high-bit entries
// (block b of the stage at dq + 256 b / aq + 512 b).  half is warp-uniform.
template <int TYPE>
__device__ __forceinline__ void slice32(const uint8_t* p, const uint8_t* dq, const uint8_t* aq, int sub, int half,
                                        uint32_t* v);

// Packed-half helpers: a 4- or 6-bit code c placed in the low mantissa bits of 0x6400 is the
// exact fp16 value 1024 + c, so code -> fp16 costs one byte permute and one logic op per pair.
__device__ __forceinline__ __half2 as_h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }
__device__ __forceinline__ uint32_t as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t lop_or3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xFE;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));  // a | b | c
    return r;
}

// Q4_K: y = d*sc*q - dmin*m over sub-block 2*sub + half (the low nibbles of the slice's 32 qs
// bytes for half 0, the high nibbles for half 1).  Per pair: the two codes land in 1024 + q
// (exact), 1024 is subtracted exactly, and one fused multiply-add by the fp16-rounded sub-block
// scale and min gives the value (the scale, the min and the result each round once to fp16;
// the f32 path rounds the result only, and the difference is well inside the layer tolerance).
template <>
__device__ __forceinline__ void slice32<T_Q4_K>(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(p);
    const float d = h2f((uint16_t)(dd & 0xFFFF)), dmin = h2f((uint16_t)(dd >> 16));
    int sc, mn;
    scale_min_k4(2 * sub + half, p + 4, sc, mn);
    const __half2 D = __float2half2_rn(__fmul_rn(d, (float)sc)), M = __float2half2_rn(-__fmul_rn(dmin, (float)mn));
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

template <>
__device__ __forceinline__ void slice32<T_Q5_K>(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
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

// Q6_K main plane row: ql[128] | qh[64] | scales[16]; d from the block-scale plane.  Slice
// `sub` covers quadrants 2*(sub&1) and 2*(sub&1)+1 of the 128-element half sub>>1; `half`
// picks one: its low bits are the low (sub even) or high (sub odd) nibbles of ql[0..31]
// (half 0) or ql[32..63] (half 1) of that half, its two high bits sit at bits 2*quadrant of qh.
template <>
__device__ __forceinline__ void slice32<T_Q6_K>(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
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

// Q4_0 main plane row: qs[8 x 16]; half = block 2*sub + half (low nibbles -> elements 0..15,
// high nibbles -> 16..31).
template <>
__device__ __forceinline__ void slice32<T_Q4_0>(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
    const int b = 2 * sub + half;
    const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 256 * b));
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

// Q5_0 main plane row: qs[8 x 16]; high bits and scales from their planes.
template <>
__device__ __forceinline__ void slice32<T_Q5_0>(const uint8_t* p, const uint8_t* dq, const uint8_t* aq, int sub,
                                                int half, uint32_t* v) {
    const int b = 2 * sub + half;
    const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 256 * b));
    const uint32_t qh = *reinterpret_cast<const uint32_t*>(aq + 512 * b);
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

// Q8_0 main plane row: qs[8 x 32]; half = block 2*sub + half.
template <>
__device__ __forceinline__ void slice32<T_Q8_0>(const uint8_t* p, const uint8_t* dq, const uint8_t*, int sub, int half,
                                                uint32_t* v) {
    const int b = 2 * sub + half;
    const float d = h2f(*reinterpret_cast<const uint16_t*>(dq + 256 * b));
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

template <>
__device__ __forceinline__ void slice32<T_DENSE>(const uint8_t* p, const uint8_t*, const uint8_t*, int sub, int half,
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

template <int TYPE, int NMAT>
struct TcGeom {
    static constexpr int B_STAGE = TC_BN * 128;  // bytes per token tile stage
    static constexpr int RAW_STAGE = NMAT * RawStage<TYPE>::BYTES;
    // down keeps one stage less so that two of its CTAs fit on an SM (one drains while the other
    // computes); gate/up fills the tensor memory with its two accumulators and runs alone
    static constexpr int NST = NMAT == 2 ? TC_NST : TC_NST - 1;
    static constexpr int SMEM = NST * B_STAGE + TC_RST * RAW_STAGE + 1024;
    // converter warps per matrix: 4 decode whole 64-element slices; 8 would split each slice
    // into two 32-element halves (measured slower on B200: the per-slice waits and arrivals
    // double while the decode itself does not shrink)
    static constexpr int CW = 4;
    static constexpr int CONV = 32 * CW * NMAT;  // converter / epilogue threads
    static constexpr int THREADS = 128 + CONV;
    static constexpr int MIN_BLOCKS = NMAT == 2 ? 1 : 2;
    static constexpr uint32_t TMEM_COLS = NMAT == 2 ? 512 : 256;
    static constexpr int A_COL0 = NMAT * TC_BN;  // A ring after the accumulators
};

template <int TYPE, int NMAT>
__global__ void __launch_bounds__(TcGeom<TYPE, NMAT>::THREADS, TcGeom<TYPE, NMAT>::MIN_BLOCKS)
    tc_grouped_kernel(const __grid_constant__ GroupedParams p, const __grid_constant__ TcMaps maps) {
    using G = TcGeom<TYPE, NMAT>;
    using RS = RawStage<TYPE>;
    constexpr int RK = Raw<TYPE>::RK, PITCH = Raw<TYPE>::PITCH, SUBS = RK / TC_KS;
    constexpr int NST = G::NST;
    extern __shared__ uint8_t dsmem[];
    __shared__ __align__(8) uint64_t bar_raw_full[TC_RST], bar_raw_empty[TC_RST];
    __shared__ __align__(8) uint64_t bar_a_full[NST], bar_b_full[NST], bar_empty[NST];
    __shared__ __align__(8) uint64_t bar_acc;
    __shared__ uint32_t tmem_holder;
    __shared__ int s_tok[TC_BN], s_rexp[TC_BN];
    __shared__ float s_w[TC_BN];
    __shared__ volatile int s_abort;

    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;  // uniform exit before any barrier or TMEM use
    const int4 ti = p.tiles[tile];
    const int e = ti.x, row0 = ti.y, nrows = ti.z;
    const int n_eff = (nrows + 15) & ~15;
    const int fb = blockIdx.x;
    const int sh = e >= p.E ? 1 : 0;  // shared expert: its own single-expert stacks
    const DevMat& M0 = NMAT == 2 ? (sh ? p.sgate : p.gate) : (sh ? p.sdown : p.down);
    const int grow0 = (sh ? 0 : e) * (int)M0.rows + fb * TC_M;  // first weight row of the CTA
    const int K = NMAT == 2 ? p.H : p.I;
    const int nk = K / TC_KS, nraw = K / RK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const uint32_t sbase = (smem_u32(dsmem) + 1023u) & ~1023u;  // 1024-B aligned (SW128 atoms)
    uint8_t* gbase = dsmem + (sbase - smem_u32(dsmem));
    const uint32_t bring = sbase, rawring = sbase + NST * G::B_STAGE;
    uint8_t* raw_g = gbase + NST * G::B_STAGE;

    // TMA of raw stage j (all planes of all matrices) into ring slot j % TC_RST
    auto issue_raw = [&](int j) {
        const int s = j % TC_RST;
        const uint32_t bar = smem_u32(&bar_raw_full[s]);
        mbar_arrive_expect_tx(bar, (uint32_t)G::RAW_STAGE);
#pragma unroll
        for (int m = 0; m < NMAT; m++) {
            const WMaps& wm = maps.w[sh][m];
            const uint32_t dst = rawring + (uint32_t)(s * NMAT + m) * RS::BYTES;
            tma_2d(dst, &wm.main, j * (Raw<TYPE>::MB / 2), grow0, bar);
            if (Raw<TYPE>::DBLK) tma_2d(dst + RS::DOFF, &wm.d, grow0, j * Raw<TYPE>::DBLK, bar);
            if (Raw<TYPE>::AUX) tma_2d(dst + RS::AOFF, &wm.aux, grow0, j * Raw<TYPE>::AUX, bar);
        }
    };
    if (tid == 0) {
        for (int i = 0; i < TC_RST; i++) {
            mbar_init(smem_u32(&bar_raw_full[i]), 1);
            mbar_init(smem_u32(&bar_raw_empty[i]), G::CW * NMAT);
        }
        for (int i = 0; i < NST; i++) {
            mbar_init(smem_u32(&bar_a_full[i]), G::CW * NMAT);
            mbar_init(smem_u32(&bar_b_full[i]), 1);
            mbar_init(smem_u32(&bar_empty[i]), 1);
        }
        mbar_init(smem_u32(&bar_acc), 1);
        s_abort = 0;
        fence_mbar_init();
        // the first raw stages need no free-slot wait: start them before the prologue's loads
        for (int j = 0; j < TC_RST && j < nraw; j++) issue_raw(j);
    }
    for (int n = tid; n < TC_BN; n += G::THREADS) {
        int tok = 0, rexp = 0;
        float w = 0.0f;
        if (n < nrows) {
            const int r = row0 + n;
            tok = __ldg(p.row_tok + r);
            const int slot = __ldg(p.row_slot + r);
            w = (slot < p.k) ? __ldg(p.topk_w + (size_t)tok * p.k + slot) : 1.0f;
            if (NMAT == 1) rexp = __ldg(p.rowexp + r);
        }
        s_tok[n] = tok;
        s_w[n] = w;
        s_rexp[n] = rexp;
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_holder), G::TMEM_COLS);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tbase = tmem_holder;

    auto fail = [&]() {
        s_abort = 1;
        atomicOr(p.status, (unsigned)DERR_TIMEOUT);
    };

    if (warp == 0) {
        // ---------------- TMA producer: raw weight superblocks ----------------
        if (lane == 0) {
            for (int j = TC_RST; j < nraw; j++) {
                if (s_abort) break;
                if (!mbar_wait(smem_u32(&bar_raw_empty[j % TC_RST]), ((j / TC_RST) + 1) & 1)) {
                    fail();
                    break;
                }
                issue_raw(j);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(TC_M, n_eff);
            for (int kt = 0; kt < nk; kt++) {
                const int s = kt % NST;
                const uint32_t ph = (kt / NST) & 1;
                if (s_abort) break;
                if (!mbar_wait(smem_u32(&bar_a_full[s]), ph) || !mbar_wait(smem_u32(&bar_b_full[s]), ph)) {
                    fail();
                    break;
                }
                fence_after_sync();
                const uint32_t bst = bring + (uint32_t)s * G::B_STAGE;
#pragma unroll
                for (int m = 0; m < NMAT; m++)
#pragma unroll
                    for (int ks = 0; ks < TC_KS / 16; ks++)
                        mma_ts(tbase + (uint32_t)(m * TC_BN), tbase + (uint32_t)(G::A_COL0 + (s * NMAT + m) * 32 + ks * 8),
                               smem_desc_sw128(bst + ks * 32), idesc, (kt | ks) != 0);
                mma_commit(smem_u32(&bar_empty[s]));
            }
            mma_commit(smem_u32(&bar_acc));  // also fires when aborted: every issued MMA has finished
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---------------- token tiles: one thread streams them with TMA onto b_full ----------------
        if (tid == 64) {
            for (int kt = 0; kt < nk; kt++) {
                const int s = kt % NST;
                if (s_abort) break;
                if (kt >= NST && !mbar_wait(smem_u32(&bar_empty[s]), ((kt / NST) + 1) & 1)) {
                    fail();
                    break;
                }
                const uint32_t bar = smem_u32(&bar_b_full[s]);
                mbar_arrive_expect_tx(bar, (uint32_t)G::B_STAGE);
                tma_2d(bring + (uint32_t)s * G::B_STAGE, &maps.b, kt * TC_KS, row0, bar);
            }
        }
    } else {
        // ---------------- converters: one thread per weight row ----------------
        // warp (4 + cw) writes TMEM lanes 32 * (warp & 3) (a warp may only reach its quarter).
        // Software-pipelined by one stage: the tensor-memory store of slice kt completes while
        // slice kt + 1 is decoded, and only then is stage kt reported full (two register sets).
        constexpr int CW = G::CW;
        static_assert(CW == 4, "one converter warp per lane quarter and matrix");
        const int cw = warp - 4, m = cw / CW, q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
        bool ok = true;
        int pend = -1;  // stage whose store is in flight
        auto report = [&](uint32_t* vp) {  // the pending store (of vp) has landed: stage full
            tmem_st_wait_hold(vp);
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_a_full[pend % NST]));
            pend = -1;
        };
        auto stage = [&](int kt, uint32_t* v, uint32_t* vp) {
            const int j = kt / SUBS, sub = kt % SUBS, s = kt % NST;
            if (s_abort) { ok = false; return; }
            if (sub == 0 && !mbar_wait(smem_u32(&bar_raw_full[j % TC_RST]), (j / TC_RST) & 1)) {
                fail();
                ok = false;
                return;
            }
            if (kt >= NST && !mbar_wait(smem_u32(&bar_empty[s]), ((kt / NST) + 1) & 1)) {
                fail();
                ok = false;
                return;
            }
            const uint8_t* mat = raw_g + (size_t)((j % TC_RST) * NMAT + m) * RS::BYTES;
            const uint8_t *rp = mat + r * PITCH, *rd = mat + RS::DOFF + r * 2, *ra = mat + RS::AOFF + r * 4;
            slice32<TYPE>(rp, rd, ra, sub, 0, v);
            slice32<TYPE>(rp, rd, ra, sub, 1, v + 16);
            if (sub == SUBS - 1) {  // every lane has read its last bytes of this raw slot
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bar_raw_empty[j % TC_RST]));
            }
            if (pend >= 0) report(vp);
            tmem_st32(tlane + (uint32_t)(G::A_COL0 + (s * NMAT + m) * 32), v);
            pend = kt;
        };
        uint32_t v0[32], v1[32];
        for (int kt = 0; kt < nk && ok; kt += 2) {  // nk is a multiple of 4
            stage(kt, v0, v1);
            if (ok) stage(kt + 1, v1, v0);
        }
        if (pend >= 0) report((pend & 1) ? v1 : v0);
        // ---------------- epilogue ----------------
        const bool acc_ok = mbar_wait(smem_u32(&bar_acc), 0);
        if (!acc_ok) fail();
        fence_after_sync();
        const bool work = acc_ok && !s_abort;
        if (NMAT == 2) {
            // SwiGLU in f32 into a shared staging tile hs[n][f] (the rings are free now)
            float* hs = reinterpret_cast<float*>(gbase);
            constexpr int HLD = TC_M + 4;  // 16-B aligned rows; lanes of one read hit distinct banks
            // token chunk c (32 columns) of the accumulators: warps of a lane quarter share them out
            for (int c = cw >> 2; c * 32 < n_eff; c += G::CONV / 128) {
                uint32_t g[32], u[32];
                tmem_ld32(tlane + (uint32_t)(c * 32), g);
                tmem_ld32(tlane + (uint32_t)(TC_BN + c * 32), u);
                tmem_ld_wait();
                if (work) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        float gv = __uint_as_float(g[i]), uv = __uint_as_float(u[i]);
                        // SiLU (src/moe.rs:44-51) with the fast exponential: the result is
                        // rounded to fp16 next, far coarser than the approximation
                        hs[(c * 32 + i) * HLD + r] = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
                    }
                }
            }
            asm volatile("bar.sync 1, %0;\n" ::"n"(G::CONV) : "memory");
            if (work) {
                // per (row, 64-feature block): exponent, fp16 values, block/row exponents
                const int nblk = p.I / HBLK;
                const int ct = tid - 128;
                for (int pi = ct; pi < nrows * 2; pi += G::CONV) {
                    const int blk = pi >= nrows ? 1 : 0, n = pi - blk * nrows;  // consecutive lanes: rows
                    const float* src = hs + n * HLD + blk * 64;
                    const float4* s4 = reinterpret_cast<const float4*>(src);
                    float amax = 0.0f;
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float4 t = s4[i];
                        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
                    }
                    int ex = -127;
                    if (amax > 0.0f) {
                        int e2;
                        frexpf(amax, &e2);
                        ex = max(-100, min(100, e2 - 14));
                    }
                    const float sc = exp2i(-ex);
                    const size_t rr = (size_t)(row0 + n);
                    uint4* dst = reinterpret_cast<uint4*>(p.h + rr * p.I + fb * TC_M + blk * 64);
#pragma unroll
                    for (int j2 = 0; j2 < 8; j2++) {
                        const float4 a = s4[2 * j2], b = s4[2 * j2 + 1];
                        dst[j2] = make_uint4(pack_f16x2(__fmul_rn(a.x, sc), __fmul_rn(a.y, sc)),
                                             pack_f16x2(__fmul_rn(a.z, sc), __fmul_rn(a.w, sc)),
                                             pack_f16x2(__fmul_rn(b.x, sc), __fmul_rn(b.y, sc)),
                                             pack_f16x2(__fmul_rn(b.z, sc), __fmul_rn(b.w, sc)));
                    }
                    p.hexp[rr * nblk + fb * 2 + blk] = (int8_t)ex;
                    atomicMax(p.rowexp + rr, ex);
                }
            }
        } else {
            // y tile through shared memory, ys[n][f] (the rings are idle once bar_acc has fired),
            // so that each warp then writes whole 512-B token rows with 16-B stores or vector
            // reductions. Scaling by 2^rowexp is exact, so w * (acc * 2^e) == acc * (w * 2^e).
            float* ys = reinterpret_cast<float*>(gbase);
            constexpr int YLD = TC_M + 4;
            for (int c = cw >> 2; c * 32 < n_eff; c += G::CONV / 128) {
                uint32_t a[32];
                tmem_ld32(tlane + (uint32_t)(c * 32), a);
                tmem_ld_wait();
                if (!work) continue;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const int n = c * 32 + i;
                    const float sc = p.y ? exp2i(s_rexp[n]) : __fmul_rn(s_w[n], exp2i(s_rexp[n]));
                    ys[n * YLD + r] = __fmul_rn(__uint_as_float(a[i]), sc);
                }
            }
            asm volatile("bar.sync 1, %0;\n" ::"n"(G::CONV) : "memory");
            if (work) {
                const int f = fb * TC_M + 4 * lane;
                for (int n = cw; n < nrows; n += G::CONV / 32) {  // one token row per epilogue warp
                    const float4 v = *reinterpret_cast<const float4*>(ys + n * YLD + 4 * lane);
                    if (p.y) *reinterpret_cast<float4*>(p.y + (size_t)(row0 + n) * p.H + f) = v;
                    else atomicAdd(reinterpret_cast<float4*>(p.out + (size_t)s_tok[n] * p.H + f), v);
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        tmem_dealloc(tbase, G::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------
// h to one scale per row.  The gate/up CTAs each see 128 features of a row, so they store h as
// fp16 x 2^hexp per 64-feature block; once all of them are done the row's common exponent
// (rowexp = max over its blocks) is known and every block is brought to it here, once, so the
// down kernel's token tiles go from global memory to the MMA untouched.  Multiplying by
// 2^(hexp - rowexp) <= 1 is exact down to the fp16 subnormal range; blocks more than 24 binades
// below the row's largest would be flushed by it anyway and are zeroed.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rescale_h_kernel(__half* __restrict__ h, const int8_t* __restrict__ hexp,
                                                        const int* __restrict__ rowexp, const int* __restrict__ n_rows,
                                                        int I) {
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (r >= *n_rows) return;
    const int re = __ldg(rowexp + r), nblk = I / HBLK;
    uint4* row = reinterpret_cast<uint4*>(h + (size_t)r * I);
    for (int c = lane; c < I / 8; c += 32) {
        const int dexp = (int)__ldg(hexp + (size_t)r * nblk + c / 8) - re;
        if (dexp == 0) continue;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (dexp >= -24) {
            v = row[c];
            const __half2 sc = __float2half2_rn(exp2i(dexp));
            __half2* h2 = reinterpret_cast<__half2*>(&v);
#pragma unroll
            for (int i = 0; i < 4; i++) h2[i] = __hmul2(h2[i], sc);
        }
        row[c] = v;
    }
}

cudaError_t launch_rescale_h(const GroupedParams& p, int max_rows, cudaStream_t s) {
    if (max_rows <= 0) return cudaSuccess;
    rescale_h_kernel<<<(max_rows + 7) / 8, 256, 0, s>>>(p.h, p.hexp, p.rowexp, p.n_rows, p.I);
    return cudaGetLastError();
}

template <int TYPE, int NMAT>
static cudaError_t go_tc(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    using G = TcGeom<TYPE, NMAT>;
    auto k = tc_grouped_kernel<TYPE, NMAT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((NMAT == 2 ? p.I : p.H) / TC_M, max_tiles);
    k<<<grid, G::THREADS, G::SMEM, s>>>(p, maps);
    return cudaGetLastError();
}

#define RMOE_TC_SWITCH(T, ...)                                     \
    switch (T) {                                                   \
        case T_Q4_0: { constexpr int TT = T_Q4_0; __VA_ARGS__; }   \
        case T_Q5_0: { constexpr int TT = T_Q5_0; __VA_ARGS__; }   \
        case T_Q8_0: { constexpr int TT = T_Q8_0; __VA_ARGS__; }   \
        case T_Q4_K: { constexpr int TT = T_Q4_K; __VA_ARGS__; }   \
        case T_Q5_K: { constexpr int TT = T_Q5_K; __VA_ARGS__; }   \
        case T_Q6_K: { constexpr int TT = T_Q6_K; __VA_ARGS__; }   \
        case T_DENSE: { constexpr int TT = T_DENSE; __VA_ARGS__; } \
        default: return cudaErrorInvalidValue;                     \
    }

cudaError_t launch_tc_gateup(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    RMOE_TC_SWITCH(p.gate.type, return go_tc<TT, 2>(p, maps, max_tiles, s))
}

cudaError_t launch_tc_down(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    RMOE_TC_SWITCH(p.down.type, return go_tc<TT, 1>(p, maps, max_tiles, s))
}

}  // namespace rmoe
