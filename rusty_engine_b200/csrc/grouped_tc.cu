// grouped_tc.cu -- tensor-core (tcgen05) grouped expert products for large batches (prefill).
//
//   gate/up: h[row, f] = silu(gate_f . x_row) * (up_f . x_row)   (src/moe.rs:280-299)
//   down:    out[tok] += w_slot * (down . h_row)                  (src/moe.rs:373-380)
//
// Both work on tiles of <= 256 expert-sorted rows (one expert each) and 128-feature blocks of
// the expert's weights, with MMA M = 128 (weight rows), N = the tile's rows (rounded to 16),
// K = 64 per stage, fp16 operands and f32 accumulators in tensor memory.
//
// gate/up (tc_grouped_kernel<TYPE, 2>, one CTA per (tile, block), one CTA per SM):
//   warp 0      TMA producer: one 2-D tensor copy per matrix and plane brings the raw GGUF
//               bytes of the CTA's 128 gate and 128 up rows for one raw stage into a ring;
//   warp 1      allocates tensor memory and issues tcgen05.mma (one elected thread), A (the
//               dequantized weights) and B (the token tile) both from shared memory, into the
//               gate and up accumulators (2 x 256 columns);
//   warp 2      one thread streams the expert-sorted x tiles with a 128-B-swizzled 2-D TMA;
//   warps 4-11  one thread per weight row decodes 64 K-elements of its row per stage from the
//               raw ring and writes them, 128-B-swizzled and K-major, as the MMA's A tile; after
//               the last stage the same warps run SwiGLU and store h as fp16 x 2^e per (row,
//               64-feature block).
// down (tc_down_kernel<TYPE>, persistent, one CTA per SM walking (tile, block) items): the same
//   producer / MMA / h-tile / converter roles, two accumulators so that four epilogue warps
//   drain item i (y scaled by the routing weight, 16-B vector reductions into out) while item
//   i + 1 is decoded and multiplied.
// Every wait is bounded: on a timeout a kernel records DERR_TIMEOUT in the status word, skips
// the remaining work, waits for its own MMAs and frees its tensor memory.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rmoe {
using namespace tc;

static constexpr int TC_M = 128;   // weight rows per matrix per CTA (= TMEM lanes, = TMA box rows)
static constexpr int TC_BN = 256;  // expert-sorted rows per tile at most (MMA N, rounded to 16 per tile)
static constexpr int TC_KS = 64;   // K elements per MMA stage (one 128-B swizzle row of fp16)
static constexpr int TC_RST = 2;   // raw weight stages in flight

int tc_tile_rows() { return TC_BN; }

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
static bool maps_for(const DevMat& M, WMaps& o, uint32_t rows) {
    using R = Raw<TYPE>;
    // main plane as u16 [trows][main_stride / 2]; box = PITCH bytes x `rows` rows (past the row
    // end the box reads zeros)
    bool ok = encode2d(o.main, CU_TENSOR_MAP_DATA_TYPE_UINT16, M.main, M.main_stride / 2, M.trows, M.main_stride,
                       R::PITCH / 2, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (R::DBLK)
        ok = ok && encode2d(o.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, M.dpl, M.trows, M.dstride, M.trows * 2, rows, R::DBLK,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    if (R::AUX)
        ok = ok && encode2d(o.aux, CU_TENSOR_MAP_DATA_TYPE_UINT32, M.aux, M.trows, M.dstride, M.trows * 4, rows, R::AUX,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    return ok;
}

bool make_weight_maps(const DevMat& M, WMaps& out, uint32_t rows) {
    memset(&out, 0, sizeof out);
    switch (M.type) {
        case T_Q4_K: return maps_for<T_Q4_K>(M, out, rows);
        case T_Q5_K: return maps_for<T_Q5_K>(M, out, rows);
        case T_Q6_K: return maps_for<T_Q6_K>(M, out, rows);
        case T_Q4_0: return maps_for<T_Q4_0>(M, out, rows);
        case T_Q5_0: return maps_for<T_Q5_0>(M, out, rows);
        case T_Q8_0: return maps_for<T_Q8_0>(M, out, rows);
        case T_DENSE: return maps_for<T_DENSE>(M, out, rows);
        default: return false;
    }
}

bool make_rows_map(const __half* base, uint64_t rows, uint32_t width, CUtensorMap& out) {
    return encode2d(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, width, rows, (uint64_t)width * 2, TC_KS, TC_BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

bool make_f32_rows_map(const float* base, uint64_t rows, uint32_t width, uint32_t box_w, uint32_t box_rows,
                       CUtensorMap& out) {
    return encode2d(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, width, rows, (uint64_t)width * 4, box_w, box_rows,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int TYPE, int NMAT>
struct TcGeom {
    static_assert(NMAT == 2, "the gate and up matrices");
    static constexpr int B_STAGE = TC_BN * 128;  // bytes per token tile stage
    static constexpr int RAW_STAGE = NMAT * RawStage<TYPE, TC_M>::BYTES;
    // the two accumulators (2 x 256 columns) fill the tensor memory, so the dequantized weight
    // tiles go to shared memory (128-B-swizzled like the token tiles) and two stages fit
    static constexpr int A_STAGE = NMAT * TC_M * 128;  // bytes per stage
    static constexpr int NA = 2;                       // weight-tile stages
    static constexpr int SMEM_MAX = 232448;            // opt-in shared memory per block
    static constexpr int LIM = SMEM_MAX - 4096, BASE = NA * A_STAGE + 1024;
    // token-tile and raw stages: (3, 2) where they fit (the TMA latency of a token tile from L2
    // spans about two MMA stages), then (2, 2), (2, 1)
    static constexpr bool F32 = BASE + 3 * B_STAGE + 2 * RAW_STAGE <= LIM;
    static constexpr bool F22 = BASE + 2 * B_STAGE + 2 * RAW_STAGE <= LIM;
    static constexpr int NB = F32 ? 3 : 2;
    static constexpr int RST = (F32 || F22) ? 2 : 1;
    static constexpr int SMEM = BASE + NB * B_STAGE + RST * RAW_STAGE;
    // converter warps per stage-parity group (two groups; a thread decodes one gate and one up
    // row of every other stage)
    static constexpr int CW = 4;
    static constexpr int CONV = 32 * CW * NMAT;  // converter / epilogue threads
    static constexpr int THREADS = 128 + CONV;
    static constexpr int MIN_BLOCKS = 1;
    static constexpr uint32_t TMEM_COLS = 512;
    static_assert(SMEM <= SMEM_MAX - 4096, "shared memory budget (static part included)");
    static_assert(SMEM - 1024 >= TC_BN * (TC_M + 4) * 4, "epilogue staging tile fits in the rings");
};

template <int TYPE, int NMAT>
__global__ void __launch_bounds__(TcGeom<TYPE, NMAT>::THREADS, TcGeom<TYPE, NMAT>::MIN_BLOCKS)
    tc_grouped_kernel(const __grid_constant__ GroupedParams p, const __grid_constant__ TcMaps maps) {
    using G = TcGeom<TYPE, NMAT>;
    using RS = RawStage<TYPE, TC_M>;
    constexpr int RK = Raw<TYPE>::RK, PITCH = Raw<TYPE>::PITCH, SUBS = RK / TC_KS;
    constexpr int NA = G::NA, NB = G::NB, RST = G::RST;
    extern __shared__ uint8_t dsmem[];
    __shared__ __align__(8) uint64_t bar_raw_full[RST], bar_raw_empty[RST];
    __shared__ __align__(8) uint64_t bar_a_full[NA], bar_a_empty[NA], bar_b_full[NB], bar_b_empty[NB];
    __shared__ __align__(8) uint64_t bar_acc;
    __shared__ uint32_t tmem_holder;
    __shared__ volatile int s_abort;

    // launched with programmatic dependent launch after the x gather: the tile list and the
    // weights may be read at once, the token tiles only after pdl_wait (token-tile producer)
    pdl_trigger();
    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;  // uniform exit before any barrier or TMEM use
    const int4 ti = p.tiles[tile];
    const int e = ti.x, row0 = ti.y, nrows = ti.z;
    const int n_eff = (nrows + 15) & ~15;
    const int fb = blockIdx.x;
    const int sh = e >= p.E ? 1 : 0;  // shared expert: its own single-expert stacks
    const DevMat& M0 = sh ? p.sgate : p.gate;
    const int grow0 = (sh ? 0 : e) * (int)M0.rows + fb * TC_M;  // first weight row of the CTA
    const int K = p.H;
    const int nk = K / TC_KS, nraw = K / RK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const uint32_t sbase = (smem_u32(dsmem) + 1023u) & ~1023u;  // 1024-B aligned (SW128 atoms)
    uint8_t* gbase = dsmem + (sbase - smem_u32(dsmem));
    // [B ring | A ring | raw ring], every tile 1024-B aligned
    const uint32_t bring = sbase, aring = sbase + NB * G::B_STAGE, rawring = aring + NA * G::A_STAGE;
    uint8_t* a_g = gbase + NB * G::B_STAGE;
    uint8_t* raw_g = a_g + NA * G::A_STAGE;

    // TMA of raw stage j (all planes of all matrices) into ring slot j % RST
    auto issue_raw = [&](int j) {
        const int s = j % RST;
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
        for (int i = 0; i < RST; i++) {
            mbar_init(smem_u32(&bar_raw_full[i]), 1);
            mbar_init(smem_u32(&bar_raw_empty[i]), G::CW * NMAT);
        }
        for (int i = 0; i < NA; i++) {
            mbar_init(smem_u32(&bar_a_full[i]), G::CW);  // the four warps of one stage-parity group
            mbar_init(smem_u32(&bar_a_empty[i]), 1);
        }
        for (int i = 0; i < NB; i++) {
            mbar_init(smem_u32(&bar_b_full[i]), 1);
            mbar_init(smem_u32(&bar_b_empty[i]), 1);
        }
        mbar_init(smem_u32(&bar_acc), 1);
        s_abort = 0;
        fence_mbar_init();
        // the first raw stages need no free-slot wait: start them before the prologue's loads
        for (int j = 0; j < RST && j < nraw; j++) issue_raw(j);
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
            for (int j = RST; j < nraw; j++) {
                if (s_abort) break;
                if (!mbar_wait(smem_u32(&bar_raw_empty[j % RST]), ((j / RST) + 1) & 1)) {
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
                const int sa = kt % NA, sb = kt % NB;
                if (s_abort) break;
                if (!mbar_wait(smem_u32(&bar_a_full[sa]), (kt / NA) & 1) ||
                    !mbar_wait(smem_u32(&bar_b_full[sb]), (kt / NB) & 1)) {
                    fail();
                    break;
                }
                fence_after_sync();
                const uint32_t bst = bring + (uint32_t)sb * G::B_STAGE;
#pragma unroll
                for (int m = 0; m < NMAT; m++)
#pragma unroll
                    for (int ks = 0; ks < TC_KS / 16; ks++)
                        mma_ss(tbase + (uint32_t)(m * TC_BN),
                               smem_desc_sw128(aring + (uint32_t)(sa * NMAT + m) * (TC_M * 128) + ks * 32),
                               smem_desc_sw128(bst + ks * 32), idesc, (kt | ks) != 0);
                mma_commit(smem_u32(&bar_a_empty[sa]));
                mma_commit(smem_u32(&bar_b_empty[sb]));
            }
            mma_commit(smem_u32(&bar_acc));  // also fires when aborted: every issued MMA has finished
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---------------- token tiles: one thread streams them with TMA onto b_full ----------------
        if (tid == 64) {
            pdl_wait();  // the expert-sorted token rows are the previous kernel's output
            for (int kt = 0; kt < nk; kt++) {
                const int s = kt % NB;
                if (s_abort) break;
                if (kt >= NB && !mbar_wait(smem_u32(&bar_b_empty[s]), ((kt / NB) + 1) & 1)) {
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
        // Two groups of four warps take alternate stages (group g the stages kt = g mod 2, so it
        // always fills A slot g): each thread decodes 64 K-elements of its gate row and of its up
        // row per stage, and has two MMA stages of time for it, which hides the latency of the
        // raw loads, the stores and the proxy fence of one stage behind the other group's.
        // Warp (4 + cw): group cw / 4, rows 32 (warp & 3) .. +31 (the epilogue reads the
        // accumulators of those TMEM lanes, which a warp may only reach in its own quarter).
        constexpr int CW = G::CW;
        static_assert(CW == 4 && NA == 2 && SUBS % 2 == 0, "two stage-parity groups of four warps");
        const int cw = warp - 4, g = cw >> 2, q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
        for (int kt = g; kt < nk; kt += 2) {
            const int j = kt / SUBS, sub = kt % SUBS, s = kt % NA;
            if (s_abort) break;
            if (sub == g && !mbar_wait(smem_u32(&bar_raw_full[j % RST]), (j / RST) & 1)) {
                fail();
                break;
            }
            if (kt >= NA && !mbar_wait(smem_u32(&bar_a_empty[s]), ((kt / NA) + 1) & 1)) {
                fail();
                break;
            }
#pragma unroll
            for (int m = 0; m < NMAT; m++) {
                const uint8_t* mat = raw_g + (size_t)((j % RST) * NMAT + m) * RS::BYTES;
                const uint8_t *rp = mat + r * PITCH, *rd = mat + RS::DOFF + r * 2, *ra = mat + RS::AOFF + r * 4;
                uint32_t v[32];
                slice32<TYPE, TC_M>(rp, rd, ra, sub, 0, v);
                slice32<TYPE, TC_M>(rp, rd, ra, sub, 1, v + 16);
                if (m == NMAT - 1 && sub == SUBS - 2 + g) {  // this group's last read of the raw slot
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&bar_raw_empty[j % RST]));
                }
                // row r of the 128-B-swizzled K-major tile: 16-B chunk c at (c ^ (r & 7)) * 16
                uint8_t* at = a_g + (size_t)(s * NMAT + m) * (TC_M * 128) + r * 128;
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4*>(at + ((c ^ (r & 7)) << 4)) =
                        make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            }
            fence_proxy_async_smem();  // generic-proxy writes -> the MMA's async-proxy reads
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_a_full[s]));
        }
        // ---------------- epilogue ----------------
        const bool acc_ok = mbar_wait(smem_u32(&bar_acc), 0);
        if (!acc_ok) fail();
        fence_after_sync();
        const bool work = acc_ok && !s_abort;
        {
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
                // per (row, 64-feature block): exponent, fp16 values, block/row exponents; h is
                // written in the down kernel's operand order (K-permuted for a Q6_K down stack)
                const int nblk = p.I / HBLK;
                const bool kperm = p.down.type == T_Q6_K;
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
                    if (kperm) {  // features in tc_down's Q6_K operand order (kperm_pos)
#pragma unroll
                        for (int j2 = 0; j2 < 8; j2++) {
                            const float4 a = s4[2 * j2], b = s4[2 * j2 + 1];
                            dst[j2] = make_uint4(pack_f16x2(__fmul_rn(a.x, sc), __fmul_rn(a.z, sc)),
                                                 pack_f16x2(__fmul_rn(a.y, sc), __fmul_rn(a.w, sc)),
                                                 pack_f16x2(__fmul_rn(b.x, sc), __fmul_rn(b.z, sc)),
                                                 pack_f16x2(__fmul_rn(b.y, sc), __fmul_rn(b.w, sc)));
                        }
                    } else {
#pragma unroll
                        for (int j2 = 0; j2 < 8; j2++) {
                            const float4 a = s4[2 * j2], b = s4[2 * j2 + 1];
                            dst[j2] = make_uint4(pack_f16x2(__fmul_rn(a.x, sc), __fmul_rn(a.y, sc)),
                                                 pack_f16x2(__fmul_rn(a.z, sc), __fmul_rn(a.w, sc)),
                                                 pack_f16x2(__fmul_rn(b.x, sc), __fmul_rn(b.y, sc)),
                                                 pack_f16x2(__fmul_rn(b.z, sc), __fmul_rn(b.w, sc)));
                        }
                    }
                    p.hexp[rr * nblk + fb * 2 + blk] = (int8_t)ex;
                    atomicMax(p.rowexp + rr, ex);
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
    pdl_trigger();
    pdl_wait();  // h and its exponents are gate/up's output
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (r >= *n_rows) return;
    const int re = rowexp[r], nblk = I / HBLK;
    uint4* row = reinterpret_cast<uint4*>(h + (size_t)r * I);
    for (int c = lane; c < I / 8; c += 32) {
        const int dexp = (int)hexp[(size_t)r * nblk + c / 8] - re;
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
    return launch_pdl(rescale_h_kernel, dim3((max_rows + 7) / 8), dim3(256), 0, s, p.h, (const int8_t*)p.hexp,
                      (const int*)p.rowexp, (const int*)p.n_rows, p.I);
}

template <int TYPE, int NMAT>
static cudaError_t go_tc(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    using G = TcGeom<TYPE, NMAT>;
    auto k = tc_grouped_kernel<TYPE, NMAT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((NMAT == 2 ? p.I : p.H) / TC_M, max_tiles);
    return launch_pdl(k, grid, dim3(G::THREADS), G::SMEM, s, p, maps);
}

// ---------------------------------------------------------------------------------------------
// down, persistent.  One CTA per SM walks the (tile, 128-feature block) items of the launch
// (item = tile * H/128 + block, strided by the grid, so the CTAs working on one tile at a time
// share its h rows in L2).  Two 256-column TMEM accumulators let the epilogue of item i run on
// its own four warps while item i + 1 is decoded and multiplied; the dequantized weight tiles
// therefore go to shared memory (the SS form of the MMA).  Warps:
//   0 raw TMA producer, 1 MMA issuer, 2 h-tile TMA, 4-7 converters (one weight row per thread),
//   8-11 epilogue: TMEM -> 32-token shared chunks -> scaled 16-B stores or vector reductions.
// ---------------------------------------------------------------------------------------------
template <int TYPE>
struct DownGeom {
    using RS = RawStage<TYPE, TC_M>;
    static constexpr int NA = 2, RST = 2;  // weight-tile and raw stages
    static constexpr int B_STAGE = TC_BN * 128, A_STAGE = TC_M * 128;
    // the epilogue's transpose buffers (YB of them): 32-token chunks
    static constexpr int YLD = TC_M + 4, YCH = 32, Y_STAGE = YCH * YLD * 4, YB = 2;
    static constexpr int FIXED = NA * A_STAGE + RST * RS::BYTES + YB * Y_STAGE + 1024;
    // h-tile stages: three where they fit (the 4-6-bit types), else two
    static constexpr int NB = FIXED + 3 * B_STAGE <= 232448 - 4096 ? 3 : 2;
    static constexpr int A_OFF = NB * B_STAGE, RAW_OFF = A_OFF + NA * A_STAGE, Y_OFF = RAW_OFF + RST * RS::BYTES;
    static constexpr int SMEM = Y_OFF + YB * Y_STAGE + 1024;
    // warps 0-3: producer / MMA / h tiles / idle; CW converter warps (two groups taking
    // alternate stages: the decode, not the MMA, is the long pole of a K = 64 stage); 4 epilogue
    // warps
    static constexpr int CW = 8;
    static constexpr int THREADS = (4 + CW + 4) * 32;
    static_assert(SMEM <= 232448 - 4096, "shared memory budget");
    static_assert(A_OFF % 1024 == 0 && RAW_OFF % 128 == 0 && Y_OFF % 16 == 0, "alignment");
};

template <int TYPE>
__global__ void __launch_bounds__(512, 1)
    tc_down_kernel(const __grid_constant__ GroupedParams p, const __grid_constant__ TcMaps maps) {
    using D = DownGeom<TYPE>;
    using RS = RawStage<TYPE, TC_M>;
    constexpr int RK = Raw<TYPE>::RK, PITCH = Raw<TYPE>::PITCH, SUBS = RK / TC_KS, NA = D::NA, NB = D::NB, RST = D::RST;
    constexpr int CW = D::CW, EPI0 = 4 + CW;  // converter warps 4 .. EPI0 - 1, epilogue warps EPI0 ..
    static_assert(D::THREADS == 512, "warp roles");
    extern __shared__ uint8_t dsmem[];
    __shared__ __align__(8) uint64_t bar_raw_full[RST], bar_raw_empty[RST];
    __shared__ __align__(8) uint64_t bar_a_full[NA], bar_a_empty[NA], bar_b_full[NB], bar_b_empty[NB];
    __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2], bar_fin;
    __shared__ uint32_t tmem_holder;
    __shared__ volatile int s_abort, s_epi_stop;

    // launched with programmatic dependent launch after the h rescale: the tile list and the
    // weights may be read at once (the weight stream and the decode start early), h and the row
    // exponents only after pdl_wait (the h-tile producer and the epilogue warps wait)
    pdl_trigger();
    const int nfb = p.H / TC_M;
    const int n_items = *p.n_tiles * nfb;
    if ((int)blockIdx.x >= n_items) return;  // uniform exit before any barrier or TMEM use
    const int K = p.I, nk = K / TC_KS, nraw = K / RK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t sbase = (smem_u32(dsmem) + 1023u) & ~1023u;
    uint8_t* gbase = dsmem + (sbase - smem_u32(dsmem));
    const uint32_t bring = sbase, aring = sbase + D::A_OFF, rawring = sbase + D::RAW_OFF;
    uint8_t* a_g = gbase + D::A_OFF;
    uint8_t* raw_g = gbase + D::RAW_OFF;
    float* ys_g = reinterpret_cast<float*>(gbase + D::Y_OFF);

    if (tid == 0) {
        for (int i = 0; i < RST; i++) {
            mbar_init(smem_u32(&bar_raw_full[i]), 1);
            mbar_init(smem_u32(&bar_raw_empty[i]), CW);
        }
        for (int i = 0; i < NA; i++) {
            mbar_init(smem_u32(&bar_a_full[i]), CW / 2);  // the warps of one stage-parity group
            mbar_init(smem_u32(&bar_a_empty[i]), 1);
        }
        for (int i = 0; i < NB; i++) {
            mbar_init(smem_u32(&bar_b_full[i]), 1);
            mbar_init(smem_u32(&bar_b_empty[i]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&bar_acc_full[i]), 1);
            mbar_init(smem_u32(&bar_acc_empty[i]), 4);
        }
        mbar_init(smem_u32(&bar_fin), 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_holder), 512);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tbase = tmem_holder;
    auto fail = [&]() {
        s_abort = 1;
        atomicOr(p.status, (unsigned)DERR_TIMEOUT);
    };
    // the (expert, first row, rows, feature block) of an item
    auto info = [&](int item, int& e, int& row0, int& nrows, int& fb) {
        const int4 ti = p.tiles[item / nfb];
        e = ti.x; row0 = ti.y; nrows = ti.z; fb = item % nfb;
    };

    if (warp == 0) {
        // ---------------- raw weight producer ----------------
        if (lane == 0) {
            int gj = 0;
            for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
                int e, row0, nrows, fb;
                info(item, e, row0, nrows, fb);
                const int sh = e >= p.E ? 1 : 0;
                const DevMat& M = sh ? p.sdown : p.down;
                const int grow0 = (sh ? 0 : e) * (int)M.rows + fb * TC_M;
                const WMaps& wm = maps.w[sh][0];
                for (int j = 0; j < nraw; j++, gj++) {
                    const int s = gj % RST;
                    if (gj >= RST && !mbar_wait(smem_u32(&bar_raw_empty[s]), ((gj / RST) + 1) & 1)) {
                        fail();
                        break;
                    }
                    const uint32_t bar = smem_u32(&bar_raw_full[s]), dst = rawring + (uint32_t)s * RS::BYTES;
                    mbar_arrive_expect_tx(bar, (uint32_t)RS::BYTES);
                    tma_2d(dst, &wm.main, j * (Raw<TYPE>::MB / 2), grow0, bar);
                    if (Raw<TYPE>::DBLK) tma_2d(dst + RS::DOFF, &wm.d, grow0, j * Raw<TYPE>::DBLK, bar);
                    if (Raw<TYPE>::AUX) tma_2d(dst + RS::AOFF, &wm.aux, grow0, j * Raw<TYPE>::AUX, bar);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int gk = 0, it = 0;
            for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x, it++) {
                int e, row0, nrows, fb;
                info(item, e, row0, nrows, fb);
                const int acc = it & 1;
                if (it >= 2 && !mbar_wait(smem_u32(&bar_acc_empty[acc]), ((it / 2) + 1) & 1)) {
                    fail();
                    break;
                }
                fence_after_sync();
                const uint32_t idesc = idesc_f16(TC_M, (nrows + 15) & ~15);
                bool ok = true;
                for (int kt = 0; kt < nk; kt++, gk++) {
                    const int sa = gk % NA, sb = gk % NB;
                    if (s_abort || !mbar_wait(smem_u32(&bar_a_full[sa]), (gk / NA) & 1) ||
                        !mbar_wait(smem_u32(&bar_b_full[sb]), (gk / NB) & 1)) {
                        if (!s_abort) fail();
                        ok = false;
                        break;
                    }
                    fence_after_sync();
#pragma unroll
                    for (int ks = 0; ks < TC_KS / 16; ks++)
                        mma_ss(tbase + (uint32_t)(acc * TC_BN), smem_desc_sw128(aring + (uint32_t)sa * D::A_STAGE + ks * 32),
                               smem_desc_sw128(bring + (uint32_t)sb * D::B_STAGE + ks * 32), idesc, (kt | ks) != 0);
                    mma_commit(smem_u32(&bar_a_empty[sa]));
                    mma_commit(smem_u32(&bar_b_empty[sb]));
                }
                if (!ok) break;
                mma_commit(smem_u32(&bar_acc_full[acc]));
            }
            mma_commit(smem_u32(&bar_fin));  // every MMA this thread issued has finished when it fires
            if (!mbar_wait(smem_u32(&bar_fin), 0)) fail();
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---------------- h tiles ----------------
        if (lane == 0) {
            pdl_wait();  // h (rescaled) is the previous kernels' output
            int gk = 0;
            for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
                int e, row0, nrows, fb;
                info(item, e, row0, nrows, fb);
                for (int kt = 0; kt < nk; kt++, gk++) {
                    const int s = gk % NB;
                    if (gk >= NB && !mbar_wait(smem_u32(&bar_b_empty[s]), ((gk / NB) + 1) & 1)) {
                        fail();
                        break;
                    }
                    const uint32_t bar = smem_u32(&bar_b_full[s]);
                    mbar_arrive_expect_tx(bar, (uint32_t)D::B_STAGE);
                    tma_2d(bring + (uint32_t)s * D::B_STAGE, &maps.b, kt * TC_KS, row0, bar);
                }
            }
        }
        __syncwarp();
    } else if (warp >= 4 && warp < EPI0) {
        // ---------------- converters: one weight row per thread, alternate stages --------
        // group g = (warp - 4) / 4 decodes the stages of parity g (every item has an even number
        // of stages, so group g always fills A slot g); each thread decodes 64 K-elements of its
        // row per stage with two MMA stages of time for it
        static_assert(CW == 8 && NA == 2 && SUBS % 2 == 0, "two stage-parity groups of four warps");
        const int cq = warp - 4, r = (cq & 3) * 32 + lane, g = cq >> 2;
        int gk = 0, gj = 0;
        for (int item = blockIdx.x; item < n_items && !s_abort; item += gridDim.x) {
            bool ok = true;
            for (int kt = 0; kt < nk; kt++, gk++) {
                const int sub = kt % SUBS, s = gk % NA, jj = gj, rs = jj % RST;
                if (sub == SUBS - 1) gj++;  // both groups count every raw stage
                if ((kt & 1) != g) continue;
                if (s_abort) { ok = false; break; }
                if (sub == g && !mbar_wait(smem_u32(&bar_raw_full[rs]), (jj / RST) & 1)) { fail(); ok = false; break; }
                if (gk >= NA && !mbar_wait(smem_u32(&bar_a_empty[s]), ((gk / NA) + 1) & 1)) { fail(); ok = false; break; }
                const uint8_t* mat = raw_g + (size_t)rs * RS::BYTES;
                uint32_t v[32];
                if constexpr (TYPE == T_Q6_K) {  // K-permuted pairs: the h / x operand is stored to match
                    slice32_q6k_kperm<TC_M>(mat + r * PITCH, mat + RS::DOFF + r * 2, sub, 0, v);
                    slice32_q6k_kperm<TC_M>(mat + r * PITCH, mat + RS::DOFF + r * 2, sub, 1, v + 16);
                } else {
                    slice32<TYPE, TC_M>(mat + r * PITCH, mat + RS::DOFF + r * 2, mat + RS::AOFF + r * 4, sub, 0, v);
                    slice32<TYPE, TC_M>(mat + r * PITCH, mat + RS::DOFF + r * 2, mat + RS::AOFF + r * 4, sub, 1, v + 16);
                }
                if (sub == SUBS - 2 + g) {  // this group's last read of the raw slot
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&bar_raw_empty[rs]));
                }
                uint8_t* at = a_g + (size_t)s * D::A_STAGE + r * 128;
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4*>(at + ((c ^ (r & 7)) << 4)) =
                        make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bar_a_full[s]));
            }
            if (!ok) break;
        }
    } else if (warp >= EPI0) {
        // ---------------- epilogue ----------------
        pdl_wait();  // the row exponents below are gate/up's output
        const int q = warp & 3;
        const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
        int it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, it++) {
            // the four warps share named barrier 2, so they stop together: one thread samples the
            // abort flag between two barriers (the first also ends every read of the previous
            // item's staging chunks)
            if (warp == EPI0 && lane == 0) s_epi_stop = s_abort;
            asm volatile("bar.sync 2, 128;\n" ::: "memory");
            const bool stop = s_epi_stop;
            asm volatile("bar.sync 2, 128;\n" ::: "memory");
            if (stop) break;
            int e, row0, nrows, fb;
            info(item, e, row0, nrows, fb);
            const int acc = it & 1;
            // this warp writes tokens c * 32 + q * 8 + t (t < 8) of every chunk c; lane l holds
            // (token, scale) for chunk l / 8 (first) and l / 8 + 4 (second), t = l % 8
            int tok[2];
            float sc[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int n = ((lane >> 3) + 4 * h) * 32 + q * 8 + (lane & 7);
                tok[h] = 0;
                sc[h] = 0.0f;
                if (n < nrows) {
                    const int rr = row0 + n;
                    tok[h] = __ldg(p.row_tok + rr);
                    const int slot = __ldg(p.row_slot + rr);
                    const float w = p.y ? 1.0f : ((slot < p.k) ? __ldg(p.topk_w + (size_t)tok[h] * p.k + slot) : 1.0f);
                    sc[h] = __fmul_rn(w, exp2i(__ldg(p.rowexp + rr)));  // exact: 2^e
                }
            }
            const bool ok = mbar_wait(smem_u32(&bar_acc_full[acc]), (it / 2) & 1);
            if (!ok) fail();
            fence_after_sync();
            const int n_eff = (nrows + 15) & ~15;
            for (int c = 0; c * 32 < n_eff; c++) {
                uint32_t a[32];
                tmem_ld32(tlane + (uint32_t)(acc * TC_BN + c * 32), a);
                tmem_ld_wait();
                float* ys = ys_g + (D::YB == 2 ? (c & 1) * (D::YCH * D::YLD) : 0);
                if (D::YB == 1 && c > 0) asm volatile("bar.sync 2, 128;\n" ::: "memory");  // chunk c - 1 read
#pragma unroll
                for (int i = 0; i < 32; i++) ys[i * D::YLD + q * 32 + lane] = __uint_as_float(a[i]);
                asm volatile("bar.sync 2, 128;\n" ::: "memory");
                if (ok && !s_abort) {
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const int n = c * 32 + q * 8 + t;
                        const int src = (c & 3) * 8 + t;
                        const int tk = __shfl_sync(0xffffffffu, c < 4 ? tok[0] : tok[1], src);
                        const float scl = __shfl_sync(0xffffffffu, c < 4 ? sc[0] : sc[1], src);
                        if (n < nrows) {
                            float4 v = *reinterpret_cast<const float4*>(ys + (q * 8 + t) * D::YLD + 4 * lane);
                            v.x = __fmul_rn(v.x, scl); v.y = __fmul_rn(v.y, scl);
                            v.z = __fmul_rn(v.z, scl); v.w = __fmul_rn(v.w, scl);
                            const int f = fb * TC_M + 4 * lane;
                            if (p.y) *reinterpret_cast<float4*>(p.y + (size_t)(row0 + n) * p.H + f) = v;
                            else atomicAdd(reinterpret_cast<float4*>(p.out + (size_t)tk * p.H + f), v);
                        }
                    }
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        tmem_dealloc(tbase, 512);
    }
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

template <int TYPE>
static cudaError_t go_down(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    using D = DownGeom<TYPE>;
    auto k = tc_down_kernel<TYPE>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, D::SMEM);
    if (e != cudaSuccess) return e;
    const int items = max_tiles * (p.H / TC_M);
    return launch_pdl(k, dim3(std::min(items, sm_count())), dim3(D::THREADS), D::SMEM, s, p, maps);
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
    RMOE_TC_SWITCH(p.down.type, return go_down<TT>(p, maps, max_tiles, s))
}

}  // namespace rmoe
