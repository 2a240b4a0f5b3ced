// grouped_small.cu -- grouped expert products for small per-expert row counts (decode).
//
// One CTA = one (tile of <= NT expert-sorted rows, block of 64 weight rows).  At decode sizes
// the layer is a weight stream: every touched expert's GGUF bytes are read once, so the kernel
// is built to keep that stream moving.  A ring of SB_RSTG raw stages (one 256-element
// superblock column of the CTA's 64 rows, all planes, plus the tile's token rows) is filled
// with cp.async while earlier stages are decoded; each landed stage is decoded to fp16 (the
// same half-slice decoders as the tensor-core kernels) into a 128-B-swizzled shared tile and
// four warps run mma.sync m16n8k16 (fp16 in, f32 accumulate) over it.  NT, the MMA width in
// tokens, is 8 or 16: a decode step touches a handful of rows per expert.
//
//   gate/up kernel: h[row, f] = silu(gate_f . x) * (up_f . x)      (src/moe.rs:280-299)
//                   stored as fp16 * 2^e with e per (row, 64-feature block), and the row's
//                   largest e folded into rowexp[row] (atomicMax)
//   down kernel:    y = down . h[row] with every h block brought to the row's common scale
//                   once it has landed; out[tok] += w_slot * y * 2^rowexp  (src/moe.rs:373-380)
#include "common.cuh"
#include "decode.cuh"
#include "kernels.h"

namespace rmoe {

static constexpr int SB_M = 64;          // weight rows per CTA (per matrix)
static constexpr int SB_THREADS = 256;   // 8 warps: all decode; warp w multiplies rows 16 (w & 3).., tokens 8 (w >> 2)..
static constexpr int SB_KS = 64;         // K elements per decoded sub-slice
static constexpr int SB_SMEM_MAX = 110 * 1024;  // two CTAs per SM

int small_tile_rows(int T) { return T <= 8 ? 8 : 16; }
int small_tile_rows_min() { return 8; }

__device__ __forceinline__ void cpa16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
// 16-B copy reading `bytes` (0 or 16) from src; the rest of the 16 B is zero-filled
__device__ __forceinline__ void cpa16_zfill(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <int TYPE, int NT, int NMAT>
struct SmallGeom {
    using R = Raw<TYPE>;
    using RS = RawStage<TYPE, SB_M>;
    static constexpr int SK = R::RK;                       // K elements per stage
    static constexpr int SUBS = SK / SB_KS;                // decoded sub-slices per stage
    static constexpr int A_WARP = NMAT * 16 * SB_KS * 2;   // a warp's decoded sub-slice (its 16 rows)
    static constexpr int B_BYTES = NT * SK * 2;            // token tile per stage
    static constexpr int STAGE = NMAT * RS::BYTES + B_BYTES;
    static constexpr int FIXED = 8 * A_WARP;
    // ring depth (even: the two K halves take a stage each): the deepest of 6 / 4 / 2 that keeps
    // two CTAs per SM
    static constexpr int RSTG = FIXED + 6 * STAGE <= SB_SMEM_MAX ? 6 : FIXED + 4 * STAGE <= SB_SMEM_MAX ? 4 : 2;
    static constexpr int RAW_OFF = 0;
    static constexpr int B_OFF = RSTG * NMAT * RS::BYTES;
    static constexpr int A_OFF = B_OFF + RSTG * B_BYTES;
    static constexpr int SMEM = A_OFF + FIXED;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(NT * (HBLK + 1) * 4 <= SMEM && 4 * 32 * NMAT * (NT / 2) * 4 <= SMEM, "epilogue staging");
    static_assert(B_OFF % 128 == 0 && A_OFF % 128 == 0, "alignment");
};

// byte offset of 16-B chunk c of row r in a [rows][SK] fp16 tile with the 128-B XOR swizzle
template <int SK>
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)(r * SK * 2 + ((c ^ (r & 7)) << 4));
}

// cp.async one raw stage j (256- or 128-element column) of the CTA's 64 rows of matrix M
template <int TYPE>
__device__ __forceinline__ void stage_raw(const DevMat& M, uint64_t grow0, int j, uint32_t dst, int tid) {
    using R = Raw<TYPE>;
    using RS = RawStage<TYPE, SB_M>;
    constexpr int PPR = R::MB / 16;  // 16-B pieces per row
    for (int q = tid; q < SB_M * PPR; q += SB_THREADS) {
        const int r = q / PPR, c = q - r * PPR;
        cpa16(dst + r * R::PITCH + c * 16, M.main + (grow0 + r) * M.main_stride + (uint64_t)j * R::MB + c * 16);
    }
    if (R::DBLK)
        for (int q = tid; q < R::DBLK * SB_M * 2 / 16; q += SB_THREADS) {
            const int b = q / (SB_M * 2 / 16), c = q % (SB_M * 2 / 16);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(M.dpl + ((uint64_t)j * R::DBLK + b) * M.trows + grow0);
            cpa16(dst + RS::DOFF + b * SB_M * 2 + c * 16, src + c * 16);
        }
    if (R::AUX)
        for (int q = tid; q < R::AUX * SB_M * 4 / 16; q += SB_THREADS) {
            const int b = q / (SB_M * 4 / 16), c = q % (SB_M * 4 / 16);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(M.aux + ((uint64_t)j * R::AUX + b) * M.trows + grow0);
            cpa16(dst + RS::AOFF + b * SB_M * 4 + c * 16, src + c * 16);
        }
}

// cp.async the stage-j columns of the tile's token rows (x by token for gate/up, h by row for
// down) into a swizzled [NT][SK] tile; rows past nrows are zero-filled.
template <int NT, int SK>
__device__ __forceinline__ void stage_b(const __half* base, const int* s_src, int width, int nrows, int j, uint32_t dst,
                                        int tid) {
    constexpr int CPR = SK / 8;
    for (int q = tid; q < NT * CPR; q += SB_THREADS) {
        const int n = q / CPR, c = q - n * CPR;
        const bool live = n < nrows;
        const __half* src = base + (live ? (size_t)s_src[n] * width + (size_t)j * SK + c * 8 : 0);
        cpa16_zfill(dst + swz<SK>(n, c), src, live ? 16u : 0u);
    }
}

// A warp decodes sub-slice `sub` (64 K-elements) of its 16 weight rows (rows 16 rg .. of the
// raw stage at `raw`) for NMAT matrices into its own fp16 tile at `at` ([NMAT][16][64], 128-B
// swizzle): lane l takes row l & 15, half l >> 4.
template <int TYPE, int NMAT>
__device__ __forceinline__ void decode_warp(const uint8_t* raw, int rg, int sub, uint8_t* at, int lane) {
    using R = Raw<TYPE>;
    using RS = RawStage<TYPE, SB_M>;
    const int row = lane & 15, half = lane >> 4, r = rg * 16 + row;
#pragma unroll
    for (int m = 0; m < NMAT; m++) {
        const uint8_t* rm = raw + m * RS::BYTES;
        uint32_t v[16];
        slice32<TYPE, SB_M>(rm + r * R::PITCH, rm + RS::DOFF + r * 2, rm + RS::AOFF + r * 4, sub, half, v);
        uint8_t* am = at + m * (16 * SB_KS * 2);
#pragma unroll
        for (int c = 0; c < 4; c++)
            *reinterpret_cast<uint4*>(am + swz<SB_KS>(row, half * 4 + c)) =
                make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
}

// A warp's MMAs over one decoded sub-slice for one matrix: acc[NT/8][4] += A(its 16 rows) x
// B(all NT tokens, K columns 64 sub.. of the stage's token tile)
template <int NT, int SK>
__device__ __forceinline__ void mma_warp(uint32_t a_base, uint32_t b_base, int sub, int lane, float (*acc)[4]) {
#pragma unroll
    for (int ks = 0; ks < SB_KS / 16; ks++) {
        uint32_t a[4];
        {
            const int mi = lane >> 3, r = (lane & 7) + (mi & 1) * 8, c = ks * 2 + (mi >> 1);
            ldmatrix_x4(a_base + swz<SB_KS>(r, c), a[0], a[1], a[2], a[3]);
        }
        if (NT == 8) {
            uint32_t b0, b1;
            const int n = lane & 7, c = sub * (SB_KS / 8) + ks * 2 + ((lane >> 3) & 1);
            ldmatrix_x2(b_base + swz<SK>(n, c), b0, b1);
            mma_f16_16816(acc[0], a, b0, b1);
        } else {
#pragma unroll
            for (int nt = 0; nt < NT / 16; nt++) {
                uint32_t b0, b1, b2, b3;
                const int mi = lane >> 3, n = nt * 16 + (lane & 7) + (mi >> 1) * 8;
                const int c = sub * (SB_KS / 8) + ks * 2 + (mi & 1);
                ldmatrix_x4(b_base + swz<SK>(n, c), b0, b1, b2, b3);
                mma_f16_16816(acc[nt * 2 + 0], a, b0, b1);
                mma_f16_16816(acc[nt * 2 + 1], a, b2, b3);
            }
        }
    }
}

// Multiply 8 packed fp16 values by 2^d (d <= 0), in f32, rounding back to fp16.
__device__ __forceinline__ uint4 scale_h8(uint4 v, int d) {
    if (d == 0) return v;
    if (d < -40) return make_uint4(0, 0, 0, 0);
    float s = exp2i(d);
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __half22float2(*reinterpret_cast<__half2*>(&w[i]));
        w[i] = pack_f16x2(__fmul_rn(f.x, s), __fmul_rn(f.y, s));
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// SwiGLU values hs[NT][64] (f32, smem) -> fp16 blocks with per-(row, block) exponent; rowexp
// gets the row maximum.
template <int NT>
__device__ __forceinline__ void store_h_block(const float* hs, int row0, int nrows, int fblk, const GroupedParams& p,
                                              int tid) {
    const int nblk = p.I / HBLK;
    // two threads per row, 32 features each
    for (int q = tid; q < NT * 2; q += SB_THREADS) {
        int n = q >> 1, half = q & 1;
        const float* src = hs + n * (HBLK + 1) + half * 32;
        float amax = 0.0f;
#pragma unroll 8
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        if (n < nrows) {
            int e = block_exp(amax);
            float s = exp2i(-e);
            size_t r = (size_t)(row0 + n);
            uint4* dst = reinterpret_cast<uint4*>(p.h + r * p.I + fblk * HBLK + half * 32);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float* v = src + j * 8;
                dst[j] = make_uint4(pack_f16x2(__fmul_rn(v[0], s), __fmul_rn(v[1], s)),
                                    pack_f16x2(__fmul_rn(v[2], s), __fmul_rn(v[3], s)),
                                    pack_f16x2(__fmul_rn(v[4], s), __fmul_rn(v[5], s)),
                                    pack_f16x2(__fmul_rn(v[6], s), __fmul_rn(v[7], s)));
            }
            if (half == 0) {
                p.hexp[r * nblk + fblk] = (int8_t)e;
                atomicMax(p.rowexp + r, e);
            }
        }
    }
}

template <int TYPE, int NT, int NMAT>
__global__ void __launch_bounds__(SB_THREADS, 2) small_kernel(GroupedParams p) {
    using G = SmallGeom<TYPE, NT, NMAT>;
    using RS = RawStage<TYPE, SB_M>;
    constexpr int SK = G::SK, RSTG = G::RSTG, SUBS = G::SUBS;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_src[NT], s_rexp[NT];
    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;
    const int4 ti = p.tiles[tile];
    const int e = ti.x, row0 = ti.y, nrows = ti.z;
    const bool sh = e >= p.E;
    const DevMat& M0 = NMAT == 2 ? (sh ? p.sgate : p.gate) : (sh ? p.sdown : p.down);
    const DevMat& M1 = NMAT == 2 ? (sh ? p.sup : p.up) : M0;
    const uint64_t grow0 = (uint64_t)(sh ? 0 : e) * M0.rows + (uint64_t)blockIdx.x * SB_M;
    const int K = NMAT == 2 ? p.H : p.I;
    const int nst = K / SK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rg = warp & 3, kh = warp >> 2;  // rows 16 rg .. 16 rg + 15; stages of parity kh
    const uint32_t sbase = smem_u32(smem);
    uint8_t* a_mine = smem + G::A_OFF + warp * G::A_WARP;

    for (int n = tid; n < NT; n += SB_THREADS) {
        const bool live = n < nrows;
        s_src[n] = NMAT == 2 ? (live ? __ldg(p.row_tok + row0 + n) : 0) : row0 + n;
        s_rexp[n] = (NMAT == 1 && live) ? __ldg(p.rowexp + row0 + n) : 0;
    }
    __syncthreads();
    const __half* bsrc = NMAT == 2 ? p.xb : p.h;
    const int bwidth = NMAT == 2 ? p.H : p.I;

    auto issue = [&](int j) {
        if (j < nst) {
            const int slot = j % RSTG;
            const uint32_t raw = sbase + G::RAW_OFF + slot * NMAT * RS::BYTES;
            stage_raw<TYPE>(M0, grow0, j, raw, tid);
            if (NMAT == 2) stage_raw<TYPE>(M1, grow0, j, raw + RS::BYTES, tid);
            stage_b<NT, SK>(bsrc, s_src, bwidth, nrows, j, sbase + G::B_OFF + slot * G::B_BYTES, tid);
        }
        cpa_commit();  // one group per stage (possibly empty), so the wait count stays fixed
    };

    float acc[NMAT][NT / 8][4];
#pragma unroll
    for (int m = 0; m < NMAT; m++)
#pragma unroll
        for (int i = 0; i < NT / 8; i++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[m][i][q] = 0.0f;

    // stages are taken in pairs, the even one by warps 0-3, the odd one by warps 4-7; inside a
    // stage every warp decodes and multiplies its own 16 rows (no CTA barrier)
    for (int j = 0; j < RSTG; j++) issue(j);
    for (int j0 = 0; j0 < nst; j0 += 2) {
        cpa_wait<RSTG - 2>();  // this thread's copies of stages j0, j0 + 1 have landed
        __syncthreads();       // ... everyone's
        if (NMAT == 1) {
            // h blocks to the row's common scale (exact power-of-two multiplies)
            const int nblk = p.I / HBLK;
            for (int q = tid; q < 2 * nrows * (SK / 8); q += SB_THREADS) {
                const int jj = j0 + q / (nrows * (SK / 8)), rem = q % (nrows * (SK / 8));
                const int n = rem / (SK / 8), c = rem - n * (SK / 8);
                if (jj >= nst) continue;
                const int blk = (jj * SK + c * 8) / HBLK;
                const int d = (int)__ldg(p.hexp + (size_t)(row0 + n) * nblk + blk) - s_rexp[n];
                uint4* ptr = reinterpret_cast<uint4*>(smem + G::B_OFF + (jj % RSTG) * G::B_BYTES + swz<SK>(n, c));
                *ptr = scale_h8(*ptr, d);
            }
            __syncthreads();
        }
        const int j = j0 + kh;
        if (j < nst) {
            const int slot = j % RSTG;
            const uint8_t* raw = smem + G::RAW_OFF + slot * NMAT * RS::BYTES;
            const uint32_t bt = sbase + G::B_OFF + slot * G::B_BYTES;
#pragma unroll 1
            for (int sub = 0; sub < SUBS; sub++) {
                decode_warp<TYPE, NMAT>(raw, rg, sub, a_mine, lane);
                __syncwarp();
#pragma unroll
                for (int m = 0; m < NMAT; m++)
                    mma_warp<NT, SK>(smem_u32(a_mine) + m * (16 * SB_KS * 2), bt, sub, lane, acc[m]);
                __syncwarp();  // the tile is read before the next sub-slice overwrites it
            }
        }
        __syncthreads();  // both stages consumed: their slots take the next pair
        issue(j0 + RSTG);
        issue(j0 + RSTG + 1);
    }
    cpa_wait<0>();
    __syncthreads();

    // the two K halves: warps 4-7 hand their sums to warps 0-3 (added in that fixed order)
    float* red = reinterpret_cast<float*>(smem);
    constexpr int PER = NMAT * (NT / 8) * 4;
    if (kh == 1) {
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int i = 0; i < NT / 8; i++)
#pragma unroll
                for (int q = 0; q < 4; q++) red[((rg * 32 + lane) * PER) + (m * (NT / 8) + i) * 4 + q] = acc[m][i][q];
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
        for (int m = 0; m < NMAT; m++)
#pragma unroll
            for (int i = 0; i < NT / 8; i++)
#pragma unroll
                for (int q = 0; q < 4; q++)
                    acc[m][i][q] = __fadd_rn(acc[m][i][q], red[((rg * 32 + lane) * PER) + (m * (NT / 8) + i) * 4 + q]);
    }
    __syncthreads();  // the reduction buffer is free for the epilogue staging

    const int g = lane >> 2, tq = lane & 3;
    if (NMAT == 2) {
        // SwiGLU in f32 (silu(g) * u, src/moe.rs:280-283) into smem hs[n][f]
        float* hs = reinterpret_cast<float*>(smem);
        if (kh == 0)
#pragma unroll
            for (int i = 0; i < NT / 8; i++)
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int n = i * 8 + tq * 2 + (q & 1);
                    const int f = rg * 16 + g + (q >> 1) * 8;
                    hs[n * (HBLK + 1) + f] = silu_ref(acc[0][i][q]) * acc[NMAT - 1][i][q];
                }
        __syncthreads();
        store_h_block<NT>(hs, row0, nrows, blockIdx.x, p, tid);
    } else if (kh == 0) {
        const int f0 = blockIdx.x * SB_M + rg * 16 + g;
#pragma unroll
        for (int i = 0; i < NT / 8; i++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int n = i * 8 + tq * 2 + (q & 1);
                const int f = f0 + (q >> 1) * 8;
                if (n < nrows) {
                    const int r = row0 + n;
                    const float yv = __fmul_rn(acc[0][i][q], exp2i(s_rexp[n]));
                    if (p.y) {
                        p.y[(size_t)r * p.H + f] = yv;
                    } else {
                        const int tok = __ldg(p.row_tok + r), slot = __ldg(p.row_slot + r);
                        const float w = (slot < p.k) ? __ldg(p.topk_w + (size_t)tok * p.k + slot) : 1.0f;
                        atomicAdd(p.out + (size_t)tok * p.H + f, __fmul_rn(w, yv));
                    }
                }
            }
    }
}

template <int TYPE, int NT, int NMAT>
static cudaError_t go_small(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    using G = SmallGeom<TYPE, NT, NMAT>;
    auto k = small_kernel<TYPE, NT, NMAT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((NMAT == 2 ? p.I : p.H) / SB_M, max_tiles);
    k<<<grid, SB_THREADS, G::SMEM, s>>>(p);
    return cudaGetLastError();
}

template <int NMAT>
static cudaError_t go_small_nt(int type, const GroupedParams& p, int max_tiles, int nt, cudaStream_t s) {
#define RMOE_SMALL_NT(TT)                                                      \
    return nt == 8 ? go_small<TT, 8, NMAT>(p, max_tiles, s) : go_small<TT, 16, NMAT>(p, max_tiles, s)
    switch (type) {
        case T_Q4_0: RMOE_SMALL_NT(T_Q4_0);
        case T_Q5_0: RMOE_SMALL_NT(T_Q5_0);
        case T_Q8_0: RMOE_SMALL_NT(T_Q8_0);
        case T_Q4_K: RMOE_SMALL_NT(T_Q4_K);
        case T_Q5_K: RMOE_SMALL_NT(T_Q5_K);
        case T_Q6_K: RMOE_SMALL_NT(T_Q6_K);
        case T_DENSE: RMOE_SMALL_NT(T_DENSE);
        default: return cudaErrorInvalidValue;
    }
#undef RMOE_SMALL_NT
}

cudaError_t launch_small_gateup(const GroupedParams& p, int max_tiles, int nt, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    return go_small_nt<2>(p.gate.type, p, max_tiles, nt, s);
}

cudaError_t launch_small_down(const GroupedParams& p, int max_tiles, int nt, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    return go_small_nt<1>(p.down.type, p, max_tiles, nt, s);
}

}  // namespace rmoe
