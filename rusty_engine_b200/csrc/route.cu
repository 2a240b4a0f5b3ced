// route.cu -- router logits, top-k and dispatch (expert-sorted rows + GEMM tile list).
//
// Router logits, two modes.
//   * exact (RMOE_FLAG_EXACT_ROUTER): bit-identical to rusty-engine's moe::matvec
//     (src/moe.rs:271-277): each logit is a sequential f32 sum over H of w*x with separate
//     multiply and add roundings (Rust never contracts), accumulated in ascending k -- small
//     batches with one thread per (token, expert) chain fed by a cp.async ring, large batches
//     with a register-tiled product (32 tokens x 64 experts per CTA, 4 x 4 outputs per thread)
//     keeping that order for every output;
//   * fast (default): the same products summed with fused multiply-adds (small batches: a
//     warp per expert, K split over the lanes and folded by a shuffle tree; large batches: the
//     tiled product with FFMA).  Logits differ from the sequential sums by a few ulp, so a
//     top-k choice can differ only where two logits lie within that distance (the near-tie
//     exception of the parity contract).
// Top-k is rusty-engine's stable descending argsort (src/moe.rs:75-93): larger score first,
// equal scores by lower expert index; softmax over the chosen k (src/moe.rs:61-72) or the
// sigmoid renormalisation (src/moe.rs:97-117).
//
// Dispatch: the top-k kernel counts each CTA's picks per expert and the in-CTA rank of every
// pick in token order; a scan kernel (a CTA per expert) turns the counts into per-(CTA, expert)
// offsets, and its last CTA to finish (atomic ticket, no spin-wait) writes the expert offsets
// and the tile list; a scatter kernel then places every (token, slot) at offset + rank, so rows
// are in ascending token order inside each expert.  Batches of at most 64 tokens take a single
// launch for all of it (route_fused_small_kernel).
#include <algorithm>

#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace rmoe {

static constexpr int TK_TOK = 8;  // tokens per top-k CTA (C2 route: 4: 0.117 ms; 8: 0.111; 16: 0.118; 32: 0.143)
static constexpr int TK_THREADS = 256;

// ---------------------------------------------------------------------------------------
// logits, small batches (T <= 64): CTA = 16 experts x 8 tokens, one thread per logit.  Each
// logit is one sequential chain of H dependent adds, so the router's latency is that chain;
// everything else is kept off it: all 128 threads stream 256-element chunks of the 16 weight
// rows and 8 token rows into a 4-deep cp.async ring, and the chains read them from shared
// memory (rows padded to 1040 B, so the 16 rows a warp reads land in distinct banks).
// ---------------------------------------------------------------------------------------
static constexpr int LC_EB = 16, LC_TB = 8, LC_KC = 256, LC_ST = 4, LC_LD = LC_KC + 4, LC_THREADS = 128;
static constexpr int LC_SMEM = LC_ST * (LC_EB + LC_TB) * LC_LD * 4;

__device__ __forceinline__ void lc_cpa16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(LC_THREADS) logits_chain_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ w, int T, int H, int E,
                                                                   float* __restrict__ logits, __half* __restrict__ xb,
                                                                   unsigned* status) {
    extern __shared__ __align__(16) float lsm[];  // [LC_ST][LC_EB weight rows + LC_TB token rows][LC_LD]
    const int e0 = blockIdx.x * LC_EB, t0 = blockIdx.y * LC_TB;
    const int ne = min(LC_EB, E - e0), nt = min(LC_TB, T - t0);
    const int tid = threadIdx.x;
    const int nchunk = H / LC_KC;
    auto issue = [&](int c) {
        if (c < nchunk) {
            float* buf = lsm + (c % LC_ST) * (LC_EB + LC_TB) * LC_LD;
            for (int q = tid; q < (LC_EB + LC_TB) * (LC_KC / 4); q += LC_THREADS) {
                const int row = q / (LC_KC / 4), pc = q % (LC_KC / 4);
                const bool wrow = row < LC_EB;
                const int idx = wrow ? row : row - LC_EB;
                const bool live = idx < (wrow ? ne : nt);
                const float* src = wrow ? w + (size_t)(e0 + (live ? idx : 0)) * H : x + (size_t)(t0 + (live ? idx : 0)) * H;
                lc_cpa16(smem_u32(buf + row * LC_LD + pc * 4), src + (size_t)c * LC_KC + pc * 4, live ? 16u : 0u);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    for (int c = 0; c < LC_ST - 1; c++) issue(c);
    const int ce = tid % LC_EB, ct = tid / LC_EB;
    const bool chain = ce < ne && ct < nt;
    float s = 0.0f;
    for (int c = 0; c < nchunk; c++) {
        asm volatile("cp.async.wait_group %0;\n" ::"n"(LC_ST - 2) : "memory");
        __syncthreads();  // chunk c landed for everyone; chunk c - 1 fully read
        issue(c + LC_ST - 1);
        const float* buf = lsm + (c % LC_ST) * (LC_EB + LC_TB) * LC_LD;
        if (chain) {
            const float4* wr = reinterpret_cast<const float4*>(buf + ce * LC_LD);
            const float4* xr = reinterpret_cast<const float4*>(buf + (LC_EB + ct) * LC_LD);
#pragma unroll 16
            for (int i = 0; i < LC_KC / 4; i++) {
                const float4 a = wr[i], b = xr[i];
                s = __fadd_rn(s, __fmul_rn(a.x, b.x));
                s = __fadd_rn(s, __fmul_rn(a.y, b.y));
                s = __fadd_rn(s, __fmul_rn(a.z, b.z));
                s = __fadd_rn(s, __fmul_rn(a.w, b.w));
            }
        }
        if (xb && blockIdx.x == 0) {
            // fp16 MMA operand; |x| beyond the fp16 range is reported, never silently inf
            for (int q = tid; q < nt * (LC_KC / 4); q += LC_THREADS) {
                const int t = q / (LC_KC / 4), pc = q % (LC_KC / 4);
                const float4 v = *reinterpret_cast<const float4*>(buf + (LC_EB + t) * LC_LD + pc * 4);
                if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f && fabsf(v.w) <= 65504.f))
                    atomicOr(status, (unsigned)DERR_FP16_RANGE);
                *reinterpret_cast<uint2*>(xb + (size_t)(t0 + t) * H + (size_t)c * LC_KC + pc * 4) =
                    make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
            }
        }
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (chain) logits[(size_t)(t0 + ct) * E + e0 + ce] = s;
}

// ---------------------------------------------------------------------------------------
// logits, large batches: CTA = 32 tokens x 64 experts, 128 threads, 4 x 4 outputs each
// (thread (tx, ty) owns experts e0 + tx + 16j and tokens t0 + ty + 8i; the 16 weight rows a
// quarter-warp reads sit 144 B apart, so 16-B shared loads hit distinct banks), K tiles of 32
// in a 3-deep cp.async ring.  Small CTAs so that several share an SM: the sequential chains
// are latency-bound and want many warps.
// ---------------------------------------------------------------------------------------
static constexpr int LT_TOK = 32, LT_EXP = 64, LT_K = 32, LT_THREADS = 128, LT_LD = LT_K + 4, LT_ST = 3;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

template <bool EXACT>
__global__ void __launch_bounds__(LT_THREADS) logits_tiled_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ w, int T, int H, int E,
                                                                  float* __restrict__ logits, __half* __restrict__ xb,
                                                                  unsigned* status) {
    __shared__ __align__(16) float xs[LT_ST][LT_TOK][LT_LD];
    __shared__ __align__(16) float ws[LT_ST][LT_EXP][LT_LD];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * LT_TOK, e0 = blockIdx.y * LT_EXP;
    const int tx = tid & 15, ty = tid >> 4;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    const int nk = H / LT_K;
    auto issue = [&](int kt) {
        if (kt < nk) {
            const int buf = kt % LT_ST, k0 = kt * LT_K;
            for (int q = tid; q < LT_TOK * LT_K / 4; q += LT_THREADS) {
                const int r = q / (LT_K / 4), c = (q % (LT_K / 4)) * 4;
                cp_async16(&xs[buf][r][c], x + (size_t)min(t0 + r, T - 1) * H + k0 + c);
            }
            for (int q = tid; q < LT_EXP * LT_K / 4; q += LT_THREADS) {
                const int r = q / (LT_K / 4), c = (q % (LT_K / 4)) * 4;
                cp_async16(&ws[buf][r][c], w + (size_t)min(e0 + r, E - 1) * H + k0 + c);
            }
        }
        cp_async_commit();
    };
    for (int kt = 0; kt < LT_ST - 1; kt++) issue(kt);
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt % LT_ST;
        cp_async_wait<LT_ST - 2>();
        __syncthreads();  // tile kt landed for everyone; tile kt - 1 fully read
        issue(kt + LT_ST - 1);
        if (blockIdx.y == 0 && xb) {  // the fp16 copy of x (GEMM operand), once per token tile
            for (int q = tid; q < LT_TOK * LT_K / 4; q += LT_THREADS) {
                const int r = q / (LT_K / 4), c = (q % (LT_K / 4)) * 4;
                if (t0 + r < T) {
                    const float4 v = *reinterpret_cast<const float4*>(&xs[buf][r][c]);
                    if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f &&
                          fabsf(v.w) <= 65504.f))
                        atomicOr(status, (unsigned)DERR_FP16_RANGE);
                    *reinterpret_cast<uint2*>(xb + (size_t)(t0 + r) * H + kt * LT_K + c) =
                        make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
                }
            }
        }
#pragma unroll 2
        for (int kq = 0; kq < LT_K; kq += 4) {
            float4 xv[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) xv[i] = *reinterpret_cast<const float4*>(&xs[buf][ty + 8 * i][kq]);
#pragma unroll
            for (int j = 0; j < 4; j++) wv[j] = *reinterpret_cast<const float4*>(&ws[buf][tx + 16 * j][kq]);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float a = acc[i][j];
                    if (EXACT) {
                        a = __fadd_rn(a, __fmul_rn(wv[j].x, xv[i].x));
                        a = __fadd_rn(a, __fmul_rn(wv[j].y, xv[i].y));
                        a = __fadd_rn(a, __fmul_rn(wv[j].z, xv[i].z));
                        a = __fadd_rn(a, __fmul_rn(wv[j].w, xv[i].w));
                    } else {
                        a = fmaf(wv[j].x, xv[i].x, a);
                        a = fmaf(wv[j].y, xv[i].y, a);
                        a = fmaf(wv[j].z, xv[i].z, a);
                        a = fmaf(wv[j].w, xv[i].w, a);
                    }
                    acc[i][j] = a;
                }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int t = t0 + ty + 8 * i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int e = e0 + tx + 16 * j;
            if (e < E) logits[(size_t)t * E + e] = acc[i][j];
        }
    }
}

// ---------------------------------------------------------------------------------------
// logits, large batches, fast mode: an FFMA register-tiled product, CTA = 128 tokens x 128
// experts x one of LG_S K-splits (the batch's 4096 tokens give 32 token tiles, so splitting K
// fills the GPU), 256 threads with 8 x 8 outputs each (token rows ty*4 + {0..3} and 64 + ty*4 +
// {0..3}, experts tx*4 + {0..3} and 64 + tx*4 + {0..3}).  k-tiles of 16 are staged transposed in
// shared memory, the next tile's loads held in registers while the current one is multiplied.
// Each split writes its partial sums; the top-k kernel adds the splits in order.  The first
// expert tile also writes the fp16 copy of its tokens' K range.
// ---------------------------------------------------------------------------------------
static constexpr int LG_M = 128, LG_N = 128, LG_K = 16, LG_S = LOGIT_SPLITS, LG_THREADS = 256, LG_LD = LG_M + 4;

__global__ void __launch_bounds__(LG_THREADS, 2) logits_ffma_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ w, int T, int H, int E,
                                                                 float* __restrict__ part, __half* __restrict__ xb,
                                                                 unsigned* status) {
    __shared__ __align__(16) float xs[2][LG_K][LG_LD];
    __shared__ __align__(16) float wsm[2][LG_K][LG_LD];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const int t0 = blockIdx.x * LG_M, e0 = blockIdx.y * LG_N, sp = blockIdx.z;
    const int klen = H / LG_S, kbeg = sp * klen;
    // loader: rows lr and lr + 64 of the x and w tiles, k-quad lq of the 16-wide k-tile
    const int lr = tid >> 2, lq = tid & 3;
    const float* xr0 = x + (size_t)min(t0 + lr, T - 1) * H + kbeg + 4 * lq;
    const float* xr1 = x + (size_t)min(t0 + lr + 64, T - 1) * H + kbeg + 4 * lq;
    const float* wr0 = w + (size_t)min(e0 + lr, E - 1) * H + kbeg + 4 * lq;
    const float* wr1 = w + (size_t)min(e0 + lr + 64, E - 1) * H + kbeg + 4 * lq;
    const bool write_xb = xb && blockIdx.y == 0;
    float4 ra[4];
    auto load = [&](int kt) {
        const int ko = kt * LG_K;
        ra[0] = __ldg(reinterpret_cast<const float4*>(xr0 + ko));
        ra[1] = __ldg(reinterpret_cast<const float4*>(xr1 + ko));
        ra[2] = __ldg(reinterpret_cast<const float4*>(wr0 + ko));
        ra[3] = __ldg(reinterpret_cast<const float4*>(wr1 + ko));
    };
    auto store = [&](int buf, int kt) {
        const float* a0 = &ra[0].x;
        const float* a1 = &ra[1].x;
        const float* b0 = &ra[2].x;
        const float* b1 = &ra[3].x;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            xs[buf][4 * lq + i][lr] = a0[i];
            xs[buf][4 * lq + i][lr + 64] = a1[i];
            wsm[buf][4 * lq + i][lr] = b0[i];
            wsm[buf][4 * lq + i][lr + 64] = b1[i];
        }
        if (write_xb) {  // fp16 MMA operand; |x| beyond the fp16 range is reported, never silently inf
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float4 v = ra[h];
                const int t = t0 + lr + 64 * h;
                if (t < T) {
                    if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f &&
                          fabsf(v.w) <= 65504.f))
                        atomicOr(status, (unsigned)DERR_FP16_RANGE);
                    *reinterpret_cast<uint2*>(xb + (size_t)t * H + kbeg + kt * LG_K + 4 * lq) =
                        make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
                }
            }
        }
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
    const int nk = klen / LG_K;
    load(0);
    store(0, 0);
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load(kt + 1);
#pragma unroll
        for (int k = 0; k < LG_K; k++) {
            const float4 a0 = *reinterpret_cast<const float4*>(&xs[buf][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&xs[buf][k][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&wsm[buf][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&wsm[buf][k][64 + tx * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < nk) store(buf ^ 1, kt + 1);
        __syncthreads();
    }
    float* out = part + (size_t)sp * T * E;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int t = t0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (t >= T) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int e = e0 + h * 64 + tx * 4;
            float* o = out + (size_t)t * E + e;
            if (e + 3 < E && (E & 3) == 0) {
                *reinterpret_cast<float4*>(o) = make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (e + j < E) o[j] = acc[i][4 * h + j];
            }
        }
    }
}

// The router logits of token t into row[0 .. E) (shared memory), one warp: the logits as
// written, or the LG_S split partial sums added in split order (written back as the logits).
__device__ __forceinline__ void logit_row(const RouteParams& p, int t, int lane, float* row) {
    const int E = p.E;
    if (p.logits_part) {
        const size_t stride = (size_t)p.T * E;
        for (int e0 = 0; e0 < E; e0 += 128) {  // all loads of four columns in flight, then the sums
            float v[4][LG_S];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int e = e0 + 32 * u + lane;
#pragma unroll
                for (int sp = 0; sp < LG_S; sp++)
                    v[u][sp] = e < E ? __ldcg(p.logits_part + sp * stride + (size_t)t * E + e) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int e = e0 + 32 * u + lane;
                float sum = v[u][0];
#pragma unroll
                for (int sp = 1; sp < LG_S; sp++) sum = __fadd_rn(sum, v[u][sp]);
                if (e < E) {
                    row[e] = sum;
                    p.logits[(size_t)t * E + e] = sum;
                }
            }
        }
    } else {
        for (int e = lane; e < E; e += 32) row[e] = p.logits[(size_t)t * E + e];
    }
    __syncwarp();
}

// (top-k of one token and the near-tie refinement of the fast router: topk.cuh)

// ---------------------------------------------------------------------------------------
// top-k + counts (+ last-CTA scan and tile list)
// ---------------------------------------------------------------------------------------
// cta_cnt is expert-major, [E][ncp] with ncp = ncta rounded up to 16 (zero padding): CTA b's
// pick count for expert e at e * ncp + b; scan_counts_kernel turns every expert's run of counts
// into exclusive prefixes (rows before CTA b's first row of that expert), so a pick's row =
// expert_off[e] + cta_cnt[e * ncp + b] + local rank.
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
    }
    return v;
}

// Expert offsets and the tile list (expert, first row, rows) from the per-expert row counts
// cnt_s[0..NE) (NE = E + the shared expert), by every thread of the CTA (one per expert, a
// block-wide scan).  An expert's rows are split into the fewest tiles of <= tile_rows rows, of
// equal size rounded up to 16 (the MMA N granularity) except the last, so no tile is nearly
// empty.  Offsets also go to off_s when given.
__device__ void build_tiles(const RouteParams& p, const int* cnt_s, int* off_s) {
    __shared__ int s_w[2][32];  // per-warp totals, then exclusive offsets, of rows and tiles
    __shared__ int s_run[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nw = nthr >> 5;
    const int NE = p.E + (p.has_shared ? 1 : 0);
    if (tid == 0) s_run[0] = s_run[1] = 0;
    __syncthreads();
    for (int e0 = 0; e0 < NE; e0 += nthr) {
        const int e = e0 + tid;
        const int c = e < NE ? cnt_s[e] : 0;
        const int n0 = (c + p.tile_rows - 1) / p.tile_rows;
        const int tr = c ? min(p.tile_rows, ((c + n0 - 1) / n0 + 15) & ~15) : 1;
        const int nt = (c + tr - 1) / tr;
        const int ic = warp_incl_scan(c, lane), itl = warp_incl_scan(nt, lane);
        if (lane == 31) {
            s_w[0][warp] = ic;
            s_w[1][warp] = itl;
        }
        __syncthreads();
        if (warp == 0) {
            const int a = lane < nw ? s_w[0][lane] : 0, b = lane < nw ? s_w[1][lane] : 0;
            const int ia = warp_incl_scan(a, lane), ib = warp_incl_scan(b, lane);
            if (lane < nw) {
                s_w[0][lane] = ia - a;
                s_w[1][lane] = ib - b;
            }
        }
        __syncthreads();
        const int off = s_run[0] + s_w[0][warp] + ic - c, tb = s_run[1] + s_w[1][warp] + itl - nt;
        if (e < NE) {
            p.expert_off[e] = off;
            if (off_s) off_s[e] = off;
            for (int j = 0; j < nt; j++)
                if (tb + j < p.max_tiles) p.tiles[tb + j] = make_int4(e, off + j * tr, min(tr, c - j * tr), 0);
        }
        __syncthreads();  // s_run and s_w read by everyone
        if (tid == nthr - 1) {  // the running totals after this chunk
            s_run[0] = off + c;
            s_run[1] = tb + nt;
        }
        __syncthreads();
    }
    if (tid == 0) {
        const int run = s_run[0];
        int tiles = s_run[1];
        p.expert_off[NE] = run;
        if (off_s) off_s[NE] = run;
        *p.n_rows = run;
        if (tiles > p.max_tiles) {
            atomicOr(p.status, (unsigned)DERR_TILES_OVERFLOW);
            tiles = p.max_tiles;
        }
        *p.n_tiles = tiles;
    }
}

__global__ void __launch_bounds__(TK_THREADS) topk_count_kernel(RouteParams p) {
    extern __shared__ __align__(16) float tk_stage[];  // rescoring stage (p.stage_floats)
    __shared__ int ids_s[TK_TOK * MAX_K];
    __shared__ float row_s[TK_THREADS / 32][MAX_E];
    __shared__ AmbTok amb[TK_TOK];
    __shared__ int amb_list[TK_TOK], amb_n;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * TK_TOK;
    const int E = p.E, H = p.H, k = p.k;
    const int ntok = min(TK_TOK, p.T - t0);
    const int ncta = gridDim.x;
    const bool refine = !p.given && refine_on(p);
    if (tid == 0) amb_n = 0;
    __syncthreads();

    for (int tl = warp; tl < ntok; tl += TK_THREADS / 32) {
        int t = t0 + tl;
        if (p.given) {
            if (lane < k) ids_s[tl * k + lane] = p.topk_id[(size_t)t * k + lane];
            continue;
        }
        logit_row(p, t, lane, row_s[warp]);
        int id;
        if (!refine) {
            id = warp_topk(row_s[warp], E, k, p.gate, lane, p.topk_w + (size_t)t * k);
        } else if (!warp_topk_try(p, t, row_s[warp], lane, p.topk_w + (size_t)t * k, id, amb[tl])) {
            if (lane == 0) amb_list[atomicAdd(&amb_n, 1)] = tl;  // near-tie: rescored below
            __syncwarp();
            continue;
        }
        if (lane < k) {
            p.topk_id[(size_t)t * k + lane] = id;
            ids_s[tl * k + lane] = id;
        }
        __syncwarp();  // the row is read before the warp's next token overwrites it
    }
    __syncthreads();
    if (amb_n) {  // CTA-uniform
        cta_rescore_batch(p, amb, amb_list, amb_n, tk_stage, p.stage_floats, p.logits, 0, E);
        for (int i = warp; i < amb_n; i += TK_THREADS / 32) {
            const int tl = amb_list[i], t = t0 + tl;
            for (int e = lane; e < E; e += 32) row_s[warp][e] = p.logits[(size_t)t * E + e];
            __syncwarp();
            const int id = warp_topk(row_s[warp], E, k, p.gate, lane, p.topk_w + (size_t)t * k);
            if (lane < k) {
                p.topk_id[(size_t)t * k + lane] = id;
                ids_s[tl * k + lane] = id;
            }
            __syncwarp();
        }
        __syncthreads();
    }
    // zero the output rows this CTA owns when the combine accumulates with atomics (the x
    // gather kernel does it instead when it runs)
    if (p.out_zero && !p.xs) {
        for (int tl = 0; tl < ntok; tl++)
            for (int i = tid * 4; i < H; i += TK_THREADS * 4)
                *reinterpret_cast<float4*>(p.out_zero + (size_t)(t0 + tl) * H + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    // in-CTA rank of every pick in token order: one thread per expert scans the CTA's
    // TK_TOK * k picks in order
    const int ncp = route_cnt_stride(ncta);
    for (int e = tid; e < E; e += TK_THREADS) {
        int c = 0;
        for (int i = 0; i < ntok * k; i++)
            if (ids_s[i] == e) p.local_rank[(size_t)t0 * k + i] = c++;
        p.cta_cnt[(size_t)e * ncp + blockIdx.x] = c;
        if (blockIdx.x == 0)
            for (int b = ncta; b < ncp; b++) p.cta_cnt[(size_t)e * ncp + b] = 0;
    }
}

// Per-expert scan of the top-k CTAs' counts, one CTA per expert: cta_cnt[e][b] becomes the rows of
// expert e that come before CTA b's (token order), the expert's total goes to expert_off[e];
// the last CTA to finish (atomic ticket, no waiting) turns the totals into expert offsets and
// the tile list.
static constexpr int SC_THREADS = 256;
__global__ void __launch_bounds__(SC_THREADS) scan_counts_kernel(RouteParams p, int ncta) {
    __shared__ int warp_s[SC_THREADS / 32];
    __shared__ int cnt_s[MAX_E + 2];
    __shared__ unsigned ticket_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, e = blockIdx.x;
    const int ncp = route_cnt_stride(ncta);
    int* row = p.cta_cnt + (size_t)e * ncp;
    int run = 0;
    for (int b0 = 0; b0 < ncta; b0 += SC_THREADS) {
        const int b = b0 + tid;
        const int c = b < ncta ? __ldcg(row + b) : 0;
        const int incl = warp_incl_scan(c, lane);
        if (lane == 31) warp_s[warp] = incl;
        __syncthreads();
        int before = run;
        for (int w = 0; w < warp; w++) before += warp_s[w];
        if (b < ncta) row[b] = before + incl - c;
        int total = 0;
        for (int w = 0; w < SC_THREADS / 32; w++) total += warp_s[w];
        run += total;
        __syncthreads();
    }
    if (tid == 0) p.expert_off[e] = run;
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket_s = atomicAdd(p.ticket, 1u);
    __syncthreads();
    if (ticket_s != gridDim.x - 1) return;
    __threadfence();
    for (int i = tid; i < p.E; i += SC_THREADS) cnt_s[i] = __ldcg(p.expert_off + i);
    if (tid == 0 && p.has_shared) cnt_s[p.E] = p.shared_n;
    __syncthreads();
    build_tiles(p, cnt_s, nullptr);
    if (tid == 0) *p.ticket = 0u;  // re-arm for the next launch (stream-ordered)
}

// Place every (token, slot) at its expert-sorted row; CTA b handles the picks top-k CTA b made.
__global__ void __launch_bounds__(TK_THREADS) scatter_rows_kernel(RouteParams p) {
    const int t0 = blockIdx.x * TK_TOK, k = p.k, ncp = route_cnt_stride(gridDim.x);
    const int nent = min(TK_TOK, p.T - t0) * k;
    for (int i = threadIdx.x; i < nent; i += TK_THREADS) {
        int gi = t0 * k + i;
        int t = gi / k;
        const int e = p.topk_id[gi];
        if (e >= p.E) {  // empty pick (given routing)
            p.slot_row[gi] = -1;
            continue;
        }
        int pos = p.expert_off[e] + p.cta_cnt[(size_t)e * ncp + blockIdx.x] + p.local_rank[gi];
        p.row_tok[pos] = t;
        p.row_slot[pos] = gi - t * k;
        p.slot_row[gi] = pos;
        p.rowexp[pos] = -127;
    }
    if (p.has_shared) {
        const int base = p.expert_off[p.E] - p.shared_t0;
        for (int tl = threadIdx.x; tl < TK_TOK && t0 + tl < p.T; tl += TK_THREADS) {
            const int t = t0 + tl;
            if (t < p.shared_t0 || t >= p.shared_t0 + p.shared_n) continue;
            p.row_tok[base + t] = t;
            p.row_slot[base + t] = k;
            p.rowexp[base + t] = -127;
        }
    }
}

// Expert-sorted fp16 copy of x for the tensor-core path: one warp per token reads its fp16 row
// once (4 KB column chunks) and writes it to each of its rows (k picks + the shared expert);
// the same warp zeroes the token's output row for the atomic combine.
static constexpr int GX_CHUNK = 8;  // 16-B units per lane per chunk
__global__ void __launch_bounds__(256) gather_x_kernel(RouteParams p) {
    pdl_trigger();  // the gate/up kernel may take its SM slots; it waits for this grid's rows
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= p.T) return;
    const int k = p.k, per = k + (p.has_shared ? 1 : 0), units = p.H / 8;
    const int dst_row = lane < k ? p.slot_row[(size_t)t * k + lane] : 0;  // lane j < k: row of pick j
    const int shared_row =
        p.has_shared && t >= p.shared_t0 && t < p.shared_t0 + p.shared_n ? p.expert_off[p.E] + t - p.shared_t0 : -1;
    const uint4* src = reinterpret_cast<const uint4*>(p.xb + (size_t)t * p.H);
    for (int u0 = 0; u0 < units; u0 += 32 * GX_CHUNK) {
        uint4 v[GX_CHUNK];
#pragma unroll
        for (int c = 0; c < GX_CHUNK; c++) {
            const int u = u0 + 32 * c + lane;
            if (u < units) v[c] = src[u];
        }
        for (int j = 0; j < per; j++) {
            const int pos = j < k ? __shfl_sync(0xffffffffu, dst_row, j) : shared_row;
            if (pos < 0) continue;  // empty pick
            uint4* dst = reinterpret_cast<uint4*>(p.xs + (size_t)pos * p.H);
#pragma unroll
            for (int c = 0; c < GX_CHUNK; c++) {
                const int u = u0 + 32 * c + lane;
                if (u < units) dst[u] = v[c];
            }
        }
    }
    if (p.out_zero) {
        float4* o = reinterpret_cast<float4*>(p.out_zero + (size_t)t * p.H);
        for (int u = lane; u < p.H / 4; u += 32) o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// ---------------------------------------------------------------------------------------
// Whole dispatch for a small batch (T <= 64) in one CTA: top-k of every token, per-expert
// counts and token-order ranks, offsets and tiles, row placement -- all through shared memory.
// ---------------------------------------------------------------------------------------
static constexpr int RS_MAX_T = 64, RS_THREADS = 1024;

// Dispatch of a small batch inside one CTA, from the token-order picks ids_s[0 .. T k): per
// expert counts and the token-order rank of every pick (warps match the expert ids of 32-pick
// chunks; per-chunk counts are scanned over the chunks per expert), offsets and tiles, row
// placement.  scratch: [ceil(T k / 32)][E] chunk counts, then T k ranks.
__device__ void dispatch_small(const RouteParams& p, const int* ids_s, int* cnt_s, int* off_s, int* scratch) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarp = nthr >> 5;
    const int T = p.T, E = p.E, k = p.k, np = T * k, nch = (np + 31) / 32;
    int* ccnt = scratch;
    int* rank_s = scratch + nch * E;
    for (int q = tid; q < nch * E; q += nthr) ccnt[q] = 0;
    __syncthreads();
    for (int q = warp; q < nch; q += nwarp) {
        const int i = q * 32 + lane;
        const int id = i < np ? ids_s[i] : -1;
        const unsigned m = __match_any_sync(0xffffffffu, id);
        const int r = __popc(m & ((1u << lane) - 1u));
        if (i < np) {
            rank_s[i] = r;
            if (id < E && r == 0) ccnt[q * E + id] = __popc(m);  // ids >= E: empty picks (given routing)
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += nthr) {  // exclusive prefix over the chunks, in token order
        int run = 0;
        for (int q = 0; q < nch; q++) {
            const int c = ccnt[q * E + e];
            ccnt[q * E + e] = run;
            run += c;
        }
        cnt_s[e] = run;
    }
    if (tid == 0 && p.has_shared) cnt_s[E] = p.shared_n;
    __syncthreads();
    build_tiles(p, cnt_s, off_s);
    __syncthreads();
    for (int i = tid; i < np; i += nthr) {
        const int id = ids_s[i];
        if (id >= E) {  // empty pick (given routing)
            p.slot_row[i] = -1;
            continue;
        }
        const int t = i / k, pos = off_s[id] + ccnt[(i >> 5) * E + id] + rank_s[i];
        p.row_tok[pos] = t;
        p.row_slot[pos] = i - t * k;
        p.slot_row[i] = pos;
        p.rowexp[pos] = -127;
    }
    if (p.has_shared)
        for (int t = p.shared_t0 + tid; t < p.shared_t0 + p.shared_n; t += nthr) {
            const int pos = off_s[E] + t - p.shared_t0;
            p.row_tok[pos] = t;
            p.row_slot[pos] = k;
            p.rowexp[pos] = -127;
        }
}

// Dispatch of at most 64 picks (no shared expert, every expert's rows within one tile) by one
// warp, two picks per lane: a pick's expert-sorted row is its rank by (expert, pick index), and
// each touched expert is one tile, placed by the number of touched experts below it (short
// rolled loops over the picks, exchanged by shuffles).
static constexpr int DT_MAX = 64;
__device__ void dispatch_tiny(const RouteParams& p, const int* ids_s, int lane) {
    const int np = p.T * p.k;
    int id[2], pos[2] = {0, 0}, rows[2] = {0, 0};
    bool first[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int i = lane + 32 * h;
        id[h] = i < np ? ids_s[i] : 0x7fffffff;
        first[h] = i < np;
    }
    for (int j = 0; j < np; j++) {
        const int o = __shfl_sync(0xffffffffu, j < 32 ? id[0] : id[1], j & 31);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const bool before = j < lane + 32 * h;
            pos[h] += (o < id[h]) || (o == id[h] && before);
            rows[h] += o == id[h];
            if (o == id[h] && before) first[h] = false;
        }
    }
    const unsigned heads0 = __ballot_sync(0xffffffffu, first[0]), heads1 = __ballot_sync(0xffffffffu, first[1]);
    int below[2] = {0, 0};  // touched experts with a smaller id
    for (int j = 0; j < np; j++) {
        const int o = __shfl_sync(0xffffffffu, j < 32 ? id[0] : id[1], j & 31);
        const bool f = ((j < 32 ? heads0 : heads1) >> (j & 31)) & 1u;
#pragma unroll
        for (int h = 0; h < 2; h++) below[h] += f && o < id[h];
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int i = lane + 32 * h;
        if (i < np) {
            const int t = i / p.k;
            p.row_tok[pos[h]] = t;
            p.row_slot[pos[h]] = i - t * p.k;
            p.slot_row[i] = pos[h];
            p.rowexp[pos[h]] = -127;
            if (first[h]) p.tiles[below[h]] = make_int4(id[h], pos[h], rows[h], 0);
        }
    }
    if (lane == 0) {
        *p.n_rows = np;
        *p.n_tiles = __popc(heads0) + __popc(heads1);
    }
}

static size_t dispatch_small_scratch(int T, int E, int k) {
    const int np = T * k, nch = (np + 31) / 32;
    return ((size_t)nch * E + np) * 4;
}

__global__ void __launch_bounds__(RS_THREADS) route_small_kernel(RouteParams p) {
    extern __shared__ int rs_scratch[];
    __shared__ int ids_s[RS_MAX_T * MAX_K];
    __shared__ int cnt_s[MAX_E + 2], off_s[MAX_E + 2];
    pdl_trigger();  // the expert kernels may take their SM slots now; they wait for this grid
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = p.T, E = p.E, k = p.k, H = p.H;
    for (int t = warp; t < T; t += RS_THREADS / 32) {
        if (p.given) {
            if (lane < k) ids_s[t * k + lane] = p.topk_id[(size_t)t * k + lane];
            continue;
        }
        const int id = warp_topk(p.logits + (size_t)t * E, E, k, p.gate, lane, p.topk_w + (size_t)t * k);
        if (lane < k) {
            p.topk_id[(size_t)t * k + lane] = id;
            ids_s[t * k + lane] = id;
        }
    }
    if (p.out_zero && !p.xs)
        for (int i = tid * 4; i < T * H; i += RS_THREADS * 4)
            *reinterpret_cast<float4*>(p.out_zero + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    dispatch_small(p, ids_s, cnt_s, off_s, rs_scratch);
}

// ---------------------------------------------------------------------------------------
// Whole routing of a small batch in fast mode, one launch.  CTA (expert group, token group) =
// 8 / KQ experts x 8 tokens, a warp per (expert, K slice): the token rows are staged in shared
// memory (the first expert group also writes their fp16 copy and zeroes their output rows),
// every warp forms its slice's partial logits from FFMA sums folded by shuffles, and the
// slices are added in slice order.  Routing proper (KQ = 4: 2 experts per CTA) spreads the
// router rows and the shared-memory reads of x over E / 2 CTAs; the logits-only mode for
// mid-size batches (KQ = 1: 8 experts per CTA) keeps the x staging per CTA low.  The last CTA
// of each token group to finish (atomic ticket, no waiting) runs top-k for those tokens; the
// last of those runs the dispatch for the whole batch and resets the tickets.
// ---------------------------------------------------------------------------------------
static constexpr int RF_WARPS = 8, RF_TOK = 8, RF_THREADS = 32 * RF_WARPS;
static constexpr int RF_WCH = 16;  // float4 of the expert row each lane holds at a time
__host__ __device__ constexpr int rf_kq(int mode) { return mode == 0 ? 1 : 4; }

static int rf_stage_off(int E) { return (RF_TOK * E + 3) & ~3; }  // floats before the rescoring stage
static size_t route_fused_smem(int T, int H, int E, int k) {
    const size_t need = std::max(std::max((size_t)RF_TOK * H * 4, (size_t)RF_TOK * E * 4), dispatch_small_scratch(T, E, k));
    return std::max(need, (size_t)(rf_stage_off(E) + rescore_stage_floats(H)) * 4);
}

// A read-only 16-B load issued exactly once: the router rows are reused by every token of the
// group from registers, and a plain __ldg may be re-issued inside the token loop (to save
// registers), which puts a global-memory round trip in every iteration.
__device__ __forceinline__ float4 ldg_once(const float4* src) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];\n" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(src));
    return v;
}

template <int MODE>  // 0: logits (and the fp16 copy) only; 1: + top-k; 2: + the dispatch
__global__ void __launch_bounds__(RF_THREADS) route_fused_small_kernel(RouteParams p) {
    constexpr int KQ = rf_kq(MODE), NEXP = RF_WARPS / KQ, JS = 32 * KQ;  // JS: float4 stride of a lane
    extern __shared__ __align__(16) float fsm[];
    __shared__ int ids_s[RS_MAX_T * MAX_K];
    __shared__ int cnt_s[MAX_E + 2], off_s[MAX_E + 2];
    __shared__ float part_s[RF_WARPS][RF_TOK], pn_s[KQ][RF_TOK];
    __shared__ unsigned ticket_s;
    pdl_trigger();  // the expert kernels may take their SM slots now; they wait for this grid
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = p.T, H = p.H, E = p.E, k = p.k;
    const int t0 = blockIdx.y * RF_TOK, nt = min(RF_TOK, T - t0);
    const int n4 = H / 4;

    // 0. this warp's slice of its expert row (float4 kq * 32 + lane + JS u): the first RF_WCH
    //    per lane in flight before anything waits
    const int el = warp / KQ, kq = warp % KQ;
    const int e = blockIdx.x * NEXP + el;
    const float4* wr = reinterpret_cast<const float4*>(p.router_w + (size_t)min(e, E - 1) * H) + kq * 32 + lane;
    const int nj = (n4 - kq * 32 - lane + JS - 1) / JS;  // float4 of the slice this lane holds
    float4 wv[RF_WCH];
#pragma unroll
    for (int u = 0; u < RF_WCH; u++) wv[u] = u < nj ? ldg_once(wr + JS * u) : make_float4(0.f, 0.f, 0.f, 0.f);

    // 1. the token group's rows -> shared memory: 16-B asynchronous copies, every one in flight
    //    before any is waited for (a short rolled loop: this code runs once per launch, and
    //    straight-line code fetched once costs more than the copies themselves)
    float4* xs4 = reinterpret_cast<float4*>(fsm);
    const float4* xg = reinterpret_cast<const float4*>(p.x + (size_t)t0 * H);
    for (int q = tid; q < nt * n4; q += RF_THREADS)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(xs4 + q)), "l"(xg + q) : "memory");
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
    if (blockIdx.x == 0)  // fp16 MMA operand (|x| beyond the fp16 range is reported, never silently inf)
        for (int q = tid; q < nt * n4; q += RF_THREADS) {
            const float4 v = xs4[q];
            if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f && fabsf(v.w) <= 65504.f))
                atomicOr(p.status, (unsigned)DERR_FP16_RANGE);
            *reinterpret_cast<uint2*>(p.xb + (size_t)t0 * H + 4 * q) =
                make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
            if (MODE == 2 && p.out_zero)
                *reinterpret_cast<float4*>(p.out_zero + (size_t)t0 * H + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
        }

    // 2. logits: the lane's float4 of the slice against every token of the group; a slice of
    //    at most RF_WCH float4 per lane stays in registers and the token loop is rolled (four
    //    partial sums per lane, so the FMA chains are short), longer rows go in chunks of
    //    RF_WCH with the token sums carried in registers.  The first expert's warps also form
    //    ||x_t||^2 slice by slice for the near-tie window of the top-k step.
    const float4* xl = xs4 + kq * 32 + lane;
    if (e < E && nj <= RF_WCH) {
        for (int t = 0; t < nt; t++) {
            const float4* xr = xl + t * n4;
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll
            for (int u = 0; u < RF_WCH; u++)
                if (u < nj) {
                    const float4 a = wv[u], b = xr[JS * u];
                    s0 = fmaf(a.x, b.x, s0);
                    s1 = fmaf(a.y, b.y, s1);
                    s2 = fmaf(a.z, b.z, s2);
                    s3 = fmaf(a.w, b.w, s3);
                    if (el == 0) {
                        q0 = fmaf(b.x, b.x, fmaf(b.y, b.y, q0));
                        q1 = fmaf(b.z, b.z, fmaf(b.w, b.w, q1));
                    }
                }
            float v = (s0 + s1) + (s2 + s3), n2 = q0 + q1;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                v += __shfl_xor_sync(0xffffffffu, v, off);
                n2 += __shfl_xor_sync(0xffffffffu, n2, off);
            }
            if (lane == 0) {
                part_s[warp][t] = v;
                if (el == 0) pn_s[kq][t] = n2;
            }
        }
    } else if (e < E) {
        float acc[RF_TOK], nacc[RF_TOK];
#pragma unroll
        for (int t = 0; t < RF_TOK; t++) acc[t] = nacc[t] = 0.0f;
        for (int u0 = 0; u0 < nj; u0 += RF_WCH) {
            if (u0 > 0)
#pragma unroll
                for (int u = 0; u < RF_WCH; u++)
                    wv[u] = u0 + u < nj ? ldg_once(wr + JS * (u0 + u)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < RF_WCH; u++)
                if (u0 + u < nj)
#pragma unroll
                    for (int t = 0; t < RF_TOK; t++)
                        if (t < nt) {
                            const float4 a = wv[u], b = xl[t * n4 + JS * (u0 + u)];
                            acc[t] = fmaf(a.x, b.x, acc[t]);
                            acc[t] = fmaf(a.y, b.y, acc[t]);
                            acc[t] = fmaf(a.z, b.z, acc[t]);
                            acc[t] = fmaf(a.w, b.w, acc[t]);
                            if (el == 0) nacc[t] = fmaf(b.x, b.x, fmaf(b.y, b.y, fmaf(b.z, b.z, fmaf(b.w, b.w, nacc[t]))));
                        }
        }
#pragma unroll
        for (int t = 0; t < RF_TOK; t++)
            if (t < nt) {
                float v = acc[t], n2 = nacc[t];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    v += __shfl_xor_sync(0xffffffffu, v, off);
                    n2 += __shfl_xor_sync(0xffffffffu, n2, off);
                }
                if (lane == 0) {
                    part_s[warp][t] = v;
                    if (el == 0) pn_s[kq][t] = n2;
                }
            }
    }
    __syncthreads();
    __shared__ float xn2_s[RF_TOK];
    if (kq == 0 && e < E && lane < nt) {  // the slices in slice order
        float v = part_s[warp][lane];
#pragma unroll
        for (int q = 1; q < KQ; q++) v += part_s[warp + q][lane];
        p.logits[(size_t)(t0 + lane) * E + e] = v;
    }
    if (warp == 0 && lane < nt) {
        float n2 = pn_s[0][lane];
#pragma unroll
        for (int q = 1; q < KQ; q++) n2 += pn_s[q][lane];
        xn2_s[lane] = n2;
    }

    // 3. the token group's last CTA: top-k of its tokens
    if (MODE == 0) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket_s = atomicAdd(p.ticket + 1 + blockIdx.y, 1u);
    __syncthreads();
    if (ticket_s != gridDim.x - 1) return;
    __threadfence();
    if (tid == 0) p.ticket[1 + blockIdx.y] = 0u;  // every CTA of the group has taken its ticket
    float* lg = fsm;  // the group's logits, read past L1 (other CTAs wrote them)
    for (int q = tid; q < nt * E; q += RF_THREADS) lg[q] = __ldcg(p.logits + (size_t)t0 * E + q);
    __syncthreads();
    __shared__ AmbTok amb[RF_TOK];
    __shared__ int amb_list[RF_TOK], amb_n;
    if (tid == 0) amb_n = 0;
    __syncthreads();
    if (warp < nt) {
        const int t = t0 + warp;
        int id;
        bool done = true;
        if (!refine_on(p)) {
            id = warp_topk(lg + warp * E, E, k, p.gate, lane, p.topk_w + (size_t)t * k);
        } else if (!warp_topk_try(p, t, lg + warp * E, lane, p.topk_w + (size_t)t * k, id, amb[warp],
                                  sqrtf(xn2_s[warp]))) {
            done = false;
            if (lane == 0) amb_list[atomicAdd(&amb_n, 1)] = warp;  // near-tie: rescored below
        }
        if (done && lane < k) {
            p.topk_id[(size_t)t * k + lane] = id;
            ids_s[t * k + lane] = id;
        }
    }
    __syncthreads();
    if (amb_n) {  // CTA-uniform; the stage follows the group's logit rows, which it updates
        cta_rescore_batch(p, amb, amb_list, amb_n, fsm + ((RF_TOK * E + 3) & ~3), p.stage_floats, lg, t0, E);
        for (int i = warp; i < amb_n; i += RF_THREADS / 32) {
            const int w = amb_list[i], t = t0 + w;
            const int id = warp_topk(lg + w * E, E, k, p.gate, lane, p.topk_w + (size_t)t * k);
            if (lane < k) {
                p.topk_id[(size_t)t * k + lane] = id;
                ids_s[t * k + lane] = id;
            }
        }
        __syncthreads();
    }

    // 4. the last token group: dispatch of the whole batch (a single group is its own last)
    if (MODE == 1) return;
    if (gridDim.y > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) ticket_s = atomicAdd(p.ticket, 1u);
        __syncthreads();
        if (ticket_s != gridDim.y - 1) return;
        __threadfence();
        for (int i = tid; i < T * k; i += RF_THREADS) ids_s[i] = __ldcg(p.topk_id + i);
        if (tid == 0) p.ticket[0] = 0u;  // every token group has taken its ticket
    }
    __syncthreads();
    if (T * k <= DT_MAX && !p.has_shared && T <= p.tile_rows) {
        if (warp == 0) dispatch_tiny(p, ids_s, lane);
    } else {
        dispatch_small(p, ids_s, cnt_s, off_s, reinterpret_cast<int*>(fsm));
    }
}

static cudaError_t launch_route_fused(const RouteParams& p0, int mode, cudaStream_t s) {
    RouteParams p = p0;
    const size_t sm = mode == 0 ? (size_t)RF_TOK * p.H * 4 : route_fused_smem(p.T, p.H, p.E, p.k);
    p.stage_floats = (int)(sm / 4) - rf_stage_off(p.E);
    auto k = mode == 0 ? route_fused_small_kernel<0> : mode == 1 ? route_fused_small_kernel<1> : route_fused_small_kernel<2>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    const int nexp = RF_WARPS / rf_kq(mode);
    k<<<dim3((p.E + nexp - 1) / nexp, (p.T + RF_TOK - 1) / RF_TOK), RF_THREADS, sm, s>>>(p);
    return cudaGetLastError();
}

// Dynamic shared memory of a top-k kernel that may rescore near-ties (sets p.stage_floats).
template <typename K>
static cudaError_t rescore_smem(K kernel, RouteParams& p, size_t& sm) {
    sm = 0;
    p.stage_floats = 0;
    if (!refine_on(p) || p.given) return cudaSuccess;
    p.stage_floats = rescore_stage_floats(p.H);
    sm = (size_t)p.stage_floats * 4;
    // static + dynamic beyond 48 KB needs the opt-in, whatever the dynamic part alone is
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
}

int route_grid(int T) { return (T + TK_TOK - 1) / TK_TOK; }

// Batches from which the fast router's logits come from the K-split FFMA product (with fewer
// tokens its CTAs could not fill the GPU; the warp-per-expert kernel takes them).
static constexpr int LG_MIN_T = 1024;
static bool use_split(const RouteParams& p) { return !p.exact && p.logits_part && p.T >= LG_MIN_T; }

// Router logits (and the fp16 copy of x).  Exact: the chained per-logit kernel for small
// batches, the register-tiled one otherwise; fast: the warp-per-expert kernel below LG_MIN_T
// tokens, the K-split product above (on the tensor cores with split-fp32 operands where the
// shapes allow, else with FFMA; the register-tiled one when there is no partial-sum buffer).
static cudaError_t launch_logits(const RouteParams& p, cudaStream_t s) {
    if (!p.exact && p.T < LG_MIN_T) return launch_route_fused(p, 0, s);
    if (p.T <= RS_MAX_T) {
        cudaError_t e = cudaFuncSetAttribute(logits_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LC_SMEM);
        if (e != cudaSuccess) return e;
        dim3 grid((p.E + LC_EB - 1) / LC_EB, (p.T + LC_TB - 1) / LC_TB);
        logits_chain_kernel<<<grid, LC_THREADS, LC_SMEM, s>>>(p.x, p.router_w, p.T, p.H, p.E, p.logits, p.xb, p.status);
    } else if (use_split(p)) {
        if (logits_tc_supported(p)) return launch_logits_tc(p, s);
        dim3 grid((p.T + LG_M - 1) / LG_M, (p.E + LG_N - 1) / LG_N, LG_S);
        logits_ffma_kernel<<<grid, LG_THREADS, 0, s>>>(p.x, p.router_w, p.T, p.H, p.E, p.logits_part, p.xb, p.status);
    } else {
        dim3 grid((p.T + LT_TOK - 1) / LT_TOK, (p.E + LT_EXP - 1) / LT_EXP);
        if (p.exact)
            logits_tiled_kernel<true><<<grid, LT_THREADS, 0, s>>>(p.x, p.router_w, p.T, p.H, p.E, p.logits, p.xb, p.status);
        else
            logits_tiled_kernel<false><<<grid, LT_THREADS, 0, s>>>(p.x, p.router_w, p.T, p.H, p.E, p.logits, p.xb, p.status);
    }
    return cudaGetLastError();
}

__global__ void route_only_kernel(const float* logits, int T, int E, int k, int gate, int* ids, float* w);

// Top-k of every token's logits (one warp per token), summing the K-split partials first when
// the split product made them.
__global__ void __launch_bounds__(256) route_rows_kernel(RouteParams p) {
    extern __shared__ __align__(16) float rr_stage[];  // rescoring stage (p.stage_floats)
    __shared__ float row_s[8][MAX_E];
    __shared__ AmbTok amb[8];
    __shared__ int amb_list[8], amb_n;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t0 = blockIdx.x * 8, t = t0 + warp;
    if (threadIdx.x == 0) amb_n = 0;
    __syncthreads();
    if (t < p.T) {
        logit_row(p, t, lane, row_s[warp]);
        int id;
        bool done = true;
        if (!refine_on(p)) {
            id = warp_topk(row_s[warp], p.E, p.k, p.gate, lane, p.topk_w + (size_t)t * p.k);
        } else if (!warp_topk_try(p, t, row_s[warp], lane, p.topk_w + (size_t)t * p.k, id, amb[warp])) {
            done = false;
            if (lane == 0) amb_list[atomicAdd(&amb_n, 1)] = warp;  // near-tie: rescored below
        }
        if (done && lane < p.k) p.topk_id[(size_t)t * p.k + lane] = id;
    }
    __syncthreads();
    if (amb_n) {  // CTA-uniform; rows of row_s are this CTA's tokens, MAX_E apart
        cta_rescore_batch(p, amb, amb_list, amb_n, rr_stage, p.stage_floats, &row_s[0][0], t0, MAX_E);
        for (int i = warp; i < amb_n; i += 8) {
            const int w = amb_list[i], tt = t0 + w;
            const int id = warp_topk(row_s[w], p.E, p.k, p.gate, lane, p.topk_w + (size_t)tt * p.k);
            if (lane < p.k) p.topk_id[(size_t)tt * p.k + lane] = id;
        }
    }
}

cudaError_t launch_router_topk(const RouteParams& p0, cudaStream_t s) {
    if (p0.T > 0 && p0.T <= RS_MAX_T && !p0.exact) return launch_route_fused(p0, 1, s);
    RouteParams p = p0;
    if (!use_split(p)) p.logits_part = nullptr;
    cudaError_t e = launch_logits(p, s);
    if (e != cudaSuccess || p.T <= 0) return e;
    size_t sm;
    if ((e = rescore_smem(route_rows_kernel, p, sm)) != cudaSuccess) return e;
    route_rows_kernel<<<(p.T + 7) / 8, 256, sm, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_route_dispatch(const RouteParams& p0, cudaStream_t s) {
    cudaError_t e;
    RouteParams p = p0;
    if (!use_split(p)) p.logits_part = nullptr;  // the top-k kernel sums partials only after the K-split product
    if (p.T <= RS_MAX_T && !p.given && !p.exact) {
        // logits, top-k and dispatch in one launch
        if ((e = launch_route_fused(p, 2, s)) != cudaSuccess) return e;
    } else {
        if (!p.given && (e = launch_logits(p, s)) != cudaSuccess) return e;
        if (p.T <= RS_MAX_T) {
            const size_t sm = dispatch_small_scratch(p.T, p.E, p.k);
            if (sm > 48 * 1024 &&
                (e = cudaFuncSetAttribute(route_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm)) !=
                    cudaSuccess)
                return e;
            route_small_kernel<<<1, RS_THREADS, sm, s>>>(p);  // the whole dispatch in one CTA
        } else {
            size_t sm;
            if ((e = rescore_smem(topk_count_kernel, p, sm)) != cudaSuccess) return e;
            topk_count_kernel<<<route_grid(p.T), TK_THREADS, sm, s>>>(p);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            scan_counts_kernel<<<p.E, SC_THREADS, 0, s>>>(p, route_grid(p.T));
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            scatter_rows_kernel<<<route_grid(p.T), TK_THREADS, 0, s>>>(p);
        }
    }
    if ((e = cudaGetLastError()) != cudaSuccess || !p.xs) return e;
    gather_x_kernel<<<(p.T + 7) / 8, 256, 0, s>>>(p);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Group routing over precomputed logits (one warp per token): route_noaux_tc
// (src/moe.rs:192-268; noaux != 0) and route_group (src/moe.rs:127-190; noaux == 0).
//   scores s_i = sigmoid(logits_i + bias_i) (bias_i = 0 past the bias length);
//   contiguous groups, expert i in group i * ng / E; a group's score is the sum of its top-2
//   scores (noaux: updated in ascending expert order with the reference's >= / > rule) or of
//   all its scores (ascending f32 sum);
//   the top_k_group groups by a stable descending sort (ties to the lower group) are eligible
//   (all of them when top_k_group < 0);
//   the top k eligible experts by a stable descending sort, weights s / (sum of the picked s
//   in pick order); picks beyond the eligible experts get id 0xFFFFFFFF and weight 0.
// ---------------------------------------------------------------------------------------
static constexpr int RG_WARPS = 8;

template <int NS>  // NS >= ceil(E / 32)
__global__ void __launch_bounds__(RG_WARPS * 32) route_grouped_kernel(const float* __restrict__ logits,
                                                                      const float* __restrict__ bias, int nbias,
                                                                      int T, int E, int k, int ng, int tkg,
                                                                      int noaux, unsigned* ids, float* w) {
    __shared__ float s_sc[RG_WARPS][MAX_E];
    __shared__ float s_gs[RG_WARPS][RG_MAX_G];
    __shared__ unsigned char s_ok[RG_WARPS][RG_MAX_G];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = blockIdx.x * RG_WARPS + warp;
    if (t >= T) return;  // warp-uniform
    float* sc = s_sc[warp];
    for (int e = lane; e < E; e += 32) {
        const float x = logits[(size_t)t * E + e] + (e < nbias ? bias[e] : 0.0f);
        sc[e] = 1.0f / (1.0f + expf(-x));  // sigmoid, src/moe.rs:44-51
    }
    __syncwarp();
    for (int g = lane; g < ng; g += 32) {
        const int b = (g * E + ng - 1) / ng, en = ((g + 1) * E + ng - 1) / ng;  // i * ng / E == g
        float sum = 0.0f, t1 = -FLT_MAX, t2 = -FLT_MAX;
        for (int i = b; i < en; i++) {
            const float v = sc[i];
            if (noaux) {
                if (v >= t1) {
                    t2 = t1;
                    t1 = v;
                } else if (v > t2) {
                    t2 = v;
                }
            } else {
                sum = __fadd_rn(sum, v);
            }
        }
        s_gs[warp][g] = noaux ? __fadd_rn(t1, t2 == -FLT_MAX ? 0.0f : t2) : sum;
    }
    __syncwarp();
    for (int g = lane; g < ng; g += 32) {
        bool ok = true;
        if (tkg >= 0) {
            const float v = s_gs[warp][g];
            int rank = 0;
            for (int h = 0; h < ng; h++) {
                const float u = s_gs[warp][h];
                rank += (u > v || (u == v && h < g)) ? 1 : 0;
            }
            ok = rank < tkg;
        }
        s_ok[warp][g] = ok ? 1 : 0;
    }
    __syncwarp();
    unsigned key[NS];
#pragma unroll
    for (int q = 0; q < NS; q++) {
        const int e = lane + 32 * q;
        key[q] = (e < E && s_ok[warp][e * ng / E]) ? score_key(sc[e]) : 0u;
    }
    float chosen = 0.0f;
    int chosen_id = -1;
    for (int j = 0; j < k; j++) {
        unsigned bk = 0u;
        int bq = 0;
#pragma unroll
        for (int q = 0; q < NS; q++)
            if (key[q] > bk) {
                bk = key[q];
                bq = q;
            }
        const unsigned m = __reduce_max_sync(0xffffffffu, bk);
        if (m == 0u) break;  // no eligible expert left (warp-uniform)
        const int win = (int)__reduce_min_sync(0xffffffffu, bk == m ? (unsigned)(lane + 32 * bq) : 0xffffffffu);
        if ((win & 31) == lane)
#pragma unroll
            for (int q = 0; q < NS; q++)
                if (q == (win >> 5)) key[q] = 0u;
        if (lane == j) {
            chosen = key_score(m);
            chosen_id = win;
        }
    }
    float wsum = 0.0f;  // the picked scores summed in pick order, as the reference's iterator sum
    for (int j = 0; j < k; j++) {
        const float v = __shfl_sync(0xffffffffu, chosen, j);
        if (__shfl_sync(0xffffffffu, chosen_id, j) >= 0) wsum = __fadd_rn(wsum, v);
    }
    if (lane < k) {
        ids[(size_t)t * k + lane] = chosen_id >= 0 ? (unsigned)chosen_id : 0xffffffffu;
        w[(size_t)t * k + lane] = (chosen_id < 0 || wsum == 0.0f) ? 0.0f : __fdiv_rn(chosen, wsum);
    }
}

cudaError_t launch_route_grouped(const float* logits, const float* bias, int nbias, int T, int E, int k, int ng,
                                 int tkg, int noaux, unsigned* ids, float* w, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const dim3 grid((T + RG_WARPS - 1) / RG_WARPS), block(RG_WARPS * 32);
    const int ns = (E + 31) / 32;
    if (ns <= 4)
        route_grouped_kernel<4><<<grid, block, 0, s>>>(logits, bias, nbias, T, E, k, ng, tkg, noaux, ids, w);
    else
        route_grouped_kernel<MAX_E / 32><<<grid, block, 0, s>>>(logits, bias, nbias, T, E, k, ng, tkg, noaux, ids, w);
    return cudaGetLastError();
}

// route() over precomputed logits (one warp per token).
__global__ void route_only_kernel(const float* logits, int T, int E, int k, int gate, int* ids, float* w) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    int id = warp_topk(logits + (size_t)warp * E, E, k, gate, lane, w + (size_t)warp * k);
    if (lane < k) ids[(size_t)warp * k + lane] = id;
}

cudaError_t launch_route_only(const float* logits, int T, int E, int k, int gate, int* ids, float* w,
                              cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    route_only_kernel<<<(T + 7) / 8, 256, 0, s>>>(logits, T, E, k, gate, ids, w);
    return cudaGetLastError();
}

}  // namespace rmoe
