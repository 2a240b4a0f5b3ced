// logits_tc.cu -- router logits of large batches on the tensor cores (tcgen05 kind::tf32),
// fast router mode:
//
//   logits[t, e] = sum_k x[t, k] * w[e, k]          (moe::matvec, src/moe.rs:271-277)
//
// Each fp32 operand a is split into a_hi = a with its 13 low mantissa bits cleared (exactly a
// tf32 value) and a_lo = a - a_hi (exact in fp32), and
//
//   x . w  ~=  x_hi . w_hi + x_hi . w_lo + x_lo . w_hi
//
// The dropped x_lo . w_lo term and the tf32 reading of the lo parts are below 2^-21 of each
// product.  The tensor cores' f32 accumulation rounds every MMA's sum into the accumulator
// toward zero (measured on B200: a 256-deep K chain of such adds drifts by ~1e-5, above the
// sequential f32 sums' own error), so the chains are kept short: per 32-element K stage the
// four x_hi . w_hi MMAs go afresh into one accumulator and the eight small cross-term MMAs into
// another (their rounding is 2^-10 smaller), double-buffered across stages, and four fold
// warps add each stage's two sums into per-token f32 registers with round-to-nearest, in stage
// order.  The router's w_hi / w_lo are split once when the layer is created; x is split in
// shared memory.
//
// CTA = 128 tokens x all E (<= 128) experts x one of LT_S K-splits; the split partial sums go
// to part[split][t][e] and the top-k kernel adds them in split order, exactly as for the FFMA
// product.  The CTA also writes its tokens' K range of the fp16 copy of x (the expert GEMMs' B
// operand), with the fp16 range check.
//   warp 0       TMA producer: per 32-element K stage, the 128 x rows and the E rows of w_hi
//                and w_lo, 128-B swizzled (rows past T read zeros);
//   warp 1       allocates tensor memory, issues 3 x 4 tcgen05.mma (M 128, N E, K 8) per stage
//                into the accumulator pair (stage & 1);
//   warps 4-7    split x in place into x_hi and a second tile x_lo, write x's fp16 copy;
//   warps 8-11   fold each stage's accumulator into the token's running sums (lane = token),
//                then write the partial-sum row.
// Every wait is bounded (1 s): on a timeout the kernel records DERR_TIMEOUT and winds down.
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rmoe {
using namespace tc;

static constexpr int LT_M = 128;   // tokens per CTA (MMA M, TMEM lanes)
static constexpr int LT_KS = 32;   // fp32 K elements per stage: one 128-B swizzle row
static constexpr int LT_S = LOGIT_SPLITS;  // K-splits: the partial-sum planes of logits_part
static constexpr int LT_THREADS = 384;
static constexpr int LT_MAX_E = 128;  // the fold warps hold E running sums per token in registers
static constexpr int LT_LIM = 232448 - 4096;

static constexpr int lt_stage_bytes(int E) { return 2 * LT_M * 128 + 2 * E * 128; }
static int lt_stages(int E) { return 3 * lt_stage_bytes(E) + 1024 <= LT_LIM ? 3 : 2; }  // 3 for E <= 128

struct LtMaps {
    CUtensorMap x, wh, wl;
};

// Instruction descriptor, kind::tf32: tf32 A and B, f32 accumulator, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4)                      // D format f32
           | (2u << 7) | (2u << 10)       // A, B format tf32
           | ((uint32_t)(N >> 3) << 17)   // N >> 3
           | ((uint32_t)(M >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void lt_tma(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ float tf32_hi(float a) { return __uint_as_float(__float_as_uint(a) & 0xffffe000u); }

__global__ void __launch_bounds__(LT_THREADS, 1)
    logits_tc_kernel(const __grid_constant__ LtMaps maps, int T, int H, int E, int NS, float* __restrict__ part,
                     __half* __restrict__ xb, unsigned* status) {
    extern __shared__ uint8_t dsmem[];
    __shared__ __align__(8) uint64_t bar_full[3], bar_conv[3], bar_empty[3];
    __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2], bar_fin;
    __shared__ uint32_t tmem_holder;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * LT_M, sp = blockIdx.y;
    const int klen = H / LT_S, kbeg = sp * klen, nst = klen / LT_KS;
    const int SB = lt_stage_bytes(E), XB = LT_M * 128, WB = E * 128;
    const uint32_t sbase = (smem_u32(dsmem) + 1023u) & ~1023u;  // 1024-B aligned (SW128 atoms)
    uint8_t* gbase = dsmem + (sbase - smem_u32(dsmem));
    // stage s at sbase + s * SB: [x (x_hi once split) | x_lo | w_hi | w_lo]
    // tensor memory: accumulator pair a at columns 2aE (x_hi . w_hi) and 2aE + E (cross terms)
    uint32_t ncols = 32;
    while (ncols < 4u * (uint32_t)E) ncols <<= 1;

    if (tid == 0) {
        for (int i = 0; i < NS; i++) {
            mbar_init(smem_u32(&bar_full[i]), 1);
            mbar_init(smem_u32(&bar_conv[i]), 4);
            mbar_init(smem_u32(&bar_empty[i]), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&bar_acc_full[i]), 1);
            mbar_init(smem_u32(&bar_acc_empty[i]), 4);
        }
        mbar_init(smem_u32(&bar_fin), 1);
        s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_holder), ncols);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tbase = tmem_holder;
    auto fail = [&]() {
        s_abort = 1;
        atomicOr(status, (unsigned)DERR_TIMEOUT);
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (int st = 0; st < nst; st++) {
                const int s = st % NS;
                if (s_abort) break;
                if (st >= NS && !mbar_wait(smem_u32(&bar_empty[s]), ((st / NS) + 1) & 1)) {
                    fail();
                    break;
                }
                const uint32_t bar = smem_u32(&bar_full[s]), dst = sbase + (uint32_t)(s * SB);
                const int kx = kbeg + st * LT_KS;  // a multiple of 32 elements: 128-B aligned
                mbar_arrive_expect_tx(bar, (uint32_t)(XB + 2 * WB));
                lt_tma(dst, &maps.x, kx, t0, bar);
                lt_tma(dst + 2 * XB, &maps.wh, kx, 0, bar);
                lt_tma(dst + 2 * XB + WB, &maps.wl, kx, 0, bar);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32(LT_M, E);
            for (int st = 0; st < nst; st++) {
                const int s = st % NS, a = st & 1;
                if (s_abort) break;
                if (!mbar_wait(smem_u32(&bar_full[s]), (st / NS) & 1) ||
                    !mbar_wait(smem_u32(&bar_conv[s]), (st / NS) & 1) ||
                    (st >= 2 && !mbar_wait(smem_u32(&bar_acc_empty[a]), ((st / 2) + 1) & 1))) {
                    fail();
                    break;
                }
                fence_after_sync();
                const uint32_t xh = sbase + (uint32_t)(s * SB), xl = xh + XB, wh = xl + XB, wl = wh + WB;
                const uint32_t dh = tbase + (uint32_t)(2 * a * E), dx = dh + (uint32_t)E;
#pragma unroll
                for (int kk = 0; kk < LT_KS / 8; kk++) {
                    const uint32_t o = (uint32_t)kk * 32;  // 8 fp32 = 32 B per K step
                    mma_tf32(dh, smem_desc_sw128(xh + o), smem_desc_sw128(wh + o), idesc, kk != 0);
                    mma_tf32(dx, smem_desc_sw128(xh + o), smem_desc_sw128(wl + o), idesc, kk != 0);
                    mma_tf32(dx, smem_desc_sw128(xl + o), smem_desc_sw128(wh + o), idesc, 1);
                }
                mma_commit(smem_u32(&bar_empty[s]));
                mma_commit(smem_u32(&bar_acc_full[a]));
            }
            mma_commit(smem_u32(&bar_fin));  // every MMA this thread issued has finished when it fires
            if (!mbar_wait(smem_u32(&bar_fin), 0)) fail();
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ---------------- x split + fp16 copy ----------------
        // A warp takes 4 rows x 8 16-B chunks per step (512 contiguous bytes: no bank conflicts).
        // Physical chunk pc of row r holds K elements 4 (pc ^ (r & 7)) .. +3 of the stage (SW128).
        const int cw = warp - 4, pc = lane & 7;
        for (int st = 0; st < nst; st++) {
            const int s = st % NS;
            if (s_abort) break;
            if (!mbar_wait(smem_u32(&bar_full[s]), (st / NS) & 1)) {
                fail();
                break;
            }
            uint8_t* xs = gbase + (size_t)s * SB;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = cw * 32 + i * 4 + (lane >> 3);
                float4* ph = reinterpret_cast<float4*>(xs + r * 128 + pc * 16);
                float4* pl = reinterpret_cast<float4*>(xs + XB + r * 128 + pc * 16);
                const float4 v = *ph;
                const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                *ph = h;
                *pl = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
                const int t = t0 + r;
                if (xb && t < T) {  // fp16 MMA operand; |x| beyond the fp16 range is reported
                    if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f &&
                          fabsf(v.w) <= 65504.f))
                        atomicOr(status, (unsigned)DERR_FP16_RANGE);
                    const int k = kbeg + st * LT_KS + 4 * (pc ^ (r & 7));
                    *reinterpret_cast<uint2*>(xb + (size_t)t * H + k) =
                        make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
                }
            }
            fence_proxy_async_smem();  // generic-proxy writes -> the MMA's async-proxy reads
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_conv[s]));
        }
    } else if (warp >= 8) {
        // ---------------- fold: stage accumulators -> running sums -> partial sums ----------------
        const int q = warp & 3, t = t0 + q * 32 + lane;
        const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
        float sum[LT_MAX_E / 32][32];
#pragma unroll
        for (int c = 0; c < LT_MAX_E / 32; c++)
#pragma unroll
            for (int i = 0; i < 32; i++) sum[c][i] = 0.0f;
        bool ok = true;
        for (int st = 0; st < nst; st++) {
            const int a = st & 1;
            if (s_abort || !mbar_wait(smem_u32(&bar_acc_full[a]), (st / 2) & 1)) {
                if (!s_abort) fail();
                ok = false;
                break;
            }
            fence_after_sync();
#pragma unroll
            for (int c = 0; c < LT_MAX_E / 32; c++) {
                if (c * 32 < E) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {  // the stage's x_hi . w_hi sum, then its cross terms
                        uint32_t v[32];
                        tmem_ld32(tlane + (uint32_t)((2 * a + h) * E + c * 32), v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) sum[c][i] = __fadd_rn(sum[c][i], __uint_as_float(v[i]));
                    }
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[a]));
        }
        if (ok && t < T) {
            float* out = part + (size_t)sp * T * E + (size_t)t * E;
#pragma unroll
            for (int c = 0; c < LT_MAX_E / 32; c++)
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (c * 32 + 4 * j < E)
                        *reinterpret_cast<float4*>(out + c * 32 + 4 * j) =
                            make_float4(sum[c][4 * j], sum[c][4 * j + 1], sum[c][4 * j + 2], sum[c][4 * j + 3]);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        tmem_dealloc(tbase, ncols);
    }
}

bool logits_tc_supported(const RouteParams& p) {
    return p.router_wh && p.router_wl && p.logits_part && p.E >= 16 && p.E <= LT_MAX_E && p.E % 16 == 0 &&
           p.H % (LT_S * LT_KS) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && p.T > 0;
}

cudaError_t launch_logits_tc(const RouteParams& p, cudaStream_t s) {
    if (!logits_tc_supported(p)) return cudaErrorNotSupported;
    LtMaps m;
    memset(&m, 0, sizeof m);
    if (!make_f32_rows_map(p.x, (uint64_t)p.T, (uint32_t)p.H, LT_KS, LT_M, m.x) ||
        !make_f32_rows_map(p.router_wh, (uint64_t)p.E, (uint32_t)p.H, LT_KS, (uint32_t)p.E, m.wh) ||
        !make_f32_rows_map(p.router_wl, (uint64_t)p.E, (uint32_t)p.H, LT_KS, (uint32_t)p.E, m.wl))
        return cudaErrorNotSupported;
    const int NS = lt_stages(p.E);
    const int smem = NS * lt_stage_bytes(p.E) + 1024;
    cudaError_t e = cudaFuncSetAttribute(logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((p.T + LT_M - 1) / LT_M, LT_S);
    logits_tc_kernel<<<grid, LT_THREADS, smem, s>>>(m, p.T, p.H, p.E, NS, p.logits_part, p.xb, p.status);
    return cudaGetLastError();
}

}  // namespace rmoe
