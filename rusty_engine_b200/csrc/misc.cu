// misc.cu -- deterministic combine and the stand-alone dequant operator.
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

// Deterministic combine (src/moe.rs:373-386): out[t] = 0; out[t] += w_j * y_j for j in the
// token's chosen order (multiply, then add: one rounding each, as in Rust); then + shared.
__global__ void combine_kernel(CombineParams p) {
    const int t = blockIdx.x;
    const int* sr = p.slot_row + (size_t)t * p.k;
    const float* wt = p.topk_w + (size_t)t * p.k;
    for (int i = threadIdx.x; i < p.H; i += blockDim.x) {
        float o = 0.0f;
        for (int j = 0; j < p.k; j++)
            if (sr[j] >= 0) o = __fadd_rn(o, __fmul_rn(wt[j], p.y[(size_t)sr[j] * p.H + i]));  // < 0: empty pick
        if (p.has_shared && t >= p.shared_t0 && t < p.shared_t0 + p.shared_n)
            o = __fadd_rn(o, p.y[(size_t)(p.expert_off[p.E] + t - p.shared_t0) * p.H + i]);
        p.out[(size_t)t * p.H + i] = o;
    }
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t s) {
    if (p.T <= 0) return cudaSuccess;
    combine_kernel<<<p.T, 256, 0, s>>>(p);
    return cudaGetLastError();
}

// ---- quant::dequant on raw GGUF bytes (src/quant.rs:363-453), one thread per block ----
__device__ __forceinline__ float rdh(const uint8_t* b) { return h2f((uint16_t)(b[0] | (b[1] << 8))); }

__global__ void dequant_raw_kernel(int type, const uint8_t* src, uint64_t nblocks, float* dst) {
    uint64_t bi = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (bi >= nblocks) return;
    switch (type) {
        case T_F32: {
            dst[bi] = reinterpret_cast<const float*>(src)[bi];
            break;
        }
        case T_F16: dst[bi] = rdh(src + 2 * bi); break;
        case T_BF16: {
            uint32_t v = (uint32_t)(src[2 * bi] | (src[2 * bi + 1] << 8)) << 16;
            dst[bi] = __uint_as_float(v);
            break;
        }
        case T_Q4_0: {
            const uint8_t* b = src + bi * 18;
            float* o = dst + bi * 32;
            float d = rdh(b);
            for (int j = 0; j < 16; j++) {
                o[j] = __fmul_rn((float)((int)(b[2 + j] & 0xF) - 8), d);
                o[j + 16] = __fmul_rn((float)((int)(b[2 + j] >> 4) - 8), d);
            }
            break;
        }
        case T_Q5_0: {
            const uint8_t* b = src + bi * 22;
            float* o = dst + bi * 32;
            float d = rdh(b);
            uint32_t qh = b[2] | (b[3] << 8) | (b[4] << 16) | ((uint32_t)b[5] << 24);
            for (int j = 0; j < 16; j++) {
                int x0 = (int)((b[6 + j] & 0xF) | (((qh >> j) & 1u) << 4)) - 16;
                int x1 = (int)((b[6 + j] >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16;
                o[j] = __fmul_rn((float)x0, d);
                o[j + 16] = __fmul_rn((float)x1, d);
            }
            break;
        }
        case T_Q8_0: {
            const uint8_t* b = src + bi * 34;
            float* o = dst + bi * 32;
            float d = rdh(b);
            for (int j = 0; j < 32; j++) o[j] = __fmul_rn((float)(int8_t)b[2 + j], d);
            break;
        }
        case T_Q4_K:
        case T_Q5_K: {
            const int bb = type == T_Q4_K ? 144 : 176;
            const uint8_t* b = src + bi * bb;
            float* o = dst + bi * 256;
            float d = rdh(b), mn = rdh(b + 2);
            const uint8_t* qs = b + (type == T_Q4_K ? 16 : 48);
            const uint8_t* qh = b + 16;
            for (int grp = 0; grp < 4; grp++) {
                int sc0, m0, sc1, m1;
                scale_min_k4(grp * 2, b + 4, sc0, m0);
                scale_min_k4(grp * 2 + 1, b + 4, sc1, m1);
                float d1 = __fmul_rn(d, (float)sc0), dm1 = __fmul_rn(mn, (float)m0);
                float d2 = __fmul_rn(d, (float)sc1), dm2 = __fmul_rn(mn, (float)m1);
                for (int l = 0; l < 32; l++) {
                    int lo = qs[grp * 32 + l] & 0xF, hi = qs[grp * 32 + l] >> 4;
                    if (type == T_Q5_K) {
                        lo += (qh[l] & (1u << (2 * grp))) ? 16 : 0;
                        hi += (qh[l] & (2u << (2 * grp))) ? 16 : 0;
                    }
                    o[grp * 64 + l] = __fsub_rn(__fmul_rn(d1, (float)lo), dm1);
                    o[grp * 64 + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)hi), dm2);
                }
            }
            break;
        }
        case T_Q6_K: {
            const uint8_t* b = src + bi * 210;
            float* o = dst + bi * 256;
            float d = rdh(b + 208);
            for (int half = 0; half < 2; half++) {
                const uint8_t* ql = b + half * 64;
                const uint8_t* qh = b + 128 + half * 32;
                const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + half * 8);
                float* oo = o + half * 128;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int q1 = (int)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                    int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    oo[l] = __fmul_rn(__fmul_rn(d, (float)sc[is]), (float)q1);
                    oo[l + 32] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
                    oo[l + 64] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
                    oo[l + 96] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
                }
            }
            break;
        }
        default: break;
    }
}

cudaError_t launch_dequant_raw(int type, const void* src, uint64_t nblocks, float* dst, cudaStream_t s) {
    if (nblocks == 0) return cudaSuccess;
    unsigned grid = (unsigned)((nblocks + 255) / 256);
    dequant_raw_kernel<<<grid, 256, 0, s>>>(type, static_cast<const uint8_t*>(src), nblocks, dst);
    return cudaGetLastError();
}

__global__ void f32_to_f16_kernel(const float* x, __half* y, uint64_t n) {
    uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(x[i]);
}

cudaError_t launch_f32_to_f16(const float* x, __half* y, uint64_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    f32_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

}  // namespace rmoe
