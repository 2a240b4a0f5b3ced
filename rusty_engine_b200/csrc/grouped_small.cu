// grouped_small.cu -- grouped expert products for small per-expert row counts (decode).
//
// One CTA = one (tile of <= NT expert-sorted rows, block of 64 weight rows).  Weights are
// read straight from the device planes, decoded to fp16 (chunk8<TYPE>) into an XOR-swizzled
// shared tile, activations are gathered by token into a second swizzled tile, and four warps
// run mma.sync m16n8k16 (fp16 in, f32 accumulate).  The weight stream is the only HBM
// traffic that grows with the layer, so this path is bandwidth-bound at decode batch sizes.
//
//   gate/up kernel: h[row, f] = silu(gate_f . x) * (up_f . x)      (src/moe.rs:280-299)
//                   stored as fp16 * 2^e with e per (row, 64-feature block), and the row's
//                   largest e folded into rowexp[row] (atomicMax)
//   down kernel:    y = down . h[row] with every h block brought to the row's common scale
//                   while it is staged; out[tok] += w_slot * y * 2^rowexp  (src/moe.rs:373-380)
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

static constexpr int SM_BM = 64;       // weight rows per CTA (per matrix)
static constexpr int SM_KC = 128;      // K elements per stage
static constexpr int SM_THREADS = 128; // 4 warps x 16 rows
static constexpr int SM_CPR = SM_KC / 8;
static constexpr int SM_NT = 64;       // rows (tokens) per tile

int small_tile_rows() { return SM_NT; }

__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * SM_KC * 2 + ((c ^ (r & 7)) << 4)); }

template <int TYPE>
__device__ __forceinline__ void load_weights(const DevMat& M, uint64_t row0, int k0, uint8_t* As, int tid) {
    for (int q = tid; q < SM_BM * SM_CPR; q += SM_THREADS) {
        int r = q / SM_CPR, c = q % SM_CPR;
        uint4 v = chunk8<TYPE>(M, row0 + r, (uint32_t)(k0 / 8 + c));
        *reinterpret_cast<uint4*>(As + swz(r, c)) = v;
    }
}

// x rows gathered by token (fp16, [T, H]); rows >= nrows are zero.
template <int NT>
__device__ __forceinline__ void load_x(const __half* xb, const int* row_tok, int row0, int nrows, int H, int k0,
                                       uint8_t* Bs, int tid) {
    for (int q = tid; q < NT * SM_CPR; q += SM_THREADS) {
        int n = q / SM_CPR, c = q % SM_CPR;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < nrows) {
            size_t r = (size_t)__ldg(row_tok + row0 + n);
            v = __ldg(reinterpret_cast<const uint4*>(xb + r * H + k0 + c * 8));
        }
        *reinterpret_cast<uint4*>(Bs + swz(n, c)) = v;
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

// h rows (fp16 * 2^hexp per block) staged at the row's common scale 2^rowexp.
template <int NT>
__device__ __forceinline__ void load_h(const __half* h, const int8_t* hexp, const int* rexp_s, int row0, int nrows,
                                       int I, int k0, uint8_t* Bs, int tid) {
    const int nblk = I / HBLK;
    for (int q = tid; q < NT * SM_CPR; q += SM_THREADS) {
        int n = q / SM_CPR, c = q % SM_CPR;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < nrows) {
            size_t r = (size_t)(row0 + n);
            int k = k0 + c * 8;
            v = __ldg(reinterpret_cast<const uint4*>(h + r * I + k));
            v = scale_h8(v, (int)__ldg(hexp + r * nblk + k / HBLK) - rexp_s[n]);
        }
        *reinterpret_cast<uint4*>(Bs + swz(n, c)) = v;
    }
}

// One K stage of MMAs for one weight tile: acc[NT/8][4] += A(16 rows of warp) x B(NT)
template <int NT>
__device__ __forceinline__ void mma_stage(const uint8_t* As, const uint8_t* Bs, int warp, int lane,
                                          float (*acc)[4]) {
    const uint32_t a_base = smem_u32(As), b_base = smem_u32(Bs);
#pragma unroll
    for (int ks = 0; ks < SM_KC / 16; ks++) {
        uint32_t a[4];
        {
            int mi = lane >> 3, r = warp * 16 + (lane & 7) + (mi & 1) * 8, c = ks * 2 + (mi >> 1);
            ldmatrix_x4(a_base + swz(r, c), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int nt = 0; nt < NT / 16; nt++) {
            uint32_t b0, b1, b2, b3;
            int mi = lane >> 3, n = nt * 16 + (lane & 7) + (mi >> 1) * 8, c = ks * 2 + (mi & 1);
            ldmatrix_x4(b_base + swz(n, c), b0, b1, b2, b3);
            mma_f16_16816(acc[nt * 2 + 0], a, b0, b1);
            mma_f16_16816(acc[nt * 2 + 1], a, b2, b3);
        }
    }
}

// Exponent e with max|v| * 2^-e in [2^13, 2^14): a zero block gets -127 (never the row max
// unless the whole row is zero).
__device__ __forceinline__ int block_exp(float amax) {
    if (!(amax > 0.0f)) return -127;
    int e;
    frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    e -= 14;
    return max(-100, min(100, e));
}

// Epilogue shared by the gate/up kernels: SwiGLU values hs[NT][64] (f32, smem) -> fp16
// blocks with per-(row, block) exponent; rowexp gets the row maximum.
template <int NT, int THREADS>
__device__ __forceinline__ void store_h_block(const float* hs, int row0, int nrows, int fblk, const GroupedParams& p,
                                              int tid) {
    const int nblk = p.I / HBLK;
    // two threads per row, 32 features each
    for (int q = tid; q < NT * 2; q += THREADS) {
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

template <int TYPE, int NT>
__global__ void __launch_bounds__(SM_THREADS) small_gateup_kernel(GroupedParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* Ag = smem;
    uint8_t* Au = smem + SM_BM * SM_KC * 2;
    uint8_t* Bs = smem + 2 * SM_BM * SM_KC * 2;
    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;
    const int4 ti = p.tiles[tile];
    const int e = ti.x, row0 = ti.y, nrows = ti.z;
    const DevMat& G = (e < p.E) ? p.gate : p.sgate;
    const DevMat& U = (e < p.E) ? p.up : p.sup;
    const uint64_t wrow0 = (uint64_t)(e < p.E ? e : 0) * G.rows + (uint64_t)blockIdx.x * SM_BM;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    float accg[NT / 8][4], accu[NT / 8][4];
#pragma unroll
    for (int i = 0; i < NT / 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) accg[i][j] = accu[i][j] = 0.0f;

    for (int k0 = 0; k0 < p.H; k0 += SM_KC) {
        load_weights<TYPE>(G, wrow0, k0, Ag, tid);
        load_weights<TYPE>(U, wrow0, k0, Au, tid);
        load_x<NT>(p.xb, p.row_tok, row0, nrows, p.H, k0, Bs, tid);
        __syncthreads();
        mma_stage<NT>(Ag, Bs, warp, lane, accg);
        mma_stage<NT>(Au, Bs, warp, lane, accu);
        __syncthreads();
    }
    // SwiGLU in f32 (silu(g) * u, src/moe.rs:280-283) into smem hs[n][f]
    float* hs = reinterpret_cast<float*>(smem);
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT / 8; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int n = nt * 8 + tq * 2 + (j & 1);
            int f = warp * 16 + g + (j >> 1) * 8;
            hs[n * (HBLK + 1) + f] = silu_ref(accg[nt][j]) * accu[nt][j];
        }
    __syncthreads();
    store_h_block<NT, SM_THREADS>(hs, row0, nrows, blockIdx.x, p, tid);
}

template <int TYPE, int NT>
__global__ void __launch_bounds__(SM_THREADS) small_down_kernel(GroupedParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* Ad = smem;
    uint8_t* Bs = smem + SM_BM * SM_KC * 2;
    __shared__ int rexp_s[NT];
    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;
    const int4 ti = p.tiles[tile];
    const int e = ti.x, row0 = ti.y, nrows = ti.z;
    const DevMat& D = (e < p.E) ? p.down : p.sdown;
    const uint64_t wrow0 = (uint64_t)(e < p.E ? e : 0) * D.rows + (uint64_t)blockIdx.x * SM_BM;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int n = tid; n < NT; n += SM_THREADS) rexp_s[n] = (n < nrows) ? __ldg(p.rowexp + row0 + n) : 0;
    __syncthreads();

    float acc[NT / 8][4];
#pragma unroll
    for (int i = 0; i < NT / 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < p.I; k0 += SM_KC) {
        load_weights<TYPE>(D, wrow0, k0, Ad, tid);
        load_h<NT>(p.h, p.hexp, rexp_s, row0, nrows, p.I, k0, Bs, tid);
        __syncthreads();
        mma_stage<NT>(Ad, Bs, warp, lane, acc);
        __syncthreads();
    }
    const int g = lane >> 2, tq = lane & 3;
    const int f0 = blockIdx.x * SM_BM + warp * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NT / 8; nt++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int n = nt * 8 + tq * 2 + (j & 1);
            int f = f0 + (j >> 1) * 8;
            if (n < nrows) {
                int r = row0 + n;
                float yv = __fmul_rn(acc[nt][j], exp2i(rexp_s[n]));
                if (p.y) {
                    p.y[(size_t)r * p.H + f] = yv;
                } else {
                    int tok = __ldg(p.row_tok + r), slot = __ldg(p.row_slot + r);
                    float w = (slot < p.k) ? __ldg(p.topk_w + (size_t)tok * p.k + slot) : 1.0f;
                    atomicAdd(p.out + (size_t)tok * p.H + f, __fmul_rn(w, yv));
                }
            }
        }
    }
}

template <int NT>
static size_t smem_gateup() {
    size_t mma = (size_t)(2 * SM_BM + NT) * SM_KC * 2, epi = (size_t)NT * (HBLK + 1) * 4;
    return mma > epi ? mma : epi;
}
template <int NT>
static size_t smem_down() { return (size_t)(SM_BM + NT) * SM_KC * 2; }

template <int TYPE, int NT>
static cudaError_t go_gateup(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    auto k = small_gateup_kernel<TYPE, NT>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_gateup<NT>());
    dim3 grid(p.I / SM_BM, max_tiles);
    k<<<grid, SM_THREADS, smem_gateup<NT>(), s>>>(p);
    return cudaGetLastError();
}

template <int TYPE, int NT>
static cudaError_t go_down(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    auto k = small_down_kernel<TYPE, NT>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_down<NT>());
    dim3 grid(p.H / SM_BM, max_tiles);
    k<<<grid, SM_THREADS, smem_down<NT>(), s>>>(p);
    return cudaGetLastError();
}

#define RMOE_TYPE_SWITCH(T, ...)                                   \
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

cudaError_t launch_small_gateup(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    RMOE_TYPE_SWITCH(p.gate.type, return go_gateup<TT, SM_NT>(p, max_tiles, s))
}

cudaError_t launch_small_down(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    RMOE_TYPE_SWITCH(p.down.type, return go_down<TT, SM_NT>(p, max_tiles, s))
}

}  // namespace rmoe
