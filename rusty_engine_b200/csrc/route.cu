// route.cu -- router GEMV + top-k + dispatch in one launch.
//
// Router logits are bit-identical to rusty-engine's moe::matvec (src/moe.rs:271-277): each
// logit is a sequential f32 sum over H of w*x with separate multiply and add roundings (Rust
// never contracts), accumulated in ascending k.  The GEMV is register-tiled (32 tokens x 128
// experts per CTA, 4x4 outputs per thread) but every output keeps that exact order.
// Top-k is rusty-engine's stable descending argsort (src/moe.rs:75-93): larger score first,
// equal scores by lower expert index; softmax over the chosen k (src/moe.rs:61-72) or the
// sigmoid renormalisation (src/moe.rs:97-117).
//
// Dispatch: each CTA counts its tokens' picks per expert and the in-CTA rank of every pick
// in token order; the last CTA to finish (atomic ticket, no spin-wait) scans the counts and
// writes the expert-sorted row list (ascending token order inside each expert, so the layout
// is deterministic) and the GEMM tile list.
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

static constexpr int RT_TOK = 32;   // tokens per CTA
static constexpr int RT_EXP = 128;  // experts per register tile pass
static constexpr int RT_K = 32;     // k-tile
static constexpr int RT_THREADS = 256;

// Top-k of one token's E logits held in `lg` (shared or global memory), one warp.
// Order = stable descending argsort (larger first, ties to the lower index), the rusty-engine
// top_k / top_k_sigmoid contract (src/moe.rs:75-117).  Lane j < k returns the j-th expert id;
// lane 0 writes the k weights to w_out in chosen order.
__device__ int warp_topk(const float* lg, int E, int k, int gate, int lane, float* w_out) {
    float v[MAX_E / 32];
    unsigned taken = 0;
#pragma unroll
    for (int s = 0; s < MAX_E / 32; s++) {
        int e = lane + 32 * s;
        float x = (e < E) ? lg[e] : 0.0f;
        if (gate == 1 && e < E) x = 1.0f / (1.0f + expf(-x));  // sigmoid (src/moe.rs:44-46)
        v[s] = x;
        if (e >= E) taken |= 1u << s;
    }
    const int NONE = 0x7fffffff;
    float chosen_score = 0.0f;
    int chosen_id = 0;
    for (int j = 0; j < k; j++) {
        float best = 0.0f;
        int bid = NONE;
#pragma unroll
        for (int s = 0; s < MAX_E / 32; s++) {
            // s ascending = index ascending, so a strict '>' keeps the lowest index on ties
            if (!((taken >> s) & 1u) && (bid == NONE || v[s] > best)) {
                best = v[s];
                bid = lane + 32 * s;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            float ob = __shfl_xor_sync(0xffffffffu, best, off);
            int oi = __shfl_xor_sync(0xffffffffu, bid, off);
            bool better = (oi != NONE) && (bid == NONE || ob > best || (ob == best && oi < bid));
            if (better) { best = ob; bid = oi; }
        }
        if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
        if (lane == j) { chosen_score = best; chosen_id = bid; }
    }
    float sc[MAX_K];
#pragma unroll
    for (int j = 0; j < MAX_K; j++) sc[j] = __shfl_sync(0xffffffffu, chosen_score, j);
    if (lane == 0) {
        if (gate == 1) {
            float wsum = 0.0f;
            for (int j = 0; j < k; j++) wsum = __fadd_rn(wsum, sc[j]);
            for (int j = 0; j < k; j++) w_out[j] = (wsum == 0.0f) ? 0.0f : __fdiv_rn(sc[j], wsum);
        } else {
            // softmax_in_place (src/moe.rs:61-72): max fold, exp(v - max), sequential sum, divide
            float mx = -INFINITY;
            for (int j = 0; j < k; j++) mx = fmaxf(mx, sc[j]);
            float sum = 0.0f;
            for (int j = 0; j < k; j++) sum = __fadd_rn(sum, expf(__fsub_rn(sc[j], mx)));
            for (int j = 0; j < k; j++) {
                float ex = expf(__fsub_rn(sc[j], mx));
                w_out[j] = (sum != 0.0f) ? __fdiv_rn(ex, sum) : ex;
            }
        }
    }
    return chosen_id;
}

__global__ void __launch_bounds__(RT_THREADS) route_dispatch_kernel(RouteParams p) {
    __shared__ float xs[RT_K][RT_TOK + 4];
    __shared__ __align__(16) float ws[RT_K][RT_EXP + 4];
    extern __shared__ float dyn[];  // logits [RT_TOK][E + 1]
    __shared__ int ids_s[RT_TOK * 32];
    __shared__ unsigned int ticket_s;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * RT_TOK;
    const int E = p.E, H = p.H, k = p.k;
    const int LS = E + 1;

    // ---- logits: exact sequential-order f32 sums ----
    const int tx = tid & 31, ty = tid >> 5;  // experts 4tx..4tx+3, tokens 4ty..4ty+3
    for (int e0 = 0; e0 < E; e0 += RT_EXP) {
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
        for (int k0 = 0; k0 < H; k0 += RT_K) {
            // x tile: 32 tokens x 32 k (and the fp16 copy of x, written once when e0 == 0)
            for (int i = tid; i < RT_TOK * RT_K; i += RT_THREADS) {
                int tl = i / RT_K, kk = i % RT_K;
                int t = t0 + tl;
                float v = (t < p.T) ? p.x[(size_t)t * H + k0 + kk] : 0.0f;
                xs[kk][tl] = v;
                if (e0 == 0 && t < p.T && p.xb) {
                    // fp16 MMA operand; |x| beyond the fp16 range is reported, never silently inf
                    if (!(fabsf(v) <= 65504.0f)) atomicOr(p.status, (unsigned)DERR_FP16_RANGE);
                    p.xb[(size_t)t * H + k0 + kk] = __float2half_rn(v);
                }
            }
            // w tile: 128 experts x 32 k, transposed into ws[k][e]
            for (int i = tid; i < RT_EXP * RT_K / 4; i += RT_THREADS) {
                int el = i / (RT_K / 4), kq = (i % (RT_K / 4)) * 4;
                int e = e0 + el;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (e < E) v = __ldg(reinterpret_cast<const float4*>(p.router_w + (size_t)e * H + k0 + kq));
                ws[kq + 0][el] = v.x;
                ws[kq + 1][el] = v.y;
                ws[kq + 2][el] = v.z;
                ws[kq + 3][el] = v.w;
            }
            __syncthreads();
#pragma unroll 4
            for (int kk = 0; kk < RT_K; kk++) {
                float4 w4 = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
                float xv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) xv[i] = xs[kk][ty * 4 + i];
                float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(wv[j], xv[i]));
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int e = e0 + tx * 4 + j;
                if (e < E) dyn[(ty * 4 + i) * LS + e] = acc[i][j];
            }
    }
    __syncthreads();

    // optional logits dump (tests)
    if (p.logits_out) {
        for (int i = tid; i < RT_TOK * E; i += RT_THREADS) {
            int tl = i / E, e = i % E;
            if (t0 + tl < p.T) p.logits_out[(size_t)(t0 + tl) * E + e] = dyn[tl * LS + e];
        }
    }

    // ---- top-k per token: one warp per token ----
    for (int tl = warp; tl < RT_TOK; tl += RT_THREADS / 32) {
        int t = t0 + tl;
        if (t >= p.T) break;
        int id = warp_topk(dyn + tl * LS, E, k, p.gate, lane, p.topk_w + (size_t)t * k);
        if (lane < k) {
            p.topk_id[(size_t)t * k + lane] = id;
            ids_s[tl * k + lane] = id;
        }
    }
    // zero the output rows this CTA owns when the combine accumulates with atomics
    if (p.out_zero) {
        for (int tl = 0; tl < RT_TOK; tl++) {
            int t = t0 + tl;
            if (t >= p.T) break;
            for (int i = tid * 4; i < H; i += RT_THREADS * 4)
                *reinterpret_cast<float4*>(p.out_zero + (size_t)t * H + i) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    __syncthreads();

    // ---- per-CTA counts and in-CTA ranks (token order) ----
    const int ntok = min(RT_TOK, p.T - t0);
    for (int e = tid; e < E; e += RT_THREADS) {
        int c = 0;
        for (int i = 0; i < ntok * k; i++)
            if (ids_s[i] == e) p.local_rank[(size_t)t0 * k + i] = c++;
        p.cta_cnt[(size_t)blockIdx.x * E + e] = c;
    }

    // ---- last CTA: scan + expert-sorted rows + tile list ----
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket_s = atomicAdd(p.ticket, 1u);
    __syncthreads();
    if (ticket_s != gridDim.x - 1) return;
    __threadfence();

    const int ncta = gridDim.x;
    const int NE = E + (p.has_shared ? 1 : 0);
    __shared__ int off_s[MAX_E + 2];
    __shared__ int cnt_s[MAX_E + 2];
    for (int e = tid; e < E; e += RT_THREADS) {
        int c = 0;
        for (int b = 0; b < ncta; b++) c += __ldcg(p.cta_cnt + (size_t)b * E + e);
        cnt_s[e] = c;
    }
    if (tid == 0 && p.has_shared) cnt_s[E] = p.T;
    __syncthreads();
    if (tid == 0) {
        int run = 0, tiles = 0;
        for (int e = 0; e < NE; e++) {
            off_s[e] = run;
            p.expert_off[e] = run;
            run += cnt_s[e];
            tiles += (cnt_s[e] + p.tile_rows - 1) / p.tile_rows;
        }
        off_s[NE] = run;
        p.expert_off[NE] = run;
        *p.n_rows = run;
        if (tiles > p.max_tiles) {
            atomicOr(p.status, (unsigned)DERR_TILES_OVERFLOW);
            tiles = p.max_tiles;
        }
        *p.n_tiles = tiles;
    }
    __syncthreads();
    // per-(cta, expert) offsets, expert-major so rows stay in token order
    for (int e = tid; e < E; e += RT_THREADS) {
        int run = off_s[e];
        for (int b = 0; b < ncta; b++) {
            int c = __ldcg(p.cta_cnt + (size_t)b * E + e);
            p.cta_cnt[(size_t)b * E + e] = run;  // reuse as offsets
            run += c;
        }
    }
    __syncthreads();
    __threadfence_block();
    const int nent = p.T * k;
    for (int i = tid; i < nent; i += RT_THREADS) {
        int t = i / k;
        int e = __ldcg(p.topk_id + i);
        int pos = __ldcg(p.cta_cnt + (size_t)(t / RT_TOK) * E + e) + __ldcg(p.local_rank + i);
        p.row_tok[pos] = t;
        p.row_slot[pos] = i - t * k;
        p.slot_row[i] = pos;
        p.rowexp[pos] = -127;
    }
    if (p.has_shared) {
        for (int t = tid; t < p.T; t += RT_THREADS) {
            p.row_tok[off_s[E] + t] = t;
            p.row_slot[off_s[E] + t] = k;
            p.rowexp[off_s[E] + t] = -127;
        }
    }
    // tile list: (expert, first row, rows) with at most tile_rows rows per tile
    if (tid < 32) {
        // warp-serial over experts keeps this simple; NE <= MAX_E + 1
        int base = 0;
        for (int e = 0; e < NE; e++) {
            int c = cnt_s[e];
            int nt = (c + p.tile_rows - 1) / p.tile_rows;
            for (int j = lane; j < nt; j += 32) {
                int ti = base + j;
                if (ti < p.max_tiles) {
                    int r0 = j * p.tile_rows;
                    p.tiles[ti] = make_int4(e, off_s[e] + r0, min(p.tile_rows, c - r0), 0);
                }
            }
            base += nt;
        }
    }
    if (tid == 0) *p.ticket = 0u;  // re-arm for the next launch (stream-ordered)
}

size_t route_smem_bytes(int E) { return (size_t)RT_TOK * (E + 1) * sizeof(float); }
int route_grid(int T) { return (T + RT_TOK - 1) / RT_TOK; }

cudaError_t launch_route_dispatch(const RouteParams& p, cudaStream_t s) {
    size_t smem = route_smem_bytes(p.E);
    cudaFuncSetAttribute(route_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    route_dispatch_kernel<<<route_grid(p.T), RT_THREADS, smem, s>>>(p);
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
