// topk.cuh -- top-k of one token's router logits (one warp) and the fast router's near-tie
// refinement, shared by the routing kernels (route.cu) and the one-launch small-batch layer.
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

// ---------------------------------------------------------------------------------------
// top-k of one token's E logits (one warp)
// ---------------------------------------------------------------------------------------
// Routing weights of one token's k picks (one warp; lane j < k holds pick j's score and writes
// w_out[j]).  The sums run in pick order on every lane (the same sequential f32 additions as
// the reference), each lane then forms its own weight.
__device__ __forceinline__ void pick_weights(float chosen_score, int k, int gate, int lane, float* w_out) {
    if (gate == 1) {
        float wsum = 0.0f;
        for (int j = 0; j < k; j++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, chosen_score, j));
        if (lane < k) w_out[lane] = (wsum == 0.0f) ? 0.0f : __fdiv_rn(chosen_score, wsum);
    } else {
        // softmax_in_place (src/moe.rs:61-72): max fold, exp(v - max), sequential sum, divide
        float mx = -INFINITY;
        for (int j = 0; j < k; j++) mx = fmaxf(mx, __shfl_sync(0xffffffffu, chosen_score, j));
        const float ex = (lane < k) ? expf(__fsub_rn(chosen_score, mx)) : 0.0f;
        float sum = 0.0f;
        for (int j = 0; j < k; j++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, j));
        if (lane < k) w_out[lane] = (sum != 0.0f) ? __fdiv_rn(ex, sum) : ex;
    }
}

// The score top-k ranks: the logit, or its sigmoid (src/moe.rs:44-46) for the sigmoid gate.
__device__ __forceinline__ float gate_score(float x, int gate) { return gate == 1 ? 1.0f / (1.0f + expf(-x)) : x; }

// Scores as unsigned keys in the same order (-0 and +0 equal, as the float compare has them);
// 0 is left free to mark a taken or absent entry.
__device__ __forceinline__ unsigned score_key(float v) {
    const unsigned u = __float_as_uint(v + 0.0f);
    const unsigned k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return k ? k : 1u;
}
__device__ __forceinline__ float key_score(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// The n best scores of one token's E logits (one warp).  Order = stable descending argsort
// (larger first, ties to the lower index), the rusty-engine top_k / top_k_sigmoid contract
// (src/moe.rs:75-117).  Lane j < n gets the j-th expert id and its score.
template <int NS>  // NS >= ceil(E / 32) logits per lane
__device__ __forceinline__ void warp_select_n(const float* lg, int E, int n, int gate, int lane, float& chosen_score,
                                              int& chosen_id) {
    unsigned key[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) {
        const int e = lane + 32 * s;
        key[s] = e < E ? score_key(gate_score(lg[e], gate)) : 0u;
    }
    chosen_score = 0.0f;
    chosen_id = 0;
    for (int j = 0; j < n; j++) {
        // this lane's best (s ascending = index ascending, so a strict '>' keeps the lower
        // index), then the warp's largest key and, among the lanes holding it, the lowest index
        unsigned bk = 0u;
        int bs = 0;
#pragma unroll
        for (int s = 0; s < NS; s++)
            if (key[s] > bk) {
                bk = key[s];
                bs = s;
            }
        const unsigned m = __reduce_max_sync(0xffffffffu, bk);
        const int win = (int)__reduce_min_sync(0xffffffffu, bk == m ? (unsigned)(lane + 32 * bs) : 0xffffffffu);
        if ((win & 31) == lane)
#pragma unroll
            for (int s = 0; s < NS; s++)
                if (s == (win >> 5)) key[s] = 0u;
        if (lane == j) {
            chosen_score = key_score(m);
            chosen_id = win;
        }
    }
}

// One token's top-k (one warp): lane j < k returns the j-th expert id and writes pick j's
// weight to w_out[j].
template <int NS>
__device__ int warp_topk_n(const float* lg, int E, int k, int gate, int lane, float* w_out) {
    float chosen_score;
    int chosen_id;
    warp_select_n<NS>(lg, E, k, gate, lane, chosen_score, chosen_id);
    pick_weights(chosen_score, k, gate, lane, w_out);
    return chosen_id;
}

__device__ __forceinline__ int warp_topk(const float* lg, int E, int k, int gate, int lane, float* w_out) {
    const int ns = (E + 31) / 32;
    if (ns <= 1) return warp_topk_n<1>(lg, E, k, gate, lane, w_out);
    if (ns <= 2) return warp_topk_n<2>(lg, E, k, gate, lane, w_out);
    if (ns <= 4) return warp_topk_n<4>(lg, E, k, gate, lane, w_out);
    if (ns <= 8) return warp_topk_n<8>(lg, E, k, gate, lane, w_out);
    return warp_topk_n<MAX_E / 32>(lg, E, k, gate, lane, w_out);
}

// ---------------------------------------------------------------------------------------
// Near-tie refinement of the fast router.
//
// A fast logit differs from moe::matvec's sequential f32 sum (src/moe.rs:271-277) by
// summation error.  Both sums are within a few units of u * ||w_e|| * ||x_t|| (u = 2^-24) of
// the exact value (at the BASELINE shapes the largest distance seen is about 14 units, nearly
// all of it the sequential sum's own rounding), so a
// top-k choice made on fast logits can differ from the reference's only where two of the
// k + 1 best scores lie within that distance.  For a token where any two adjacent scores of
// its k + 1 best are closer than tau = REFINE_UNITS units (the ratio of tau to the largest
// error is what the GPU tests check), every expert whose fast score lies within tau of the
// (k+1)-th best is rescored with the exact sequential chain, bit-identical to moe::matvec, and
// top-k runs again: experts further down are more than tau / 2 below k + 1 others under any
// of the sums and cannot be chosen.  The ids are then the reference's, near-ties included.
// Two steps: each warp checks its tokens (warp_topk_try) and defers the close ones; after the
// CTA's warps are done, the whole CTA rescores the deferred tokens (cta_rescore_batch), so the rows
// come in with the CTA's full memory parallelism and only the chain itself is serial.
// For the sigmoid gate the distances are taken between scores (sigmoid has slope <= 1/4,
// plus a few ulp for the rounding of the score itself).
// ---------------------------------------------------------------------------------------
static constexpr float REFINE_UNITS = 64.0f;

// ||x_t||_2 (one warp) from the token's fp16 copy (written by the logits step before any top-k
// runs; 16-B loads through L2, all of a lane's in flight at once).  It only sizes the
// refinement window, so the fp16 rounding of x does not matter.
__device__ __forceinline__ float warp_row_norm(const __half* __restrict__ xb, int H, int lane) {
    const uint4* x8 = reinterpret_cast<const uint4*>(xb);
    float s = 0.0f;
#pragma unroll 8
    for (int j = lane; j < H / 8; j += 32) {
        const uint4 v = __ldcg(x8 + j);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
            s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    return sqrtf(s);
}

// Whether the fast router refines at all (exact logits need no refinement).
__host__ __device__ __forceinline__ bool refine_on(const RouteParams& p) {
    return !p.exact && p.x && p.xb && p.router_wmax > 0.0f;
}

// One token whose fast top-k met a near-tie, as the first step hands it to the second: the
// experts to rescore (at most RF_MAXM; nm = -1: more than that, then every expert scoring at
// least thr is rescored).
static constexpr int RF_MAXM = 32;
struct AmbTok {
    int t, nm;
    float thr;
    int mem[RF_MAXM];
};

// First step, one warp per token: top-k of token t from its fast logits in row[0 .. E).  When
// no two of the k + 1 best scores are within the window, lane j < k gets the j-th id in `id`,
// the weights are written to w_out, and the call returns true.  Otherwise it fills `a` (a
// shared-memory slot) and returns false; the CTA then rescores (cta_rescore_batch) and reruns
// warp_topk on the token's row.  The sorted k + 1 best split into groups at every gap of at
// least the window; only groups of two or more can be misordered, so only their experts are
// rescored, plus, when such a group reaches the (k+1)-th best, every expert below it within
// the window (one of them may belong in the top k).
template <int NS>
__device__ bool warp_topk_try_n(const RouteParams& p, int t, const float* row, int lane, float* w_out, int& id,
                                AmbTok& a, float xn) {
    const int E = p.E, k = p.k, gate = p.gate;
    if (xn < 0.0f) xn = warp_row_norm(p.xb + (size_t)t * p.H, p.H, lane);
    const int n = min(k + 1, E);
    float sc;
    warp_select_n<NS>(row, E, n, gate, lane, sc, id);
    const float tau_l = REFINE_UNITS * 5.9604645e-8f * p.router_wmax * xn;
    const float tau = gate == 1 ? 0.25f * tau_l + 4.7683716e-7f : tau_l;  // + 8 ulp of 1.0
    const float next = __shfl_down_sync(0xffffffffu, sc, 1);
    const bool close = lane + 1 < n && !(sc - next >= tau);  // ranks lane and lane + 1
    const unsigned cm = __ballot_sync(0xffffffffu, close);
    if (!cm) {
        pick_weights(sc, k, gate, lane, w_out);
        return true;
    }
    const bool in = lane < n && (((cm >> lane) & 1u) || (lane > 0 && ((cm >> (lane - 1)) & 1u)));
    const unsigned im = __ballot_sync(0xffffffffu, in);
    int nm = __popc(im);
    if (in) a.mem[__popc(im & ((1u << lane) - 1u))] = id;
    const float sk = __shfl_sync(0xffffffffu, sc, n - 1);
    const float thr = k < E ? sk - tau : -INFINITY;
    if (k < E && ((cm >> (n - 2)) & 1u)) {  // the group reaches the (k+1)-th best
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            bool top = false;  // one of the k + 1 best already
            for (int j = 0; j < n; j++) top |= __shfl_sync(0xffffffffu, id, j) == e;
            const float se = e < E ? gate_score(row[e], gate) : -INFINITY;
            const bool b = e < E && !top && !(se < thr);
            const unsigned bm = __ballot_sync(0xffffffffu, b);
            const int at = nm + __popc(bm & ((1u << lane) - 1u));
            if (b && at < RF_MAXM) a.mem[at] = e;
            nm += __popc(bm);
        }
    }
    if (lane == 0) {
        a.t = t;
        a.nm = nm <= RF_MAXM ? nm : -1;
        a.thr = thr;
    }
    __syncwarp();
    return false;
}

// xn: ||x_t||_2 where the caller has it, else negative (the warp reads the token's fp16 copy).
__device__ __forceinline__ bool warp_topk_try(const RouteParams& p, int t, const float* row, int lane, float* w_out,
                                              int& id, AmbTok& a, float xn = -1.0f) {
    const int ns = (p.E + 31) / 32;
    if (ns <= 1) return warp_topk_try_n<1>(p, t, row, lane, w_out, id, a, xn);
    if (ns <= 2) return warp_topk_try_n<2>(p, t, row, lane, w_out, id, a, xn);
    if (ns <= 4) return warp_topk_try_n<4>(p, t, row, lane, w_out, id, a, xn);
    if (ns <= 8) return warp_topk_try_n<8>(p, t, row, lane, w_out, id, a, xn);
    return warp_topk_try_n<MAX_E / 32>(p, t, row, lane, w_out, id, a, xn);
}

// Second step, the whole CTA (every thread calls it, with the same arguments): the listed
// experts of the deferred tokens are rescored with moe::matvec's sequential chain
// (src/moe.rs:271-277): products rounded, then added in ascending k to a running f32 sum that
// starts at 0, no contraction.  As many tokens as `stage` (stage_floats floats of shared
// memory, at least 2 H) holds go at once: their x rows and listed router rows are loaded with
// 16-B loads all in flight, every thread forms products in place, and one thread per
// (token, expert) adds its products in ascending k -- only those chains are serial, and they
// run side by side.  A token with more than RF_MAXM experts to rescore (nm = -1) goes alone,
// in rounds, over every expert scoring at least its thr (its row read back from `logits`).
// The tokens are slots[list[0 .. na)]; token t's logits are row t - row0 of `logits` (row
// stride ld, global or shared memory, holding the fast ones on entry), where the exact ones
// are written.
static constexpr int RF_JMAX = 128;  // (token, expert) chains per round
static __device__ void cta_rescore_batch(const RouteParams& p, const AmbTok* slots, const int* list, int na,
                                         float* stage, int stage_floats, float* logits, int row0, int ld) {
    __shared__ int s_tok[RF_JMAX], s_e[RF_JMAX], s_xrow[RF_JMAX], s_erow[RF_JMAX];
    __shared__ int s_nj, s_next, s_cursor;
    const int E = p.E, H = p.H, gate = p.gate, h4 = H / 4;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int cap = min(stage_floats / H, RF_JMAX + 1);  // rows the stage holds
    float4* st4 = reinterpret_cast<float4*>(stage);
    if (cap < 2) {  // no room for x and one expert row: the tokens keep their fast logits
        if (tid == 0 && p.status) atomicOr(p.status, (unsigned)DERR_TIMEOUT);
        __syncthreads();
        return;
    }
    __syncthreads();
    if (tid == 0) s_cursor = 0;
    int i0 = 0;
    // every round consumes at least one expert of token i0 or moves past it, so the rounds are
    // bounded; the bound is enforced all the same (status word, then the remaining tokens keep
    // their fast logits)
    const int max_rounds = na * (E + 2);
    for (int round = 0; i0 < na; round++) {
        if (round >= max_rounds) {
            if (tid == 0 && p.status) atomicOr(p.status, (unsigned)DERR_TIMEOUT);
            break;
        }
        __syncthreads();
        if (tid == 0) {
            int nj = 0, i = i0, rows = 0;
            const AmbTok& a0 = slots[list[i0]];
            if (s_cursor > 0 || a0.nm < 0 || 1 + a0.nm > cap) {
                // token i0 alone, a round of at most cap - 1 of its experts from the cursor:
                // its list, or (over-full list) every expert scoring at least thr
                int c = s_cursor;
                if (a0.nm >= 0) {
                    for (; c < a0.nm && nj < cap - 1; c++, nj++) s_e[nj] = a0.mem[c];
                    s_cursor = c < a0.nm ? c : 0;
                    i = c < a0.nm ? i0 : i0 + 1;
                } else {
                    for (; c < E && nj < cap - 1; c++) {
                        const float se = gate_score(logits[(size_t)(a0.t - row0) * ld + c], gate);
                        if (!(se < a0.thr)) s_e[nj++] = c;
                    }
                    s_cursor = c < E ? c : 0;
                    i = c < E ? i0 : i0 + 1;
                }
                for (int j = 0; j < nj; j++) {
                    s_tok[j] = i0;
                    s_xrow[j] = 0;
                    s_erow[j] = 1 + j;
                }
            } else {  // whole tokens while their rows fit
                for (; i < na; i++) {
                    const int nm = slots[list[i]].nm;
                    if (nm < 0 || rows + 1 + nm > cap || nj + nm > RF_JMAX) break;
                    for (int j = 0; j < nm; j++) {
                        s_tok[nj + j] = i;
                        s_e[nj + j] = slots[list[i]].mem[j];
                        s_xrow[nj + j] = rows;
                        s_erow[nj + j] = rows + 1 + j;
                    }
                    rows += 1 + nm;
                    nj += nm;
                }
            }
            s_nj = nj;
            s_next = i;
        }
        __syncthreads();
        const int nj = s_nj;
        // the x rows (one per token of the round: its first job loads it) and the expert rows,
        // every 16-B load of the round issued before any is used
        for (int q = tid; q < 2 * nj * h4; q += nthr) {
            const int j = q / (2 * h4), r = q - j * 2 * h4, w = r >= h4, c = r - w * h4;
            if (!w && j > 0 && s_tok[j - 1] == s_tok[j]) continue;  // x row loaded by the token's first job
            const float* src = w ? p.router_w + (size_t)s_e[j] * H : p.x + (size_t)slots[list[s_tok[j]]].t * H;
            st4[(size_t)(w ? s_erow[j] : s_xrow[j]) * h4 + c] = __ldg(reinterpret_cast<const float4*>(src) + c);
        }
        __syncthreads();
        for (int q = tid; q < nj * h4; q += nthr) {  // products, each rounded, in place
            const int j = q / h4, c = q - j * h4;
            float4 a = st4[(size_t)s_erow[j] * h4 + c];
            const float4 b = st4[(size_t)s_xrow[j] * h4 + c];
            a.x = __fmul_rn(a.x, b.x);
            a.y = __fmul_rn(a.y, b.y);
            a.z = __fmul_rn(a.z, b.z);
            a.w = __fmul_rn(a.w, b.w);
            st4[(size_t)s_erow[j] * h4 + c] = a;
        }
        __syncthreads();
        for (int j = tid; j < nj; j += nthr) {  // the chains, side by side
            const float4* pr = st4 + (size_t)s_erow[j] * h4;
            float s = 0.0f;
#pragma unroll 8
            for (int c = 0; c < h4; c++) {
                const float4 a = pr[c];
                s = __fadd_rn(s, a.x);
                s = __fadd_rn(s, a.y);
                s = __fadd_rn(s, a.z);
                s = __fadd_rn(s, a.w);
            }
            logits[(size_t)(slots[list[s_tok[j]]].t - row0) * ld + s_e[j]] = s;
        }
        __syncthreads();
        if (tid == 0 && p.refined && s_next > i0) atomicAdd(p.refined, (unsigned)(s_next - i0));
        i0 = s_next;
    }
    __syncthreads();
}

// Shared memory the rescoring stage takes for rows of H floats: about 88 KB (11 rows at
// H = 2048, 5 at H = 4096; at least 2), so that a CTA's deferred tokens usually go in one round.
__host__ __device__ inline int rescore_stage_floats(int H) {
    const int rows = max(2, min(16, 90112 / (4 * H)));
    return rows * H;
}

}  // namespace rmoe
