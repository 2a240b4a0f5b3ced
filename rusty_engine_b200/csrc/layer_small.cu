// layer_small.cu -- the whole MoE layer for a decode batch (T <= 16 tokens, Q4_K / Q6_K experts)
// in one launch.
//
// At decode sizes the layer is a chain of dependent steps (router logits -> top-k -> dispatch ->
// gate/up -> down), each only a few microseconds of work, so separate launches spend most of
// the layer in launch and drain gaps.  Here one cooperative launch (every CTA resident at once)
// runs the chain with two grid-wide barriers:
//   A. router logits, one warp per expert over all T tokens (fast FFMA sums); the fp16 copy of
//      x (range-checked), the output rows zeroed, the SwiGLU row exponents reset;
//   -- barrier --
//   B. in every CTA: top-k of every token with the near-tie refinement (topk.cuh), then the
//      dispatch in shared memory: picks sorted by (expert, token order), one tile per expert
//      (an expert holds at most T <= 16 rows of the batch), the shared expert last;
//      C. gate/up + SwiGLU items (tile, weight-row block), dealt round-robin over the CTAs,
//      each the decode kernels' tile body (gemv.cuh);
//   -- barrier --
//   D. down + weighted combine items the same way (atomic adds into the zeroed output).
// Every CTA computes the same routing from the same logits, so the dispatch needs no third
// barrier; only CTA 0 writes the routing out (rmoe_layer_routing) and counts refinements (the
// logits written out, rmoe_layer_logits, are the fast sums, before any refinement).
// The barrier waits are bounded (1 s of globaltimer), after which a CTA records DERR_TIMEOUT in
// the status word and goes on.
#include <algorithm>

#include "gemv.cuh"
#include "topk.cuh"

namespace rmoe {

static constexpr int LS_MAX_T = 16;
static constexpr int LS_WCH = 16;            // float4 of a router row a lane holds at a time
static constexpr int LS_XSTAGE = 64 * 1024;  // shared memory for staged token rows (bytes)
static constexpr int LS_MAX_ROWS = LS_MAX_T * (MAX_K + 1);

struct SmallLayerParams {
    RouteParams r;       // x, router_w, T, H, E, k, gate, has_shared, xb, rowexp, logits, out_zero,
                         // topk_id, topk_w, status, refined, router_wmax
    GroupedParams g;     // expert stacks, h / hexp / rowexp, out
    unsigned* bar;       // grid barrier words: arrivals, generation (zero at first use)
    int depth_gu, ring_gu, depth_dn, ring_dn;
    int stage_floats;    // shared memory after the logit rows, for rescoring near-ties
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ls_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// Grid-wide barrier of a cooperative launch: bar[0] counts arrivals, bar[1] is the generation.
// The last CTA to arrive resets the count and moves the generation on; the others wait for
// that, at most 1 s, then record DERR_TIMEOUT and go on.
__device__ void ls_grid_barrier(unsigned* bar, unsigned* status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned gen = ld_acquire_gpu(bar + 1);
        __threadfence();  // this CTA's writes before its arrival
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);  // nobody arrives again before the generation moves
            __threadfence();
            st_release_gpu(bar + 1, gen + 1);
        } else {
            const uint64_t t0 = ls_globaltimer();
            for (uint32_t i = 0; ld_acquire_gpu(bar + 1) == gen; i++) {
                if ((i & 255) == 255 && ls_globaltimer() - t0 > 1000000000ull) {
                    atomicOr(status, (unsigned)DERR_TIMEOUT);
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
}

template <int TG, int TD, int NT, int KSG, int KSD>
__global__ void __launch_bounds__(GV_THREADS, 2) layer_small_kernel(SmallLayerParams sp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_ids[LS_MAX_T * MAX_K];
    __shared__ float s_wts[LS_MAX_T * MAX_K];
    __shared__ int s_rtok[LS_MAX_ROWS], s_rslot[LS_MAX_ROWS], s_rid[LS_MAX_ROWS];
    __shared__ int4 s_tiles[LS_MAX_ROWS];
    __shared__ int s_ntiles;
    const RouteParams& p = sp.r;
    const int T = p.T, H = p.H, E = p.E, k = p.k;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gtid = blockIdx.x * GV_THREADS + tid, gthreads = gridDim.x * GV_THREADS;
    const int gwarp = gtid >> 5, gwarps = gthreads >> 5;
    const int n4 = H / 4;

    // ---- A. logits (lane l sums elements 4 l + 128 j of its expert for every token) ----------
    // CTA b < ceil(E / 8): warp w scores expert 8 b + w.  Its first router chunk (16 float4 a
    // lane) is loaded before anything waits; the tokens are staged in shared memory LS_XG at a
    // time (every load of a group in flight at once), so no load sits behind an FMA chain.
    if (blockIdx.x * 8 < E) {
        const int e = blockIdx.x * 8 + warp;
        const float4* wr = reinterpret_cast<const float4*>(p.router_w + (size_t)min(e, E - 1) * H);
        float4 wv[LS_WCH];
#pragma unroll
        for (int u = 0; u < LS_WCH; u++) {
            const int j = lane + 32 * u;
            wv[u] = j < n4 ? __ldg(wr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float4* xs4 = reinterpret_cast<float4*>(smem);
        const int G = max(1, min(T, LS_XSTAGE / (H * 4)));
        float mine = 0.0f;
        for (int tg = 0; tg < T; tg += G) {
            const int ng = min(G, T - tg);
            __syncthreads();  // the previous group's rows are no longer read
            const float4* xg = reinterpret_cast<const float4*>(p.x + (size_t)tg * H);
            for (int q0 = 0; q0 < ng * n4; q0 += 8 * GV_THREADS) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int q = q0 + u * GV_THREADS + tid;
                    v[u] = q < ng * n4 ? __ldg(xg + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int q = q0 + u * GV_THREADS + tid;
                    if (q < ng * n4) xs4[q] = v[u];
                }
            }
            __syncthreads();
            if (e < E) {
                float acc[LS_MAX_T];
#pragma unroll
                for (int t = 0; t < LS_MAX_T; t++) acc[t] = 0.0f;
                for (int j0 = 0; j0 < n4; j0 += 32 * LS_WCH) {
                    if (j0 > 0)
#pragma unroll
                        for (int u = 0; u < LS_WCH; u++) {
                            const int j = j0 + lane + 32 * u;
                            wv[u] = j < n4 ? __ldg(wr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                    for (int u = 0; u < LS_WCH; u++) {
                        const int j = j0 + lane + 32 * u;
                        if (j < n4)
#pragma unroll
                            for (int t = 0; t < LS_MAX_T; t++)
                                if (t < ng) {
                                    const float4 a = wv[u], b = xs4[t * n4 + j];
                                    acc[t] = fmaf(a.x, b.x, acc[t]);
                                    acc[t] = fmaf(a.y, b.y, acc[t]);
                                    acc[t] = fmaf(a.z, b.z, acc[t]);
                                    acc[t] = fmaf(a.w, b.w, acc[t]);
                                }
                    }
                }
#pragma unroll
                for (int t = 0; t < LS_MAX_T; t++)
                    if (t < ng) {
                        float v = acc[t];
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                        if (lane == tg + t) mine = v;
                    }
                if (n4 > 32 * LS_WCH)  // the chunk registers hold the last chunk: reload the first
#pragma unroll
                    for (int u = 0; u < LS_WCH; u++) {
                        const int j = lane + 32 * u;
                        wv[u] = j < n4 ? __ldg(wr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
            }
        }
        if (e < E && lane < T) p.logits[(size_t)lane * E + e] = mine;
    }
    {
        // fp16 MMA operand (|x| beyond the fp16 range is reported, never silently inf), zeroed
        // output rows for the atomic combine, reset row exponents
        const float4* x4 = reinterpret_cast<const float4*>(p.x);
        for (int q = gtid; q < T * n4; q += gthreads) {
            const float4 v = __ldg(x4 + q);
            if (!(fabsf(v.x) <= 65504.f && fabsf(v.y) <= 65504.f && fabsf(v.z) <= 65504.f && fabsf(v.w) <= 65504.f))
                atomicOr(p.status, (unsigned)DERR_FP16_RANGE);
            *reinterpret_cast<uint2*>(p.xb + 4 * (size_t)q) = make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
            reinterpret_cast<float4*>(p.out_zero)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int rows = T * k + (p.has_shared ? T : 0);
        for (int r = gtid; r < rows; r += gthreads) p.rowexp[r] = -127;
    }
    ls_grid_barrier(sp.bar, p.status);

    // ---- B. routing and dispatch, in every CTA --------------------------------------------
    float* rows_s = reinterpret_cast<float*>(smem);  // [T][E] logits
    for (int q = tid; q < T * E; q += GV_THREADS) rows_s[q] = __ldcg(p.logits + q);
    __syncthreads();
    // every CTA refines from the same fast logits (the written-out logits stay the fast ones,
    // since other CTAs may still be reading them); one CTA counts the refinements
    RouteParams rp = p;
    rp.logits = nullptr;
    if (blockIdx.x != 0) rp.refined = nullptr;
    __shared__ AmbTok amb[LS_MAX_T];
    __shared__ int amb_list[LS_MAX_T], amb_n;
    if (tid == 0) amb_n = 0;
    __syncthreads();
    for (int t = warp; t < T; t += GV_THREADS / 32) {
        int id;
        if (!refine_on(rp)) {
            id = warp_topk(rows_s + (size_t)t * E, E, k, p.gate, lane, s_wts + t * k);
        } else if (!warp_topk_try(rp, t, rows_s + (size_t)t * E, lane, s_wts + t * k, id, amb[t])) {
            if (lane == 0) amb_list[atomicAdd(&amb_n, 1)] = t;  // near-tie: rescored below
            continue;
        }
        if (lane < k) s_ids[t * k + lane] = id;
    }
    __syncthreads();
    if (amb_n) {  // CTA-uniform; the stage follows the logit rows, which it updates
        cta_rescore_batch(rp, amb, amb_list, amb_n, rows_s + ((T * E + 3) & ~3), sp.stage_floats, rows_s, 0, E);
        for (int i = warp; i < amb_n; i += GV_THREADS / 32) {
            const int t = amb_list[i];
            const int id = warp_topk(rows_s + (size_t)t * E, E, k, p.gate, lane, s_wts + t * k);
            if (lane < k) s_ids[t * k + lane] = id;
        }
        __syncthreads();
    }
    const int np = T * k, nrows = np + (p.has_shared ? T : 0);
    if (blockIdx.x == 0)
        for (int i = tid; i < np; i += GV_THREADS) {
            p.topk_id[i] = s_ids[i];
            p.topk_w[i] = s_wts[i];
        }
    // rank of every pick by (expert, pick index): rows of an expert in token order
    for (int i = tid; i < np; i += GV_THREADS) {
        const int id = s_ids[i];
        int rank = 0;
        for (int j = 0; j < np; j++) {
            const int o = s_ids[j];
            rank += (o < id) || (o == id && j < i);
        }
        s_rtok[rank] = i / k;
        s_rslot[rank] = i - (i / k) * k;
        s_rid[rank] = id;
    }
    for (int t = tid; t < nrows - np; t += GV_THREADS) {  // the shared expert's rows, last
        s_rtok[np + t] = t;
        s_rslot[np + t] = k;
        s_rid[np + t] = E;
    }
    __syncthreads();
    if (warp == 0) {  // one tile per expert: (expert, first row, rows)
        int base = 0;
        for (int r0 = 0; r0 < nrows; r0 += 32) {
            const int r = r0 + lane;
            const bool start = r < nrows && (r == 0 || s_rid[r] != s_rid[r - 1]);
            const unsigned m = __ballot_sync(0xffffffffu, start);
            if (start) s_tiles[base + __popc(m & ((1u << lane) - 1u))] = make_int4(s_rid[r], r, 0, 0);
            base += __popc(m);
        }
        __syncwarp();
        for (int ti = lane; ti < base; ti += 32) {
            const int end = ti + 1 < base ? s_tiles[ti + 1].y : nrows;
            s_tiles[ti].z = end - s_tiles[ti].y;
        }
        if (lane == 0) s_ntiles = base;
    }
    __syncthreads();

    GroupedParams gp = sp.g;
    gp.row_tok = s_rtok;
    gp.row_slot = s_rslot;
    gp.topk_w = s_wts;
    const int ntiles = s_ntiles;

    // ---- C. gate/up + SwiGLU items ------------------------------------------------------------
    {
        constexpr int RB = GvGeom<TG, NT, 2, KSG>::RB;
        const int nrb = sp.g.I / RB;
        for (int it = blockIdx.x; it < ntiles * nrb; it += gridDim.x) {
            __syncthreads();  // the previous item's shared memory is free
            const int4 ti = s_tiles[it / nrb];
            gv_tile<TG, NT, 2, KSG, false>(gp, ti.x, ti.y, ti.z, it % nrb, sp.depth_gu, sp.ring_gu, smem);
        }
    }
    ls_grid_barrier(sp.bar, p.status);

    // ---- D. down + weighted combine items -----------------------------------------------------
    {
        constexpr int RB = GvGeom<TD, NT, 1, KSD>::RB;
        const int nrb = sp.g.H / RB;
        for (int it = blockIdx.x; it < ntiles * nrb; it += gridDim.x) {
            __syncthreads();
            const int4 ti = s_tiles[it / nrb];
            gv_tile<TD, NT, 1, KSD, false>(gp, ti.x, ti.y, ti.z, it % nrb, sp.depth_dn, sp.ring_dn, smem);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// Shared-memory layout of one gv_tile configuration (as go_gv in grouped_gemv.cu sizes it).
template <int TYPE, int NT, int NMAT, int KS>
static void gv_layout(int K, int& depth, int& ring_off, size_t& smem) {
    using G = GvGeom<TYPE, NT, NMAT, KS>;
    const size_t bbytes = (size_t)K * NT * 2;
    const size_t dbytes = Gv<TYPE>::DPL ? (size_t)NMAT * (K / 256) * G::RB * 2 : 0;
    ring_off = (int)((bbytes + dbytes + 127) & ~(size_t)127);
    depth = 4;
    while (depth > 2 && (size_t)ring_off + (size_t)depth * G::SLOT > GV_SMEM_TWO) depth--;
    smem = (size_t)ring_off + (size_t)depth * G::SLOT;
}

template <int TG, int TD, int NT, int KSG, int KSD>
static cudaError_t go_small(SmallLayerParams sp, int* grid_cache, cudaStream_t s) {
    const int H = sp.g.H, I = sp.g.I;
    if (I % GvGeom<TG, NT, 2, KSG>::RB || H % GvGeom<TD, NT, 1, KSD>::RB) return cudaErrorNotSupported;
    size_t sm_gu, sm_dn;
    gv_layout<TG, NT, 2, KSG>(H, sp.depth_gu, sp.ring_gu, sm_gu);
    gv_layout<TD, NT, 1, KSD>(I, sp.depth_dn, sp.ring_dn, sm_dn);
    const int rows_floats = (sp.r.T * sp.r.E + 3) & ~3;
    const size_t sm_route = (size_t)(rows_floats + 2 * sp.r.H) * 4;  // the rescoring stage takes what is left
    const int xg = std::max(1, std::min(sp.r.T, LS_XSTAGE / (H * 4)));  // staged token rows (phase A)
    const size_t smem = std::max(std::max(std::max(sm_gu, sm_dn), sm_route), (size_t)xg * H * 4);
    sp.stage_floats = (int)(smem / 4) - rows_floats;
    if (smem > 227 * 1024) return cudaErrorNotSupported;
    auto kfn = layer_small_kernel<TG, TD, NT, KSG, KSD>;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (*grid_cache <= 0) {
        int dev = 0, nsm = 0, per = 0, coop = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kfn, GV_THREADS, smem)) != cudaSuccess) return e;
        if (!coop || per < 1) return cudaErrorNotSupported;
        *grid_cache = nsm * per;
    }
    void* args[] = {&sp};
    return cudaLaunchCooperativeKernel((const void*)kfn, dim3(*grid_cache), dim3(GV_THREADS), args, smem, s);
}

template <int TG, int TD>
static cudaError_t go_small_types(const SmallLayerParams& sp, int* grid_cache, cudaStream_t s) {
    const int T = sp.r.T;
    if (T <= 2) return go_small<TG, TD, 8, 4, 2>(sp, grid_cache + 0, s);
    if (T <= 8) return go_small<TG, TD, 8, 2, 1>(sp, grid_cache + 1, s);
    return go_small<TG, TD, 16, 1, 1>(sp, grid_cache + 2, s);
}

bool layer_small_supported(int gate_type, int down_type, int T, int E, int k) {
    const bool tg = gate_type == T_Q4_K || gate_type == T_Q6_K, td = down_type == T_Q4_K || down_type == T_Q6_K;
    return tg && td && T >= 1 && T <= LS_MAX_T && k <= MAX_K && E <= MAX_E;
}

cudaError_t launch_layer_small(const RouteParams& r, const GroupedParams& g, unsigned* bar, int* grid_cache,
                               cudaStream_t s) {
    SmallLayerParams sp{};
    sp.r = r;
    sp.g = g;
    sp.bar = bar;
    const int tg = g.gate.type, td = g.down.type;
    if (tg == T_Q4_K && td == T_Q6_K) return go_small_types<T_Q4_K, T_Q6_K>(sp, grid_cache, s);
    if (tg == T_Q4_K && td == T_Q4_K) return go_small_types<T_Q4_K, T_Q4_K>(sp, grid_cache, s);
    if (tg == T_Q6_K && td == T_Q6_K) return go_small_types<T_Q6_K, T_Q6_K>(sp, grid_cache, s);
    if (tg == T_Q6_K && td == T_Q4_K) return go_small_types<T_Q6_K, T_Q4_K>(sp, grid_cache, s);
    return cudaErrorNotSupported;
}

}  // namespace rmoe
