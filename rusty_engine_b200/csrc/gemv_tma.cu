// gemv_tma.cu -- the decode-size grouped expert products (Q4_K / Q6_K) with the weight stream
// on the tensor memory accelerator, for batches large enough to fill the GPU with 128-row
// blocks (several tokens per launch).
//
// The products, fragment order and decode are those of gemv.cuh (dequantisation in the
// registers that feed mma.sync); what changes is how the weights arrive.  At decode batch sizes
// the per-lane cp.async ring of gv_kernel issues a few 8- and 16-byte requests per lane per
// unit, and its copy stream, not the decode, caps its HBM rate (with the decode taken out it
// still reached only ~2.5 TB/s at 64 tokens).  Here
// one producer warp brings each raw block of the CTA's 128 weight rows (the tensor-core path's
// weight maps: 128 rows x one Q4_K unit / one Q6_K superblock, plus the Q6_K d plane) into a
// ring of shared-memory stages with 2-D TMA copies, completion counted on an mbarrier per
// stage; the consumer warps (16 rows each: eight for 128-row blocks, four for gate/up's 64-row
// blocks) read their fragments from the stage, decode, multiply and release the stage (one
// arrival per warp) for the producer to refill.
//
// Items = (tile of <= NT expert-sorted rows, block of RB weight rows of the expert), K whole.
// Gate/up runs one item per CTA; down is persistent (two CTAs per SM), each CTA walking a
// contiguous range of items: the producer streams the raw blocks of one item after another
// through the same ring, and the consumers stage a tile's token rows once for all of its row
// blocks in the range.
//   gate/up: h[row, f] = silu(gate_f . x) * (up_f . x)      (src/moe.rs:280-299), stored as fp16
//            x 2^e with e per (row, 16-feature block); the row's largest e goes to rowexp[row]
//   down:    y = down . h[row], every h block brought to the row's exponent while it is staged;
//            out[tok] += w_slot * y * 2^rowexp                  (src/moe.rs:373-380)
// Every mbarrier wait is bounded: on a timeout the CTA records DERR_TIMEOUT, stops, and the
// producer waits (bounded) for the copies it issued before the CTA exits.
#include <algorithm>

#include "gemv.cuh"
#include "tc_ptx.cuh"

namespace rmoe {
using namespace tc;

// CTA = CONS consumer warps (row groups of 16 rows: RB = 16 CONS weight rows, the height of the
// maps' boxes) + one producer warp.  CONS = 8 (128 rows, two CTAs per SM) everywhere; gate/up
// with 8-row tiles also has CONS = 4 (64 rows, three CTAs per SM): twice the items, so the last
// partial wave of a launch is half as long.
static constexpr int GVT_MAXD = 8;  // ring stages at most
__host__ __device__ constexpr int gvt_ctas_per_sm(int cons) { return cons == 4 ? 3 : 2; }

__host__ __device__ constexpr bool gvt_persistent(int nmat) { return nmat == 1; }

template <int TYPE, int NMAT, int RB>
struct GvtGeom {
    using R = Raw<TYPE>;
    using RS = RawStage<TYPE, RB>;
    static constexpr int STAGE = NMAT * RS::BYTES;  // one raw block of every matrix
    static constexpr int UPB = R::RK / GV_UK;       // 128-element units per raw block
    static_assert(R::RK % GV_UK == 0 && RS::BYTES % 128 == 0, "stage geometry");
};

template <int TYPE, int NT, int NMAT, int CONS>
__global__ void __launch_bounds__(32 * (CONS + 1), gvt_ctas_per_sm(CONS))
    gvt_kernel(const __grid_constant__ GroupedParams p, const __grid_constant__ TcMaps maps, int depth, int ring_off) {
    constexpr int RB = 16 * CONS;
    using D = Gv<TYPE>;
    using G = GvtGeom<TYPE, NMAT, RB>;
    using RS = typename G::RS;
    using R = Raw<TYPE>;
    constexpr int NTT = NT / 8, UPB = G::UPB, NCT = 32 * CONS;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[GVT_MAXD], empty[GVT_MAXD];
    __shared__ int s_tok[NT], s_rexp[NT];
    __shared__ float s_w[NT];
    __shared__ volatile int s_abort;
    __shared__ int s_consumed;

    // launch order (programmatic dependent launch) as gv_kernel: gate/up waits for the routing
    // kernel, then lets the down kernel start; the down kernel streams its weights at once and
    // waits for gate/up before it touches h
    if (NMAT == 2) {
        pdl_wait();
        pdl_trigger();
    }
    // this CTA's items (tile * nrb + row block).  Down (persistent): a contiguous range, so that
    // consecutive items share their tile's token rows (staged once) and the weight ring streams
    // across items.  Gate/up: one item per CTA (grid = row blocks x tile slots), which measured
    // faster for its 16-stage items than the persistent walk.
    constexpr bool PERSIST = gvt_persistent(NMAT);
    const int rows_out = NMAT == 2 ? p.I : p.H, nrb = rows_out / RB;
    int it0, it1;
    if (PERSIST) {
        const int n_items = *p.n_tiles * nrb;
        it0 = (int)((long long)blockIdx.x * n_items / gridDim.x);
        it1 = (int)((long long)(blockIdx.x + 1) * n_items / gridDim.x);  // ranges differ by one item at most
    } else {
        it0 = (int)blockIdx.y < *p.n_tiles ? (int)blockIdx.y * nrb + (int)blockIdx.x : 0;
        it1 = (int)blockIdx.y < *p.n_tiles ? it0 + 1 : 0;
    }
    if (it0 >= it1) return;  // uniform exit before any barrier
    const int K = NMAT == 2 ? p.H : p.I;
    const int nraw = K / R::RK;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t ring = smem_u32(smem) + (uint32_t)ring_off;
    const int total_stages = (it1 - it0) * nraw;

    if (tid == 0) {
        for (int i = 0; i < depth; i++) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), CONS);
        }
        s_abort = 0;
        s_consumed = total_stages;
        fence_mbar_init();
    }
    __syncthreads();

    int issued = 0;  // producer: stages whose copies were issued
    if (warp == CONS) {
        // ---------------- producer: one raw block of every matrix per stage ----------------
        if (lane == 0) {
            int gj = 0;
            for (int item = it0; item < it1 && !s_abort; item++) {
                const int4 ti = p.tiles[item / nrb];
                const bool sh = ti.x >= p.E;
                const DevMat& M0 = NMAT == 2 ? (sh ? p.sgate : p.gate) : (sh ? p.sdown : p.down);
                const int grow0 = (sh ? 0 : ti.x) * (int)M0.rows + (item % nrb) * RB;
                for (int j = 0; j < nraw; j++, gj++) {
                    const int s = gj % depth;
                    if (gj >= depth && !mbar_wait(smem_u32(&empty[s]), ((gj / depth) + 1) & 1)) {
                        s_abort = 1;
                        atomicOr(p.status, (unsigned)DERR_TIMEOUT);
                        break;
                    }
                    if (s_abort) break;
                    const uint32_t bar = smem_u32(&full[s]);
                    mbar_arrive_expect_tx(bar, (uint32_t)G::STAGE);
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        const WMaps& wm = maps.w[sh ? 1 : 0][m];
                        const uint32_t dst = ring + (uint32_t)(s * G::STAGE + m * RS::BYTES);
                        tma_2d(dst, &wm.main, j * (R::MB / 2), grow0, bar);
                        if (R::DBLK) tma_2d(dst + RS::DOFF, &wm.d, grow0, j * R::DBLK, bar);
                    }
                    issued = gj + 1;
                }
            }
        }
    } else {
        // ---------------- consumers ----------------
        const int rg = warp, g = lane >> 2, c = lane & 3;
        uint2* bsm = reinterpret_cast<uint2*>(smem);
        int cur_tile = -1, row0 = 0, nrows = 0, gj = 0;
        int s = 0;               // ring slot of stage gj (kept incrementally: depth is a runtime value)
        uint32_t phase = 0;      // parity of the full[s] phase stage gj completes
        if (NMAT == 1) pdl_wait();  // h, its exponents and the row exponents are gate/up's output
        for (int item = it0; item < it1; item++) {
            const int tile = item / nrb, rblk = item % nrb;
            if (tile != cur_tile) {
                // the previous tile's token rows and tables are no longer read by any warp
                asm volatile("bar.sync 1, %0;\n" ::"n"(NCT) : "memory");
                const int4 ti = p.tiles[tile];
                cur_tile = tile;
                row0 = ti.y;
                nrows = ti.z;
                for (int n = tid; n < NT; n += NCT) {
                    int tok = 0, rexp = 0;
                    float w = 0.0f;
                    if (n < nrows) {
                        const int r = row0 + n;
                        tok = p.row_tok[r];
                        if (NMAT == 1) {
                            const int slot = p.row_slot[r];
                            w = slot < p.k ? p.topk_w[(size_t)tok * p.k + slot] : 1.0f;
                            rexp = __ldcg(p.rowexp + r);
                        }
                    }
                    s_tok[n] = tok;
                    s_w[n] = w;
                    s_rexp[n] = rexp;
                }
                asm volatile("bar.sync 1, %0;\n" ::"n"(NCT) : "memory");
                // token operand in fragment order (as gv_tile): entry ((u * 8 + s) * NTT + t) * 32 + lane
                const int cpr = K / 8;
                const int hstride = p.I / GV_EBLK;
                const int total = nrows * cpr;
                constexpr int SB = 4;
                for (int i0 = 0; i0 < total; i0 += SB * NCT) {
                    uint4 v[SB];
                    int d[SB];
#pragma unroll
                    for (int u = 0; u < SB; u++) {
                        const int i = i0 + u * NCT + tid;
                        d[u] = 0;
                        if (i < total) {
                            const int n = i / cpr, j = i - n * cpr;
                            if (NMAT == 2) {
                                v[u] = __ldcg(reinterpret_cast<const uint4*>(p.xb + (size_t)s_tok[n] * K + 8 * j));
                            } else {
                                const size_t r = (size_t)(row0 + n);
                                v[u] = __ldcg(reinterpret_cast<const uint4*>(p.h + r * p.I + 8 * j));
                                d[u] = (int)__ldcg(p.hexp + r * hstride + (8 * j) / GV_EBLK);
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < SB; u++) {
                        const int i = i0 + u * NCT + tid;
                        if (i >= total) continue;
                        const int n = i / cpr, j = i - n * cpr;
                        uint4 w = v[u];
                        if (NMAT == 1) {
                            const int dd = d[u] - s_rexp[n];
                            const uint2 lo = gv_scale4(make_uint2(w.x, w.y), dd), hi = gv_scale4(make_uint2(w.z, w.w), dd);
                            w = make_uint4(lo.x, lo.y, hi.x, hi.y);
                        }
#pragma unroll
                        for (int hf = 0; hf < 2; hf++) {
                            const int kk = 8 * j + 4 * hf;
                            int cc, st;
                            D::inv(kk & (GV_UK - 1), cc, st);
                            const uint32_t x01 = hf ? w.z : w.x, x23 = hf ? w.w : w.y;
                            bsm[(((kk / GV_UK) * 8 + st) * NTT + (n >> 3)) * 32 + (n & 7) * 4 + cc] =
                                make_uint2(__byte_perm(x01, x23, 0x5410), __byte_perm(x01, x23, 0x7632));
                        }
                    }
                }
                asm volatile("bar.sync 1, %0;\n" ::"n"(NCT) : "memory");
            }

            float acc[NMAT][NTT][4];
#pragma unroll
            for (int m = 0; m < NMAT; m++)
#pragma unroll
                for (int t = 0; t < NTT; t++)
#pragma unroll
                    for (int q = 0; q < 4; q++) acc[m][t][q] = 0.0f;
            const int ntl = (nrows + 7) >> 3;  // n-tiles holding live token rows

            for (int j = 0; j < nraw; j++, gj++) {
                if (s_abort || !mbar_wait(smem_u32(&full[s]), phase)) {
                    if (!s_abort) {
                        s_abort = 1;
                        atomicOr(p.status, (unsigned)DERR_TIMEOUT);
                    }
                    if (lane == 0) atomicMin(&s_consumed, gj);
                    break;
                }
                const uint8_t* st = smem + ring_off + (size_t)s * G::STAGE;
#pragma unroll
                for (int uu = 0; uu < UPB; uu++) {
                    const int u = j * UPB + uu;
                    const uint2* bu = bsm + (size_t)u * 8 * NTT * 32 + lane;
#pragma unroll
                    for (int m = 0; m < NMAT; m++) {
                        uint32_t afr[8][4];
#pragma unroll
                        for (int r = 0; r < 2; r++) {
                            const int row = 16 * rg + g + 8 * r;
                            const uint8_t* rp = st + m * RS::BYTES + row * R::PITCH;
                            uint4 q16[D::N16 > 0 ? D::N16 : 1];
                            uint2 q8[D::N8 > 0 ? D::N8 : 1];
#pragma unroll
                            for (int jj = 0; jj < D::N16; jj++) q16[jj] = *reinterpret_cast<const uint4*>(rp + D::off16(uu, c, jj));
#pragma unroll
                            for (int jj = 0; jj < D::N8; jj++) q8[jj] = *reinterpret_cast<const uint2*>(rp + D::off8(uu, c, jj));
                            const uint16_t db =
                                D::DPL ? *reinterpret_cast<const uint16_t*>(st + m * RS::BYTES + RS::DOFF + row * 2) : 0;
                            if (r == 0) D::template decode<0>(q16, q8, c, db, afr);
                            else D::template decode<1>(q16, q8, c, db, afr);
                        }
#pragma unroll
                        for (int s8 = 0; s8 < 8; s8++) {
#pragma unroll
                            for (int t = 0; t < NTT; t++) {
                                if (NTT == 1 || t < ntl) {
                                    const uint2 b = bu[(s8 * NTT + t) * 32];
                                    mma_f16_16816(acc[m][t], afr[s8], b.x, b.y);
                                }
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&empty[s]));  // this warp is done with the stage
                if (++s == depth) {
                    s = 0;
                    phase ^= 1u;
                }
            }
            // after a timeout the warps skip the stages and the stores but keep walking the items,
            // so that every consumer warp takes the same named-barrier steps
            if (s_abort) continue;

            // accumulator (m, t, q): weight row 16 rg + g + 8 (q >> 1), token row 8 t + 2 c + (q & 1)
            const int fb = rblk * CONS + rg;  // 16-row block of the output features
            const int f = fb * 16 + g;
            if (NMAT == 2) {
                const int hstride = p.I / GV_EBLK;
#pragma unroll
                for (int t = 0; t < NTT; t++) {
                    float hv[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) hv[q] = silu_ref(acc[0][t][q]) * acc[NMAT - 1][t][q];  // src/moe.rs:280-283
                    float m0 = fmaxf(fabsf(hv[0]), fabsf(hv[2])), m1 = fmaxf(fabsf(hv[1]), fabsf(hv[3]));
#pragma unroll
                    for (int off = 4; off < 32; off <<= 1) {
                        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
                        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
                    }
#pragma unroll
                    for (int jn = 0; jn < 2; jn++) {
                        const int n = 8 * t + 2 * c + jn;
                        if (n < nrows) {
                            const int ex = block_exp(jn ? m1 : m0);
                            const float sc = exp2i(-ex);
                            const size_t r = (size_t)(row0 + n);
                            p.h[r * p.I + f] = __float2half_rn(__fmul_rn(hv[jn], sc));
                            p.h[r * p.I + f + 8] = __float2half_rn(__fmul_rn(hv[jn + 2], sc));
                            if (g == 0) {
                                p.hexp[r * hstride + fb] = (int8_t)ex;
                                atomicMax(p.rowexp + r, ex);
                            }
                        }
                    }
                }
            } else {
#pragma unroll
                for (int t = 0; t < NTT; t++)
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int n = 8 * t + 2 * c + (q & 1);
                        if (n < nrows) {
                            const int fo = f + 8 * (q >> 1);
                            const float yv = __fmul_rn(acc[0][t][q], exp2i(s_rexp[n]));
                            if (p.y) p.y[(size_t)(row0 + n) * p.H + fo] = yv;
                            else atomicAdd(p.out + (size_t)s_tok[n] * p.H + fo, __fmul_rn(s_w[n], yv));
                        }
                    }
            }
        }
    }
    // a CTA that stopped early exits only after the copies it issued have landed
    __syncthreads();
    if (warp == CONS && lane == 0 && s_abort)
        for (int j = s_consumed; j < issued; j++)
            if (!mbar_wait(smem_u32(&full[j % depth]), (j / depth) & 1, 100000000ull)) break;
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int TYPE, int NT, int NMAT, int CONS>
static cudaError_t go_gvt(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s) {
    constexpr int RB = 16 * CONS;
    using G = GvtGeom<TYPE, NMAT, RB>;
    const int K = NMAT == 2 ? p.H : p.I, rows = NMAT == 2 ? p.I : p.H;
    if (rows % RB || K % Raw<TYPE>::RK) return cudaErrorNotSupported;
    const size_t ring_off = ((size_t)K * NT * 2 + 127) & ~(size_t)127;
    // shared memory that keeps gvt_ctas_per_sm CTAs on an SM
    const size_t budget = CONS == 4 ? (size_t)74 * 1024 : (size_t)GV_SMEM_TWO;
    if (ring_off >= budget) return cudaErrorNotSupported;
    int depth = (int)std::min<size_t>(GVT_MAXD, (budget - ring_off) / G::STAGE);
    if (depth < 2) return cudaErrorNotSupported;
    const size_t smem = ring_off + (size_t)depth * G::STAGE;
    auto k = gvt_kernel<TYPE, NT, NMAT, CONS>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // down: persistent, two CTAs per SM (the shared-memory budget), each walking a range of items
    static int n_sm = 0;
    if (!n_sm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
        if (n_sm <= 0) n_sm = 148;
    }
    const int items = max_tiles * (rows / RB);
    const dim3 grid = gvt_persistent(NMAT) ? dim3(std::min(items, 2 * n_sm)) : dim3(rows / RB, max_tiles);
    return launch_pdl(k, grid, dim3(32 * (CONS + 1)), smem, s, p, maps, depth, (int)ring_off);
}

template <int NMAT, int CONS>
static cudaError_t go_gvt_type(int type, const GroupedParams& p, const TcMaps& maps, int max_tiles, int nt,
                               cudaStream_t s) {
    switch (type) {
        case T_Q4_K:
            return nt == 8 ? go_gvt<T_Q4_K, 8, NMAT, CONS>(p, maps, max_tiles, s)
                           : go_gvt<T_Q4_K, 16, NMAT, CONS>(p, maps, max_tiles, s);
        case T_Q6_K:
            return nt == 8 ? go_gvt<T_Q6_K, 8, NMAT, CONS>(p, maps, max_tiles, s)
                           : go_gvt<T_Q6_K, 16, NMAT, CONS>(p, maps, max_tiles, s);
        default: return cudaErrorNotSupported;
    }
}

cudaError_t launch_gvt_gateup(const GroupedParams& p, const TcMaps& maps, const TcMaps* maps64, int max_tiles, int nt,
                              cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    if (maps64 && nt == 8) {
        const cudaError_t e = go_gvt_type<2, 4>(p.gate.type, p, *maps64, max_tiles, nt, s);
        if (e != cudaErrorNotSupported) return e;
    }
    return go_gvt_type<2, 8>(p.gate.type, p, maps, max_tiles, nt, s);
}

cudaError_t launch_gvt_down(const GroupedParams& p, const TcMaps& maps, int max_tiles, int nt, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    return go_gvt_type<1, 8>(p.down.type, p, maps, max_tiles, nt, s);
}

}  // namespace rmoe
