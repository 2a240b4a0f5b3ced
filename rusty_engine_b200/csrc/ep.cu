// ep.cu -- expert-parallel layers: the experts split over G ranks (one GPU each), NCCL
// send/recv exchanges between them.
//
// Each rank holds a subset of the experts and the whole router.  The placement is either the
// caller's (expert_rank[e] = the rank holding e, e.g. balanced by measured expert loads) or
// round-robin (rank r holds experts r, r + G, r + 2G, ..., so the most popular experts of a
// skewed load land on different ranks); a rank's local ids number its experts in ascending
// global order.  A forward on rank r takes r's own T tokens:
//   1. router logits + top-k over all E experts (the same kernels as a whole layer);
//   2. plan: for every destination rank d, which tokens have at least one pick on d (each such
//      token is sent to d once, however many of its picks d holds) and their order (token
//      order, by a per-destination scan);
//   3. counts exchange (one int per peer) and one device-to-host read of the counts, which
//      size the payload calls (the pack of step 4 is queued behind that read and runs while the
//      host waits);
//   4. pack + exchange: a row per (token, destination): the token's fp16 activations followed
//      by its k picks as seen by d (d's local expert id, or the empty id = d's expert count, and
//      the weight);
//   5. d runs its local experts over the rows it received with the given routing (the grouped
//      tensor-core or small-batch kernels), producing per received row the weighted sum of its
//      local picks' outputs (f32);
//   6. those partial sums go back to the token's rank, which adds them in ascending rank order.
// A shared expert (src/moe.rs:381-386) is replicated on every rank: each rank sends every one of
// its tokens to itself and runs the shared expert on exactly those rows, so each token gets it
// once, at weight 1, inside its own rank's partial sum.
// There is no counterpart in the reference (its moe_layer_forward runs in one process,
// src/moe.rs:360-388); the sum over a token's experts is regrouped by rank, which changes
// only the f32 summation order.
#include <nccl.h>
#include <stdlib.h>

#include <chrono>
#include <thread>
#include <vector>

#include "../../include/rmoe.h"
#include "kernels.h"
#include "layer_impl.h"

namespace rmoe {

struct EpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    Owned tok_own;  // per-token buffers, sized for capT tokens
    uint32_t capT = 0, lastT = 0;
    __half* xb = nullptr;
    float* logits = nullptr;
    float* logits_part = nullptr;  // K-split partial router logits (large batches)
    int* topk_id = nullptr;
    float* topk_w = nullptr;
    float* xin = nullptr;    // host-IO staging
    float* xout = nullptr;
    int* pos = nullptr;      // [T][G]: row of the token in d's block, -1 when not sent to d
    int* cnt = nullptr;      // [2G]: send counts, then receive counts
    unsigned* status = nullptr;
    unsigned* ticket = nullptr;  // router last-CTA counters (0 between launches)
    int* h_cnt = nullptr;    // pinned copy of cnt
    int* map = nullptr;      // device [E rank of e][E local id of e][G experts on rank d]
    Owned send_own, recv_own;
    uint64_t cap_send = 0, cap_recv = 0;  // rows
    uint8_t* sendbuf = nullptr;
    float* ret = nullptr;    // [send rows][H] partial sums coming back
    uint8_t* recvbuf = nullptr;
    float* part = nullptr;   // [recv rows][H] partial sums computed here
    int timeout_ms = 120000;      // no progress for this long: the communicator is aborted
    cudaEvent_t ev = nullptr;     // host waits go through this event
    ~EpState() {
        if (ev) cudaEventDestroy(ev);
        if (h_cnt) cudaFreeHost(h_cnt);
        if (comm) ncclCommDestroy(comm);
    }
};

static inline uint32_t row_bytes(uint32_t H, uint32_t k) { return (H * 2 + k * 8 + 15) & ~15u; }

// Largest worst-case send buffer (tokens x ranks rows) that is allocated so that the pack can
// be queued before the host has read the counts.
static constexpr uint64_t PACK_EARLY_BYTES = 1ull << 30;

// 2. one CTA per destination: flags and the exclusive scan over tokens (every token goes to
// rank `self_all` itself when that is >= 0: the shared expert runs there)
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int* topk_id, int T, int k, const int* rank_of, int G,
                                                       int* pos, int* cnt, int self_all) {
    __shared__ int warp_sum[32];
    __shared__ int carry_s;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += 1024) {
        const int t = t0 + tid;
        int f = 0;
        if (t < T) {
            for (int j = 0; j < k; j++) f |= rank_of[topk_id[(size_t)t * k + j]] == d;
            if (d == self_all) f = 1;
        }
        int inc = f;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += o;
        }
        if (lane == 31) warp_sum[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            int v = warp_sum[lane];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, v, off);
                if (lane >= off) v += o;
            }
            warp_sum[lane] = v;  // inclusive over warps
        }
        __syncthreads();
        const int before = carry_s + (warp ? warp_sum[warp - 1] : 0) + inc - f;
        if (t < T) pos[(size_t)t * G + d] = f ? before : -1;
        __syncthreads();
        if (tid == 0) carry_s += warp_sum[31];
        __syncthreads();
    }
    if (tid == 0) cnt[d] = carry_s;
}

// 4. one warp per (token, destination): the row for d
__global__ void __launch_bounds__(256) ep_pack_kernel(const __half* xb, const int* topk_id, const float* topk_w,
                                                      const int* pos, const int* cnt, int T, int H, int k,
                                                      const int* map, int E, int G, uint32_t rb, uint8_t* sendbuf) {
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wid >= T * G) return;
    const int t = wid / G, d = wid - t * G;
    const int pr = pos[(size_t)t * G + d];
    if (pr < 0) return;
    int soff = 0;
    for (int q = 0; q < d; q++) soff += cnt[q];
    uint8_t* row = sendbuf + (size_t)(soff + pr) * rb;
    const uint4* src = reinterpret_cast<const uint4*>(xb + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(row);
    for (int u = lane; u < H / 8; u += 32) dst[u] = src[u];
    if (lane < k) {
        const int id = topk_id[(size_t)t * k + lane];
        const bool mine = map[id] == d;
        reinterpret_cast<int*>(row + (size_t)H * 2)[lane] = mine ? map[E + id] : map[2 * E + d];
        reinterpret_cast<float*>(row + (size_t)H * 2 + k * 4)[lane] = mine ? topk_w[(size_t)t * k + lane] : 0.0f;
    }
}

// 5a. one warp per received row: activations and routing into the local workspace
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* recvbuf, int R, int H, int k, uint32_t rb,
                                                        __half* xb, int* topk_id, float* topk_w) {
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (r >= R) return;
    const uint8_t* row = recvbuf + (size_t)r * rb;
    const uint4* src = reinterpret_cast<const uint4*>(row);
    uint4* dst = reinterpret_cast<uint4*>(xb + (size_t)r * H);
    for (int u = lane; u < H / 8; u += 32) dst[u] = src[u];
    if (lane < k) {
        topk_id[(size_t)r * k + lane] = reinterpret_cast<const int*>(row + (size_t)H * 2)[lane];
        topk_w[(size_t)r * k + lane] = reinterpret_cast<const float*>(row + (size_t)H * 2 + k * 4)[lane];
    }
}

// 6. out[t] = sum over the ranks d the token went to, ascending, of the partial sum from d
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* ret, const int* pos, const int* cnt, int T, int H,
                                                         int G, float* out) {
    const int t = blockIdx.x;
    int rows[16];
    int soff = 0;
    for (int d = 0; d < G; d++) {
        const int pr = pos[(size_t)t * G + d];
        rows[d] = pr < 0 ? -1 : soff + pr;
        soff += cnt[d];
    }
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int d = 0; d < G; d++) {
            if (rows[d] < 0) continue;
            const float4 v = *reinterpret_cast<const float4*>(ret + (size_t)rows[d] * H + i);
            o.x = __fadd_rn(o.x, v.x);
            o.y = __fadd_rn(o.y, v.y);
            o.z = __fadd_rn(o.z, v.z);
            o.w = __fadd_rn(o.w, v.w);
        }
        *reinterpret_cast<float4*>(out + (size_t)t * H + i) = o;
    }
}

static rmoe_status nccl_fail(ncclResult_t r, const char* what) {
    return fail(RMOE_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

// Failure detection.  The communicator is non-blocking, and every host wait of an
// expert-parallel call polls both the GPU work and the communicator's asynchronous error: an
// NCCL error, or no progress for timeout_ms (a peer rank that stopped, so the exchange kernels
// wait for it), aborts the communicator -- which ends its kernels -- and the call returns
// RMOE_ERR_NCCL; every later call on the handle returns the same.
static rmoe_status ep_abort(EpState& P, rmoe_status st) {
    if (P.comm) ncclCommAbort(P.comm);
    P.comm = nullptr;
    return st;
}

static rmoe_status ep_poll(EpState& P, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    // The count read of every forward waits here for tens of microseconds: the first 2 ms of a
    // wait poll back to back (a 50-us sleep would add its whole length to each forward), later
    // polls sleep between queries.
    for (;;) {
        cudaError_t q = P.ev ? cudaEventQuery(P.ev) : cudaSuccess;
        ncclResult_t a = ncclSuccess;
        if (ncclCommGetAsyncError(P.comm, &a) != ncclSuccess || (a != ncclSuccess && a != ncclInProgress))
            return ep_abort(P, nccl_fail(a, what));
        if (q == cudaSuccess && a == ncclSuccess) return RMOE_OK;
        if (q != cudaSuccess && q != cudaErrorNotReady) return cuda_fail(q, what);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms > P.timeout_ms)
            return ep_abort(P, fail(RMOE_ERR_NCCL, "%s: no progress for %d ms (a peer rank stopped?); the communicator "
                                                   "was aborted", what, P.timeout_ms));
        if (ms < 2) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// After ncclGroupEnd on the non-blocking communicator: wait until the group is enqueued.
static rmoe_status ep_enqueued(EpState& P, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return RMOE_OK;
    if (r != ncclInProgress) return ep_abort(P, nccl_fail(r, what));
    cudaEvent_t keep = P.ev;
    P.ev = nullptr;  // poll the communicator alone
    rmoe_status st = ep_poll(P, what);
    P.ev = keep;
    return st;
}

// Wait, bounded, for the work queued on s so far.
static rmoe_status ep_sync(EpState& P, cudaStream_t s, const char* what) {
    cudaError_t e = cudaEventRecord(P.ev, s);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return ep_poll(P, what);
}

static rmoe_status ep_token_buffers(rmoe_layer* L, uint32_t T) {
    EpState& P = *L->ep;
    if (T <= P.capT) return RMOE_OK;
    cudaDeviceSynchronize();
    P.tok_own.~Owned();
    new (&P.tok_own) Owned();
    const uint32_t cap = (T + 255) / 256 * 256, G = P.world;
    bool ok = true;
    auto A = [&](size_t n) { void* p = P.tok_own.alloc(n); ok = ok && p; return p; };
    P.xb = (__half*)A((size_t)cap * L->H * 2);
    P.xin = (float*)A((size_t)cap * L->H * 4);
    P.xout = (float*)A((size_t)cap * L->H * 4);
    P.logits = (float*)A((size_t)cap * L->E_router * 4);
    P.logits_part = (float*)A((size_t)LOGIT_SPLITS * cap * L->E_router * 4);
    P.topk_id = (int*)A((size_t)cap * L->k * 4);
    P.topk_w = (float*)A((size_t)cap * L->k * 4);
    P.pos = (int*)A((size_t)cap * G * 4);
    P.cnt = (int*)A((size_t)2 * G * 4);
    P.status = (unsigned*)A(16);
    P.ticket = (unsigned*)A(64);
    if (!ok) return fail(RMOE_ERR_OOM, "expert-parallel token buffers for %u tokens", cap);
    cudaMemset(P.status, 0, 16);
    cudaMemset(P.ticket, 0, 64);
    P.capT = cap;
    return RMOE_OK;
}

static rmoe_status grow(Owned& own, uint64_t rows, uint64_t& cap, uint32_t rb, uint32_t H, uint8_t** buf, float** f) {
    if (rows <= cap) return RMOE_OK;
    cudaDeviceSynchronize();
    own.~Owned();
    new (&own) Owned();
    const uint64_t c = (rows + 255) / 256 * 256;
    *buf = (uint8_t*)own.alloc(c * rb);
    *f = (float*)own.alloc(c * H * 4);
    if (!*buf || !*f) {
        cap = 0;
        return fail(RMOE_ERR_OOM, "expert-parallel exchange buffers for %llu rows", (unsigned long long)c);
    }
    cap = c;
    return RMOE_OK;
}

rmoe_status ep_forward(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s, uint32_t flags) {
    EpState& P = *L->ep;
    const int G = P.world, H = (int)L->H, k = (int)L->k;
    const uint32_t rb = row_bytes(L->H, L->k);
    if (!P.comm) return fail(RMOE_ERR_NCCL, "expert-parallel layer: the communicator was aborted by an earlier failure");
    rmoe_status st = ep_token_buffers(L, T ? T : 1);
    if (st) return st;
    cudaError_t e;
    // 1. router + top-k over all experts
    RouteParams rp{};
    rp.x = x; rp.router_w = L->router_w; rp.router_wh = L->router_wh; rp.router_wl = L->router_wl; rp.T = (int)T; rp.H = H; rp.E = (int)L->E_router; rp.k = k;
    rp.exact = (flags & RMOE_FLAG_EXACT_ROUTER) ? 1 : 0;
    rp.gate = (int)L->gate_kind; rp.xb = P.xb; rp.logits = P.logits; rp.topk_id = P.topk_id; rp.topk_w = P.topk_w;
    rp.logits_part = rp.exact ? nullptr : P.logits_part;
    rp.status = P.status; rp.ticket = P.ticket;
    rp.router_wmax = L->router_wmax; rp.refined = P.status + 1;
    if (T && (e = launch_router_topk(rp, s)) != cudaSuccess) return cuda_fail(e, "ep router launch");
    // 2. plan
    ep_plan_kernel<<<G, 1024, 0, s>>>(P.topk_id, (int)T, k, P.map, G, P.pos, P.cnt, L->has_shared ? P.rank : -1);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "ep plan launch");
    // 3. counts
    ncclResult_t r = ncclGroupStart();
    for (int q = 0; q < G && r == ncclSuccess; q++) {
        r = ncclSend(P.cnt + q, 1, ncclInt32, q, P.comm, s);
        if (r == ncclSuccess) r = ncclRecv(P.cnt + G + q, 1, ncclInt32, q, P.comm, s);
    }
    ncclResult_t r2 = ncclGroupEnd();
    if (r != ncclSuccess) return ep_abort(P, nccl_fail(r, "ep counts exchange"));
    if ((st = ep_enqueued(P, r2, "ep counts exchange"))) return st;
    if ((e = cudaMemcpyAsync(P.h_cnt, P.cnt, 2 * G * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
        return cuda_fail(e, "ep counts");
    if ((e = cudaEventRecord(P.ev, s)) != cudaSuccess) return cuda_fail(e, "ep counts");
    // 4a. pack: it needs only the device-side counts, so with a send buffer sized for the worst
    // case (every token sent to every rank; up to PACK_EARLY_BYTES) it is queued behind the
    // count read and runs while the host waits for the counts
    const bool early = T && (uint64_t)T * G * rb <= PACK_EARLY_BYTES;
    auto pack = [&]() -> rmoe_status {
        ep_pack_kernel<<<(T * G + 7) / 8, 256, 0, s>>>(P.xb, P.topk_id, P.topk_w, P.pos, P.cnt, (int)T, H, k, P.map,
                                                       (int)L->E_router, G, rb, P.sendbuf);
        cudaError_t le = cudaGetLastError();
        return le == cudaSuccess ? RMOE_OK : cuda_fail(le, "ep pack launch");
    };
    if (early) {
        if ((st = grow(P.send_own, (uint64_t)T * G, P.cap_send, rb, L->H, &P.sendbuf, &P.ret))) return st;
        if ((st = pack())) return st;
    }
    if ((st = ep_poll(P, "ep counts"))) return st;
    std::vector<uint64_t> soff(G + 1, 0), roff(G + 1, 0);
    for (int q = 0; q < G; q++) {
        soff[q + 1] = soff[q] + (uint64_t)P.h_cnt[q];
        roff[q + 1] = roff[q] + (uint64_t)P.h_cnt[G + q];
    }
    const uint64_t S = soff[G], R = roff[G];
    if ((st = grow(P.send_own, S, P.cap_send, rb, L->H, &P.sendbuf, &P.ret))) return st;
    if ((st = grow(P.recv_own, R, P.cap_recv, rb, L->H, &P.recvbuf, &P.part))) return st;
    // 4b. pack (when not queued early) + exchange
    if (T && !early && (st = pack())) return st;
    r = ncclGroupStart();
    for (int q = 0; q < G && r == ncclSuccess; q++) {
        if (P.h_cnt[q]) r = ncclSend(P.sendbuf + soff[q] * rb, (size_t)P.h_cnt[q] * rb, ncclUint8, q, P.comm, s);
        if (r == ncclSuccess && P.h_cnt[G + q])
            r = ncclRecv(P.recvbuf + roff[q] * rb, (size_t)P.h_cnt[G + q] * rb, ncclUint8, q, P.comm, s);
    }
    r2 = ncclGroupEnd();
    if (r != ncclSuccess) return ep_abort(P, nccl_fail(r, "ep dispatch exchange"));
    if ((st = ep_enqueued(P, r2, "ep dispatch exchange"))) return st;
    // 5. local experts over the received rows
    if (R) {
        if ((st = ensure_workspace(L, (uint32_t)R, flags & RMOE_FLAG_DETERMINISTIC))) return st;
        ep_unpack_kernel<<<(unsigned)((R + 7) / 8), 256, 0, s>>>(P.recvbuf, (int)R, H, k, rb, L->ws.xb, L->ws.topk_id,
                                                                 L->ws.topk_w);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "ep unpack launch");
        // the rows this rank sent itself (all its tokens, in token order, when the layer has a
        // shared expert) also take the shared expert, at weight 1 (src/moe.rs:381-386)
        if ((st = layer_forward_device(L, nullptr, (uint32_t)R, P.part, s, flags & ~RMOE_FLAG_STAGE_TIMING, true,
                                       (uint32_t)roff[P.rank], L->has_shared ? (int64_t)P.h_cnt[G + P.rank] : 0)))
            return st;
    }
    // 6. partial sums back, combined in rank order
    r = ncclGroupStart();
    for (int q = 0; q < G && r == ncclSuccess; q++) {
        if (P.h_cnt[G + q])
            r = ncclSend(P.part + roff[q] * H, (size_t)P.h_cnt[G + q] * H, ncclFloat32, q, P.comm, s);
        if (r == ncclSuccess && P.h_cnt[q])
            r = ncclRecv(P.ret + soff[q] * H, (size_t)P.h_cnt[q] * H, ncclFloat32, q, P.comm, s);
    }
    r2 = ncclGroupEnd();
    if (r != ncclSuccess) return ep_abort(P, nccl_fail(r, "ep combine exchange"));
    if ((st = ep_enqueued(P, r2, "ep combine exchange"))) return st;
    if (T) {
        ep_combine_kernel<<<T, 256, 0, s>>>(P.ret, P.pos, P.cnt, (int)T, H, G, out);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "ep combine launch");
    }
    P.lastT = T;
    L->last_T = T;
    return RMOE_OK;
}

// Host buffers in and out, copies inside the call (synchronises the stream).
rmoe_status ep_forward_host(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s, uint32_t flags) {
    EpState& P = *L->ep;
    if (!P.comm) return fail(RMOE_ERR_NCCL, "expert-parallel layer: the communicator was aborted by an earlier failure");
    rmoe_status st = ep_token_buffers(L, T ? T : 1);
    if (st) return st;
    cudaError_t e = cudaMemcpyAsync(P.xin, x, (size_t)T * L->H * 4, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "x upload");
    if ((st = ep_forward(L, P.xin, T, P.xout, s, flags & ~RMOE_FLAG_HOST_IO))) return st;
    if ((e = cudaMemcpyAsync(out, P.xout, (size_t)T * L->H * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
        return cuda_fail(e, "out download");
    if ((st = ep_sync(P, s, "forward"))) return st;
    return RMOE_OK;
}

unsigned* ep_status(rmoe_layer* L) { return L->ep ? L->ep->status : nullptr; }

void ep_free(rmoe_layer* L) {
    delete L->ep;
    L->ep = nullptr;
}

}  // namespace rmoe

using namespace rmoe;

extern "C" {

rmoe_status rmoe_ep_unique_id(uint8_t id[128]) {
    if (!id) return fail(RMOE_ERR_INVALID, "null id buffer");
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(RMOE_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    static_assert(sizeof(u.internal) == 128, "NCCL unique id is 128 bytes");
    for (int i = 0; i < 128; i++) id[i] = (uint8_t)u.internal[i];
    return RMOE_OK;
}

rmoe_status rmoe_ep_layer_create(const rmoe_layer_desc* d, int32_t rank, int32_t world_size, const uint8_t id[128],
                                 rmoe_layer** out) {
    if (d && world_size >= 1 && d->n_experts % (uint32_t)world_size)
        return fail(RMOE_ERR_INVALID, "%u experts do not split evenly over %d ranks", d->n_experts, world_size);
    return rmoe_ep_layer_create_placed(d, rank, world_size, id, nullptr, out);
}

rmoe_status rmoe_ep_layer_create_placed(const rmoe_layer_desc* d, int32_t rank, int32_t world_size,
                                        const uint8_t id[128], const int32_t* expert_rank, rmoe_layer** out) {
    if (!out) return fail(RMOE_ERR_INVALID, "null output handle pointer");
    *out = nullptr;
    rmoe_status s = validate_desc(d);
    if (s) return s;
    if (!id) return fail(RMOE_ERR_INVALID, "null NCCL unique id");
    if (world_size < 1 || world_size > 16 || rank < 0 || rank >= world_size)
        return fail(RMOE_ERR_INVALID, "rank %d / world size %d (1..16 ranks)", rank, world_size);
    // the placement table: rank of each expert, its local id there, the expert count per rank
    const uint32_t E = d->n_experts, G = (uint32_t)world_size;
    std::vector<int> map(2 * E + G, 0);
    std::vector<uint32_t> mine;
    for (uint32_t e = 0; e < E; e++) {
        const int32_t r = expert_rank ? expert_rank[e] : (int32_t)(e % G);
        if (r < 0 || r >= world_size)
            return fail(RMOE_ERR_INVALID, "expert_rank[%u] = %d is not a rank of %d", e, r, world_size);
        map[e] = r;
        map[E + e] = map[2 * E + r]++;
        if (r == rank) mine.push_back(e);
    }
    for (uint32_t r = 0; r < G; r++)
        if (!map[2 * E + r]) return fail(RMOE_ERR_INVALID, "rank %u holds no expert (every rank needs at least one)", r);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(RMOE_ERR_CUDA, "no CUDA device");
    if (d->device < 0 || d->device >= ndev) return fail(RMOE_ERR_INVALID, "device %d out of range", d->device);
    DeviceGuard g(d->device);
    rmoe_layer* L = new rmoe_layer();
    L->device = d->device;
    L->H = d->hidden; L->I = d->inter;
    L->E_router = d->n_experts;
    L->E = L->E_local = (uint32_t)mine.size();
    L->k = d->top_k < d->n_experts ? d->top_k : d->n_experts;
    L->gate_kind = d->gate;
    L->has_shared = d->has_shared ? 1 : 0;  // the shared expert is replicated on every rank
    if ((s = layer_upload(d, mine.data(), L->E, L))) { delete L; return s; }
    int* dmap = static_cast<int*>(L->own.alloc(map.size() * sizeof(int)));
    if (!dmap) { delete L; return fail(RMOE_ERR_OOM, "expert placement table"); }
    cudaError_t me = cudaMemcpy(dmap, map.data(), map.size() * sizeof(int), cudaMemcpyHostToDevice);
    if (me != cudaSuccess) { delete L; return cuda_fail(me, "expert placement table"); }
    L->ep = new EpState();
    L->ep->map = dmap;
    L->ep->rank = rank;
    L->ep->world = world_size;
    if (cudaMallocHost(&L->ep->h_cnt, 2 * world_size * sizeof(int)) != cudaSuccess) {
        delete L;
        return fail(RMOE_ERR_OOM, "pinned count buffer");
    }
    if (const char* t = getenv("RMOE_EP_TIMEOUT_MS")) {
        const long v = strtol(t, nullptr, 10);
        if (v > 0) L->ep->timeout_ms = (int)v;
    }
    if (cudaEventCreateWithFlags(&L->ep->ev, cudaEventDisableTiming) != cudaSuccess) {
        delete L;
        return fail(RMOE_ERR_CUDA, "expert-parallel event");
    }
    ncclUniqueId u;
    for (int i = 0; i < 128; i++) u.internal[i] = (char)id[i];
    // non-blocking communicator: the init (which waits for every rank) and every later wait are
    // polled with the timeout instead of blocking for good on a rank that never comes
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&L->ep->comm, world_size, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (L->ep->comm) ncclCommAbort(L->ep->comm);
        L->ep->comm = nullptr;
        delete L;
        return nccl_fail(r, "ncclCommInitRankConfig");
    }
    cudaEvent_t keep = L->ep->ev;
    L->ep->ev = nullptr;
    rmoe_status ist = ep_poll(*L->ep, "ncclCommInitRankConfig (waiting for every rank to join)");
    L->ep->ev = keep;
    if (ist) {
        delete L;
        return ist;
    }
    *out = L;
    return RMOE_OK;
}

}  // extern "C"

namespace rmoe {
// routing / logits of the last expert-parallel forward (this rank's tokens)
rmoe_status ep_routing(rmoe_layer* L, uint32_t T, uint32_t* ids, float* weights, float* logits) {
    EpState& P = *L->ep;
    if (T > P.lastT) return fail(RMOE_ERR_INVALID, "%u tokens requested, last forward had %u", T, P.lastT);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess && ids) e = cudaMemcpy(ids, P.topk_id, (size_t)T * L->k * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && weights) e = cudaMemcpy(weights, P.topk_w, (size_t)T * L->k * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && logits) e = cudaMemcpy(logits, P.logits, (size_t)T * L->E_router * 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "ep routing");
}
}  // namespace rmoe
