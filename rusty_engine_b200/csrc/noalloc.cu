// noalloc.cu -- the MoE layer forward for small batches with no device allocation at call time.
//
// rmoe_layer_forward sizes its per-forward scratch (routing tables, expert-sorted rows, SwiGLU
// activations) with cudaMalloc on first use and whenever the batch grows.  Some callers cannot
// allocate there: serving runtimes that reserve all device memory up front for their own pool
// (weights, KV cache), where a late cudaMalloc fails or fragments that reservation, and decode
// loops where cudaMalloc's implicit device synchronisation would stall the other streams.
// rmoe_layer_forward_noalloc runs the same kernels (router + dispatch, mma.sync gate/up, down
// with the atomic weighted combine) on scratch carved from one file-scope device array of
// RMOE_NOALLOC_SCRATCH_BYTES, which is part of the library's device image: every GPU that loads
// the library holds it until the process exits.
//
// The array's address is looked up once per device (cudaGetSymbolAddress, with that device
// current) by the first call of the entry point on that device.  The array keeps the previous
// call's contents; the entry point clears the words that must start at zero (dispatch ticket,
// status word) on the caller's stream and the kernels overwrite everything else before reading
// it.  All calls on a device share the one array, so calls that overlap on the GPU (different
// streams, or different layers on concurrent streams) race on it.
#include <string.h>

#include <mutex>

#include <algorithm>

#include "layer_impl.h"

namespace rmoe {

// The scratch itself.  In host code `g_noalloc_scratch` names a host-side stand-in for the
// symbol, not a device address: the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[RMOE_NOALLOC_SCRATCH_BYTES];

static constexpr int MAX_DEVICES = 64;
static std::mutex g_setup_mu;
static void* g_scratch_ptr[MAX_DEVICES] = {};

// Device address of the scratch on `dev` (current); set up on the first call per device.
static rmoe_status scratch_on(int dev, unsigned char** out) {
    if (dev < 0 || dev >= MAX_DEVICES) return fail(RMOE_ERR_INVALID, "device %d out of range", dev);
    std::lock_guard<std::mutex> g(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_scratch_ptr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
    return RMOE_OK;
}

// Carves 256-B-aligned pieces off the scratch; `used` is the running total, so one pass with a
// null base measures a batch's need and a second pass hands out the pointers.
struct Carver {
    unsigned char* base;
    size_t used = 0;
    template <class T>
    T* take(size_t bytes) {
        T* p = base ? reinterpret_cast<T*>(base + used) : nullptr;
        used += (bytes + 255) & ~size_t(255);
        return p;
    }
};

// The small-batch path's workspace for T tokens (the subset of Workspace those kernels read).
static void carve(Carver& c, const rmoe_layer* L, uint32_t T, uint64_t rows, int max_tiles, Workspace& w) {
    const size_t H = L->H, I = L->I, E = L->E, k = L->k;
    w.ticket = c.take<unsigned>(64);
    w.status = c.take<unsigned>(16);
    w.n_rows = c.take<int>(16);
    w.n_tiles = c.take<int>(16);
    w.xb = c.take<__half>((size_t)T * H * 2);
    w.logits = c.take<float>((size_t)T * E * 4);
    w.topk_id = c.take<int>((size_t)T * k * 4);
    w.topk_w = c.take<float>((size_t)T * k * 4);
    w.local_rank = c.take<int>((size_t)T * k * 4);
    w.slot_row = c.take<int>((size_t)T * k * 4);
    w.cta_cnt = c.take<int>((size_t)route_cnt_stride(route_grid((int)T)) * E * 4);
    w.expert_off = c.take<int>((E + 2) * 4);
    w.row_tok = c.take<int>(rows * 4);
    w.row_slot = c.take<int>(rows * 4);
    w.tiles = c.take<int4>((size_t)max_tiles * 16);
    w.h = c.take<__half>(rows * I * 2);
    w.hexp = c.take<int8_t>(rows * (I / GV_EBLK));
    w.rowexp = c.take<int>(rows * 4);
}

}  // namespace rmoe

using namespace rmoe;

extern "C" {

rmoe_status rmoe_layer_forward_noalloc(rmoe_layer* L, const float* x, uint32_t T, float* out, void* stream) {
    if (!L) return fail(RMOE_ERR_INVALID, "null layer");
    if (T == 0) return RMOE_OK;
    if (!x || !out) return fail(RMOE_ERR_INVALID, "null x / out");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(RMOE_ERR_INVALID, "device x / out must be 16-byte aligned");
    if (L->ep) return fail(RMOE_ERR_UNSUPPORTED, "noalloc forward: expert-parallel layers are not supported");
    const uint64_t rows = (uint64_t)T * L->k + (L->has_shared ? T : 0);
    const bool gv = gv_supported(L->wg.type, L->wd.type);
    const int nt = gv ? gv_tile_rows((int)T) : small_tile_rows((int)T);
    const int max_tiles = (int)(rows / nt + std::min<uint64_t>(L->E + 2, rows));
    Workspace w{};
    Carver measure{nullptr};
    carve(measure, L, T, rows, max_tiles, w);
    if (measure.used > (size_t)RMOE_NOALLOC_SCRATCH_BYTES)
        return fail(RMOE_ERR_INVALID,
                    "noalloc forward: %u tokens of this layer need %zu bytes of scratch, the static scratch holds %u; "
                    "use rmoe_layer_forward for this batch",
                    T, measure.used, (unsigned)RMOE_NOALLOC_SCRATCH_BYTES);
    DeviceGuard g(L->device);
    unsigned char* base = nullptr;
    rmoe_status st = scratch_on(L->device, &base);
    if (st) return st;
    Carver c{base};
    carve(c, L, T, rows, max_tiles, w);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(base, 0, 2 * 256, s);  // ticket and status start at zero
    if (e != cudaSuccess) return cuda_fail(e, "noalloc scratch clear");

    RouteParams rp{};
    rp.x = x;
    rp.router_w = L->router_w;
    rp.T = (int)T; rp.H = (int)L->H; rp.E = (int)L->E; rp.k = (int)L->k; rp.gate = (int)L->gate_kind;
    rp.has_shared = L->has_shared;
    rp.shared_t0 = 0; rp.shared_n = (int)T;
    rp.xb = w.xb; rp.rowexp = w.rowexp; rp.xs = nullptr; rp.logits = w.logits;
    rp.out_zero = out;  // the atomic combine accumulates into zeroed rows
    rp.topk_id = w.topk_id; rp.topk_w = w.topk_w; rp.local_rank = w.local_rank; rp.cta_cnt = w.cta_cnt;
    rp.ticket = w.ticket; rp.expert_off = w.expert_off; rp.row_tok = w.row_tok; rp.row_slot = w.row_slot;
    rp.slot_row = w.slot_row; rp.n_rows = w.n_rows; rp.tiles = w.tiles; rp.n_tiles = w.n_tiles;
    rp.max_tiles = max_tiles; rp.tile_rows = nt; rp.status = w.status;
    rp.router_wmax = L->router_wmax; rp.refined = w.status + 1;
    if ((e = launch_route_dispatch(rp, s)) != cudaSuccess) return cuda_fail(e, "noalloc route_dispatch launch");

    GroupedParams gp{};
    gp.gate = L->wg; gp.up = L->wu; gp.down = L->wd;
    gp.sgate = L->swg; gp.sup = L->swu; gp.sdown = L->swd;
    gp.H = (int)L->H; gp.I = (int)L->I; gp.E = (int)L->E; gp.k = (int)L->k;
    gp.xb = w.xb; gp.row_tok = w.row_tok; gp.row_slot = w.row_slot; gp.tiles = w.tiles; gp.n_tiles = w.n_tiles;
    gp.topk_w = w.topk_w; gp.h = w.h; gp.hexp = w.hexp; gp.rowexp = w.rowexp;
    gp.y = nullptr; gp.out = out; gp.status = w.status;
    // the layer's own kernel choice: TMA-streamed decode kernels from GVT_MIN_T tokens (their
    // tensor maps live in the layer), the per-lane-copy ones below, the generic small kernels
    // for the other formats
    const bool gvt = gv && T >= GVT_MIN_T;
    TcMaps gmaps;
    memset(&gmaps, 0, sizeof gmaps);
    gmaps.w[0][0] = L->mg; gmaps.w[0][1] = L->mu; gmaps.w[1][0] = L->smg; gmaps.w[1][1] = L->smu;
    TcMaps gmaps64;
    memset(&gmaps64, 0, sizeof gmaps64);
    gmaps64.w[0][0] = L->mg64; gmaps64.w[0][1] = L->mu64; gmaps64.w[1][0] = L->smg64; gmaps64.w[1][1] = L->smu64;
    e = gvt ? launch_gvt_gateup(gp, gmaps, (L->maps64 && T <= GVT64_MAX_T) ? &gmaps64 : nullptr, max_tiles, nt, s)
            : cudaErrorNotSupported;
    if (e == cudaErrorNotSupported)
        e = gv ? launch_gv_gateup(gp, max_tiles, nt, (int)T, s) : launch_small_gateup(gp, max_tiles, nt, s);
    if (e != cudaSuccess) return cuda_fail(e, "noalloc gate/up launch");
    gmaps.w[0][0] = L->md; gmaps.w[1][0] = L->smd;
    e = gvt ? launch_gvt_down(gp, gmaps, max_tiles, nt, s) : cudaErrorNotSupported;
    if (e == cudaErrorNotSupported)
        e = gv ? launch_gv_down(gp, max_tiles, nt, (int)T, s) : launch_small_down(gp, max_tiles, nt, s);
    if (e != cudaSuccess) return cuda_fail(e, "noalloc down launch");
    return RMOE_OK;
}

// Device errors of the last rmoe_layer_forward_noalloc on `device`: the status word in the static
// scratch, read with a plain copy (no allocation) after synchronising the device.
rmoe_status rmoe_noalloc_status(int32_t device) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(RMOE_ERR_INVALID, "device %d out of range", device);
    DeviceGuard g(device);
    unsigned char* base = nullptr;
    rmoe_status st = scratch_on(device, &base);
    if (st) return st;
    Carver c{base};
    c.take<unsigned>(64);  // the dispatch tickets, then the status words (the order carve() uses)
    unsigned* status = c.take<unsigned>(16);
    cudaError_t e = cudaDeviceSynchronize();
    unsigned v = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&v, status, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "noalloc status read");
    if (v) {
        cudaMemset(status, 0, 4);
        return fail(RMOE_ERR_DEVICE, "noalloc forward: device status 0x%x%s", v,
                    (v & DERR_FP16_RANGE) ? " (an x value beyond the fp16 range)" : "");
    }
    return RMOE_OK;
}

}  // extern "C"
