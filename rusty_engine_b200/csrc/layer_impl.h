// layer_impl.h -- host-side layer handle and helpers shared by layer.cu and ep.cu.
#pragma once
#include <cuda_runtime.h>

#include <new>
#include <vector>

#include "../../include/rmoe.h"
#include "kernels.h"

namespace rmoe {

// cudaMalloc'd blocks owned by a handle, freed together.
struct Owned {
    std::vector<void*> ptrs;
    void* alloc(size_t n);
    Owned() = default;
    Owned(const Owned&) = delete;
    Owned& operator=(const Owned&) = delete;
    ~Owned();
};

// Makes `dev` current for the scope and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = 0, cur = 0;
    explicit DeviceGuard(int dev);
    ~DeviceGuard();
};

// Per-forward scratch, sized for ws_T tokens.
struct Workspace {
    float* xin = nullptr;     // host-IO staging of x
    float* xout = nullptr;    // host-IO staging of out
    __half* xb = nullptr;
    int* topk_id = nullptr;
    float* topk_w = nullptr;
    int* local_rank = nullptr;
    int* cta_cnt = nullptr;
    unsigned* ticket = nullptr;
    unsigned* status = nullptr;
    int* expert_off = nullptr;
    int* row_tok = nullptr;
    int* row_slot = nullptr;
    int* slot_row = nullptr;
    int* n_rows = nullptr;
    int* n_tiles = nullptr;
    int4* tiles = nullptr;
    __half* h = nullptr;
    int8_t* hexp = nullptr;
    int* rowexp = nullptr;
    __half* xs = nullptr;   // expert-sorted x (tensor-core path)
    float* y = nullptr;
    float* logits = nullptr;
    float* logits_part = nullptr;  // K-split partial router logits (large batches, fast router)
};

struct EpState;  // expert-parallel state (ep.cu)

}  // namespace rmoe

struct rmoe_layer {
    int device = 0;
    uint32_t H = 0, I = 0, E = 0, k = 0, gate_kind = 0;
    int has_shared = 0;
    uint32_t E_local = 0;
    uint32_t E_router = 0;      // experts the router scores (E, or all experts of an EP layer)
    rmoe::EpState* ep = nullptr;  // expert-parallel state (null for a whole layer)
    rmoe::DevMat wg{}, wu{}, wd{}, swg{}, swu{}, swd{};
    rmoe::WMaps mg{}, mu{}, md{}, smg{}, smu{}, smd{};  // TMA maps of the stacks above
    rmoe::WMaps mg64{}, mu64{}, smg64{}, smu64{};       // gate/up with 64-row boxes (decode kernels)
    bool maps64 = false;
    CUtensorMap hmap{}, xsmap{};                          // TMA maps of the workspace h and xs
    float* router_w = nullptr;
    float* router_wh = nullptr;  // router_w split for the tensor-core logits (hi | lo, [E, H] each)
    float* router_wl = nullptr;
    float router_wmax = 0.0f;    // max over experts of ||router row||_2 (fast-router near-tie window)
    rmoe::Owned own;       // weights
    rmoe::Owned ws_own;    // workspace
    rmoe::Workspace ws;
    uint32_t ws_T = 0;
    bool ws_had_y = false;
    int max_tiles = 0;
    uint32_t last_T = 0;
    bool last_tc = false;  // the last forward ran the tcgen05 kernels
    int small_grid[3] = {0, 0, 0};  // co-resident grid sizes of the one-launch decode layer
    cudaEvent_t ev[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    bool ev_valid = false, ev_combine = false;
    // host-IO pipeline: copy streams (in, out) and per-chunk events, made on first use
    cudaStream_t io_stream[2] = {nullptr, nullptr};
    cudaEvent_t io_ev[2 * 8 + 1] = {};
    ~rmoe_layer();
};

namespace rmoe {
rmoe_status fail(rmoe_status s, const char* fmt, ...);
rmoe_status cuda_fail(cudaError_t e, const char* what);
bool block_geom(uint32_t t, uint32_t& el, uint32_t& by);
rmoe_status upload_mat(const rmoe_tensor& t, uint32_t rows, uint32_t K, uint32_t experts, const char* name, Owned& own,
                       DevMat& out);
rmoe_status validate_desc(const rmoe_layer_desc* d);
rmoe_status layer_upload(const rmoe_layer_desc* d, const uint32_t* ids, uint32_t e_count, rmoe_layer* L);
rmoe_status ensure_workspace(rmoe_layer* L, uint32_t T, bool need_y);
// given: the workspace's xb / topk_id / topk_w already hold T rows' routing (x unused; ids >= E
// are empty picks) -- the expert-parallel local step
// shared_t0 / shared_n: the tokens that get the shared expert (all T when shared_n < 0)
rmoe_status layer_forward_device(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s, uint32_t flags,
                                 bool given = false, uint32_t shared_t0 = 0, int64_t shared_n = -1);
rmoe_status ep_forward(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s, uint32_t flags);
rmoe_status ep_forward_host(rmoe_layer* L, const float* x, uint32_t T, float* out, cudaStream_t s, uint32_t flags);
rmoe_status ep_routing(rmoe_layer* L, uint32_t T, uint32_t* ids, float* weights, float* logits);
void ep_free(rmoe_layer* L);
unsigned* ep_status(rmoe_layer* L);  // the expert-parallel state's status words (null before a forward)
int canon_type(uint32_t t);
}  // namespace rmoe
