// kernels.h -- parameter blocks and launchers shared by the host orchestration (layer.cu)
// and the kernel translation units.
#pragma once
#include <cuda_bf16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "common.cuh"

namespace rmoe {

// Launch with programmatic dependent launch allowed: the kernel's CTAs may start while the
// previous kernel of the stream finishes; the kernel itself waits (pdl_wait) before it reads
// anything that kernel writes.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

static constexpr int MAX_E = 512;  // experts per layer this build supports
static constexpr int LOGIT_SPLITS = 4;  // K-splits of the large-batch fast router (logits_part planes)
static constexpr int MAX_K = 32;   // top-k this build supports
static constexpr int RG_MAX_G = 64; // expert groups the group router supports

struct RouteParams {
    const float* x;         // [T, H] f32
    const float* router_w;  // [E, H] f32
    const float* router_wh; // optional [E, H]: router_w with the 13 low mantissa bits cleared
    const float* router_wl; // optional [E, H]: router_w - router_wh (the tensor-core logits)
    int T, H, E, k, gate, has_shared;
    int shared_t0, shared_n;  // tokens [shared_t0, shared_t0 + shared_n) get a shared-expert row
                              // (all T normally; the expert-parallel local step gives the range
                              // of the rows a rank sent to itself)
    __half* xb;             // [T, H] fp16 copy of x (GEMM B operand)
    int* rowexp;            // [rows] SwiGLU row exponents, set to -127 by the dispatch
    __half* xs;             // optional [rows, H]: x rows in expert-sorted order (tensor-core path)
    float* logits;          // [T, E] router logits
    float* logits_part;     // optional [8, T, E]: K-split partial logits of the fast large-batch
                            // router (the top-k kernel sums them into logits); null (always in
                            // exact mode): the logits kernel writes logits directly
    float* out_zero;        // optional: rows of `out` to zero (atomic combine)
    int* topk_id;           // [T, k]
    float* topk_w;          // [T, k]
    int* local_rank;        // [T, k] scratch
    int* cta_cnt;           // [E, route_cnt_stride(route_grid(T))] scratch: counts, then prefixes
    unsigned int* ticket;   // last-CTA counters, 0 between launches: [0] per launch, [1 + g] per
                            // 8-token group (16 words)
    int* expert_off;        // [E + 2]
    int* row_tok;           // [rows] token of each expert-sorted row
    int* row_slot;          // [rows] slot (k for the shared expert)
    int* slot_row;          // [T, k] row of each (token, slot)
    int* n_rows;            // total rows
    int4* tiles;            // (expert, first row, rows, 0)
    int* n_tiles;
    int max_tiles;
    int tile_rows;          // rows per tile
    unsigned int* status;   // device status word (DevErr bits)
    int given;              // 1: topk_id / topk_w are filled in already (x and logits unused);
                            // ids >= E are empty picks and get no row
    int exact;              // 1: logits bit-identical to moe::matvec (sequential sums)
    float router_wmax;      // max over experts of ||router row||_2 (sizes the fast router's
                            // near-tie window; 0 turns the refinement off)
    unsigned int* refined;  // optional counter of tokens whose near-tie logits were rescored
    int stage_floats;       // dynamic shared memory the top-k kernel has for rescoring (floats)
};

// Grouped expert products over the expert-sorted rows.
struct GroupedParams {
    DevMat gate, up, down;        // routed experts
    DevMat sgate, sup, sdown;     // shared expert (type < 0 when absent)
    int H, I, E, k;
    const __half* xb;             // [T, H]
    const int* row_tok;
    const int* row_slot;
    const int4* tiles;
    const int* n_tiles;
    const int* n_rows;            // expert-sorted rows in use
    const float* topk_w;          // [T, k]
    __half* h;                    // [rows, I] SwiGLU activations, fp16 * 2^hexp
    int8_t* hexp;                 // [rows, I / 16] block exponents (I / 64 used by the tensor-core path)
    int* rowexp;                  // [rows] max block exponent per row
    float* y;                     // [rows, H] expert outputs (deterministic combine) or null
    float* out;                   // [T, H] atomic combine target (when y is null)
    unsigned int* status;
};

struct CombineParams {
    const float* y;       // [rows, H]
    const int* slot_row;  // [T, k]
    const float* topk_w;  // [T, k]
    int T, H, k, has_shared;
    int shared_t0, shared_n;  // tokens with a shared-expert row (see RouteParams)
    const int* expert_off;    // [E + 2]: the shared expert's first row at expert_off[E]
    int E;
    float* out;
};

int route_grid(int T);
// row stride of the per-(expert, top-k CTA) count table: CTAs rounded up to 16
__host__ __device__ inline int route_cnt_stride(int ncta) { return (ncta + 15) & ~15; }
cudaError_t launch_route_dispatch(const RouteParams& p, cudaStream_t s);
// router logits and top-k only (topk_id, topk_w, xb): no dispatch tables
cudaError_t launch_router_topk(const RouteParams& p, cudaStream_t s);

// small-batch (mma.sync) grouped kernels; nt = rows per tile (8 or 16, small_tile_rows(T) for
// a batch of T tokens; the dispatch must use the same value)
int small_tile_rows(int T);
int small_tile_rows_min();
cudaError_t launch_small_gateup(const GroupedParams& p, int max_tiles, int nt, cudaStream_t s);
cudaError_t launch_small_down(const GroupedParams& p, int max_tiles, int nt, cudaStream_t s);

// decode GEMV kernels (Q4_K / Q6_K experts, dequant in the mma.sync operand registers), same
// tiles as the small-batch kernels; h blocks of GV_EBLK features
bool gv_supported(int gate_type, int down_type);
int gv_tile_rows(int T);
cudaError_t launch_gv_gateup(const GroupedParams& p, int max_tiles, int nt, int T, cudaStream_t s);
cudaError_t launch_gv_down(const GroupedParams& p, int max_tiles, int nt, int T, cudaStream_t s);

// The whole layer for a decode batch (T <= 16, Q4_K / Q6_K experts, fast router, atomic
// combine) in one cooperative launch (layer_small.cu).  bar: two zeroed words that persist
// between launches; grid_cache: three ints (0 at first use) caching the co-resident grid size.
// cudaErrorNotSupported where the shapes or the device do not allow it.
bool layer_small_supported(int gate_type, int down_type, int T, int E, int k);
cudaError_t launch_layer_small(const RouteParams& r, const GroupedParams& g, unsigned* bar, int* grid_cache,
                               cudaStream_t s);

// TMA descriptors of one weight-matrix stack: main plane (viewed as u16, 128-row boxes), the
// block-scale plane and the Q5_0 high-bit plane (both [block][row], 128-row boxes).
struct WMaps {
    CUtensorMap main, d, aux;
};

// Everything the tcgen05 kernels read through TMA: [routed | shared expert][matrix 0 | 1]
// weight maps and the token operand b: the expert-sorted x rows (gate/up) or the SwiGLU
// activations h (down), [rows, width] fp16 in 64 x 128 boxes with the 128-B swizzle.
struct alignas(64) TcMaps {
    WMaps w[2][2];
    CUtensorMap b;
};

// The same decode products with the weight stream on TMA (gemv_tma.cu): CTA = (tile, 128-row
// block), weights from the stacks' maps (maps.w), same tiles, h layout and launch order as the
// gv launchers.  cudaErrorNotSupported where the shapes do not fit (then use those).
// Decode batches of at least GVT_MIN_T tokens use them (a single token fills the GPU only with
// the K-split CTAs of gv_kernel).
static constexpr uint32_t GVT_MIN_T = 2;
// ... and gate/up runs 64-row blocks (maps64) for batches of at most GVT64_MAX_T tokens
static constexpr uint32_t GVT64_MAX_T = 16;
// maps64: the same stacks with 64-row boxes (null: none); 8-row tiles of gate/up then run
// 64-row blocks, three CTAs per SM (finer items, so the last wave is shorter)
cudaError_t launch_gvt_gateup(const GroupedParams& p, const TcMaps& maps, const TcMaps* maps64, int max_tiles, int nt,
                              cudaStream_t s);
cudaError_t launch_gvt_down(const GroupedParams& p, const TcMaps& maps, int max_tiles, int nt, cudaStream_t s);

// Build the maps of one stack (after upload_mat) / of the h workspace; false on a driver error.
bool make_weight_maps(const DevMat& M, WMaps& out, uint32_t rows = 128);  // rows: box height
bool make_rows_map(const __half* base, uint64_t rows, uint32_t width, CUtensorMap& out);
// fp32 [rows, width] row-major, 128-B-swizzled boxes of box_w (32) x box_rows
bool make_f32_rows_map(const float* base, uint64_t rows, uint32_t width, uint32_t box_w, uint32_t box_rows,
                       CUtensorMap& out);
// large-batch fast-router logits on the tensor cores (split partial sums into logits_part);
// cudaErrorNotSupported where the shapes or the pointers do not allow it
// route_noaux_tc / route_group over precomputed logits (one warp per token)
cudaError_t launch_route_grouped(const float* logits, const float* bias, int nbias, int T, int E, int k, int ng,
                                 int tkg, int noaux, unsigned* ids, float* w, cudaStream_t s);
bool logits_tc_supported(const RouteParams& p);
cudaError_t launch_logits_tc(const RouteParams& p, cudaStream_t s);

// large-batch (tcgen05) grouped kernels; tile_rows = rows per tile
int tc_tile_rows();
cudaError_t launch_tc_gateup(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s);
cudaError_t launch_tc_down(const GroupedParams& p, const TcMaps& maps, int max_tiles, cudaStream_t s);
// between the two: h blocks to their row's common exponent (rows beyond *n_rows untouched)
cudaError_t launch_rescale_h(const GroupedParams& p, int max_rows, cudaStream_t s);

cudaError_t launch_combine(const CombineParams& p, cudaStream_t s);
cudaError_t launch_dequant_raw(int type, const void* src, uint64_t nblocks, float* dst, cudaStream_t s);
cudaError_t launch_route_only(const float* logits, int T, int E, int k, int gate, int* ids, float* w, cudaStream_t s);
cudaError_t launch_f32_to_f16(const float* x, __half* y, uint64_t n, cudaStream_t s);

}  // namespace rmoe
