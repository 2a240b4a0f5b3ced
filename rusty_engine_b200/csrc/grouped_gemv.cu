// grouped_gemv.cu -- decode-size grouped expert products for Q4_K / Q6_K experts (the kernel
// wrappers and their launchers; the device code is in gemv.cuh).
#include "gemv.cuh"

namespace rmoe {

template <int TYPE, int NT, int NMAT, int KS>
__global__ void __launch_bounds__(GV_THREADS, 2) gv_kernel(GroupedParams p, int depth, int ring_off) {
    extern __shared__ __align__(128) uint8_t smem[];
    // Launch order (programmatic dependent launch): gate/up waits for the routing kernel, then
    // lets the down kernel start; the down kernel may read everything routing wrote (the tiles,
    // token rows, routing weights) and stream its weights at once, and waits for gate/up before
    // it touches h.
    if (NMAT == 2) {
        pdl_wait();
        pdl_trigger();
    }
    const int tile = blockIdx.y;
    if (tile >= *p.n_tiles) return;
    const int4 ti = p.tiles[tile];
    gv_tile<TYPE, NT, NMAT, KS, true>(p, ti.x, ti.y, ti.z, blockIdx.x, depth, ring_off, smem);
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
bool gv_supported(int gate_type, int down_type) {
    auto ok = [](int t) { return t == T_Q4_K || t == T_Q6_K; };
    return ok(gate_type) && ok(down_type);
}

template <int TYPE, int NT, int NMAT, int KS>
static cudaError_t go_gv(const GroupedParams& p, int max_tiles, cudaStream_t s) {
    using G = GvGeom<TYPE, NT, NMAT, KS>;
    const int K = NMAT == 2 ? p.H : p.I, rows = NMAT == 2 ? p.I : p.H;
    if (rows % G::RB || K % 256) return cudaErrorInvalidValue;
    const size_t bbytes = (size_t)K * NT * 2;
    const size_t dbytes = Gv<TYPE>::DPL ? (size_t)NMAT * (K / 256) * G::RB * 2 : 0;
    const size_t ring_off = (bbytes + dbytes + 127) & ~(size_t)127;
    int depth = 4;
    while (depth > 2 && ring_off + (size_t)depth * G::SLOT > GV_SMEM_TWO) depth--;
    const size_t smem = ring_off + (size_t)depth * G::SLOT;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    auto k = gv_kernel<TYPE, NT, NMAT, KS>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(k, dim3(rows / G::RB, max_tiles), dim3(GV_THREADS), smem, s, p, depth, (int)ring_off);
}

template <int NMAT, int KS>
static cudaError_t go_gv_type(int type, const GroupedParams& p, int max_tiles, int nt, cudaStream_t s) {
    switch (type) {
        case T_Q4_K: return nt == 8 ? go_gv<T_Q4_K, 8, NMAT, KS>(p, max_tiles, s) : go_gv<T_Q4_K, 16, NMAT, KS>(p, max_tiles, s);
        case T_Q6_K: return nt == 8 ? go_gv<T_Q6_K, 8, NMAT, KS>(p, max_tiles, s) : go_gv<T_Q6_K, 16, NMAT, KS>(p, max_tiles, s);
        default: return cudaErrorInvalidValue;
    }
}

int gv_tile_rows(int T) { return T <= 64 ? 8 : 16; }

// K slices per CTA: more slices (so more, narrower CTAs) when a few tiles must fill the GPU,
// fewer (wider CTAs, each token tile staged for more weight rows) otherwise
cudaError_t launch_gv_gateup(const GroupedParams& p, int max_tiles, int nt, int T, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    return T <= 2   ? go_gv_type<2, 4>(p.gate.type, p, max_tiles, nt, s)
           : T <= 8 ? go_gv_type<2, 2>(p.gate.type, p, max_tiles, nt, s)
                    : go_gv_type<2, 1>(p.gate.type, p, max_tiles, nt, s);
}

cudaError_t launch_gv_down(const GroupedParams& p, int max_tiles, int nt, int T, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    if (nt != 8 && nt != 16) return cudaErrorInvalidValue;
    return T <= 2 ? go_gv_type<1, 2>(p.down.type, p, max_tiles, nt, s) : go_gv_type<1, 1>(p.down.type, p, max_tiles, nt, s);
}

}  // namespace rmoe
