// qmat.cu -- resident quantized matrices: QMat (src/qmat.rs:30-308) on the GPU.
//
// A handle holds one m x n GGUF matrix in the device layout of the expert stacks (uploaded
// once) and runs QMat::matmul / matvec products on it: Out[rows x m] = X[rows x n] . W^T.  It
// drives the expert kernels as a one-expert stack: from 128 rows (m % 128 == 0, n % 256 == 0)
// the tcgen05 down-product kernel (256-row tiles, each weight decoded once per tile and
// 128-row block), below that the mma.sync kernel (16-row tiles), both with deterministic
// stores.  The per-call index tables (row -> token, tiles) are written by a small kernel on the
// caller's stream, so a forward makes no host copies; the workspace grows with cudaMalloc (the
// call synchronises the device then) and is reused.
#include <string.h>

#include <algorithm>

#include "layer_impl.h"

namespace rmoe {

// rows i -> token i, slot 0; the tile list (expert 0, first row, rows)
__global__ void qmat_prep_kernel(int rows, int NT, int4* tiles, int* ntiles, int* rowtok, int* rowslot) {
    const int ntl = (rows + NT - 1) / NT;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
        rowtok[i] = i;
        rowslot[i] = 0;
        if (i < ntl) tiles[i] = make_int4(0, i * NT, min(NT, rows - i * NT), 0);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *ntiles = ntl;
}

// X rows -> the fp16 MMA operand, one warp per row.  QMat::matmul is f32 throughout
// (src/qmat.rs:169-308), so a row whose largest |x| is at or beyond 2^15 is carried as
// fp16 x 2^e: scaled by the exact power of two 2^-e that brings its maximum into [2^13, 2^14),
// e written as the row exponent and as every block exponent, which the product kernels fold
// back into the output (y * 2^e).  Rows inside the fp16 range keep e = 0 (no scaling).
// Non-finite x cannot be carried and sets DERR_FP16_RANGE in the status word.  kperm: the row
// is stored in the tensor-core down kernel's K-permuted order for a Q6_K matrix (kperm_pos).
__global__ void __launch_bounds__(256) qmat_x_kernel(const float* __restrict__ x, int rows, int n,
                                                     __half* __restrict__ xb, int8_t* __restrict__ hexp,
                                                     int* __restrict__ rexp, unsigned* status, int kperm) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float* xr = x + (size_t)r * n;
    float mx = 0.0f;
    bool finite = true;
    for (int i = lane; i < n; i += 32) {
        const float v = fabsf(__ldg(xr + i));
        finite = finite && v <= 3.4028235e38f;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (!__all_sync(0xffffffffu, finite)) {
        if (lane == 0) atomicOr(status, (unsigned)DERR_FP16_RANGE);
        mx = 0.0f;
    }
    const int e = mx >= 32768.0f ? (int)((__float_as_uint(mx) >> 23) & 0xffu) - 127 - 13 : 0;
    const float sc = exp2i(-e);  // exact
    for (int i = lane; i < n; i += 32)
        xb[(size_t)r * n + (kperm ? kperm_pos(i) : i)] = __float2half_rn(__fmul_rn(__ldg(xr + i), sc));
    for (int b = lane; b < n / HBLK; b += 32) hexp[(size_t)r * (n / HBLK) + b] = (int8_t)e;
    if (lane == 0) rexp[r] = e;
}

}  // namespace rmoe

using namespace rmoe;

struct rmoe_qmat {
    int device = 0;
    uint32_t type = 0, m = 0, n = 0;
    Owned own;  // the weights
    DevMat W;
    TcMaps maps;
    bool tc_ok = false;  // shapes allow the tcgen05 path
    Owned ws_own;        // the per-call workspace, for ws_rows rows
    uint32_t ws_rows = 0;
    __half* xb = nullptr;
    int *rowtok = nullptr, *rowslot = nullptr, *rexp = nullptr, *nt = nullptr;
    int8_t* hexp = nullptr;
    int4* tiles = nullptr;
    unsigned* status = nullptr;
    CUtensorMap xmap;  // TMA map of xb (tcgen05 path), for ws_rows rows
};

static rmoe_status qmat_workspace(rmoe_qmat* q, uint32_t rows) {
    if (rows <= q->ws_rows) return RMOE_OK;
    const uint32_t cap = (rows + 255) / 256 * 256;
    cudaDeviceSynchronize();  // the old workspace may be in use by queued work
    q->ws_own.~Owned();
    new (&q->ws_own) Owned();
    q->ws_rows = 0;
    Owned& o = q->ws_own;
    bool ok = true;
    auto A = [&](size_t b) { void* p = o.alloc(b); ok = ok && p; return p; };
    q->xb = (__half*)A((size_t)cap * q->n * 2);
    q->rowtok = (int*)A((size_t)cap * 4);
    q->rowslot = (int*)A((size_t)cap * 4);
    q->rexp = (int*)A((size_t)cap * 4);
    q->hexp = (int8_t*)A((size_t)cap * (q->n / HBLK));
    q->tiles = (int4*)A((size_t)(cap / 16 + 1) * 16);
    q->nt = (int*)A(16);
    q->status = (unsigned*)A(16);
    if (!ok) return fail(RMOE_ERR_OOM, "qmat workspace cudaMalloc failed for %u rows", cap);
    if (cudaMemset(q->status, 0, 16) != cudaSuccess) return fail(RMOE_ERR_CUDA, "qmat workspace clear");
    if (q->tc_ok && !make_rows_map(q->xb, cap, q->n, q->xmap))
        return fail(RMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the qmat token rows");
    q->ws_rows = cap;
    return RMOE_OK;
}

extern "C" {

RMOE_API rmoe_status rmoe_qmat_create(uint32_t ggml_type, const void* w_host, uint64_t w_nbytes, uint32_t m, uint32_t n,
                                      int32_t device, rmoe_qmat** out) {
    if (!out) return fail(RMOE_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (m % 64) return fail(RMOE_ERR_UNSUPPORTED, "m %u must be a multiple of 64", m);
    DeviceGuard g(device);
    rmoe_qmat* q = new rmoe_qmat();
    q->device = device;
    q->type = ggml_type;
    q->m = m;
    q->n = n;
    rmoe_tensor tt{ggml_type, w_host, w_nbytes, {n, m, 1}};
    rmoe_status s = upload_mat(tt, m, n, 1, "qmat", q->own, q->W);
    if (s) {
        delete q;
        return s;
    }
    memset(&q->maps, 0, sizeof q->maps);
    q->tc_ok = m % 128 == 0 && n % 256 == 0 && make_weight_maps(q->W, q->maps.w[0][0]);
    *out = q;
    return RMOE_OK;
}

RMOE_API rmoe_status rmoe_qmat_forward(rmoe_qmat* q, const float* x, uint32_t rows, float* out, void* stream) {
    if (!q) return fail(RMOE_ERR_INVALID, "null qmat");
    if (rows == 0) return RMOE_OK;
    if (!x || !out) return fail(RMOE_ERR_INVALID, "null x / out");
    // the product kernels store Out with 16-B vector stores; x is read as f32
    if (reinterpret_cast<uintptr_t>(out) & 15) return fail(RMOE_ERR_INVALID, "device out must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(x) & 3) return fail(RMOE_ERR_INVALID, "device x must be 4-byte aligned");
    DeviceGuard g(q->device);
    rmoe_status st = qmat_workspace(q, rows);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc = q->tc_ok && rows >= 128;
    const int NT = tc ? tc_tile_rows() : 16;
    const int ntiles = (int)((rows + NT - 1) / NT);
    qmat_prep_kernel<<<std::min<uint32_t>((rows + 255) / 256, 1024), 256, 0, s>>>((int)rows, NT, q->tiles, q->nt,
                                                                              q->rowtok, q->rowslot);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        qmat_x_kernel<<<(rows + 7) / 8, 256, 0, s>>>(x, (int)rows, (int)q->n, q->xb, q->hexp, q->rexp, q->status,
                                                     tc && q->W.type == T_Q6_K ? 1 : 0);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return cuda_fail(e, "qmat prepare");
    GroupedParams gp{};
    gp.down = q->W;
    gp.sdown.type = -1;
    gp.H = (int)q->m; gp.I = (int)q->n; gp.E = 1; gp.k = 1;
    gp.h = q->xb; gp.hexp = q->hexp; gp.rowexp = q->rexp; gp.row_tok = q->rowtok; gp.row_slot = q->rowslot;
    gp.tiles = q->tiles; gp.n_tiles = q->nt; gp.y = out; gp.status = q->status;
    if (tc) {
        TcMaps maps = q->maps;
        maps.b = q->xmap;
        e = launch_tc_down(gp, maps, ntiles, s);
    } else {
        e = launch_small_down(gp, ntiles, NT, s);
    }
    return e == cudaSuccess ? RMOE_OK : cuda_fail(e, "qmat launch");
}

RMOE_API rmoe_status rmoe_qmat_status(rmoe_qmat* q) {
    if (!q) return fail(RMOE_ERR_INVALID, "null qmat");
    if (!q->status) return RMOE_OK;
    DeviceGuard g(q->device);
    unsigned hs = 0;
    cudaError_t e = cudaMemcpy(&hs, q->status, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "qmat status");
    if (hs) {
        cudaMemset(q->status, 0, 4);
        return fail(RMOE_ERR_DEVICE, "qmat: device status 0x%x%s", hs,
                    (hs & DERR_FP16_RANGE) ? " (an x value beyond the fp16 range)" : "");
    }
    return RMOE_OK;
}

RMOE_API void rmoe_qmat_destroy(rmoe_qmat* q) {
    if (!q) return;
    DeviceGuard g(q->device);
    cudaDeviceSynchronize();
    delete q;
}

RMOE_API rmoe_status rmoe_qmat_matmul(uint32_t t, const void* w_host, uint64_t w_nbytes, uint32_t m, uint32_t n,
                                      const float* x, uint32_t rows, float* out, void* stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    rmoe_qmat* q = nullptr;
    rmoe_status s = rmoe_qmat_create(t, w_host, w_nbytes, m, n, dev, &q);
    if (s) return s;
    s = rmoe_qmat_forward(q, x, rows, out, stream);
    if (!s) {
        cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        s = e == cudaSuccess ? rmoe_qmat_status(q) : cuda_fail(e, "qmat");
    }
    rmoe_qmat_destroy(q);
    return s;
}

}  // extern "C"
