// common.cuh -- shared device-side definitions for the MoE-layer kernels (sm_100a).
//
// Device weight layout ("planes"): GGUF expert tensors are re-strided once at layer creation
// so that every load a kernel issues is naturally aligned, without changing the byte count.
//   Q4_K (12): main plane [row][half-superblock] of 80 B = four (fp16 d*sc, fp16 -dmin*m)
//              pairs (sub-blocks 0..3 of those 128 elements), then their 64 quant bytes.
//   Q5_K (13): unchanged GGUF superblocks (176 B).
//   Q6_K (14): main plane [row][sb] of 208 B = ql[128] | qh[64] | scales[16] (the GGUF
//              superblock minus its trailing f16 d), d plane [sb][row] f16.
//   Q4_0 (2):  main plane [row][blk] of 16 B qs, d plane [blk][row] f16.
//   Q5_0 (6):  main plane [row][blk] of 16 B qs, aux plane [blk][row] u32 qh, d plane.
//   Q8_0 (8):  main plane [row][blk] of 32 B int8, d plane.
//   F32/F16/BF16 (0/1/30): main plane [row][K] fp16 (the MMA operand type), internal code T_DENSE.
// Element values decoded from these planes are bit-identical (in f32) to quant::dequant
// (rusty-engine src/quant.rs:106-357); the kernels then round them to fp16 (round to nearest
// even) for the tensor-core MMA.  fp16 keeps 11 significant bits against bf16's 8, and every
// operand is range-checked: weights at layer creation, activations by the router, and the
// SwiGLU activations carry a power-of-two scale per (row, 64-feature block) so they never
// overflow fp16.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace rmoe {

enum GgmlType : int {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30,
    T_DENSE = 100  // device-only: an fp16 plane holding F32/F16/BF16 experts
};

// Storage position of K index i in the K-permuted operand order of the tensor-core Q6_K down
// product (positions 1 and 2 of every group of four swapped; its own inverse).
__host__ __device__ __forceinline__ int kperm_pos(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

// Status word bits written by kernels when a device-side check fails (never trap).
enum DevErr : uint32_t { DERR_NONE = 0, DERR_BAD_EXPERT = 1, DERR_ROWS_OVERFLOW = 2, DERR_TILES_OVERFLOW = 4,
                         DERR_TIMEOUT = 8, DERR_FP16_RANGE = 16 };

// Rows of SwiGLU activations are stored as fp16 * 2^e per 64-feature block (tensor-core and
// small-batch kernels) or per 16-feature block (the decode GEMV kernels).
static constexpr int HBLK = 64;
static constexpr int GV_EBLK = 16;

// One stack of expert matrices (E experts x rows x K) in the device layout above.
struct DevMat {
    const uint8_t* main;   // main plane
    const uint32_t* aux;   // Q5_0 qh plane (else null)
    const __half* dpl;     // block-scale plane (Q4_0/Q5_0/Q8_0/Q6_K; else null)
    uint64_t main_stride;  // bytes per row in the main plane
    uint32_t dstride;      // blocks per row (d / aux planes)
    uint64_t trows;        // rows in the whole stack (experts x rows); d / aux planes are [block][trows]
    uint32_t rows;         // rows per expert
    uint32_t K;            // elements per row (multiple of 256)
    int32_t type;
};

// --------------------------------------------------------------------------------------
// f16 -> f32 widening.  The hardware conversion is exact for every binary16 pattern (as is
// rusty-engine's bit-level f16_to_f32, src/quant.rs:25-45): both map each half to the
// unique f32 with the same value (NaN payloads aside).
// --------------------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// 2^e as an exact float for e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// Exponent e with max|v| * 2^-e in [2^13, 2^14): a zero block gets -127 (never the row max
// unless the whole row is zero).
__device__ __forceinline__ int block_exp(float amax) {
    if (!(amax > 0.0f)) return -127;
    int e;
    frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    e -= 14;
    return max(-100, min(100, e));
}

// get_scale_min_k4 (src/quant.rs:250-258) on the 12-byte scale array.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// --------------------------------------------------------------------------------------
// small PTX helpers
// --------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// D = A(16x16 fp16, row) * B(16x8 fp16, col) + D (fp32)
__device__ __forceinline__ void mma_f16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Programmatic dependent launch.  pdl_wait: block until the preceding kernel of the stream has
// completed and its writes are visible (returns at once when this launch did not allow the
// overlap).  pdl_trigger: the next kernel of the stream, if launched with the overlap allowed,
// may start its CTAs once every CTA of this grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// SiLU as rusty-engine computes it (src/moe.rs:44-51): x * (1 / (1 + exp(-x))).
__device__ __forceinline__ float silu_ref(float x) { return x * (1.0f / (1.0f + expf(-x))); }

}  // namespace rmoe
