/*
 * rmoe.h -- C ABI of the B200-native MoE-layer path (router, dispatch, grouped expert
 * products over GGUF-quantized experts, combine).
 *
 * Every entry point is plain C: pointers, sizes and status codes; no CUDA, NCCL or torch
 * types cross this boundary (streams are passed as void*, NCCL ids as 128 raw bytes).
 * Citations are to the rusty-engine function each entry point replaces.
 *
 * Error convention: every call returns rmoe_status; RMOE_OK is 0.  On failure the
 * thread-local message is in rmoe_last_error() (rusty-engine returns
 * EngineError{message}, src/core.rs:56-68, where it does not panic).  No call aborts or
 * unwinds across the boundary.  Calls on one handle are stream-ordered; use one handle
 * per device per host thread.
 */
#ifndef RMOE_H
#define RMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RMOE_API __attribute__((visibility("default")))
#else
#define RMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    RMOE_OK = 0,
    RMOE_ERR_INVALID = 1,     /* bad argument: shape, type, size, null pointer, k > E ... */
    RMOE_ERR_UNSUPPORTED = 2, /* a ggml type / shape this build has no kernel for */
    RMOE_ERR_CUDA = 3,        /* a CUDA runtime error (message carries cudaGetErrorString) */
    RMOE_ERR_NCCL = 4,        /* an NCCL error in the expert-parallel path */
    RMOE_ERR_DEVICE = 5,      /* a device-side check failed (kernel status word) */
    RMOE_ERR_OOM = 6
} rmoe_status;

/* Gate (src/moe.rs:19-25): softmax over the chosen k logits, or per-expert sigmoid
 * renormalised over the chosen k. */
typedef enum { RMOE_GATE_SOFTMAX = 0, RMOE_GATE_SIGMOID = 1 } rmoe_gate;

/* ggml type codes accepted for expert tensors (src/quant.rs:75-88). */
enum {
    RMOE_GGML_F32 = 0, RMOE_GGML_F16 = 1, RMOE_GGML_Q4_0 = 2, RMOE_GGML_Q5_0 = 6,
    RMOE_GGML_Q8_0 = 8, RMOE_GGML_Q4_K = 12, RMOE_GGML_Q5_K = 13, RMOE_GGML_Q6_K = 14,
    RMOE_GGML_BF16 = 30
};

/* One GGUF tensor as it lies in the file (src/gguf.rs:102-124 TensorEntry): type, the raw
 * bytes (host memory), their length, and the GGUF dims, innermost first.
 * ffn_{gate,up}_exps: dims {H, I, E}; ffn_down_exps: {I, H, E} (src/model.rs:366-391).
 * Shared-expert tensors (*_shexp): {H, I} / {I, H}. */
typedef struct {
    uint32_t ggml_type;
    const void* data;
    uint64_t nbytes;
    uint64_t dims[3];
} rmoe_tensor;

/* Layer description: the arguments of moe_layer_forward (src/moe.rs:360-368) with the
 * experts given as GGUF tensors instead of f32 ExpertWeights. */
typedef struct {
    uint32_t hidden;      /* H (dmodel) */
    uint32_t inter;       /* I (expert SwiGLU width) */
    uint32_t n_experts;   /* E */
    uint32_t top_k;       /* k (RouterConfig.top_k) */
    uint32_t gate;        /* rmoe_gate (RouterConfig.gate) */
    const float* router_w;/* ffn_gate_inp, E rows x H f32, host memory */
    rmoe_tensor gate_exps, up_exps, down_exps;
    uint32_t has_shared;  /* shared expert added at weight 1 (src/moe.rs:381-386) */
    rmoe_tensor gate_shexp, up_shexp, down_shexp;
    int32_t device;       /* CUDA ordinal the handle lives on */
} rmoe_layer_desc;

typedef struct rmoe_layer rmoe_layer;

/* Forward flags. */
enum {
    RMOE_FLAG_HOST_IO = 1u << 0,       /* x / out are host pointers: copied in and out inside
                                          the call, which then synchronises the stream */
    RMOE_FLAG_DETERMINISTIC = 1u << 1, /* combine sums expert outputs per token in chosen
                                          order (the reference order) instead of atomics */
    RMOE_FLAG_FORCE_SMALL = 1u << 2,   /* always use the small-batch (decode) kernels */
    RMOE_FLAG_FORCE_LARGE = 1u << 3,   /* always use the large-batch (prefill) kernels */
    RMOE_FLAG_ROUTING_OUT = 1u << 4,   /* also fill the routing buffers (rmoe_layer_routing) */
    RMOE_FLAG_STAGE_TIMING = 1u << 5,  /* record CUDA events between the pipeline stages
                                          (read back with rmoe_layer_stage_ms) */
    RMOE_FLAG_EXACT_ROUTER = 1u << 6   /* router logits bit-identical to moe::matvec (sequential
                                          f32 sums, src/moe.rs:271-277); without it the logits
                                          are sums in another order (FFMA, or from 1024 tokens
                                          tensor-core products of hi/lo-split fp32 operands)
                                          within the f32 summation error of the exact sums; a
                                          token whose best k + 1 scores hold a near-tie of that
                                          size has those logits rescored with the sequential
                                          sums, so top-k ids match the reference either way */
};

/* Create a layer handle: validates the description on the host, copies router and expert
 * bytes to HBM once (re-strided into the device layout) and owns that memory.
 * Replaces building ExpertWeights for moe_layer_forward (src/moe.rs:348-353) and
 * QMat::from_bytes for the expert tensors (src/qmat.rs:51-58). */
RMOE_API rmoe_status rmoe_layer_create(const rmoe_layer_desc* desc, rmoe_layer** out);

/* moe_layer_forward (src/moe.rs:360-388) for T tokens at once: out[t] = sum over the top-k
 * routed experts of weight * down(swiglu(gate x_t, up x_t)) (+ the shared expert).
 * x: T x H f32, out: T x H f32 (device pointers unless RMOE_FLAG_HOST_IO).  stream is a
 * cudaStream_t (NULL = legacy default stream).  T = 0 is a no-op. */
RMOE_API rmoe_status rmoe_layer_forward(rmoe_layer* layer, const float* x, uint32_t T, float* out,
                               void* stream, uint32_t flags);

/* Size of the library's static device scratch used by rmoe_layer_forward_noalloc: 8 MiB, held
 * on every GPU that loads the library until the process exits. */
#define RMOE_NOALLOC_SCRATCH_BYTES (8u << 20)

/* No counterpart in the reference.  The same layer forward as rmoe_layer_forward for a small
 * batch, allocating no device memory: for callers that cannot call cudaMalloc at forward time
 * (serving runtimes that reserved the device's memory up front for their own pool, decode
 * loops that must not take cudaMalloc's implicit device synchronisation).  x and out are
 * 16-byte-aligned device pointers (T x H f32); it runs the small-batch kernels with the atomic
 * combine, in-stream and without synchronising.  Its scratch is one static device array of
 * RMOE_NOALLOC_SCRATCH_BYTES; a batch whose scratch would not fit is rejected with
 * RMOE_ERR_INVALID and a message giving the bytes it needs (about 2.4 MB for 64 tokens of an
 * H 2048 / E 128 / k 8 / I 768 layer).  The first call on a device looks up the array's
 * address (cudaGetSymbolAddress), so make that first call before any stream capture.  Every
 * call on a device shares the array: calls that overlap on the GPU race on it.  It does not
 * update what rmoe_layer_routing / rmoe_layer_logits / rmoe_layer_stage_ms report; its device
 * errors are read with rmoe_noalloc_status. */
RMOE_API rmoe_status rmoe_layer_forward_noalloc(rmoe_layer* layer, const float* x, uint32_t T, float* out,
                                                void* stream);

/* Device errors of the last rmoe_layer_forward_noalloc call on `device` (an x value beyond the
 * fp16 range, a tile-list overflow), which that call cannot report itself since it does not
 * wait for its kernels.  Synchronises the device and reads the status word kept in the static
 * scratch, allocating nothing; RMOE_ERR_DEVICE (then the word is cleared) when one is set.
 * The next noalloc call on the device clears the word, so read it in between.  No counterpart
 * in the reference (its CPU path has no device errors). */
RMOE_API rmoe_status rmoe_noalloc_status(int32_t device);

/* Routing of the last forward with RMOE_FLAG_ROUTING_OUT: expert ids (T x k, chosen order)
 * and weights (T x k), copied to host buffers.  Mirrors route() (src/moe.rs:120-125). */
RMOE_API rmoe_status rmoe_layer_routing(rmoe_layer* layer, uint32_t T, uint32_t* ids, float* weights);

/* Router logits (T x E f32: the exact moe::matvec values under RMOE_FLAG_EXACT_ROUTER) of the
 * last forward that had RMOE_FLAG_ROUTING_OUT, copied to a host buffer.  A debugging aid with no counterpart in
 * the reference (its logits never leave moe_layer_forward). */
RMOE_API rmoe_status rmoe_layer_logits(rmoe_layer* layer, uint32_t T, float* logits);

/* Tokens whose fast-router top-k met a near-tie since the last call (or since the handle's
 * workspace was last sized), read and reset; synchronises the device.  For such a token the
 * logits of the experts around its k-th pick are rescored with moe::matvec's sequential f32
 * sums (src/moe.rs:271-277) before top-k, so its ids are the reference's.  A debugging aid
 * with no counterpart in the reference. */
RMOE_API rmoe_status rmoe_layer_router_refined(rmoe_layer* layer, uint32_t* count);

/* Stage durations of the last forward that had RMOE_FLAG_STAGE_TIMING, in milliseconds,
 * from CUDA events recorded on the forward's stream: ms[0] route+dispatch, ms[1] gate/up
 * (+SwiGLU), ms[2] down (+atomic combine), ms[3] deterministic combine (0 if not run).
 * Synchronises on the last event.  No counterpart in the reference (its RUSTY_PROFILE stage
 * timers, src/profile.rs:15-89, are the analogue). */
RMOE_API rmoe_status rmoe_layer_stage_ms(rmoe_layer* layer, float ms[4]);

/* Release the handle and all device memory it owns. */
RMOE_API void rmoe_layer_destroy(rmoe_layer* layer);

/* Thread-local message of the last failed call on this thread ("" if none). */
RMOE_API const char* rmoe_last_error(void);

/* ---- stand-alone operators (the reference functions the layer is built from) --------- */

/* quant::dequant (src/quant.rs:363-453) on the GPU: n GGUF bytes of type t -> f32.
 * src/dst are device pointers; dst holds numel(t, nbytes) floats. */
RMOE_API rmoe_status rmoe_dequant(uint32_t ggml_type, const void* src, uint64_t nbytes, float* dst,
                         void* stream);

/* QMat::matmul (src/qmat.rs:169-182) on the GPU: W[m x n] (GGUF bytes, host pointer, type t)
 * times X[rows x n] f32 -> Out[rows x m] f32.  X/Out are device pointers.  rows = 1 is
 * QMat::matvec (src/qmat.rs:80-82).  Weights are uploaded per call (a convenience path;
 * the layer handle and rmoe_qmat keep their weights resident), synchronising the stream.
 * From 128 rows, with m % 128 == 0 and n % 256 == 0, the product runs on the tcgen05 kernel of
 * the layer's down projection. */
RMOE_API rmoe_status rmoe_qmat_matmul(uint32_t ggml_type, const void* w_host, uint64_t w_nbytes,
                             uint32_t m, uint32_t n, const float* x, uint32_t rows, float* out,
                             void* stream);

/* A resident quantized matrix (QMat, src/qmat.rs:30-58): W[m x n] GGUF bytes (host pointer)
 * uploaded once to `device`; m % 64 == 0, n a multiple of the type's block. */
typedef struct rmoe_qmat rmoe_qmat;
RMOE_API rmoe_status rmoe_qmat_create(uint32_t ggml_type, const void* w_host, uint64_t w_nbytes, uint32_t m,
                             uint32_t n, int32_t device, rmoe_qmat** out);
/* QMat::matmul (src/qmat.rs:169-308): Out[rows x m] = X[rows x n] . W^T, device pointers,
 * stream-ordered, no synchronisation (the workspace grows with cudaMalloc when rows exceed
 * every earlier call's, and the call synchronises the device then).  From 128 rows, with
 * m % 128 == 0 and n % 256 == 0, the tcgen05 kernel; below, the mma.sync kernel. */
RMOE_API rmoe_status rmoe_qmat_forward(rmoe_qmat* q, const float* x, uint32_t rows, float* out, void* stream);
/* Device errors of the forwards so far (an x value beyond the fp16 range, a timed-out wait);
 * synchronises with the device.  RMOE_ERR_DEVICE clears the recorded status. */
RMOE_API rmoe_status rmoe_qmat_status(rmoe_qmat* q);
RMOE_API void rmoe_qmat_destroy(rmoe_qmat* q);

/* route() (src/moe.rs:120-125) over T rows of E logits (device pointers): ids/weights are
 * T x k in chosen order. */
RMOE_API rmoe_status rmoe_route(const float* logits, uint32_t T, uint32_t E, uint32_t k, uint32_t gate,
                       uint32_t* ids, float* weights, void* stream);

/* route_noaux_tc (src/moe.rs:192-268; noaux != 0) or route_group (src/moe.rs:127-190;
 * noaux == 0) over T rows of E logits, device pointers: scores sigmoid(logit + bias) (bias of
 * length nbias, 0 past it, may be null when nbias is 0); experts in n_groups contiguous groups
 * (expert i in group i * n_groups / E); a group scores the sum of its top-2 scores (noaux) or
 * of all its scores; only the top_k_group best groups are eligible (every group when
 * top_k_group < 0); the top k eligible experts by score, weights renormalised over the picks.
 * ids / weights are T x k in chosen order; picks beyond the eligible experts get id
 * 0xFFFFFFFF and weight 0 (the reference returns fewer picks).  n_groups <= 64, k <= 32. */
RMOE_API rmoe_status rmoe_route_grouped(const float* logits, const float* bias, uint32_t nbias, uint32_t T,
                               uint32_t E, uint32_t k, uint32_t n_groups, int32_t top_k_group, int32_t noaux,
                               uint32_t* ids, float* weights, void* stream);

/* ---- expert parallelism (no counterpart in the reference: its B9 dist-MoE is planned,
 *      docs/roadmap.md:235-246) ---------------------------------------------------------- */

/* 128-byte NCCL unique id, made on one rank and shared with all ranks out of band. */
RMOE_API rmoe_status rmoe_ep_unique_id(uint8_t id[128]);

/* Create this rank's shard of an expert-parallel layer (a collective: every rank calls it with
 * the same id): experts are dealt round-robin, E / world_size per rank (rank r holds experts
 * r, r + W, r + 2W, ...), so a skewed load spreads over the ranks; the router is replicated.
 * desc carries the FULL tensors (each rank uploads only its experts).  E must divide by W,
 * W <= 16.  A shared expert is replicated on every rank and applied by each rank to its own
 * tokens.  rmoe_layer_forward on the handle takes this rank's T tokens
 * (device or RMOE_FLAG_HOST_IO buffers) and returns their complete layer outputs; it exchanges
 * rows with the other ranks over NCCL and reads the per-rank row counts back to the host
 * once (the call synchronises the stream there).
 * Failure detection: the communicator is non-blocking; the create (which waits for every
 * rank to join) and every host wait of a forward give up after RMOE_EP_TIMEOUT_MS
 * milliseconds without progress (environment variable, default 120000), or at once on an NCCL
 * error: the communicator is then aborted (its kernels end) and the call returns
 * RMOE_ERR_NCCL, as does every later forward on the handle. */
RMOE_API rmoe_status rmoe_ep_layer_create(const rmoe_layer_desc* desc, int32_t rank, int32_t world_size,
                                 const uint8_t id[128], rmoe_layer** out);

/* rmoe_ep_layer_create with the caller's expert placement: expert_rank[e] (n_experts entries,
 * the same table on every rank) is the rank that holds expert e; every rank must hold at least
 * one expert, and the experts need not split evenly.  A rank numbers its experts in ascending
 * global order.  Placing by measured expert loads (e.g. the per-expert pick counts of a
 * calibration batch, spread by a greedy largest-first fill) keeps the busiest rank near the
 * mean under skewed routing, where the round-robin deal can leave one rank with 1.5x the mean
 * at 8 ranks.  expert_rank == NULL is the round-robin deal.  No counterpart in the reference
 * (its MoE layer runs in one process). */
RMOE_API rmoe_status rmoe_ep_layer_create_placed(const rmoe_layer_desc* desc, int32_t rank, int32_t world_size,
                                                 const uint8_t id[128], const int32_t* expert_rank,
                                                 rmoe_layer** out);

/* ---- GGUF expert binding (MmapModel::open / tensor_bytes, src/loader.rs:33-102; the MoE
 *      tensors of a block, src/model.rs:366-391) ---------------------------------------------- */

/* A GGUF file mapped read-only with its parsed header (version 2 or 3).  Parse errors are
 * RMOE_ERR_INVALID with "gguf parse error at <byte offset>: <what>" (src/gguf.rs:174-178). */
typedef struct rmoe_gguf rmoe_gguf;
RMOE_API rmoe_status rmoe_gguf_open(const char* path, rmoe_gguf** out);
RMOE_API void rmoe_gguf_close(rmoe_gguf* g);

/* A tensor's type, dims (up to 3; unused dims are 1) and bytes inside the mapping:
 * [aligned data start + offset, + bytes_for_numel(type, numel)), bounds-checked
 * (MmapModel::tensor_bytes, src/loader.rs:97-102).  Valid until rmoe_gguf_close. */
RMOE_API rmoe_status rmoe_gguf_tensor(const rmoe_gguf* g, const char* name, rmoe_tensor* out);

/* An integer metadata value by its full key (e.g. "qwen3moe.expert_count"). */
RMOE_API rmoe_status rmoe_gguf_meta_uint(const rmoe_gguf* g, const char* key, uint64_t* out);

/* The layer description of MoE block `block`: blk.N.ffn_gate_inp [H, E] (router; F32 used in
 * place, F16 / BF16 widened to f32 in memory the rmoe_gguf handle owns), ffn_{gate,up}_exps
 * [H, I, E], ffn_down_exps [I, H, E] and, when all three exist, ffn_{gate,up,down}_shexp
 * ([H, I], [H, I], [I, H]).  top_k = {arch}.expert_used_count, the expert count is checked
 * against {arch}.expert_count where present (then general.*, src/model.rs:131-147), gate =
 * sigmoid when {arch}.expert_gating_func is 2, else softmax; device 0.  The description
 * points into the mapping: pass it to rmoe_layer_create before rmoe_gguf_close. */
RMOE_API rmoe_status rmoe_gguf_moe_layer_desc(rmoe_gguf* g, uint32_t block, rmoe_layer_desc* out);

/* Self-test of the tensor-core kernels' bounded waits (no counterpart in the reference): one
 * CTA on `device` allocates tensor memory, waits on an mbarrier that nothing arrives at with a
 * limit of limit_us (1 .. 1000000) instead of the kernels' 1 s, then records DERR_TIMEOUT,
 * frees the tensor memory and returns, as the product kernels do when a wait runs out.
 * Returns RMOE_ERR_DEVICE with the timeout in the message (what a product call whose wait ran
 * out reports); the context stays usable.  RMOE_ERR_CUDA for any other outcome. */
RMOE_API rmoe_status rmoe_selftest_bounded_wait(int32_t device, uint32_t limit_us);

/* Build info: "sm_100a <git-describe> <kernels...>". */
RMOE_API const char* rmoe_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* RMOE_H */
