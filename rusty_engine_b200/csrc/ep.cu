// ep.cu -- expert-parallel layer shards (NCCL all-to-all dispatch / combine).
#include <nccl.h>

#include "../../include/rmoe.h"
#include "layer_impl.h"

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

rmoe_status rmoe_ep_layer_create(const rmoe_layer_desc* desc, int32_t rank, int32_t world_size, const uint8_t id[128],
                                 rmoe_layer** out) {
    (void)desc; (void)rank; (void)world_size; (void)id;
    if (out) *out = nullptr;
    return fail(RMOE_ERR_UNSUPPORTED, "expert-parallel layers are not built yet");
}

}  // extern "C"
