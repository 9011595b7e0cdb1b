// session_sharded.cu -- multi-GPU decode session (row-sharded projections, KV-head-sharded
// attention, all-gathers between ranks).
#include "capi_internal.h"
#include "session_internal.h"

using namespace satori;

void session_destroy_sharding(satori_session *s) { (void)s; }

extern "C" int satori_nccl_unique_id(void *out128)
{
    (void)out128;
    return set_error(SATORI_ERR_NOT_SUPPORTED, "sharded sessions are not built yet");
}

extern "C" int satori_session_create_sharded(satori_ctx *ctx, const satori_model_desc *desc, int context, int rank,
                                             int world, const void *nccl_unique_id, satori_session **out)
{
    (void)ctx; (void)desc; (void)context; (void)rank; (void)world; (void)nccl_unique_id; (void)out;
    return set_error(SATORI_ERR_NOT_SUPPORTED, "sharded sessions are not built yet");
}
