// dit_shard.cpp -- multi-GPU window-sharded forward (NCCL over NVLink).
#include "dit_shard.h"

namespace s2b {

DitB200::ShardState::~ShardState() {}

int DitB200::shard_init(const uint8_t id[128], int world, int rank) {
    (void)id; (void)world; (void)rank;
    return fail(ERR_UNSUPPORTED, "window-sharded mode is not built yet");
}

int DitB200::shard_forward(const float* vid_patch, int Lv, const float* txt, int TXT, float t, float* sr_out) {
    (void)vid_patch; (void)Lv; (void)txt; (void)TXT; (void)t; (void)sr_out;
    return fail(ERR_UNSUPPORTED, "window-sharded mode is not built yet");
}

}  // namespace s2b

extern "C" int s2b_nccl_unique_id(uint8_t id[128]) {
    (void)id;
    return s2b::ERR_UNSUPPORTED;
}
