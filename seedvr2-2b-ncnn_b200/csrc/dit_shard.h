// dit_shard.h -- per-context state of the multi-GPU window-sharded forward.
#pragma once
#include "dit_b200.h"

namespace s2b {

struct DitB200::ShardState {
    int world = 1, rank = 0;
    void* comm = nullptr;          // ncclComm_t (NCCL is loaded at run time)
    ~ShardState();
};

}  // namespace s2b
