// attn_rows.cuh -- per-row facts of an attention launch shared by the
// attention kernels: keys attended, KV-cache slot, shard ownership.
#pragma once

#include "kernels.h"

namespace slm {

// keys attended by row r: pos+1, never beyond the cache nor the launch's
// max_len (which sizes the grid and the softmax's shared memory)
__device__ __forceinline__ int row_len(const AttnArgs &a, int r) {
    int p = a.pos ? a.pos[r] : a.pos_const;
    int L = p + 1;
    L = L < a.max_seq ? L : a.max_seq;
    return L < a.max_len ? L : a.max_len;
}
__device__ __forceinline__ size_t row_slot(const AttnArgs &a, int r) {
    return a.slot ? (size_t)a.slot[r] : 0;
}
// whether this rank computes (row r, KV head g) of a sharded batched prefill
__device__ __forceinline__ bool unit_owned(const AttnArgs &a, int r, int g) {
    return a.shard_n <= 1 ||
           ((r / a.rows_per_seq) * a.num_kv_heads + g) % a.shard_n == a.shard_r;
}

}  // namespace slm
