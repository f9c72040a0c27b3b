// shard.cpp - how the batched decode path is split across GPUs (one process
// per GPU). The reference is single-GPU (src/models.rs:51-53); these rules are
// new: sequences are independent, so small-KV-head models shard by sequence
// with no data-path collective; wide models shard by KV head and all-gather
// the per-head outputs.
#include <algorithm>
#include <numeric>
#include <vector>

#include "../lc_host.h"

extern "C" int lc_shard_sequences(const int *context_lens, int batch, int num_ranks,
                                  int *rank_of) {
    if (!context_lens || !rank_of || batch < 0 || num_ranks <= 0) return LC_ERR_INVALID_ARGUMENT;
    std::vector<int> order(batch);
    std::iota(order.begin(), order.end(), 0);
    // Longest first; equal lengths keep index order.
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return context_lens[a] > context_lens[b]; });
    std::vector<long long> load(num_ranks, 0);
    for (int b : order) {
        int best = 0;
        for (int r = 1; r < num_ranks; ++r)
            if (load[r] < load[best]) best = r;
        rank_of[b] = best;
        load[best] += std::max(context_lens[b], 0);
    }
    return LC_OK;
}

extern "C" int lc_shard_kv_heads(int num_q_heads, int num_kv_heads, int num_ranks, int rank,
                                 int *first_kv_head, int *num_local_kv_heads) {
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_ranks <= 0 || rank < 0 ||
        rank >= num_ranks || !first_kv_head || !num_local_kv_heads)
        return LC_ERR_INVALID_ARGUMENT;
    if (num_q_heads % num_kv_heads || num_kv_heads % num_ranks) return LC_ERR_UNSUPPORTED_SHAPE;
    const int per = num_kv_heads / num_ranks;
    *first_kv_head = rank * per;
    *num_local_kv_heads = per;
    return LC_OK;
}
