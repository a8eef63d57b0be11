// Token permute: the eager expert dispatch order of Qwen3_5MoeExperts.forward
// (transformers qwen3_5_moe modeling :730-744) -- ascending expert, then
// slot-major, then token -- as a stable counting sort inside one CTA.
//
// Routes are numbered r = slot * T + token (slot-major).  Warp w owns the
// contiguous r-range [w*chunk, (w+1)*chunk).  Pass 1 counts, per warp and
// expert, with __match_any_sync over 32 routes at a time; a column scan over
// warps plus an exclusive scan over experts gives every warp the first
// position of each of its experts; pass 2 repeats the walk and places each
// route at that position plus its rank among equal experts to its left in the
// 32-route step.  Because r-ranges and steps are visited in increasing r, the
// placement is stable, which is exactly the (expert, slot, token) order.
#include "common.cuh"
#include "kernels.cuh"
#include "routing.cuh"

namespace lrb {

__global__ void __launch_bounds__(1024) permute_kernel(const int64_t *__restrict__ idx, int tokens, int top_k,
                                                       int experts, int32_t *__restrict__ offsets,
                                                       int32_t *__restrict__ perm_token,
                                                       int32_t *__restrict__ perm_slot,
                                                       int32_t *__restrict__ route_pos,
                                                       int32_t *__restrict__ active,
                                                       int32_t *__restrict__ num_active,
                                                       int32_t *__restrict__ bad_routes) {
    extern __shared__ int32_t smem[];
    __shared__ int scratch[33];
    permute_block(GlobalIdx{idx, top_k}, tokens, top_k, experts, offsets, perm_token, perm_slot, route_pos, active,
                  num_active, bad_routes, smem, scratch);
}

int permute_smem_bytes(int warps, int experts) {
    return static_cast<int>(sizeof(int32_t) * static_cast<size_t>(warps + 1) * experts);
}

int launch_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets, int32_t *perm_token,
                   int32_t *perm_slot, int32_t *route_pos, int32_t *active, int32_t *num_active, int32_t *bad_routes,
                   cudaStream_t stream) {
    const int smem = permute_smem_bytes(32, experts);
    static bool configured = false;
    if (!configured) {
        LRB_CUDA(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      permute_smem_bytes(32, 1024)));
        configured = true;
    }
    permute_kernel<<<1, 1024, smem, stream>>>(idx, tokens, top_k, experts, offsets, perm_token, perm_slot, route_pos,
                                               active, num_active, bad_routes);
    LRB_LAUNCHED("permute_kernel");
    return MOE_OK;
}

}  // namespace lrb

extern "C" int moe_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets,
                           int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                           int32_t *num_active, int32_t *bad_routes, void *stream) {
    LRB_REQUIRE(experts >= 1 && experts <= 1024, "moe_permute: experts %d outside [1, 1024]", experts);
    LRB_REQUIRE(top_k >= 1 && tokens >= 0, "moe_permute: bad tokens %d / top_k %d", tokens, top_k);
    LRB_REQUIRE(static_cast<int64_t>(tokens) * top_k < (1 << 30), "moe_permute: too many routes");
    LRB_REQUIRE(idx && offsets && perm_token && perm_slot && route_pos && active && num_active,
                "moe_permute: null output");
    if (int rc = lrb::require_sm100()) return rc;
    if (tokens == 0) {
        LRB_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (experts + 1), lrb::as_stream(stream)));
        LRB_CUDA(cudaMemsetAsync(num_active, 0, sizeof(int32_t), lrb::as_stream(stream)));
        if (bad_routes) LRB_CUDA(cudaMemsetAsync(bad_routes, 0, sizeof(int32_t), lrb::as_stream(stream)));
        return MOE_OK;
    }
    return lrb::launch_permute(idx, tokens, top_k, experts, offsets, perm_token, perm_slot, route_pos, active,
                               num_active, bad_routes, lrb::as_stream(stream));
}
