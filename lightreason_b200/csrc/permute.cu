// Token permute: the eager expert dispatch order of Qwen3_5MoeExperts.forward
// (transformers qwen3_5_moe modeling :730-744) -- ascending expert, then
// slot-major, then token -- as a stable counting sort in one CTA.
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

namespace lrb {

namespace {
constexpr int kPermuteThreads = 1024;
constexpr int kPermuteWarps = kPermuteThreads / 32;
}  // namespace

__global__ void __launch_bounds__(kPermuteThreads) permute_kernel(const int64_t *__restrict__ idx, int tokens,
                                                                  int top_k, int experts,
                                                                  int32_t *__restrict__ offsets,
                                                                  int32_t *__restrict__ perm_token,
                                                                  int32_t *__restrict__ perm_slot,
                                                                  int32_t *__restrict__ route_pos,
                                                                  int32_t *__restrict__ active,
                                                                  int32_t *__restrict__ num_active,
                                                                  int32_t *__restrict__ bad_routes) {
    extern __shared__ int32_t smem[];
    int32_t *cnt = smem;                                 // [warps][experts]
    int32_t *total = smem + kPermuteWarps * experts;     // [experts]
    __shared__ int32_t warp_sums[kPermuteWarps];
    __shared__ int32_t bad;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int routes = tokens * top_k;
    const int chunk = ((routes + kPermuteWarps * 32 - 1) / (kPermuteWarps * 32)) * 32;
    const int r_begin = warp * chunk, r_end = min(routes, r_begin + chunk);

    for (int i = threadIdx.x; i < kPermuteWarps * experts; i += kPermuteThreads) cnt[i] = 0;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();

    // Pass 1: per-warp expert histogram.
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e = -1;
        if (r < r_end) {
            const int t = r % tokens, k = r / tokens;
            const int64_t v = idx[static_cast<size_t>(t) * top_k + k];
            if (v >= 0 && v < experts) e = static_cast<int>(v);
            else atomicAdd(&bad, 1);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e] += __popc(peers);
    }
    __syncthreads();

    // Column scan over warps, then an exclusive scan of the totals over experts.
    for (int e = threadIdx.x; e < experts; e += kPermuteThreads) {
        int run = 0;
        for (int w = 0; w < kPermuteWarps; ++w) {
            const int c = cnt[w * experts + e];
            cnt[w * experts + e] = run;
            run += c;
        }
        total[e] = run;
    }
    __syncthreads();
    // experts <= kPermuteThreads: one value per thread.
    const int my_total = threadIdx.x < experts ? total[threadIdx.x] : 0;
    int incl = my_total;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, s);
        if (lane >= s) incl += o;
    }
    if (lane == 31) warp_sums[warp] = incl;
    const unsigned has = __ballot_sync(0xffffffffu, my_total > 0);
    __syncthreads();
    if (warp == 0) {
        const int ws = warp_sums[lane];
        int wincl = ws;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, wincl, s);
            if (lane >= s) wincl += o;
        }
        warp_sums[lane] = wincl - ws;  // exclusive prefix of warp totals
    }
    __syncthreads();
    const int excl = warp_sums[warp] + incl - my_total;
    if (threadIdx.x < experts) {
        offsets[threadIdx.x] = excl;
        if (threadIdx.x == experts - 1) offsets[experts] = excl + my_total;
        for (int w = 0; w < kPermuteWarps; ++w) cnt[w * experts + threadIdx.x] += excl;
    }
    // Active experts, ascending: the same scan on the 0/1 "has routes" flags.
    __syncthreads();
    if (lane == 0) warp_sums[warp] = __popc(has);
    __syncthreads();
    if (warp == 0) {
        const int ws = warp_sums[lane];
        int wincl = ws;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, wincl, s);
            if (lane >= s) wincl += o;
        }
        warp_sums[lane] = wincl - ws;
        if (lane == 31) *num_active = wincl;
    }
    __syncthreads();
    if (my_total > 0) active[warp_sums[warp] + __popc(has & ((1u << lane) - 1))] = threadIdx.x;

    // Pass 2: stable placement.
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e = -1, t = 0, k = 0;
        if (r < r_end) {
            t = r % tokens;
            k = r / tokens;
            const int64_t v = idx[static_cast<size_t>(t) * top_k + k];
            if (v >= 0 && v < experts) e = static_cast<int>(v);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        int p = -1;
        if (e >= 0) p = cnt[warp * experts + e] + __popc(peers & ((1u << lane) - 1));
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e] += __popc(peers);
        __syncwarp();
        if (r < r_end) {
            route_pos[static_cast<size_t>(t) * top_k + k] = p;
            if (p >= 0) {
                perm_token[p] = t;
                perm_slot[p] = k;
            }
        }
    }
    if (bad_routes && threadIdx.x == 0) *bad_routes = bad;
}

int launch_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets, int32_t *perm_token,
                   int32_t *perm_slot, int32_t *route_pos, int32_t *active, int32_t *num_active, int32_t *bad_routes,
                   cudaStream_t stream) {
    const size_t smem = sizeof(int32_t) * static_cast<size_t>(kPermuteWarps + 1) * experts;
    static bool configured = false;
    if (!configured) {
        LRB_CUDA(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(sizeof(int32_t) * (kPermuteWarps + 1) * 1024)));
        configured = true;
    }
    permute_kernel<<<1, kPermuteThreads, smem, stream>>>(idx, tokens, top_k, experts, offsets, perm_token, perm_slot,
                                                          route_pos, active, num_active, bad_routes);
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
