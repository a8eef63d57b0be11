// Token permute: the eager expert dispatch order of Qwen3_5MoeExperts.forward
// (transformers qwen3_5_moe modeling :730-744) -- ascending expert, then
// slot-major, then token -- as a stable counting sort: inside one CTA for up
// to kOneCtaRoutes routes, else across the GPU in three launches (below).
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

constexpr int64_t kOneCtaRoutes = 2048;  // at most this many routes: the one-CTA sort

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

// Wide permute: the route order r is cut into chunks of kChunk routes, one per
// warp.  count: each warp writes its chunk's per-expert counts to hist[c][e];
// column scan (a CTA per 32 experts): hist[c][e] becomes the count of expert e
// in the earlier chunks, and the last CTA turns the column totals into the
// expert offsets, active experts and the dropped-route count; place: each warp
// re-walks its chunk and puts every route at offsets[e] + hist[c][e] plus its
// rank among the equal experts before it.  The scattered position writes spread over many SMs.
constexpr int kChunk = 128;
constexpr int kWarpsPerCta = 8;

__global__ void __launch_bounds__(256) permute_count_kernel(const int64_t *__restrict__ idx, int tokens, int top_k,
                                                            int experts, int chunks, int32_t *__restrict__ hist) {
    extern __shared__ int32_t cnt_smem[];
    grid_dependency_wait();
    grid_dependency_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * kWarpsPerCta + warp;
    if (c == 0 && lane == 0) hist[static_cast<size_t>(chunks) * experts + experts] = 0;  // the column scan's counter
    if (c >= chunks) return;
    int32_t *cnt = cnt_smem + warp * experts;
    for (int e = lane; e < experts; e += 32) cnt[e] = 0;
    __syncwarp();
    const int routes = tokens * top_k;
    int64_t v[kChunk / 32];
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
        const int r = c * kChunk + 32 * j + lane;
        v[j] = r < routes ? idx[static_cast<size_t>(r % tokens) * top_k + r / tokens] : -1;
    }
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
        const int e = v[j] >= 0 && v[j] < experts ? static_cast<int>(v[j]) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[e] += __popc(peers);
        __syncwarp();
    }
    for (int e = lane; e < experts; e += 32) hist[static_cast<size_t>(c) * experts + e] = cnt[e];
}

// Column scan: CTA b owns experts [32b, 32b + 32), one per lane, and its 32
// warps split the chunks.  hist[c][e] becomes the count of expert e in the
// chunks before c; the column totals go to totals[e].  The last CTA to finish
// (a counter zeroed by the count kernel) scans the totals into the expert
// offsets, the active experts and the dropped-route count.
__global__ void __launch_bounds__(1024) permute_colscan_kernel(int32_t *__restrict__ hist, int chunks, int experts,
                                                               int routes, int32_t *__restrict__ totals,
                                                               int32_t *__restrict__ done,
                                                               int32_t *__restrict__ offsets,
                                                               int32_t *__restrict__ active,
                                                               int32_t *__restrict__ num_active,
                                                               int32_t *__restrict__ bad_routes) {
    __shared__ int part[32][33];
    __shared__ int scratch[100];
    __shared__ int last;
    grid_dependency_wait();
    grid_dependency_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * 32 + lane;
    const bool col = e < experts;
    const int per = (chunks + 31) / 32;
    const int c_begin = min(chunks, warp * per), c_end = min(chunks, c_begin + per);
    constexpr int kU = 8;
    int sum = 0;
    for (int c = c_begin; c < c_end; c += kU) {
        int v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) v[u] = col && c + u < c_end ? hist[static_cast<size_t>(c + u) * experts + e] : 0;
#pragma unroll
        for (int u = 0; u < kU; ++u) sum += v[u];
    }
    part[warp][lane] = sum;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 32; ++w) {
        const int v = part[w][lane];
        if (w < warp) before += v;
        total += v;
    }
    if (col) {
        int run = before;
        for (int c = c_begin; c < c_end; c += kU) {
            int v[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) v[u] = c + u < c_end ? hist[static_cast<size_t>(c + u) * experts + e] : 0;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                if (c + u < c_end) {
                    hist[static_cast<size_t>(c + u) * experts + e] = run;
                    run += v[u];
                }
            }
        }
        if (warp == 0) totals[e] = total;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int x = threadIdx.x;
    int t = 0;
    if (x < experts) t = __ldcg(totals + x);
    int3 all;
    const int3 ex = block_exclusive_scan3(make_int3(t, t > 0 ? 1 : 0, 0), scratch, &all);
    if (x < experts) {
        offsets[x] = ex.x;
        if (x == experts - 1) offsets[experts] = ex.x + t;
        if (t > 0) active[ex.y] = x;
    }
    if (x == 0) {
        *num_active = all.y;
        if (bad_routes) *bad_routes = routes - all.x;
    }
}

__global__ void __launch_bounds__(256) permute_place_kernel(const int64_t *__restrict__ idx, int tokens, int top_k,
                                                            int experts, int chunks,
                                                            const int32_t *__restrict__ hist,
                                                            const int32_t *__restrict__ offsets,
                                                            int32_t *__restrict__ perm_token,
                                                            int32_t *__restrict__ perm_slot,
                                                            int32_t *__restrict__ route_pos) {
    extern __shared__ int32_t base_smem[];
    grid_dependency_wait();
    grid_dependency_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * kWarpsPerCta + warp;
    if (c >= chunks) return;
    int32_t *base = base_smem + warp * experts;
    for (int e = lane; e < experts; e += 32) base[e] = hist[static_cast<size_t>(c) * experts + e] + offsets[e];
    __syncwarp();
    const int routes = tokens * top_k;
    int64_t v[kChunk / 32];
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
        const int r = c * kChunk + 32 * j + lane;
        v[j] = r < routes ? idx[static_cast<size_t>(r % tokens) * top_k + r / tokens] : -1;
    }
#pragma unroll
    for (int j = 0; j < kChunk / 32; ++j) {
        const int r = c * kChunk + 32 * j + lane;
        const int e = v[j] >= 0 && v[j] < experts ? static_cast<int>(v[j]) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        int p = -1;
        if (e >= 0) p = base[e] + __popc(peers & ((1u << lane) - 1));
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) base[e] += __popc(peers);
        __syncwarp();
        if (r < routes) {
            const int t = r % tokens, k = r / tokens;
            route_pos[static_cast<size_t>(t) * top_k + k] = p;
            if (p >= 0) {
                perm_token[p] = t;
                perm_slot[p] = k;
            }
        }
    }
}

int permute_hist_ints(int tokens, int top_k, int experts) {
    const int64_t routes = static_cast<int64_t>(tokens) * top_k;
    // chunk counts, then the column totals and the column scan's counter
    return routes <= kOneCtaRoutes ? 0 : static_cast<int>((routes + kChunk - 1) / kChunk) * experts + experts + 1;
}

int permute_smem_bytes(int warps, int experts) {
    return static_cast<int>(sizeof(int32_t) * static_cast<size_t>(warps + 1) * experts);
}

int launch_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets, int32_t *perm_token,
                   int32_t *perm_slot, int32_t *route_pos, int32_t *active, int32_t *num_active, int32_t *bad_routes,
                   cudaStream_t stream, int32_t *hist) {
    const int64_t routes = static_cast<int64_t>(tokens) * top_k;
    if (hist && routes > kOneCtaRoutes && experts <= 1024) {
        const int chunks = static_cast<int>((routes + kChunk - 1) / kChunk);
        const int ctas = (chunks + kWarpsPerCta - 1) / kWarpsPerCta;
        const size_t smem = sizeof(int32_t) * kWarpsPerCta * experts;
        if (smem > 48 * 1024) {
            const int most = static_cast<int>(sizeof(int32_t) * kWarpsPerCta * 1024);
            if (int rc = ensure_dynamic_smem(permute_count_kernel, most, "cudaFuncSetAttribute(permute_count)"))
                return rc;
            if (int rc = ensure_dynamic_smem(permute_place_kernel, most, "cudaFuncSetAttribute(permute_place)"))
                return rc;
        }
        if (int rc = launch_pdl(permute_count_kernel, dim3(ctas), dim3(256), smem, stream, "permute_count_kernel", idx,
                                tokens, top_k, experts, chunks, hist))
            return rc;
        int32_t *totals = hist + static_cast<size_t>(chunks) * experts;
        if (int rc = launch_pdl(permute_colscan_kernel, dim3((experts + 31) / 32), dim3(1024), 0, stream,
                                "permute_colscan_kernel", hist, chunks, experts, static_cast<int>(routes), totals,
                                totals + experts, offsets, active, num_active, bad_routes))
            return rc;
        return launch_pdl(permute_place_kernel, dim3(ctas), dim3(256), smem, stream, "permute_place_kernel", idx,
                          tokens, top_k, experts, chunks, hist, offsets, perm_token, perm_slot, route_pos);
    }
    const int smem = permute_smem_bytes(32, experts);
    if (int rc = ensure_dynamic_smem(permute_kernel, permute_smem_bytes(32, 1024), "cudaFuncSetAttribute(permute)"))
        return rc;
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
    // an empty batch still writes offsets (zeros) and num_active (0); its
    // per-route arrays may be NULL
    LRB_REQUIRE(offsets && active && num_active && (tokens == 0 || (idx && perm_token && perm_slot && route_pos)),
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

extern "C" int moe_permute_hist_ints(int tokens, int top_k, int experts) {
    if (tokens <= 0 || top_k <= 0 || experts <= 0) return 0;
    return lrb::permute_hist_ints(tokens, top_k, experts);
}

extern "C" int moe_permute_wide(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets,
                                int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                                int32_t *num_active, int32_t *bad_routes, int32_t *hist, void *stream) {
    LRB_REQUIRE(experts >= 1 && experts <= 1024, "moe_permute_wide: experts %d outside [1, 1024]", experts);
    LRB_REQUIRE(top_k >= 1 && tokens >= 0, "moe_permute_wide: bad tokens %d / top_k %d", tokens, top_k);
    LRB_REQUIRE(static_cast<int64_t>(tokens) * top_k < (1 << 30), "moe_permute_wide: too many routes");
    LRB_REQUIRE(!lrb::permute_hist_ints(tokens, top_k, experts) || hist,
                "moe_permute_wide: hist (moe_permute_hist_ints ints) is required at this size");
    if (tokens == 0 || !lrb::permute_hist_ints(tokens, top_k, experts))
        return moe_permute(idx, tokens, top_k, experts, offsets, perm_token, perm_slot, route_pos, active, num_active,
                           bad_routes, stream);
    LRB_REQUIRE(idx && offsets && perm_token && perm_slot && route_pos && active && num_active,
                "moe_permute_wide: null output");
    if (int rc = lrb::require_sm100()) return rc;
    return lrb::launch_permute(idx, tokens, top_k, experts, offsets, perm_token, perm_slot, route_pos, active,
                               num_active, bad_routes, lrb::as_stream(stream), hist);
}
