// Work plan of the grouped expert kernel, built by one CTA after routing: the
// groups (active experts in ascending id, then the shared expert), per-phase
// item prefix sums, zeroed dependency counters, the expert -> group map used by
// the combine, and the route -> token entries of the shared rows.
#pragma once

#include "common.cuh"
#include "kernels.cuh"
#include "routing.cuh"

namespace lrb {

struct PlanArgs {
    const int32_t *active, *num_active, *offsets;
    int use_slots, shared, routes, tokens, bn, ks, mb1, mb2, halves;
    int combine;  // 1: the grouped kernel runs the ordered combine (phase 3)
    GroupedGroup *groups;
    GroupedPlan *plan;
    int32_t *off1, *off2, *done1, *done2, *split_cnt;
    int split_cnt_len;
    int32_t *route_token, *group_of_expert;
    int32_t *stage_error;         // zeroed here: the host-staging kernels run after the plan
    const int32_t *router_error;  // folded into plan->error when non-null (the router ran before)
};

// Executed by every thread of one CTA.
__device__ __forceinline__ void plan_block(const PlanArgs &a, int *scratch) {
    const int n = *a.num_active;
    const int ng = n + (a.shared ? 1 : 0);
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        GroupedGroup G;
        if (g < n) {
            const int e = a.active[g];
            G.weight = a.use_slots ? g : e;
            G.begin = a.offsets[e];
            G.count = a.offsets[e + 1] - a.offsets[e];
            a.group_of_expert[e] = g;
        } else {
            G.weight = -1;
            G.begin = a.routes;
            G.count = a.tokens;
        }
        G.ntiles = (G.count + a.bn - 1) / a.bn;
        a.groups[g] = G;
        a.done1[g] = 0;
        a.done2[g] = 0;
    }
    if (a.shared)
        for (int t = threadIdx.x; t < a.tokens; t += blockDim.x) a.route_token[a.routes + t] = t;
    for (int i = threadIdx.x; i < a.split_cnt_len; i += blockDim.x) a.split_cnt[i] = 0;
    // Item prefix sums over the groups, blockDim.x groups at a time.
    int carry1 = 0, carry2 = 0;
    for (int base = 0; base < ng; base += blockDim.x) {
        const int g = base + threadIdx.x;
        int c1 = 0, c2 = 0;
        if (g < ng) {
            const int count = g < n ? a.offsets[a.active[g] + 1] - a.offsets[a.active[g]] : a.tokens;
            const int ntiles = (count + a.bn - 1) / a.bn;
            c1 = a.mb1 * a.ks * ntiles;
            c2 = a.mb2 * ntiles;
        }
        int t1 = 0, t2 = 0;
        const int e1 = block_exclusive_scan(c1, scratch, &t1);
        const int e2 = block_exclusive_scan(c2, scratch, &t2);
        if (g < ng) {
            a.off1[g] = carry1 + e1;
            a.off2[g] = carry2 + e2;
        }
        carry1 += t1;
        carry2 += t2;
    }
    if (threadIdx.x == 0) {
        a.off1[ng] = carry1;
        a.off2[ng] = carry2;
        a.plan->num_groups = ng;
        a.plan->items1 = carry1;
        a.plan->items2 = carry2;
        a.plan->items3 = a.combine ? a.tokens * a.halves : 0;
        a.plan->work = 0;
        a.plan->error = a.router_error ? *a.router_error : 0;
        if (a.stage_error) *a.stage_error = 0;
        a.plan->done2_total = 0;
        a.plan->xs_ready = 0;
        a.plan->act_ready = 0;
        a.plan->work2 = 0;
    }
    __syncthreads();
}

// permute_block and plan_block in one pass for the decode routing kernel:
// the expert thread that owns a column of the counting table also writes its
// group of the plan, with one three-way scan (route offsets, active-expert
// positions, token-tile prefix) in place of the five scans and the global
// re-reads of the two blocks run back to back.  Same outputs, same values.
// blockDim.x >= experts; cnt as for permute_block; scratch >= 100 ints.
template <class IdxOf>
__device__ void route_plan_block(IdxOf idx_of, int tokens, int top_k, int experts, int32_t *offsets,
                                 int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                                 int32_t *num_active, int32_t *bad_routes, const PlanArgs &a, int32_t *cnt,
                                 int *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int routes = tokens * top_k;
    const int warps = max(1, min(static_cast<int>(blockDim.x >> 5), (routes + 31) / 32));
    const int chunk = ((routes + warps * 32 - 1) / (warps * 32)) * 32;
    const int r_begin = warp < warps ? warp * chunk : routes;
    const int r_end = warp < warps ? min(routes, r_begin + chunk) : routes;
    int *bad_total = scratch + 99;

    for (int i = threadIdx.x; i < warps * experts; i += blockDim.x) cnt[i] = 0;
    if (threadIdx.x == 0) *bad_total = 0;
    __syncthreads();
    int bad = 0;
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e = -1;
        if (r < r_end) {
            const int64_t v = idx_of(r % tokens, r / tokens);
            if (v >= 0 && v < experts) e = static_cast<int>(v);
            else bad++;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e] += __popc(peers);
    }
    bad = __reduce_add_sync(0xffffffffu, bad);
    if (lane == 0 && bad) atomicAdd(bad_total, bad);
    __syncthreads();
    const int e = threadIdx.x;
    int total_e = 0;
    if (e < experts) {
        for (int w = 0; w < warps; ++w) {
            const int c = cnt[w * experts + e];
            cnt[w * experts + e] = total_e;
            total_e += c;
        }
    }
    const int nt_e = (total_e + a.bn - 1) / a.bn;
    int3 tot;
    const int3 ex = block_exclusive_scan3(make_int3(total_e, total_e > 0 ? 1 : 0, nt_e), scratch, &tot);
    const int n = tot.y;
    if (e < experts) {
        offsets[e] = ex.x;
        if (e == experts - 1) offsets[experts] = ex.x + total_e;
        for (int w = 0; w < warps; ++w) cnt[w * experts + e] += ex.x;
        if (total_e > 0) {
            const int g = ex.y;
            active[g] = e;
            GroupedGroup G;
            G.weight = a.use_slots ? g : e;
            G.begin = ex.x;
            G.count = total_e;
            G.ntiles = nt_e;
            a.groups[g] = G;
            a.done1[g] = 0;
            a.done2[g] = 0;
            a.off1[g] = a.mb1 * a.ks * ex.z;
            a.off2[g] = a.mb2 * ex.z;
            a.group_of_expert[e] = g;
        }
    }
    if (threadIdx.x == 0) {
        *num_active = n;
        if (bad_routes) *bad_routes = *bad_total;
        const int ng = n + (a.shared ? 1 : 0);
        int t1 = a.mb1 * a.ks * tot.z, t2 = a.mb2 * tot.z;
        if (a.shared) {
            GroupedGroup G;
            G.weight = -1;
            G.begin = a.routes;
            G.count = a.tokens;
            G.ntiles = (a.tokens + a.bn - 1) / a.bn;
            a.groups[n] = G;
            a.done1[n] = 0;
            a.done2[n] = 0;
            a.off1[n] = t1;
            a.off2[n] = t2;
            t1 += a.mb1 * a.ks * G.ntiles;
            t2 += a.mb2 * G.ntiles;
        }
        a.off1[ng] = t1;
        a.off2[ng] = t2;
        a.plan->num_groups = ng;
        a.plan->items1 = t1;
        a.plan->items2 = t2;
        a.plan->items3 = a.combine ? a.tokens * a.halves : 0;
        a.plan->work = 0;
        a.plan->error = a.router_error ? *a.router_error : 0;
        if (a.stage_error) *a.stage_error = 0;
        a.plan->done2_total = 0;
        a.plan->xs_ready = 0;
        a.plan->act_ready = 0;
        a.plan->work2 = 0;
    }
    if (a.shared)
        for (int t = threadIdx.x; t < a.tokens; t += blockDim.x) a.route_token[a.routes + t] = t;
    for (int i = threadIdx.x; i < a.split_cnt_len; i += blockDim.x) a.split_cnt[i] = 0;
    __syncthreads();
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e2 = -1, t = 0, k = 0;
        if (r < r_end) {
            t = r % tokens;
            k = r / tokens;
            const int64_t v = idx_of(t, k);
            if (v >= 0 && v < experts) e2 = static_cast<int>(v);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e2);
        int p = -1;
        if (e2 >= 0) p = cnt[warp * experts + e2] + __popc(peers & ((1u << lane) - 1));
        __syncwarp();
        if (e2 >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e2] += __popc(peers);
        __syncwarp();
        if (r < r_end) {
            route_pos[static_cast<size_t>(t) * top_k + k] = p;
            if (p >= 0) {
                perm_token[p] = t;
                perm_slot[p] = k;
            }
        }
    }
    __syncthreads();
}

}  // namespace lrb
