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
    }
    __syncthreads();
}

}  // namespace lrb
