// Internal launchers shared between the translation units of libmoe_b200.so.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace lrb {

// Weights of one work group of the expert kernels: the routed expert whose
// routes occupy positions [begin, begin + count), or the shared expert.
struct Group {
    const uint16_t *gate;  // [I, H]
    const uint16_t *up;    // [I, H]
    const uint16_t *down;  // [H, I]
    int32_t begin;
    int32_t count;
};

// Groups resolved on the device (layer path): groups[g] for g < *num_groups;
// route_token[p] is the token of route position p.
struct DeviceGroups {
    const Group *groups;
    const int32_t *num_groups;
    const int32_t *route_token;
    __device__ __forceinline__ int n() const { return *num_groups; }
    __device__ __forceinline__ Group get(int g) const { return groups[g]; }
    __device__ __forceinline__ int token(int p) const { return route_token[p]; }
    __device__ __forceinline__ void on_start() const {}
};

// Groups passed by value (pointer-table entry points, one route per group).
constexpr int kMaxParamGroups = 128;
struct ParamGroups {
    Group groups[kMaxParamGroups];
    int32_t tokens[kMaxParamGroups];
    int32_t count;
    __device__ __forceinline__ int n() const { return count; }
    __device__ __forceinline__ Group get(int g) const { return groups[g]; }
    __device__ __forceinline__ int token(int p) const { return tokens[p]; }
    __device__ __forceinline__ void on_start() const {}
};

// Grouped tensor-core experts (grouped.cu).
struct GroupedGroup {
    int32_t weight;  // index into the expert bank (expert id or HBM slot); -1 = shared expert
    int32_t begin;   // first route position
    int32_t count;   // routes
    int32_t ntiles;  // token tiles of width BN
};
struct GroupedPlan {
    int32_t num_groups, items1, items2, items3, work, error, done2_total;
    int32_t xs_ready;   // epilogue warps that finished the in-kernel token gather
    int32_t act_ready;  // CTAs of the fused decode kernel that published their activations
    int32_t work2;      // item counter of a launch that runs phases 2-3 only
};

// The grouped kernel's plan read as pointer groups, for the warp-per-row
// expert kernels at the narrowest widths: weight index -> bank rows (expert
// id or HBM slot; -1 = the shared expert), the host-staging error folded
// into the plan's error word once.
struct PlanGroups {
    const GroupedGroup *groups;
    GroupedPlan *plan;
    const int32_t *route_token;
    const uint16_t *gate_up, *down, *sh_gate, *sh_up, *sh_down;
    int64_t gate_up_stride, down_stride;  // elements per bank entry
    int inner, hidden;
    const int32_t *stage_error;
    __device__ __forceinline__ int n() const { return plan->num_groups; }
    __device__ __forceinline__ Group get(int g) const { return resolve(groups[g]); }
    __device__ __forceinline__ Group resolve(const GroupedGroup G) const {
        Group r;
        if (G.weight >= 0) {
            r.gate = gate_up + static_cast<int64_t>(G.weight) * gate_up_stride;
            r.up = r.gate + static_cast<int64_t>(inner) * hidden;
            r.down = down + static_cast<int64_t>(G.weight) * down_stride;
        } else {
            r.gate = sh_gate;
            r.up = sh_up;
            r.down = sh_down;
        }
        r.begin = G.begin;
        r.count = G.count;
        return r;
    }
    __device__ __forceinline__ int token(int p) const { return route_token[p]; }
    __device__ __forceinline__ void on_start() const {
        if (stage_error) {
            const int e = *stage_error;
            if (e) atomicCAS(&plan->error, 0, e);
        }
    }
};
struct GroupedLaunch {
    const uint16_t *gate_up, *down;  // banks: [bank_experts, 2I, H], [bank_experts, H, I]
    int64_t gate_up_stride, down_stride;
    int bank_experts;
    const uint16_t *sh_gate, *sh_up, *sh_down;  // shared expert (may be null)
    const uint16_t *xs;                          // [rows, H] tokens in route order
    uint16_t *act, *y, *out;                     // [rows, I], [rows, H], [T, H]
    int rows;
    const GroupedGroup *groups;
    GroupedPlan *plan;
    const int32_t *off1, *off2;
    int32_t *done1, *done2, *split_cnt;
    float *part;
    const int32_t *route_pos;
    const int64_t *idx;
    const uint16_t *scores, *sig;
    const int32_t *group_of_expert;
    const int32_t *route_token;  // [rows] route -> token
    uint16_t *rows_out;            // [T, H]: write y per token (top_k 1, no shared), or null
    const int32_t *stage_error;    // nonzero: the host staging gave up; folded into plan->error
    const uint16_t *x;             // gather_x: tokens [T, H], gathered into xs by the kernel itself
    int gather_x;
    // Address tables (or null): row p of the plan is read from src_rows[p] and
    // its down output (no combine) stored to dst_rows[p]; row_ready[g] counts
    // the rows of group g gathered (zeroed by the plan).
    const int64_t *src_rows, *dst_rows;
    int32_t *row_ready;
    int32_t *error_out;  // or null: set to 3 when a wait of the kernel gave up
    int tokens, top_k, hidden, inner, bn, ks, ctas;
    // CTA pairs (grouped_pairs_for): the plan's items are 256 gate/up rows
    // (mb1 = inner / 256) and 512 down rows (mb2 = hidden / 512)
    int pairs;
    // which items this launch runs: 3 (0) all, 1 phase 1 only, 2 phases 2-3
    // only (after a phase-1 launch of the same plan)
    int phases;
};
struct PlanArgs;
int grouped_bn_for(int tokens);
int grouped_pair_clusters();
bool grouped_pairs_for(int bn, int ks, int inner, int hidden);
int grouped_ks_for(int tokens);
int grouped_tiles_max(int tokens, int experts, int top_k, int inner);
size_t grouped_part_floats(int tokens, int experts, int top_k, int inner);
int launch_grouped_plan(const PlanArgs &a, cudaStream_t stream);
int launch_gather_tokens(const uint16_t *x, const int32_t *route_token, const int32_t *offsets, int experts,
                         int routes, int shared_rows, int hidden, uint16_t *xs, cudaStream_t stream);
int launch_grouped(const GroupedLaunch &L, cudaStream_t stream);

// Expert-parallel exchange over peer memory (ep_p2p.cu); fields as moe_ep_p2p.
struct EpP2PArgs {
    const int64_t *peers;
    int64_t off_flags_publish, off_flags_return, off_count, off_meta, off_tokens, off_ret;
    int world, rank, capacity, hidden, top_k, experts, local_experts, own_rows;
    uint32_t *step;
    int32_t *sync, *error;
    const int32_t *placement;  // (owner << 16) | local index per expert, or null: contiguous
};
// BF16 tensor map: dims[0] innermost, 128-byte swizzle, box {64, box_rows(, 1)}.
int make_map_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides_bytes,
                  uint32_t box_rows);
// part != null: FP32 partials [ks][T][E] (router_select sums them); else BF16 logits.
int launch_router_tc(const uint16_t *x, const uint16_t *router, int tokens, int hidden, int experts,
                     uint16_t *logits, float *part, int ks, int32_t *error, cudaStream_t stream);
int router_tc_splits(int tokens, int experts);
int sm_count();

int launch_stage_row_codec(const int64_t *descriptors, const int32_t *active, const int32_t *num_active, int experts,
                           int max_slots, uint16_t *gate_up_slots, uint16_t *down_slots, int64_t gate_up_bytes,
                           int64_t down_bytes, int32_t *error, cudaStream_t stream,
                           const int32_t *slot_of_entry = nullptr, int bank0 = 0, int banks = 2);
// A non-blocking stream per device for work the library overlaps with the
// caller's stream (created on first use, kept for the process).
cudaStream_t side_stream();

int launch_router_logits(const uint16_t *x, const uint16_t *router, const uint16_t *gate_w, int tokens, int hidden,
                         int experts, uint16_t *logits, uint16_t *sig, cudaStream_t stream);
// With gate_w, also sig[t] = bf16(sigmoid(bf16(x[t] . gate_w))) (one warp per token).
// part != null: logits = bf16(sum over ks splits of part[k][t][e]) are formed
// (and stored to `logits`) before the selection.
int launch_router_select(const uint16_t *logits, const float *bias, int tokens, int experts, int top_k,
                         int64_t *idx, float *scores_f32, uint16_t *scores_bf16, cudaStream_t stream,
                         const uint16_t *x = nullptr, const uint16_t *gate_w = nullptr, int hidden = 0,
                         uint16_t *sig = nullptr, const float *part = nullptr, int ks = 1);
int check_router_args(int tokens, int hidden, int experts, int top_k);

// Decode routing (T <= kDecodeMaxTokens): split-K router partials, then one CTA
// that sums them, selects, permutes and plans.
constexpr int kDecodeMaxTokens = 64;
constexpr int kRouterSplit = 4;
// zero_words: n_zero int32 words set to 0 once the previous kernel in the
// stream is complete (the fused decode kernel's plan words when it routes
// itself), or null.
int launch_router_split(const uint16_t *x, const uint16_t *router, const uint16_t *gate_w, int tokens, int hidden,
                        int experts, float *part, cudaStream_t stream, int32_t *zero_words = nullptr,
                        int n_zero = 0);
struct DecodeRouteArgs {
    const float *part;            // [kRouterSplit][T][E+1] router partials (null with route_in)
    const float *bias;
    const int64_t *route_in;      // given ids (skip selection) or null
    uint16_t *logits, *sig, *scores;
    int64_t *idx;
    int tokens, experts, top_k, has_gate;
    int32_t *offsets, *perm_token, *perm_slot, *route_pos, *active, *num_active, *bad_routes;
};
int launch_route_decode(const DecodeRouteArgs &r, const PlanArgs &plan, cudaStream_t stream);

// Scratch ints the wide (multi-CTA) permute needs in `hist` (0: one CTA suffices).
int permute_hist_ints(int tokens, int top_k, int experts);
int launch_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets, int32_t *perm_token,
                   int32_t *perm_slot, int32_t *route_pos, int32_t *active, int32_t *num_active, int32_t *bad_routes,
                   cudaStream_t stream,
                   int32_t *hist = nullptr);

template <class Src>
int launch_experts(const Src &src, int max_groups, const uint16_t *x, int hidden, int inner, uint16_t *act,
                   uint16_t *y, cudaStream_t stream, cudaEvent_t between);

int launch_combine(const uint16_t *y, const int32_t *route_pos, const uint16_t *scores, int tokens, int top_k,
                   int hidden, const uint16_t *shared_y, const uint16_t *sig, uint16_t *out, cudaStream_t stream);

// The fused expert stage for T <= kFusedDecodeMaxTokens (csrc/decode.cu):
// gate/up, down and the ordered combine in one persistent launch over the
// routing plan.  fused_decode_fits: the shape and widths it takes (its shared
// memory holds the token rows, every activation row and a ring of weight rows).
// With route != null the kernel also routes (experts <= 256): it reads the
// router's FP32 partials, selects and plans in every CTA, and writes the
// routing outputs below (sig then receives the shared-expert gate); the plan
// words from error to act_ready must have been zeroed after the previous
// kernel (router_split's zero_words).
constexpr int kFusedDecodeMaxTokens = 2;
struct FusedDecodeRoute {
    const float *part;   // [kRouterSplit][T][E + 1] router partials
    const float *bias;   // [E] or null
    int experts;
    uint16_t *logits;    // [T, E]
    int64_t *idx;        // [T, K]
    uint16_t *scores;    // [T, K]
    int32_t *route_pos;  // [T, K]
    int32_t *counters;   // [0] distinct routed experts, [1] dropped routes
};
bool fused_decode_fits(int tokens, int top_k, int hidden, int inner, int max_groups, bool shared);
int launch_fused_decode(const PlanGroups &src, int max_groups, const uint16_t *x, uint16_t *act,
                        const int32_t *route_pos, const uint16_t *scores, uint16_t *sig, uint16_t *out,
                        int tokens, int top_k, int hidden, int inner, cudaStream_t stream,
                        const FusedDecodeRoute *route = nullptr);

}  // namespace lrb
