// One MoE layer on the device: router -> permute -> (host-resident gather) ->
// grouped SwiGLU experts + shared expert + ordered combine.  Every step reads
// its routing from device memory, so a call is a short chain of launches with
// no host synchronisation and can be captured in a CUDA graph.  Consecutive
// kernels use programmatic dependent launch, so each one's prologue overlaps
// its predecessor.
//
// T <= 2: split-K router partials, then one fused kernel that selects and
// plans in every CTA and runs gate/up, down and the combine (with host-staged
// experts or given routes the one-CTA routing kernel plans first; the
// warp-per-row GEMVs and the combine for shapes it cannot hold).  T <= 16: the
// same routing, then the grouped kernel, which gathers the token rows and
// runs the combine itself (so too up to 64 tokens, after the spread-out
// routing).  Wider calls: tensor-core router, selection, permute and plan as
// separate kernels, a token gather, the grouped kernel and the combine.
#include <algorithm>
#include <cstddef>

#include "common.cuh"
#include "kernels.cuh"
#include "plan.cuh"

namespace lrb {

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Byte offsets of the scratch arrays inside the caller's workspace.
struct Layout {
    size_t logits, sig, idx, scores, offsets, route_token, perm_slot, route_pos, active, counters, groups, plan, off1,
        off2, done1, done2, split_cnt, gofe, rpart, part, xs, act, y, perm_hist, rsplit, stage_e, stage_s, total;
    int router_ks;
    int split_len;
};

// Routing in one fused CTA (router_split + route_decode) or across the GPU
// (router_tc + router_select + permute + plan).  The one-CTA routing wins up to
// 16 tokens; at 64 the spread-out path is 23% faster for a whole 40-layer
// decode step (measured), as the single CTA serialises per-token work.
constexpr int kFusedRoutingMaxTokens = 16;
bool decode_routing(int tokens, int experts) { return tokens <= kFusedRoutingMaxTokens && experts <= 256; }

// At the narrowest widths the experts run without the tensor-core grouped
// kernel: as fused_decode_kernel (csrc/decode.cu), or, for shapes it cannot
// hold in shared memory, as warp-per-row GEMVs and the standalone combine.
constexpr int kGemvMaxTokens = 2;
bool gemv_experts(int tokens, bool rows_mode) { return tokens <= kGemvMaxTokens && !rows_mode; }

Layout layout(int tokens, int experts, int top_k, int hidden, int inner) {
    const size_t T = tokens, E = experts, K = top_k, R = T * K;
    Layout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes);
        return at;
    };
    L.logits = take(T * E * 2);
    L.sig = take(T * 2);
    L.idx = take(R * 8);
    L.scores = take(R * 2);
    L.offsets = take((E + 1) * 4);
    L.route_token = take((R + T) * 4);
    L.perm_slot = take(R * 4);
    L.route_pos = take(R * 4);
    L.active = take(E * 4);
    L.counters = take(8 * 4);  // num_active, bad_routes, host-stage error, slot overflow, router error, misses
    L.stage_e = take(E * 4);
    L.stage_s = take(E * 4);
    L.groups = take((E + 1) * sizeof(GroupedGroup));
    L.plan = take(sizeof(GroupedPlan));
    L.off1 = take((E + 2) * 4);
    L.off2 = take((E + 2) * 4);
    L.done1 = take((E + 1) * 4);
    L.done2 = take((E + 1) * 4);
    L.split_len = grouped_tiles_max(tokens, experts, top_k, inner) * 4;
    L.split_cnt = take(static_cast<size_t>(L.split_len) * 4);
    L.gofe = take(E * 4);
    L.perm_hist = take(static_cast<size_t>(permute_hist_ints(tokens, top_k, experts)) * 4);
    L.router_ks = !decode_routing(tokens, experts) ? router_tc_splits(tokens, experts) : 1;
    L.rsplit = take(L.router_ks > 1 ? static_cast<size_t>(L.router_ks) * T * E * 4 : 0);
    L.rpart = take(tokens <= kDecodeMaxTokens ? static_cast<size_t>(kRouterSplit) * T * (E + 1) * 4 : 0);
    L.part = take(grouped_part_floats(tokens, experts, top_k, inner) * 4);
    L.xs = take((R + T) * hidden * 2);
    L.act = take((R + T) * inner * 2);
    L.y = take((R + T) * hidden * 2);
    L.total = o;
    return L;
}

template <class T>
T *at(void *base, size_t offset) {
    return reinterpret_cast<T *>(static_cast<char *>(base) + offset);
}

// Work forked from the caller's stream onto the library's side stream and
// joined back: begin() creates the two events (allowed while the caller's
// stream captures; the side stream then joins the capture through the first
// wait), to_side() orders the side stream after the caller's work so far,
// side_done() marks the side work's end, join() makes the caller's stream wait
// for it.  The events are destroyed on every exit path; a wait already
// enqueued keeps its dependency.
struct SideFork {
    cudaStream_t side = nullptr;
    cudaEvent_t forked = nullptr, done = nullptr;

    int begin(cudaStream_t) {
        side = side_stream();
        LRB_REQUIRE(side != nullptr, "moe_layer_forward: no side stream on this device");
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        cudaError_t e = cudaEventCreateWithFlags(&forked, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
        cudaThreadExchangeStreamCaptureMode(&mode);
        if (e != cudaSuccess) return cuda_error(e, "cudaEventCreateWithFlags(side fork)");
        return MOE_OK;
    }
    int to_side(cudaStream_t s) {
        LRB_CUDA(cudaEventRecord(forked, s));
        LRB_CUDA(cudaStreamWaitEvent(side, forked, 0));
        return MOE_OK;
    }
    int side_done() {
        LRB_CUDA(cudaEventRecord(done, side));
        return MOE_OK;
    }
    int join(cudaStream_t s) {
        LRB_CUDA(cudaStreamWaitEvent(s, done, 0));
        return MOE_OK;
    }
    ~SideFork() {
        if (!forked && !done) return;
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        if (forked) cudaEventDestroy(forked);
        if (done) cudaEventDestroy(done);
        cudaThreadExchangeStreamCaptureMode(&mode);
    }
};

}  // namespace

// Copy every active expert's gate_up and down rows from the mapped host banks
// into HBM slot g (g-th active expert).  Grid (stripes, banks, max_slots), bank
// bank0 + blockIdx.y (0 gate_up, 1 down);
// 16-byte loads over the host link, four in flight per thread.
// Entry g < *num_active copies expert active[g] into slot slot_of_entry[g]
// (or slot g when slot_of_entry is null).
__global__ void __launch_bounds__(256) stage_experts_kernel(const int32_t *__restrict__ active,
                                                            const int32_t *__restrict__ num_active,
                                                            const int32_t *__restrict__ slot_of_entry,
                                                            const uint16_t *host_gate_up, const uint16_t *host_down,
                                                            int64_t gate_up_stride, int64_t down_stride,
                                                            int64_t gate_up_bytes, int64_t down_bytes,
                                                            uint16_t *gate_up_slots, uint16_t *down_slots,
                                                            int32_t *overflow, int bank0) {
    grid_dependency_wait();
    grid_dependency_trigger();
    const int g = blockIdx.z;
    const int n = *num_active;
    if (g == 0 && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *overflow = n > static_cast<int>(gridDim.z);
    if (g >= n) return;
    const int64_t e = active[g];
    const bool gu = bank0 + static_cast<int>(blockIdx.y) == 0;
    const uint4 *src = reinterpret_cast<const uint4 *>(gu ? host_gate_up + e * gate_up_stride
                                                          : host_down + e * down_stride);
    const int64_t bytes = gu ? gate_up_bytes : down_bytes;
    const int64_t slot = slot_of_entry ? slot_of_entry[g] : g;
    uint4 *dst = reinterpret_cast<uint4 *>(gu ? gate_up_slots + slot * (gate_up_bytes / 2)
                                              : down_slots + slot * (down_bytes / 2));
    const int64_t units = bytes / 16;
    const int64_t begin = units * blockIdx.x / gridDim.x, end = units * (blockIdx.x + 1) / gridDim.x;
    int64_t i = begin + threadIdx.x;
    for (; i + 3 * blockDim.x < end; i += 4 * blockDim.x) {
        uint4 v0 = ld_stream(src + i), v1 = ld_stream(src + i + blockDim.x);
        uint4 v2 = ld_stream(src + i + 2 * blockDim.x), v3 = ld_stream(src + i + 3 * blockDim.x);
        dst[i] = v0;
        dst[i + blockDim.x] = v1;
        dst[i + 2 * blockDim.x] = v2;
        dst[i + 3 * blockDim.x] = v3;
    }
    for (; i < end; i += blockDim.x) dst[i] = ld_stream(src + i);
}

// Expert cache (moe_layer_io.expert_cache): the slot banks keep experts across
// calls.  State: slot_of[E] (-1: not cached), expert_of[S] (-1: empty),
// stamp[S] (the call that last used the slot), then step, total routed-expert
// uses and total misses.  One CTA, after the plan: hits stamp their slots;
// misses take, in ascending expert order, the least recently used slots not
// used by this call (ties to the lower slot), and become the stage list; every
// routed group's weight index becomes its slot.  Needs S >= the routed groups
// of the call and S <= 1024.
__global__ void __launch_bounds__(1024) cache_plan_kernel(const int32_t *__restrict__ active,
                                                          const int32_t *__restrict__ num_active,
                                                          GroupedGroup *__restrict__ groups, int32_t *__restrict__ cache,
                                                          int experts, int slots, int32_t *__restrict__ stage_e,
                                                          int32_t *__restrict__ stage_s, int32_t *__restrict__ stage_n) {
    __shared__ unsigned long long keys[1024];
    __shared__ int miss_e[1024];
    __shared__ int scratch[33];
    grid_dependency_wait();
    grid_dependency_trigger();
    int32_t *slot_of = cache, *expert_of = cache + experts, *stamp = cache + experts + slots;
    int32_t *meta = cache + experts + 2 * slots;
    const int step = meta[0] + 1;
    const int n = *num_active;
    const int g = threadIdx.x;
    int e = -1;
    bool miss = false;
    if (g < n) {
        e = active[g];
        const int s = slot_of[e];
        if (s >= 0) stamp[s] = step;
        else miss = true;
    }
    __syncthreads();
    int n_miss = 0;
    const int m = block_exclusive_scan(miss ? 1 : 0, scratch, &n_miss);
    if (miss) miss_e[m] = e;
    int P = 1;
    while (P < slots) P <<= 1;
    for (int s = threadIdx.x; s < P; s += blockDim.x) {
        unsigned long long k = ~0ull;
        if (s < slots) {
            const unsigned used = stamp[s] == step ? 0x7fffffffu : static_cast<unsigned>(stamp[s]);
            k = (static_cast<unsigned long long>(used) << 32) | static_cast<unsigned>(s);
        }
        keys[s] = k;
    }
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int i = threadIdx.x;
            if (i < P) {
                const int o = i ^ j;
                if (o > i) {
                    const bool up = (i & k) == 0;
                    const unsigned long long a = keys[i], b = keys[o];
                    if ((a > b) == up) {
                        keys[i] = b;
                        keys[o] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (threadIdx.x < n_miss) {
        const int v = static_cast<int>(keys[threadIdx.x] & 0xffffffffull);
        const int ne = miss_e[threadIdx.x];
        const int old = expert_of[v];
        if (old >= 0) slot_of[old] = -1;
        slot_of[ne] = v;
        expert_of[v] = ne;
        stamp[v] = step;
        stage_e[threadIdx.x] = ne;
        stage_s[threadIdx.x] = v;
    }
    __syncthreads();
    if (g < n) groups[g].weight = slot_of[e];
    if (threadIdx.x == 0) {
        *stage_n = n_miss;
        meta[0] = step;
        meta[1] += n;
        meta[2] += n_miss;
    }
}

}  // namespace lrb

extern "C" {

size_t moe_layer_workspace_bytes(int tokens, int experts, int top_k, int hidden, int inner, int shared_inner) {
    (void)shared_inner;
    if (tokens < 0 || experts <= 0 || top_k <= 0 || hidden <= 0 || inner <= 0) return 0;
    return lrb::layout(tokens, experts, top_k, hidden, inner).total;
}

int moe_layer_forward(const moe_layer_weights *w, const uint16_t *x, int tokens, uint16_t *out,
                      const moe_layer_io *io, void *workspace, size_t workspace_bytes, void *stream) {
    using namespace lrb;
    // an empty batch is a no-op: x, out and the workspace may then be NULL
    LRB_REQUIRE(w && (tokens == 0 || (x && out)), "moe_layer_forward: weights, x and out are required");
    const moe_layer_io none{};
    if (!io) io = &none;
    const int E = w->experts, H = w->hidden, I = w->inner, K = w->top_k;
    if (int rc = check_router_args(tokens, H, E, K)) return rc;
    LRB_REQUIRE(I == 256 || I == 512 || I == 1024, "moe_layer_forward: inner %d not in {256, 512, 1024}", I);
    LRB_REQUIRE(H % 1024 == 0, "moe_layer_forward: hidden %d is not a multiple of 1024", H);
    const bool routed_in = io->route_in != nullptr;
    const bool shared = !routed_in && w->shared_gate != nullptr;
    const bool rows_mode = io->rows_mode != 0;
    LRB_REQUIRE(!rows_mode || (routed_in && K == 1), "moe_layer_forward: rows_mode needs route_in and top_k == 1");
    LRB_REQUIRE(!routed_in || rows_mode || io->weights_in, "moe_layer_forward: route_in needs weights_in");
    LRB_REQUIRE(K <= 16, "moe_layer_forward: top_k %d > 16", K);
    LRB_REQUIRE(routed_in || w->router, "moe_layer_forward: router weights required without route_in");
    LRB_REQUIRE(!shared || (w->shared_up && w->shared_down && w->shared_gate_w && w->shared_inner == I),
                "moe_layer_forward: shared expert needs gate/up/down/gate_w with shared_inner == inner");
    const bool packed_host = io->host_descriptors != nullptr;
    const bool staged = io->host_gate_up != nullptr || packed_host;
    LRB_REQUIRE(!staged || ((packed_host || io->host_down) && io->gate_up_slots && io->down_slots),
                "moe_layer_forward: host banks need slot banks");
    const int R = tokens * K;
    const int max_groups = std::min(E, R);
    LRB_REQUIRE(!staged || io->max_slots >= max_groups, "moe_layer_forward: max_slots %d < min(E, T*top_k) = %d",
                staged ? io->max_slots : 0, max_groups);
    const bool cached = io->expert_cache != nullptr;
    LRB_REQUIRE(!cached || (staged && io->max_slots <= 1024),
                "moe_layer_forward: expert_cache needs host banks and at most 1024 slots");
    LRB_REQUIRE(staged || (w->gate_up && w->down), "moe_layer_forward: expert banks required");
    const int64_t gu_stride = w->gate_up_stride ? w->gate_up_stride : static_cast<int64_t>(2) * I * H;
    const int64_t dn_stride = w->down_stride ? w->down_stride : static_cast<int64_t>(H) * I;
    // Rows are read with 16-byte loads, TMA and bulk copies: a misaligned base
    // is an argument error here rather than a fault on the device.
    auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    LRB_REQUIRE(a16(x) && a16(out) && a16(w->router) && a16(w->gate_up) && a16(w->down) && a16(w->shared_gate) &&
                    a16(w->shared_up) && a16(w->shared_down) && a16(w->shared_gate_w) && a16(io->host_gate_up) &&
                    a16(io->host_down) && a16(io->gate_up_slots) && a16(io->down_slots) && gu_stride % 8 == 0 &&
                    dn_stride % 8 == 0,
                "moe_layer_forward: row pointers must be 16-byte aligned and expert strides multiples of 8");
    if (tokens == 0) return MOE_OK;
    const Layout L = layout(tokens, E, K, H, I);
    LRB_REQUIRE(workspace && workspace_bytes >= L.total, "moe_layer_forward: workspace %zu < %zu bytes",
                workspace_bytes, L.total);
    if (int rc = require_sm100()) return rc;
    cudaStream_t s = as_stream(stream);
    // Under stream capture an ordinary record is only a dependency node; an
    // external record node keeps the event usable for timing each replay.
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (io->stage_events) LRB_CUDA(cudaStreamIsCapturing(s, &capturing));
    auto mark_on = [&](int i, cudaStream_t st) -> int {
        if (io->stage_events && i < io->num_stage_events && io->stage_events[i])
            LRB_CUDA(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(io->stage_events[i]), st,
                                              capturing == cudaStreamCaptureStatusActive ? cudaEventRecordExternal
                                                                                         : cudaEventRecordDefault));
        return MOE_OK;
    };
    auto mark = [&](int i) -> int { return mark_on(i, s); };
    if (int rc = mark(0)) return rc;

    void *ws = workspace;
    const bool decode = decode_routing(tokens, E);
    const int bn = grouped_bn_for(tokens), ks = grouped_ks_for(tokens);
    uint16_t *sig = at<uint16_t>(ws, L.sig);
    uint16_t *logits = io->logits_out ? io->logits_out : at<uint16_t>(ws, L.logits);
    int64_t *idx = routed_in ? const_cast<int64_t *>(io->route_in)
                             : io->idx_out ? io->idx_out : at<int64_t>(ws, L.idx);
    uint16_t *scores = routed_in ? const_cast<uint16_t *>(io->weights_in)
                                 : io->scores_out ? io->scores_out : at<uint16_t>(ws, L.scores);
    int32_t *offsets = at<int32_t>(ws, L.offsets), *route_token = at<int32_t>(ws, L.route_token);
    int32_t *route_pos = at<int32_t>(ws, L.route_pos), *active = at<int32_t>(ws, L.active);
    int32_t *counters = at<int32_t>(ws, L.counters);
    GroupedGroup *groups = at<GroupedGroup>(ws, L.groups);
    GroupedPlan *plan = at<GroupedPlan>(ws, L.plan);

    PlanArgs pa{};
    pa.active = active;
    pa.num_active = counters + 0;
    pa.offsets = offsets;
    pa.use_slots = staged;
    pa.shared = shared;
    pa.routes = R;
    pa.tokens = tokens;
    pa.bn = bn;
    pa.ks = ks;
    // items of the grouped kernel: 128 gate/up rows and 256 down rows, twice
    // that for CTA pairs
    const bool pairs = grouped_pairs_for(bn, ks, I, H);
    pa.mb1 = I / (pairs ? 256 : 128);
    pa.mb2 = H / (pairs ? 512 : 256);
    pa.halves = H / 1024;
    pa.groups = groups;
    pa.plan = plan;
    pa.off1 = at<int32_t>(ws, L.off1);
    pa.off2 = at<int32_t>(ws, L.off2);
    pa.done1 = at<int32_t>(ws, L.done1);
    pa.done2 = at<int32_t>(ws, L.done2);
    pa.split_cnt = at<int32_t>(ws, L.split_cnt);
    pa.split_cnt_len = L.split_len;
    pa.route_token = route_token;
    pa.group_of_expert = at<int32_t>(ws, L.gofe);
    pa.stage_error = counters + 2;
    pa.router_error = decode ? nullptr : counters + 4;
    // Decode widths combine inside the expert kernel (one launch less on the
    // latency path); wider calls run the standalone combine after it, whose
    // parallelism the persistent kernel's epilogue warps cannot match.
    const bool gemv = gemv_experts(tokens, rows_mode != 0);
    const bool fused_combine = tokens <= kDecodeMaxTokens && !rows_mode && !gemv;
    pa.combine = fused_combine ? 1 : 0;
    // At the narrowest widths with HBM-resident experts the fused decode kernel
    // also routes (every CTA selects and plans from the router partials), so
    // route_decode_kernel and its launch gap leave the chain; router_split then
    // zeroes the plan words the fused kernel counts on (error .. act_ready).
    const int gemv_groups = std::min(E, R) + (shared ? 1 : 0);
    const bool self_route = gemv && decode && !routed_in && !staged && E <= 256 &&
                            fused_decode_fits(tokens, K, H, I, gemv_groups, shared);
    static_assert(offsetof(GroupedPlan, act_ready) == offsetof(GroupedPlan, error) + 3 * sizeof(int32_t),
                  "plan words error .. act_ready are contiguous");

    if (decode) {
        float *rpart = at<float>(ws, L.rpart);
        if (!routed_in) {
            if (int rc = launch_router_split(x, w->router, shared ? w->shared_gate_w : nullptr, tokens, H, E, rpart,
                                             s, self_route ? &plan->error : nullptr, self_route ? 4 : 0))
                return rc;
        }
        if (int rc = mark(1)) return rc;
        DecodeRouteArgs ra{};
        ra.part = routed_in ? nullptr : rpart;
        ra.bias = w->router_bias;
        ra.route_in = routed_in ? io->route_in : nullptr;
        ra.logits = logits;
        ra.sig = sig;
        ra.scores = scores;
        ra.idx = idx;
        ra.tokens = tokens;
        ra.experts = E;
        ra.top_k = K;
        ra.has_gate = shared;
        ra.offsets = offsets;
        ra.perm_token = route_token;
        ra.perm_slot = at<int32_t>(ws, L.perm_slot);
        ra.route_pos = route_pos;
        ra.active = active;
        ra.num_active = counters + 0;
        ra.bad_routes = counters + 1;
        if (!self_route)
            if (int rc = launch_route_decode(ra, pa, s)) return rc;
        if (int rc = mark(2)) return rc;
    } else {
        LRB_CUDA(cudaMemsetAsync(counters + 4, 0, sizeof(int32_t), s));
        if (!routed_in) {
            // tensor-core logits, then selection and the shared-expert gate
            float *rsplit = L.router_ks > 1 ? at<float>(ws, L.rsplit) : nullptr;
            if (int rc = launch_router_tc(x, w->router, tokens, H, E, logits, rsplit, L.router_ks, counters + 4, s))
                return rc;
            if (int rc = launch_router_select(logits, w->router_bias, tokens, E, K, idx, nullptr, scores, s, x,
                                              shared ? w->shared_gate_w : nullptr, H, shared ? sig : nullptr, rsplit,
                                              L.router_ks))
                return rc;
        }
        if (int rc = mark(1)) return rc;
        if (int rc = launch_permute(idx, tokens, K, E, offsets, route_token, at<int32_t>(ws, L.perm_slot), route_pos,
                                    active, counters + 0, counters + 1, s, at<int32_t>(ws, L.perm_hist)))
            return rc;
        if (int rc = launch_grouped_plan(pa, s)) return rc;
        if (int rc = mark(2)) return rc;
    }

    const uint16_t *gu_base = w->gate_up, *dn_base = w->down;
    int64_t gu_str = gu_stride, dn_str = dn_stride;
    // stage list: every active expert into slot g, or with the cache only the misses into their slots
    const int32_t *stage_list = active, *stage_count = counters + 0, *stage_slot = nullptr;
    if (cached) {
        int32_t *se = at<int32_t>(ws, L.stage_e), *ss = at<int32_t>(ws, L.stage_s);
        if (int rc = launch_pdl(cache_plan_kernel, dim3(1), dim3(1024), 0, s, "cache_plan_kernel", active,
                                counters + 0, groups, io->expert_cache, E, io->max_slots, se, ss, counters + 5))
            return rc;
        stage_list = se;
        stage_slot = ss;
        stage_count = counters + 5;
    }
    auto stage_banks = [&](int bank0, int banks, cudaStream_t st) -> int {
        if (packed_host)
            return launch_stage_row_codec(io->host_descriptors, stage_list, stage_count, E, max_groups,
                                          io->gate_up_slots, io->down_slots, static_cast<int64_t>(2) * I * H * 2,
                                          static_cast<int64_t>(H) * I * 2, counters + 2, st, stage_slot, bank0, banks);
        return launch_pdl(stage_experts_kernel, dim3(64, banks, max_groups), dim3(256), 0, st, "stage_experts_kernel",
                          stage_list, stage_count, stage_slot, io->host_gate_up, io->host_down, gu_stride, dn_stride,
                          static_cast<int64_t>(2) * I * H * 2, static_cast<int64_t>(H) * I * 2, io->gate_up_slots,
                          io->down_slots, counters + 3, bank0);
    };
    // Host-resident experts on the grouped path: the gate/up banks cross the
    // host link first on the caller's stream; the down banks follow on the
    // library's side stream while the grouped kernel runs phase 1 (gate/up,
    // which reads no down bank), and phases 2-3 wait for them.  The link stays
    // busy throughout and the gate/up products leave the critical path.
    const bool split = staged && !gemv;
    SideFork fork;
    if (staged) {
        if (split) {
            if (int rc = fork.begin(s)) return rc;
            if (int rc = stage_banks(0, 1, s)) return rc;
            if (int rc = fork.to_side(s)) return rc;
            if (int rc = stage_banks(1, 1, fork.side)) return rc;
            if (int rc = mark_on(3, fork.side)) return rc;  // both banks staged
            if (int rc = fork.side_done()) return rc;
        } else {
            if (int rc = stage_banks(0, 2, s)) return rc;
            if (int rc = mark(3)) return rc;
        }
        gu_base = io->gate_up_slots;
        dn_base = io->down_slots;
        gu_str = static_cast<int64_t>(2) * I * H;
        dn_str = static_cast<int64_t>(H) * I;
    } else if (int rc = mark(3)) {
        return rc;
    }
    uint16_t *xs = at<uint16_t>(ws, L.xs), *act = at<uint16_t>(ws, L.act), *y = at<uint16_t>(ws, L.y);
    // At decode widths the grouped kernel gathers the token rows itself (its
    // epilogue warps are idle while the first weight tiles stream in).
    if (!fused_combine && !gemv)
        if (int rc = launch_gather_tokens(x, route_token, offsets, E, R, shared ? tokens : 0, H, xs, s)) return rc;
    if (int rc = mark(4)) return rc;
    if (gemv) {
        PlanGroups pg{groups, plan, route_token, gu_base, dn_base, shared ? w->shared_gate : nullptr,
                      shared ? w->shared_up : nullptr, shared ? w->shared_down : nullptr, gu_str, dn_str, I, H,
                      self_route ? nullptr : counters + 2};
        const int max_groups = gemv_groups;
        if (fused_decode_fits(tokens, K, H, I, max_groups, shared)) {
            const FusedDecodeRoute fr{at<float>(ws, L.rpart), w->router_bias, E, logits, idx, scores, route_pos,
                                      counters};
            if (int rc = launch_fused_decode(pg, max_groups, x, act, route_pos, scores, shared ? sig : nullptr, out,
                                             tokens, K, H, I, s, self_route ? &fr : nullptr))
                return rc;
            if (int rc = mark(5)) return rc;
        } else {
            if (int rc = launch_experts(pg, max_groups, x, H, I, act, y, s, nullptr)) return rc;
            if (int rc = mark(5)) return rc;
            if (int rc = launch_combine(y, route_pos, scores, tokens, K, H,
                                        shared ? y + static_cast<size_t>(R) * H : nullptr, shared ? sig : nullptr, out,
                                        s))
                return rc;
        }
        if (io->status) LRB_CUDA(cudaMemcpyAsync(io->status, &plan->error, sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
        if (int rc = mark(6)) return rc;
        return mark(7);
    }
    GroupedLaunch GL{};
    GL.gate_up = gu_base;
    GL.down = dn_base;
    GL.gate_up_stride = gu_str;
    GL.down_stride = dn_str;
    GL.bank_experts = staged ? io->max_slots : E;
    GL.sh_gate = shared ? w->shared_gate : nullptr;
    GL.sh_up = shared ? w->shared_up : nullptr;
    GL.sh_down = shared ? w->shared_down : nullptr;
    GL.xs = xs;
    GL.act = act;
    GL.y = y;
    GL.out = out;
    GL.rows = R + (shared ? tokens : 0);
    GL.groups = groups;
    GL.plan = plan;
    GL.off1 = pa.off1;
    GL.off2 = pa.off2;
    GL.done1 = pa.done1;
    GL.done2 = pa.done2;
    GL.split_cnt = pa.split_cnt;
    GL.part = at<float>(ws, L.part);
    GL.route_pos = route_pos;
    GL.idx = idx;
    GL.scores = scores;
    GL.sig = shared ? sig : nullptr;
    GL.group_of_expert = pa.group_of_expert;
    GL.route_token = route_token;
    GL.rows_out = rows_mode ? out : nullptr;
    GL.stage_error = counters + 2;
    GL.x = x;
    GL.gather_x = fused_combine ? 1 : 0;
    GL.tokens = tokens;
    GL.top_k = K;
    GL.hidden = H;
    GL.inner = I;
    GL.bn = bn;
    GL.ks = ks;
    GL.ctas = sm_count();
    GL.pairs = pairs;
    GL.phases = split ? 1 : 3;
    if (int rc = launch_grouped(GL, s)) return rc;
    if (split) {
        if (int rc = fork.join(s)) return rc;  // the down banks are in their slots
        GL.phases = 2;
        GL.gather_x = 0;  // phase 1 gathered the token rows
        if (int rc = launch_grouped(GL, s)) return rc;
    }
    if (int rc = mark(5)) return rc;
    if (!fused_combine && !rows_mode) {
        if (int rc = launch_combine(y, route_pos, scores, tokens, K, H, shared ? y + static_cast<size_t>(R) * H : nullptr,
                                    shared ? sig : nullptr, out, s))
            return rc;
    }
    if (io->status) LRB_CUDA(cudaMemcpyAsync(io->status, &plan->error, sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    if (int rc = mark(6)) return rc;
    return mark(7);
}

}  // extern "C"
