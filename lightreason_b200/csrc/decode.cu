// The expert stage of one layer step at the narrowest decode widths, fused:
// gate/up, the SiLU gate, down and the ordered combine in one persistent
// kernel, one CTA per SM (modeling_qwen3_5_moe.py:745-750 and :788-790;
// edge35b/cpu_experts.c:59-68; edge35b/fused_experts.py:27-37).
//
// Why one kernel: at T <= 2 the step moves ~57 MB of weights (8 routed experts
// and the shared one) and nothing else of size, so the time goes to the
// dependency chain (gate/up -> down -> combine as three launches, each with a
// grid-completion wait) and to streaming weights through registers.  Here a
// producer thread per CTA streams the CTA's share of the weights into a
// shared-memory ring with bulk copies of 16-32 KB (the per-SM copy rate grows
// with the bytes of each ring handoff), eight consumer warps in two groups of
// four do the dot products out of the ring, and the only grid-wide wait is the
// one the math needs: down reads every activation of its group.
//
// Work split (the same formula in every CTA, no table): the gate/up rows go to
// the CTAs as quads (rows 4k..4k+3 of one group's gate and up), evenly, since
// the grid-wide wait follows them -- the shared expert's quads first, by a
// split of their own that needs no routing, so each CTA issues them before it
// waits for the router and they stream while the routing runs; then the
// routed groups' quads.  The hidden columns are cut into units of 8;
// CTA c owns units c, c + A, ... (A = CTAs) and computes down rows 8u..8u+7 of
// EVERY group, so it holds every routed row of its columns and runs the
// ordered combine for them itself -- no second grid wait and no y round trip
// through global memory.  Ring items: the CTA's quads (gate rows, then up
// rows: 16H bytes; warp j of the consumer group that takes the item handles
// row pair j), then its down chunks (8 rows x I of one group and unit, 16I
// bytes) four to an item (warp j takes chunk j).  The down chunks enter the
// ring as the last quads leave it, so at decode widths they are in shared
// memory by the time the grid-wide wait ends.
//
// Phase A (quads): act[row] = bf16(bf16(silu(bf16(gate))) * bf16(up)) per
// routed token of the group, the eager rounding points; stored to global
// memory.  Then the CTA publishes (fence + counter) and waits until every CTA
// has (bounded, 2 s).  Phase B (chunks): every activation row is staged in
// shared memory once, y[row][col] = bf16(down . act[row]) for each row of the
// group, kept in shared memory.  Combine: per (token, 8 columns) the routed
// rows in ascending route position (the order is ranked once per token at
// start), acc = bf16(acc + bf16(y * w)), then the gated shared row, as the
// standalone combine kernel does.
//
// Routing in the kernel (HBM-resident experts, no given routes): every CTA
// also sums the router's K-quarter partials, selects the top-k of each token
// and builds the eager-order plan in shared memory (fused_route), so the
// one-CTA routing kernel and its launch gap leave the chain; CTA 0 writes the
// ids, weights, logits and shared-expert gate.  Before its grid-dependency wait
// each CTA also asks L2 for its slice of the shared expert's rows.
//
// Every wait is bounded; on timeout the CTA raises the plan's error word,
// skips the rest of its math, waits (bounded) for its own copies in flight and
// returns.  All CTAs must be resident at once: the grid is one CTA per SM,
// the kernel takes most of an SM's shared memory, and it is launched with the
// cooperative attribute so that the launch waits until every CTA fits.
#include <algorithm>

#include <climits>

#include "common.cuh"
#include "kernels.cuh"
#include "routing.cuh"
#include "sm100.cuh"

namespace lrb {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kFusedThreads = kConsumers + 32;  // + the producer warp
constexpr int kSub = 4;                         // warps (row pairs, down chunks) per ring item
constexpr int kGroups = kConsumerWarps / kSub;  // consumer groups; they take the ring items in turn
constexpr int kUnit = 8;                        // hidden columns per unit (rows of a down chunk)
constexpr int kMaxSlots = 32;
constexpr int kFusedMaxTopK = 16;
constexpr uint64_t kFusedWaitNs = 2000000000ull;  // 2 s: far beyond any legal wait

struct FusedParams {
    PlanGroups src;
    const uint16_t *x;          // [T, H] token rows
    uint16_t *act;              // [rows, I] activations, phase A -> phase B
    const int32_t *route_pos;   // [T, K] route position of (token, slot), -1 = dropped
    const uint16_t *scores;     // [T, K] BF16 routing weights
    uint16_t *sig;              // [T] BF16 shared-expert gate (written here when route != 0)
    uint16_t *out;              // [T, H]
    int tokens, top_k, rows;    // rows = T * K (+ T with a shared expert)
    int max_groups, slots, units_max, has_shared;
    // route != 0: the routing runs in the kernel (every CTA selects from the
    // router's FP32 partials and plans in shared memory; CTA 0 writes the
    // routing outputs); route_pos, scores and src's group table are unused.
    int route, experts;
    const float *part;          // [4][T][E + 1] router partials (column E: the shared-expert gate)
    const float *bias;          // [E] selection bias or null
    uint16_t *logits_out;       // [T, E]
    int64_t *idx_out;           // [T, K]
    uint16_t *scores_out;       // [T, K]
    int32_t *route_pos_out;     // [T, K]
    int32_t *counters;          // [0] distinct routed experts, [1] dropped routes
};

// Shared-memory layout in bytes, computed the same way on host and device.
struct FusedLayout {
    int slot_bytes, ring, xs, acts, ys, grp, tok, pos, spos, wt, swt, sig, bars, total;
};
__host__ __device__ inline int fused_align16(int v) { return (v + 15) & ~15; }
__host__ __device__ inline FusedLayout fused_layout(int slots, int T, int H, int I, int rows, int max_groups, int K,
                                                    int units_max) {
    FusedLayout L{};
    L.slot_bytes = 4 * kSub * H > 16 * kSub * I ? 4 * kSub * H : 16 * kSub * I;
    int o = 0;
    L.ring = o;
    o += slots * L.slot_bytes;
    L.xs = o;
    o += fused_align16(T * H * 2);
    L.acts = o;
    o += fused_align16(rows * I * 2);
    L.ys = o;
    o += fused_align16(units_max * rows * kUnit * 2);
    L.grp = o;
    o += fused_align16(max_groups * static_cast<int>(sizeof(GroupedGroup)));
    L.tok = o;
    o += fused_align16(rows * 4);
    L.pos = o;
    o += fused_align16(T * K * 4);
    L.spos = o;
    o += fused_align16(T * K * 4);
    L.wt = o;
    o += fused_align16(T * K * 2);
    L.swt = o;
    o += fused_align16(T * K * 2);
    L.sig = o;
    o += fused_align16(T * 2);
    L.bars = o;
    o += 2 * kMaxSlots * 8 + 16;  // full[], empty[], abort flag, group count
    L.total = o;
    return L;
}

__device__ __forceinline__ uint64_t fused_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool fused_wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = fused_now();
    for (uint32_t i = 1;; ++i) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if ((i & 63) == 0 && fused_now() - t0 > kFusedWaitNs) {
            *abort = 1;
            return false;
        }
    }
}

// Routing for T <= 2 inside the kernel, the arithmetic of route_decode_kernel
// and route_plan_block (csrc/router.cu, csrc/plan.cuh): logits = bf16(the sum
// of the K-quarter partials in order), top-k on logits + bias, BF16 weights,
// the shared-expert gate bf16(sigmoid(bf16 logit)); routes r = k * T + t placed
// in ascending expert order, stable in r (the eager order); one group per
// distinct expert in ascending order, the shared expert's group last.  Warp t
// selects for token t, then warp 0 plans (at most 32 routes: one per lane).
// Every thread of the CTA calls it; sel holds T * K ints of scratch.
template <int VPL>
__device__ __forceinline__ void fused_route(const FusedParams &P, GroupedGroup *grp, int32_t *tok, int32_t *pos_s,
                                            uint16_t *wt_s, uint16_t *sig_s, int32_t *sel, int *n_groups) {
    const int T = P.tokens, K = P.top_k, E = P.experts, R = T * K, cols = E + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool out = blockIdx.x == 0;
    if (warp < T) {
        const int t = warp;
        const float *__restrict__ part = P.part;
        const float *__restrict__ bias = P.bias;
        // every load of the token first (one L2 round trip), then the sums
        float p[VPL][kRouterSplit], b[VPL], gp[kRouterSplit];
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            const int e = min(lane + 32 * v, E - 1);
#pragma unroll
            for (int k = 0; k < kRouterSplit; ++k) p[v][k] = part[(static_cast<size_t>(k) * T + t) * cols + e];
            b[v] = bias ? bias[e] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kRouterSplit; ++k) gp[k] = part[(static_cast<size_t>(k) * T + t) * cols + E];
        float z[VPL];
        uint16_t lg[VPL];
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < kRouterSplit; ++k) sum += p[v][k];
            lg[v] = f2bf(sum);
            z[v] = lane + 32 * v < E ? bf2f(lg[v]) + b[v] : -INFINITY;
        }
        uint16_t sg = 0;
        if (P.has_shared) {
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < kRouterSplit; ++k) sum += gp[k];
            sg = f2bf(sigmoid_f32(bf2f(f2bf(sum))));
            if (lane == 0) sig_s[t] = sg;
        }
        int e;
        float w;
        warp_topk<VPL>([&](int j) { return z[j >> 5]; }, E, K, &e, &w);
        if (lane < K) {
            sel[t * K + lane] = e;
            wt_s[t * K + lane] = f2bf(w);
        }
        if (out) {
#pragma unroll
            for (int v = 0; v < VPL; ++v)
                if (lane + 32 * v < E) P.logits_out[static_cast<size_t>(t) * E + lane + 32 * v] = lg[v];
            if (lane == 0 && P.has_shared) P.sig[t] = sg;
            if (lane < K) {
                P.idx_out[static_cast<size_t>(t) * K + lane] = e;
                P.scores_out[static_cast<size_t>(t) * K + lane] = f2bf(w);
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        int e = INT_MAX, t = 0, k = 0;
        if (lane < R) {
            t = lane % T;
            k = lane / T;
            e = sel[t * K + k];
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const bool leader = lane < R && lane == __ffs(peers) - 1;
        const unsigned leaders = __ballot_sync(0xffffffffu, leader);
        int p = 0, g = 0;
        for (int j = 0; j < R; ++j) {
            const int ej = __shfl_sync(0xffffffffu, e, j);
            p += (ej < e || (ej == e && j < lane)) ? 1 : 0;
            g += (((leaders >> j) & 1u) && ej < e) ? 1 : 0;
        }
        const int routed = __popc(leaders);
        if (lane < R) {
            pos_s[t * K + k] = p;
            tok[p] = t;
            if (out) P.route_pos_out[t * K + k] = p;
        }
        if (leader) {
            GroupedGroup G;
            G.weight = e;
            G.begin = p;
            G.count = __popc(peers);
            G.ntiles = 1;
            grp[g] = G;
        }
        if (P.has_shared && lane < T) tok[R + lane] = lane;
        if (lane == 0) {
            int n = routed;
            if (P.has_shared) {
                GroupedGroup G;
                G.weight = -1;
                G.begin = R;
                G.count = T;
                G.ntiles = 1;
                grp[n++] = G;
            }
            *n_groups = n;
            if (out) {
                P.counters[0] = routed;
                P.counters[1] = 0;
                P.src.plan->num_groups = n;
            }
        }
    }
    __syncthreads();
}

// The consumer warps only (the producer warp leaves early).
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

template <int NW, int NI>
__global__ void __launch_bounds__(kFusedThreads, 1) fused_decode_kernel(const FusedParams P) {
    constexpr int H = NW * 256, I = NI * 256;
    constexpr int HU = H / 8, IU = I / 8;  // 16-byte units of a row
    constexpr int QPG = I / kSub;          // quads per group
    extern __shared__ __align__(128) uint8_t smem[];
    const int T = P.tokens, K = P.top_k, rows = P.rows, S = P.slots;
    const FusedLayout L = fused_layout(S, T, H, I, rows, P.max_groups, K, P.units_max);
    uint8_t *ring = smem + L.ring;
    uint4 *xs = reinterpret_cast<uint4 *>(smem + L.xs);
    uint4 *acts = reinterpret_cast<uint4 *>(smem + L.acts);
    uint16_t *ys = reinterpret_cast<uint16_t *>(smem + L.ys);
    GroupedGroup *grp = reinterpret_cast<GroupedGroup *>(smem + L.grp);
    int32_t *tok = reinterpret_cast<int32_t *>(smem + L.tok);
    int32_t *pos_s = reinterpret_cast<int32_t *>(smem + L.pos);
    int32_t *spos = reinterpret_cast<int32_t *>(smem + L.spos);
    uint16_t *wt_s = reinterpret_cast<uint16_t *>(smem + L.wt);
    uint16_t *swt = reinterpret_cast<uint16_t *>(smem + L.swt);
    uint16_t *sig_s = reinterpret_cast<uint16_t *>(smem + L.sig);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kMaxSlots;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + kMaxSlots);
    int *n_groups = reinterpret_cast<int *>(empty + kMaxSlots) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(&full[s], 1);
            sm100::mbar_init(&empty[s], kSub);
        }
        *abort = 0;
        sm100::fence_barrier_init();
    }
    // The shared expert's rows do not depend on the routing: this CTA's quads
    // of its gate/up rows enter the ring (slots 0..) and its slice of the down
    // rows goes to L2 while the routing kernels still run.
    const int A = gridDim.x, c = blockIdx.x;
    const bool sh = P.has_shared && P.src.sh_gate;
    const int sq0 = sh ? QPG * c / A : 0, nsq = sh ? QPG * (c + 1) / A - sq0 : 0;
    const int npre = min(nsq, S);  // issued before the wait (ring slots 0..npre-1, first use)
    __syncthreads();  // barriers initialised before the producer's first copy
    if (warp == kConsumerWarps && lane == 0) {
        for (int it = 0; it < npre; ++it) {
            const size_t r0 = static_cast<size_t>(sq0 + it) * kSub;
            uint8_t *dst = ring + it * L.slot_bytes;
            sm100::mbar_expect_tx(&full[it], 4 * kSub * H);
            sm100::bulk_load(dst, P.src.sh_gate + r0 * H, 2 * kSub * H, &full[it]);
            sm100::bulk_load(dst + 2 * kSub * H, P.src.sh_up + r0 * H, 2 * kSub * H, &full[it]);
        }
    }
    if (threadIdx.x == 64 && sh) prefetch_l2_slice(P.src.sh_down, static_cast<size_t>(H) * I * 2);
    grid_dependency_wait();  // the plan (or the router partials) come from the routing kernels
    grid_dependency_trigger();
    if (P.route) {
        fused_route<8>(P, grp, tok, pos_s, wt_s, sig_s, spos, n_groups);  // group table in place
    } else {
        if (blockIdx.x == 0 && threadIdx.x == 0) P.src.on_start();
        if (threadIdx.x == 32) *n_groups = P.src.n();
        for (int g = threadIdx.x; g < P.max_groups; g += blockDim.x) grp[g] = P.src.groups[g];
        __syncthreads();  // group table in place: the producer can start
    }

    // ---- work split (identical in every thread of every CTA): items 0..nsq-1
    // are the CTA's shared-expert quads (the shared group is the last group),
    // then its share of the routed groups' quads, then its down chunks
    const int n = min(*n_groups, P.max_groups);
    const int nr = n - (sh ? 1 : 0);  // routed groups
    constexpr int HW = H / kUnit;  // column units
    const int my_units = HW / A + (c < HW % A ? 1 : 0);
    const int64_t quads = static_cast<int64_t>(nr) * QPG;
    const int64_t qa0 = quads * c / A;
    const int nquads = nsq + static_cast<int>(quads * (c + 1) / A - qa0);
    // quad item it -> (group, first row)
    auto quad_of = [&](int it, int *g, int *r0) {
        if (it < nsq) {
            *g = n - 1;
            *r0 = (sq0 + it) * kSub;
        } else {
            const int64_t k = qa0 + (it - nsq);
            *g = static_cast<int>(k / QPG);
            *r0 = static_cast<int>(k % QPG) * kSub;
        }
    };
    const int nchunks = my_units * n;  // chunk ci: unit ci / n, group ci % n
    const int items = nquads + (nchunks + kSub - 1) / kSub;

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            int issued = npre;  // the first shared quads went out before the routing
            for (int it = npre; it < items; ++it) {
                const int s = it % S;
                if (it >= S && !fused_wait_bar(&empty[s], ((it / S) - 1) & 1, abort)) break;
                uint8_t *dst = ring + s * L.slot_bytes;
                if (it < nquads) {
                    int g, q0;
                    quad_of(it, &g, &q0);
                    const Group G = P.src.resolve(grp[g]);
                    const size_t r0 = static_cast<size_t>(q0);
                    sm100::mbar_expect_tx(&full[s], 4 * kSub * H);
                    sm100::bulk_load(dst, G.gate + r0 * H, 2 * kSub * H, &full[s]);
                    sm100::bulk_load(dst + 2 * kSub * H, G.up + r0 * H, 2 * kSub * H, &full[s]);
                } else {
                    const int ci0 = (it - nquads) * kSub, nc = min(kSub, nchunks - ci0);
                    sm100::mbar_expect_tx(&full[s], nc * 16 * I);
                    for (int jj = 0; jj < nc; ++jj) {
                        const int ci = ci0 + jj;
                        const Group G = P.src.resolve(grp[ci % n]);
                        const size_t u = c + (ci / n) * A;
                        sm100::bulk_load(dst + jj * 16 * I, G.down + u * kUnit * I, 16 * I, &full[s]);
                    }
                }
                issued = it + 1;
            }
            // Every copy this thread issued lands before the CTA leaves.
            for (int it = max(0, issued - S); it < issued; ++it) {
                const uint64_t t0 = fused_now();
                while (!sm100::mbar_try_wait(&full[it % S], (it / S) & 1) && fused_now() - t0 < kFusedWaitNs) {
                }
            }
        }
        return;
    }

    // ----------------------------------- consumers: token rows, route order
    if (!P.route) {
        for (int i = threadIdx.x; i < rows; i += kConsumers) tok[i] = P.src.route_token[i];
        for (int i = threadIdx.x; i < T * K; i += kConsumers) {
            const int p = P.route_pos[i];
            pos_s[i] = (p >= 0 && p < rows) ? p : -1;
            wt_s[i] = P.scores[i];
        }
        if (P.has_shared)
            for (int t = threadIdx.x; t < T; t += kConsumers) sig_s[t] = P.sig[t];
    }
    for (int i = threadIdx.x; i < T * HU; i += kConsumers) xs[i] = ld_cached(P.x + static_cast<size_t>(i) * 8);
    consumers_sync();
    // Each token's routes in ascending position (dropped ones last, ties in
    // slot order: the stable order of the standalone combine's sort).
    for (int i = threadIdx.x; i < T * K; i += kConsumers) {
        const int t = i / K, k = i % K;
        const unsigned me = static_cast<unsigned>(pos_s[i]);
        int rank = 0;
        for (int k2 = 0; k2 < K; ++k2) {
            const unsigned o = static_cast<unsigned>(pos_s[t * K + k2]);
            rank += (o < me || (o == me && k2 < k)) ? 1 : 0;
        }
        spos[t * K + rank] = pos_s[i];
        swt[t * K + rank] = wt_s[i];
    }
    const int wg = warp / kSub, j = warp % kSub;

    // ------------------------------------------------ phase A: gate/up quads
    int it = wg;
    for (; it < nquads; it += kGroups) {
        const int s = it % S;
        if (!fused_wait_bar(&full[s], (it / S) & 1, abort)) break;
        int g, q0;
        quad_of(it, &g, &q0);
        const GroupedGroup G = grp[g];
        const int r = q0 + j;
        const uint4 *gs = reinterpret_cast<const uint4 *>(ring + s * L.slot_bytes) + j * HU;
        const uint4 *us = gs + kSub * HU;
        for (int jj = 0; jj < G.count; ++jj) {
            const int t = min(max(tok[G.begin + jj], 0), T - 1);
            const uint4 *xr = xs + t * HU;
            float ag = 0.f, au = 0.f;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const uint4 a = xr[lane + 32 * i];
                ag = dot8(gs[lane + 32 * i], a, ag);
                au = dot8(us[lane + 32 * i], a, au);
            }
            ag = warp_sum(ag);
            au = warp_sum(au);
            if (lane == 0) {
                const float gv = rbf(ag), uv = rbf(au);
                const float sv = rbf(silu_f32(gv));
                P.act[static_cast<size_t>(G.begin + jj) * I + r] = f2bf(sv * uv);
            }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&empty[s]);
    }

    // ------------------------------- publish the activations, wait for all
    consumers_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&P.src.plan->act_ready, 1);
        if (!*abort) {
            const uint64_t t0 = fused_now();
            while (sm100::ld_acquire(&P.src.plan->act_ready) < A) {
                if (fused_now() - t0 > kFusedWaitNs) {
                    *abort = 1;
                    break;
                }
            }
        }
    }
    consumers_sync();
    if (!*abort) {
        const uint4 *act16 = reinterpret_cast<const uint4 *>(P.act);
        for (int i = threadIdx.x; i < rows * IU; i += kConsumers) acts[i] = __ldcg(act16 + i);
    }
    consumers_sync();

    // ------------------------------------------- phase B: down chunks -> ys
    if (!*abort) {
        for (; it < items; it += kGroups) {
            const int s = it % S;
            if (!fused_wait_bar(&full[s], (it / S) & 1, abort)) break;
            const int ci = (it - nquads) * kSub + j, ul = ci / n;
            const GroupedGroup G = grp[ci % n];
            const uint4 *ds = reinterpret_cast<const uint4 *>(ring + s * L.slot_bytes) + j * 8 * IU;
            for (int jj = 0; ci < nchunks && jj < G.count; ++jj) {
                const int row = G.begin + jj;
                uint4 a[NI];
#pragma unroll
                for (int i = 0; i < NI; ++i) a[i] = acts[row * IU + lane + 32 * i];
                float acc[8];
#pragma unroll
                for (int q8 = 0; q8 < 8; ++q8) {
                    acc[q8] = 0.f;
#pragma unroll
                    for (int i = 0; i < NI; ++i) acc[q8] = dot8(ds[q8 * IU + lane + 32 * i], a[i], acc[q8]);
                    acc[q8] = warp_sum(acc[q8]);
                }
                if (lane < 8) {
                    float v = acc[0];
#pragma unroll
                    for (int q8 = 1; q8 < 8; ++q8)
                        if (lane == q8) v = acc[q8];
                    ys[(ul * rows + row) * kUnit + lane] = f2bf(v);
                }
            }
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&empty[s]);
        }
    }
    consumers_sync();

    // ---------------------------- ordered combine of my columns, a unit a task
    if (!*abort) {
        for (int task = threadIdx.x; task < T * my_units; task += kConsumers) {
            const int t = task / my_units, ul = task % my_units;
            const uint4 *yu = reinterpret_cast<const uint4 *>(ys + ul * rows * kUnit);
            constexpr int kRowU = kUnit / 8;  // uint4 per ys row
            uint4 o = make_uint4(0, 0, 0, 0);
            for (int k = 0; k < K; ++k) {
                const int p = spos[t * K + k];
                if (p < 0) break;  // dropped routes sort last
                const uint4 v = yu[p * kRowU];
                const uint32_t w2 = bf16x2_splat(swt[t * K + k]);
                o.x = bf16x2_mul_add(o.x, v.x, w2);
                o.y = bf16x2_mul_add(o.y, v.y, w2);
                o.z = bf16x2_mul_add(o.z, v.z, w2);
                o.w = bf16x2_mul_add(o.w, v.w, w2);
            }
            if (P.has_shared) {
                const uint4 v = yu[(T * K + t) * kRowU];
                const uint32_t s2 = bf16x2_splat(sig_s[t]);
                o.x = bf16x2_mul_add(o.x, v.x, s2);
                o.y = bf16x2_mul_add(o.y, v.y, s2);
                o.z = bf16x2_mul_add(o.z, v.z, s2);
                o.w = bf16x2_mul_add(o.w, v.w, s2);
            }
            const int col = (c + ul * A) * kUnit;
            *reinterpret_cast<uint4 *>(P.out + static_cast<size_t>(t) * H + col) = o;
        }
    }
    if (threadIdx.x == 0 && *abort) atomicCAS(&P.src.plan->error, 0, 1);
}

template <int NW, int NI>
int launch_fused(const FusedParams &p, int smem, cudaStream_t stream) {
    if (int rc = ensure_dynamic_smem(fused_decode_kernel<NW, NI>, smem_optin(), "cudaFuncSetAttribute(fused_decode)"))
        return rc;
    return launch_pdl_cooperative(fused_decode_kernel<NW, NI>, dim3(sm_count()), dim3(kFusedThreads),
                                  static_cast<size_t>(smem), stream, "fused_decode_kernel", p);
}

template <int NW>
int launch_fused_i(const FusedParams &p, int inner, int smem, cudaStream_t stream) {
    switch (inner) {
        case 256: return launch_fused<NW, 1>(p, smem, stream);
        case 512: return launch_fused<NW, 2>(p, smem, stream);
        case 1024: return launch_fused<NW, 4>(p, smem, stream);
        default: return set_error(MOE_EINVAL, "fused decode: inner %d not in {256, 512, 1024}", inner);
    }
}

}  // namespace

bool fused_decode_fits(int tokens, int top_k, int hidden, int inner, int max_groups, bool shared) {
    if (tokens < 1 || tokens > kFusedDecodeMaxTokens || top_k < 1 || top_k > kFusedMaxTopK) return false;
    if ((hidden != 1024 && hidden != 2048 && hidden != 4096) || (inner != 256 && inner != 512 && inner != 1024))
        return false;
    const int A = sm_count();
    if (A <= 0) return false;
    const int rows = tokens * top_k + (shared ? tokens : 0);
    const int units_max = (hidden / kUnit + A - 1) / A;
    const FusedLayout L0 = fused_layout(0, tokens, hidden, inner, rows, max_groups, top_k, units_max);
    const int slots = std::min(kMaxSlots, (smem_optin() - L0.total) / L0.slot_bytes) / kGroups * kGroups;
    return slots >= 4;
}

int launch_fused_decode(const PlanGroups &src, int max_groups, const uint16_t *x, uint16_t *act,
                        const int32_t *route_pos, const uint16_t *scores, uint16_t *sig, uint16_t *out,
                        int tokens, int top_k, int hidden, int inner, cudaStream_t stream,
                        const FusedDecodeRoute *route) {
    if (!fused_decode_fits(tokens, top_k, hidden, inner, max_groups, sig != nullptr))
        return set_error(MOE_EINVAL, "fused decode: tokens %d / top_k %d / shape %dx%d out of range", tokens, top_k,
                         hidden, inner);
    if (route && (!route->part || route->experts < 1 || route->experts > 256 || tokens * top_k > 32 ||
                  !route->logits || !route->idx || !route->scores || !route->route_pos || !route->counters))
        return set_error(MOE_EINVAL, "fused decode: in-kernel routing needs partials and outputs, experts <= 256");
    FusedParams p{};
    if (route) {
        p.route = 1;
        p.experts = route->experts;
        p.part = route->part;
        p.bias = route->bias;
        p.logits_out = route->logits;
        p.idx_out = route->idx;
        p.scores_out = route->scores;
        p.route_pos_out = route->route_pos;
        p.counters = route->counters;
    }
    p.has_shared = sig != nullptr ? 1 : 0;
    p.src = src;
    p.x = x;
    p.act = act;
    p.route_pos = route_pos;
    p.scores = scores;
    p.sig = sig;
    p.out = out;
    p.tokens = tokens;
    p.top_k = top_k;
    p.rows = tokens * top_k + (sig ? tokens : 0);
    p.max_groups = max_groups;
    const int A = sm_count();
    p.units_max = (hidden / kUnit + A - 1) / A;
    const FusedLayout L0 = fused_layout(0, tokens, hidden, inner, p.rows, max_groups, top_k, p.units_max);
    // A multiple of the consumer groups: slot s then only ever holds the items of
    // group s % kGroups, which that group consumes in order, so no consumer
    // waits on a slot phase that another group has not consumed yet (a wait
    // two phases ahead would pass on the older phase of the same parity).
    p.slots = std::min(kMaxSlots, (smem_optin() - L0.total) / L0.slot_bytes) / kGroups * kGroups;
    const int smem = fused_layout(p.slots, tokens, hidden, inner, p.rows, max_groups, top_k, p.units_max).total;
    switch (hidden) {
        case 1024: return launch_fused_i<4>(p, inner, smem, stream);
        case 2048: return launch_fused_i<8>(p, inner, smem, stream);
        case 4096: return launch_fused_i<16>(p, inner, smem, stream);
        default: return set_error(MOE_EINVAL, "fused decode: hidden %d not in {1024, 2048, 4096}", hidden);
    }
}

}  // namespace lrb
