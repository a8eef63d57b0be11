// Grouped SwiGLU experts and the ordered combine on the 5th-generation tensor
// cores, in one persistent launch.
//
// For every active expert group g (routed experts in ascending id, then the
// shared expert) and its routes p:
//   phase 1  act[p, :] = bf16(bf16(silu(bf16(x_p . Wg))) * bf16(x_p . Wu))
//   phase 2  y[p, :]   = bf16(act_p . Wd)
// and for every token t (phase 3, the ordered combine):
//   out[t] = bf16(acc + bf16(sig_t * y[shared row t])) after
//   acc = bf16(acc + bf16(y_p * w_p)) over t's routes in ascending expert id
// (modeling_qwen3_5_moe.py:745-750, :788-790; edge35b/fused_experts.py:27-37).
// The weights are the M = 128 operand (rows of gate/up/down) and the group's
// routed tokens the N operand ("swap AB"), so decode widths (a handful of
// tokens per expert) and prefill widths (hundreds) share one tile shape.
//
// Work items, handed out in this order from a device counter (a launch may
// run phase 1 only, or phases 2-3 only after a phase-1 launch of the plan, so
// that other work can run between them):
//   phase 1  (group, 128-row block of gate and of up, token tile, K split)
//   phase 2  (group, 256-row block of down, token tile)
//   phase 3  (token, 1024-column half; decode widths only)
// Both matrix phases issue two M = 128 products per K step on one shared token
// tile (gate and up rows, or two halves of the down block), so every token
// tile loaded from L2 feeds 256 weight rows.
// A phase-2 item waits until its group's activations are published, a phase-3
// item until the outputs of all of its token's groups are; phase-1 items wait
// on nothing, so the queue cannot deadlock.  When few experts are active
// (small T) the K dimension of phase 1 is split so that every SM streams
// weights; the last split of a tile sums the FP32 partials in split order, so
// results do not depend on timing.
//
// Per CTA (256 threads, one CTA per SM): warp 0 issues TMA loads of 64-wide K
// slices (128B swizzle) into a ring of stages; warp 1 allocates TMEM and issues
// tcgen05.mma (M=128, N=BN, K=16) into a double-buffered FP32 accumulator;
// warps 2-5 read the accumulator with tcgen05.ld, write BF16 results and run
// the combine; warps 6-7 gather the token rows in address-table mode.  Every
// wait is bounded (globaltimer); on timeout the CTA raises the plan's error
// word, drains its own TMA and MMA work and returns.
//
// Address-table mode (src_rows / dst_rows, the expert-parallel step): row p
// of the plan is read from the 16-byte-aligned address src_rows[p] -- this
// GPU's memory or a peer's over NVLink -- and its down output is stored to
// dst_rows[p], again local or a peer's.  Warps 6-7 of every CTA copy the rows
// into the route-ordered buffer in plan order, two rows in flight per warp,
// and count each finished row into its group; a phase-1 item's token tiles
// wait only for its own group's rows, so the tensor cores start on the first
// groups while later rows are still crossing the links.  The caller's next
// kernel, once this grid is complete, releases the peers with a system-scope
// release, which orders the epilogue's stores into their memory before it.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include <climits>

#include "common.cuh"
#include "kernels.cuh"
#include "plan.cuh"
#include "sm100.cuh"

namespace lrb {

namespace {

constexpr int kBM = 128;                // weight rows per tile (MMA M)
constexpr int kBK = 64;                 // K per stage: one 128-byte swizzle atom of BF16
constexpr int kATile = kBM * kBK * 2;   // 16 KiB
constexpr int kThreads = 256;           // warps 0 TMA, 1 MMA, 2-5 epilogue, 6-7 row gather
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any legal wait
constexpr int kCombineCols = 1024;       // columns per phase-3 item (128 threads x 8)
constexpr int kSmemGroups = 257;         // plans up to this many groups are staged in shared memory

}  // namespace

// PAIR: a cluster of two CTAs works each item together (tcgen05.mma
// cta_group::2): each CTA holds 128 of the item's 256 weight rows of an M =
// 256 product and half of its token tile, so a token tile feeds 512 weight
// rows per load and every CTA reads fewer operand bytes per FLOP from shared
// memory, the limit of the single-CTA tile at prefill widths.
template <int BN, bool PAIR = false, bool TOKM = false>
struct GroupedShape {
    static constexpr int kBRows = PAIR ? BN / 2 : BN;  // token rows of a tile held by one CTA
    static constexpr int kBTile = kBRows * kBK * 2 < 1024 ? 1024 : kBRows * kBK * 2;
    static constexpr int kStage = 2 * kATile + kBTile;
    static constexpr int kStages = PAIR ? 5 : BN >= 256 ? 3 : BN >= 128 ? 4 : (BN >= 64 ? 5 : 6);
    // accumulator buffers of (gate, up): two, so the epilogue of one item
    // overlaps the products of the next, while they fit the 512 TMEM columns
    static constexpr int kBufs = 4 * BN <= 512 ? 2 : 1;
    static constexpr int kTmemCols = 2 * BN * kBufs < 32 ? 32 : 2 * BN * kBufs;
    static constexpr int kPlanBytes = 2 * (kSmemGroups + 1) * 4 + kSmemGroups * 16;
    // tokens-as-M in address-table mode: 4 KB per epilogue warp to turn its
    // 32 rows x 64 columns into 128-byte row segments for the stores into the
    // senders' memory
    static constexpr int kEpiBytes = TOKM ? 4 * 4096 : 0;
    static constexpr int kSmem = kStages * kStage + 1024 /*align*/ + 512 /*barriers*/ + kPlanBytes + kEpiBytes;
};

struct GroupedSmemTail {
    uint64_t full[8], empty[8], tfull[2], tempty[2], ifull[4], iempty[4], drain;
    int item[4];
    uint32_t tmem_base;
    int abort;
};

struct GroupedParams {
    const GroupedGroup *groups;
    GroupedPlan *plan;
    const int32_t *off1, *off2;   // [num_groups + 1] item prefixes of phases 1 and 2
    int32_t *done1, *done2;       // [num_groups] published epilogue-warp results
    int32_t *split_cnt;           // [phase-1 tiles * 4] arrivals of K splits
    float *part;                  // [phase-1 tiles, ks, 2, BN, 128] FP32 partials
    uint16_t *act, *y, *out;      // [rows, I], [rows, H], [T, H]
    const int32_t *route_pos;     // [T, K]
    const int64_t *idx;           // [T, K]
    const uint16_t *scores;       // [T, K] BF16
    const uint16_t *sig;          // [T] BF16 or null (no shared expert)
    const int32_t *group_of_expert;  // [E]
    const int32_t *route_token;      // [rows] route -> token
    uint16_t *rows_out;              // [T, H] per-token y rows instead of y (top_k 1), or null
    const int32_t *stage_error;      // host-staging error word, or null
    const uint16_t *x;               // gather_x: token rows [T, H]
    const uint16_t *sh_gate, *sh_up, *sh_down;  // shared expert rows (null: none), prefetched to L2 at start
    uint16_t *xs;                    // gather_x: route-ordered rows the kernel fills
    int gather_x, gather_need;       // gather in the kernel; epilogue warps that must publish it
    const int64_t *src_rows;         // address-table mode: row p is read from src_rows[p] (or null)
    const int64_t *dst_rows;         // and its down output stored to dst_rows[p]
    int32_t *row_ready;              // [num_groups] rows gathered per group (address-table mode)
    int32_t *error_out;              // or null: set to 3 when a wait of this kernel gave up
    int tokens, top_k, hidden, inner, ks;
    int phases;                      // 3 all items, 1 phase 1 only, 2 phases 2-3 only
};

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t i = 1;; ++i) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if ((i & 63) == 0 && now_ns() - t0 > kWaitNs) {
            *abort = 1;
            return false;
        }
    }
}

// wait_bar with cluster-scope acquire (barriers other CTAs of the pair arrive on
// after writing this CTA's shared memory).
__device__ __forceinline__ bool wait_bar_cluster(uint64_t *bar, uint32_t parity, volatile int *abort) {
    if (sm100::mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t i = 1;; ++i) {
        if (sm100::mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort) return false;
        if ((i & 63) == 0 && now_ns() - t0 > kWaitNs) {
            *abort = 1;
            return false;
        }
    }
}

// Bounded wait until *counter >= need (acquire).  false on timeout/abort.
__device__ __forceinline__ bool wait_count(const int32_t *counter, int need, volatile int *abort) {
    if (sm100::ld_acquire(counter) >= need) return true;
    const uint64_t t0 = now_ns();
    while (sm100::ld_acquire(counter) < need) {
        if (*abort || now_ns() - t0 > kWaitNs) return false;
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ int find_group(const int32_t *off, int n, int item) {
    int lo = 0, hi = n;  // largest g with off[g] <= item
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off[mid] <= item) lo = mid;
        else hi = mid;
    }
    return lo;
}

struct ItemPos {
    int phase, g, mb, nt, ks, tile;  // tile: phase-1 tile index (for split partials)
};

// off1/off2/groups point at the shared-memory copy of the plan (or at the
// global one when it is too large to stage).
struct PlanView {
    const int32_t *off1, *off2;
    const GroupedGroup *groups;
};

__device__ __forceinline__ ItemPos decode_item(const GroupedParams &P, const PlanView &V, int n_groups, int items1,
                                               int items2, int item, int mb1, int mb2) {
    ItemPos r{};
    if (item < items1) {
        r.phase = 1;
        r.g = find_group(V.off1, n_groups, item);
        const int local = item - V.off1[r.g];
        r.ks = local % P.ks;
        const int rest = local / P.ks;
        r.mb = rest % mb1;
        r.nt = rest / mb1;
        r.tile = V.off1[r.g] / P.ks + rest;
    } else if (item < items1 + items2) {
        const int j = item - items1;
        r.phase = 2;
        r.g = find_group(V.off2, n_groups, j);
        const int local = j - V.off2[r.g];
        r.mb = local % mb2;
        r.nt = local / mb2;
    } else {
        r.phase = 3;
        r.g = item - items1 - items2;  // token * halves + half
    }
    return r;
}

// The ordered combine of 8 columns [c, c + 8) of token t (phase 3): the sum
// over the token's routes in ascending route position of bf16(y[pos] * w),
// rounded to BF16 after every add, then + bf16(sig[t] * shared row).  KMAX >=
// top_k fixes every index at compile time, so the routes live in registers
// and every load of a stage is in flight at once.  The route positions and
// weights are read before waiting for `done` to reach `need` (lane 0 polls,
// bounded).  Out of line on purpose: the epilogue warps run it once at kernel
// start on token 0 with store = false, so its code is cached when the real
// combine runs after the weight stream.  Returns false when the wait gave up.
template <int KMAX>
__device__ __noinline__ bool combine_cols(const int32_t *__restrict__ route_pos, const uint16_t *__restrict__ scores,
                                          const uint16_t *y, const uint16_t *__restrict__ sig, uint16_t *out,
                                          int hidden, int top_k, int shared_row, int t, int c, const int32_t *done,
                                          int need, volatile int *abort, bool store) {
    const int lane = threadIdx.x & 31;
    int pos[KMAX];
    uint16_t wb[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        pos[k] = INT_MAX;  // past top_k: sorts last, never summed
        wb[k] = 0;
        if (k < top_k) {
            const size_t o = static_cast<size_t>(t) * top_k + k;
            pos[k] = route_pos[o];
            wb[k] = scores[o];
        }
    }
    bool ok = true;
    if (lane == 0) ok = wait_count(done, need, abort);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) return false;
    __threadfence();
    // ascending route position (insertion sort without early exit: a pair
    // already in order is never swapped)
#pragma unroll
    for (int a = 1; a < KMAX; ++a) {
#pragma unroll
        for (int b = a; b > 0; --b) {
            if (pos[b] < pos[b - 1]) {
                const int tp = pos[b];
                pos[b] = pos[b - 1];
                pos[b - 1] = tp;
                const uint16_t tw = wb[b];
                wb[b] = wb[b - 1];
                wb[b - 1] = tw;
            }
        }
    }
    uint4 shv = make_uint4(0, 0, 0, 0);
    if (sig) shv = __ldcg(reinterpret_cast<const uint4 *>(y + static_cast<size_t>(shared_row) * hidden + c));
    // packed BF16 pairs: acc = bf16(acc + bf16(v * w)) per route, ascending position
    uint4 o = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k0 = 0; k0 < KMAX; k0 += 8) {
        if (k0 >= top_k) break;
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = k0 + j;
            v[j] = make_uint4(0, 0, 0, 0);
            if (pos[k] >= 0 && pos[k] != INT_MAX)
                v[j] = __ldcg(reinterpret_cast<const uint4 *>(y + static_cast<size_t>(pos[k]) * hidden + c));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = k0 + j;
            if (pos[k] < 0 || pos[k] == INT_MAX) continue;
            const uint32_t w2 = bf16x2_splat(wb[k]);
            o.x = bf16x2_mul_add(o.x, v[j].x, w2);
            o.y = bf16x2_mul_add(o.y, v[j].y, w2);
            o.z = bf16x2_mul_add(o.z, v[j].z, w2);
            o.w = bf16x2_mul_add(o.w, v[j].w, w2);
        }
    }
    if (sig) {
        const uint32_t s2 = bf16x2_splat(sig[t]);
        o.x = bf16x2_mul_add(o.x, shv.x, s2);
        o.y = bf16x2_mul_add(o.y, shv.y, s2);
        o.z = bf16x2_mul_add(o.z, shv.z, s2);
        o.w = bf16x2_mul_add(o.w, shv.w, s2);
    }
    if (store) *reinterpret_cast<uint4 *>(out + static_cast<size_t>(t) * hidden + c) = o;
    return true;
}

// combine_cols at the smallest KMAX that holds top_k (<= 32).
__device__ __forceinline__ bool combine_cols_k(const int32_t *route_pos, const uint16_t *scores, const uint16_t *y,
                                               const uint16_t *sig, uint16_t *out, int hidden, int top_k,
                                               int shared_row, int t, int c, const int32_t *done, int need,
                                               volatile int *abort, bool store) {
    if (top_k <= 8)
        return combine_cols<8>(route_pos, scores, y, sig, out, hidden, top_k, shared_row, t, c, done, need, abort,
                               store);
    if (top_k <= 16)
        return combine_cols<16>(route_pos, scores, y, sig, out, hidden, top_k, shared_row, t, c, done, need, abort,
                                store);
    return combine_cols<32>(route_pos, scores, y, sig, out, hidden, top_k, shared_row, t, c, done, need, abort,
                            store);
}

// TOKM (128-token tiles, single CTA): the token tile is the M = 128 operand
// and the item's 256 weight rows one N = 256 operand (gate rows then up rows,
// or the two halves of the down block, which lie back to back in the stage),
// one product per K step.  The accumulator row of a lane is then one token:
// the gate and up values of a column sit in the same thread, and each thread
// stores its token's outputs as contiguous 16-byte vectors instead of one
// BF16 per token column; the token tile is also read once per K step instead
// of twice.  Same tiles, items and stage contents as the swapped layout.
template <int BN, bool PAIR, bool TOKM>
__global__ void __launch_bounds__(kThreads, 1)
    swiglu_grouped_kernel(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dn,
                          const __grid_constant__ CUtensorMap tm_sg, const __grid_constant__ CUtensorMap tm_su,
                          const __grid_constant__ CUtensorMap tm_sd, const __grid_constant__ CUtensorMap tm_x,
                          const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_x16,
                          const __grid_constant__ CUtensorMap tm_act16, const GroupedParams P) {
    static_assert(!TOKM || (BN == 128 && !PAIR), "tokens-as-M runs single CTAs on 128-token tiles");
    using S = GroupedShape<BN, PAIR, TOKM>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    GroupedSmemTail *tail = reinterpret_cast<GroupedSmemTail *>(smem + S::kStages * S::kStage);
    volatile int *abort = &tail->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // paired mode: this CTA's rank in its pair; rank 0 fetches the items and
    // issues the products of both
    const int cta = PAIR ? static_cast<int>(sm100::cluster_ctarank()) : 0;
    const bool leader = cta == 0;

    // Prologue (overlaps the previous kernel under programmatic launch).
    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            sm100::mbar_init(&tail->full[s], 1);
            sm100::mbar_init(&tail->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(&tail->tfull[b], 1);
            sm100::mbar_init(&tail->tempty[b], PAIR ? 8 : 4);  // the epilogue warps of the pair
        }
        for (int i = 0; i < 4; ++i) {
            sm100::mbar_init(&tail->ifull[i], 1);
            // MMA + 4 epilogue warps; paired: the peer's producer and epilogue too
            sm100::mbar_init(&tail->iempty[i], PAIR ? 10 : 5);
        }
        sm100::mbar_init(&tail->drain, 1);
        tail->abort = 0;
        sm100::fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        sm100::tma_prefetch_map(&tm_gu);
        sm100::tma_prefetch_map(&tm_dn);
        sm100::tma_prefetch_map(&tm_sg);
        sm100::tma_prefetch_map(&tm_su);
        sm100::tma_prefetch_map(&tm_sd);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            sm100::tmem_alloc_pair(&tail->tmem_base, S::kTmemCols);
            sm100::tmem_relinquish_pair();
        } else {
            sm100::tmem_alloc(&tail->tmem_base, S::kTmemCols);
            sm100::tmem_relinquish();
        }
    }
    // The shared expert's rows do not depend on the routing: this CTA's slice
    // of them goes to L2 while the routing kernels still run.
    if (threadIdx.x == 64 && P.sh_gate) {
        prefetch_l2_slice(P.sh_gate, static_cast<size_t>(P.inner) * P.hidden * 2);
        prefetch_l2_slice(P.sh_up, static_cast<size_t>(P.inner) * P.hidden * 2);
        prefetch_l2_slice(P.sh_down, static_cast<size_t>(P.hidden) * P.inner * 2);
    }
    sm100::tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) sm100::cluster_sync();  // the peer's barriers exist before any remote arrive
    sm100::tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    grid_dependency_wait();  // routing and token gather are complete from here on
    grid_dependency_trigger();
    if (blockIdx.x == 0 && threadIdx.x == 0 && P.stage_error) {
        const int e = *P.stage_error;
        if (e) atomicCAS(&P.plan->error, 0, e);
    }

    const int n_groups = P.plan->num_groups;
    const int items1 = P.plan->items1, items2 = P.plan->items2;
    const int total = items1 + items2 + P.plan->items3;
    // weight rows per item: phase 1 kBM of gate and of up (2 kBM paired),
    // phase 2 2 kBM of down (4 kBM paired)
    const int mb1 = P.inner / (PAIR ? 2 * kBM : kBM), mb2 = P.hidden / (PAIR ? 4 * kBM : 2 * kBM);
    // Stage the plan in shared memory: every item decode then costs a few
    // shared loads instead of a chain of dependent global ones.
    PlanView V{P.off1, P.off2, P.groups};
    if (n_groups <= kSmemGroups) {
        int32_t *s_off1 = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(tail) + 512);
        int32_t *s_off2 = s_off1 + kSmemGroups + 1;
        GroupedGroup *s_groups = reinterpret_cast<GroupedGroup *>(s_off2 + kSmemGroups + 1);
        for (int i = threadIdx.x; i <= n_groups; i += blockDim.x) {
            s_off1[i] = P.off1[i];
            s_off2[i] = P.off2[i];
            if (i < n_groups) s_groups[i] = P.groups[i];
        }
        V = PlanView{s_off1, s_off2, s_groups};
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            // weights are read once per step: evict them first, so the
            // activations, plan and code stay in L2 under the stream
            const uint64_t wpol = sm100::l2_evict_first_policy(), npol = sm100::l2_evict_normal_policy();
            bool xs_seen = false;  // the in-kernel gather was observed complete
            uint32_t stage = 0, sphase = 0;
            uint32_t issued_parity[8];
            bool issued[8] = {false, false, false, false, false, false, false, false};
            // the items of this launch: [lo, hi), fetched from their own counter
            const int lo = P.phases == 2 ? items1 : 0, hi = P.phases == 1 ? items1 : total;
            int32_t *ctr = P.phases == 2 ? &P.plan->work2 : &P.plan->work;
            int next = leader ? lo + atomicAdd(ctr, 1) : 0;
            for (int it = 0;; ++it) {
                const int slot = it & 3;
                int item;
                if (PAIR && !leader) {
                    // the leader hands this CTA the pair's item
                    if (!wait_bar_cluster(&tail->ifull[slot], (it >> 2) & 1, abort)) break;
                    item = tail->item[slot];
                    sm100::mbar_arrive_cluster(sm100::mapa(&tail->iempty[slot], 0));
                } else {
                    item = next;
                    if (item >= hi) item = -1;
                    else next = lo + atomicAdd(ctr, 1);  // in flight while this item streams
                    if (PAIR ? !wait_bar_cluster(&tail->iempty[slot], ((it >> 2) & 1) ^ 1, abort)
                             : !wait_bar(&tail->iempty[slot], ((it >> 2) & 1) ^ 1, abort))
                        break;
                    tail->item[slot] = item;
                    if constexpr (PAIR) {
                        sm100::st_cluster_u32(sm100::mapa(&tail->item[slot], 1), static_cast<uint32_t>(item));
                        sm100::mbar_arrive_cluster(sm100::mapa(&tail->ifull[slot], 1));
                    }
                    sm100::mbar_arrive(&tail->ifull[slot]);
                }
                if (item < 0) break;
                const ItemPos ip = decode_item(P, V, n_groups, items1, items2, item, mb1, mb2);
                if (ip.phase == 3) continue;  // combine: no operand loads
                const GroupedGroup G = V.groups[ip.g];
                const int kspan = (ip.phase == 1 ? P.hidden / P.ks : P.inner) / kBK;
                const int kb0 = ip.phase == 1 ? ip.ks * kspan : 0;
                // this CTA's first weight row (paired: its 128 of the item's 256)
                const int row0 = PAIR ? ip.mb * (ip.phase == 1 ? 2 * kBM : 4 * kBM) + cta * kBM
                                      : ip.mb * (ip.phase == 1 ? kBM : 2 * kBM);
                // a group of one token tile reads each weight tile once: evict it
                // first; with several tiles the later ones re-read it from L2
                const uint64_t ipol = G.ntiles == 1 ? wpol : npol;
                // Token tiles are loaded (and multiplied) only as wide as their
                // rows, rounded up to 16 (32 paired, each CTA holding half): a
                // full tile in one box, a partial one in boxes of 16 rows.
                const int nmma = PAIR ? (min(BN, G.count - ip.nt * BN) + 31) & ~31
                                      : (min(BN, G.count - ip.nt * BN) + 15) & ~15;
                const int nb = PAIR ? nmma / 2 : nmma;  // token rows this CTA loads
                const int tok0 = G.begin + ip.nt * BN + cta * nb;
                const uint32_t bytes = (PAIR ? 2 : 1) * (2 * kATile + nb * kBK * 2);  // on the leader's barrier
                auto load_b = [&](const CUtensorMap *full_map, const CUtensorMap *map16, uint8_t *dst, uint64_t *bar,
                                  int k0) {
                    if constexpr (PAIR) {
                        const uint32_t lb = sm100::mapa(bar, 0);
                        if (nb == S::kBRows) {
                            sm100::tma_load_2d_pair(dst, full_map, lb, k0, tok0, npol);
                        } else {
                            for (int r = 0; r < nb; r += 16)
                                sm100::tma_load_2d_pair(dst + r * kBK * 2, map16, lb, k0, tok0 + r, npol);
                        }
                    } else if (nb == BN) {
                        sm100::tma_load_2d(dst, full_map, bar, k0, tok0);
                    } else {
                        for (int r = 0; r < nb; r += 16) sm100::tma_load_2d(dst + r * kBK * 2, map16, bar, k0, tok0 + r);
                    }
                };
                // weight tiles: a bank expert (3-D map) or the shared expert
                // (2-D); every call names its map, so each TMA instruction reads
                // a fixed kernel-parameter descriptor
                auto load_w3 = [&](uint8_t *dst, const CUtensorMap *map, uint64_t *bar, int k0, int r, int e) {
                    if constexpr (PAIR) sm100::tma_load_3d_pair(dst, map, sm100::mapa(bar, 0), k0, r, e, ipol);
                    else sm100::tma_load_3d_hint(dst, map, bar, k0, r, e, ipol);
                };
                auto load_w2 = [&](uint8_t *dst, const CUtensorMap *map, uint64_t *bar, int k0, int r) {
                    if constexpr (PAIR) sm100::tma_load_2d_pair(dst, map, sm100::mapa(bar, 0), k0, r, ipol);
                    else sm100::tma_load_2d_hint(dst, map, bar, k0, r, ipol);
                };
                // Weight tiles stream right away; activation tiles wait for their
                // producers: phase 2 for the group's phase 1 (every phase-1 tile
                // once per epilogue warp), phase 1 for the in-kernel gather.
                const bool p1 = ip.phase == 1;
                const bool tables = P.src_rows != nullptr;
                bool dep_ok = p1 ? (!tables && (xs_seen || !P.gather_x)) : false;
                const int32_t *dep_ctr = p1 ? (tables ? &P.row_ready[ip.g] : &P.plan->xs_ready) : &P.done1[ip.g];
                // phase 2 waits for every epilogue warp of the group's phase-1 items
                const int need = p1 ? (tables ? G.count : P.gather_need) : (PAIR ? 8 : 4) * mb1 * G.ntiles;
                const CUtensorMap *bmap = p1 ? &tm_x : &tm_act, *bmap16 = p1 ? &tm_x16 : &tm_act16;
                int pending[8];
                int n_pending = 0;
                bool ok = true;
                for (int kb = kb0; kb < kb0 + kspan; ++kb) {
                    if (!dep_ok && n_pending > 0 && !sm100::mbar_try_wait(&tail->empty[stage], sphase ^ 1)) {
                        // out of free stages: the earlier stages need their activation tiles
                        if (!wait_count(dep_ctr, need, abort)) {
                            *abort = 1;
                            atomicExch(&P.plan->error, 2);
                            ok = false;
                            break;
                        }
                        sm100::fence_proxy_async_global();
                        dep_ok = true;
                        for (int j = 0; j < n_pending; ++j) {
                            const int ps = pending[j] & 0xff, pk = pending[j] >> 8;
                            load_b(bmap, bmap16, smem + ps * S::kStage + 2 * kATile, &tail->full[ps], pk * kBK);
                        }
                        n_pending = 0;
                    }
                    if (!wait_bar(&tail->empty[stage], sphase ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + stage * S::kStage;
                    uint64_t *fb = &tail->full[stage];
                    if (leader) sm100::mbar_expect_tx(fb, bytes);
                    const int k0 = kb * kBK;
                    // the second down block starts kBM rows on (2 kBM paired: the
                    // other M = 256 product)
                    const int row1 = row0 + (PAIR ? 2 * kBM : kBM);
                    if (ip.phase == 1) {
                        if (G.weight >= 0) {
                            load_w3(st, &tm_gu, fb, k0, row0, G.weight);
                            load_w3(st + kATile, &tm_gu, fb, k0, P.inner + row0, G.weight);
                        } else {
                            load_w2(st, &tm_sg, fb, k0, row0);
                            load_w2(st + kATile, &tm_su, fb, k0, row0);
                        }
                    } else {
                        if (G.weight >= 0) {
                            load_w3(st, &tm_dn, fb, k0, row0, G.weight);
                            load_w3(st + kATile, &tm_dn, fb, k0, row1, G.weight);
                        } else {
                            load_w2(st, &tm_sd, fb, k0, row0);
                            load_w2(st + kATile, &tm_sd, fb, k0, row1);
                        }
                    }
                    if (!dep_ok && sm100::ld_acquire(dep_ctr) >= need) {
                        sm100::fence_proxy_async_global();
                        dep_ok = true;
                        for (int j = 0; j < n_pending; ++j) {
                            const int ps = pending[j] & 0xff, pk = pending[j] >> 8;
                            load_b(bmap, bmap16, smem + ps * S::kStage + 2 * kATile, &tail->full[ps], pk * kBK);
                        }
                        n_pending = 0;
                    }
                    if (dep_ok) load_b(bmap, bmap16, st + 2 * kATile, fb, k0);
                    else pending[n_pending++] = stage | (kb << 8);
                    issued[stage] = true;
                    issued_parity[stage] = sphase;
                    if (++stage == S::kStages) {
                        stage = 0;
                        sphase ^= 1;
                    }
                }
                if (ok && n_pending > 0) {
                    if (!wait_count(dep_ctr, need, abort)) {
                        *abort = 1;
                        atomicExch(&P.plan->error, 2);
                        ok = false;
                    } else {
                        sm100::fence_proxy_async_global();
                        dep_ok = true;
                        for (int j = 0; j < n_pending; ++j) {
                            const int ps = pending[j] & 0xff, pk = pending[j] >> 8;
                            load_b(bmap, bmap16, smem + ps * S::kStage + 2 * kATile, &tail->full[ps], pk * kBK);
                        }
                        n_pending = 0;
                    }
                }
                if (p1 && dep_ok && !tables) xs_seen = true;
                if (!ok) break;
            }
            if (PAIR && *abort) {
                // A pair's loads complete on the leader's barriers, which the
                // peer cannot watch: give every load in flight a bounded time
                // to land (far above any load latency) before the CTA leaves.
                const uint64_t t0 = now_ns();
                while (now_ns() - t0 < 200000) __nanosleep(1000);
            } else if (*abort) {
                // Let every load this thread issued land before the CTA leaves.
                for (int s = 0; s < S::kStages; ++s) {
                    if (!issued[s]) continue;
                    const uint64_t t0 = now_ns();
                    while (!sm100::mbar_try_wait(&tail->full[s], issued_parity[s]) && now_ns() - t0 < kWaitNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------- MMA issuer
        // (paired: the leader's, for both CTAs)
        if (lane == 0 && leader) {
            uint32_t stage = 0, sphase = 0;
            int acc = 0;
            bool any = false;
            for (int it = 0;; ++it) {
                const int slot = it & 3;
                if (!wait_bar(&tail->ifull[slot], (it >> 2) & 1, abort)) break;
                const int item = tail->item[slot];
                sm100::mbar_arrive(&tail->iempty[slot]);
                if (item < 0) break;
                const ItemPos ip = decode_item(P, V, n_groups, items1, items2, item, mb1, mb2);
                if (ip.phase == 3) continue;
                const int kspan = (ip.phase == 1 ? P.hidden / P.ks : P.inner) / kBK;
                const GroupedGroup G = V.groups[ip.g];
                const int nmma = PAIR ? (min(BN, G.count - ip.nt * BN) + 31) & ~31
                                      : (min(BN, G.count - ip.nt * BN) + 15) & ~15;
                // TOKM: M = 128 token rows (a partial tile's stale rows give
                // accumulator rows nobody reads), N = 256 weight rows
                const uint32_t idesc = TOKM ? sm100::idesc_bf16_f32(kBM, 2 * kBM)
                                            : sm100::idesc_bf16_f32(PAIR ? 2 * kBM : kBM, nmma);
                const int buf = acc % S::kBufs;
                if (PAIR ? !wait_bar_cluster(&tail->tempty[buf], ((acc / S::kBufs) & 1) ^ 1, abort)
                         : !wait_bar(&tail->tempty[buf], ((acc / S::kBufs) & 1) ^ 1, abort))
                    break;
                sm100::tc_fence_after();
                const uint32_t d_gate = tmem + buf * 2 * BN, d_up = d_gate + BN;
                bool ok = true;
                for (int kb = 0; kb < kspan; ++kb) {
                    if (!wait_bar(&tail->full[stage], sphase, abort)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    const uint32_t base = sm100::smem_u32(smem + stage * S::kStage);
                    const uint64_t a0 = sm100::desc_kmajor_sw128(base);
                    const uint64_t a1 = sm100::desc_kmajor_sw128(base + kATile);
                    const uint64_t b = sm100::desc_kmajor_sw128(base + 2 * kATile);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t accumulate = (kb | kk) != 0;
                        if constexpr (TOKM) {
                            sm100::mma_bf16(d_gate, b + 2 * kk, a0 + 2 * kk, idesc, accumulate);
                        } else if constexpr (PAIR) {
                            sm100::mma_bf16_pair(d_gate, a0 + 2 * kk, b + 2 * kk, idesc, accumulate);
                            sm100::mma_bf16_pair(d_up, a1 + 2 * kk, b + 2 * kk, idesc, accumulate);
                        } else {
                            sm100::mma_bf16(d_gate, a0 + 2 * kk, b + 2 * kk, idesc, accumulate);
                            sm100::mma_bf16(d_up, a1 + 2 * kk, b + 2 * kk, idesc, accumulate);
                        }
                    }
                    // the stage is free in both CTAs once these products are done
                    if constexpr (PAIR) sm100::mma_commit_pair(&tail->empty[stage], 3);
                    else sm100::mma_commit(&tail->empty[stage]);
                    any = true;
                    if (++stage == S::kStages) {
                        stage = 0;
                        sphase ^= 1;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) sm100::mma_commit_pair(&tail->tfull[buf], 3);
                else sm100::mma_commit(&tail->tfull[buf]);
                ++acc;
            }
            if (*abort && any) {
                // Wait for this thread's MMAs before TMEM is released.
                if constexpr (PAIR) sm100::mma_commit_pair(&tail->drain, 1);
                else sm100::mma_commit(&tail->drain);
                const uint64_t t0 = now_ns();
                while (!sm100::mbar_try_wait(&tail->drain, 0) && now_ns() - t0 < kWaitNs) {
                }
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------- epilogue + combine
        const int q = warp & 3;           // TMEM lane quadrant this warp may read
        const int et = threadIdx.x - 64;  // 0..127
        int acc = 0;
        // an accumulator buffer is free again (paired: on the leader, which
        // issues the next products into both CTAs' TMEM)
        auto release_acc = [&](uint64_t *bar) {
            if constexpr (PAIR) sm100::mbar_arrive_cluster(sm100::mapa(bar, 0));
            else sm100::mbar_arrive(bar);
        };
        if (P.gather_x) {
            // The token gather of the routed and shared rows (xs[p] = x[token
            // of route p]), spread over every CTA's epilogue warps while the
            // producers start the weight stream; phase-1 activation loads wait
            // for all of them to publish.
            const int shared = V.groups[n_groups - 1].weight < 0 ? 1 : 0;
            const int nr = n_groups - shared;
            const int placed = nr > 0 ? V.groups[nr - 1].begin + V.groups[nr - 1].count : 0;
            const int routes = P.tokens * P.top_k, units = P.hidden / 8;
            const int64_t total_units = static_cast<int64_t>(placed + (shared ? P.tokens : 0)) * units;
            for (int64_t i = static_cast<int64_t>(blockIdx.x) * 128 + et; i < total_units;
                 i += static_cast<int64_t>(gridDim.x) * 128) {
                const int qr = static_cast<int>(i / units), cu = static_cast<int>(i % units);
                const int p = qr < placed ? qr : routes + (qr - placed);
                const int tk = p < routes ? P.route_token[p] : p - routes;
                reinterpret_cast<uint4 *>(P.xs)[static_cast<int64_t>(p) * units + cu] =
                    ld_cached(P.x + static_cast<size_t>(tk) * P.hidden + cu * 8);
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                sm100::fence_proxy_async_global();
                atomicAdd(&P.plan->xs_ready, 1);
            }
        }
        if (P.plan->items3 > 0)  // warm the combine's code: token 0, nothing stored, no wait
            combine_cols_k(P.route_pos, P.scores, P.y, P.sig, P.out, P.hidden, P.top_k,
                           P.sig ? V.groups[n_groups - 1].begin : 0, 0, et * 8, &P.plan->done2_total, 0, abort, false);
        for (int it = 0;; ++it) {
            const int slot = it & 3;
            if (PAIR ? !wait_bar_cluster(&tail->ifull[slot], (it >> 2) & 1, abort)
                     : !wait_bar(&tail->ifull[slot], (it >> 2) & 1, abort))
                break;
            const int item = tail->item[slot];
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) sm100::mbar_arrive_cluster(sm100::mapa(&tail->iempty[slot], 0));
                else sm100::mbar_arrive(&tail->iempty[slot]);
            }
            if (item < 0) break;
            const ItemPos ip = decode_item(P, V, n_groups, items1, items2, item, mb1, mb2);

            if ((PAIR || TOKM) && (ip.phase == 3 || P.ks > 1)) {  // never planned so (host check)
                *abort = 1;
                break;
            }
            if (ip.phase == 3) {
                const int halves = P.hidden / kCombineCols;
                const int t = ip.g / halves, c = (ip.g % halves) * kCombineCols + et * 8;
                const int shared_row = P.sig ? V.groups[n_groups - 1].begin + t : 0;
                // every route row and shared row exists once all phase-2 items
                // (4 epilogue warps each) have published
                if (!combine_cols_k(P.route_pos, P.scores, P.y, P.sig, P.out, P.hidden, P.top_k, shared_row, t, c,
                                    &P.plan->done2_total, 4 * items2, abort, true)) {
                    *abort = 1;
                    atomicExch(&P.plan->error, 3);
                    break;
                }
                continue;
            }

            const GroupedGroup G = V.groups[ip.g];
            const int buf = acc % S::kBufs;
            if (!wait_bar(&tail->tfull[buf], (acc / S::kBufs) & 1, abort)) break;
            __syncwarp();
            sm100::tc_fence_after();
            const int row = (PAIR ? ip.mb * (ip.phase == 1 ? 2 * kBM : 4 * kBM) + cta * kBM
                                  : ip.mb * (ip.phase == 1 ? kBM : 2 * kBM)) +
                            q * 32 + lane;
            const int p0 = G.begin + ip.nt * BN;
            const int nvalid = min(BN, G.count - ip.nt * BN);
            const uint32_t t_gate = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 2 * BN;
            if constexpr (TOKM) {
                // lane = token p0 + q * 32 + lane of the tile; columns = the
                // item's 256 weight rows
                const int tk = q * 32 + lane;
                const bool valid = tk < nvalid;
                if (q * 32 < nvalid) {  // warp-uniform: a warp with no token of the tile reads nothing
                    if (ip.phase == 1) {
                        uint16_t *dst = P.act + static_cast<size_t>(p0 + tk) * P.inner + ip.mb * kBM;
#pragma unroll 1
                        for (int c0 = 0; c0 < kBM; c0 += 16) {
                            float g[16], u[16];
                            __syncwarp();
                            sm100::tmem_ld16(t_gate + c0, g);
                            sm100::tmem_ld16(t_gate + kBM + c0, u);
                            sm100::tmem_wait_ld();
                            uint32_t pk[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float a0v = rbf(silu_f32(rbf(g[2 * j]))) * rbf(u[2 * j]);
                                const float a1v = rbf(silu_f32(rbf(g[2 * j + 1]))) * rbf(u[2 * j + 1]);
                                pk[j] = static_cast<uint32_t>(f2bf(a0v)) | (static_cast<uint32_t>(f2bf(a1v)) << 16);
                            }
                            if (valid) {
                                uint4 *o = reinterpret_cast<uint4 *>(dst + c0);
                                o[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                                o[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                            }
                        }
                    } else if (P.dst_rows) {
                        // address tables: the rows go to the senders' memory
                        // over NVLink; 64 columns of the warp's 32 rows pass
                        // through shared memory so that eight lanes store one
                        // row's 128 contiguous bytes (one lane per row would
                        // send 32 separate 16-byte pieces per instruction)
                        uint8_t *stg = smem + S::kStages * S::kStage + 512 + S::kPlanBytes + (warp - 2) * 4096;
                        const int64_t mine = valid ? P.dst_rows[p0 + tk] : 0;
#pragma unroll 1
                        for (int c0 = 0; c0 < 2 * kBM; c0 += 64) {
#pragma unroll
                            for (int sub = 0; sub < 4; ++sub) {
                                float v[16];
                                __syncwarp();
                                sm100::tmem_ld16(t_gate + c0 + sub * 16, v);
                                sm100::tmem_wait_ld();
                                uint32_t pk[8];
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    pk[j] = static_cast<uint32_t>(f2bf(v[2 * j])) |
                                            (static_cast<uint32_t>(f2bf(v[2 * j + 1])) << 16);
                                // piece p of row r at slot p ^ (r & 7): the lanes'
                                // writes spread over the banks
                                uint8_t *row = stg + lane * 128;
                                const int p0s = 2 * sub, sw = lane & 7;
                                *reinterpret_cast<uint4 *>(row + ((p0s ^ sw) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                                *reinterpret_cast<uint4 *>(row + (((p0s + 1) ^ sw) << 4)) =
                                    make_uint4(pk[4], pk[5], pk[6], pk[7]);
                            }
                            __syncwarp();
#pragma unroll
                            for (int it = 0; it < 8; ++it) {
                                const int r = it * 4 + (lane >> 3), seg = lane & 7;  // row of the warp, 16-byte piece
                                const int64_t rowp = __shfl_sync(0xffffffffu, mine, r);
                                const uint4 val = *reinterpret_cast<const uint4 *>(stg + r * 128 + ((seg ^ (r & 7)) << 4));
                                if (q * 32 + r < nvalid)
                                    reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(rowp) + ip.mb * 2 * kBM +
                                                              c0)[seg] = val;
                            }
                            __syncwarp();
                        }
                    } else {
                        uint16_t *dst = nullptr;  // this token's output row
                        if (valid) {
                            if (P.rows_out) dst = P.rows_out + static_cast<size_t>(P.route_token[p0 + tk]) * P.hidden;
                            else dst = P.y + static_cast<size_t>(p0 + tk) * P.hidden;
                            dst += ip.mb * 2 * kBM;
                        }
#pragma unroll 1
                        for (int c0 = 0; c0 < 2 * kBM; c0 += 16) {
                            float v[16];
                            __syncwarp();
                            sm100::tmem_ld16(t_gate + c0, v);
                            sm100::tmem_wait_ld();
                            uint32_t pk[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                pk[j] = static_cast<uint32_t>(f2bf(v[2 * j])) |
                                        (static_cast<uint32_t>(f2bf(v[2 * j + 1])) << 16);
                            if (valid) {
                                uint4 *o = reinterpret_cast<uint4 *>(dst + c0);
                                o[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                                o[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                            }
                        }
                    }
                }
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tail->tempty[buf]);
                ++acc;
            } else if (ip.phase == 1 && P.ks > 1) {
                // Write this split's FP32 partials; the last split of the tile
                // sums all of them in split order and writes the activations.
                float *mine = P.part + (static_cast<size_t>(ip.tile) * P.ks + ip.ks) * 2 * BN * kBM;
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    if (c0 >= nvalid) break;  // warp-uniform: columns past the tile's rows
                    float g[16], u[16];
                    __syncwarp();
                    sm100::tmem_ld16(t_gate + c0, g);
                    sm100::tmem_ld16(t_gate + BN + c0, u);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        mine[(c0 + j) * kBM + q * 32 + lane] = g[j];
                        mine[(BN + c0 + j) * kBM + q * 32 + lane] = u[j];
                    }
                }
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tail->tempty[buf]);
                ++acc;
                __threadfence();
                __syncwarp();
                int arrived = 0;
                if (lane == 0) arrived = atomicAdd(&P.split_cnt[ip.tile * 4 + q], 1);
                arrived = __shfl_sync(0xffffffffu, arrived, 0);
                if (arrived != P.ks - 1) continue;  // not the last split: nothing to publish yet
                __threadfence();
                const float *all = P.part + static_cast<size_t>(ip.tile) * P.ks * 2 * BN * kBM;
                for (int j = 0; j < nvalid; ++j) {
                    float gs = 0.f, us = 0.f;
                    for (int s = 0; s < P.ks; ++s) {
                        gs += __ldcg(all + (static_cast<size_t>(s) * 2 * BN + j) * kBM + q * 32 + lane);
                        us += __ldcg(all + (static_cast<size_t>(s) * 2 * BN + BN + j) * kBM + q * 32 + lane);
                    }
                    const float gv = rbf(gs), uv = rbf(us);
                    P.act[static_cast<size_t>(p0 + j) * P.inner + row] = f2bf(rbf(silu_f32(gv)) * uv);
                }
            } else if (ip.phase == 1) {
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    if (c0 >= nvalid) break;  // warp-uniform: columns past the tile's rows
                    float g[16], u[16];
                    __syncwarp();
                    sm100::tmem_ld16(t_gate + c0, g);
                    sm100::tmem_ld16(t_gate + BN + c0, u);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (c0 + j < nvalid) {
                            const float gv = rbf(g[j]), uv = rbf(u[j]);
                            P.act[static_cast<size_t>(p0 + c0 + j) * P.inner + row] = f2bf(rbf(silu_f32(gv)) * uv);
                        }
                    }
                }
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tail->tempty[buf]);
                ++acc;
            } else {
                // rows_out: column c of the tile is route p0 + c, whose token the
                // lanes hold (lane c % 32 of register c / 32) and broadcast; in
                // address-table mode they hold the row's destination address.
                constexpr int kTokRegs = BN < 32 ? 1 : BN / 32;
                int tok[kTokRegs];
                long long dsta[kTokRegs];
                if (P.dst_rows) {
#pragma unroll
                    for (int i = 0; i < kTokRegs; ++i) {
                        const int c = i * 32 + lane;
                        dsta[i] = c < nvalid ? P.dst_rows[p0 + c] : 0;
                    }
                } else if (P.rows_out) {
#pragma unroll
                    for (int i = 0; i < kTokRegs; ++i) {
                        const int c = i * 32 + lane;
                        tok[i] = c < nvalid ? P.route_token[p0 + c] : 0;
                    }
                }
                // accumulator 0 holds down rows `row`, accumulator 1 rows `row +
                // 128` (`row + 256` paired: the second M = 256 product)
                const int row2 = row + (PAIR ? 2 * kBM : kBM);
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    if (c0 >= nvalid) break;  // warp-uniform
                    float v[16], v2[16];
                    __syncwarp();
                    sm100::tmem_ld16(t_gate + c0, v);
                    sm100::tmem_ld16(t_gate + BN + c0, v2);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (c0 + j >= nvalid) continue;  // warp-uniform
                        uint16_t *dst;
                        if (P.dst_rows) {
                            dst = reinterpret_cast<uint16_t *>(
                                __shfl_sync(0xffffffffu, dsta[(c0 + j) >> 5], (c0 + j) & 31));
                        } else if (P.rows_out) {
                            const int t = __shfl_sync(0xffffffffu, tok[(c0 + j) >> 5], (c0 + j) & 31);
                            dst = P.rows_out + static_cast<size_t>(t) * P.hidden;
                        } else {
                            dst = P.y + static_cast<size_t>(p0 + c0 + j) * P.hidden;
                        }
                        dst[row] = f2bf(v[j]);
                        dst[row2] = f2bf(v2[j]);
                    }
                }
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(&tail->tempty[buf]);
                ++acc;
            }
            // Publish this warp's 32 rows: each lane fences its own stores, then
            // one release per warp (no cross-warp barrier, so an aborting warp
            // can never strand the others).
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                sm100::fence_proxy_async_global();
                if (ip.phase == 1) atomicAdd(&P.done1[ip.g], 1);
                else atomicAdd(&P.plan->done2_total, 1);
            }
        }
    } else if (P.src_rows && !*abort) {
        // ------------------------------------------ row gather (address tables)
        // Rows in plan order over every CTA's two gather warps, two rows in
        // flight per warp; each finished row counts into its group.
        const int n_rows = V.groups[n_groups - 1].begin + V.groups[n_groups - 1].count;
        const int units = P.hidden / 8;  // 16-byte units of a row (128 or more, a multiple of 32)
        const int gw = blockIdx.x * 2 + (warp - 6), ngw = gridDim.x * 2;
        auto group_of = [&](int p) {  // the group whose rows hold p (groups are contiguous, ascending)
            int lo = 0, hi = n_groups;
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (V.groups[mid].begin <= p) lo = mid;
                else hi = mid;
            }
            return lo;
        };
        for (int q0 = gw; q0 < n_rows; q0 += 2 * ngw) {
            const int q1 = q0 + ngw;
            const bool two = q1 < n_rows;
            const uint4 *s0 = reinterpret_cast<const uint4 *>(P.src_rows[q0]);
            const uint4 *s1 = two ? reinterpret_cast<const uint4 *>(P.src_rows[q1]) : s0;
            uint4 *d0 = reinterpret_cast<uint4 *>(P.xs) + static_cast<int64_t>(q0) * units;
            uint4 *d1 = reinterpret_cast<uint4 *>(P.xs) + static_cast<int64_t>(q1) * units;
            for (int c0 = 0; c0 < units; c0 += 8 * 32) {
                uint4 a[8], b[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + u * 32 < units) a[u] = __ldcg(s0 + c0 + u * 32 + lane);
                if (two) {
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (c0 + u * 32 < units) b[u] = __ldcg(s1 + c0 + u * 32 + lane);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + u * 32 < units) d0[c0 + u * 32 + lane] = a[u];
                if (two) {
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (c0 + u * 32 < units) d1[c0 + u * 32 + lane] = b[u];
                }
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                sm100::fence_proxy_async_global();
                atomicAdd(&P.row_ready[group_of(q0)], 1);
                if (two) atomicAdd(&P.row_ready[group_of(q1)], 1);
            }
        }
    }

    sm100::tc_fence_before();
    __syncthreads();
    // paired: no CTA leaves (or frees TMEM) while the other may still arrive
    // on its barriers or the leader's products still write its TMEM
    if constexpr (PAIR) sm100::cluster_sync();
    if (warp == 1) {
        __syncwarp();
        sm100::tc_fence_after();
        if constexpr (PAIR) sm100::tmem_dealloc_pair(tmem, S::kTmemCols);
        else sm100::tmem_dealloc(tmem, S::kTmemCols);
    }
    if (threadIdx.x == 0 && *abort) {
        atomicCAS(&P.plan->error, 0, 1);
        if (P.error_out) atomicCAS(P.error_out, 0, 3);
    }
}

// Standalone plan for the general (prefill) path; the decode path runs the
// same plan_block inside its fused routing kernel.
__global__ void __launch_bounds__(1024) grouped_plan_kernel(PlanArgs a) {
    __shared__ int scratch[33];
    grid_dependency_wait();
    grid_dependency_trigger();
    plan_block(a, scratch);
}

// xs[p] = x[route_token[p]] for the placed routes (p < offsets[experts]) and,
// when the shared expert runs, xs[routes + t] = x[t]; 16 bytes per thread.
// One warp per row: the row's token is read once, then the 16-byte units of
// the row (hidden / 8, 8 per lane at hidden 2048) are all loaded before any
// is stored.
__global__ void __launch_bounds__(256) gather_tokens_kernel(const uint16_t *__restrict__ x,
                                                            const int32_t *__restrict__ route_token,
                                                            const int32_t *__restrict__ offsets, int experts,
                                                            int routes, int shared_rows, int hidden,
                                                            uint16_t *__restrict__ xs) {
    grid_dependency_wait();
    grid_dependency_trigger();
    const int lane = threadIdx.x & 31;
    const int units = hidden / 8;
    const int placed = offsets[experts];
    // rows to fill: the placed routes, then the shared rows (routes past the
    // placed ones were dropped and own no row)
    const int rows = placed + shared_rows;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < rows; q += warps) {
        const int p = q < placed ? q : routes + (q - placed);
        const int t = p < routes ? route_token[p] : p - routes;
        const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * hidden);
        uint4 *dst = reinterpret_cast<uint4 *>(xs + static_cast<size_t>(p) * hidden);
        for (int c0 = 0; c0 < units; c0 += 8 * 32) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < units) v[u] = ld_cached(src + c);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < units) dst[c] = v[u];
            }
        }
    }
}

// ------------------------------------------------------------ host side ---

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

// BF16 tensor map: dims[0] innermost (K), 128-byte swizzle, box {64, box_rows(, 1)}.
int make_map_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides_bytes,
             uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(MOE_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    cuuint64_t d[3], s[2];
    cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), box_rows, 1}, es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) d[i] = dims[i];
    for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base), d, s, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(MOE_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return MOE_OK;
}

namespace {

template <int BN, bool PAIR, bool TOKM = false>
int launch_bn(const GroupedLaunch &L, cudaStream_t stream) {
    using S = GroupedShape<BN, PAIR, TOKM>;
    CUtensorMap gu{}, dn{}, sg{}, su{}, sd{}, xm{}, am{}, xm16{}, am16{};
    const uint64_t H = L.hidden, I = L.inner, rows = static_cast<uint64_t>(L.rows);
    {
        const uint64_t dims[3] = {H, 2 * I, static_cast<uint64_t>(L.bank_experts)};
        const uint64_t str[2] = {H * 2, static_cast<uint64_t>(L.gate_up_stride) * 2};
        if (int rc = make_map_bf16(&gu, L.gate_up, 3, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[3] = {I, H, static_cast<uint64_t>(L.bank_experts)};
        const uint64_t str[2] = {I * 2, static_cast<uint64_t>(L.down_stride) * 2};
        if (int rc = make_map_bf16(&dn, L.down, 3, dims, str, kBM)) return rc;
    }
    const void *sgp = L.sh_gate ? L.sh_gate : L.gate_up, *sup = L.sh_up ? L.sh_up : L.gate_up;
    const void *sdp = L.sh_down ? L.sh_down : L.down;
    {
        const uint64_t dims[2] = {H, I}, str[1] = {H * 2};
        if (int rc = make_map_bf16(&sg, sgp, 2, dims, str, kBM)) return rc;
        if (int rc = make_map_bf16(&su, sup, 2, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[2] = {I, H}, str[1] = {I * 2};
        if (int rc = make_map_bf16(&sd, sdp, 2, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[2] = {H, rows}, str[1] = {H * 2};
        if (int rc = make_map_bf16(&xm, L.xs, 2, dims, str, S::kBRows)) return rc;
        if (int rc = make_map_bf16(&xm16, L.xs, 2, dims, str, 16)) return rc;
    }
    {
        const uint64_t dims[2] = {I, rows}, str[1] = {I * 2};
        if (int rc = make_map_bf16(&am, L.act, 2, dims, str, S::kBRows)) return rc;
        if (int rc = make_map_bf16(&am16, L.act, 2, dims, str, 16)) return rc;
    }
    if (int rc = ensure_dynamic_smem(swiglu_grouped_kernel<BN, PAIR, TOKM>, S::kSmem, "cudaFuncSetAttribute(grouped)"))
        return rc;
    GroupedParams P{};
    P.groups = L.groups;
    P.plan = L.plan;
    P.off1 = L.off1;
    P.off2 = L.off2;
    P.done1 = L.done1;
    P.done2 = L.done2;
    P.split_cnt = L.split_cnt;
    P.part = L.part;
    P.act = L.act;
    P.y = L.y;
    P.out = L.out;
    P.route_pos = L.route_pos;
    P.idx = L.idx;
    P.scores = L.scores;
    P.sig = L.sig;
    P.group_of_expert = L.group_of_expert;
    P.route_token = L.route_token;
    P.rows_out = L.rows_out;
    P.stage_error = L.stage_error;
    P.x = L.x;
    P.sh_gate = L.sh_gate && L.sh_up && L.sh_down ? L.sh_gate : nullptr;
    P.sh_up = L.sh_up;
    P.sh_down = L.sh_down;
    P.xs = const_cast<uint16_t *>(L.xs);
    P.gather_x = L.gather_x;
    P.gather_need = 4 * L.ctas;
    P.src_rows = L.src_rows;
    P.dst_rows = L.dst_rows;
    P.row_ready = L.row_ready;
    P.error_out = L.error_out;
    P.tokens = L.tokens;
    P.top_k = L.top_k;
    P.hidden = L.hidden;
    P.inner = L.inner;
    P.ks = L.ks;
    P.phases = L.phases == 1 || L.phases == 2 ? L.phases : 3;
    if constexpr (PAIR) {
        const int pairs = std::min(L.ctas / 2, grouped_pair_clusters());
        return launch_pdl_cluster2(swiglu_grouped_kernel<BN, true, false>, dim3(2 * pairs), dim3(kThreads), S::kSmem, stream,
                                   "swiglu_grouped_kernel", gu, dn, sg, su, sd, xm, am, xm16, am16, P);
    }
    return launch_pdl(swiglu_grouped_kernel<BN, false, TOKM>, dim3(L.ctas), dim3(kThreads), S::kSmem, stream,
                      "swiglu_grouped_kernel", gu, dn, sg, su, sd, xm, am, xm16, am16, P);
}

}  // namespace

// How many CTA pairs of the paired kernel can be resident at once on the
// current device (clusters of two must share a GPC), 0 if none; cached per
// device.
int grouped_pair_clusters() {
    static std::mutex mu;
    static int cached[64];
    static bool known[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (known[dev]) return cached[dev];
    using S = GroupedShape<128, true>;
    int n = 0;
    // the first query may come while a stream of this thread is being
    // captured: relaxed mode lets these non-stream calls run
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (ensure_dynamic_smem(swiglu_grouped_kernel<128, true, false>, S::kSmem, "cudaFuncSetAttribute(grouped)") ==
        MOE_OK) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * sm_count());
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = S::kSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, swiglu_grouped_kernel<128, true, false>, &cfg) != cudaSuccess) n = 0;
    }
    cudaThreadExchangeStreamCaptureMode(&mode);
    cudaGetLastError();  // a failed query leaves no sticky error
    cached[dev] = n;
    known[dev] = true;
    return n;
}

bool grouped_swap_forced() {
    const char *v = getenv("LRB_GROUPED_SWAP");
    return v && v[0] == '1';
}

// The paired kernel (weights as an M = 256 operand split over two CTAs) can
// serve the prefill widths (token tiles of 128, no K split, no in-kernel
// gather or combine) when the widths divide into 256-row gate/up and 512-row
// down blocks and pairs can be resident; the plan's item counts (mb1, mb2)
// follow the choice.  It gives the same results as the single-CTA kernels and
// measured no faster than them (the operand traffic it saves is not what
// bounds the kernel), so it runs only with LRB_GROUPED_PAIRS=1 in the
// environment (read at every call, so one process can run both).
bool grouped_pairs_for(int bn, int ks, int inner, int hidden) {
    const char *v = getenv("LRB_GROUPED_PAIRS");
    const bool enabled = v && v[0] == '1';
    return enabled && bn == 128 && ks == 1 && inner % (2 * kBM) == 0 && hidden % (4 * kBM) == 0 &&
           grouped_pair_clusters() > 0;
}

int grouped_bn_for(int tokens) { return tokens <= 16 ? 16 : tokens <= 64 ? 32 : tokens <= 512 ? 64 : 128; }
// K splits of the phase-1 items at the narrowest grouped widths, so that
// more SMs stream weights while few experts are active: two up to 4 tokens,
// none from 5 (one box, grouped-kernel step at T = 4 / 8 / 16 with 1, 2 or 4
// splits: 66.5 / 62.0 / 64.0, 76.1 / 79.1 / 81.0 and 99.6 / 109.2 / 110.4 us;
// the FP32 partials and their last-split sum cost more than the extra SMs
// gain from T = 5 on).  LRB_GROUPED_KS=1, 2 or 4 (read at every call)
// overrides the choice for 3 to 16 tokens, for measurement.
int grouped_ks_for(int tokens) {
    if (tokens > 2 && tokens <= 16) {
        const char *v = getenv("LRB_GROUPED_KS");
        if (v && (v[0] == '1' || v[0] == '2' || v[0] == '4') && v[1] == 0) return v[0] - '0';
    }
    return tokens <= 4 ? 2 : 1;
}

// Upper bound of phase-1 tiles times splits times 2 * BN * 128 floats.
size_t grouped_part_floats(int tokens, int experts, int top_k, int inner) {
    const int ks = grouped_ks_for(tokens);
    if (ks == 1) return 0;
    return static_cast<size_t>(grouped_tiles_max(tokens, experts, top_k, inner)) * ks * 2 * grouped_bn_for(tokens) *
           kBM;
}

int grouped_tiles_max(int tokens, int experts, int top_k, int inner) {
    const int bn = grouped_bn_for(tokens);
    const int groups = std::min(experts, tokens * top_k) + 1;
    const int rows = tokens * top_k + tokens;
    return (inner / kBM) * (groups + rows / bn + 1);
}

int launch_grouped_plan(const PlanArgs &a, cudaStream_t stream) {
    return launch_pdl(grouped_plan_kernel, dim3(1), dim3(1024), 0, stream, "grouped_plan_kernel", a);
}

int launch_gather_tokens(const uint16_t *x, const int32_t *route_token, const int32_t *offsets, int experts,
                         int routes, int shared_rows, int hidden, uint16_t *xs, cudaStream_t stream) {
    const int64_t rows = static_cast<int64_t>(routes) + shared_rows;  // a bound on the rows to fill
    const int grid = static_cast<int>(std::min<int64_t>((rows + 7) / 8, static_cast<int64_t>(sm_count()) * 8));
    if (grid == 0) return MOE_OK;
    return launch_pdl(gather_tokens_kernel, dim3(grid), dim3(256), 0, stream, "gather_tokens_kernel", x,
                      route_token, offsets, experts, routes, shared_rows, hidden, xs);
}

int launch_grouped(const GroupedLaunch &L, cudaStream_t stream) {
    LRB_REQUIRE(L.hidden % kBM == 0 && L.inner % kBM == 0 && L.hidden % kCombineCols == 0,
                "grouped: hidden must be a multiple of 1024 and inner of 128");
    LRB_REQUIRE((L.src_rows == nullptr) == (L.dst_rows == nullptr) && (!L.src_rows || (L.row_ready && !L.gather_x)),
                "grouped: address tables need both tables and the row counters, without gather_x");
    LRB_REQUIRE(L.ks == 1 || L.ks == 2 || L.ks == 4, "grouped: K split %d not in {1, 2, 4}", L.ks);
    LRB_REQUIRE(L.top_k <= 32, "grouped: top_k %d > 32", L.top_k);
    if (L.pairs) {
        LRB_REQUIRE(L.bn == 128 && L.ks == 1 && !L.gather_x && L.inner % (2 * kBM) == 0 && L.hidden % (4 * kBM) == 0 &&
                        L.ctas >= 2,
                    "grouped: the paired kernel needs 128-token tiles, no K split and no in-kernel gather");
        return launch_bn<128, true>(L, stream);
    }
    switch (L.bn) {
        case 16: return launch_bn<16, false>(L, stream);
        case 32: return launch_bn<32, false>(L, stream);
        case 64: return launch_bn<64, false>(L, stream);
        case 128:
            // 128-token tiles run tokens-as-M unless LRB_GROUPED_SWAP=1
            // (the swapped layout, for comparison; the results are the same)
            if (L.ks == 1 && !L.gather_x && !grouped_swap_forced()) return launch_bn<128, false, true>(L, stream);
            return launch_bn<128, false>(L, stream);
        default: return set_error(MOE_EINVAL, "grouped: unsupported token tile %d", L.bn);
    }
}

}  // namespace lrb

extern "C" int moe_grouped_paired(int tokens, int inner, int hidden) {
    if (tokens <= 0 || inner <= 0 || hidden <= 0) return 0;
    return lrb::grouped_pairs_for(lrb::grouped_bn_for(tokens), lrb::grouped_ks_for(tokens), inner, hidden) ? 1 : 0;
}
