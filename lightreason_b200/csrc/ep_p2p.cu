// Expert-parallel exchange over NVLink peer memory, fused with the experts
// and without host synchronisation: every rank owns one symmetric buffer (same
// layout on all ranks, mapped into every peer by CUDA IPC), and the ranks'
// kernels meet through release/acquire flags in those buffers.
//
// Symmetric buffer of rank q (W ranks, C = capacity routes per sender, T0 =
// own token rows):
//   flags_publish uint32 [W]      step at which rank s published its routes to q
//   flags_return  uint32 [W]      step at which rank d finished q's rows
//   count         int32  [W]      routes rank s sent to q this step
//   meta          int32  [W][C][4] (local expert on q, return row on s, token on s, 0)
//   tokens        bf16   [T0][H]  q's own token rows, read by the owners
//   ret           bf16   [C][H]   q's routes' expert rows, by position
//
// One step on rank r (the step number lives in device memory and advances at
// the end of the step, so a captured CUDA graph replays correctly):
//   route    the tensor-core router's FP32 partials, then one warp per own
//            token selects its experts (the layer's selection), copies the
//            token row to r.tokens and gives its routes the return rows
//            t * K + (rank of the route's expert among the token's K), so
//            the ordered combine, which sums in ascending row, adds them in
//            ascending expert id (the eager order); each route to expert e
//            goes to its owner d (e / El, or the placement table's entry) as
//            an entry of d.meta[r] (local expert, return row, token), slots
//            taken per CTA with one atomic per
//            destination; the last CTA writes d.count[r] and releases
//            d.flags_publish[r] = step.  No token row moves here, and no
//            permute of the own routes is needed.
//   experts  plan (one CTA): wait for every flags_publish[s] == step, then lay
//            out one group per local expert with routes (ascending id; within
//            it sender by sender; within a sender in the order the plan's
//            row cursors hand out, which no result depends on) and
//            the shared expert's group of the own tokens last, and for every
//            row the address it is read from (sender s's tokens row) and the
//            address its down output goes to (s.ret[row], or for a shared row
//            the caller's shared_rows[t]).  Then the grouped tensor-core
//            kernel in address-table mode: its gather warps pull the rows
//            over NVLink as the weights start streaming, and its epilogue
//            stores every down row straight into the sender's ret.
//   finish   releases s.flags_return[r] = step for every s (r's reads of their
//            tokens and its writes into their ret are complete), waits for
//            every flags_return[d] == step (r.ret is complete), advances the
//            step; the ordered combine then reads ret.
// Buffer reuse across steps is ordered by the flags: a rank overwrites its
// tokens and the owners' meta only in the next step, after every owner
// released it in finish, i.e. after the owners' kernels that read them.
// Every wait is bounded (globaltimer): on timeout the kernel stores an error
// code in *error and carries on without the missing data, so a missing peer
// cannot hang the GPU.
//
// The reference runs its MoE layer on one GPU; this exchange has no
// counterpart there.
#include "common.cuh"
#include "kernels.cuh"
#include "routing.cuh"

namespace lrb {

namespace {

constexpr uint64_t kPeerWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until flags[i] == step for every i < world (thread-level, bounded).
__device__ __forceinline__ bool wait_flags(const uint32_t *flags, int world, uint32_t step) {
    const uint64_t t0 = gtime();
    for (int i = 0; i < world; ++i) {
        while (ld_acquire_sys(flags + i) != step) {
            if (gtime() - t0 > kPeerWaitNs) return false;
            __nanosleep(128);
        }
    }
    return true;
}

__device__ __forceinline__ uint8_t *peer_base(const EpP2PArgs &a, int q) {
    return reinterpret_cast<uint8_t *>(a.peers[q]);
}

// One row copy by a warp in 16-byte units, eight loads per lane in flight
// before their stores.
__device__ __forceinline__ void warp_copy_row(const uint16_t *src, uint16_t *dst, int hidden, int lane) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const int n = hidden / 8;
    int v = lane;
    for (; v + 7 * 32 < n; v += 8 * 32) {
        uint4 r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = __ldg(s + v + 32 * i);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[v + 32 * i] = r[i];
    }
    for (; v < n; v += 32) d[v] = __ldg(s + v);
}

// Last-CTA election: once every thread of the CTA is past its stores, one
// thread counts the CTA in with an acquire-release add at GPU scope, so the
// last CTA has every CTA's stores ordered before it; its system-scope release
// of a flag then passes them on to the peer that acquires the flag (release
// and acquire are cumulative along that chain).  No sequentially consistent
// system fence is needed; such a fence costs microseconds here.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t *p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ bool last_cta(int32_t *counter) {
    __shared__ int is_last;
    __syncthreads();
    if (threadIdx.x == 0) is_last = atom_add_acq_rel_gpu(counter, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    return is_last != 0;
}

}  // namespace

// Selection of the own tokens and publication of their routes, see the file
// comment.  One warp per token, eight tokens per CTA; send_cnt (sync + 2,
// zero at entry) counts the slots taken per destination and is zeroed again
// by the last CTA.
template <int VPL>
__global__ void __launch_bounds__(256) ep_p2p_select_kernel(EpP2PArgs a, const uint16_t *__restrict__ x, int tokens,
                                                            const float *__restrict__ part, int ks,
                                                            const float *__restrict__ bias,
                                                            const uint16_t *__restrict__ gate_w,
                                                            uint16_t *__restrict__ logits, int64_t *__restrict__ idx,
                                                            uint16_t *__restrict__ scores, uint16_t *__restrict__ sig,
                                                            int32_t *__restrict__ route_pos) {
    __shared__ int cta_cnt[64], cta_base[64];
    grid_dependency_wait();
    grid_dependency_trigger();
    const uint32_t step = *a.step;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int El = a.local_experts, K = a.top_k, W = a.world;
    int32_t *send_cnt = a.sync + 2;
    if (threadIdx.x < W) cta_cnt[threadIdx.x] = 0;
    __syncthreads();
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    int e = -1, row = -1, d = 0, le = 0, slot = 0;
    if (t < tokens) {
        float w;
        select_token<VPL>(t, logits, bias, tokens, a.experts, K, idx, nullptr, scores, x, gate_w, a.hidden, sig, part,
                          ks, &e, &w);
        uint16_t *own = reinterpret_cast<uint16_t *>(peer_base(a, a.rank) + a.off_tokens);
        warp_copy_row(x + static_cast<size_t>(t) * a.hidden, own + static_cast<size_t>(t) * a.hidden, a.hidden, lane);
        // the return row: rank of this route's expert among the token's K
        int rank = 0;
        for (int j = 0; j < K; ++j) {
            const int ej = __shfl_sync(0xffffffffu, e, j);
            rank += (lane < K && ej < e) ? 1 : 0;
        }
        if (lane < K) {
            row = t * K + rank;
            route_pos[static_cast<size_t>(t) * K + lane] = row;
            if (a.placement) {
                const int pl = __ldg(a.placement + e);
                d = pl >> 16;
                le = pl & 0xffff;
                if (d < 0 || d >= W || le >= El) {  // a malformed table: the route is dropped, the step fails
                    atomicExch(a.error, 4);
                    row = -1;
                }
            } else {
                d = e / El;
                le = e - d * El;
            }
            if (row >= 0) slot = atomicAdd(&cta_cnt[d], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x < W && cta_cnt[threadIdx.x] > 0)
        cta_base[threadIdx.x] = atomicAdd(&send_cnt[threadIdx.x], cta_cnt[threadIdx.x]);
    __syncthreads();
    if (row >= 0) {
        const int j = cta_base[d] + slot;
        if (j < a.capacity) {  // cannot be exceeded: a rank sends at most own_rows * K routes
            int4 *meta = reinterpret_cast<int4 *>(peer_base(a, d) + a.off_meta) + static_cast<size_t>(a.rank) * a.capacity;
            meta[j] = make_int4(le, row, t, 0);
        }
    }
    if (last_cta(a.sync + 0)) {
        if (threadIdx.x < W) {
            const int dd = threadIdx.x;
            uint8_t *dst = peer_base(a, dd);
            reinterpret_cast<int32_t *>(dst + a.off_count)[a.rank] = min(send_cnt[dd], a.capacity);
            send_cnt[dd] = 0;
            st_release_sys(reinterpret_cast<uint32_t *>(dst + a.off_flags_publish) + a.rank, step);
        }
        if (threadIdx.x == 0) a.sync[0] = 0;
    }
}

// The owner's plan (one CTA of 1024 threads), see the file comment.  cnt is
// the [El][W] table of routes per (local expert, sender); E = El * W <= 1024.
struct EpPlanOut {
    GroupedGroup *groups;
    GroupedPlan *plan;
    int32_t *off1, *off2, *done1, *done2, *row_ready;
    int64_t *src_rows, *dst_rows;
    uint16_t *shared_rows;
    uint16_t *trash_row;  // one row [H] that catches a malformed entry's output
    int32_t *stats;  // [2 + W]: rows received, local experts with rows, rows per sender
    int tokens, bn, mb1, mb2;
};

__global__ void __launch_bounds__(1024) ep_p2p_plan_kernel(EpP2PArgs a, EpPlanOut o) {
    __shared__ int cnt[1024], base[1024];
    __shared__ int sent[64];
    __shared__ int scratch[100];
    __shared__ int ok;
    grid_dependency_wait();
    grid_dependency_trigger();
    const uint32_t step = *a.step;
    const int W = a.world, El = a.local_experts, E = El * W, C = a.capacity;
    uint8_t *self = peer_base(a, a.rank);
    if (threadIdx.x == 0) {
        ok = wait_flags(reinterpret_cast<const uint32_t *>(self + a.off_flags_publish), W, step);
        if (!ok) atomicExch(a.error, 1);
    }
    for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const int32_t *count = reinterpret_cast<const int32_t *>(self + a.off_count);
    const int4 *meta = reinterpret_cast<const int4 *>(self + a.off_meta);
    if (threadIdx.x < W) sent[threadIdx.x] = ok ? min(max(__ldcg(count + threadIdx.x), 0), C) : 0;
    __syncthreads();
    // routes per (local expert, sender); the entries of a sender are in its
    // permuted order, so ascending in local expert
    for (int s = 0; s < W; ++s)
        for (int j0 = 0; j0 < sent[s]; j0 += 4 * static_cast<int>(blockDim.x)) {
            // four entries per thread with their loads in flight together;
            // equal experts within a warp are counted once
            int les[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + u * blockDim.x + threadIdx.x;
                les[u] = j < sent[s] ? __ldcg(meta + static_cast<size_t>(s) * C + j).x : -1;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int le = les[u] >= 0 && les[u] < El ? les[u] : -1;
                const unsigned same = __match_any_sync(0xffffffffu, le);
                if (le >= 0 && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&cnt[le * W + s], __popc(same));
            }
        }
    __syncthreads();
    // base[le][s]: the first row of sender s's routes in expert le's group
    // (scan in (le, s) order); it then serves as the row cursor of that run
    const int i = threadIdx.x;
    const int v_ls = i < E ? cnt[i] : 0;
    int3 tot_a;
    const int3 sa = block_exclusive_scan3(make_int3(v_ls, 0, 0), scratch, &tot_a);
    const int routed = tot_a.x, b = sa.x;
    if (i < E) base[i] = b;
    __syncthreads();
    // groups: local experts with rows in ascending id, then the shared expert
    int tot_le = 0;
    if (i < El)
        for (int s = 0; s < W; ++s) tot_le += cnt[i * W + s];
    const int nt = (tot_le + o.bn - 1) / o.bn;
    int3 tot_b;
    const int3 sb = block_exclusive_scan3(make_int3(tot_le > 0 ? 1 : 0, tot_le > 0 ? o.mb1 * nt : 0,
                                                    tot_le > 0 ? o.mb2 * nt : 0), scratch, &tot_b);
    const int n_active = tot_b.x, t1 = tot_b.y, t2 = tot_b.z;
    const int g = sb.x, e1 = sb.y, e2 = sb.z;
    if (i < El && tot_le > 0) {
        GroupedGroup G;
        G.weight = i;
        G.begin = base[i * W];
        G.count = tot_le;
        G.ntiles = nt;
        o.groups[g] = G;
        o.off1[g] = e1;
        o.off2[g] = e2;
        o.done1[g] = 0;
        o.done2[g] = 0;
        o.row_ready[g] = 0;
    }
    if (threadIdx.x == 0) {
        GroupedGroup G;  // the shared expert: bank entry El, the own tokens
        G.weight = El;
        G.begin = routed;
        G.count = o.tokens;
        G.ntiles = (o.tokens + o.bn - 1) / o.bn;
        const int n = n_active;
        o.groups[n] = G;
        o.off1[n] = t1;
        o.off2[n] = t2;
        o.done1[n] = 0;
        o.done2[n] = 0;
        o.row_ready[n] = 0;
        o.off1[n + 1] = t1 + o.mb1 * G.ntiles;
        o.off2[n + 1] = t2 + o.mb2 * G.ntiles;
        o.plan->num_groups = n + 1;
        o.plan->items1 = t1 + o.mb1 * G.ntiles;
        o.plan->items2 = t2 + o.mb2 * G.ntiles;
        o.plan->items3 = 0;
        o.plan->work = 0;
        o.plan->error = ok ? 0 : 4;
        o.plan->done2_total = 0;
        o.plan->xs_ready = 0;
        o.plan->act_ready = 0;
        o.plan->work2 = 0;
        if (o.stats) {
            o.stats[0] = routed;
            o.stats[1] = n_active;
        }
    }
    if (o.stats && threadIdx.x < W) o.stats[2 + threadIdx.x] = sent[threadIdx.x];
    // the address tables: routed rows, then the shared rows.  Every routed row
    // first gets a harmless pair (the own first token row, the trash row), so
    // no row is left with a stale address even if a sender's entries were
    // malformed; valid entries then overwrite each of them once.
    const int64_t rowb = static_cast<int64_t>(a.hidden) * 2;
    const int64_t own = a.peers[a.rank] + a.off_tokens;
    for (int r = threadIdx.x; r < routed; r += blockDim.x) {
        o.src_rows[r] = own;
        o.dst_rows[r] = reinterpret_cast<int64_t>(o.trash_row);
    }
    __syncthreads();
    for (int s = 0; s < W; ++s) {
        const int64_t peer = a.peers[s];
        for (int j0 = 0; j0 < sent[s]; j0 += blockDim.x) {
            const int j = j0 + threadIdx.x;
            int4 m = make_int4(-1, -1, -1, 0);
            if (j < sent[s]) m = __ldcg(meta + static_cast<size_t>(s) * C + j);
            const bool ok_m = m.x >= 0 && m.x < El && m.y >= 0 && m.y < C && m.z >= 0 && m.z < a.own_rows;
            // a row from the run's cursor; equal experts within a warp take
            // consecutive rows with one shared-memory atomic
            const int key = ok_m ? m.x : -1;
            const unsigned same = __match_any_sync(0xffffffffu, key);
            const int leader = __ffs(same) - 1;
            int first_row = 0;
            if (ok_m && (threadIdx.x & 31) == leader) first_row = atomicAdd(&base[m.x * W + s], __popc(same));
            first_row = __shfl_sync(0xffffffffu, first_row, leader);
            const int row = first_row + __popc(same & ((1u << (threadIdx.x & 31)) - 1u));
            if (!ok_m || row < 0 || row >= routed) continue;
            o.src_rows[row] = peer + a.off_tokens + m.z * rowb;
            o.dst_rows[row] = peer + a.off_ret + m.y * rowb;
        }
    }
    for (int t = threadIdx.x; t < o.tokens; t += blockDim.x) {
        o.src_rows[routed + t] = own + t * rowb;
        o.dst_rows[routed + t] = reinterpret_cast<int64_t>(o.shared_rows) + t * rowb;
    }
}

__global__ void ep_p2p_finish_kernel(EpP2PArgs a) {
    grid_dependency_wait();
    const uint32_t step = *a.step;
    if (threadIdx.x < a.world) {
        // this rank's reads of the peers' tokens and its stores into their ret
        // (the expert kernel, complete before the dependency wait above) are
        // ordered before this release
        st_release_sys(reinterpret_cast<uint32_t *>(peer_base(a, threadIdx.x) + a.off_flags_return) + a.rank, step);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint8_t *self = peer_base(a, a.rank);
        if (!wait_flags(reinterpret_cast<const uint32_t *>(self + a.off_flags_return), a.world, step))
            atomicExch(a.error, 2);
        *a.step = step + 1;
    }
}

}  // namespace lrb

namespace {

int check_p2p(const moe_ep_p2p *p) {
    LRB_REQUIRE(p && p->peers && p->step && p->sync && p->error, "ep_p2p: null argument");
    LRB_REQUIRE(p->world >= 1 && p->world <= 64 && p->rank >= 0 && p->rank < p->world,
                "ep_p2p: rank %d / world %d out of range", p->rank, p->world);
    LRB_REQUIRE(p->experts % p->world == 0 && p->local_experts == p->experts / p->world && p->experts <= 1024,
                "ep_p2p: %d experts do not shard over %d ranks (at most 1024 experts)", p->experts, p->world);
    LRB_REQUIRE(p->hidden > 0 && p->hidden % 1024 == 0 && p->capacity > 0 && p->top_k >= 1 && p->own_rows > 0 &&
                    p->capacity >= p->own_rows * p->top_k,
                "ep_p2p: bad shape (hidden %d, capacity %d, own rows %d, top_k %d)", p->hidden, p->capacity,
                p->own_rows, p->top_k);
    LRB_REQUIRE(p->off_tokens % 16 == 0 && p->off_ret % 16 == 0 && p->off_meta % 16 == 0,
                "ep_p2p: token rows, ret and meta offsets must be 16-byte aligned");
    return MOE_OK;
}

lrb::EpP2PArgs args_of(const moe_ep_p2p *p) {
    lrb::EpP2PArgs a{};
    a.peers = p->peers;
    a.off_flags_publish = p->off_flags_publish;
    a.off_flags_return = p->off_flags_return;
    a.off_count = p->off_count;
    a.off_meta = p->off_meta;
    a.off_tokens = p->off_tokens;
    a.off_ret = p->off_ret;
    a.world = p->world;
    a.rank = p->rank;
    a.capacity = p->capacity;
    a.hidden = p->hidden;
    a.top_k = p->top_k;
    a.experts = p->experts;
    a.local_experts = p->local_experts;
    a.own_rows = p->own_rows;
    a.step = p->step;
    a.sync = p->sync;
    a.error = p->error;
    a.placement = p->placement;
    return a;
}

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Workspace of moe_ep_p2p_experts: the plan of the grouped kernel, the
// address tables and the route-ordered rows and activations, for the most
// rows an owner can receive (every sender's capacity) plus its own tokens.
struct ExpertsLayout {
    size_t groups, plan, off1, off2, done1, done2, ready, split, src, dst, trash, xs, act, total;
    int rows;
};
ExpertsLayout experts_layout(const moe_ep_p2p *p, int inner) {
    ExpertsLayout L{};
    const size_t G = static_cast<size_t>(p->local_experts) + 1;
    L.rows = p->own_rows + p->world * p->capacity;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes);
        return at;
    };
    L.groups = take(G * sizeof(lrb::GroupedGroup));
    L.plan = take(sizeof(lrb::GroupedPlan));
    L.off1 = take((G + 1) * 4);
    L.off2 = take((G + 1) * 4);
    L.done1 = take(G * 4);
    L.done2 = take(G * 4);
    L.ready = take(G * 4);
    L.split = take(16);
    L.src = take(static_cast<size_t>(L.rows) * 8);
    L.dst = take(static_cast<size_t>(L.rows) * 8);
    L.trash = take(static_cast<size_t>(p->hidden) * 2);
    L.xs = take(static_cast<size_t>(L.rows) * p->hidden * 2);
    L.act = take(static_cast<size_t>(L.rows) * inner * 2);
    L.total = o;
    return L;
}

template <class T>
T *at(void *base, size_t offset) {
    return reinterpret_cast<T *>(static_cast<char *>(base) + offset);
}

}  // namespace

extern "C" {

int moe_ipc_alloc(size_t bytes, void **ptr, void *handle) {
    LRB_REQUIRE(ptr && handle && bytes > 0, "moe_ipc_alloc: bad arguments");
    void *p = nullptr;
    LRB_CUDA(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return lrb::cuda_error(e, "moe_ipc_alloc");
    }
    *ptr = p;
    return MOE_OK;
}

int moe_ipc_free(void *ptr) {
    if (ptr) LRB_CUDA(cudaFree(ptr));
    return MOE_OK;
}

int moe_ipc_open(const void *handle, void **ptr) {
    LRB_REQUIRE(handle && ptr, "moe_ipc_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    LRB_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return MOE_OK;
}

int moe_ipc_close(void *ptr) {
    if (ptr) LRB_CUDA(cudaIpcCloseMemHandle(ptr));
    return MOE_OK;
}

size_t moe_ep_p2p_route_workspace_bytes(const moe_ep_p2p *p, int tokens) {
    if (check_p2p(p) != MOE_OK || tokens < 0) return 0;
    return moe_router_workspace_bytes(tokens, p->experts);
}

int moe_ep_p2p_route(const moe_ep_p2p *p, const uint16_t *x, int tokens, const uint16_t *router, const float *bias,
                     const uint16_t *shared_gate_w, uint16_t *logits, int64_t *idx, uint16_t *scores, uint16_t *sig,
                     int32_t *route_pos, void *workspace, size_t workspace_bytes, void *stream) {
    using namespace lrb;
    if (int rc = check_p2p(p)) return rc;
    if (int rc = check_router_args(tokens, p->hidden, p->experts, p->top_k)) return rc;
    LRB_REQUIRE(p->top_k <= 16, "moe_ep_p2p_route: top_k %d > 16", p->top_k);
    LRB_REQUIRE(x && router && logits && idx && scores && route_pos, "moe_ep_p2p_route: null input");
    LRB_REQUIRE(!shared_gate_w || sig, "moe_ep_p2p_route: shared_gate_w needs a sig output");
    LRB_REQUIRE(tokens <= p->own_rows, "moe_ep_p2p_route: tokens %d > own rows %d", tokens, p->own_rows);
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0, "moe_ep_p2p_route: x must be 16-byte aligned");
    if (int rc = require_sm100()) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int E = p->experts, H = p->hidden;
    // the logits: tensor-core partials (summed by the selection) at prefill
    // widths, the decode logits kernel for one or two tokens
    const float *part = nullptr;
    int ks = 1;
    const uint16_t *gate_sel = shared_gate_w;
    if (tokens > kDecodeMaxTokens) {
        const size_t need = moe_router_workspace_bytes(tokens, E);
        if (need > 0 && workspace && workspace_bytes >= need) {
            ks = router_tc_splits(tokens, E);
            part = static_cast<const float *>(workspace);
        }
        if (int rc = launch_router_tc(x, router, tokens, H, E, logits, const_cast<float *>(part), ks, nullptr, s))
            return rc;
    } else if (tokens > 0) {
        if (int rc = launch_router_logits(x, router, shared_gate_w, tokens, H, E, logits, sig, s)) return rc;
        gate_sel = nullptr;  // sig came with the logits
    }
    const dim3 grid(static_cast<unsigned>(std::max(1, (tokens + 7) / 8)));
    if (E <= 256)
        return launch_pdl(ep_p2p_select_kernel<8>, grid, dim3(256), 0, s, "ep_p2p_select_kernel", args_of(p), x,
                          tokens, part, ks, bias, gate_sel, logits, idx, scores, sig, route_pos);
    return launch_pdl(ep_p2p_select_kernel<32>, grid, dim3(256), 0, s, "ep_p2p_select_kernel", args_of(p), x,
                      tokens, part, ks, bias, gate_sel, logits, idx, scores, sig, route_pos);
}

size_t moe_ep_p2p_workspace_bytes(const moe_ep_p2p *p, int inner) {
    if (check_p2p(p) != MOE_OK || (inner != 256 && inner != 512 && inner != 1024)) return 0;
    return experts_layout(p, inner).total;
}

int moe_ep_p2p_experts(const moe_ep_p2p *p, const uint16_t *gate_up, const uint16_t *down, int inner, int tokens,
                       uint16_t *shared_rows, int32_t *stats, void *workspace, size_t workspace_bytes,
                       void *const *kernel_events, void *stream) {
    using namespace lrb;
    if (int rc = check_p2p(p)) return rc;
    LRB_REQUIRE(gate_up && down && shared_rows, "moe_ep_p2p_experts: null input");
    LRB_REQUIRE(inner == 256 || inner == 512 || inner == 1024, "moe_ep_p2p_experts: inner %d not in {256, 512, 1024}",
                inner);
    LRB_REQUIRE(tokens >= 1 && tokens <= p->own_rows, "moe_ep_p2p_experts: tokens %d outside [1, %d]", tokens,
                p->own_rows);
    auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    LRB_REQUIRE(a16(gate_up) && a16(down) && a16(shared_rows) && a16(workspace),
                "moe_ep_p2p_experts: banks, shared_rows and workspace must be 16-byte aligned");
    const ExpertsLayout L = experts_layout(p, inner);
    LRB_REQUIRE(workspace && workspace_bytes >= L.total, "moe_ep_p2p_experts: workspace %zu < %zu bytes",
                workspace_bytes, L.total);
    if (int rc = require_sm100()) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int H = p->hidden, I = inner, El = p->local_experts;
    const int bn = grouped_bn_for(L.rows);
    EpPlanOut o{};
    o.groups = at<GroupedGroup>(workspace, L.groups);
    o.plan = at<GroupedPlan>(workspace, L.plan);
    o.off1 = at<int32_t>(workspace, L.off1);
    o.off2 = at<int32_t>(workspace, L.off2);
    o.done1 = at<int32_t>(workspace, L.done1);
    o.done2 = at<int32_t>(workspace, L.done2);
    o.row_ready = at<int32_t>(workspace, L.ready);
    o.src_rows = at<int64_t>(workspace, L.src);
    o.dst_rows = at<int64_t>(workspace, L.dst);
    o.shared_rows = shared_rows;
    o.trash_row = at<uint16_t>(workspace, L.trash);
    o.stats = stats;
    o.tokens = tokens;
    o.bn = bn;
    const bool pairs = grouped_pairs_for(bn, 1, I, H);
    o.mb1 = I / (pairs ? 256 : 128);
    o.mb2 = H / (pairs ? 512 : 256);
    if (int rc = launch_pdl(ep_p2p_plan_kernel, dim3(1), dim3(1024), 0, s, "ep_p2p_plan_kernel", args_of(p), o))
        return rc;
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (kernel_events) LRB_CUDA(cudaStreamIsCapturing(s, &capturing));
    auto mark = [&](int i) -> int {
        if (kernel_events && kernel_events[i])
            LRB_CUDA(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(kernel_events[i]), s,
                                              capturing == cudaStreamCaptureStatusActive ? cudaEventRecordExternal
                                                                                         : cudaEventRecordDefault));
        return MOE_OK;
    };
    if (int rc = mark(0)) return rc;
    GroupedLaunch GL{};
    GL.gate_up = gate_up;
    GL.down = down;
    GL.gate_up_stride = static_cast<int64_t>(2) * I * H;
    GL.down_stride = static_cast<int64_t>(H) * I;
    GL.bank_experts = El + 1;
    GL.xs = at<uint16_t>(workspace, L.xs);
    GL.act = at<uint16_t>(workspace, L.act);
    GL.rows = L.rows;
    GL.groups = o.groups;
    GL.plan = o.plan;
    GL.off1 = o.off1;
    GL.off2 = o.off2;
    GL.done1 = o.done1;
    GL.done2 = o.done2;
    GL.split_cnt = at<int32_t>(workspace, L.split);
    GL.src_rows = o.src_rows;
    GL.dst_rows = o.dst_rows;
    GL.row_ready = o.row_ready;
    GL.error_out = p->error;
    GL.tokens = tokens;
    GL.top_k = 1;
    GL.hidden = H;
    GL.inner = I;
    GL.bn = bn;
    GL.ks = 1;  // the plan's item counts have no K split
    GL.ctas = sm_count();
    GL.pairs = pairs;
    if (int rc = launch_grouped(GL, s)) return rc;
    return mark(1);
}

int moe_ep_p2p_finish(const moe_ep_p2p *p, void *stream) {
    if (int rc = check_p2p(p)) return rc;
    return lrb::launch_pdl(lrb::ep_p2p_finish_kernel, dim3(1), dim3(64), 0, static_cast<cudaStream_t>(stream),
                           "ep_p2p_finish_kernel", args_of(p));
}

}  // extern "C"
