// Expert-parallel exchange over NVLink peer memory, without host
// synchronisation: every rank owns one symmetric buffer (same layout on all
// ranks, mapped into every peer by CUDA IPC), and the ranks' kernels meet
// through release/acquire flags in those buffers.
//
// Symmetric buffer of rank q (W ranks, C = capacity rows per source, T0 own
// token rows):
//   flags_dispatch uint32 [W]   step at which rank s finished writing into q
//   flags_return   uint32 [W]   step at which rank d finished returning q's rows
//   count          int32  [W]   rows rank s wrote into q this step
//   meta           int32  [W][C][2]  (local expert on q, position on s)
//   rows           bf16   [T0 + W*C][H]  q's own tokens, then rank s's rows at
//                                        T0 + s*C: the local layer's input
//   ret            bf16   [C][H]     q's own routes' expert rows, by position
//
// One step on rank r (the step number lives in device memory and advances at
// the end of the step, so a captured CUDA graph replays correctly):
//   dispatch  route position p of expert e goes to rank d = e / El, slot
//             j = p - offsets[d * El]: row x[perm_token[p]] -> d.rx[r][j],
//             (e % El, p) -> d.meta[r][j]; the last CTA writes d.count[r] and
//             releases d.flags_dispatch[r] = step.
//   collect   copy the own tokens into rows[0, T); wait for every
//             flags_dispatch[s] == step; route_in of every row = its local
//             expert (own tokens: the shared expert, El; rows no sender wrote:
//             -1, dropped by the layer, whose token gather is the one
//             compaction) and the peer address each received row returns to.
//   return    after the local layer (rows mode): each received row -> its
//             sender's ret[p]; the last CTA releases s.flags_return[r] = step.
//   finish    wait for every flags_return[d] == step, advance the step; the
//             ordered combine then reads ret.
// Every wait is bounded (globaltimer): on timeout the kernel stores an error
// code in *error and returns, so a missing peer cannot hang the GPU.
//
// The reference runs its MoE layer on one GPU; this exchange has no
// counterpart there.
#include "common.cuh"
#include "kernels.cuh"

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

// Last-CTA election: every CTA fences its (peer) stores, then counts itself in.
__device__ __forceinline__ bool last_cta(int32_t *counter) {
    __shared__ int is_last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(counter, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    return is_last != 0;
}

}  // namespace

__global__ void __launch_bounds__(256) ep_p2p_dispatch_kernel(EpP2PArgs a, const uint16_t *__restrict__ x,
                                                              const int64_t *__restrict__ idx,
                                                              const int32_t *__restrict__ offsets,
                                                              const int32_t *__restrict__ perm_token,
                                                              const int32_t *__restrict__ perm_slot) {
    grid_dependency_wait();
    const uint32_t step = *a.step;
    const int lane = threadIdx.x & 31;
    const int routes = offsets[a.experts];
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int El = a.local_experts;
    for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < routes; p += warps) {
        const int t = perm_token[p], k = perm_slot[p];
        const int e = static_cast<int>(idx[static_cast<size_t>(t) * a.top_k + k]);
        const int d = e / El;
        const int j = p - offsets[d * El];
        uint8_t *dst = peer_base(a, d);
        const size_t slot = static_cast<size_t>(a.rank) * a.capacity + j;
        warp_copy_row(x + static_cast<size_t>(t) * a.hidden,
                      reinterpret_cast<uint16_t *>(dst + a.off_rx) + (a.own_rows + slot) * a.hidden, a.hidden, lane);
        if (lane == 0) {
            int32_t *meta = reinterpret_cast<int32_t *>(dst + a.off_meta) + slot * 2;
            meta[0] = e % El;
            meta[1] = p;
        }
    }
    if (last_cta(a.sync + 0)) {
        if (threadIdx.x < a.world) {
            const int d = threadIdx.x;
            uint8_t *dst = peer_base(a, d);
            const int lo = min(d * El, a.experts), hi = min((d + 1) * El, a.experts);
            reinterpret_cast<int32_t *>(dst + a.off_count)[a.rank] = offsets[hi] - offsets[lo];
            __threadfence_system();
            st_release_sys(reinterpret_cast<uint32_t *>(dst + a.off_flags_dispatch) + a.rank, step);
        }
        if (threadIdx.x == 0) a.sync[0] = 0;
    }
}

// route_in [own_rows + W*C] int64 and ret_addr [W*C] int64, both indexed like
// the rows region (the layer's input and output rows).
__global__ void __launch_bounds__(256) ep_p2p_collect_kernel(EpP2PArgs a, const uint16_t *__restrict__ x,
                                                             int tokens, int64_t *__restrict__ route_in,
                                                             int64_t *__restrict__ ret_addr) {
    grid_dependency_wait();
    __shared__ int ok;
    const uint32_t step = *a.step;
    uint8_t *self = peer_base(a, a.rank);
    uint16_t *rows = reinterpret_cast<uint16_t *>(self + a.off_rx);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    // own tokens first: the shared expert's rows (no wait needed)
    for (int t = gw; t < a.own_rows; t += warps) {
        if (t < tokens) warp_copy_row(x + static_cast<size_t>(t) * a.hidden, rows + static_cast<size_t>(t) * a.hidden,
                                      a.hidden, lane);
        if (lane == 0) route_in[t] = t < tokens ? a.local_experts : -1;
    }
    if (threadIdx.x == 0) {
        ok = wait_flags(reinterpret_cast<const uint32_t *>(self + a.off_flags_dispatch), a.world, step);
        if (!ok) atomicExch(a.error, 1);
    }
    __syncthreads();
    if (!ok) return;
    const int32_t *count = reinterpret_cast<const int32_t *>(self + a.off_count);
    const int32_t *meta = reinterpret_cast<const int32_t *>(self + a.off_meta);
    const int slots = a.world * a.capacity;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < slots; i += gridDim.x * blockDim.x) {
        const int q = i / a.capacity, j = i - q * a.capacity;
        if (j < count[q]) {
            route_in[a.own_rows + i] = meta[static_cast<size_t>(i) * 2];
            ret_addr[i] = a.peers[q] + a.off_ret + static_cast<int64_t>(meta[static_cast<size_t>(i) * 2 + 1]) *
                                                       a.hidden * 2;
        } else {
            route_in[a.own_rows + i] = -1;
        }
    }
}

// rows [W*C, H]: the local layer's unweighted rows of the received slots
// (the layer's output rows past the own tokens).
__global__ void __launch_bounds__(256) ep_p2p_return_kernel(EpP2PArgs a, const uint16_t *__restrict__ rows,
                                                            const int64_t *__restrict__ ret_addr) {
    grid_dependency_wait();
    const uint32_t step = *a.step;
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int32_t *count = reinterpret_cast<const int32_t *>(peer_base(a, a.rank) + a.off_count);
    if (*a.error == 0) {
        const int slots = a.world * a.capacity;
        for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < slots; i += warps) {
            const int q = i / a.capacity, j = i - q * a.capacity;
            if (j < count[q])
                warp_copy_row(rows + static_cast<size_t>(i) * a.hidden, reinterpret_cast<uint16_t *>(ret_addr[i]),
                              a.hidden, lane);
        }
    }
    if (last_cta(a.sync + 1)) {
        if (threadIdx.x < a.world) {
            uint8_t *src = peer_base(a, threadIdx.x);
            st_release_sys(reinterpret_cast<uint32_t *>(src + a.off_flags_return) + a.rank, step);
        }
        if (threadIdx.x == 0) a.sync[1] = 0;
    }
}

__global__ void ep_p2p_finish_kernel(EpP2PArgs a) {
    grid_dependency_wait();
    const uint32_t step = *a.step;
    uint8_t *self = peer_base(a, a.rank);
    if (threadIdx.x == 0) {
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
    LRB_REQUIRE(p->experts % p->world == 0 && p->local_experts == p->experts / p->world,
                "ep_p2p: %d experts do not shard over %d ranks", p->experts, p->world);
    LRB_REQUIRE(p->hidden > 0 && p->hidden % 8 == 0 && p->capacity > 0 && p->top_k >= 1, "ep_p2p: bad shape");
    return MOE_OK;
}

lrb::EpP2PArgs args_of(const moe_ep_p2p *p) {
    lrb::EpP2PArgs a{};
    a.peers = p->peers;
    a.off_flags_dispatch = p->off_flags_dispatch;
    a.off_flags_return = p->off_flags_return;
    a.off_count = p->off_count;
    a.off_meta = p->off_meta;
    a.off_rx = p->off_rx;
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

    return a;
}

int copy_grid() { return lrb::sm_count() * 2; }

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

int moe_ep_p2p_dispatch(const moe_ep_p2p *p, const uint16_t *x, const int64_t *idx, const int32_t *offsets,
                        const int32_t *perm_token, const int32_t *perm_slot, void *stream) {
    if (int rc = check_p2p(p)) return rc;
    LRB_REQUIRE(x && idx && offsets && perm_token && perm_slot, "moe_ep_p2p_dispatch: null input");
    return lrb::launch_pdl(lrb::ep_p2p_dispatch_kernel, dim3(copy_grid()), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), "ep_p2p_dispatch_kernel", args_of(p), x, idx, offsets,
                           perm_token, perm_slot);
}

int moe_ep_p2p_collect(const moe_ep_p2p *p, const uint16_t *x, int tokens, int64_t *route_in, int64_t *ret_addr,
                       void *stream) {
    if (int rc = check_p2p(p)) return rc;
    LRB_REQUIRE(x && route_in && ret_addr && tokens >= 0 && tokens <= p->own_rows,
                "moe_ep_p2p_collect: bad input (tokens %d, own rows %d)", tokens, p->own_rows);
    return lrb::launch_pdl(lrb::ep_p2p_collect_kernel, dim3(copy_grid()), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), "ep_p2p_collect_kernel", args_of(p), x, tokens,
                           route_in, ret_addr);
}

int moe_ep_p2p_return(const moe_ep_p2p *p, const uint16_t *rows, const int64_t *ret_addr, void *stream) {
    if (int rc = check_p2p(p)) return rc;
    LRB_REQUIRE(rows && ret_addr, "moe_ep_p2p_return: null input");
    return lrb::launch_pdl(lrb::ep_p2p_return_kernel, dim3(copy_grid()), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), "ep_p2p_return_kernel", args_of(p), rows, ret_addr);
}

int moe_ep_p2p_finish(const moe_ep_p2p *p, void *stream) {
    if (int rc = check_p2p(p)) return rc;
    return lrb::launch_pdl(lrb::ep_p2p_finish_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                           "ep_p2p_finish_kernel", args_of(p));
}

}  // extern "C"
