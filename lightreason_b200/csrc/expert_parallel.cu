// Expert-parallel dispatch and combine around the NCCL all-to-all exchange.
//
// Rank r owns the experts [r*El, (r+1)*El).  After the local router and the
// eager permute (ascending expert, slot-major, token), route position p of the
// home rank belongs to the rank owning its expert, and the positions of one
// destination rank are contiguous -- so the permuted order is also the send
// order, and the per-destination counts are differences of the permute's
// expert offsets.
//
//   dispatch  send_rows[p] = x[perm_token[p]]; send_meta[p] = the local
//             expert id on the owning rank; send_counts[d] = routes owned by d.
//   unpack    the received ids as the route_in of a one-slot moe_layer_forward
//             in rows mode, which returns the unweighted row y per received row.
//   combine   the layer's own ordered combine over the returned rows in the
//             home rank's permuted order: bf16(acc + bf16(y * w)) in ascending
//             position (= ascending global expert, then slot), then the gated
//             shared-expert row -- the rounding order of
//             Qwen3_5MoeExperts.forward (modeling_qwen3_5_moe :749-750) and
//             Qwen3_5MoeSparseMoeBlock.forward (:788-790).
//
// The reference runs its MoE layer on one GPU; these kernels have no
// counterpart there.
#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

// One warp per route position: 16-byte row copy plus the expert id.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const uint16_t *__restrict__ x, const int64_t *__restrict__ idx, const int32_t *__restrict__ offsets, const int32_t *__restrict__ perm_token,
    const int32_t *__restrict__ perm_slot, int top_k, int experts, int hidden, int world, int local_experts,
    uint16_t *__restrict__ send_rows, int32_t *__restrict__ send_meta, int64_t *__restrict__ send_counts) {
    grid_dependency_wait();
    if (blockIdx.x == 0 && threadIdx.x < world) {
        const int d = threadIdx.x;
        const int lo = min(d * local_experts, experts), hi = min((d + 1) * local_experts, experts);
        send_counts[d] = offsets[hi] - offsets[lo];
    }
    const int routes = offsets[experts];
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int vecs = hidden / 8;
    for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < routes; p += warps) {
        const int t = perm_token[p], k = perm_slot[p];
        const uint4 *src = reinterpret_cast<const uint4 *>(x + static_cast<size_t>(t) * hidden);
        uint4 *dst = reinterpret_cast<uint4 *>(send_rows + static_cast<size_t>(p) * hidden);
        for (int v = lane; v < vecs; v += 32) dst[v] = __ldg(src + v);
        if (lane == 0) send_meta[p] = static_cast<int>(idx[static_cast<size_t>(t) * top_k + k]) % local_experts;
    }
}

__global__ void ep_unpack_kernel(const int32_t *__restrict__ meta, int rows, int64_t *__restrict__ route_in) {
    grid_dependency_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) route_in[i] = meta[i];
}

}  // namespace lrb

extern "C" int moe_ep_dispatch(const uint16_t *x, const int64_t *idx, const int32_t *offsets,
                               const int32_t *perm_token, const int32_t *perm_slot, int tokens, int top_k,
                               int experts, int hidden, int world, uint16_t *send_rows, int32_t *send_meta,
                               int64_t *send_counts, void *stream) {
    LRB_REQUIRE(x && idx && offsets && perm_token && perm_slot && send_rows && send_meta && send_counts,
                "moe_ep_dispatch: null pointer");
    LRB_REQUIRE(world >= 1 && world <= 256 && experts % world == 0 && experts / world <= 32768,
                "moe_ep_dispatch: %d experts do not shard over %d ranks", experts, world);
    LRB_REQUIRE(hidden > 0 && hidden % 8 == 0 && tokens >= 0 && top_k >= 1 && top_k <= 32,
                "moe_ep_dispatch: bad shape");
    const int routes = tokens * top_k;
    const int blocks = std::max(1, std::min((routes + 7) / 8, lrb::sm_count() * 8));
    return lrb::launch_pdl(lrb::ep_dispatch_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                           "ep_dispatch_kernel", x, idx, offsets, perm_token, perm_slot, top_k, experts,
                           hidden, world, experts / world, send_rows, send_meta, send_counts);
}

extern "C" int moe_ep_unpack(const int32_t *meta, int rows, int64_t *route_in, void *stream) {
    LRB_REQUIRE(rows >= 0 && (rows == 0 || (meta && route_in)), "moe_ep_unpack: bad arguments");
    if (rows == 0) return MOE_OK;
    const int blocks = std::min((rows + 255) / 256, lrb::sm_count() * 4);
    return lrb::launch_pdl(lrb::ep_unpack_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                           "ep_unpack_kernel", meta, rows, route_in);
}

extern "C" int moe_ep_combine(const uint16_t *ret, const int32_t *route_pos, const uint16_t *scores,
                              const uint16_t *shared_rows, const uint16_t *sig, int tokens, int top_k, int hidden,
                              uint16_t *out, void *stream) {
    LRB_REQUIRE(ret && route_pos && scores && out && (!shared_rows || sig), "moe_ep_combine: null pointer");
    LRB_REQUIRE(hidden > 0 && hidden % 8 == 0 && tokens >= 0 && top_k >= 1 && top_k <= 16,
                "moe_ep_combine: bad shape");
    return lrb::launch_combine(ret, route_pos, scores, tokens, top_k, hidden, shared_rows, sig, out,
                               static_cast<cudaStream_t>(stream));
}
