// Expert-parallel dispatch and combine around the NCCL all-to-all exchange.
//
// Rank r owns the experts [r*El, (r+1)*El).  After the local router and the
// eager permute (ascending expert, slot-major, token), route position p of the
// home rank belongs to the rank owning its expert, and the positions of one
// destination rank are contiguous -- so the permuted order is also the send
// order, and the per-destination counts are differences of the permute's
// expert offsets.
//
//   dispatch  send_rows[p] = x[perm_token[p]]; send_meta[p] = local expert id
//             << 16 | BF16 routing weight; send_counts[d] = routes owned by d.
//   unpack    the receiver's (local expert, weight) pairs as the route_in /
//             weights_in of a one-slot moe_layer_forward, whose ordered combine
//             returns bf16(y * w) per received row.
//   combine   out[t] = the eager fold over t's routes in ascending position
//             (= ascending global expert, then slot), each already weighted,
//             then + the gated shared-expert row: bf16 after every add, the
//             rounding order of Qwen3_5MoeExperts.forward (modeling_qwen3_5_moe
//             :749-750) and Qwen3_5MoeSparseMoeBlock.forward (:788-790).
//
// The reference runs its MoE layer on one GPU; these kernels have no
// counterpart there.
#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

// One warp per route position: 16-byte row copy plus the metadata word.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const uint16_t *__restrict__ x, const int64_t *__restrict__ idx, const uint16_t *__restrict__ scores,
    const int32_t *__restrict__ offsets, const int32_t *__restrict__ perm_token,
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
        if (lane == 0) {
            const int e = static_cast<int>(idx[static_cast<size_t>(t) * top_k + k]);
            send_meta[p] = ((e % local_experts) << 16) | scores[static_cast<size_t>(t) * top_k + k];
        }
    }
}

__global__ void ep_unpack_kernel(const int32_t *__restrict__ meta, int rows, int64_t *__restrict__ route_in,
                                 uint16_t *__restrict__ weights_in) {
    grid_dependency_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
        const uint32_t m = static_cast<uint32_t>(meta[i]);
        route_in[i] = m >> 16;
        weights_in[i] = static_cast<uint16_t>(m & 0xFFFFu);
    }
}

// One thread per (token, 8 columns).
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint16_t *__restrict__ ret,
                                                         const int32_t *__restrict__ route_pos,
                                                         const uint16_t *__restrict__ shared_rows, int tokens,
                                                         int top_k, int hidden, uint16_t *__restrict__ out) {
    grid_dependency_wait();
    const int chunks = hidden / 8;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= tokens * chunks) return;
    const int t = i / chunks, c = (i % chunks) * 8;
    int pos[32];
    for (int k = 0; k < top_k; ++k) pos[k] = route_pos[static_cast<size_t>(t) * top_k + k];
    for (int a = 1; a < top_k; ++a)
        for (int b = a; b > 0 && pos[b] < pos[b - 1]; --b) {
            const int tp = pos[b];
            pos[b] = pos[b - 1];
            pos[b - 1] = tp;
        }
    float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < top_k; ++k) {
        if (pos[k] < 0) continue;
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(ret + static_cast<size_t>(pos[k]) * hidden + c));
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            o8[2 * h] = rbf(o8[2 * h] + bf16_lo(vw[h]));
            o8[2 * h + 1] = rbf(o8[2 * h + 1] + bf16_hi(vw[h]));
        }
    }
    if (shared_rows) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(shared_rows + static_cast<size_t>(t) * hidden + c));
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            o8[2 * h] = rbf(o8[2 * h] + bf16_lo(vw[h]));
            o8[2 * h + 1] = rbf(o8[2 * h + 1] + bf16_hi(vw[h]));
        }
    }
    uint4 o;
    o.x = pack_bf16x2(o8[0], o8[1]);
    o.y = pack_bf16x2(o8[2], o8[3]);
    o.z = pack_bf16x2(o8[4], o8[5]);
    o.w = pack_bf16x2(o8[6], o8[7]);
    *reinterpret_cast<uint4 *>(out + static_cast<size_t>(t) * hidden + c) = o;
}

}  // namespace lrb

extern "C" int moe_ep_dispatch(const uint16_t *x, const int64_t *idx, const uint16_t *scores, const int32_t *offsets,
                               const int32_t *perm_token, const int32_t *perm_slot, int tokens, int top_k,
                               int experts, int hidden, int world, uint16_t *send_rows, int32_t *send_meta,
                               int64_t *send_counts, void *stream) {
    LRB_REQUIRE(x && idx && scores && offsets && perm_token && perm_slot && send_rows && send_meta && send_counts,
                "moe_ep_dispatch: null pointer");
    LRB_REQUIRE(world >= 1 && world <= 256 && experts % world == 0 && experts / world <= 32768,
                "moe_ep_dispatch: %d experts do not shard over %d ranks", experts, world);
    LRB_REQUIRE(hidden > 0 && hidden % 8 == 0 && tokens >= 0 && top_k >= 1 && top_k <= 32,
                "moe_ep_dispatch: bad shape");
    const int routes = tokens * top_k;
    const int blocks = std::max(1, std::min((routes + 7) / 8, lrb::sm_count() * 8));
    return lrb::launch_pdl(lrb::ep_dispatch_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                           "ep_dispatch_kernel", x, idx, scores, offsets, perm_token, perm_slot, top_k, experts,
                           hidden, world, experts / world, send_rows, send_meta, send_counts);
}

extern "C" int moe_ep_unpack(const int32_t *meta, int rows, int64_t *route_in, uint16_t *weights_in, void *stream) {
    LRB_REQUIRE(rows >= 0 && (rows == 0 || (meta && route_in && weights_in)), "moe_ep_unpack: bad arguments");
    if (rows == 0) return MOE_OK;
    const int blocks = std::min((rows + 255) / 256, lrb::sm_count() * 4);
    return lrb::launch_pdl(lrb::ep_unpack_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                           "ep_unpack_kernel", meta, rows, route_in, weights_in);
}

extern "C" int moe_ep_combine(const uint16_t *ret, const int32_t *route_pos, const uint16_t *shared_rows,
                              int tokens, int top_k, int hidden, uint16_t *out, void *stream) {
    LRB_REQUIRE(ret && route_pos && out, "moe_ep_combine: null pointer");
    LRB_REQUIRE(hidden > 0 && hidden % 8 == 0 && tokens >= 0 && top_k >= 1 && top_k <= 32,
                "moe_ep_combine: bad shape");
    if (tokens == 0) return MOE_OK;
    const int threads = tokens * (hidden / 8);
    return lrb::launch_pdl(lrb::ep_combine_kernel, dim3((threads + 255) / 256), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), "ep_combine_kernel", ret, route_pos, shared_rows, tokens,
                           top_k, hidden, out);
}
