// Router: BF16 logits GEMV/GEMM + softmax/top-k/renormalise, and the sigmoid
// shared-expert gate (transformers qwen3_5_moe modeling :762-770, :779, :788).
#include <climits>

#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

// One warp per output row (expert e < E, or the shared-expert gate row e == E)
// and a block of TOKENS_PER_CTA tokens per grid row.  The weight row lives in
// registers (NW 16-byte words per lane); token rows come through L1.  Each
// logit is the FP32 warp sum rounded once to BF16, i.e. F.linear on BF16.
template <int NW>
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t *__restrict__ x,
                                                            const uint16_t *__restrict__ router,
                                                            const uint16_t *__restrict__ gate_w,
                                                            int tokens, int experts, int tokens_per_cta,
                                                            uint16_t *__restrict__ logits,
                                                            uint16_t *__restrict__ sig) {
    constexpr int H = NW * 256;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int rows = experts + (gate_w != nullptr);
    if (row >= rows) return;
    const uint16_t *wrow = row < experts ? router + static_cast<size_t>(row) * H : gate_w;
    uint4 w[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = ld_cached(wrow + (lane + 32 * i) * 8);
    const int t_begin = blockIdx.y * tokens_per_cta;
    const int t_end = min(tokens, t_begin + tokens_per_cta);
    for (int t0 = t_begin; t0 < t_end; t0 += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (t0 + j < t_end) {
                const uint16_t *xr = x + static_cast<size_t>(t0 + j) * H;
#pragma unroll
                for (int i = 0; i < NW; ++i) acc[j] = dot8(w[i], ld_cached(xr + (lane + 32 * i) * 8), acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = warp_sum(acc[j]);
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int t = t0 + j;
                if (t >= t_end) break;
                if (row < experts) {
                    logits[static_cast<size_t>(t) * experts + row] = f2bf(acc[j]);
                } else {
                    sig[t] = f2bf(sigmoid_f32(rbf(acc[j])));
                }
            }
        }
    }
}

// One warp per token.  z = float(bf16 logit) + bias; softmax over z; top_k by z
// descending with exact ties to the lower expert id (softmax is monotonic, so
// this is torch.topk's selection on p); w_k = p_k / sum_k p_k summed in slot
// order.  VPL = logits per lane (experts <= 32 * VPL).
template <int VPL>
__global__ void __launch_bounds__(256) router_select_kernel(const uint16_t *__restrict__ logits,
                                                            const float *__restrict__ bias, int tokens,
                                                            int experts, int top_k, int64_t *__restrict__ idx,
                                                            float *__restrict__ scores_f32,
                                                            uint16_t *__restrict__ scores_bf16) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    float z[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
        const int e = lane + 32 * v;
        z[v] = -INFINITY;
        if (e < experts) {
            z[v] = bf2f(logits[static_cast<size_t>(t) * experts + e]) + (bias ? bias[e] : 0.0f);
            m = fmaxf(m, z[v]);
        }
    }
#pragma unroll
    for (int s = 16; s; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    float denom = 0.0f;
#pragma unroll
    for (int v = 0; v < VPL; ++v)
        if (lane + 32 * v < experts) denom += expf(z[v] - m);
    denom = warp_sum(denom);

    uint32_t taken = 0;
    float my_p = 0.0f;
    int my_e = 0;
    for (int k = 0; k < top_k; ++k) {
        float bz = -INFINITY;
        int be = INT_MAX;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            const int e = lane + 32 * v;
            if (e < experts && !(taken & (1u << v)) && (z[v] > bz || be == INT_MAX)) {
                bz = z[v];
                be = e;
            }
        }
#pragma unroll
        for (int s = 16; s; s >>= 1) {
            const float oz = __shfl_xor_sync(0xffffffffu, bz, s);
            const int oe = __shfl_xor_sync(0xffffffffu, be, s);
            if (oz > bz || (oz == bz && oe < be)) {
                bz = oz;
                be = oe;
            }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == k) {
            my_p = expf(bz - m) / denom;
            my_e = be;
        }
    }
    float sum = 0.0f;
    for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, my_p, k);
    if (lane < top_k) {
        const float w = my_p / sum;
        const size_t o = static_cast<size_t>(t) * top_k + lane;
        idx[o] = my_e;
        if (scores_f32) scores_f32[o] = w;
        if (scores_bf16) scores_bf16[o] = f2bf(w);
    }
}

int launch_router_logits(const uint16_t *x, const uint16_t *router, const uint16_t *gate_w, int tokens,
                         int hidden, int experts, uint16_t *logits, uint16_t *sig, cudaStream_t stream) {
    const int rows = experts + (gate_w != nullptr);
    const int tokens_per_cta = tokens <= 16 ? 16 : 64;
    dim3 grid((rows + 7) / 8, (tokens + tokens_per_cta - 1) / tokens_per_cta);
    switch (hidden) {
        case 2048:
            router_logits_kernel<8><<<grid, 256, 0, stream>>>(x, router, gate_w, tokens, experts, tokens_per_cta,
                                                               logits, sig);
            break;
        case 1024:
            router_logits_kernel<4><<<grid, 256, 0, stream>>>(x, router, gate_w, tokens, experts, tokens_per_cta,
                                                               logits, sig);
            break;
        case 4096:
            router_logits_kernel<16><<<grid, 256, 0, stream>>>(x, router, gate_w, tokens, experts, tokens_per_cta,
                                                                logits, sig);
            break;
        default:
            return set_error(MOE_EINVAL, "router: hidden %d not in {1024, 2048, 4096}", hidden);
    }
    LRB_LAUNCHED("router_logits_kernel");
    return MOE_OK;
}

int launch_router_select(const uint16_t *logits, const float *bias, int tokens, int experts, int top_k,
                         int64_t *idx, float *scores_f32, uint16_t *scores_bf16, cudaStream_t stream) {
    const int grid = (tokens + 7) / 8;
    if (experts <= 256) {
        router_select_kernel<8><<<grid, 256, 0, stream>>>(logits, bias, tokens, experts, top_k, idx, scores_f32,
                                                           scores_bf16);
    } else if (experts <= 1024) {
        router_select_kernel<32><<<grid, 256, 0, stream>>>(logits, bias, tokens, experts, top_k, idx, scores_f32,
                                                            scores_bf16);
    } else {
        return set_error(MOE_EINVAL, "router: experts %d > 1024", experts);
    }
    LRB_LAUNCHED("router_select_kernel");
    return MOE_OK;
}

int check_router_args(int tokens, int hidden, int experts, int top_k) {
    LRB_REQUIRE(tokens >= 0, "router: tokens %d < 0", tokens);
    LRB_REQUIRE(experts >= 1 && experts <= 1024, "router: experts %d outside [1, 1024]", experts);
    LRB_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= experts, "router: top_k %d outside [1, min(32, experts)]",
                top_k);
    LRB_REQUIRE(hidden == 1024 || hidden == 2048 || hidden == 4096, "router: hidden %d not in {1024, 2048, 4096}",
                hidden);
    return MOE_OK;
}

}  // namespace lrb

extern "C" {

int moe_router_topk(const uint16_t *x, const uint16_t *router, const float *bias, const uint16_t *shared_gate_w,
                    int tokens, int hidden, int experts, int top_k, uint16_t *logits, int64_t *idx,
                    float *scores_f32, uint16_t *scores_bf16, uint16_t *sig, void *stream) {
    if (int rc = lrb::check_router_args(tokens, hidden, experts, top_k)) return rc;
    LRB_REQUIRE(x && router && logits && idx, "moe_router_topk: x, router, logits and idx are required");
    LRB_REQUIRE(!shared_gate_w || sig, "moe_router_topk: shared_gate_w needs a sig output");
    if (tokens == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    cudaStream_t s = lrb::as_stream(stream);
    if (int rc = lrb::launch_router_logits(x, router, shared_gate_w, tokens, hidden, experts, logits, sig, s))
        return rc;
    return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, s);
}

int moe_router_select(const uint16_t *logits, const float *bias, int tokens, int experts, int top_k, int64_t *idx,
                      float *scores_f32, uint16_t *scores_bf16, void *stream) {
    if (int rc = lrb::check_router_args(tokens, 2048, experts, top_k)) return rc;
    LRB_REQUIRE(logits && idx, "moe_router_select: logits and idx are required");
    if (tokens == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16,
                                     lrb::as_stream(stream));
}

}  // extern "C"
