// Router: BF16 logits GEMV/GEMM + softmax/top-k/renormalise, and the sigmoid
// shared-expert gate (transformers qwen3_5_moe modeling :762-770, :779, :788).
#include <algorithm>
#include <climits>

#include "common.cuh"
#include "kernels.cuh"
#include "plan.cuh"
#include "routing.cuh"

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

// One warp per token: softmax / top-k / renormalise of routing.cuh warp_topk,
// and (gate_w != null) the shared-expert gate sig = bf16(sigmoid(bf16(x . w)))
// (modeling_qwen3_5_moe :779, :788), FP32 lane partials summed by warp_sum.
template <int VPL>
__global__ void __launch_bounds__(256) router_select_kernel(const uint16_t *__restrict__ logits,
                                                            const float *__restrict__ bias, int tokens,
                                                            int experts, int top_k, int64_t *__restrict__ idx,
                                                            float *__restrict__ scores_f32,
                                                            uint16_t *__restrict__ scores_bf16,
                                                            const uint16_t *__restrict__ x,
                                                            const uint16_t *__restrict__ gate_w, int hidden,
                                                            uint16_t *__restrict__ sig,
                                                            const float *__restrict__ part, int ks) {
    grid_dependency_wait();
    grid_dependency_trigger();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    int e;
    float w;
    select_token<VPL>(t, logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, x, gate_w, hidden, sig,
                      part, ks, &e, &w);
}

// Decode widths: every (row, K quarter) pair is one warp over all tokens, so
// ~130 CTAs share the 1 MiB router read.  Each CTA stages its K quarter of up
// to 16 token rows in shared memory with all loads in flight at once (one L2
// round trip instead of one per token), the warps' router rows having been
// requested before the wait on the previous kernel.  FP32 partials go to
// part[ks][t][row] (row E = shared-expert gate); the routing kernel sums the
// quarters in a fixed order.
template <int NW>
__global__ void __launch_bounds__(256) router_split_kernel(const uint16_t *__restrict__ x,
                                                           const uint16_t *__restrict__ router,
                                                           const uint16_t *__restrict__ gate_w, int tokens,
                                                           int experts, float *__restrict__ part,
                                                           int32_t *__restrict__ zero_words, int n_zero) {
    constexpr int H = NW * 256 * kRouterSplit;
    constexpr int kUnits = NW * 32;                 // 16-byte units of one token's K quarter
    constexpr int kTB = 16;                         // tokens staged per round
    constexpr int kPer = kTB * kUnits / 256;        // staging loads per thread
    __shared__ uint4 xs[kTB][kUnits];
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int ks = blockIdx.y;
    const int rows = experts + (gate_w != nullptr);
    const bool active = row < rows;
    grid_dependency_trigger();
    uint4 w[NW];
    if (active) {
        const uint16_t *wrow =
            (row < experts ? router + static_cast<size_t>(row) * H : gate_w) + ks * (H / kRouterSplit);
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = ld_stream(wrow + (lane + 32 * i) * 8);
    }
    grid_dependency_wait();  // x may come from the previous kernel
    if (zero_words && blockIdx.x == 0 && blockIdx.y == 0 && static_cast<int>(threadIdx.x) < n_zero)
        zero_words[threadIdx.x] = 0;
    for (int t0 = 0; t0 < tokens; t0 += kTB) {
        const int nt = min(kTB, tokens - t0);
        uint4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * 256, t = min(i / kUnits, nt - 1);
            v[u] = ld_cached(x + static_cast<size_t>(t0 + t) * H + ks * (H / kRouterSplit) + (i % kUnits) * 8);
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * 256;
            xs[i / kUnits][i % kUnits] = v[u];
        }
        __syncthreads();
        if (active) {
            float acc[kTB];
#pragma unroll
            for (int j = 0; j < kTB; ++j) {
                acc[j] = 0.f;
#pragma unroll
                for (int i = 0; i < NW; ++i) acc[j] = dot8(w[i], xs[j][lane + 32 * i], acc[j]);
            }
#pragma unroll
            for (int j = 0; j < kTB; ++j) acc[j] = warp_sum(acc[j]);
            float out = acc[0];
#pragma unroll
            for (int j = 1; j < kTB; ++j)
                if (lane == j) out = acc[j];
            if (lane < nt) part[(static_cast<size_t>(ks) * tokens + t0 + lane) * (experts + 1) + row] = out;
        }
        __syncthreads();
    }
}

// One CTA: logits (sum of the quarters, rounded once to BF16 -- F.linear),
// shared-expert gate, per-token top-k, the eager-order permute and the grouped
// kernel's plan.  With route_in the selection is skipped.
template <int VPL>
__global__ void __launch_bounds__(1024) route_decode_kernel(DecodeRouteArgs r, PlanArgs plan) {
    extern __shared__ float dyn[];
    __shared__ int scratch[100];
    const int T = r.tokens, E = r.experts, K = r.top_k;
    float *z = dyn;                                                   // [T][E]
    int32_t *sidx = reinterpret_cast<int32_t *>(z + T * E);           // [T][K]
    int32_t *cnt = sidx + T * K;                                      // permute scratch
    grid_dependency_wait();
    grid_dependency_trigger();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (!r.route_in) {
        // Thread (g, e): column e < E of tokens g, g + G, ...; four tokens per
        // round with all their partial loads in flight (no division: the
        // column width CW is a power of two).  Threads t < T also sum the
        // shared-expert gate column E of token t.
        constexpr int CW = 32 * VPL;
        const int cols = E + 1, G = blockDim.x / CW;
        const int e = threadIdx.x % CW, g = threadIdx.x / CW;
        const bool gate_thread = r.has_gate && static_cast<int>(threadIdx.x) < T;
        float gp[kRouterSplit];
        if (gate_thread) {
#pragma unroll
            for (int k = 0; k < kRouterSplit; ++k) gp[k] = r.part[(static_cast<size_t>(k) * T + threadIdx.x) * cols + E];
        }
        if (e < E) {
            const float be = r.bias ? r.bias[e] : 0.0f;
            for (int t0 = g; t0 < T; t0 += 4 * G) {
                float p[4][kRouterSplit];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = min(t0 + u * G, T - 1);
#pragma unroll
                    for (int k = 0; k < kRouterSplit; ++k) p[u][k] = r.part[(static_cast<size_t>(k) * T + t) * cols + e];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int t = t0 + u * G;
                    if (t >= T) break;
                    float sum = 0.f;
#pragma unroll
                    for (int k = 0; k < kRouterSplit; ++k) sum += p[u][k];
                    const uint16_t lg = f2bf(sum);
                    r.logits[static_cast<size_t>(t) * E + e] = lg;
                    z[t * E + e] = bf2f(lg) + be;
                }
            }
        }
        if (gate_thread) {
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < kRouterSplit; ++k) sum += gp[k];
            r.sig[threadIdx.x] = f2bf(sigmoid_f32(bf2f(f2bf(sum))));
        }
        __syncthreads();
        for (int t = warp; t < T; t += blockDim.x >> 5) {
            int e;
            float w;
            const float *zr = z + t * E;
            warp_topk<VPL>([&](int j) { return zr[j]; }, E, K, &e, &w);
            if (lane < K) {
                sidx[t * K + lane] = e;
                r.idx[static_cast<size_t>(t) * K + lane] = e;
                r.scores[static_cast<size_t>(t) * K + lane] = f2bf(w);
            }
        }
    } else {
        for (int i = threadIdx.x; i < T * K; i += blockDim.x) sidx[i] = static_cast<int32_t>(r.route_in[i]);
    }
    __syncthreads();
    route_plan_block([&](int t, int k) -> int64_t { return sidx[t * K + k]; }, T, K, E, r.offsets, r.perm_token,
                     r.perm_slot, r.route_pos, r.active, r.num_active, r.bad_routes, plan, cnt, scratch);
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
                         int64_t *idx, float *scores_f32, uint16_t *scores_bf16, cudaStream_t stream,
                         const uint16_t *x, const uint16_t *gate_w, int hidden, uint16_t *sig, const float *part,
                         int ks) {
    const int grid = (tokens + 7) / 8;
    if (gate_w && (!x || !sig || hidden % 256)) return set_error(MOE_EINVAL, "router: bad shared-gate arguments");
    if (experts <= 256)
        return launch_pdl(router_select_kernel<8>, dim3(grid), dim3(256), 0, stream, "router_select_kernel", logits,
                          bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, x, gate_w, hidden, sig, part,
                          ks);
    if (experts <= 1024)
        return launch_pdl(router_select_kernel<32>, dim3(grid), dim3(256), 0, stream, "router_select_kernel", logits,
                          bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, x, gate_w, hidden, sig, part,
                          ks);
    return set_error(MOE_EINVAL, "router: experts %d > 1024", experts);
}

int launch_router_split(const uint16_t *x, const uint16_t *router, const uint16_t *gate_w, int tokens, int hidden,
                        int experts, float *part, cudaStream_t stream, int32_t *zero_words, int n_zero) {
    const int rows = experts + (gate_w != nullptr);
    const dim3 grid((rows + 7) / 8, kRouterSplit);
    switch (hidden) {
        case 2048:
            return launch_pdl(router_split_kernel<2>, grid, dim3(256), 0, stream, "router_split_kernel", x, router,
                              gate_w, tokens, experts, part, zero_words, n_zero);
        case 1024:
            return launch_pdl(router_split_kernel<1>, grid, dim3(256), 0, stream, "router_split_kernel", x, router,
                              gate_w, tokens, experts, part, zero_words, n_zero);
        case 4096:
            return launch_pdl(router_split_kernel<4>, grid, dim3(256), 0, stream, "router_split_kernel", x, router,
                              gate_w, tokens, experts, part, zero_words, n_zero);
        default:
            return set_error(MOE_EINVAL, "router: hidden %d not in {1024, 2048, 4096}", hidden);
    }
}

int route_decode_smem(int tokens, int experts, int top_k) {
    return static_cast<int>(sizeof(float) * tokens * experts + sizeof(int32_t) * tokens * top_k +
                            sizeof(int32_t) * std::max(33 * experts, 1024));
}

int launch_route_decode(const DecodeRouteArgs &r, const PlanArgs &plan, cudaStream_t stream) {
    LRB_REQUIRE(r.tokens <= kDecodeMaxTokens, "route_decode: tokens %d > %d", r.tokens, kDecodeMaxTokens);
    const int smem = route_decode_smem(r.tokens, r.experts, r.top_k);
    const int v = r.experts <= 256 ? 0 : 1;
    {
        const int most = route_decode_smem(kDecodeMaxTokens, v ? 1024 : 256, 32);
        const int rc = v == 0 ? ensure_dynamic_smem(route_decode_kernel<8>, most, "cudaFuncSetAttribute(route_decode)")
                              : ensure_dynamic_smem(route_decode_kernel<32>, most, "cudaFuncSetAttribute(route_decode)");
        if (rc) return rc;
    }
    if (v == 0)
        return launch_pdl(route_decode_kernel<8>, dim3(1), dim3(1024), smem, stream, "route_decode_kernel", r, plan);
    return launch_pdl(route_decode_kernel<32>, dim3(1), dim3(1024), smem, stream, "route_decode_kernel", r, plan);
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
    LRB_REQUIRE(router && (tokens == 0 || (x && logits && idx)),
                "moe_router_topk: x, router, logits and idx are required");
    LRB_REQUIRE(!shared_gate_w || sig, "moe_router_topk: shared_gate_w needs a sig output");
    if (tokens == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    cudaStream_t s = lrb::as_stream(stream);
    if (tokens > lrb::kDecodeMaxTokens) {
        // prefill widths: tensor-core logits, then selection + shared gate
        if (int rc = lrb::launch_router_tc(x, router, tokens, hidden, experts, logits, nullptr, 1, nullptr, s))
            return rc;
        return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, s, x,
                                         shared_gate_w, hidden, sig);
    }
    if (int rc = lrb::launch_router_logits(x, router, shared_gate_w, tokens, hidden, experts, logits, sig, s))
        return rc;
    return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, s);
}

size_t moe_router_workspace_bytes(int tokens, int experts) {
    if (tokens <= lrb::kDecodeMaxTokens || experts <= 0) return 0;
    const int ks = lrb::router_tc_splits(tokens, experts);
    return ks > 1 ? static_cast<size_t>(ks) * tokens * experts * sizeof(float) : 0;
}

int moe_router_topk_ws(const uint16_t *x, const uint16_t *router, const float *bias, const uint16_t *shared_gate_w,
                       int tokens, int hidden, int experts, int top_k, uint16_t *logits, int64_t *idx,
                       float *scores_f32, uint16_t *scores_bf16, uint16_t *sig, void *workspace,
                       size_t workspace_bytes, void *stream) {
    const size_t need = moe_router_workspace_bytes(tokens, experts);
    if (need == 0 || !workspace || workspace_bytes < need)
        return moe_router_topk(x, router, bias, shared_gate_w, tokens, hidden, experts, top_k, logits, idx,
                               scores_f32, scores_bf16, sig, stream);
    if (int rc = lrb::check_router_args(tokens, hidden, experts, top_k)) return rc;
    LRB_REQUIRE(x && router && logits && idx, "moe_router_topk_ws: x, router, logits and idx are required");
    LRB_REQUIRE(!shared_gate_w || sig, "moe_router_topk_ws: shared_gate_w needs a sig output");
    if (int rc = lrb::require_sm100()) return rc;
    cudaStream_t s = lrb::as_stream(stream);
    const int ks = lrb::router_tc_splits(tokens, experts);
    float *part = static_cast<float *>(workspace);
    if (int rc = lrb::launch_router_tc(x, router, tokens, hidden, experts, logits, part, ks, nullptr, s)) return rc;
    return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16, s, x,
                                     shared_gate_w, hidden, sig, part, ks);
}

int moe_router_select(const uint16_t *logits, const float *bias, int tokens, int experts, int top_k, int64_t *idx,
                      float *scores_f32, uint16_t *scores_bf16, void *stream) {
    if (int rc = lrb::check_router_args(tokens, 2048, experts, top_k)) return rc;
    LRB_REQUIRE(tokens == 0 || (logits && idx), "moe_router_select: logits and idx are required");
    if (tokens == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    return lrb::launch_router_select(logits, bias, tokens, experts, top_k, idx, scores_f32, scores_bf16,
                                     lrb::as_stream(stream));
}

}  // extern "C"
