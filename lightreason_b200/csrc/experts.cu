// Expert projections at decode and small-batch widths, and the ordered combine.
//
// gate/up: one warp per (group, row r): the gate row r and up row r of the
// group's expert stay in registers (16-byte streaming loads), and every routed
// token is dotted against both; bf16(gate), bf16(up), bf16(silu), bf16(s*u)
// are the eager rounding points (modeling_qwen3_5_moe.py:745-746,
// edge35b/cpu_experts.c:59-62).  down: one warp per (group, output row) over
// the group's activation rows (:747, cpu_experts.c:68).  The weight stream
// dominates (6 MiB per expert), so each weight byte is loaded exactly once.
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

template <int NW, class Src>
__global__ void __launch_bounds__(256) gate_up_kernel(const Src src, const uint16_t *__restrict__ x, int inner,
                                                      uint16_t *__restrict__ act) {
    constexpr int H = NW * 256;
    const int g = blockIdx.y;
    if (g >= src.n()) return;
    const Group G = src.get(g);
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= inner || G.count <= 0) return;
    uint4 wg[NW], wu[NW];
    const uint16_t *gr = G.gate + static_cast<size_t>(row) * H;
    const uint16_t *ur = G.up + static_cast<size_t>(row) * H;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
        wg[i] = ld_stream(gr + (lane + 32 * i) * 8);
        wu[i] = ld_stream(ur + (lane + 32 * i) * 8);
    }
    for (int j0 = 0; j0 < G.count; j0 += 4) {
        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j0 + j < G.count) {
                const uint16_t *xr = x + static_cast<size_t>(src.token(G.begin + j0 + j)) * H;
#pragma unroll
                for (int i = 0; i < NW; ++i) {
                    const uint4 a = ld_cached(xr + (lane + 32 * i) * 8);
                    ag[j] = dot8(wg[i], a, ag[j]);
                    au[j] = dot8(wu[i], a, au[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ag[j] = warp_sum(ag[j]);
            au[j] = warp_sum(au[j]);
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j0 + j >= G.count) break;
                const float gv = rbf(ag[j]), uv = rbf(au[j]);
                const float s = rbf(silu_f32(gv));
                act[static_cast<size_t>(G.begin + j0 + j) * inner + row] = f2bf(s * uv);
            }
        }
    }
}

template <int NI, class Src>
__global__ void __launch_bounds__(256) down_kernel(const Src src, const uint16_t *__restrict__ act, int hidden,
                                                   uint16_t *__restrict__ y) {
    constexpr int I = NI * 256;
    const int g = blockIdx.y;
    if (g >= src.n()) return;
    const Group G = src.get(g);
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= hidden || G.count <= 0) return;
    uint4 wd[NI];
    const uint16_t *dr = G.down + static_cast<size_t>(row) * I;
#pragma unroll
    for (int i = 0; i < NI; ++i) wd[i] = ld_stream(dr + (lane + 32 * i) * 8);
    for (int j0 = 0; j0 < G.count; j0 += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j0 + j < G.count) {
                const uint16_t *ar = act + static_cast<size_t>(G.begin + j0 + j) * I;
#pragma unroll
                for (int i = 0; i < NI; ++i) acc[j] = dot8(wd[i], ld_cached(ar + (lane + 32 * i) * 8), acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = warp_sum(acc[j]);
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j0 + j >= G.count) break;
                y[static_cast<size_t>(G.begin + j0 + j) * hidden + row] = f2bf(acc[j]);
            }
        }
    }
}

template <class Src>
int launch_experts(const Src &src, int max_groups, const uint16_t *x, int hidden, int inner, uint16_t *act,
                   uint16_t *y, cudaStream_t stream, cudaEvent_t between) {
    if (max_groups <= 0) return MOE_OK;
    const dim3 gu_grid((inner + 7) / 8, max_groups), dn_grid((hidden + 7) / 8, max_groups);
    if (hidden == 2048) gate_up_kernel<8, Src><<<gu_grid, 256, 0, stream>>>(src, x, inner, act);
    else if (hidden == 1024) gate_up_kernel<4, Src><<<gu_grid, 256, 0, stream>>>(src, x, inner, act);
    else if (hidden == 4096) gate_up_kernel<16, Src><<<gu_grid, 256, 0, stream>>>(src, x, inner, act);
    else return set_error(MOE_EINVAL, "experts: hidden %d not in {1024, 2048, 4096}", hidden);
    LRB_LAUNCHED("gate_up_kernel");
    if (between) LRB_CUDA(cudaEventRecord(between, stream));
    if (inner == 512) down_kernel<2, Src><<<dn_grid, 256, 0, stream>>>(src, act, hidden, y);
    else if (inner == 256) down_kernel<1, Src><<<dn_grid, 256, 0, stream>>>(src, act, hidden, y);
    else if (inner == 1024) down_kernel<4, Src><<<dn_grid, 256, 0, stream>>>(src, act, hidden, y);
    else return set_error(MOE_EINVAL, "experts: inner %d not in {256, 512, 1024}", inner);
    LRB_LAUNCHED("down_kernel");
    return MOE_OK;
}

template int launch_experts<DeviceGroups>(const DeviceGroups &, int, const uint16_t *, int, int, uint16_t *,
                                          uint16_t *, cudaStream_t, cudaEvent_t);
template int launch_experts<ParamGroups>(const ParamGroups &, int, const uint16_t *, int, int, uint16_t *,
                                         uint16_t *, cudaStream_t, cudaEvent_t);

// Per token: the routed contributions in ascending route position (= ascending
// expert id), acc = bf16(acc + bf16(y * w)) as index_add_ on BF16 does
// (modeling_qwen3_5_moe.py:749-750; edge35b/fused_experts.py:27-37), then the
// gated shared expert, acc = bf16(acc + bf16(sig * shared)) (:788-790).
// One thread per (token, 8 columns): a warp covers 256 columns of one token,
// and every thread issues all of its row loads before the ordered sums.  KMAX
// (8 or 16) bounds top_k; MINB CTAs stay resident on an SM without spills.
template <int KMAX, int MINB>
__global__ void __launch_bounds__(256, MINB) combine_kernel(const uint16_t *__restrict__ y,
                                                      const int32_t *__restrict__ route_pos,
                                                      const uint16_t *__restrict__ scores, int tokens, int top_k,
                                                      int hidden, const uint16_t *__restrict__ shared_y,
                                                      const uint16_t *__restrict__ sig, uint16_t *__restrict__ out) {
    grid_dependency_wait();
    const int chunks = hidden / 8;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(tokens) * chunks) return;
    const int t = static_cast<int>(i / chunks), c = static_cast<int>(i % chunks) * 8;
    int pos[KMAX];
    uint16_t wt[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        pos[k] = k < top_k ? __ldg(route_pos + static_cast<size_t>(t) * top_k + k) : -1;
        wt[k] = k < top_k ? __ldg(scores + static_cast<size_t>(t) * top_k + k) : 0;
    }
#pragma unroll
    for (int a = 1; a < KMAX; ++a) {
#pragma unroll
        for (int b = a; b > 0; --b) {
            // -1 (no route) sorts last
            const bool swap = static_cast<unsigned>(pos[b]) < static_cast<unsigned>(pos[b - 1]);
            const int p0 = pos[b - 1], p1 = pos[b];
            const uint16_t w0 = wt[b - 1], w1 = wt[b];
            pos[b - 1] = swap ? p1 : p0;
            pos[b] = swap ? p0 : p1;
            wt[b - 1] = swap ? w1 : w0;
            wt[b] = swap ? w0 : w1;
        }
    }
    uint4 v[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
        v[k] = pos[k] >= 0 ? __ldcg(reinterpret_cast<const uint4 *>(y + static_cast<size_t>(pos[k]) * hidden + c))
                           : make_uint4(0, 0, 0, 0);
    const uint4 sv = shared_y ? __ldcg(reinterpret_cast<const uint4 *>(shared_y + static_cast<size_t>(t) * hidden + c))
                              : make_uint4(0, 0, 0, 0);
    // packed BF16 pairs: acc = bf16(acc + bf16(v * w)) per route, ascending position
    uint4 o = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        if (pos[k] < 0) continue;
        const uint32_t w2 = bf16x2_splat(wt[k]);
        o.x = bf16x2_mul_add(o.x, v[k].x, w2);
        o.y = bf16x2_mul_add(o.y, v[k].y, w2);
        o.z = bf16x2_mul_add(o.z, v[k].z, w2);
        o.w = bf16x2_mul_add(o.w, v[k].w, w2);
    }
    if (shared_y) {
        const uint32_t s2 = bf16x2_splat(sig[t]);
        o.x = bf16x2_mul_add(o.x, sv.x, s2);
        o.y = bf16x2_mul_add(o.y, sv.y, s2);
        o.z = bf16x2_mul_add(o.z, sv.z, s2);
        o.w = bf16x2_mul_add(o.w, sv.w, s2);
    }
    *reinterpret_cast<uint4 *>(out + static_cast<size_t>(t) * hidden + c) = o;
}

int launch_combine(const uint16_t *y, const int32_t *route_pos, const uint16_t *scores, int tokens, int top_k,
                   int hidden, const uint16_t *shared_y, const uint16_t *sig, uint16_t *out, cudaStream_t stream) {
    if (tokens == 0) return MOE_OK;
    if (top_k > 16 || hidden % 8) return set_error(MOE_EINVAL, "combine: top_k %d > 16", top_k);
    const int64_t threads = static_cast<int64_t>(tokens) * (hidden / 8);
    const dim3 grid(static_cast<unsigned>((threads + 255) / 256));
    if (top_k <= 8)
        return launch_pdl(combine_kernel<8, 3>, grid, dim3(256), 0, stream, "combine_kernel", y, route_pos, scores,
                          tokens, top_k, hidden, shared_y, sig, out);
    return launch_pdl(combine_kernel<16, 2>, grid, dim3(256), 0, stream, "combine_kernel", y, route_pos, scores, tokens,
                      top_k, hidden, shared_y, sig, out);
}

namespace {

int expert_pairs(const uint16_t *const *gate_up, const uint16_t *const *down, const uint16_t *input,
                 const int32_t *token_ids, uint16_t *output, int tokens, int experts, void *workspace,
                 size_t workspace_bytes, void *stream, const char *name) {
    constexpr int H = 2048, I = 512;
    LRB_REQUIRE(experts >= 0 && experts <= kMaxParamGroups, "%s: experts %d outside [0, %d]", name, experts,
                kMaxParamGroups);
    LRB_REQUIRE(tokens >= 1 && tokens <= 16, "%s: tokens %d outside [1, 16]", name, tokens);
    if (experts == 0) return MOE_OK;
    LRB_REQUIRE(gate_up && down && input && output, "%s: null pointer", name);
    LRB_REQUIRE(workspace && workspace_bytes >= static_cast<size_t>(experts) * I * sizeof(uint16_t),
                "%s: workspace must hold experts * 512 BF16 activations", name);
    ParamGroups src;
    memset(&src, 0, sizeof src);
    src.count = experts;
    for (int e = 0; e < experts; ++e) {
        LRB_REQUIRE(gate_up[e] && down[e], "%s: null weight pointer for expert %d", name, e);
        const int t = token_ids ? token_ids[e] : 0;
        LRB_REQUIRE(t >= 0 && t < tokens, "%s: token id %d outside [0, %d)", name, t, tokens);
        src.groups[e] = Group{gate_up[e], gate_up[e] + static_cast<size_t>(I) * H, down[e], e, 1};
        src.tokens[e] = t;
    }
    if (int rc = require_sm100()) return rc;
    return launch_experts(src, experts, input, H, I, static_cast<uint16_t *>(workspace), output, as_stream(stream),
                          nullptr);
}

}  // namespace

}  // namespace lrb

extern "C" {

int moe_expert_rows(const uint16_t *const *gate_up, const uint16_t *const *down, const uint16_t *input,
                    uint16_t *output, int experts, void *workspace, size_t workspace_bytes, void *stream) {
    return lrb::expert_pairs(gate_up, down, input, nullptr, output, 1, experts, workspace, workspace_bytes, stream,
                             "moe_expert_rows");
}

int moe_expert_block_rows(const uint16_t *const *gate_up, const uint16_t *const *down, const uint16_t *input,
                          const int32_t *token_ids, uint16_t *output, int tokens, int experts, void *workspace,
                          size_t workspace_bytes, void *stream) {
    if (experts > 0 && !token_ids) return lrb::set_error(MOE_EINVAL, "moe_expert_block_rows: token_ids is required");
    return lrb::expert_pairs(gate_up, down, input, token_ids, output, tokens, experts, workspace, workspace_bytes,
                             stream, "moe_expert_block_rows");
}

}  // extern "C"
