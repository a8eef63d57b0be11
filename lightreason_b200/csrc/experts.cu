// Expert projections at decode and small-batch widths, and the ordered combine.
//
// gate/up: one warp per (group, row r): the gate row r and up row r of the
// group's expert stay in registers (16-byte streaming loads), and every routed
// token is dotted against both; bf16(gate), bf16(up), bf16(silu), bf16(s*u)
// are the eager rounding points (modeling_qwen3_5_moe.py:745-746,
// edge35b/cpu_experts.c:59-62).  down: one warp per (group, 4 output rows)
// over the group's activation rows (:747, cpu_experts.c:68).  The weight stream
// dominates (6 MiB per expert), so each weight byte is loaded exactly once.
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

// gate/up: one warp per row r of one group (the CTA's group): the gate row
// and the up row stay in registers; the group's token rows are staged in
// shared memory four at a time, so a warp holds only its 2 x 4 KiB of weights
// and two CTAs fit on an SM with every weight load in flight.
template <int NW, class Src>
__global__ void __launch_bounds__(256, 2) gate_up_kernel(const Src src, const uint16_t *__restrict__ x, int inner,
                                                         uint16_t *__restrict__ act) {
    constexpr int H = NW * 256;
    __shared__ uint4 xs[4][H / 8];
    const int g = blockIdx.y;
    grid_dependency_wait();  // the groups come from the routing kernels before
    grid_dependency_trigger();
    if (blockIdx.x == 0 && g == 0 && threadIdx.x == 0) src.on_start();
    if (g >= src.n()) return;
    const Group G = src.get(g);
    if (G.count <= 0) return;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const bool live = row < inner;
    uint4 wg[NW], wu[NW];
    if (live) {
        const uint16_t *gr = G.gate + static_cast<size_t>(row) * H;
        const uint16_t *ur = G.up + static_cast<size_t>(row) * H;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            wg[i] = ld_stream(gr + (lane + 32 * i) * 8);
            wu[i] = ld_stream(ur + (lane + 32 * i) * 8);
        }
    }
    for (int j0 = 0; j0 < G.count; j0 += 4) {
        const int nj = min(4, G.count - j0);
        __syncthreads();  // the previous round's token rows are consumed
        for (int i = threadIdx.x; i < nj * (H / 8); i += blockDim.x) {
            const int j = i / (H / 8), c = i % (H / 8);
            xs[j][c] = ld_cached(x + static_cast<size_t>(src.token(G.begin + j0 + j)) * H + c * 8);
        }
        __syncthreads();
        if (!live) continue;
        for (int j = 0; j < nj; ++j) {
            float ag = 0.f, au = 0.f;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const uint4 a = xs[j][lane + 32 * i];
                ag = dot8(wg[i], a, ag);
                au = dot8(wu[i], a, au);
            }
            ag = warp_sum(ag);
            au = warp_sum(au);
            if (lane == 0) {
                const float gv = rbf(ag), uv = rbf(au);
                const float s = rbf(silu_f32(gv));
                act[static_cast<size_t>(G.begin + j0 + j) * inner + row] = f2bf(s * uv);
            }
        }
    }
}

// down: one warp per four output rows of one group, their 4 x 1 KiB of
// weights requested before the activations exist (programmatic launch: the
// groups were complete before the gate/up kernel started, so this kernel may
// read them while that kernel still runs; only the activations wait).
template <int NI, class Src>
__global__ void __launch_bounds__(256, 3) down_kernel(const Src src, const uint16_t *__restrict__ act, int hidden,
                                                   uint16_t *__restrict__ y) {
    constexpr int I = NI * 256;
    constexpr int R = 4;  // rows per warp
    const int g = blockIdx.y;
    if (g >= src.n()) {
        grid_dependency_wait();
        return;
    }
    const Group G = src.get(g);
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * 8 + (threadIdx.x >> 5)) * R;
    if (row0 >= hidden || G.count <= 0) {
        grid_dependency_wait();
        return;
    }
    uint4 wd[R][NI];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint16_t *dr = G.down + static_cast<size_t>(min(row0 + r, hidden - 1)) * I;
#pragma unroll
        for (int i = 0; i < NI; ++i) wd[r][i] = ld_stream(dr + (lane + 32 * i) * 8);
    }
    grid_dependency_wait();
    grid_dependency_trigger();
    for (int j = 0; j < G.count; ++j) {
        const uint16_t *ar = act + static_cast<size_t>(G.begin + j) * I;
        uint4 a[NI];
#pragma unroll
        for (int i = 0; i < NI; ++i) a[i] = ld_cached(ar + (lane + 32 * i) * 8);
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            acc[r] = 0.f;
#pragma unroll
            for (int i = 0; i < NI; ++i) acc[r] = dot8(wd[r][i], a[i], acc[r]);
            acc[r] = warp_sum(acc[r]);
        }
        if (lane < R && row0 + lane < hidden) {
            float v = acc[0];
#pragma unroll
            for (int r = 1; r < R; ++r)
                if (lane == r) v = acc[r];
            y[static_cast<size_t>(G.begin + j) * hidden + row0 + lane] = f2bf(v);
        }
    }
}

template <class Src>
int launch_experts(const Src &src, int max_groups, const uint16_t *x, int hidden, int inner, uint16_t *act,
                   uint16_t *y, cudaStream_t stream, cudaEvent_t between) {
    if (max_groups <= 0) return MOE_OK;
    const dim3 gu_grid((inner + 7) / 8, max_groups), dn_grid((hidden + 31) / 32, max_groups);
    int rc;
    if (hidden == 2048) rc = launch_pdl(gate_up_kernel<8, Src>, gu_grid, dim3(256), 0, stream, "gate_up_kernel", src, x, inner, act);
    else if (hidden == 1024) rc = launch_pdl(gate_up_kernel<4, Src>, gu_grid, dim3(256), 0, stream, "gate_up_kernel", src, x, inner, act);
    else if (hidden == 4096) rc = launch_pdl(gate_up_kernel<16, Src>, gu_grid, dim3(256), 0, stream, "gate_up_kernel", src, x, inner, act);
    else return set_error(MOE_EINVAL, "experts: hidden %d not in {1024, 2048, 4096}", hidden);
    if (rc) return rc;
    if (between) LRB_CUDA(cudaEventRecord(between, stream));
    if (inner == 512) rc = launch_pdl(down_kernel<2, Src>, dn_grid, dim3(256), 0, stream, "down_kernel", src, act, hidden, y);
    else if (inner == 256) rc = launch_pdl(down_kernel<1, Src>, dn_grid, dim3(256), 0, stream, "down_kernel", src, act, hidden, y);
    else if (inner == 1024) rc = launch_pdl(down_kernel<4, Src>, dn_grid, dim3(256), 0, stream, "down_kernel", src, act, hidden, y);
    else return set_error(MOE_EINVAL, "experts: inner %d not in {256, 512, 1024}", inner);
    return rc;
}

template int launch_experts<DeviceGroups>(const DeviceGroups &, int, const uint16_t *, int, int, uint16_t *,
                                          uint16_t *, cudaStream_t, cudaEvent_t);
template int launch_experts<ParamGroups>(const ParamGroups &, int, const uint16_t *, int, int, uint16_t *,
                                         uint16_t *, cudaStream_t, cudaEvent_t);
template int launch_experts<PlanGroups>(const PlanGroups &, int, const uint16_t *, int, int, uint16_t *,
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

// sig[t] = bf16(sigmoid(bf16(x[t] . w))): the shared-expert gate
// (modeling_qwen3_5_moe.py:779), one warp per token, FP32 accumulation in
// the lane order of the router's gate dot.
__global__ void __launch_bounds__(256) shared_gate_kernel(const uint16_t *__restrict__ x,
                                                          const uint16_t *__restrict__ w, int tokens, int hidden,
                                                          uint16_t *__restrict__ sig) {
    grid_dependency_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= tokens) return;
    const uint16_t *xr = x + static_cast<size_t>(t) * hidden;
    float acc = 0.f;
    for (int c0 = 0; c0 < hidden; c0 += 8 * 256) {
        uint4 wv[8], xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = c0 + u * 256 + lane * 8;
            wv[u] = c < hidden ? ld_cached(w + c) : make_uint4(0, 0, 0, 0);
            xv[u] = c < hidden ? ld_cached(xr + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (c0 + u * 256 + lane * 8 < hidden) acc = dot8(wv[u], xv[u], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) sig[t] = f2bf(sigmoid_f32(rbf(acc)));
}

}  // namespace

}  // namespace lrb

extern "C" {

int moe_combine(const uint16_t *y, const int32_t *route_pos, const uint16_t *scores, const uint16_t *shared_rows,
                const uint16_t *sig, int tokens, int top_k, int hidden, uint16_t *out, void *stream) {
    LRB_REQUIRE(tokens == 0 || (y && route_pos && scores && out && (!shared_rows || sig)), "moe_combine: null pointer");
    LRB_REQUIRE(hidden > 0 && hidden % 8 == 0 && tokens >= 0 && top_k >= 1 && top_k <= 16,
                "moe_combine: bad shape");
    if (tokens == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    return lrb::launch_combine(y, route_pos, scores, tokens, top_k, hidden, shared_rows, sig, out,
                               lrb::as_stream(stream));
}

size_t moe_shared_expert_workspace_bytes(int tokens, int inner) {
    return tokens > 0 && inner > 0 ? static_cast<size_t>(tokens) * inner * sizeof(uint16_t) : 0;
}

int moe_shared_expert(const uint16_t *x, const uint16_t *gate, const uint16_t *up, const uint16_t *down,
                      const uint16_t *gate_w, int tokens, int hidden, int inner, uint16_t *out, uint16_t *sig,
                      void *workspace, size_t workspace_bytes, void *stream) {
    LRB_REQUIRE(gate && up && down && (tokens == 0 || (x && out && (!gate_w || sig))), "moe_shared_expert: null pointer");
    LRB_REQUIRE(tokens >= 0 && tokens <= lrb::kMaxParamGroups, "moe_shared_expert: tokens %d outside [0, %d]", tokens,
                lrb::kMaxParamGroups);
    LRB_REQUIRE((hidden == 1024 || hidden == 2048 || hidden == 4096) && (inner == 256 || inner == 512 || inner == 1024),
                "moe_shared_expert: shapes %d x %d unsupported", hidden, inner);
    if (tokens == 0) return MOE_OK;
    LRB_REQUIRE(workspace && workspace_bytes >= moe_shared_expert_workspace_bytes(tokens, inner),
                "moe_shared_expert: workspace below moe_shared_expert_workspace_bytes");
    if (int rc = lrb::require_sm100()) return rc;
    lrb::ParamGroups src;
    memset(&src, 0, sizeof src);
    src.count = 1;
    src.groups[0] = lrb::Group{gate, up, down, 0, tokens};
    for (int t = 0; t < tokens; ++t) src.tokens[t] = t;
    cudaStream_t s = lrb::as_stream(stream);
    if (int rc = lrb::launch_experts(src, 1, x, hidden, inner, static_cast<uint16_t *>(workspace), out, s, nullptr))
        return rc;
    if (!gate_w) return MOE_OK;
    return lrb::launch_pdl(lrb::shared_gate_kernel, dim3((tokens + 7) / 8), dim3(256), 0, s, "shared_gate_kernel", x,
                           gate_w, tokens, hidden, sig);
}

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
