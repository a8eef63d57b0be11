// Device-side routing helpers shared by the permute kernel and the fused
// decode routing kernel: a CTA-wide exclusive scan, the stable counting-sort
// permute of the eager dispatch order, and per-token top-k selection.
#pragma once

#include "common.cuh"

namespace lrb {

// Exclusive scan of one int per thread over the CTA (blockDim.x <= 1024).
// `scratch` holds >= 33 ints of shared memory.  Returns the exclusive prefix;
// *total receives the CTA-wide sum.  Every thread of the CTA must call it.
__device__ __forceinline__ int block_exclusive_scan(int v, int *scratch, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    int incl = v;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, s);
        if (lane >= s) incl += o;
    }
    __syncthreads();
    if (lane == 31) scratch[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int ws = lane < warps ? scratch[lane] : 0;
        int wincl = ws;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, wincl, s);
            if (lane >= s) wincl += o;
        }
        scratch[lane] = wincl - ws;
        if (lane == 31) scratch[32] = wincl;
    }
    __syncthreads();
    const int r = scratch[warp] + incl - v;
    *total = scratch[32];
    __syncthreads();
    return r;
}

// Exclusive scan of three ints per thread over the CTA in one pass (the three
// shuffle chains interleave, so it costs about one scan).  `scratch` holds
// >= 99 ints of shared memory; *total receives the CTA-wide sums.
__device__ __forceinline__ int3 block_exclusive_scan3(int3 v, int *scratch, int3 *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    int a = v.x, b = v.y, c = v.z;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const int oa = __shfl_up_sync(0xffffffffu, a, s);
        const int ob = __shfl_up_sync(0xffffffffu, b, s);
        const int oc = __shfl_up_sync(0xffffffffu, c, s);
        if (lane >= s) {
            a += oa;
            b += ob;
            c += oc;
        }
    }
    __syncthreads();
    if (lane == 31) {
        scratch[warp] = a;
        scratch[33 + warp] = b;
        scratch[66 + warp] = c;
    }
    __syncthreads();
    if (warp == 0) {
        const int wa = lane < warps ? scratch[lane] : 0, wb = lane < warps ? scratch[33 + lane] : 0,
                  wc = lane < warps ? scratch[66 + lane] : 0;
        int ia = wa, ib = wb, ic = wc;
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const int oa = __shfl_up_sync(0xffffffffu, ia, s);
            const int ob = __shfl_up_sync(0xffffffffu, ib, s);
            const int oc = __shfl_up_sync(0xffffffffu, ic, s);
            if (lane >= s) {
                ia += oa;
                ib += ob;
                ic += oc;
            }
        }
        scratch[lane] = ia - wa;
        scratch[33 + lane] = ib - wb;
        scratch[66 + lane] = ic - wc;
        if (lane == 31) {
            scratch[32] = ia;
            scratch[65] = ib;
            scratch[98] = ic;
        }
    }
    __syncthreads();
    const int3 r = make_int3(scratch[warp] + a - v.x, scratch[33 + warp] + b - v.y, scratch[66 + warp] + c - v.z);
    *total = make_int3(scratch[32], scratch[65], scratch[98]);
    __syncthreads();
    return r;
}

// The whole permute, executed by every thread of one CTA (blockDim.x is a
// multiple of 32, >= experts).  idx_of(t, k) yields the expert id of (token,
// slot).  cnt: shared [warps * experts + experts] ints; scratch: 33 ints.
// Only the first ceil(routes / 32) warps own routes (and counting tables), so
// few routes cost few table columns.
template <class IdxOf>
__device__ void permute_block(IdxOf idx_of, int tokens, int top_k, int experts, int32_t *offsets,
                              int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos, int32_t *active,
                              int32_t *num_active, int32_t *bad_routes, int32_t *cnt, int *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int routes = tokens * top_k;
    const int warps = max(1, min(static_cast<int>(blockDim.x >> 5), (routes + 31) / 32));
    int32_t *total = cnt + warps * experts;
    const int chunk = ((routes + warps * 32 - 1) / (warps * 32)) * 32;
    const int r_begin = warp < warps ? warp * chunk : routes;
    const int r_end = warp < warps ? min(routes, r_begin + chunk) : routes;

    for (int i = threadIdx.x; i < warps * experts; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    int bad = 0;
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e = -1;
        if (r < r_end) {
            const int64_t v = idx_of(r % tokens, r / tokens);
            if (v >= 0 && v < experts) e = static_cast<int>(v);
            else bad++;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e] += __popc(peers);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < experts; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < warps; ++w) {
            const int c = cnt[w * experts + e];
            cnt[w * experts + e] = run;
            run += c;
        }
        total[e] = run;
    }
    __syncthreads();
    const int my_total = threadIdx.x < experts ? total[threadIdx.x] : 0;
    int all = 0;
    const int excl = block_exclusive_scan(my_total, scratch, &all);
    if (threadIdx.x < experts) {
        offsets[threadIdx.x] = excl;
        if (threadIdx.x == experts - 1) offsets[experts] = excl + my_total;
        for (int w = 0; w < warps; ++w) cnt[w * experts + threadIdx.x] += excl;
    }
    int n_active = 0;
    const int apos = block_exclusive_scan(my_total > 0 ? 1 : 0, scratch, &n_active);
    if (my_total > 0) active[apos] = threadIdx.x;
    if (threadIdx.x == 0) *num_active = n_active;
    __syncthreads();
    for (int r0 = r_begin; r0 < r_end; r0 += 32) {
        const int r = r0 + lane;
        int e = -1, t = 0, k = 0;
        if (r < r_end) {
            t = r % tokens;
            k = r / tokens;
            const int64_t v = idx_of(t, k);
            if (v >= 0 && v < experts) e = static_cast<int>(v);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        int p = -1;
        if (e >= 0) p = cnt[warp * experts + e] + __popc(peers & ((1u << lane) - 1));
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * experts + e] += __popc(peers);
        __syncwarp();
        if (r < r_end) {
            route_pos[static_cast<size_t>(t) * top_k + k] = p;
            if (p >= 0) {
                perm_token[p] = t;
                perm_slot[p] = k;
            }
        }
    }
    if (bad_routes) {
        int n_bad = 0;
        block_exclusive_scan(bad, scratch, &n_bad);
        if (threadIdx.x == 0) *bad_routes = n_bad;
    }
    __syncthreads();
}

struct GlobalIdx {
    const int64_t *idx;
    int top_k;
    __device__ __forceinline__ int64_t operator()(int t, int k) const {
        return idx[static_cast<size_t>(t) * top_k + k];
    }
};


// Top-k of one token by one warp (modeling_qwen3_5_moe.py:762-770 plus the
// per-expert bias): z[e] = logit + bias is given through z_of(e) for e <
// experts (<= 32 * VPL); softmax over z; selection by z descending with exact
// ties to the lower expert id; w_k = p_k / sum_k p_k in slot order.  Lane k <
// top_k returns slot k's expert in *e_out and its weight in *w_out.
// Order-preserving unsigned key of a float (larger float, larger key), with
// -0 ranked as +0 so that the two compare equal as floats do.
__device__ __forceinline__ uint32_t topk_key(float f) {
    uint32_t b = __float_as_uint(f);
    if (b == 0x80000000u) b = 0;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float topk_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int VPL, class ZOf>
__device__ __forceinline__ void warp_topk(ZOf z_of, int experts, int top_k, int *e_out, float *w_out) {
    const int lane = threadIdx.x & 31;
    float z[VPL];
    uint32_t key[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
        const int e = lane + 32 * v;
        z[v] = -INFINITY;
        key[v] = 0;
        if (e < experts) {
            z[v] = z_of(e);
            m = fmaxf(m, z[v]);
            key[v] = topk_key(z[v]);
        }
    }
#pragma unroll
    for (int s = 16; s; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    float denom = 0.0f;
#pragma unroll
    for (int v = 0; v < VPL; ++v)
        if (lane + 32 * v < experts) denom += expf(z[v] - m);
    denom = warp_sum(denom);
    // Selection rounds: each lane's best untaken key (its lowest expert on a
    // tie), the warp's largest key by one redux, and the lowest expert holding
    // it by a second.
    uint32_t taken = 0, my_key = 0;
    int my_e = 0;
    for (int k = 0; k < top_k; ++k) {
        uint32_t bk = 0;
        int be = 0x7fffffff;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            if (!(taken & (1u << v)) && key[v] > bk) {
                bk = key[v];
                be = lane + 32 * v;
            }
        }
        const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
        const int we = __reduce_min_sync(0xffffffffu, bk == wk ? be : 0x7fffffff);
        if ((we & 31) == lane) taken |= 1u << (we >> 5);
        if (lane == k) {
            my_key = wk;
            my_e = we;
        }
    }
    // slot probabilities, every lane at once (lanes >= top_k unused)
    const float my_p = lane < top_k ? expf(topk_value(my_key) - m) / denom : 0.0f;
    float sum = 0.0f;
    for (int k = 0; k < top_k; ++k) sum += __shfl_sync(0xffffffffu, my_p, k);
    *e_out = my_e;
    *w_out = my_p / sum;
}

// The selection of one token by one warp (router_select_kernel, and the
// expert-parallel selection that also publishes the routes): its logits (or
// the FP32 K-split partials, summed in split order and rounded once to BF16,
// F.linear) + bias, softmax, top-k, renormalised BF16 weights, and with
// gate_w the shared-expert gate sig = bf16(sigmoid(bf16(x . w)))
// (modeling_qwen3_5_moe :762-770, :779, :788).  Lane k < top_k returns the
// k-th expert and its FP32 weight.
template <int VPL>
__device__ __forceinline__ void select_token(int t, const uint16_t *__restrict__ logits,
                                             const float *__restrict__ bias, int tokens, int experts, int top_k,
                                             int64_t *__restrict__ idx, float *__restrict__ scores_f32,
                                             uint16_t *__restrict__ scores_bf16, const uint16_t *__restrict__ x,
                                             const uint16_t *__restrict__ gate_w, int hidden,
                                             uint16_t *__restrict__ sig, const float *__restrict__ part, int ks,
                                             int *e_out, float *w_out) {
    const int lane = threadIdx.x & 31;
    uint16_t *row = const_cast<uint16_t *>(logits) + static_cast<size_t>(t) * experts;
    // Every load of the token issued up front: its logits (or the FP32 K-split
    // partials, summed in split order and rounded once to BF16, F.linear),
    // and the shared-expert gate operands, in rounds of 8 per lane.
    float z[VPL];
    if (part) {
        float p[VPL][4];
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            const int j = min(lane + 32 * v, experts - 1);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                p[v][k] = k < ks ? part[(static_cast<size_t>(k) * tokens + t) * experts + j] : 0.f;
        }
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            const int j = lane + 32 * v;
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (k < ks) s += p[v][k];
            const uint16_t lg = f2bf(s);
            if (j < experts) row[j] = lg;
            z[v] = bf2f(lg) + (bias && j < experts ? bias[j] : 0.0f);
        }
    } else {
        uint16_t lg[VPL];
#pragma unroll
        for (int v = 0; v < VPL; ++v) lg[v] = row[min(lane + 32 * v, experts - 1)];
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
            const int j = lane + 32 * v;
            z[v] = bf2f(lg[v]) + (bias && j < experts ? bias[j] : 0.0f);
        }
    }
    if (gate_w) {
        const uint16_t *xr = x + static_cast<size_t>(t) * hidden;
        float acc = 0.f;
        for (int c0 = 0; c0 < hidden; c0 += 8 * 256) {
            uint4 wv[8], xv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * 256 + lane * 8;
                wv[u] = c < hidden ? ld_cached(gate_w + c) : make_uint4(0, 0, 0, 0);
                xv[u] = c < hidden ? ld_cached(xr + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c0 + u * 256 + lane * 8 < hidden) acc = dot8(wv[u], xv[u], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) sig[t] = f2bf(sigmoid_f32(rbf(acc)));
    }
    int e;
    float w;
    warp_topk<VPL>([&](int j) { return z[j >> 5]; }, experts, top_k, &e, &w);
    if (lane < top_k) {
        const size_t o = static_cast<size_t>(t) * top_k + lane;
        idx[o] = e;
        if (scores_f32) scores_f32[o] = w;
        if (scores_bf16) scores_bf16[o] = f2bf(w);
    }
    *e_out = e;
    *w_out = w;
}


}  // namespace lrb
