// Grouped SwiGLU experts on the 5th-generation tensor cores.
//
// One persistent launch computes, for every active expert group g (routed
// experts in ascending id, then the shared expert):
//   phase 1  act[p, :]  = bf16(bf16(silu(bf16(x_p . Wg))) * bf16(x_p . Wu))
//   phase 2  y[p, :]    = bf16(act_p . Wd)
// for the routes p of the group (modeling_qwen3_5_moe.py:745-748 rounding
// points).  The weights are the M = 128 operand (rows of gate/up/down), the
// group's routed tokens the N operand ("swap AB"), so decode widths (a handful
// of tokens per expert) and prefill widths (hundreds) use the same tiles.
//
// Work items: phase-1 (group, 128-row block of gate+up, token tile) and
// phase-2 (group, 128-row block of down, token tile), handed out in that order
// from a device counter.  A phase-2 item waits (bounded) until every phase-1
// item of its group has published its activations; phase-1 items never wait,
// so the queue cannot deadlock.
//
// Per CTA (192 threads, one CTA per SM): warp 0 issues TMA loads of 64-wide K
// slices (128B swizzle) into a ring of stages; warp 1 allocates TMEM and issues
// tcgen05.mma (M=128, N=BN, K=16) into a double-buffered FP32 accumulator;
// warps 2-5 read the accumulator back with tcgen05.ld and write BF16 results.
// Every wait is bounded (globaltimer); on timeout the CTA raises the plan's
// error word, drains its own TMA and MMA work and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace lrb {

namespace {

constexpr int kBM = 128;                // weight rows per tile (MMA M)
constexpr int kBK = 64;                 // K per stage: one 128-byte swizzle atom of BF16
constexpr int kATile = kBM * kBK * 2;   // 16 KiB
constexpr int kThreads = 192;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any legal wait

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

}  // namespace

template <int BN>
struct GroupedShape {
    static constexpr int kBTile = BN * kBK * 2 < 1024 ? 1024 : BN * kBK * 2;
    static constexpr int kStage = 2 * kATile + kBTile;
    static constexpr int kStages = BN >= 128 ? 4 : (BN >= 64 ? 5 : 6);
    static constexpr int kTmemCols = 4 * BN < 32 ? 32 : 4 * BN;  // two buffers of (gate, up)
    static constexpr int kSmem = kStages * kStage + 1024 /*align*/ + 512 /*barriers*/;
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
    const int32_t *off1;  // [num_groups + 1] phase-1 item prefix
    const int32_t *off2;  // [num_groups + 1] phase-2 item prefix
    int32_t *done1;       // [num_groups] finished phase-1 items
    uint16_t *act;        // [rows, inner]
    uint16_t *y;          // [rows, hidden]
    int hidden, inner;
};

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
    int phase, g, mb, nt;
};

__device__ __forceinline__ ItemPos decode_item(const GroupedParams &P, int n_groups, int items1, int item, int mb1,
                                               int mb2) {
    ItemPos r;
    if (item < items1) {
        r.phase = 1;
        r.g = find_group(P.off1, n_groups, item);
        const int local = item - P.off1[r.g];
        r.mb = local % mb1;
        r.nt = local / mb1;
    } else {
        const int j = item - items1;
        r.phase = 2;
        r.g = find_group(P.off2, n_groups, j);
        const int local = j - P.off2[r.g];
        r.mb = local % mb2;
        r.nt = local / mb2;
    }
    return r;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    swiglu_grouped_kernel(const __grid_constant__ CUtensorMap tm_gu, const __grid_constant__ CUtensorMap tm_dn,
                          const __grid_constant__ CUtensorMap tm_sg, const __grid_constant__ CUtensorMap tm_su,
                          const __grid_constant__ CUtensorMap tm_sd, const __grid_constant__ CUtensorMap tm_x,
                          const __grid_constant__ CUtensorMap tm_act, const GroupedParams P) {
    using S = GroupedShape<BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    GroupedSmemTail *tail = reinterpret_cast<GroupedSmemTail *>(smem + S::kStages * S::kStage);
    volatile int *abort = &tail->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_groups = P.plan->num_groups;
    const int items1 = P.plan->items1, total = items1 + P.plan->items2;
    const int mb1 = P.inner / kBM, mb2 = P.hidden / kBM;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            sm100::mbar_init(&tail->full[s], 1);
            sm100::mbar_init(&tail->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(&tail->tfull[b], 1);
            sm100::mbar_init(&tail->tempty[b], 4);
        }
        for (int i = 0; i < 4; ++i) {
            sm100::mbar_init(&tail->ifull[i], 1);
            sm100::mbar_init(&tail->iempty[i], 5);
        }
        sm100::mbar_init(&tail->drain, 1);
        tail->abort = 0;
        sm100::fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        sm100::tma_prefetch_map(&tm_gu);
        sm100::tma_prefetch_map(&tm_dn);
        sm100::tma_prefetch_map(&tm_x);
        sm100::tma_prefetch_map(&tm_act);
    }
    if (warp == 1) {
        sm100::tmem_alloc(&tail->tmem_base, S::kTmemCols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = tail->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t stage = 0, sphase = 0;
            uint32_t issued_parity[8];
            bool issued[8] = {false, false, false, false, false, false, false, false};
            for (int it = 0;; ++it) {
                int item = atomicAdd(&P.plan->work, 1);
                if (item >= total) item = -1;
                const int slot = it & 3;
                if (!wait_bar(&tail->iempty[slot], ((it >> 2) & 1) ^ 1, abort)) break;
                tail->item[slot] = item;
                sm100::mbar_arrive(&tail->ifull[slot]);
                if (item < 0) break;
                const ItemPos ip = decode_item(P, n_groups, items1, item, mb1, mb2);
                const GroupedGroup G = P.groups[ip.g];
                if (ip.phase == 2) {
                    // every phase-1 item of the group publishes once per epilogue warp
                    const int need = 4 * mb1 * G.ntiles;
                    const uint64_t t0 = now_ns();
                    bool ok = true;
                    while (sm100::ld_acquire(&P.done1[ip.g]) < need) {
                        if (*abort || now_ns() - t0 > kWaitNs) {
                            ok = false;
                            break;
                        }
                        __nanosleep(100);
                    }
                    if (!ok) {
                        *abort = 1;
                        atomicExch(&P.plan->error, 2);
                        break;
                    }
                    sm100::fence_proxy_async_global();
                }
                const int kblocks = (ip.phase == 1 ? P.hidden : P.inner) / kBK;
                const uint32_t bytes = (ip.phase == 1 ? 2 * kATile : kATile) + BN * kBK * 2;
                const int row0 = ip.mb * kBM;
                const int tok0 = G.begin + ip.nt * BN;
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!wait_bar(&tail->empty[stage], sphase ^ 1, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + stage * S::kStage;
                    uint64_t *fb = &tail->full[stage];
                    sm100::mbar_expect_tx(fb, bytes);
                    const int k0 = kb * kBK;
                    if (ip.phase == 1) {
                        if (G.weight >= 0) {
                            sm100::tma_load_3d(st, &tm_gu, fb, k0, row0, G.weight);
                            sm100::tma_load_3d(st + kATile, &tm_gu, fb, k0, P.inner + row0, G.weight);
                        } else {
                            sm100::tma_load_2d(st, &tm_sg, fb, k0, row0);
                            sm100::tma_load_2d(st + kATile, &tm_su, fb, k0, row0);
                        }
                        sm100::tma_load_2d(st + 2 * kATile, &tm_x, fb, k0, tok0);
                    } else {
                        if (G.weight >= 0) sm100::tma_load_3d(st, &tm_dn, fb, k0, row0, G.weight);
                        else sm100::tma_load_2d(st, &tm_sd, fb, k0, row0);
                        sm100::tma_load_2d(st + 2 * kATile, &tm_act, fb, k0, tok0);
                    }
                    issued[stage] = true;
                    issued_parity[stage] = sphase;
                    if (++stage == S::kStages) {
                        stage = 0;
                        sphase ^= 1;
                    }
                }
                if (!ok) break;
            }
            if (*abort) {
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
        if (lane == 0) {
            constexpr uint32_t idesc = sm100::idesc_bf16_f32(kBM, BN);
            uint32_t stage = 0, sphase = 0;
            int acc = 0;
            bool any = false;
            for (int it = 0;; ++it) {
                const int slot = it & 3;
                if (!wait_bar(&tail->ifull[slot], (it >> 2) & 1, abort)) break;
                const int item = tail->item[slot];
                sm100::mbar_arrive(&tail->iempty[slot]);
                if (item < 0) break;
                const ItemPos ip = decode_item(P, n_groups, items1, item, mb1, mb2);
                const int kblocks = (ip.phase == 1 ? P.hidden : P.inner) / kBK;
                const int buf = acc & 1;
                if (!wait_bar(&tail->tempty[buf], ((acc >> 1) & 1) ^ 1, abort)) break;
                sm100::tc_fence_after();
                const uint32_t d_gate = tmem + buf * 2 * BN, d_up = d_gate + BN;
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
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
                        sm100::mma_bf16(d_gate, a0 + 2 * kk, b + 2 * kk, idesc, accumulate);
                        if (ip.phase == 1) sm100::mma_bf16(d_up, a1 + 2 * kk, b + 2 * kk, idesc, accumulate);
                    }
                    sm100::mma_commit(&tail->empty[stage]);
                    any = true;
                    if (++stage == S::kStages) {
                        stage = 0;
                        sphase ^= 1;
                    }
                }
                if (!ok) break;
                sm100::mma_commit(&tail->tfull[buf]);
                ++acc;
            }
            if (*abort && any) {
                // Wait for this thread's MMAs before TMEM is released.
                sm100::mma_commit(&tail->drain);
                const uint64_t t0 = now_ns();
                while (!sm100::mbar_try_wait(&tail->drain, 0) && now_ns() - t0 < kWaitNs) {
                }
            }
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may read
        int acc = 0;
        for (int it = 0;; ++it) {
            const int slot = it & 3;
            if (!wait_bar(&tail->ifull[slot], (it >> 2) & 1, abort)) break;
            const int item = tail->item[slot];
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&tail->iempty[slot]);
            if (item < 0) break;
            const ItemPos ip = decode_item(P, n_groups, items1, item, mb1, mb2);
            const GroupedGroup G = P.groups[ip.g];
            const int buf = acc & 1;
            if (!wait_bar(&tail->tfull[buf], (acc >> 1) & 1, abort)) break;
            __syncwarp();
            sm100::tc_fence_after();
            const int row = ip.mb * kBM + q * 32 + lane;
            const int p0 = G.begin + ip.nt * BN;
            const int nvalid = min(BN, G.count - ip.nt * BN);
            const uint32_t t_gate = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 2 * BN;
            if (ip.phase == 1) {
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
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
            } else {
#pragma unroll
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    float v[16];
                    __syncwarp();
                    sm100::tmem_ld16(t_gate + c0, v);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c0 + j < nvalid) P.y[static_cast<size_t>(p0 + c0 + j) * P.hidden + row] = f2bf(v[j]);
                }
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&tail->tempty[buf]);
            ++acc;
            if (ip.phase == 1) {
                // Publish this warp's 32 activation rows: each lane fences its
                // own stores, then one release per warp (no cross-warp barrier,
                // so an aborting warp can never strand the others).
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    sm100::fence_proxy_async_global();
                    atomicAdd(&P.done1[ip.g], 1);
                }
            }
        }
    }

    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, S::kTmemCols);
    }
    if (threadIdx.x == 0 && *abort) atomicCAS(&P.plan->error, 0, 1);
}

// One CTA: groups in ascending expert id (+ shared expert last), item prefix
// sums, zeroed counters, and the route -> token map of the shared rows.
__global__ void grouped_plan_kernel(const int32_t *__restrict__ active, const int32_t *__restrict__ num_active,
                                    const int32_t *__restrict__ offsets, int use_slots, int shared, int routes,
                                    int tokens, int bn, int mb1, int mb2, GroupedGroup *__restrict__ groups,
                                    GroupedPlan *__restrict__ plan, int32_t *__restrict__ off1,
                                    int32_t *__restrict__ off2, int32_t *__restrict__ done1,
                                    int32_t *__restrict__ route_token) {
    const int n = *num_active;
    const int ng = n + (shared ? 1 : 0);
    for (int g = threadIdx.x; g < ng; g += blockDim.x) {
        GroupedGroup G;
        if (g < n) {
            const int e = active[g];
            G.weight = use_slots ? g : e;
            G.begin = offsets[e];
            G.count = offsets[e + 1] - offsets[e];
        } else {
            G.weight = -1;
            G.begin = routes;
            G.count = tokens;
        }
        G.ntiles = (G.count + bn - 1) / bn;
        groups[g] = G;
        done1[g] = 0;
    }
    for (int t = threadIdx.x; shared && t < tokens; t += blockDim.x) route_token[routes + t] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0, b = 0;
        for (int g = 0; g < ng; ++g) {
            off1[g] = a;
            off2[g] = b;
            a += mb1 * groups[g].ntiles;
            b += mb2 * groups[g].ntiles;
        }
        off1[ng] = a;
        off2[ng] = b;
        plan->num_groups = ng;
        plan->items1 = a;
        plan->items2 = b;
        plan->work = 0;
        plan->error = 0;
    }
}

// xs[p] = x[route_token[p]] for the placed routes (p < offsets[experts]) and,
// when the shared expert runs, xs[routes + t] = x[t]; 16 bytes per thread.
__global__ void __launch_bounds__(256) gather_tokens_kernel(const uint16_t *__restrict__ x,
                                                            const int32_t *__restrict__ route_token,
                                                            const int32_t *__restrict__ offsets, int experts,
                                                            int routes, int shared_rows, int hidden,
                                                            uint16_t *__restrict__ xs) {
    const int units = hidden / 8;
    const int placed = offsets[experts];
    const int64_t total = static_cast<int64_t>(routes + shared_rows) * units;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i / units), c = static_cast<int>(i % units);
        if (p < routes && p >= placed) continue;
        const int t = p < routes ? route_token[p] : p - routes;
        reinterpret_cast<uint4 *>(xs)[i] = ld_cached(x + static_cast<size_t>(t) * hidden + c * 8);
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

// BF16 tensor map: dims[0] innermost (K), 128-byte swizzle, box {64, box_rows(, 1)}.
int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides_bytes,
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

template <int BN>
int launch_bn(const GroupedLaunch &L, cudaStream_t stream) {
    using S = GroupedShape<BN>;
    CUtensorMap gu{}, dn{}, sg{}, su{}, sd{}, xm{}, am{};
    const uint64_t H = L.hidden, I = L.inner, rows = static_cast<uint64_t>(L.rows);
    {
        const uint64_t dims[3] = {H, 2 * I, static_cast<uint64_t>(L.bank_experts)};
        const uint64_t str[2] = {H * 2, static_cast<uint64_t>(L.gate_up_stride) * 2};
        if (int rc = make_map(&gu, L.gate_up, 3, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[3] = {I, H, static_cast<uint64_t>(L.bank_experts)};
        const uint64_t str[2] = {I * 2, static_cast<uint64_t>(L.down_stride) * 2};
        if (int rc = make_map(&dn, L.down, 3, dims, str, kBM)) return rc;
    }
    const void *sgp = L.sh_gate ? L.sh_gate : L.gate_up, *sup = L.sh_up ? L.sh_up : L.gate_up;
    const void *sdp = L.sh_down ? L.sh_down : L.down;
    {
        const uint64_t dims[2] = {H, I}, str[1] = {H * 2};
        if (int rc = make_map(&sg, sgp, 2, dims, str, kBM)) return rc;
        if (int rc = make_map(&su, sup, 2, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[2] = {I, H}, str[1] = {I * 2};
        if (int rc = make_map(&sd, sdp, 2, dims, str, kBM)) return rc;
    }
    {
        const uint64_t dims[2] = {H, rows}, str[1] = {H * 2};
        if (int rc = make_map(&xm, L.xs, 2, dims, str, BN)) return rc;
    }
    {
        const uint64_t dims[2] = {I, rows}, str[1] = {I * 2};
        if (int rc = make_map(&am, L.act, 2, dims, str, BN)) return rc;
    }
    static std::once_flag once[4];
    static cudaError_t attr_err[4];
    const int which = BN == 16 ? 0 : BN == 32 ? 1 : BN == 64 ? 2 : 3;
    std::call_once(once[which], [] {
        attr_err[BN == 16 ? 0 : BN == 32 ? 1 : BN == 64 ? 2 : 3] = cudaFuncSetAttribute(
            swiglu_grouped_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem);
    });
    if (attr_err[which] != cudaSuccess) return cuda_error(attr_err[which], "cudaFuncSetAttribute(grouped)");
    GroupedParams P{L.groups, L.plan, L.off1, L.off2, L.done1, L.act, L.y, L.hidden, L.inner};
    swiglu_grouped_kernel<BN><<<L.ctas, kThreads, S::kSmem, stream>>>(gu, dn, sg, su, sd, xm, am, P);
    LRB_LAUNCHED("swiglu_grouped_kernel");
    return MOE_OK;
}

}  // namespace

int grouped_bn_for(int tokens) { return tokens <= 16 ? 16 : tokens <= 64 ? 32 : tokens <= 512 ? 64 : 128; }

int launch_grouped_plan(const int32_t *active, const int32_t *num_active, const int32_t *offsets, bool use_slots,
                        bool shared, int routes, int tokens, int bn, int hidden, int inner, GroupedGroup *groups,
                        GroupedPlan *plan, int32_t *off1, int32_t *off2, int32_t *done1, int32_t *route_token,
                        cudaStream_t stream) {
    grouped_plan_kernel<<<1, 256, 0, stream>>>(active, num_active, offsets, use_slots, shared, routes, tokens, bn,
                                                inner / kBM, hidden / kBM, groups, plan, off1, off2, done1,
                                                route_token);
    LRB_LAUNCHED("grouped_plan_kernel");
    return MOE_OK;
}

int launch_gather_tokens(const uint16_t *x, const int32_t *route_token, const int32_t *offsets, int experts,
                         int routes, int shared_rows, int hidden, uint16_t *xs, cudaStream_t stream) {
    const int64_t units = static_cast<int64_t>(routes + shared_rows) * (hidden / 8);
    const int grid = static_cast<int>(std::min<int64_t>((units + 255) / 256, 148 * 16));
    if (grid == 0) return MOE_OK;
    gather_tokens_kernel<<<grid, 256, 0, stream>>>(x, route_token, offsets, experts, routes, shared_rows, hidden,
                                                    xs);
    LRB_LAUNCHED("gather_tokens_kernel");
    return MOE_OK;
}

int launch_grouped(const GroupedLaunch &L, cudaStream_t stream) {
    LRB_REQUIRE(L.hidden % kBM == 0 && L.inner % kBM == 0, "grouped: hidden and inner must be multiples of 128");
    switch (L.bn) {
        case 16: return launch_bn<16>(L, stream);
        case 32: return launch_bn<32>(L, stream);
        case 64: return launch_bn<64>(L, stream);
        case 128: return launch_bn<128>(L, stream);
        default: return set_error(MOE_EINVAL, "grouped: unsupported token tile %d", L.bn);
    }
}

}  // namespace lrb
