// Router logits at prefill widths on the tensor cores: logits[T, E] =
// bf16(x[T, H] . W[E, H]^T) with FP32 accumulation (F.linear on BF16,
// transformers qwen3_5_moe modeling :764).
//
// One CTA per (128 router rows, BN tokens, K split): the router rows are the
// M = 128 operand and the token tile the N operand, both K-major with the
// 128-byte swizzle, streamed by TMA through an 8-stage ring.  With ks > 1 K
// splits (few tokens: more CTAs than row blocks x token tiles) each CTA writes
// FP32 partials part[split][t][e], which the selection kernel sums in split
// order before the one BF16 rounding.  Warp 0 issues the loads and warp 1
// the tcgen05.mma (M=128, N=BN, K=16) into a TMEM accumulator, each stage
// handed back to the loads by a commit; all four warps then read their 32 TMEM lanes (= router rows) and write BF16 logits,
// 32 consecutive experts of one token per warp store.  Every wait is bounded:
// on timeout the CTA records an error in *error, drains its own copies and
// products, and returns.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace lrb {

namespace {

constexpr int kRows = 128, kK = 64, kStagesTc = 8;
constexpr uint64_t kRouterWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t i = 1;; ++i) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0 && now_ns() - t0 > kRouterWaitNs) return false;
    }
}

}  // namespace

template <int BN>
__global__ void __launch_bounds__(128, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, int tokens,
                     int experts, int hidden, uint16_t *__restrict__ logits, float *__restrict__ part,
                     int32_t *__restrict__ error) {
    constexpr int kA = kRows * kK * 2;
    constexpr int kB = BN * kK * 2;
    constexpr int kStage = kA + kB;
    constexpr uint32_t kCols = BN < 32 ? 32 : BN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kStagesTc], empty[kStagesTc], done;
    __shared__ uint32_t tmem_base;
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesTc; ++s) {
            sm100::mbar_init(&full[s], 1);
            sm100::mbar_init(&empty[s], 1);
        }
        sm100::mbar_init(&done, 1);
        failed = 0;
        sm100::fence_barrier_init();
        sm100::tma_prefetch_map(&tm_w);
        sm100::tma_prefetch_map(&tm_x);
    }
    if (warp == 0) {
        sm100::tmem_alloc(&tmem_base, kCols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = tmem_base;
    grid_dependency_wait();  // x may come from the previous kernel
    grid_dependency_trigger();

    const int row0 = blockIdx.x * kRows, t0 = blockIdx.y * BN;
    const int nk = hidden / kK / gridDim.z, kb_first = blockIdx.z * nk;
    volatile int *failed_v = &failed;
    if (warp == 0 && lane == 0) {
        // TMA producer: refills a stage as soon as the products reading it
        // have committed, independently of the MMA issue below
        bool issued[kStagesTc] = {};
        uint32_t issued_parity[kStagesTc] = {};
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStagesTc;
            const uint32_t ph = (kb / kStagesTc) & 1;
            if (*failed_v || !wait_bounded(&empty[s], ph ^ 1)) {
                *failed_v = 1;
                break;
            }
            uint8_t *st = smem + s * kStage;
            sm100::mbar_expect_tx(&full[s], kStage);
            sm100::tma_load_2d(st, &tm_w, &full[s], (kb_first + kb) * kK, row0);
            sm100::tma_load_2d(st + kA, &tm_x, &full[s], (kb_first + kb) * kK, t0);
            issued[s] = true;
            issued_parity[s] = ph;
        }
        if (*failed_v) {
            if (error) atomicExch(error, 6);
            // drain: every issued copy lands before the CTA leaves
            for (int s = 0; s < kStagesTc; ++s)
                if (issued[s]) wait_bounded(&full[s], issued_parity[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: products back to back, each stage released by a commit
        constexpr uint32_t idesc = sm100::idesc_bf16_f32(kRows, BN);
        bool any_mma = false;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kStagesTc;
            const uint32_t ph = (kb / kStagesTc) & 1;
            if (*failed_v || !wait_bounded(&full[s], ph)) {
                *failed_v = 1;
                if (error) atomicExch(error, 6);
                break;
            }
            sm100::tc_fence_after();
            const uint32_t base = sm100::smem_u32(smem + s * kStage);
            const uint64_t a = sm100::desc_kmajor_sw128(base), b = sm100::desc_kmajor_sw128(base + kA);
#pragma unroll
            for (int kk = 0; kk < kK / 16; ++kk)
                sm100::mma_bf16(tmem, a + 2 * kk, b + 2 * kk, idesc, (kb | kk) != 0);
            sm100::mma_commit(&empty[s]);
            any_mma = true;
        }
        if (any_mma) sm100::mma_commit(&done);
        else sm100::mbar_arrive(&done);
    }
    __syncwarp();
    const bool ready = wait_bounded(&done, 0);
    sm100::tc_fence_after();
    if (ready && !*failed_v) {
        const int row = row0 + warp * 32 + lane;
        const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            __syncwarp();
            sm100::tmem_ld16(taddr + c0, v);
            sm100::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = t0 + c0 + j;
                if (t < tokens && row < experts) {
                    if (part) part[(static_cast<size_t>(blockIdx.z) * tokens + t) * experts + row] = v[j];
                    else logits[static_cast<size_t>(t) * experts + row] = f2bf(v[j]);
                }
            }
        }
    } else if (!ready && lane == 0 && error) {
        atomicExch(error, 6);
    }
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 0 && ready) {
        __syncwarp();
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, kCols);
    }
}

int router_tc_bn(int tokens) { return tokens >= 2048 ? 64 : 32; }

int router_tc_splits(int tokens, int experts) {
    const int ctas = ((experts + kRows - 1) / kRows) * ((tokens + router_tc_bn(tokens) - 1) / router_tc_bn(tokens));
    return ctas * 4 <= sm_count() ? 4 : ctas * 2 <= sm_count() ? 2 : 1;
}

template <int BN>
int launch_router_tc_bn(const uint16_t *x, const uint16_t *router, int tokens, int hidden, int experts,
                        uint16_t *logits, float *part, int ks, int32_t *error, cudaStream_t stream) {
    constexpr int kSmem = kStagesTc * (kRows * kK * 2 + BN * kK * 2) + 1024;
    CUtensorMap tw{}, tx{};
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(experts)};
        const uint64_t str[1] = {static_cast<uint64_t>(hidden) * 2};
        if (int rc = make_map_bf16(&tw, router, 2, dims, str, kRows)) return rc;
    }
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(tokens)};
        const uint64_t str[1] = {static_cast<uint64_t>(hidden) * 2};
        if (int rc = make_map_bf16(&tx, x, 2, dims, str, BN)) return rc;
    }
    if (int rc = ensure_dynamic_smem(router_tc_kernel<BN>, kSmem, "cudaFuncSetAttribute(router_tc)")) return rc;
    const dim3 grid((experts + kRows - 1) / kRows, (tokens + BN - 1) / BN, part ? ks : 1);
    return launch_pdl(router_tc_kernel<BN>, grid, dim3(128), kSmem, stream, "router_tc_kernel", tw, tx, tokens,
                      experts, hidden, logits, part, error);
}

int launch_router_tc(const uint16_t *x, const uint16_t *router, int tokens, int hidden, int experts,
                     uint16_t *logits, float *part, int ks, int32_t *error, cudaStream_t stream) {
    LRB_REQUIRE(hidden % (kK * (part ? ks : 1)) == 0, "router: hidden %d does not split into %d K splits", hidden, ks);
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(router) % 16 == 0,
                "router: x and router must be 16-byte aligned");
    if (router_tc_bn(tokens) == 64)
        return launch_router_tc_bn<64>(x, router, tokens, hidden, experts, logits, part, ks, error, stream);
    return launch_router_tc_bn<32>(x, router, tokens, hidden, experts, logits, part, ks, error, stream);
}

}  // namespace lrb
