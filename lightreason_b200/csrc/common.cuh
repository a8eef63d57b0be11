// Shared helpers for the sm_100a MoE kernels: BF16 bit handling, streaming
// loads, warp reductions and the host-side status plumbing of the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "moe_b200.h"

namespace lrb {

// ---------------------------------------------------------------- BF16 ----
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf2f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
// Round an FP32 value to the nearest BF16 and widen it back (one eager BF16 op).
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return static_cast<uint32_t>(f2bf(lo)) | (static_cast<uint32_t>(f2bf(hi)) << 16);
}

// 16-byte loads.  Weights are read once per layer step: keep them out of L1.
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_cached(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}
// Ask L2 to fetch [p, p + bytes) from DRAM (no data returns to the SM; p and
// bytes multiples of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// This CTA's slice (blockIdx.x of gridDim.x) of [p, p + bytes) into L2 (p and
// bytes multiples of 16).
__device__ __forceinline__ void prefetch_l2_slice(const void *p, size_t bytes) {
    const size_t per = (bytes / gridDim.x + 15) & ~static_cast<size_t>(15);
    const size_t off = per * blockIdx.x;
    if (off < bytes)
        prefetch_l2_bulk(static_cast<const uint8_t *>(p) + off, static_cast<uint32_t>(per < bytes - off ? per : bytes - off));
}

// acc += dot(8 BF16 weights, 8 BF16 activations) in FP32 FMA.
__device__ __forceinline__ float dot8(uint4 w, uint4 a, float acc) {
    acc = fmaf(bf16_lo(w.x), bf16_lo(a.x), acc);
    acc = fmaf(bf16_hi(w.x), bf16_hi(a.x), acc);
    acc = fmaf(bf16_lo(w.y), bf16_lo(a.y), acc);
    acc = fmaf(bf16_hi(w.y), bf16_hi(a.y), acc);
    acc = fmaf(bf16_lo(w.z), bf16_lo(a.z), acc);
    acc = fmaf(bf16_hi(w.z), bf16_hi(a.z), acc);
    acc = fmaf(bf16_lo(w.w), bf16_lo(a.w), acc);
    acc = fmaf(bf16_hi(w.w), bf16_hi(a.w), acc);
    return acc;
}

// One eager BF16 combine step on two packed values at once: acc = bf16(acc +
// bf16(v * w)), each operation rounded to nearest even (the _rn forms are
// never contracted into an FMA, which would drop the product's rounding).
// The product of two BF16 values is exact in FP32, so the BF16 multiply
// equals rbf(float(v) * float(w)); likewise the add.
__device__ __forceinline__ uint32_t bf16x2_mul_add(uint32_t acc, uint32_t v, uint32_t w2) {
    const __nv_bfloat162 p = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162 *>(&v),
                                        *reinterpret_cast<const __nv_bfloat162 *>(&w2));
    const __nv_bfloat162 r = __hadd2_rn(*reinterpret_cast<const __nv_bfloat162 *>(&acc), p);
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t bf16x2_splat(uint16_t w) { return static_cast<uint32_t>(w) * 0x10001u; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int s = 16; s; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    return v;
}

// eager SiLU on a BF16 tensor (torch computes x / (1 + exp(-x)) in FP32 and
// rounds once), the arithmetic of edge35b/cpu_experts.c:61.
__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }
__device__ __forceinline__ float sigmoid_f32(float g) { return 1.0f / (1.0f + expf(-g)); }

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while its predecessor in the stream still runs; it must call
// grid_dependency_wait() before touching anything the predecessor writes.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// -------------------------------------------------------- host status ----
int set_error(int status, const char *fmt, ...);
int cuda_error(cudaError_t err, const char *where);
int check_launch(const char *where);
int require_sm100();
// The opt-in shared-memory limit per block of the current device.
int smem_optin();
// Raise `kernel`'s dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute belongs to the (function, device) pair, so
// it is set once per device that launches the kernel (thread-safe).
int ensure_dynamic_smem(const void *kernel, int bytes, const char *name);
template <class... KArgs>
int ensure_dynamic_smem(void (*kernel)(KArgs...), int bytes, const char *name) {
    return ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), bytes, name);
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

template <class... KArgs, class... Args>
int launch_ex(bool cooperative, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
              const char *name, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 2 : 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (err != cudaSuccess) return cuda_error(err, name);
    return MOE_OK;
}

template <class... KArgs, class... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char *name,
               Args &&...args) {
    return launch_ex(false, kernel, grid, block, smem, stream, name, std::forward<Args>(args)...);
}

// As launch_pdl, in clusters of two CTAs (gridDim.x even).
template <class... KArgs, class... Args>
int launch_pdl_cluster2(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                        const char *name, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (err != cudaSuccess) return cuda_error(err, name);
    return MOE_OK;
}

// As launch_pdl, for a kernel whose CTAs wait on one another: the cooperative
// attribute makes the launch wait until every CTA of the grid can be resident
// at once (kernels on other streams may hold SMs), so the wait cannot stall
// on a CTA that has not been scheduled.
template <class... KArgs, class... Args>
int launch_pdl_cooperative(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           const char *name, Args &&...args) {
    return launch_ex(true, kernel, grid, block, smem, stream, name, std::forward<Args>(args)...);
}

}  // namespace lrb

#define LRB_REQUIRE(cond, ...)                                         \
    do {                                                               \
        if (!(cond)) return ::lrb::set_error(MOE_EINVAL, __VA_ARGS__); \
    } while (0)

#define LRB_CUDA(call)                                                    \
    do {                                                                  \
        cudaError_t err_ = (call);                                        \
        if (err_ != cudaSuccess) return ::lrb::cuda_error(err_, #call);   \
    } while (0)

#define LRB_LAUNCHED(where)                                  \
    do {                                                     \
        int rc_ = ::lrb::check_launch(where);                \
        if (rc_ != MOE_OK) return rc_;                       \
    } while (0)
