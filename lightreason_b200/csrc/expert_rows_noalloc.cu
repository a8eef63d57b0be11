// moe_expert_block_rows_noalloc: the pointer-table expert rows of
// moe_expert_block_rows without a caller workspace.
//
// Who needs it: callers that hold nothing but raw device pointers and cannot
// obtain device memory themselves -- for example a plain C or C++ worker that
// replaces the reference's cpu_experts.c call (its signature carries the
// weight pointers, the input, the output and a count, and no buffer for the
// intermediate activations), or a serving loop that reserves all of its device
// memory at start-up and is not permitted to allocate while it serves.  Such a
// caller cannot hand moe_expert_block_rows the [pairs, 512] BF16 workspace it
// needs, so this entry point keeps that workspace inside the library.
//
// How: the activations live in a fixed array in device memory, g_pair_scratch
// below, sized for the largest table the workspace entry point accepts (128
// pairs x 512 BF16 = 128 KiB).  Every GPU that loads this library holds that
// array until the process exits.  Nothing here calls cudaMalloc, cudaFree or
// any other allocating routine.
//
// Set-up: host code cannot use the array's name as a device address (on the
// host it only names a stand-in object), so the device address is looked up
// with cudaGetSymbolAddress once per device, with that device current, the
// first time this entry point runs on it; later calls reuse the cached
// address.  Make that first call on each device before any stream capture.
// The cached address lives as long as the process: after cudaDeviceReset (or
// any reset of the device's primary context) the module is loaded again at a
// new address, so this entry point must not be used on that device again.
//
// Sharing: all calls on a device use the same array, and it keeps whatever the
// last call left in it.  Nothing in it has to start at zero: within one call,
// the gate/up kernel writes every activation the down kernel then reads, in
// stream order.  Calls whose kernels can overlap on the GPU (different streams,
// or several host threads without ordering between them) race on the array;
// order such calls on one stream, or use moe_expert_block_rows with a separate
// workspace for each.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kMaxPairs = 128;   // the pair limit of moe_expert_block_rows
constexpr int kInner = 512;      // activations per pair (cpu_experts.c INNER)
constexpr size_t kScratchBytes = static_cast<size_t>(kMaxPairs) * kInner * sizeof(uint16_t);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint16_t g_pair_scratch[kMaxPairs * kInner];

std::mutex g_setup_mutex;
void *g_scratch_address[kMaxDevices] = {};

// Device address of g_pair_scratch on the current device (looked up once).
int scratch_address(void **out) {
    int device = 0;
    LRB_CUDA(cudaGetDevice(&device));
    LRB_REQUIRE(device >= 0 && device < kMaxDevices, "moe_expert_block_rows_noalloc: device %d >= %d", device,
                kMaxDevices);
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_address[device]) {
        void *ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_pair_scratch);
        if (err != cudaSuccess) return lrb::cuda_error(err, "cudaGetSymbolAddress(g_pair_scratch)");
        g_scratch_address[device] = ptr;
    }
    *out = g_scratch_address[device];
    return MOE_OK;
}

}  // namespace

extern "C" int moe_expert_block_rows_noalloc(const uint16_t *const *gate_up, const uint16_t *const *down,
                                             const uint16_t *input, const int32_t *token_ids, uint16_t *output,
                                             int tokens, int experts, void *stream) {
    LRB_REQUIRE(experts >= 0, "moe_expert_block_rows_noalloc: experts %d < 0", experts);
    LRB_REQUIRE(static_cast<size_t>(experts) * kInner * sizeof(uint16_t) <= kScratchBytes,
                "moe_expert_block_rows_noalloc: %d pairs exceed the built-in scratch of %d pairs (%zu bytes); "
                "use moe_expert_block_rows with a workspace",
                experts, kMaxPairs, kScratchBytes);
    LRB_REQUIRE(token_ids != nullptr || tokens == 1,
                "moe_expert_block_rows_noalloc: token_ids may be NULL only for one token");
    if (experts == 0) return MOE_OK;
    void *scratch = nullptr;
    if (int rc = lrb::require_sm100()) return rc;
    if (int rc = scratch_address(&scratch)) return rc;
    if (!token_ids) return moe_expert_rows(gate_up, down, input, output, experts, scratch, kScratchBytes, stream);
    return moe_expert_block_rows(gate_up, down, input, token_ids, output, tokens, experts, scratch, kScratchBytes,
                                 stream);
}
