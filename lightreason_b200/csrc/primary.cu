// Packed primary-cache staging and refill: the selected experts of a step are
// written as BF16 rows for the expert GEMM, read from a packed cache slot on a
// hit or from the host source (or a device replica) on a miss, and a miss
// refills the slot in the same pass.  Tables and results are those of
// edge35b/bf16_gather_ada.cu stage_bf16_primary (:202-308) and
// gather_bf16_compact_tail (:312-381); the work split is this file's own.
//
// Slot format (the tile codec of cpu_bf16_reads.h:16-52, compact): tiles of
// 256 values back to back, 384 bytes for a packed tile and 512 for a raw one
// (base 255), so tile t of a row starts at t*384 + 128 * (raw tiles before t).
// The raw-tile counts come from a prefix table per (bank, expert, 32 tiles):
// (raw tiles before the group << 32) | bitmask of the group's raw tiles.
//
// Each warp owns runs of 32 consecutive tiles: its lanes first read the 32
// tiles' bases / headers / prefix words together, then the warp walks the run
// one tile at a time, 16 output bytes per lane, with the tile's parameters
// broadcast by shuffle.
#include "common.cuh"
#include "kernels.cuh"

namespace lrb {

namespace {

constexpr int kTileBytes = 512, kPackedTileBytes = 384, kStripes = 16;

__device__ __forceinline__ uint32_t raw_tiles_before(const uint64_t *prefix_row, int tile) {
    const uint64_t group = prefix_row[tile >> 5];
    return static_cast<uint32_t>(group >> 32) +
           __popc(static_cast<uint32_t>(group) & ((1u << (tile & 31)) - 1u));
}

// Tile-codec encode of 8 values (one 16-byte unit) of a packable tile: the 8
// low bytes and 8 4-bit codes (exponent offset from base | sign << 3).
__device__ __forceinline__ void tile_encode(uint4 v, uint32_t base, uint2 *low, uint32_t *codes) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t lows[4], c = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x = w[j];
        lows[j] = (x & 0xffu) | ((x >> 8) & 0xff00u);
        const uint32_t a = ((((x >> 8) & 0x7fu) - base) & 7u) | ((x >> 12) & 8u);
        const uint32_t b = ((((x >> 24) & 0x7fu) - base) & 7u) | ((x >> 28) & 8u);
        c |= (a | (b << 4)) << (8 * j);
    }
    *low = make_uint2(lows[0] | (lows[1] << 16), lows[2] | (lows[3] << 16));
    *codes = c;
}

__device__ __forceinline__ uint32_t tile_pair2(uint32_t low2, uint32_t codes2, uint32_t base) {
    const uint32_t c0 = codes2 & 0xfu, c1 = (codes2 >> 4) & 0xfu;
    const uint32_t h0 = ((base + (c0 & 7u)) | ((c0 & 8u) << 4)) & 0xffu;
    const uint32_t h1 = ((base + (c1 & 7u)) | ((c1 & 8u) << 4)) & 0xffu;
    return (low2 & 0xffu) | (h0 << 8) | (((low2 >> 8) & 0xffu) << 16) | (h1 << 24);
}

__device__ __forceinline__ uint4 tile_decode(uint2 low, uint32_t codes, uint32_t base) {
    return make_uint4(tile_pair2(low.x, codes, base), tile_pair2(low.x >> 16, codes >> 8, base),
                      tile_pair2(low.y, codes >> 16, base), tile_pair2(low.y >> 16, codes >> 24, base));
}

__device__ __forceinline__ uint4 ld16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint2 ld8(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ uint32_t ld4(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ void copy_row_units(const uint4 *src, uint4 *dst, int64_t begin, int64_t end) {
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

// plan: int32 [3, max_rows] (expert, slot, miss); layouts: int64 [banks, 5]
// (packed slot base, raw slot base, work rows base, packed slot stride, row
// bytes); sources / miss_sources: descriptors [banks, E, 3].
__global__ void __launch_bounds__(256) stage_primary_kernel(
    const int64_t *__restrict__ sources, const int64_t *__restrict__ miss_sources, const int64_t *__restrict__ layouts,
    const int64_t *__restrict__ prefix_tables, const int32_t *__restrict__ plan, const int32_t *__restrict__ count,
    int experts, int packed_slots, int max_rows) {
    const int row = blockIdx.z;
    if (row >= *count) return;
    const int bank = blockIdx.y;
    const int expert = plan[row], slot = plan[max_rows + row];
    const bool miss = plan[2 * max_rows + row] != 0;
    const bool in_packed = slot >= 0 && slot < packed_slots;
    if (!miss && slot >= packed_slots) return;  // raw-slot hit: the GEMM reads the slot in place
    const int64_t *layout = layouts + bank * 5;
    const int64_t row_bytes = layout[4];
    uint8_t *cached = slot < 0 ? nullptr
                      : in_packed ? reinterpret_cast<uint8_t *>(layout[0] + static_cast<int64_t>(slot) * layout[3])
                                  : reinterpret_cast<uint8_t *>(layout[1] + static_cast<int64_t>(slot - packed_slots) *
                                                                                row_bytes);
    uint4 *dest = slot >= packed_slots ? reinterpret_cast<uint4 *>(cached)
                                       : reinterpret_cast<uint4 *>(layout[2] + static_cast<int64_t>(row + 1) * row_bytes);
    const int64_t *src = sources + (static_cast<int64_t>(bank) * experts + expert) * 3;
    const int64_t *ref = miss_sources + (static_cast<int64_t>(bank) * experts + expert) * 3;
    const uint8_t *code = reinterpret_cast<const uint8_t *>(src[0]);
    const uint8_t *bases = reinterpret_cast<const uint8_t *>(src[1]);
    const uint4 *raw = reinterpret_cast<const uint4 *>(src[2]);
    const bool replica_packed = miss && ref[2] == -1;
    const bool replica_raw = miss && ref[1] == 0 && ref[2] != src[2];
    const uint8_t *replica = reinterpret_cast<const uint8_t *>(ref[0]);
    const uint32_t *replica_headers = reinterpret_cast<const uint32_t *>(ref[1]);
    const uint4 *replica_row = reinterpret_cast<const uint4 *>(ref[2]);
    const int tiles = static_cast<int>(row_bytes / kTileBytes);
    const int t_begin = static_cast<int>(static_cast<int64_t>(tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(tiles) * (blockIdx.x + 1) / gridDim.x);

    if (!in_packed && !replica_packed && (replica_raw || bases == nullptr)) {
        copy_row_units(replica_raw ? replica_row : raw, dest, static_cast<int64_t>(t_begin) * 32,
                       static_cast<int64_t>(t_end) * 32);
        return;
    }
    const uint64_t *prefix_row =
        reinterpret_cast<const uint64_t *>(prefix_tables[bank]) + static_cast<int64_t>(expert) * (tiles / 32);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    for (int run = t_begin + 32 * warp; run < t_end; run += 32 * warps) {
        // the run's per-tile parameters, one tile per lane
        const int my_tile = run + lane;
        uint32_t my_base = 255u, my_prior = 0u, my_roff = 0u;
        if (my_tile < t_end) {
            if (replica_packed) {
                const uint32_t header = replica_headers[my_tile];
                my_roff = static_cast<uint32_t>(my_tile) * kPackedTileBytes + (header >> 8) * 128u;
                if (!in_packed) my_base = header & 0xffu;
            }
            if (in_packed || !replica_packed) my_base = bases[my_tile];
            if (in_packed) my_prior = raw_tiles_before(prefix_row, my_tile);
        }
        const int n = min(32, t_end - run);
        for (int j = 0; j < n; ++j) {
            const int tile = run + j;
            const uint32_t base = __shfl_sync(0xffffffffu, my_base, j);
            const uint32_t prior = __shfl_sync(0xffffffffu, my_prior, j);
            const uint32_t roff = __shfl_sync(0xffffffffu, my_roff, j);
            const int64_t offset = static_cast<int64_t>(tile) * kPackedTileBytes + static_cast<int64_t>(prior) * 128;
            const int64_t i = static_cast<int64_t>(tile) * 32 + lane;
            uint4 v;
            if (base == 255u) {
                v = replica_packed           ? ld16(replica + roff + 16 * lane)
                    : (in_packed && !miss)   ? ld16(cached + offset + 16 * lane)
                    : replica_raw            ? replica_row[i]
                                             : raw[i];
                if (in_packed && miss) *reinterpret_cast<uint4 *>(cached + offset + 16 * lane) = v;
            } else {
                uint2 low;
                uint32_t codes;
                if (replica_raw) {
                    v = replica_row[i];
                    tile_encode(v, base, &low, &codes);
                } else {
                    const uint8_t *data = replica_packed           ? replica + roff
                                          : (in_packed && !miss)   ? cached + offset
                                                                   : code + static_cast<int64_t>(tile) * kPackedTileBytes;
                    low = ld8(data + 8 * lane);
                    codes = ld4(data + 256 + 4 * lane);
                    v = tile_decode(low, codes, base);
                }
                if (in_packed && miss) {
                    *reinterpret_cast<uint2 *>(cached + offset + 8 * lane) = low;
                    *reinterpret_cast<uint32_t *>(cached + offset + 256 + 4 * lane) = codes;
                }
            }
            dest[i] = v;
        }
    }
}

// entries: int32 [2, max_rows] (tail entry or -1, resident flag); tail: int64
// [banks, 2] (entry storage base, entry stride).
__global__ void __launch_bounds__(256) compact_tail_kernel(
    const int64_t *__restrict__ sources, const int64_t *__restrict__ destinations, const int64_t *__restrict__ sizes,
    const int64_t *__restrict__ prefix_tables, const int64_t *__restrict__ tail, const int32_t *__restrict__ source_ids,
    const int32_t *__restrict__ dest_ids, const int64_t *__restrict__ count, const int32_t *__restrict__ entries,
    const int64_t *__restrict__ resident, int experts, int max_rows) {
    const int row = blockIdx.z;
    if (row >= *count) return;
    const int bank = blockIdx.y;
    const int expert = source_ids[row];
    const int entry = entries[row];
    const bool is_resident = entries[max_rows + row] != 0;
    const int64_t row_bytes = sizes[bank];
    uint4 *dest = reinterpret_cast<uint4 *>(destinations[bank] + static_cast<int64_t>(dest_ids[row]) * row_bytes);
    const int64_t *d = (is_resident ? resident : sources) + (static_cast<int64_t>(bank) * experts + expert) * 3;
    const uint8_t *mapped = reinterpret_cast<const uint8_t *>(d[0]);
    const uint8_t *bases = reinterpret_cast<const uint8_t *>(d[1]);
    const uint4 *raw = reinterpret_cast<const uint4 *>(d[2]);
    uint8_t *storage = entry < 0 ? nullptr
                                 : reinterpret_cast<uint8_t *>(tail[bank * 2] + static_cast<int64_t>(entry) * tail[bank * 2 + 1]);
    const int tiles = static_cast<int>(row_bytes / kTileBytes);
    const int t_begin = static_cast<int>(static_cast<int64_t>(tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(tiles) * (blockIdx.x + 1) / gridDim.x);
    if (bases == nullptr) {
        copy_row_units(raw, dest, static_cast<int64_t>(t_begin) * 32, static_cast<int64_t>(t_end) * 32);
        return;
    }
    const bool replica = d[2] == -1;
    const uint64_t *prefix_row =
        reinterpret_cast<const uint64_t *>(prefix_tables[bank]) + static_cast<int64_t>(expert) * (tiles / 32);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    for (int run = t_begin + 32 * warp; run < t_end; run += 32 * warps) {
        const int my_tile = run + lane;
        uint32_t my_header = 0;
        if (my_tile < t_end) {
            if (replica) {
                my_header = reinterpret_cast<const uint32_t *>(bases)[my_tile];
            } else {
                my_header = bases[my_tile];
                if (storage) my_header |= raw_tiles_before(prefix_row, my_tile) << 8;
            }
        }
        const int n = min(32, t_end - run);
        for (int j = 0; j < n; ++j) {
            const int tile = run + j;
            const uint32_t header = __shfl_sync(0xffffffffu, my_header, j);
            const uint32_t base = header & 0xffu;
            const int64_t offset = static_cast<int64_t>(tile) * kPackedTileBytes + static_cast<int64_t>(header >> 8) * 128;
            const int64_t i = static_cast<int64_t>(tile) * 32 + lane;
            if (base == 255u) {
                const uint4 v = is_resident ? ld16(storage + offset + 16 * lane)
                                : replica   ? ld16(mapped + offset + 16 * lane)
                                            : raw[i];
                dest[i] = v;
                if (!is_resident && storage) *reinterpret_cast<uint4 *>(storage + offset + 16 * lane) = v;
                continue;
            }
            const uint8_t *data = is_resident ? storage + offset
                                              : mapped + (replica ? offset : static_cast<int64_t>(tile) * kPackedTileBytes);
            const uint2 low = ld8(data + 8 * lane);
            const uint32_t codes = ld4(data + 256 + 4 * lane);
            dest[i] = tile_decode(low, codes, base);
            if (!is_resident && storage) {
                *reinterpret_cast<uint2 *>(storage + offset + 8 * lane) = low;
                *reinterpret_cast<uint32_t *>(storage + offset + 256 + 4 * lane) = codes;
            }
        }
    }
}

}  // namespace lrb

extern "C" int moe_stage_primary(const int64_t *sources, const int64_t *miss_sources, const int64_t *layouts,
                                 const int64_t *prefix_tables, const int32_t *plan, const int32_t *count, int experts,
                                 int packed_slots, int max_rows, int banks, void *stream) {
    LRB_REQUIRE(sources && miss_sources && layouts && prefix_tables && plan && count,
                "moe_stage_primary: null table");
    LRB_REQUIRE(experts >= 1 && packed_slots >= 0, "moe_stage_primary: bad experts %d / packed_slots %d", experts,
                packed_slots);
    LRB_REQUIRE(banks >= 1 && banks <= 65535 && max_rows >= 0 && max_rows <= 65535,
                "moe_stage_primary: banks %d / max_rows %d out of range", banks, max_rows);
    if (max_rows == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    lrb::stage_primary_kernel<<<dim3(lrb::kStripes, banks, max_rows), 256, 0, lrb::as_stream(stream)>>>(
        sources, miss_sources, layouts, prefix_tables, plan, count, experts, packed_slots, max_rows);
    LRB_LAUNCHED("stage_primary_kernel");
    return MOE_OK;
}

extern "C" int moe_gather_compact_tail(const int64_t *sources, const int64_t *destinations, const int64_t *sizes,
                                       const int64_t *prefix_tables, const int64_t *tail, const int32_t *source_ids,
                                       const int32_t *dest_ids, const int64_t *count, const int32_t *entries,
                                       const int64_t *resident, int experts, int max_rows, int banks, void *stream) {
    LRB_REQUIRE(sources && destinations && sizes && prefix_tables && tail && source_ids && dest_ids && count &&
                    entries && resident,
                "moe_gather_compact_tail: null table");
    LRB_REQUIRE(experts >= 1, "moe_gather_compact_tail: experts %d < 1", experts);
    LRB_REQUIRE(banks >= 1 && banks <= 65535 && max_rows >= 0 && max_rows <= 65535,
                "moe_gather_compact_tail: banks %d / max_rows %d out of range", banks, max_rows);
    if (max_rows == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    lrb::compact_tail_kernel<<<dim3(lrb::kStripes, banks, max_rows), 256, 0, lrb::as_stream(stream)>>>(
        sources, destinations, sizes, prefix_tables, tail, source_ids, dest_ids, count, entries, resident, experts,
        max_rows);
    LRB_LAUNCHED("compact_tail_kernel");
    return MOE_OK;
}
