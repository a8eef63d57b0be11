// Descriptor-driven copies of expert rows into BF16 slots, with in-register
// decode of the two lossless codecs.  Tables, layouts and results are those of
// edge35b/bf16_gather_ada.cu (gather_bf16*, :36-198); the work split is this
// file's own: every CTA owns a contiguous share of one (row, bank) and every
// 16-byte unit of the row is written whatever the stripe count.
//
// Row codec (edge35b/bf16_expert_codec.py:40-51): n bytes of sign|7-bit
// fraction, n/2 bytes of 4-bit exponent deltas from `base`, then int32 escape
// indices (ascending) and their uint16 values.  A unit of 16 output bytes (8
// values) reads 8 sign/fraction bytes and 4 delta bytes.
//
// Tile codec (cpu_bf16_reads.h:16-52): 256-value tiles of 256 low bytes + 128
// bytes of 4-bit codes (3-bit offset from the tile base | sign << 3); base 255
// is a raw tile.  One warp decodes one tile, 16 output bytes per lane.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace lrb {

namespace {

template <bool L2Only>
__device__ __forceinline__ uint4 load16(const void *p) {
    if constexpr (L2Only) {
        uint4 v;
        asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
        return v;
    } else {
        return ld_stream(p);
    }
}

template <bool L2Only>
__device__ __forceinline__ uint2 load8(const void *p) {
    uint2 v;
    if constexpr (L2Only) asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    else asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

template <bool L2Only>
__device__ __forceinline__ uint32_t load4(const void *p) {
    uint32_t v;
    if constexpr (L2Only) asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    else asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// Two values of the row codec: bytes sf (sign<<7 | fraction) and a delta byte.
__device__ __forceinline__ uint32_t row_pair(uint32_t sf2, uint32_t deltas2, uint32_t base) {
    const uint32_t a = sf2 & 0xffu, b = (sf2 >> 8) & 0xffu;
    const uint32_t lo = ((a & 0x80u) << 8) | ((base + (deltas2 & 0xfu)) << 7) | (a & 0x7fu);
    const uint32_t hi = ((b & 0x80u) << 8) | ((base + ((deltas2 >> 4) & 0xfu)) << 7) | (b & 0x7fu);
    return (lo & 0xffffu) | (hi << 16);
}

__device__ __forceinline__ uint4 row_unit(uint2 sf, uint32_t deltas, uint32_t base) {
    return make_uint4(row_pair(sf.x, deltas, base), row_pair(sf.x >> 16, deltas >> 8, base),
                      row_pair(sf.y, deltas >> 16, base), row_pair(sf.y >> 16, deltas >> 24, base));
}

// Two values of the tile codec: low bytes and two 4-bit codes.
__device__ __forceinline__ uint32_t tile_pair(uint32_t low2, uint32_t codes2, uint32_t base) {
    const uint32_t c0 = codes2 & 0xfu, c1 = (codes2 >> 4) & 0xfu;
    const uint32_t h0 = ((base + (c0 & 7u)) | ((c0 & 8u) << 4)) & 0xffu;
    const uint32_t h1 = ((base + (c1 & 7u)) | ((c1 & 8u) << 4)) & 0xffu;
    return (low2 & 0xffu) | (h0 << 8) | (((low2 >> 8) & 0xffu) << 16) | (h1 << 24);
}

__device__ __forceinline__ uint4 tile_unit(uint2 low, uint32_t codes, uint32_t base) {
    return make_uint4(tile_pair(low.x, codes, base), tile_pair(low.x >> 16, codes >> 8, base),
                      tile_pair(low.y, codes >> 16, base), tile_pair(low.y >> 16, codes >> 24, base));
}

template <bool L2Only>
__device__ __forceinline__ void copy_units(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int64_t begin,
                                           int64_t end) {
    const int64_t step = blockDim.x;
    int64_t i = begin + threadIdx.x;
    for (; i + 3 * step < end; i += 4 * step) {
        const uint4 a = load16<L2Only>(src + i), b = load16<L2Only>(src + i + step);
        const uint4 c = load16<L2Only>(src + i + 2 * step), d = load16<L2Only>(src + i + 3 * step);
        dst[i] = a;
        dst[i + step] = b;
        dst[i + 2 * step] = c;
        dst[i + 3 * step] = d;
    }
    for (; i < end; i += step) dst[i] = load16<L2Only>(src + i);
}

__device__ __forceinline__ int first_not_below(const int32_t *v, int n, int64_t key) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = lo + (hi - lo) / 2;
        if (v[mid] < key) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

}  // namespace

// Decode (or copy, base < 0) this CTA's share of one row-codec row into dst:
// 16-byte output units [units*stripe/stripes, units*(stripe+1)/stripes), then
// repair the escapes that fall inside that share.
template <bool L2Only>
__device__ __forceinline__ void row_codec_share(const uint8_t *src, int64_t base, int64_t escapes, int64_t row_bytes,
                                                uint4 *dst, int stripe, int stripes) {
    const int64_t units = row_bytes >> 4;
    const int64_t begin = units * stripe / stripes, end = units * (stripe + 1) / stripes;
    if (base < 0) {
        copy_units<L2Only>(reinterpret_cast<const uint4 *>(src), dst, begin, end);
        return;
    }
    const uint8_t *deltas = src + row_bytes / 2;
    const uint32_t b32 = static_cast<uint32_t>(base);
    // Pairs of units per thread: 16 sign/fraction bytes + 8 delta bytes per
    // load pair, two pairs in flight -- wide requests over the host link.
    int64_t i = begin;
    if ((i & 1) && i < end) {
        if (threadIdx.x == 0) dst[i] = row_unit(load8<L2Only>(src + 8 * i), load4<L2Only>(deltas + 4 * i), b32);
        ++i;
    }
    const int64_t pairs_end = i + ((end - i) & ~int64_t(1));
    const int64_t step = 2 * static_cast<int64_t>(blockDim.x);
    int64_t j = i + 2 * threadIdx.x;
    for (; j + step < pairs_end; j += 2 * step) {
        const uint4 sa = load16<L2Only>(src + 8 * j), sb = load16<L2Only>(src + 8 * (j + step));
        const uint2 da = load8<L2Only>(deltas + 4 * j), db = load8<L2Only>(deltas + 4 * (j + step));
        dst[j] = row_unit(make_uint2(sa.x, sa.y), da.x, b32);
        dst[j + 1] = row_unit(make_uint2(sa.z, sa.w), da.y, b32);
        dst[j + step] = row_unit(make_uint2(sb.x, sb.y), db.x, b32);
        dst[j + step + 1] = row_unit(make_uint2(sb.z, sb.w), db.y, b32);
    }
    for (; j < pairs_end; j += step) {
        const uint4 sa = load16<L2Only>(src + 8 * j);
        const uint2 da = load8<L2Only>(deltas + 4 * j);
        dst[j] = row_unit(make_uint2(sa.x, sa.y), da.x, b32);
        dst[j + 1] = row_unit(make_uint2(sa.z, sa.w), da.y, b32);
    }
    if (pairs_end < end && threadIdx.x == 0)
        dst[pairs_end] = row_unit(load8<L2Only>(src + 8 * pairs_end), load4<L2Only>(deltas + 4 * pairs_end), b32);
    if (escapes > 0) {
        // The escape list is sorted, so this CTA repairs exactly its own values
        // after all of its decode stores are done.
        __shared__ int range[2];
        const int32_t *where = reinterpret_cast<const int32_t *>(src + row_bytes / 2 + row_bytes / 4);
        const uint16_t *value = reinterpret_cast<const uint16_t *>(where + escapes);
        if (threadIdx.x == 0) {
            range[0] = first_not_below(where, static_cast<int>(escapes), begin * 8);
            range[1] = first_not_below(where, static_cast<int>(escapes), end * 8);
        }
        __syncthreads();
        uint16_t *out = reinterpret_cast<uint16_t *>(dst);
        for (int j = range[0] + threadIdx.x; j < range[1]; j += blockDim.x) out[where[j]] = value[j];
    }
}

template <bool L2Only>
__global__ void __launch_bounds__(1024) gather_row_codec_kernel(const int64_t *__restrict__ descriptors,
                                                                 const int64_t *__restrict__ destinations,
                                                                 const int64_t *__restrict__ sizes,
                                                                 const int32_t *__restrict__ source_ids,
                                                                 const int32_t *__restrict__ destination_ids,
                                                                 const int64_t *__restrict__ count, int experts) {
    const int row = blockIdx.z;
    if (row >= *count) return;
    const int bank = blockIdx.y;
    const int64_t *d = descriptors + (static_cast<int64_t>(bank) * experts + source_ids[row]) * 3;
    const int64_t row_bytes = sizes[bank];
    uint4 *dst = reinterpret_cast<uint4 *>(destinations[bank] + static_cast<int64_t>(destination_ids[row]) * row_bytes);
    row_codec_share<L2Only>(reinterpret_cast<const uint8_t *>(d[0]), d[1], d[2], row_bytes, dst, blockIdx.x,
                            gridDim.x);
}

// The layer's host-resident stage with packed banks: active expert g (g-th
// ascending id) decodes from descriptors[bank][active[g]] into HBM slot g of
// bank 0 (gate_up) or 1 (down), bank = bank0 + blockIdx.y.  Grid (stripes,
// banks, max_slots), 256 threads.
//
// The packed bytes cross the host link as large bulk copies: thread 0 streams
// the CTA's share of the sign/fraction and exponent-delta regions into a ring
// of shared-memory stages (mbarrier completion), and the CTA decodes each stage
// into HBM while the next ones are in flight.  Shares start and end on 4-unit
// boundaries so every bulk copy is 16-byte aligned.  Raw rows (base < 0) and
// escape repair use plain loads.  Waits are bounded; a timeout raises *error.
constexpr int kStageUnits = 1024;   // 16 KiB of output per ring stage
constexpr int kStageRing = 3;

// Entry g < *num_active stages expert active[g] into slot slot_of_entry[g]
// (or slot g when slot_of_entry is null).
__global__ void __launch_bounds__(256) stage_row_codec_kernel(const int64_t *__restrict__ descriptors,
                                                              const int32_t *__restrict__ active,
                                                              const int32_t *__restrict__ num_active, int experts,
                                                              const int32_t *__restrict__ slot_of_entry,
                                                              uint16_t *gate_up_slots, uint16_t *down_slots,
                                                              int64_t gate_up_bytes, int64_t down_bytes,
                                                              int32_t *error, int bank0) {
    __shared__ __align__(128) uint8_t sf_buf[kStageRing][kStageUnits * 8];
    __shared__ __align__(128) uint8_t dl_buf[kStageRing][kStageUnits * 4];
    __shared__ __align__(8) uint64_t bars[kStageRing];
    __shared__ int range[2];
    grid_dependency_wait();
    grid_dependency_trigger();
    const int g = blockIdx.z;
    if (g >= *num_active) return;
    const int bank = bank0 + static_cast<int>(blockIdx.y);
    const int64_t *d = descriptors + (static_cast<int64_t>(bank) * experts + active[g]) * 3;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(d[0]);
    const int64_t base = d[1], escapes = d[2];
    const int64_t row_bytes = bank == 0 ? gate_up_bytes : down_bytes;
    const int64_t slot = slot_of_entry ? slot_of_entry[g] : g;
    uint4 *dst = reinterpret_cast<uint4 *>(bank == 0 ? gate_up_slots + slot * (gate_up_bytes / 2)
                                                     : down_slots + slot * (down_bytes / 2));
    const int64_t units = row_bytes >> 4;
    if (base < 0 || (units & 3)) {
        row_codec_share<false>(src, base, escapes, row_bytes, dst, blockIdx.x, gridDim.x);
        return;
    }
    const int64_t quads = units >> 2;
    const int64_t begin = 4 * (quads * blockIdx.x / gridDim.x), end = 4 * (quads * (blockIdx.x + 1) / gridDim.x);
    const uint8_t *deltas = src + row_bytes / 2;
    const uint32_t b32 = static_cast<uint32_t>(base);
    const int chunks = static_cast<int>((end - begin + kStageUnits - 1) / kStageUnits);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStageRing; ++s) sm100::mbar_init(&bars[s], 1);
        sm100::fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int c) {
        const int s = c % kStageRing;
        const int64_t u0 = begin + static_cast<int64_t>(c) * kStageUnits;
        const uint32_t n = static_cast<uint32_t>(min(static_cast<int64_t>(kStageUnits), end - u0));
        sm100::mbar_expect_tx(&bars[s], 12 * n);
        sm100::bulk_load(sf_buf[s], src + 8 * u0, 8 * n, &bars[s]);
        sm100::bulk_load(dl_buf[s], deltas + 4 * u0, 4 * n, &bars[s]);
    };
    if (threadIdx.x == 0)
        for (int c = 0; c < min(chunks, kStageRing); ++c) issue(c);
    bool ok = true;
    for (int c = 0; c < chunks; ++c) {
        const int s = c % kStageRing;
        const uint32_t parity = (c / kStageRing) & 1;
        if (!sm100::mbar_try_wait(&bars[s], parity)) {
            uint64_t t0;
            asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
            while (!sm100::mbar_try_wait(&bars[s], parity)) {
                uint64_t t;
                asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
                if (t - t0 > 2000000000ull) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) break;
        const int64_t u0 = begin + static_cast<int64_t>(c) * kStageUnits;
        const int n = static_cast<int>(min(static_cast<int64_t>(kStageUnits), end - u0));
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint2 sf = *reinterpret_cast<const uint2 *>(sf_buf[s] + 8 * i);
            const uint32_t dl = *reinterpret_cast<const uint32_t *>(dl_buf[s] + 4 * i);
            dst[u0 + i] = row_unit(sf, dl, b32);
        }
        __syncthreads();  // stage s is free again
        if (threadIdx.x == 0 && c + kStageRing < chunks) issue(c + kStageRing);
    }
    if (!ok) {
        // Let the copies this CTA issued land before it leaves; then report.
        if (threadIdx.x == 0) {
            atomicExch(error, 4);
            for (int s = 0; s < kStageRing; ++s) {
                uint64_t t0, t;
                asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
                do {
                    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
                } while (!sm100::mbar_try_wait(&bars[s], 0) && !sm100::mbar_try_wait(&bars[s], 1) &&
                         t - t0 < 2000000000ull);
            }
        }
        __syncthreads();
        return;
    }
    if (escapes > 0) {
        const int32_t *where = reinterpret_cast<const int32_t *>(src + row_bytes / 2 + row_bytes / 4);
        const uint16_t *value = reinterpret_cast<const uint16_t *>(where + escapes);
        if (threadIdx.x == 0) {
            range[0] = first_not_below(where, static_cast<int>(escapes), begin * 8);
            range[1] = first_not_below(where, static_cast<int>(escapes), end * 8);
        }
        __syncthreads();
        uint16_t *out = reinterpret_cast<uint16_t *>(dst);
        for (int j = range[0] + threadIdx.x; j < range[1]; j += blockDim.x) out[where[j]] = value[j];
    }
}

int launch_stage_row_codec(const int64_t *descriptors, const int32_t *active, const int32_t *num_active, int experts,
                           int max_slots, uint16_t *gate_up_slots, uint16_t *down_slots, int64_t gate_up_bytes,
                           int64_t down_bytes, int32_t *error, cudaStream_t stream, const int32_t *slot_of_entry,
                           int bank0, int banks) {
    return launch_pdl(stage_row_codec_kernel, dim3(64, banks, max_slots), dim3(256), 0, stream,
                      "stage_row_codec_kernel", descriptors, active, num_active, experts, slot_of_entry, gate_up_slots,
                      down_slots, gate_up_bytes, down_bytes, error, bank0);
}

template <bool AllowCompact>
__global__ void __launch_bounds__(1024) gather_tiles_kernel(const int64_t *__restrict__ descriptors,
                                                            const int64_t *__restrict__ destinations,
                                                            const int64_t *__restrict__ sizes,
                                                            const int32_t *__restrict__ source_ids,
                                                            const int32_t *__restrict__ destination_ids,
                                                            const int64_t *__restrict__ count, int experts) {
    const int row = blockIdx.z;
    if (row >= *count) return;
    const int bank = blockIdx.y;
    const int64_t *d = descriptors + (static_cast<int64_t>(bank) * experts + source_ids[row]) * 3;
    const uint8_t *packed = reinterpret_cast<const uint8_t *>(d[0]);
    const uint8_t *bases = reinterpret_cast<const uint8_t *>(d[1]);
    const uint4 *raw = reinterpret_cast<const uint4 *>(d[2]);
    const int64_t row_bytes = sizes[bank];
    uint4 *dst = reinterpret_cast<uint4 *>(destinations[bank] + static_cast<int64_t>(destination_ids[row]) * row_bytes);
    const int64_t tiles = row_bytes / 512;
    const int64_t begin = tiles * blockIdx.x / gridDim.x, end = tiles * (blockIdx.x + 1) / gridDim.x;
    if (bases == nullptr) {
        copy_units<false>(raw, dst, begin * 32, end * 32);
        return;
    }
    const bool compact = AllowCompact && d[2] == -1;
    const int lane = threadIdx.x & 31;
    for (int64_t tile = begin + (threadIdx.x >> 5); tile < end; tile += blockDim.x >> 5) {
        uint32_t header = 0;
        if (lane == 0) header = compact ? load4<false>(bases + 4 * tile) : bases[tile];
        header = __shfl_sync(0xffffffffu, header, 0);
        const uint32_t base = header & 0xffu;
        const uint8_t *tile_data = packed + tile * 384 + (compact ? static_cast<int64_t>(header >> 8) * 128 : 0);
        const int64_t i = tile * 32 + lane;
        if (base == 255u) {
            dst[i] = compact ? load16<false>(tile_data + 16 * lane) : load16<false>(raw + i);
        } else {
            dst[i] = tile_unit(load8<false>(tile_data + 8 * lane), load4<false>(tile_data + 256 + 4 * lane), base);
        }
    }
}

}  // namespace lrb

extern "C" int moe_gather_rows(const int64_t *descriptors, const int64_t *destinations, const int64_t *sizes,
                               const int32_t *source_ids, const int32_t *destination_ids, const int64_t *count,
                               int experts, int banks, int max_copies, int codec, int stripes, int threads,
                               void *stream) {
    LRB_REQUIRE(descriptors && destinations && sizes && source_ids && destination_ids && count,
                "moe_gather_rows: null table");
    LRB_REQUIRE(experts >= 1, "moe_gather_rows: experts %d < 1", experts);
    LRB_REQUIRE(banks >= 1 && banks <= 65535, "moe_gather_rows: banks %d outside [1, 65535]", banks);
    LRB_REQUIRE(max_copies >= 0 && max_copies <= 65535, "moe_gather_rows: max_copies %d outside [0, 65535]",
                max_copies);
    LRB_REQUIRE(stripes >= 1 && stripes <= (1 << 20), "moe_gather_rows: stripes %d outside [1, 2^20]", stripes);
    LRB_REQUIRE(threads >= 32 && threads <= 1024 && threads % 32 == 0,
                "moe_gather_rows: threads %d must be a multiple of 32 in [32, 1024]", threads);
    if (max_copies == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    const dim3 grid(stripes, banks, max_copies);
    cudaStream_t s = lrb::as_stream(stream);
    switch (codec) {
        case MOE_CODEC_ROW:
            lrb::gather_row_codec_kernel<false><<<grid, threads, 0, s>>>(descriptors, destinations, sizes, source_ids,
                                                                         destination_ids, count, experts);
            break;
        case MOE_CODEC_ROW_L2:
            lrb::gather_row_codec_kernel<true><<<grid, threads, 0, s>>>(descriptors, destinations, sizes, source_ids,
                                                                        destination_ids, count, experts);
            break;
        case MOE_CODEC_TILES:
            lrb::gather_tiles_kernel<false><<<grid, threads, 0, s>>>(descriptors, destinations, sizes, source_ids,
                                                                     destination_ids, count, experts);
            break;
        case MOE_CODEC_RESIDENT:
            lrb::gather_tiles_kernel<true><<<grid, threads, 0, s>>>(descriptors, destinations, sizes, source_ids,
                                                                    destination_ids, count, experts);
            break;
        default:
            return lrb::set_error(MOE_EINVAL, "moe_gather_rows: unknown codec %d", codec);
    }
    LRB_LAUNCHED("moe_gather_rows");
    return MOE_OK;
}
