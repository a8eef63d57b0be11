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
    const uint8_t *src = reinterpret_cast<const uint8_t *>(d[0]);
    const int64_t base = d[1], escapes = d[2];
    const int64_t row_bytes = sizes[bank];
    uint4 *dst = reinterpret_cast<uint4 *>(destinations[bank] + static_cast<int64_t>(destination_ids[row]) * row_bytes);
    const int64_t units = row_bytes >> 4;
    const int64_t begin = units * blockIdx.x / gridDim.x, end = units * (blockIdx.x + 1) / gridDim.x;
    if (base < 0) {
        copy_units<L2Only>(reinterpret_cast<const uint4 *>(src), dst, begin, end);
        return;
    }
    const uint8_t *deltas = src + row_bytes / 2;
    for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x)
        dst[i] = row_unit(load8<L2Only>(src + 8 * i), load4<L2Only>(deltas + 4 * i), static_cast<uint32_t>(base));
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
