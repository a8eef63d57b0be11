// Lossless BF16 codec encoders on the GPU: the same bytes as the host
// encoders (edge35b/bf16_expert_codec.py:26-84 for the row codec,
// cpu_bf16_reads.h:16-52 pack_cpu_read_tiles for the 256-value tile codec),
// for packing expert banks where they already sit in HBM.
//
// Row codec, per row of n values (n a multiple of 8): base = the start of the
// 16-exponent window holding the most values (the first such window),
// escapes = values outside it; rows with escapes > 1% of n stay raw, the
// others are packed at 16-byte-aligned offsets in row order as
//   [n sign|fraction bytes][n/2 nibble bytes][escapes int32 indices][escapes uint16 values]
// (indices ascending).  Launch chain: plan = histograms (CTA per 8192-value
// chunk, row and chunk histograms) -> window + offsets (one CTA); pack =
// per-row scan of the chunks' escape counts (from the chunk histograms) ->
// pack (CTA per chunk).  The bank is read twice: by the histograms and by
// the pack.
//
// Tile codec: per 256-value tile, base = the smallest 7-bit exponent when the
// exponents span at most 8 values (else 255, a raw tile, whose 384 packed
// bytes are zero); packed tile = 256 low bytes + 128 bytes of 4-bit codes
// (exponent - base | sign << 3), one warp per tile.
#include "common.cuh"
#include "kernels.cuh"
#include "routing.cuh"

namespace lrb {

namespace {

constexpr int kWindow = 16;
constexpr int kChunk = 8192;  // values per CTA in the per-row passes (256 threads x 32)

}  // namespace

// Row histogram (hist[row][256], accumulated) and each chunk's own histogram
// (chunk_hist[row][chunk][256]), from which the pack pass gets its escape
// counts without reading the bank again.
__global__ void __launch_bounds__(256) rowcodec_hist_kernel(const uint16_t *__restrict__ bank, int64_t n,
                                                            int32_t *__restrict__ hist,
                                                            int32_t *__restrict__ chunk_hist) {
    // one private histogram per warp: weight exponents crowd a few bins, so a
    // shared CTA histogram would serialise on them
    __shared__ int bins[8][256];
    const int row = blockIdx.y, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) (&bins[0][0])[i] = 0;
    __syncthreads();
    const uint16_t *r = bank + static_cast<int64_t>(row) * n;
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk, end = min(n, begin + kChunk);
    for (int64_t i = begin + threadIdx.x * 8; i < end; i += blockDim.x * 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(r + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            atomicAdd(&bins[warp][(w[j] >> 7) & 0xffu], 1);
            atomicAdd(&bins[warp][(w[j] >> 23) & 0xffu], 1);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        int c = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) c += bins[k][i];
        chunk_hist[(static_cast<int64_t>(row) * gridDim.x + blockIdx.x) * 256 + i] = c;
        if (c) atomicAdd(&hist[row * 256 + i], c);
    }
}

// One CTA: meta[row] = (offset or -1 for a raw row, base, escapes) and *total.
__global__ void __launch_bounds__(1024) rowcodec_plan_kernel(const int32_t *__restrict__ hist, int rows, int64_t n,
                                                             int64_t *__restrict__ meta, int64_t *__restrict__ total) {
    __shared__ int scratch[33];
    int64_t carry = 0;
    for (int r0 = 0; r0 < rows; r0 += blockDim.x) {
        const int row = r0 + threadIdx.x;
        int64_t size = 0;
        int best = 0, best_in = -1, escapes = 0;
        bool packed = false;
        if (row < rows) {
            const int32_t *h = hist + row * 256;
            int inside = 0;
            for (int b = 0; b < kWindow; ++b) inside += h[b];
            best_in = inside;
            for (int b = 1; b + kWindow <= 256; ++b) {
                inside += h[b + kWindow - 1] - h[b - 1];
                if (inside > best_in) {
                    best_in = inside;
                    best = b;
                }
            }
            escapes = static_cast<int>(n - best_in);
            packed = static_cast<int64_t>(escapes) * 100 <= n;
            if (packed) size = (3 * n / 2 + 6 * static_cast<int64_t>(escapes) + 15) & ~int64_t(15);
        }
        // 64-bit exclusive scan of the aligned sizes, 2^20-byte units plus remainders
        int hi_total = 0, lo_total = 0;
        const int hi = block_exclusive_scan(static_cast<int>(size >> 20), scratch, &hi_total);
        const int lo = block_exclusive_scan(static_cast<int>(size & ((1 << 20) - 1)), scratch, &lo_total);
        if (row < rows) {
            const int64_t off = carry + (static_cast<int64_t>(hi) << 20) + lo;
            meta[row * 3 + 0] = packed ? off : -1;
            meta[row * 3 + 1] = best;
            meta[row * 3 + 2] = escapes;
        }
        carry += (static_cast<int64_t>(hi_total) << 20) + lo_total;
    }
    if (threadIdx.x == 0) *total = carry;
}

// One CTA per row: the escapes of each chunk (its values outside the row's
// window, from its histogram) and their exclusive scan, chunk_base[row][chunk].
__global__ void __launch_bounds__(1024) rowcodec_scan_kernel(const int32_t *__restrict__ chunk_hist, int64_t n,
                                                             const int64_t *__restrict__ meta,
                                                             int32_t *__restrict__ chunk_base, int chunks) {
    __shared__ int scratch[33];
    const int row = blockIdx.x;
    if (meta[row * 3] < 0) return;
    const int base = min(max(static_cast<int>(meta[row * 3 + 1]), 0), 256 - kWindow);  // in-bounds reads only
    int carry = 0;
    for (int c0 = 0; c0 < chunks; c0 += blockDim.x) {
        const int c = c0 + threadIdx.x;
        int esc = 0;
        if (c < chunks) {
            const int32_t *h = chunk_hist + (static_cast<int64_t>(row) * chunks + c) * 256;
            int inside = 0;
#pragma unroll
            for (int b = 0; b < kWindow; ++b) inside += h[base + b];
            esc = static_cast<int>(min(static_cast<int64_t>(kChunk), n - static_cast<int64_t>(c) * kChunk)) - inside;
        }
        int total = 0;
        const int excl = block_exclusive_scan(esc, scratch, &total);
        if (c < chunks) chunk_base[static_cast<int64_t>(row) * chunks + c] = carry + excl;
        carry += total;
    }
}

__global__ void __launch_bounds__(256) rowcodec_pack_kernel(const uint16_t *__restrict__ bank, int64_t n,
                                                            const int64_t *__restrict__ meta,
                                                            const int32_t *__restrict__ chunk_base, int chunks,
                                                            uint8_t *__restrict__ packed) {
    __shared__ int scratch[33];
    const int row = blockIdx.y;
    const int64_t off = meta[row * 3];
    if (off < 0) return;
    const uint32_t base = static_cast<uint32_t>(meta[row * 3 + 1]);
    const int64_t escapes = meta[row * 3 + 2];
    const uint16_t *r = bank + static_cast<int64_t>(row) * n;
    uint8_t *out = packed + off;
    int32_t *esc_idx = reinterpret_cast<int32_t *>(out + 3 * n / 2);
    uint16_t *esc_val = reinterpret_cast<uint16_t *>(out + 3 * n / 2 + 4 * escapes);
    const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk, end = min(n, begin + kChunk);
    // each thread: 32 consecutive values, in order; escapes placed by a CTA scan
    const int64_t i0 = begin + static_cast<int64_t>(threadIdx.x) * 32;
    int my_esc = 0;
    if (i0 < end) {
        for (int k = 0; k < 32 && i0 + k < end; k += 8) {
            const uint4 v = *reinterpret_cast<const uint4 *>(r + i0 + k);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t sf[2] = {0, 0}, nib = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t x = (w[j] >> (16 * h)) & 0xffffu;
                    const uint32_t e = (x >> 7) & 0xffu;
                    const int q = 2 * j + h;  // value index within the 8
                    sf[q >> 2] |= (((x >> 8) & 0x80u) | (x & 0x7fu)) << (8 * (q & 3));
                    nib |= ((e - base) & 0xfu) << (4 * q);
                    const int d = static_cast<int>(e) - static_cast<int>(base);
                    my_esc += d < 0 || d >= kWindow;
                }
            }
            *reinterpret_cast<uint2 *>(out + i0 + k) = make_uint2(sf[0], sf[1]);
            *reinterpret_cast<uint32_t *>(out + n + (i0 + k) / 2) = nib;
        }
    }
    int total = 0;
    int pos = chunk_base[static_cast<int64_t>(row) * chunks + blockIdx.x] +
              block_exclusive_scan(my_esc, scratch, &total);
    if (i0 < end && my_esc) {
        for (int k = 0; k < 32 && i0 + k < end; ++k) {
            const uint32_t x = r[i0 + k];
            const int d = static_cast<int>((x >> 7) & 0xffu) - static_cast<int>(base);
            if ((d < 0 || d >= kWindow) && pos < escapes) {  // a meta that disagrees writes no further
                esc_idx[pos] = static_cast<int32_t>(i0 + k);
                esc_val[pos] = static_cast<uint16_t>(x);
                ++pos;
            }
        }
    }
}

// One warp per 256-value tile; the CTA adds its encoded tiles to *encoded once.
__global__ void __launch_bounds__(256) tilecodec_pack_kernel(const uint16_t *__restrict__ raw, int64_t tiles,
                                                             uint8_t *__restrict__ packed,
                                                             uint8_t *__restrict__ bases,
                                                             unsigned long long *__restrict__ encoded) {
    const int lane = threadIdx.x & 31;
    const int64_t tile = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    bool enc = false;
    if (tile < tiles) {
        const uint4 v = *reinterpret_cast<const uint4 *>(raw + tile * 256 + lane * 8);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        int lo = 127, hi = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int a = (w[j] >> 8) & 127, b = (w[j] >> 24) & 127;
            lo = min(lo, min(a, b));
            hi = max(hi, max(a, b));
        }
#pragma unroll
        for (int s = 16; s; s >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, s));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, s));
        }
        uint8_t *p = packed + tile * 384;
        uint32_t low[2] = {0, 0}, codes = 0;
        enc = hi - lo <= 7;
        if (enc) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t x = (w[j] >> (16 * h)) & 0xffffu;
                    const int q = 2 * j + h;
                    low[q >> 2] |= (x & 0xffu) << (8 * (q & 3));
                    codes |= (((((x >> 8) & 127u) - static_cast<uint32_t>(lo)) & 7u) | ((x >> 12) & 8u)) << (4 * q);
                }
            }
        }
        // a raw tile (base 255) leaves its 384 packed bytes zero
        *reinterpret_cast<uint2 *>(p + lane * 8) = make_uint2(low[0], low[1]);
        *reinterpret_cast<uint32_t *>(p + 256 + lane * 4) = codes;
        if (lane == 0) bases[tile] = enc ? static_cast<uint8_t>(lo) : uint8_t(255);
    }
    const int count = __syncthreads_count(enc && lane == 0);
    if (threadIdx.x == 0 && count) atomicAdd(encoded, static_cast<unsigned long long>(count));
}

// Compact rows of the resident tile codec.  In a compact row, tile t starts at
// byte 384 t + 128 p(t), p(t) = raw tiles (base 255) before t: every tile
// takes its 384 packed bytes, and a raw tile 128 more (its 512 source bytes).
// So the only state that crosses tiles is that running count.  One CTA per
// row: a first pass counts the row's raw tiles and checks that the row fits
// the arena at its offsets (else sizes[r] = -1 and nothing is written); then
// chunks of 1024 tiles are scanned (ballot + warp scan) into p(t), each tile's
// header (p(t) << 8) | base is written, and the warps copy the tiles with
// 16-byte stores (an encoded tile from `packed`, a raw one from `raw`).
__global__ void __launch_bounds__(1024) tilecodec_compact_kernel(const uint16_t *__restrict__ raw,
                                                                 const uint8_t *__restrict__ packed,
                                                                 const uint8_t *__restrict__ bases,
                                                                 int64_t tiles_per_row, uint8_t *__restrict__ arena,
                                                                 int64_t arena_bytes,
                                                                 const int64_t *__restrict__ data_off,
                                                                 const int64_t *__restrict__ header_off,
                                                                 int64_t *__restrict__ sizes) {
    __shared__ int warp_incl[32];
    __shared__ int prior_s[1024];
    __shared__ uint8_t base_s[1024];
    __shared__ int total_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r = blockIdx.x;
    const int64_t doff = data_off[r], hoff = header_off[r];
    const uint8_t *rb = bases + r * tiles_per_row;
    if (doff < 0) {
        if (threadIdx.x == 0) sizes[r] = 0;
        return;
    }
    if (threadIdx.x == 0) total_s = 0;
    __syncthreads();
    int mine = 0;
    for (int64_t t = threadIdx.x; t < tiles_per_row; t += blockDim.x) mine += rb[t] == 255;
    mine = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0 && mine) atomicAdd(&total_s, mine);
    __syncthreads();
    const int64_t bytes = 384 * tiles_per_row + 128 * static_cast<int64_t>(total_s);
    const bool fits = doff % 16 == 0 && hoff % 16 == 0 && hoff >= 0 && doff + bytes <= arena_bytes &&
                      hoff + 4 * tiles_per_row <= arena_bytes;
    if (threadIdx.x == 0) sizes[r] = fits ? bytes : -1;
    if (!fits) return;
    uint8_t *data = arena + doff;
    uint32_t *hdr = reinterpret_cast<uint32_t *>(arena + hoff);
    const uint8_t *rp = packed + r * tiles_per_row * 384;
    const uint16_t *rr = raw + r * tiles_per_row * 256;
    int carry = 0;
    for (int64_t c0 = 0; c0 < tiles_per_row; c0 += 1024) {
        const int64_t t = c0 + threadIdx.x;
        const uint8_t b = t < tiles_per_row ? rb[t] : uint8_t(0);
        const unsigned flags = __ballot_sync(0xffffffffu, t < tiles_per_row && b == 255);
        if (lane == 0) warp_incl[warp] = __popc(flags);
        __syncthreads();
        if (warp == 0) {
            int v = warp_incl[lane];
#pragma unroll
            for (int s = 1; s < 32; s <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, v, s);
                if (lane >= s) v += u;
            }
            warp_incl[lane] = v;
        }
        __syncthreads();
        const int prior = carry + (warp ? warp_incl[warp - 1] : 0) + __popc(flags & ((1u << lane) - 1u));
        prior_s[threadIdx.x] = prior;
        base_s[threadIdx.x] = b;
        if (t < tiles_per_row) hdr[t] = (static_cast<uint32_t>(prior) << 8) | b;
        carry += warp_incl[31];
        __syncthreads();
        const int n = static_cast<int>(tiles_per_row - c0 < 1024 ? tiles_per_row - c0 : 1024);
        for (int i = warp; i < n; i += 32) {
            const int64_t tile = c0 + i;
            uint4 *dst = reinterpret_cast<uint4 *>(data + 384 * tile + 128 * static_cast<int64_t>(prior_s[i]));
            if (base_s[i] == 255)
                dst[lane] = reinterpret_cast<const uint4 *>(rr + tile * 256)[lane];
            else if (lane < 24)
                dst[lane] = reinterpret_cast<const uint4 *>(rp + tile * 384)[lane];
        }
        __syncthreads();  // prior_s, base_s and warp_incl are rewritten by the next chunk
    }
}

}  // namespace lrb

extern "C" {

size_t moe_rowcodec_workspace_bytes(int rows, int64_t n) {
    if (rows <= 0 || n <= 0) return 0;
    const int64_t chunks = (n + lrb::kChunk - 1) / lrb::kChunk;
    // row histograms, chunk histograms, chunk escape bases
    return static_cast<size_t>(rows) * 256 * 4 + static_cast<size_t>(rows) * chunks * 257 * 4;
}

namespace {

struct RowcodecWs {
    int32_t *hist, *chunk_hist, *chunk_base;
    int chunks;
};

RowcodecWs rowcodec_ws(void *workspace, int rows, int64_t n) {
    RowcodecWs w;
    w.chunks = static_cast<int>((n + lrb::kChunk - 1) / lrb::kChunk);
    w.hist = static_cast<int32_t *>(workspace);
    w.chunk_hist = w.hist + static_cast<size_t>(rows) * 256;
    w.chunk_base = w.chunk_hist + static_cast<size_t>(rows) * w.chunks * 256;
    return w;
}

}  // namespace

int moe_rowcodec_plan(const uint16_t *bank, int rows, int64_t n, int64_t *meta, int64_t *total, void *workspace,
                      size_t workspace_bytes, void *stream) {
    LRB_REQUIRE(bank && meta && total && rows > 0 && rows < 65536 && n > 0 && n % 8 == 0 && n < (int64_t(1) << 31),
                "moe_rowcodec_plan: bad arguments");
    LRB_REQUIRE(workspace && workspace_bytes >= moe_rowcodec_workspace_bytes(rows, n),
                "moe_rowcodec_plan: workspace below moe_rowcodec_workspace_bytes");
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(bank) % 16 == 0, "moe_rowcodec_plan: bank must be 16-byte aligned");
    if (int rc = lrb::require_sm100()) return rc;
    cudaStream_t s = lrb::as_stream(stream);
    const RowcodecWs w = rowcodec_ws(workspace, rows, n);
    LRB_CUDA(cudaMemsetAsync(w.hist, 0, static_cast<size_t>(rows) * 256 * 4, s));
    lrb::rowcodec_hist_kernel<<<dim3(w.chunks, rows), 256, 0, s>>>(bank, n, w.hist, w.chunk_hist);
    LRB_LAUNCHED("rowcodec_hist_kernel");
    lrb::rowcodec_plan_kernel<<<1, 1024, 0, s>>>(w.hist, rows, n, meta, total);
    LRB_LAUNCHED("rowcodec_plan_kernel");
    return MOE_OK;
}

int moe_rowcodec_pack(const uint16_t *bank, int rows, int64_t n, const int64_t *meta, uint8_t *packed,
                      void *workspace, size_t workspace_bytes, void *stream) {
    LRB_REQUIRE(bank && meta && packed && rows > 0 && rows < 65536 && n > 0 && n % 8 == 0 &&
                    n < (int64_t(1) << 31),
                "moe_rowcodec_pack: bad arguments");
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(bank) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 16 == 0,
                "moe_rowcodec_pack: bank and packed must be 16-byte aligned");
    LRB_REQUIRE(workspace && workspace_bytes >= moe_rowcodec_workspace_bytes(rows, n),
                "moe_rowcodec_pack: workspace below moe_rowcodec_workspace_bytes");
    if (int rc = lrb::require_sm100()) return rc;
    cudaStream_t s = lrb::as_stream(stream);
    const RowcodecWs w = rowcodec_ws(workspace, rows, n);
    lrb::rowcodec_scan_kernel<<<rows, 1024, 0, s>>>(w.chunk_hist, n, meta, w.chunk_base, w.chunks);
    LRB_LAUNCHED("rowcodec_scan_kernel");
    lrb::rowcodec_pack_kernel<<<dim3(w.chunks, rows), 256, 0, s>>>(bank, n, meta, w.chunk_base, w.chunks, packed);
    LRB_LAUNCHED("rowcodec_pack_kernel");
    return MOE_OK;
}

int moe_tilecodec_pack(const uint16_t *raw, int64_t tiles, uint8_t *packed, uint8_t *bases,
                       unsigned long long *encoded, void *stream) {
    LRB_REQUIRE(raw && packed && bases && encoded && tiles >= 0, "moe_tilecodec_pack: bad arguments");
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(raw) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 8 == 0,
                "moe_tilecodec_pack: raw must be 16-byte and packed 8-byte aligned");
    if (tiles == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    const int64_t blocks = (tiles + 7) / 8;
    LRB_REQUIRE(blocks < (int64_t(1) << 31), "moe_tilecodec_pack: too many tiles");
    lrb::tilecodec_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, lrb::as_stream(stream)>>>(raw, tiles, packed,
                                                                                                 bases, encoded);
    LRB_LAUNCHED("tilecodec_pack_kernel");
    return MOE_OK;
}

int moe_tilecodec_compact(const uint16_t *raw, const uint8_t *packed, const uint8_t *bases, int rows,
                          int64_t tiles_per_row, uint8_t *arena, int64_t arena_bytes, const int64_t *data_offsets,
                          const int64_t *header_offsets, int64_t *sizes, void *stream) {
    LRB_REQUIRE(raw && packed && bases && arena && data_offsets && header_offsets && sizes && rows >= 0 &&
                    tiles_per_row > 0 && tiles_per_row < (int64_t(1) << 31) && arena_bytes > 0,
                "moe_tilecodec_compact: bad arguments");
    LRB_REQUIRE(reinterpret_cast<uintptr_t>(raw) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(arena) % 16 == 0,
                "moe_tilecodec_compact: raw, packed and arena must be 16-byte aligned");
    if (rows == 0) return MOE_OK;
    if (int rc = lrb::require_sm100()) return rc;
    lrb::tilecodec_compact_kernel<<<rows, 1024, 0, lrb::as_stream(stream)>>>(
        raw, packed, bases, tiles_per_row, arena, arena_bytes, data_offsets, header_offsets, sizes);
    LRB_LAUNCHED("tilecodec_compact_kernel");
    return MOE_OK;
}

}  // extern "C"
