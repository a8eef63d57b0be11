/*
 * moe_oracle.c -- CPU restatement of the lightreason edge35b MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in lightreason_b200/ links, loads or calls
 * this file; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs use it, and only as the checker.
 *
 * Every function names the reference code it restates (paths inside the
 * me-farza/lightreason project; "TF:" = transformers
 * models/qwen3_5_moe/modeling_qwen3_5_moe.py, the third-party eager body that
 * edge35b/expert_stream.py:28,33 pins by version and AST hash).
 *
 * Parity pins (see tests/test_oracle_pins.py):
 *   - expert rows are bit-identical to edge35b/cpu_experts.c compiled from the
 *     reference sources (oracle/Makefile target `ref`);
 *   - the whole layer agrees with the installed TF eager Qwen3_5MoeSparseMoeBlock
 *     through golden fixtures in tests/golden/ (make_golden.py);
 *   - the codecs are bit-identical to edge35b/bf16_expert_codec.py and to
 *     cpu_bf16_reads.h pack_cpu_read_tiles on the reference's own test vectors.
 *
 * Build: oracle/Makefile (gcc -O2 -mfma -ffp-contract=off -fopenmp).  fmaf() is
 * used where the reference uses a fused multiply-add and nowhere else, so that
 * the summation order below is the one that runs.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_OK 0
#define OR_EINVAL 1

/* ---------------------------------------------------------------- bf16 ---- */

/* edge35b/cpu_experts.c:11-16 from_bfloat. */
static inline float bf2f(uint16_t v) {
    uint32_t b = (uint32_t)v << 16;
    float f;
    memcpy(&f, &b, sizeof f);
    return f;
}

/* Round-to-nearest-even float -> bf16, edge35b/cpu_experts.c:18-22 for finite
 * values; NaN stays a quiet NaN as torch's conversion does. */
static inline uint16_t f2bf(float f) {
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

static inline float rbf(float f) { return bf2f(f2bf(f)); }

/* edge35b/cpu_experts.c:29-41 dot(): two 8-lane FMA chains over 16-wide
 * blocks, lane-pair add, 128-bit fold and two horizontal adds.  The order of
 * every rounding step is kept so expert rows match the reference bit for bit. */
static float dot16(const uint16_t *w, const float *x, int width) {
    float lo[8] = {0}, hi[8] = {0};
    for (int i = 0; i < width; i += 16) {
        for (int j = 0; j < 8; ++j) {
            lo[j] = fmaf(bf2f(w[i + j]), x[i + j], lo[j]);
            hi[j] = fmaf(bf2f(w[i + 8 + j]), x[i + 8 + j], hi[j]);
        }
    }
    float lanes[8], s[4];
    for (int j = 0; j < 8; ++j) lanes[j] = lo[j] + hi[j];
    for (int j = 0; j < 4; ++j) s[j] = lanes[j] + lanes[j + 4];
    return (s[0] + s[1]) + (s[2] + s[3]);
}

void or_bf16_to_f32(const uint16_t *in, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]);
}

void or_f32_to_bf16(const float *in, uint16_t *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}

/* F.linear on BF16 (TF:764, TF:709): FP32 accumulation rounded once to BF16.
 * out[t][n] = bf16(sum_k x[t][k] * w[n][k]); dot order as dot16(). */
int or_linear_bf16(const uint16_t *x, const uint16_t *w, int tokens, int rows, int width,
                   uint16_t *out) {
    if (width % 16) return OR_EINVAL;
    float *xf = (float *)malloc(sizeof(float) * (size_t)tokens * width);
    if (!xf) return OR_EINVAL;
    or_bf16_to_f32(x, xf, (int64_t)tokens * width);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)tokens * rows; ++i) {
        int t = (int)(i / rows), n = (int)(i % rows);
        out[i] = f2bf(dot16(w + (int64_t)n * width, xf + (int64_t)t * width, width));
    }
    free(xf);
    return OR_OK;
}

/* ------------------------------------------------------------- router ---- */

/*
 * TF:762-770 Qwen3_5MoeTopKRouter.forward, with the synthetic per-expert bias
 * the benchmark configs add to the FP32 logits before the softmax:
 *   z = float(bf16 logits) + bias;  p = softmax(z);  top-k;  w = p_k / sum p_k.
 * Selection orders by z descending and breaks exact ties by the lower expert
 * index.  softmax is monotonic, so this selects the same set as topk on p;
 * where torch.topk meets equal p values its order is unspecified, and the
 * parity tests compare such groups as sets.
 * Outputs: idx[t][k] (int64), scores as FP32 and as BF16 (the reference fast
 * paths take BF16 router weights: edge35b/fused_experts.py:41-42).
 */
int or_router_select(const uint16_t *logits, const float *bias, int tokens, int experts,
                     int top_k, int64_t *idx, float *scores_f32, uint16_t *scores_bf16) {
    if (experts <= 0 || experts > 4096 || top_k <= 0 || top_k > experts) return OR_EINVAL;
    for (int t = 0; t < tokens; ++t) {
        float z[4096];
        float m = -INFINITY;
        for (int e = 0; e < experts; ++e) {
            z[e] = bf2f(logits[(int64_t)t * experts + e]) + (bias ? bias[e] : 0.0f);
            if (z[e] > m) m = z[e];
        }
        float s = 0.0f;
        for (int e = 0; e < experts; ++e) s += expf(z[e] - m);
        char taken[4096];
        memset(taken, 0, (size_t)experts);
        float top[64];
        int ids[64];
        for (int k = 0; k < top_k; ++k) {
            int best = -1;
            for (int e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best < 0 || z[e] > z[best]) best = e;
            }
            taken[best] = 1;
            ids[k] = best;
            top[k] = expf(z[best] - m) / s;
        }
        float sum = 0.0f;
        for (int k = 0; k < top_k; ++k) sum += top[k];
        for (int k = 0; k < top_k; ++k) {
            float w = top[k] / sum;
            idx[(int64_t)t * top_k + k] = ids[k];
            if (scores_f32) scores_f32[(int64_t)t * top_k + k] = w;
            if (scores_bf16) scores_bf16[(int64_t)t * top_k + k] = f2bf(w);
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------ permute ---- */

/*
 * TF:730-744 eager dispatch order: one_hot(idx).permute(2,1,0) visits experts
 * in ascending order (nonzero), and torch.where(mask[e]) yields (slot, token)
 * pairs slot-major then token.  edge35b/pipeline.py:59-76 _routes restates the
 * same order.  Route position p runs over that order:
 *   offsets[e]..offsets[e+1]    the routes of expert e,
 *   perm_token[p], perm_slot[p] the route at position p,
 *   route_pos[t*K + k]          the position of (token t, slot k).
 */
int or_permute(const int64_t *idx, int tokens, int top_k, int experts, int32_t *offsets,
               int32_t *perm_token, int32_t *perm_slot, int32_t *route_pos) {
    int32_t *count = (int32_t *)calloc((size_t)experts + 1, sizeof(int32_t));
    if (!count) return OR_EINVAL;
    for (int64_t r = 0; r < (int64_t)tokens * top_k; ++r) {
        int64_t e = idx[r];
        if (e < 0 || e >= experts) { free(count); return OR_EINVAL; }
        count[e]++;
    }
    offsets[0] = 0;
    for (int e = 0; e < experts; ++e) offsets[e + 1] = offsets[e] + count[e];
    for (int e = 0; e < experts; ++e) count[e] = offsets[e];
    for (int k = 0; k < top_k; ++k) {
        for (int t = 0; t < tokens; ++t) {
            int e = (int)idx[(int64_t)t * top_k + k];
            int p = count[e]++;
            perm_token[p] = t;
            perm_slot[p] = k;
            route_pos[(int64_t)t * top_k + k] = p;
        }
    }
    free(count);
    return OR_OK;
}

/* ------------------------------------------------------------ experts ---- */

/*
 * One (expert, token) pair of edge35b/cpu_experts.c:86-103 expert_block_rows,
 * itself the eager arithmetic of TF:745-748:
 *   gate, up = bf16(W_gu x) split at I;   s = bf16(g / (1 + exp(-g)));
 *   a = bf16(s * up);                     y = bf16(W_d a).
 * gate rows are W_gu[0:I], up rows W_gu[I:2I] (the .chunk(2) of TF:746).
 */
static void expert_pair(const uint16_t *gate_rows, const uint16_t *up_rows,
                        const uint16_t *down, const float *x, int hidden, int inner,
                        uint16_t *y) {
    float *active = (float *)malloc(sizeof(float) * (size_t)inner);
    for (int r = 0; r < inner; ++r) {
        float g = rbf(dot16(gate_rows + (int64_t)r * hidden, x, hidden));
        float u = rbf(dot16(up_rows + (int64_t)r * hidden, x, hidden));
        float s = rbf(g / (1.0f + expf(-g)));
        active[r] = rbf(s * u);
    }
    for (int r = 0; r < hidden; ++r) y[r] = f2bf(dot16(down + (int64_t)r * inner, active, inner));
    free(active);
}

/*
 * Routed experts for every route position.  gate_up/down hold one pointer per
 * expert id (the layout of Qwen3_5MoeExperts.gate_up_proj[e] / down_proj[e],
 * TF:720-721).  y[p] is the BF16 down projection of route p (not yet scaled).
 */
int or_experts(const uint16_t *x, const uint16_t *const *gate_up, const uint16_t *const *down,
               const int32_t *offsets, const int32_t *perm_token, int experts, int hidden,
               int inner, int tokens, uint16_t *y) {
    if (hidden % 16 || inner % 16) return OR_EINVAL;
    float *xf = (float *)malloc(sizeof(float) * (size_t)tokens * hidden);
    if (!xf) return OR_EINVAL;
    or_bf16_to_f32(x, xf, (int64_t)tokens * hidden);
    int routes = offsets[experts];
    int32_t *expert_of = (int32_t *)malloc(sizeof(int32_t) * (size_t)(routes > 0 ? routes : 1));
    for (int e = 0; e < experts; ++e)
        for (int p = offsets[e]; p < offsets[e + 1]; ++p) expert_of[p] = e;
#pragma omp parallel for schedule(dynamic, 1)
    for (int p = 0; p < routes; ++p) {
        int e = expert_of[p];
        const uint16_t *gu = gate_up[e];
        expert_pair(gu, gu + (int64_t)inner * hidden, down[e], xf + (int64_t)perm_token[p] * hidden,
                    hidden, inner, y + (int64_t)p * hidden);
    }
    free(expert_of);
    free(xf);
    return OR_OK;
}

/* TF:698-711 Qwen3_5MoeMLP (shared expert) for every token, and the sigmoid of
 * TF:779/788 shared_expert_gate:  sig[t] = bf16(sigmoid(bf16(x . w_gate))).
 * shared_out[t] = bf16(W_down bf16(bf16(silu(bf16 g)) * bf16 u)). */
int or_shared_expert(const uint16_t *x, const uint16_t *gate_w, const uint16_t *up_w,
                     const uint16_t *down_w, const uint16_t *sgate_w, int tokens, int hidden,
                     int inner, uint16_t *shared_out, uint16_t *sig) {
    if (hidden % 16 || inner % 16) return OR_EINVAL;
    float *xf = (float *)malloc(sizeof(float) * (size_t)tokens * hidden);
    if (!xf) return OR_EINVAL;
    or_bf16_to_f32(x, xf, (int64_t)tokens * hidden);
#pragma omp parallel for schedule(dynamic, 1)
    for (int t = 0; t < tokens; ++t) {
        const float *xt = xf + (int64_t)t * hidden;
        expert_pair(gate_w, up_w, down_w, xt, hidden, inner, shared_out + (int64_t)t * hidden);
        float g = rbf(dot16(sgate_w, xt, hidden));
        sig[t] = f2bf(1.0f / (1.0f + expf(-g)));
    }
    free(xf);
    return OR_OK;
}

/*
 * TF:749-750 + TF:788-790: per token, the routed contributions in ascending
 * expert order (index_add_ on BF16: acc = bf16(acc + bf16(y * w))), then the
 * gated shared expert (bf16(sig * shared)) added in BF16.  The same ordered
 * BF16 sum is edge35b/fused_experts.py:27-37 _ordered_sum and
 * edge35b/block_experts.py:31-49 _combine.  Route positions ascend with the
 * expert id, so the loop walks each token's positions in ascending order.
 * scores are BF16 router weights; shared_out/sig may be NULL (experts only).
 */
int or_combine(const uint16_t *y, const int32_t *route_pos, const uint16_t *scores, int tokens,
               int top_k, int hidden, const uint16_t *shared_out, const uint16_t *sig,
               uint16_t *out) {
    for (int t = 0; t < tokens; ++t) {
        int order[64];
        for (int k = 0; k < top_k; ++k) order[k] = k;
        for (int a = 1; a < top_k; ++a)
            for (int b = a; b > 0 && route_pos[t * top_k + order[b]] < route_pos[t * top_k + order[b - 1]]; --b) {
                int tmp = order[b]; order[b] = order[b - 1]; order[b - 1] = tmp;
            }
        for (int h = 0; h < hidden; ++h) {
            float acc = 0.0f;
            for (int j = 0; j < top_k; ++j) {
                int k = order[j];
                float v = bf2f(y[(int64_t)route_pos[t * top_k + k] * hidden + h]);
                acc = rbf(acc + rbf(v * bf2f(scores[t * top_k + k])));
            }
            if (shared_out) acc = rbf(acc + rbf(bf2f(sig[t]) * bf2f(shared_out[(int64_t)t * hidden + h])));
            out[(int64_t)t * hidden + h] = f2bf(acc);
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------- codecs ---- */

/* edge35b/bf16_expert_codec.py:26-33 exponent_window: the 16-exponent window
 * (over the 8-bit exponent field) holding the most values; first maximum wins.
 * escapes = values outside the window. */
void or_exponent_window(const uint16_t *bits, int64_t n, int32_t *base, int64_t *escapes) {
    int64_t counts[256] = {0};
    for (int64_t i = 0; i < n; ++i) counts[(bits[i] >> 7) & 255]++;
    int64_t best = -1;
    int best_base = 0;
    for (int b = 0; b + 16 <= 256; ++b) {
        int64_t w = 0;
        for (int j = 0; j < 16; ++j) w += counts[b + j];
        if (w > best) { best = w; best_base = b; }
    }
    *base = best_base;
    *escapes = n - best;
}

/* edge35b/bf16_expert_codec.py:36-37 row_bytes. */
int64_t or_row_bytes(int64_t n, int64_t escapes) { return 3 * n / 2 + 6 * escapes; }

/* edge35b/bf16_expert_codec.py:40-51 pack_row.  Layout: n bytes of sign|7-bit
 * fraction, n/2 bytes of exponent-delta nibbles (even value low nibble), then
 * int32 escape indices and uint16 escape values. */
int or_row_pack(const uint16_t *bits, int64_t n, int32_t base, int64_t escapes, uint8_t *out) {
    if (n % 2) return OR_EINVAL;
    int64_t split = 3 * n / 2, found = 0;
    for (int64_t i = 0; i < n; ++i) {
        int delta = (int)((bits[i] >> 7) & 255) - base;
        if (delta < 0 || delta >= 16) found++;
    }
    if (found != escapes) return OR_EINVAL;
    int32_t *esc_idx = (int32_t *)(out + split);
    uint16_t *esc_val = (uint16_t *)(out + split + 4 * escapes);
    int64_t e = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint16_t b = bits[i];
        out[i] = (uint8_t)((b & 127) | ((b >> 8) & 128));
        int delta = (int)((b >> 7) & 255) - base;
        if (i % 2 == 0) out[n + i / 2] = (uint8_t)(delta & 15);
        else out[n + i / 2] |= (uint8_t)((delta & 15) << 4);
        if (delta < 0 || delta >= 16) { esc_idx[e] = (int32_t)i; esc_val[e] = b; e++; }
    }
    return OR_OK;
}

/* edge35b/bf16_expert_codec.py:54-63 restore_row, equivalently the decode of
 * bf16_gather_ada.cu:11-20,68-102 (exponent field = base + nibble, then the
 * sorted escape list overwrites its values). */
void or_row_restore(const uint8_t *packed, int64_t n, int32_t base, int64_t escapes, uint16_t *bits) {
    int64_t split = 3 * n / 2;
    for (int64_t i = 0; i < n; ++i) {
        uint16_t sf = packed[i];
        uint16_t nib = (uint16_t)((packed[n + i / 2] >> ((i & 1) * 4)) & 15);
        bits[i] = (uint16_t)(((sf & 128) << 8) | (sf & 127) | ((nib + (uint16_t)base) << 7));
    }
    const int32_t *esc_idx = (const int32_t *)(packed + split);
    const uint16_t *esc_val = (const uint16_t *)(packed + split + 4 * escapes);
    for (int64_t e = 0; e < escapes; ++e) bits[esc_idx[e]] = esc_val[e];
}

/* cpu_bf16_reads.h:16-52 pack_cpu_read_tiles: 256-value tiles; the low byte is
 * kept, the high byte becomes a 4-bit code (3-bit offset from the tile's
 * smallest 7-bit high-byte exponent, bit 3 = sign).  A tile whose exponent span
 * exceeds 7 is left raw (base 255).  Packed tile = 256 low bytes + 128 code
 * bytes at stride 384.  Returns the number of encoded tiles. */
int64_t or_tile_pack(const uint16_t *raw, uint8_t *packed, uint8_t *bases, int64_t tiles) {
    int64_t encoded = 0;
    for (int64_t tile = 0; tile < tiles; ++tile) {
        const uint16_t *w = raw + tile * 256;
        int low = 127, high = 0;
        for (int i = 0; i < 256; ++i) {
            int e = (w[i] >> 8) & 127;
            if (e < low) low = e;
            if (e > high) high = e;
        }
        if (high - low > 7) { bases[tile] = 255; continue; }
        bases[tile] = (uint8_t)low;
        uint8_t *frac = packed + tile * 384, *codes = frac + 256;
        for (int i = 0; i < 256; i += 2) {
            int a = w[i] >> 8, b = w[i + 1] >> 8;
            frac[i] = (uint8_t)(w[i] & 255);
            frac[i + 1] = (uint8_t)(w[i + 1] & 255);
            int ac = ((a & 127) - low) | ((a & 128) >> 4);
            int bc = ((b & 127) - low) | ((b & 128) >> 4);
            codes[i / 2] = (uint8_t)(ac | (bc << 4));
        }
        ++encoded;
    }
    return encoded;
}

/* Decode of one encoded 256-value tile: bf16_gather_ada.cu:117-123. */
static void tile_unpack(const uint8_t *tile_data, unsigned base, uint16_t *out) {
    const uint8_t *codes = tile_data + 256;
    for (int i = 0; i < 256; ++i) {
        unsigned code = (codes[i / 2] >> ((i & 1) * 4)) & 15;
        unsigned high = ((base + (code & 7)) | ((code & 8) << 4)) & 255;
        out[i] = (uint16_t)(tile_data[i] | (high << 8));
    }
}

/*
 * edge35b/gpu_resident_experts.py:22-42 encode: tiles packed back to back
 * (384 B each; raw fallbacks inline at 512 B) with one uint32 header per tile:
 * (raw tiles before it << 8) | base.  Returns 0 and sets *data_bytes when the
 * compact row is smaller than raw (headers counted); 1 when raw is kept.
 */
int or_compact_encode(const uint16_t *raw, int64_t tiles, uint8_t *data, uint32_t *headers,
                      int64_t *data_bytes, int64_t *encoded_tiles) {
    uint8_t *packed = (uint8_t *)malloc((size_t)tiles * 384);
    uint8_t *bases = (uint8_t *)malloc((size_t)tiles);
    int64_t enc = or_tile_pack(raw, packed, bases, tiles);
    int64_t size = 0, raw_before = 0;
    for (int64_t t = 0; t < tiles; ++t) size += bases[t] == 255 ? 512 : 384;
    *encoded_tiles = enc;
    if (size + 4 * tiles >= tiles * 512) {
        free(packed); free(bases);
        *data_bytes = tiles * 512;
        return 1;
    }
    int64_t off = 0;
    for (int64_t t = 0; t < tiles; ++t) {
        headers[t] = (uint32_t)((raw_before << 8) | bases[t]);
        if (bases[t] == 255) {
            memcpy(data + off, raw + t * 256, 512);
            off += 512;
            raw_before++;
        } else {
            memcpy(data + off, packed + t * 384, 384);
            off += 384;
        }
    }
    *data_bytes = off;
    free(packed); free(bases);
    return 0;
}

/* --------------------------------------------------------- row gathers ---- */

/*
 * Host emulation of the descriptor-driven copies of edge35b/bf16_gather_ada.cu.
 * descriptors int64 [banks][experts][3]; destinations/sizes int64 [banks];
 * source_ids/destination_ids int32 [max]; count rows are copied.  Pointers in
 * the tables are host addresses here.
 *
 * mode 0 = row codec (gather<>, :36-103): (src, base, escapes), base < 0 raw.
 * mode 1 = tile codec (gather_cpu_tiles<false>, :127-180): (packed, bases, raw),
 *          bases == 0 raw.
 * mode 2 = tile codec with compact rows (gather_cpu_tiles<true>): raw == -1
 *          marks a compact row whose bases pointer holds uint32 headers.
 */
int or_gather_rows(const int64_t *descriptors, const int64_t *destinations, const int64_t *sizes,
                   const int32_t *source_ids, const int32_t *destination_ids, int64_t count,
                   int experts, int banks, int mode) {
    for (int64_t row = 0; row < count; ++row) {
        for (int bank = 0; bank < banks; ++bank) {
            const int64_t *d = descriptors + ((int64_t)bank * experts + source_ids[row]) * 3;
            int64_t row_bytes = sizes[bank];
            uint16_t *dst = (uint16_t *)(intptr_t)(destinations[bank] + (int64_t)destination_ids[row] * row_bytes);
            int64_t n = row_bytes / 2;
            if (mode == 0) {
                const uint8_t *src = (const uint8_t *)(intptr_t)d[0];
                if (d[1] < 0) memcpy(dst, src, (size_t)row_bytes);
                else or_row_restore(src, n, (int32_t)d[1], d[2], dst);
                continue;
            }
            const uint8_t *packed = (const uint8_t *)(intptr_t)d[0];
            const uint8_t *bases = (const uint8_t *)(intptr_t)d[1];
            const uint16_t *raw = (const uint16_t *)(intptr_t)d[2];
            if (bases == NULL) { memcpy(dst, raw, (size_t)row_bytes); continue; }
            int compact = mode == 2 && d[2] == -1;
            int64_t tiles = row_bytes / 512;
            for (int64_t t = 0; t < tiles; ++t) {
                uint32_t header = compact ? ((const uint32_t *)bases)[t] : bases[t];
                unsigned base = compact ? (header & 255) : header;
                const uint8_t *tile_data = packed + t * 384 + (compact ? (int64_t)(header >> 8) * 128 : 0);
                if (base == 255) {
                    if (compact) memcpy(dst + t * 256, tile_data, 512);
                    else memcpy(dst + t * 256, raw + t * 256, 512);
                } else {
                    tile_unpack(tile_data, base, dst + t * 256);
                }
            }
        }
    }
    return OR_OK;
}

/* -------------------------------------------------------- whole layer ---- */

/*
 * TF:781-792 Qwen3_5MoeSparseMoeBlock.forward with the BF16-score router:
 * shared expert, router (+bias), eager experts, gate and final add.
 * Weights: router [E,H]; gate_up [E][2I,H] and down [E][H,I] by pointer;
 * shared gate/up [Is,H], down [H,Is]; shared_gate [H].
 */
int or_moe_layer(const uint16_t *x, const uint16_t *router_w, const float *bias,
                 const uint16_t *const *gate_up, const uint16_t *const *down,
                 const uint16_t *sh_gate, const uint16_t *sh_up, const uint16_t *sh_down,
                 const uint16_t *sh_gate_w, int tokens, int hidden, int inner, int shared_inner,
                 int experts, int top_k, uint16_t *out, int64_t *idx_out, uint16_t *scores_out,
                 uint16_t *logits_out) {
    int rc = OR_OK;
    int64_t routes = (int64_t)tokens * top_k;
    uint16_t *logits = logits_out ? logits_out : (uint16_t *)malloc(sizeof(uint16_t) * (size_t)tokens * experts);
    int64_t *idx = idx_out ? idx_out : (int64_t *)malloc(sizeof(int64_t) * (size_t)routes);
    uint16_t *scores = scores_out ? scores_out : (uint16_t *)malloc(sizeof(uint16_t) * (size_t)routes);
    int32_t *offsets = (int32_t *)malloc(sizeof(int32_t) * (size_t)(experts + 1));
    int32_t *ptok = (int32_t *)malloc(sizeof(int32_t) * (size_t)routes);
    int32_t *pslot = (int32_t *)malloc(sizeof(int32_t) * (size_t)routes);
    int32_t *rpos = (int32_t *)malloc(sizeof(int32_t) * (size_t)routes);
    uint16_t *y = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)routes * hidden);
    uint16_t *sh = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)tokens * hidden);
    uint16_t *sig = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)tokens);
    if (!logits || !idx || !scores || !offsets || !ptok || !pslot || !rpos || !y || !sh || !sig) {
        rc = OR_EINVAL;
        goto done;
    }
    if ((rc = or_linear_bf16(x, router_w, tokens, experts, hidden, logits))) goto done;
    if ((rc = or_router_select(logits, bias, tokens, experts, top_k, idx, NULL, scores))) goto done;
    if ((rc = or_permute(idx, tokens, top_k, experts, offsets, ptok, pslot, rpos))) goto done;
    if ((rc = or_experts(x, gate_up, down, offsets, ptok, experts, hidden, inner, tokens, y))) goto done;
    if ((rc = or_shared_expert(x, sh_gate, sh_up, sh_down, sh_gate_w, tokens, hidden, shared_inner, sh, sig))) goto done;
    rc = or_combine(y, rpos, scores, tokens, top_k, hidden, sh, sig, out);
done:
    if (!logits_out) free(logits);
    if (!idx_out) free(idx);
    if (!scores_out) free(scores);
    free(offsets); free(ptok); free(pslot); free(rpos); free(y); free(sh); free(sig);
    return rc;
}
