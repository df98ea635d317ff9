/*
 * CPU oracle for the Tvara decode/prefill step -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference engine's arithmetic for the
 * hot path so that tests, smoke() and bench.py's cpu_baseline leg can check
 * the CUDA path against it.  Nothing in the shipped library links or calls
 * this code.  Parity is pinned: tests/test_oracle_pins.py checks every
 * function here against the reference itself (oracle/_ref, compiled from the
 * reference sources by oracle/Makefile) and against the known-answer vectors
 * of the reference's tests/core/test_quant.cpp and tests/core/test_kv.cpp.
 *
 * Reference paths below are relative to the Tvara source tree.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* core/include/tvara/quant.hpp:14-29 -- IEEE half to float, subnormals
 * normalised by shifting the mantissa, inf/nan keep their payload. */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 31u;
    uint32_t mantissa = h & 1023u;
    uint32_t bits;
    if (exponent == 0) {
        if (!mantissa) {
            bits = sign;
        } else {
            int e = -14;
            while ((mantissa & 1024u) == 0) { mantissa <<= 1; --e; }
            bits = sign | ((uint32_t)(e + 127) << 23) | ((mantissa & 1023u) << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* core/include/tvara/quant.hpp:63-68 -- 6-bit scale/min of sub-block g. */
void orc_q4k_scale_min(const uint8_t* scales12, int g, unsigned* scale, unsigned* min) {
    if (g < 4) {
        *scale = scales12[g] & 63u;
        *min = scales12[g + 4] & 63u;
    } else {
        *scale = (scales12[g + 4] & 15u) | ((unsigned)(scales12[g - 4] >> 6) << 4);
        *min = (scales12[g + 4] >> 4) | ((unsigned)(scales12[g] >> 6) << 4);
    }
}

/* GGUF storage types used on this path (gguf.hpp:152-170). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q4_K = 12 };

/* Bytes per block and elements per block; 0 for unknown types. */
int orc_block_shape(int type, size_t* block_bytes, size_t* block_elems) {
    switch (type) {
        case ORC_F32: *block_bytes = 4; *block_elems = 1; return 1;
        case ORC_F16: *block_bytes = 2; *block_elems = 1; return 1;
        case ORC_Q4_0: *block_bytes = 18; *block_elems = 32; return 1;
        case ORC_Q8_0: *block_bytes = 34; *block_elems = 32; return 1;
        case ORC_Q4_K: *block_bytes = 144; *block_elems = 256; return 1;
        default: return 0;
    }
}

/* Dequantise `blocks` blocks of `type` into floats.
 * Q8_0: quant.hpp:40-49 (d*q); Q4_0: quant.hpp:51-61 (low nibble -> i,
 * high nibble -> i+16, d*(q-8)); Q4_K: quant.hpp:70-84
 * (d*float(sc)*float(q) - dmin*float(m), evaluated left to right in float,
 * no fused multiply-add).  F32/F16 follow model.hpp:132-133.
 * Returns 0 on success, -1 on an unknown type. */
int orc_dequantize(int type, const uint8_t* src, size_t blocks, float* out) {
    size_t b, i;
    switch (type) {
        case ORC_F32:
            memcpy(out, src, blocks * 4);
            return 0;
        case ORC_F16:
            for (b = 0; b < blocks; ++b) out[b] = orc_half_to_float(rd16(src + 2 * b));
            return 0;
        case ORC_Q8_0:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = src + b * 34;
                const float scale = orc_half_to_float(rd16(blk));
                for (i = 0; i < 32; ++i) out[b * 32 + i] = scale * (float)(int8_t)blk[2 + i];
            }
            return 0;
        case ORC_Q4_0:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = src + b * 18;
                const float scale = orc_half_to_float(rd16(blk));
                for (i = 0; i < 16; ++i) {
                    const unsigned q = blk[2 + i];
                    out[b * 32 + i] = scale * (float)((int)(q & 15u) - 8);
                    out[b * 32 + i + 16] = scale * (float)((int)(q >> 4) - 8);
                }
            }
            return 0;
        case ORC_Q4_K:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = src + b * 144;
                const float d = orc_half_to_float(rd16(blk));
                const float dmin = orc_half_to_float(rd16(blk + 2));
                int g;
                for (g = 0; g < 8; ++g) {
                    unsigned sc, m;
                    orc_q4k_scale_min(blk + 4, g, &sc, &m);
                    for (i = 0; i < 32; ++i) {
                        const unsigned packed = blk[16 + (g / 2) * 32 + i];
                        const unsigned q = (g % 2) ? (packed >> 4) : (packed & 15u);
                        volatile float a = d * (float)sc;   /* keep the reference's */
                        volatile float c = a * (float)q;    /* rounding sequence    */
                        volatile float e = dmin * (float)m;
                        out[b * 256 + g * 32 + i] = c - e;
                    }
                }
            }
            return 0;
        default:
            return -1;
    }
}

/* quant.hpp:105-110 + 163-169 -- served projection: one double-accumulated
 * dot per output row, cast to float. */
void orc_matvec_f32(const float* w, size_t rows, size_t cols, const float* x, float* out) {
    size_t r, k;
    for (r = 0; r < rows; ++r) {
        double sum = 0;
        const float* row = w + r * cols;
        for (k = 0; k < cols; ++k) sum += (double)row[k] * (double)x[k];
        out[r] = (float)sum;
    }
}

/* prefill.hpp:12-18 / quant.hpp:188-196 -- tokens x rows projection. */
void orc_matmul_f32(const float* x, size_t tokens, const float* w, size_t rows, size_t cols, float* out) {
    size_t t;
    for (t = 0; t < tokens; ++t) orc_matvec_f32(w, rows, cols, x + t * cols, out + t * rows);
}

/* quant.hpp:86-103 -- per-32 activation quantisation; scale = max|x|/127,
 * values = round-half-away(x/scale).  Returns -1 on a nonfinite input. */
int orc_quantize_activations(const float* x, size_t n, float* scales, int8_t* values) {
    size_t b, i;
    if (n % 32) return -1;
    for (b = 0; b < n / 32; ++b) {
        float maximum = 0;
        for (i = 0; i < 32; ++i) {
            const float v = x[b * 32 + i];
            if (!isfinite(v)) return -1;
            if (fabsf(v) > maximum) maximum = fabsf(v);
        }
        scales[b] = maximum / 127.f;
        for (i = 0; i < 32; ++i)
            values[b * 32 + i] = scales[b] == 0 ? 0 : (int8_t)roundf(x[b * 32 + i] / scales[b]);
    }
    return 0;
}

/* quant.hpp:112-161 -- int8-activation dots, integer block sums, double
 * total.  `row` is one packed weight row, `blocks` its block count. */
float orc_dot_quant(int type, const uint8_t* row, size_t blocks, const float* ascale, const int8_t* aval) {
    double total = 0;
    size_t b, i;
    if (type == ORC_Q8_0) {
        for (b = 0; b < blocks; ++b) {
            int32_t sum = 0;
            for (i = 0; i < 32; ++i) sum += (int32_t)(int8_t)row[b * 34 + 2 + i] * (int32_t)aval[b * 32 + i];
            total += (double)orc_half_to_float(rd16(row + b * 34)) * (double)ascale[b] * (double)sum;
        }
    } else if (type == ORC_Q4_0) {
        for (b = 0; b < blocks; ++b) {
            int32_t sum = 0;
            for (i = 0; i < 16; ++i) {
                const unsigned q = row[b * 18 + 2 + i];
                sum += ((int)(q & 15u) - 8) * (int32_t)aval[b * 32 + i];
                sum += ((int)(q >> 4) - 8) * (int32_t)aval[b * 32 + i + 16];
            }
            total += (double)orc_half_to_float(rd16(row + b * 18)) * (double)ascale[b] * (double)sum;
        }
    } else if (type == ORC_Q4_K) {
        for (b = 0; b < blocks; ++b) {
            const uint8_t* blk = row + b * 144;
            const float d = orc_half_to_float(rd16(blk)), dmin = orc_half_to_float(rd16(blk + 2));
            int g;
            for (g = 0; g < 8; ++g) {
                unsigned sc, m;
                int32_t products = 0, sum = 0;
                const int8_t* a = aval + (b * 8 + g) * 32;
                orc_q4k_scale_min(blk + 4, g, &sc, &m);
                for (i = 0; i < 32; ++i) {
                    const unsigned packed = blk[16 + (g / 2) * 32 + i];
                    const unsigned q = (g % 2) ? packed >> 4 : packed & 15u;
                    products += (int32_t)q * (int32_t)a[i];
                    sum += a[i];
                }
                total += (double)ascale[b * 8 + g] * ((double)d * sc * products - (double)dmin * m * sum);
            }
        }
    }
    return (float)total;
}

/* quant.hpp:170-186 -- matvec over packed rows with int8 activations. */
int orc_matvec_quant(int type, const uint8_t* w, size_t rows, size_t cols, const float* x, float* out) {
    size_t bb, be, r, stride;
    float* scales;
    int8_t* values;
    if (!orc_block_shape(type, &bb, &be) || be == 1 || cols % be) return -1;
    stride = cols / be * bb;
    scales = (float*)malloc(sizeof(float) * (cols / 32));
    values = (int8_t*)malloc(cols);
    if (!scales || !values || orc_quantize_activations(x, cols, scales, values)) {
        free(scales); free(values); return -1;
    }
    for (r = 0; r < rows; ++r) out[r] = orc_dot_quant(type, w + r * stride, cols / be, scales, values);
    free(scales); free(values);
    return 0;
}

/* model.hpp:57-65 -- RMSNorm, double sum of squares, float inverse,
 * out = (x*inverse)*w as two float roundings. */
void orc_rms_norm(const float* x, const float* w, size_t n, float eps, float* out) {
    double sum = 0;
    size_t i;
    for (i = 0; i < n; ++i) sum += (double)x[i] * x[i];
    const float inverse = (float)(1 / sqrt(sum / (double)n + eps));
    for (i = 0; i < n; ++i) {
        volatile float a = x[i] * inverse;
        out[i] = a * w[i];
    }
}

/* model.hpp:67-76 -- the float angle and its cosine/sine for pair i at
 * `position`; RoPE tables built from this are bit-identical to the
 * reference's per-call evaluation on the same libm. */
void orc_rope_table(size_t positions, size_t dim, float theta, float* cosines, float* sines) {
    size_t p, i;
    for (p = 0; p < positions; ++p)
        for (i = 0; i < dim / 2; ++i) {
            const float angle = (float)p / powf(theta, (float)(2 * i) / (float)dim);
            cosines[p * (dim / 2) + i] = cosf(angle);
            sines[p * (dim / 2) + i] = sinf(angle);
        }
}

/* model.hpp:67-76 -- rotate `heads` heads of x in place. */
void orc_rotary(float* x, size_t heads, size_t dim, size_t position, float theta, int interleaved) {
    size_t h, i;
    for (h = 0; h < heads; ++h)
        for (i = 0; i < dim / 2; ++i) {
            const float angle = (float)position / powf(theta, (float)(2 * i) / (float)dim);
            const float c = cosf(angle), s = sinf(angle);
            const size_t a = h * dim + (interleaved ? 2 * i : i);
            const size_t b = h * dim + (interleaved ? 2 * i + 1 : i + dim / 2);
            const float left = x[a], right = x[b];
            volatile float l1 = left * c, r1 = right * s, r2 = right * c, l2 = left * s;
            x[a] = l1 - r1;
            x[b] = r2 + l2;
        }
}

/* model.hpp:115-126 -- SwiGLU: gate *= sigmoid(gate)*up with the
 * reference's overflow-safe sigmoid. */
void orc_swiglu(float* gate, const float* up, size_t n) {
    size_t i;
    for (i = 0; i < n; ++i) {
        const float small = expf(-fabsf(gate[i]));
        const float sigmoid = gate[i] >= 0 ? 1 / (1 + small) : small / (1 + small);
        volatile float su = sigmoid * up[i];
        gate[i] *= su;
    }
}

/* attention.hpp:6-16 + 57-83 -- online-softmax attention of one query row
 * over a paged block list laid out as the reference's pool
 * (offset ((layer*2+kind)*tpb+slot)*kv_width within a block), plus an
 * optional uncommitted tail position.  visible caps the positions seen.
 * Scores and the running sums are double. */
int orc_paged_attention(const float* q, size_t heads, size_t kv_heads, size_t dim,
                        const float* pool, size_t block_elems, size_t tpb, size_t layer,
                        const int64_t* table, size_t length,
                        const float* tail_k, const float* tail_v, size_t visible, float* out) {
    const size_t width = kv_heads * dim, group = heads / kv_heads;
    const size_t total = length + (tail_k ? 1 : 0);
    size_t h, p, i;
    double* sum = (double*)malloc(sizeof(double) * dim);
    if (!sum) return -1;
    if (visible > total) visible = total;
    if (!visible) { free(sum); return -1; }
    for (h = 0; h < heads; ++h) {
        const size_t kh = h / group;
        double maximum = -INFINITY, normalizer = 0;
        for (i = 0; i < dim; ++i) sum[i] = 0;
        for (p = 0; p < visible; ++p) {
            const float *key, *value;
            if (p < length) {
                const float* blk = pool + (size_t)table[p / tpb] * block_elems;
                const size_t slot = p % tpb;
                key = blk + ((layer * 2 + 0) * tpb + slot) * width + kh * dim;
                value = blk + ((layer * 2 + 1) * tpb + slot) * width + kh * dim;
            } else {
                key = tail_k + kh * dim;
                value = tail_v + kh * dim;
            }
            double score = 0;
            for (i = 0; i < dim; ++i) score += (double)q[h * dim + i] * key[i];
            score /= sqrt((double)dim);
            const double next = score > maximum ? score : maximum;
            const double old = exp(maximum - next), weight = exp(score - next);
            normalizer = normalizer * old + weight;
            for (i = 0; i < dim; ++i) sum[i] = sum[i] * old + weight * value[i];
            maximum = next;
        }
        for (i = 0; i < dim; ++i) out[h * dim + i] = (float)(sum[i] / normalizer);
    }
    free(sum);
    return 0;
}

/* ---------------------------------------------------------------------
 * Paged KV block accounting, kv.hpp:36-165.  A pool of `max_blocks`
 * blocks with generation tags, reference counts and a LIFO free list that
 * starts as [max-1, ..., 0] so the first allocation returns block 0.
 * Block payloads are not modelled (tests compare ids, generations,
 * reference counts and the free-list state).
 * ------------------------------------------------------------------- */
typedef struct {
    size_t max_blocks, tpb;
    uint64_t* generation;
    size_t* references;
    size_t* free_list;
    size_t free_count;
    /* sequences: dense arrays indexed by id (ids start at 1). */
    size_t seq_cap;
    uint64_t next_id;
    int* live;
    size_t* length;
    size_t** blocks;     /* block ids */
    uint64_t** gens;     /* generation of each entry */
    size_t* nblocks;
    size_t* cap;
    /* CoW copies recorded by the last append: (from, to) block ids. */
    int64_t last_copy_from, last_copy_to;
} orc_cache;

orc_cache* orc_cache_new(size_t max_blocks, size_t tpb, size_t max_sequences) {
    orc_cache* c = (orc_cache*)calloc(1, sizeof(orc_cache));
    size_t i;
    c->max_blocks = max_blocks; c->tpb = tpb;
    c->generation = (uint64_t*)calloc(max_blocks, 8);
    c->references = (size_t*)calloc(max_blocks, sizeof(size_t));
    c->free_list = (size_t*)calloc(max_blocks, sizeof(size_t));
    for (i = max_blocks; i > 0; --i) c->free_list[c->free_count++] = i - 1;   /* kv.hpp:42 */
    c->seq_cap = max_sequences + 1;
    c->live = (int*)calloc(c->seq_cap, sizeof(int));
    c->length = (size_t*)calloc(c->seq_cap, sizeof(size_t));
    c->blocks = (size_t**)calloc(c->seq_cap, sizeof(size_t*));
    c->gens = (uint64_t**)calloc(c->seq_cap, sizeof(uint64_t*));
    c->nblocks = (size_t*)calloc(c->seq_cap, sizeof(size_t));
    c->cap = (size_t*)calloc(c->seq_cap, sizeof(size_t));
    return c;
}

void orc_cache_free(orc_cache* c) {
    size_t i;
    if (!c) return;
    for (i = 0; i < c->seq_cap; ++i) { free(c->blocks[i]); free(c->gens[i]); }
    free(c->generation); free(c->references); free(c->free_list); free(c->live);
    free(c->length); free(c->blocks); free(c->gens); free(c->nblocks); free(c->cap);
    free(c);
}

size_t orc_cache_available(const orc_cache* c) { return c->free_count; }
size_t orc_cache_references(const orc_cache* c, size_t id) { return id < c->max_blocks ? c->references[id] : 0; }
uint64_t orc_cache_generation(const orc_cache* c, size_t id) { return id < c->max_blocks ? c->generation[id] : 0; }

/* Copy the free list (top of stack last) into out; returns its length. */
size_t orc_cache_free_list(const orc_cache* c, size_t* out) {
    memcpy(out, c->free_list, c->free_count * sizeof(size_t));
    return c->free_count;
}

static int seq_ok(const orc_cache* c, uint64_t id) { return id && id < c->seq_cap && c->live[id]; }

/* kv.hpp:44-50: pop the free-list top, references=1, ++generation.
 * Returns the block id or -1 when exhausted. */
static int64_t pool_allocate(orc_cache* c) {
    size_t id;
    if (!c->free_count) return -1;
    id = c->free_list[--c->free_count];
    c->references[id] = 1;
    ++c->generation[id];
    return (int64_t)id;
}

/* kv.hpp:57: on the last release the id is pushed on the free list. */
static void pool_release(orc_cache* c, size_t id) {
    if (--c->references[id] == 0) c->free_list[c->free_count++] = id;
}

static void push_block(orc_cache* c, uint64_t s, size_t id) {
    if (c->nblocks[s] == c->cap[s]) {
        c->cap[s] = c->cap[s] ? 2 * c->cap[s] : 8;
        c->blocks[s] = (size_t*)realloc(c->blocks[s], c->cap[s] * sizeof(size_t));
        c->gens[s] = (uint64_t*)realloc(c->gens[s], c->cap[s] * 8);
    }
    c->blocks[s][c->nblocks[s]] = id;
    c->gens[s][c->nblocks[s]] = c->generation[id];
    ++c->nblocks[s];
}

/* kv.hpp:81 -- ids start at 1.  Returns 0 when no id is free. */
uint64_t orc_cache_create(orc_cache* c) {
    if (c->next_id + 1 >= c->seq_cap) return 0;
    const uint64_t id = ++c->next_id;
    c->live[id] = 1; c->length[id] = 0; c->nblocks[id] = 0;
    return id;
}

/* kv.hpp:91-108 -- accounting half of append: a fresh block at slot 0,
 * copy-on-write replacement of a shared partial tail.  Returns 0, -1 for
 * an unknown sequence or full table, -2 when the pool is exhausted (state
 * unchanged, kv.hpp:93-96). */
int orc_cache_append(orc_cache* c, uint64_t s) {
    size_t slot;
    c->last_copy_from = c->last_copy_to = -1;
    if (!seq_ok(c, s)) return -1;
    if (c->length[s] >= c->max_blocks * c->tpb) return -1;
    slot = c->length[s] % c->tpb;
    if (slot == 0) {
        const int64_t id = pool_allocate(c);
        if (id < 0) return -2;
        push_block(c, s, (size_t)id);
    }
    if (slot != 0 && c->references[c->blocks[s][c->nblocks[s] - 1]] > 1) {
        const size_t original = c->blocks[s][c->nblocks[s] - 1];
        const int64_t replacement = pool_allocate(c);
        if (replacement < 0) return -2;
        c->blocks[s][c->nblocks[s] - 1] = (size_t)replacement;
        c->gens[s][c->nblocks[s] - 1] = c->generation[replacement];
        pool_release(c, original);
        c->last_copy_from = (int64_t)original; c->last_copy_to = replacement;
    }
    ++c->length[s];
    return 0;
}

/* kv.hpp:121 */
int orc_cache_drop(orc_cache* c, uint64_t s) {
    size_t i;
    if (!seq_ok(c, s)) return -1;
    for (i = 0; i < c->nblocks[s]; ++i) pool_release(c, c->blocks[s][i]);
    c->live[s] = 0; c->nblocks[s] = 0; c->length[s] = 0;
    return 0;
}

/* kv.hpp:123-129 -- share every block (retain) under a new id. */
uint64_t orc_cache_fork(orc_cache* c, uint64_t s) {
    size_t i;
    uint64_t id;
    if (!seq_ok(c, s)) return 0;
    id = orc_cache_create(c);
    if (!id) return 0;
    for (i = 0; i < c->nblocks[s]; ++i) { ++c->references[c->blocks[s][i]]; push_block(c, id, c->blocks[s][i]); }
    c->length[id] = c->length[s];
    return id;
}

/* kv.hpp:131-136 -- releases blocks beyond ceil(length/tpb). */
int orc_cache_truncate(orc_cache* c, uint64_t s, size_t length) {
    size_t keep, i;
    if (!seq_ok(c, s) || length > c->length[s]) return -1;
    keep = length / c->tpb + (length % c->tpb ? 1 : 0);
    for (i = keep; i < c->nblocks[s]; ++i) pool_release(c, c->blocks[s][i]);
    c->nblocks[s] = keep;
    c->length[s] = length;
    return 0;
}

/* kv.hpp:149-159 -- a new sequence sharing the first ceil(length/tpb)
 * blocks of `s`. */
uint64_t orc_cache_import(orc_cache* c, uint64_t s, size_t length) {
    size_t count, i;
    uint64_t id;
    if (!seq_ok(c, s) || length > c->length[s]) return 0;
    count = length / c->tpb + (length % c->tpb ? 1 : 0);
    id = orc_cache_create(c);
    if (!id) return 0;
    for (i = 0; i < count; ++i) { ++c->references[c->blocks[s][i]]; push_block(c, id, c->blocks[s][i]); }
    c->length[id] = length;
    return id;
}

size_t orc_cache_length(const orc_cache* c, uint64_t s) { return seq_ok(c, s) ? c->length[s] : 0; }

/* Block table of `s` as (id, generation) pairs; returns the count. */
size_t orc_cache_table(const orc_cache* c, uint64_t s, size_t* ids, uint64_t* gens) {
    size_t i;
    if (!seq_ok(c, s)) return 0;
    for (i = 0; i < c->nblocks[s]; ++i) { ids[i] = c->blocks[s][i]; gens[i] = c->gens[s][i]; }
    return c->nblocks[s];
}

/* kv.hpp:61-64 + 138-146 -- free-list and reference invariants.
 * Returns 0 when they hold. */
int orc_cache_audit(const orc_cache* c) {
    size_t i, s;
    size_t* counts = (size_t*)calloc(c->max_blocks, sizeof(size_t));
    char* seen = (char*)calloc(c->max_blocks, 1);
    int bad = 0;
    for (i = 0; i < c->free_count; ++i) {
        const size_t id = c->free_list[i];
        if (id >= c->max_blocks || seen[id] || c->references[id]) bad = 1; else seen[id] = 1;
    }
    for (i = 0; i < c->max_blocks; ++i) if ((seen[i] != 0) != (c->references[i] == 0)) bad = 1;
    for (s = 1; s < c->seq_cap; ++s) {
        if (!c->live[s]) continue;
        if (c->nblocks[s] != c->length[s] / c->tpb + (c->length[s] % c->tpb ? 1 : 0)) bad = 1;
        for (i = 0; i < c->nblocks[s]; ++i) ++counts[c->blocks[s][i]];
    }
    for (i = 0; i < c->max_blocks; ++i) if (counts[i] != c->references[i]) bad = 1;
    free(counts); free(seen);
    return bad ? -1 : 0;
}
