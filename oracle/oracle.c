/*
 * oracle.c - CPU restatement of the reference search path. TEST INFRASTRUCTURE ONLY.
 *
 * Used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker;
 * never linked into or called by the product library. Each function cites the reference
 * file:line whose arithmetic it restates. Build: oracle/Makefile (gcc -O2 -ffp-contract=off,
 * so every a*b+c is two IEEE roundings, exactly like the reference CPU loops).
 *
 * Pinned against the reference: tests/golden/ holds outputs of the reference's own CPU code
 * (tests/cpp/cpu_reference.hpp compiled by oracle/Makefile) and its Python format tools
 * (python/zcgvs_tools/formats.py); tests/test_oracle_golden.py checks this file against them.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------------------------
 * fp16 <-> fp32 (IEEE binary16, round to nearest even). The reference rounds fp16 stores
 * with __float2half (src/cuda/convert.cu:17-23) and its tests with __float2half_rn
 * (tests/cpp/test_scan_paths.cu:47-52); both are round-to-nearest-even.
 * --------------------------------------------------------------------------------------- */
uint16_t orc_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    const int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t half = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
    return (uint16_t)(sign | half);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

void orc_convert_f16(const float* src, size_t count, uint16_t* dst) {
    for (size_t i = 0; i < count; ++i) dst[i] = orc_f32_to_f16(src[i]);
}

/* Per-matrix scale of python/zcgvs_tools/formats.py:85-91: max|x| / 127, or 1 if all zero. */
float orc_matrix_scale(const float* src, size_t count) {
    float peak = 0.0f;
    for (size_t i = 0; i < count; ++i) {
        const float a = fabsf(src[i]);
        if (a > peak) peak = a;
    }
    return peak > 0.0f ? peak / 127.0f : 1.0f;
}

/* Symmetric int8 quantisation with a given scale: clamp(rint(x * (1/scale)), -127, 127).
 * src/cuda/convert.cu:25-32 and :57-64; tests/cpp/cpu_reference.hpp:53-62. */
void orc_quantize_i8(const float* src, size_t count, float scale, int8_t* dst) {
    const float inverse = (scale > 0.0f) ? 1.0f / scale : 0.0f;
    for (size_t i = 0; i < count; ++i) {
        float q = nearbyintf(src[i] * inverse);
        if (q > 127.0f) q = 127.0f;
        if (q < -127.0f) q = -127.0f;
        dst[i] = (int8_t)q;
    }
}

/* Per-row variant (the extension used by ZCGVS_DTYPE_I8_ROW and by the BASELINE int8
 * config): each row gets its own formats.py:85-91 scale and the quantiser above. */
void orc_quantize_rows_i8(const float* src, int64_t rows, int dim, int8_t* dst, float* scales) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* row = src + (size_t)r * (size_t)dim;
        const float s = orc_matrix_scale(row, (size_t)dim);
        scales[r] = s;
        orc_quantize_i8(row, (size_t)dim, s, dst + (size_t)r * (size_t)dim);
    }
}

/* Sign-bit packing: bit b of word w is dimension 32w+b, set when x >= 0; padding bits zero.
 * src/cuda/convert.cu:34-53; tests/cpp/cpu_reference.hpp:64-78; formats.py:65-82. */
void orc_pack_binary(const float* src, int64_t rows, int dim, uint32_t* dst) {
    const int words = (dim + 31) / 32;
    memset(dst, 0, (size_t)rows * (size_t)words * sizeof(uint32_t));
    for (int64_t r = 0; r < rows; ++r) {
        for (int d = 0; d < dim; ++d) {
            if (src[(size_t)r * (size_t)dim + (size_t)d] >= 0.0f) {
                dst[(size_t)r * (size_t)words + (size_t)(d / 32)] |= (1u << (d % 32));
            }
        }
    }
}

static int popcount32(uint32_t x) {
    int n = 0;
    while (x) {
        x &= x - 1u;
        ++n;
    }
    return n;
}

/* tests/cpp/cpu_reference.hpp:80-90. */
int orc_hamming(const uint32_t* a, const uint32_t* b, int words) {
    int distance = 0;
    for (int w = 0; w < words; ++w) distance += popcount32(a[w] ^ b[w]);
    return distance;
}

/* ---------------------------------------------------------------------------------------
 * Scores of one query against every row, [n] floats.
 *   F32 / F16 / I8 (per-matrix): sequential fp32 accumulation of q * decode(x)
 *     (tests/cpp/cpu_reference.hpp:12-24; decode = include/zcgvs/cuda/decode.cuh:22-26);
 *     L2: -sum((q - x)^2) (tests/cpp/test_metrics_filter.cu:16-29).
 *   BINARY: (dim - 2 * hamming) / dim on packed sign bits of the query
 *     (include/zcgvs/cuda/decode.cuh:45-47).
 *   I8_ROW: float(int32 dot of per-row-quantised query and row) * s_query * s_row.
 *   mask[i] == 0 -> -FLT_MAX (src/cuda/similarity.cu:109-113).
 * --------------------------------------------------------------------------------------- */
/* Scores of rows [i0, i1) of the corpus (out indexed by row). */
static void scores_rows(int dtype, const void* corpus, float scale, const float* row_scales,
                        int64_t i0, int64_t n, int dim, const float* query, const uint8_t* mask, int metric,
                        float* out) {
    const int l2 = (metric == ORC_METRIC_L2);
    if (dtype == ORC_DTYPE_BINARY) {
        const int words = (dim + 31) / 32;
        uint32_t* qbits = (uint32_t*)calloc((size_t)words, sizeof(uint32_t));
        orc_pack_binary(query, 1, dim, qbits);
        const uint32_t* codes = (const uint32_t*)corpus;
        for (int64_t i = i0; i < n; ++i) {
            const int h = orc_hamming(codes + (size_t)i * (size_t)words, qbits, words);
            out[i] = (float)(dim - 2 * h) / (float)dim;
        }
        free(qbits);
    } else if (dtype == ORC_DTYPE_I8_ROW) {
        int8_t* qq = (int8_t*)malloc((size_t)dim);
        float qs = 0.0f;
        orc_quantize_rows_i8(query, 1, dim, qq, &qs);
        const int8_t* rows = (const int8_t*)corpus;
        for (int64_t i = i0; i < n; ++i) {
            const int8_t* x = rows + (size_t)i * (size_t)dim;
            int32_t dot = 0;
            for (int j = 0; j < dim; ++j) dot += (int32_t)x[j] * (int32_t)qq[j];
            const float a = (float)dot * qs;
            out[i] = a * row_scales[i];
        }
        free(qq);
    } else {
        for (int64_t i = i0; i < n; ++i) {
            float acc = 0.0f;
            for (int j = 0; j < dim; ++j) {
                float x;
                const size_t at = (size_t)i * (size_t)dim + (size_t)j;
                if (dtype == ORC_DTYPE_F16) {
                    x = orc_f16_to_f32(((const uint16_t*)corpus)[at]);
                } else if (dtype == ORC_DTYPE_I8) {
                    x = (float)((const int8_t*)corpus)[at] * scale;
                } else {
                    x = ((const float*)corpus)[at];
                }
                if (l2) {
                    const float d = query[j] - x;
                    acc += d * d;
                } else {
                    acc += x * query[j];
                }
            }
            out[i] = l2 ? -acc : acc;
        }
    }
    if (mask != NULL) {
        for (int64_t i = i0; i < n; ++i) {
            if (mask[i] == 0) out[i] = -FLT_MAX;
        }
    }
}

/* Host threads scores_one may use (orc_set_threads; 1 by default). Rows are scored
 * independently, so the thread count changes no arithmetic: every score is the same sequential
 * sum whatever the split. */
static int g_threads = 1;

void orc_set_threads(int threads) { g_threads = threads > 1 ? (threads < 256 ? threads : 256) : 1; }

struct rows_job {
    int dtype, dim, metric;
    const void* corpus;
    float scale;
    const float* row_scales;
    int64_t i0, i1;
    const float* query;
    const uint8_t* mask;
    float* out;
};

static void* rows_job_run(void* arg) {
    const struct rows_job* j = (const struct rows_job*)arg;
    scores_rows(j->dtype, j->corpus, j->scale, j->row_scales, j->i0, j->i1, j->dim, j->query, j->mask, j->metric,
                j->out);
    return NULL;
}

static void scores_one(int dtype, const void* corpus, float scale, const float* row_scales,
                       int64_t n, int dim, const float* query, const uint8_t* mask, int metric,
                       float* out) {
    const int threads = (g_threads > 1 && n >= 65536) ? g_threads : 1;
    if (threads == 1) {
        scores_rows(dtype, corpus, scale, row_scales, 0, n, dim, query, mask, metric, out);
        return;
    }
    pthread_t tid[256];
    int spawned[256];
    struct rows_job jobs[256];
    for (int t = 0; t < threads; ++t) {
        const struct rows_job j = {dtype, dim, metric, corpus, scale, row_scales, n * t / threads,
                                   n * (t + 1) / threads, query, mask, out};
        jobs[t] = j;
        spawned[t] = t > 0 && pthread_create(&tid[t], NULL, rows_job_run, &jobs[t]) == 0;
    }
    for (int t = 0; t < threads; ++t) {
        if (!spawned[t]) rows_job_run(&jobs[t]);  /* the calling thread, or a thread that failed to start */
    }
    for (int t = 1; t < threads; ++t) {
        if (spawned[t]) pthread_join(tid[t], NULL);
    }
}

void orc_scores(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n,
                int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                float* out) {
    for (int q = 0; q < batch; ++q) {
        scores_one(dtype, corpus, scale, row_scales, n, dim, queries + (size_t)q * (size_t)dim,
                   mask, metric, out + (size_t)q * (size_t)n);
    }
}

/* ---------------------------------------------------------------------------------------
 * Top-k under the total order (score descending, id ascending): the order
 * std::stable_sort(order, score[a] > score[b]) gives in tests/cpp/cpu_reference.hpp:26-34.
 * -0.0 and +0.0 are equal scores there, so both map to the key of +0.0 here (and the
 * reported score of such an entry is +0.0). Implemented with the same 64-bit key as the
 * device code: high word = order-preserving score bits, low word = ~id.
 * --------------------------------------------------------------------------------------- */
static uint32_t orderable(float s) {
    uint32_t u;
    memcpy(&u, &s, 4);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static float from_orderable(uint32_t o) {
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    float s;
    memcpy(&s, &u, 4);
    return s;
}

static uint64_t make_key(float s, uint32_t id) {
    return ((uint64_t)orderable(s) << 32) | (uint32_t)(~id);
}

static void heap_sift_down(uint64_t* h, int n, int i) {
    for (;;) {
        int smallest = i;
        const int l = 2 * i + 1, r = 2 * i + 2;
        if (l < n && h[l] < h[smallest]) smallest = l;
        if (r < n && h[r] < h[smallest]) smallest = r;
        if (smallest == i) return;
        const uint64_t t = h[i];
        h[i] = h[smallest];
        h[smallest] = t;
        i = smallest;
    }
}

static int cmp_desc(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return (x < y) - (x > y);
}

void orc_topk(const float* scores, int64_t n, int batch, int k, int id_base, int32_t* out_idx,
              float* out_scores) {
    uint64_t* heap = (uint64_t*)malloc((size_t)(k > 0 ? k : 1) * sizeof(uint64_t));
    for (int q = 0; q < batch; ++q) {
        const float* s = scores + (size_t)q * (size_t)n;
        int size = 0;
        for (int64_t i = 0; i < n; ++i) {
            const uint64_t key = make_key(s[i], (uint32_t)(id_base + i));
            if (size < k) {
                heap[size++] = key;
                if (size == k) {
                    for (int j = k / 2 - 1; j >= 0; --j) heap_sift_down(heap, k, j);
                }
            } else if (key > heap[0]) {
                heap[0] = key;
                heap_sift_down(heap, k, 0);
            }
        }
        qsort(heap, (size_t)size, sizeof(uint64_t), cmp_desc);
        for (int j = 0; j < k; ++j) {
            if (j < size) {
                out_idx[(size_t)q * k + j] = (int32_t)(~(uint32_t)heap[j]);
                out_scores[(size_t)q * k + j] = from_orderable((uint32_t)(heap[j] >> 32));
            } else {
                out_idx[(size_t)q * k + j] = -1;
                out_scores[(size_t)q * k + j] = -FLT_MAX;
            }
        }
    }
    free(heap);
}

/* Fused reference of zcgvs_scan_topk: scores_one + orc_topk per query. */
void orc_scan_topk(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n,
                   int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                   int k, int id_base, int32_t* out_idx, float* out_scores) {
    float* s = (float*)malloc((size_t)n * sizeof(float));
    for (int q = 0; q < batch; ++q) {
        scores_one(dtype, corpus, scale, row_scales, n, dim, queries + (size_t)q * (size_t)dim,
                   mask, metric, s);
        orc_topk(s, n, 1, k, id_base, out_idx + (size_t)q * k, out_scores + (size_t)q * k);
    }
    free(s);
}

/* ---------------------------------------------------------------------------------------
 * Rescore stage: the gather-rescore of src/cuda/rescore.cu:20-63 (every candidate id scored
 * against the rescore store with the fp32 query, as scores_one does for a whole corpus), the
 * second launchTopK over the [batch, m] rescored values and the id remap of :65-79, as
 * Searcher::recordPipeline chains them (src/search/searcher.cpp:266-279). Candidates outside
 * [0, n) are dropped; the top-k of the rest is taken under (score desc, id asc) on the global
 * ids, and short lists are padded with (-1, -FLT_MAX). BINARY stores are rejected by the
 * reference (src/cuda/rescore.cu:102-105); this returns -1 for them.
 * --------------------------------------------------------------------------------------- */
static float score_row(int dtype, const void* store, float scale, const float* row_scales, int dim,
                       int64_t row, const float* query, const int8_t* qq, float qs, int metric) {
    const int l2 = (metric == ORC_METRIC_L2);
    if (dtype == ORC_DTYPE_I8_ROW) {
        const int8_t* x = (const int8_t*)store + (size_t)row * (size_t)dim;
        int32_t dot = 0;
        for (int j = 0; j < dim; ++j) dot += (int32_t)x[j] * (int32_t)qq[j];
        const float a = (float)dot * qs;
        return a * row_scales[row];
    }
    float acc = 0.0f;
    for (int j = 0; j < dim; ++j) {
        float x;
        const size_t at = (size_t)row * (size_t)dim + (size_t)j;
        if (dtype == ORC_DTYPE_F16) {
            x = orc_f16_to_f32(((const uint16_t*)store)[at]);
        } else if (dtype == ORC_DTYPE_I8) {
            x = (float)((const int8_t*)store)[at] * scale;
        } else {
            x = ((const float*)store)[at];
        }
        if (l2) {
            const float d = query[j] - x;
            acc += d * d;
        } else {
            acc += x * query[j];
        }
    }
    return l2 ? -acc : acc;
}

int orc_rescore_topk(int dtype, const void* store, float scale, const float* row_scales, int64_t n,
                     int dim, const float* queries, int batch, const int32_t* candidates, int m,
                     int metric, int k, int32_t* out_idx, float* out_scores) {
    if (dtype == ORC_DTYPE_BINARY) return -1;
    uint64_t* keys = (uint64_t*)malloc((size_t)(m > 0 ? m : 1) * sizeof(uint64_t));
    int8_t* qq = (int8_t*)malloc((size_t)(dim > 0 ? dim : 1));
    for (int q = 0; q < batch; ++q) {
        const float* query = queries + (size_t)q * (size_t)dim;
        float qs = 0.0f;
        if (dtype == ORC_DTYPE_I8_ROW) orc_quantize_rows_i8(query, 1, dim, qq, &qs);
        int count = 0;
        for (int j = 0; j < m; ++j) {
            const int32_t id = candidates[(size_t)q * (size_t)m + (size_t)j];
            if (id < 0 || (int64_t)id >= n) continue;
            const float s = score_row(dtype, store, scale, row_scales, dim, id, query, qq, qs, metric);
            keys[count++] = make_key(s, (uint32_t)id);
        }
        qsort(keys, (size_t)count, sizeof(uint64_t), cmp_desc);
        for (int j = 0; j < k; ++j) {
            if (j < count) {
                out_idx[(size_t)q * k + j] = (int32_t)(~(uint32_t)keys[j]);
                out_scores[(size_t)q * k + j] = from_orderable((uint32_t)(keys[j] >> 32));
            } else {
                out_idx[(size_t)q * k + j] = -1;
                out_scores[(size_t)q * k + j] = -FLT_MAX;
            }
        }
    }
    free(qq);
    free(keys);
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * Lexical scoring, the CPU reference of tests/cpp/test_lexical.cu:71-89:
 *   orc_bm25          : scores[doc] += weight for every posting of every valid term slot, in
 *                       slot order then posting order (sequential fp32 adds); postings whose
 *                       document is outside [0, n) are skipped (src/cuda/lexical.cu:35-39),
 *                       term ids outside [0, vocab) are ignored.
 *   orc_max_positive  : max(0, max_i values[i]).
 *   orc_fuse          : dense[i] = w * dense[i] + ((1 - w) * lex[i]) * inv, inv = 1 / peak when
 *                       peak > 0 else 0, each operation rounded on its own.
 *   orc_hybrid_topk   : per query, scores_one (dense, mask -> -FLT_MAX), orc_bm25 from zero,
 *                       orc_max_positive, orc_fuse, then orc_topk: the hybrid chain of
 *                       src/search/searcher.cpp:236-263 followed by its top-k.
 * --------------------------------------------------------------------------------------- */
void orc_bm25(const int64_t* offsets, const int32_t* docs, const float* weights, int vocab, const int32_t* terms,
              int term_count, int64_t n, float* scores) {
    for (int t = 0; t < term_count; ++t) {
        const int32_t term = terms[t];
        if (term < 0 || term >= vocab) continue;
        for (int64_t p = offsets[term]; p < offsets[term + 1]; ++p) {
            const int32_t doc = docs[p];
            if (doc < 0 || (int64_t)doc >= n) continue;
            scores[doc] += weights[p];
        }
    }
}

float orc_max_positive(const float* values, int64_t count) {
    float best = 0.0f;
    for (int64_t i = 0; i < count; ++i) {
        if (values[i] > best) best = values[i];
    }
    return best;
}

void orc_fuse(float* dense, const float* lex, float peak, float w, int64_t count) {
    const float inv = peak > 0.0f ? 1.0f / peak : 0.0f;
    for (int64_t i = 0; i < count; ++i) {
        const float a = w * dense[i];
        const float b = (1.0f - w) * lex[i];
        const float c = b * inv;
        dense[i] = a + c;
    }
}

void orc_hybrid_topk(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n, int dim,
                     const float* queries, int batch, const uint8_t* mask, int metric, const int64_t* offsets,
                     const int32_t* docs, const float* weights, int vocab, const int32_t* terms, int stride,
                     float w, int k, int32_t* out_idx, float* out_scores) {
    float* dense = (float*)malloc((size_t)n * sizeof(float));
    float* lex = (float*)malloc((size_t)n * sizeof(float));
    for (int q = 0; q < batch; ++q) {
        scores_one(dtype, corpus, scale, row_scales, n, dim, queries + (size_t)q * (size_t)dim, mask, metric, dense);
        if (stride > 0 && terms != NULL) {
            memset(lex, 0, (size_t)n * sizeof(float));
            orc_bm25(offsets, docs, weights, vocab, terms + (size_t)q * (size_t)stride, stride, n, lex);
            orc_fuse(dense, lex, orc_max_positive(lex, n), w, n);
        }
        orc_topk(dense, n, 1, k, 0, out_idx + (size_t)q * k, out_scores + (size_t)q * k);
    }
    free(lex);
    free(dense);
}
