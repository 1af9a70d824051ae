/*
 * oracle.h - CPU restatement of the reference search path. TEST INFRASTRUCTURE ONLY:
 * called by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker,
 * never by the product library.
 */
#ifndef ZCGVS_ORACLE_H
#define ZCGVS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_DTYPE_F32 = 0, ORC_DTYPE_F16 = 1, ORC_DTYPE_I8 = 2, ORC_DTYPE_BINARY = 3, ORC_DTYPE_I8_ROW = 4 };
enum { ORC_METRIC_COSINE = 0, ORC_METRIC_DOT = 1, ORC_METRIC_L2 = 2 };

void orc_set_threads(int threads);
uint16_t orc_f32_to_f16(float value);
float orc_f16_to_f32(uint16_t h);
void orc_convert_f16(const float* src, size_t count, uint16_t* dst);
float orc_matrix_scale(const float* src, size_t count);
void orc_quantize_i8(const float* src, size_t count, float scale, int8_t* dst);
void orc_quantize_rows_i8(const float* src, int64_t rows, int dim, int8_t* dst, float* scales);
void orc_pack_binary(const float* src, int64_t rows, int dim, uint32_t* dst);
int orc_hamming(const uint32_t* a, const uint32_t* b, int words);
void orc_scores(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n,
                int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                float* out);
void orc_topk(const float* scores, int64_t n, int batch, int k, int id_base, int32_t* out_idx,
              float* out_scores);
void orc_scan_topk(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n,
                   int dim, const float* queries, int batch, const uint8_t* mask, int metric,
                   int k, int id_base, int32_t* out_idx, float* out_scores);

/* Rescore stage (gather + exact score + second top-k + id remap) over candidate ids
 * [batch, m]; ids outside [0, n) are dropped. Returns -1 for BINARY stores. */
int orc_rescore_topk(int dtype, const void* store, float scale, const float* row_scales, int64_t n,
                     int dim, const float* queries, int batch, const int32_t* candidates, int m,
                     int metric, int k, int32_t* out_idx, float* out_scores);

/* Lexical scoring (tests/cpp/test_lexical.cu:71-89) and the hybrid search chain. */
void orc_bm25(const int64_t* offsets, const int32_t* docs, const float* weights, int vocab, const int32_t* terms,
              int term_count, int64_t n, float* scores);
float orc_max_positive(const float* values, int64_t count);
void orc_fuse(float* dense, const float* lex, float peak, float w, int64_t count);
void orc_hybrid_topk(int dtype, const void* corpus, float scale, const float* row_scales, int64_t n, int dim,
                     const float* queries, int batch, const uint8_t* mask, int metric, const int64_t* offsets,
                     const int32_t* docs, const float* weights, int vocab, const int32_t* terms, int stride,
                     float w, int k, int32_t* out_idx, float* out_scores);

/* The synthetic index, query and dense scores of tests/cpp/test_lexical.cu:31-67, bit for bit. */
void orc_gen_lexical_test(uint32_t index_seed, int doc_count, int vocab, int max_postings, float wlo,
                          float whi, uint32_t query_seed, int term_count, int64_t* offsets, int32_t* docs,
                          float* weights, int64_t* nnz, int32_t* terms, float* dense);

/* Seeded inputs identical to the reference harnesses' randomMatrix
 * (tests/cpp/test_pipeline.cu:20-31): std::mt19937(seed), std::normal_distribution<float>(0,1),
 * then each row L2-normalised in fp32 (tests/cpp/cpu_reference.hpp:36-49). */
void orc_gen_normal_rows(int64_t rows, int dim, uint32_t seed, int normalize, float* out);
/* std::mt19937(seed) + std::uniform_real_distribution<float>(lo, hi), the generator of
 * tests/cpp/test_topk.cu:14-20 and test_metrics_filter.cu:27-37. */
void orc_gen_uniform(size_t count, uint32_t seed, float lo, float hi, float* out);

#ifdef __cplusplus
}
#endif

#endif
