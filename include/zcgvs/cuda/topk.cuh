// Top-k launcher (the reference's include/zcgvs/cuda/topk.cuh:8-43), implemented over zcgvs_topk:
// the top-k of every row of a [batch, doc_count] score matrix, (score desc, id asc), padded with
// (-FLT_MAX, -1). The four scratch buffers keep the reference signature; the kernel needs none and
// leaves them untouched.
#pragma once

#include <cuda_runtime.h>

namespace zcgvs {
namespace cuda {

int topKTileSize();                              // 1024
int topKMergeTile();                             // 4096
int topKMaxK();                                  // ZCGVS_MAX_K
int topKBlockCount(int doc_count);               // ceil(doc_count / 1024)
int topKScratchElements(int doc_count, int k);   // topKBlockCount(doc_count) * k

void launchTopK(const float* d_scores, int doc_count, int k, int batch, int* d_out_indices,
                float* d_out_values, float* d_scratch_values_a, int* d_scratch_indices_a,
                float* d_scratch_values_b, int* d_scratch_indices_b, cudaStream_t stream);

}  // namespace cuda
}  // namespace zcgvs
