// The C++ interface of include/zcgvs/ (the reference's launcher, store, index and Searcher
// declarations) implemented over the C ABI of include/zcgvs_sm100.h. Failures are rethrown as
// the reference's exception types: invalid arguments as std::invalid_argument, CUDA failures as
// zcgvs::CudaError, anything else as std::runtime_error.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <numeric>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "zcgvs/core/cuda_check.hpp"
#include "zcgvs/core/cuda_context.hpp"
#include "zcgvs/cuda/convert.cuh"
#include "zcgvs/cuda/lexical.cuh"
#include "zcgvs/cuda/rescore.cuh"
#include "zcgvs/cuda/similarity.cuh"
#include "zcgvs/cuda/topk.cuh"
#include "zcgvs/data/binary_format.hpp"
#include "zcgvs/data/corpus.hpp"
#include "zcgvs/data/embedding_store.hpp"
#include "zcgvs/data/lexical_index.hpp"
#include "zcgvs/search/searcher.hpp"
#include "zcgvs/search/sharded_searcher.hpp"
#include "zcgvs_sm100.h"

namespace zcgvs {

namespace {

void check(int status, const char* call) {
    if (status == ZCGVS_OK) return;
    const std::string message = zcgvs_last_error_message();
    if (status == ZCGVS_ERR_INVALID_ARG) throw std::invalid_argument(message);
    if (status == ZCGVS_ERR_CUDA) {
        const int code = zcgvs_last_cuda_error();
        throw CudaError(code != 0 ? static_cast<cudaError_t>(code) : cudaErrorUnknown, call, __FILE__, __LINE__);
    }
    throw std::runtime_error(message);
}

// Text of the device status word's bits (ZCGVS_DEVICE_* in zcgvs_sm100.h).
std::string describeDeviceStatus(std::uint32_t word) {
    static const std::pair<std::uint32_t, const char*> kBits[] = {
        {ZCGVS_DEVICE_TILE_WAIT_TIMEOUT, "a bounded wait for a corpus tile ran out"},
        {ZCGVS_DEVICE_DRAIN_TIMEOUT, "a bounded wait for in-flight copies ran out"},
        {ZCGVS_DEVICE_TMEM_WAIT_TIMEOUT, "a tensor-memory accumulator hand-off ran out"},
        {ZCGVS_DEVICE_CANDIDATE_OVERFLOW, "a query kept more candidates than its buffer holds (its top-k is incomplete)"},
    };
    char hex[16];
    std::snprintf(hex, sizeof(hex), "0x%x", word);
    std::string text = std::string("device status ") + hex + ":";
    std::uint32_t known = 0u;
    for (const auto& bit : kBits) {
        known |= bit.first;
        if ((word & bit.first) != 0u) text += std::string(" ") + bit.second + ";";
    }
    if ((word & ~known) != 0u) text += " unknown bits;";
    text.pop_back();
    return text;
}

// Per-query staging limit of the reference's similarity launcher (src/cuda/similarity.cu:23):
// reported by similaritySharedBytes for callers that size their own launches.
constexpr std::size_t kQueryStageLimit = 40960;
constexpr int kQueryTile = 8;
constexpr int kTopKTile = 1024;

// Reads little-endian scalars and byte ranges of a binary file, failing on a short read.
class Reader {
public:
    explicit Reader(const std::string& path) : in_(path, std::ios::binary), path_(path) {
        if (!in_) throw std::runtime_error("zcgvs: cannot open '" + path + "'");
    }
    template <typename T>
    T scalar() {
        T value{};
        bytes(&value, sizeof(T));
        return value;
    }
    void bytes(void* dst, std::size_t count) {
        in_.read(static_cast<char*>(dst), static_cast<std::streamsize>(count));
        if (!in_) throw std::runtime_error("zcgvs: '" + path_ + "' ends early");
    }
    void magic(const char (&expected)[4]) {
        char got[4];
        bytes(got, 4);
        if (std::memcmp(got, expected, 4) != 0) throw std::runtime_error("zcgvs: '" + path_ + "' has the wrong magic");
    }
    std::string text(std::size_t length) {
        std::string value(length, '\0');
        if (length > 0) bytes(value.data(), length);
        return value;
    }
    // Streams `count` bytes of the file into device memory through two pinned chunks: the read
    // of one chunk overlaps the host-to-device copy of the other, and no host copy of the whole
    // payload is made.
    void toDevice(void* device_dst, std::size_t count) {
        if (count == 0) return;
        constexpr std::size_t kChunk = std::size_t(32) << 20;
        const std::size_t chunk = std::min(count, kChunk);
        PinnedBuffer<std::uint8_t> stage[2] = {PinnedBuffer<std::uint8_t>(chunk),
                                               PinnedBuffer<std::uint8_t>(count > chunk ? chunk : 0)};
        StreamGuard copies;
        auto* dst = static_cast<std::uint8_t*>(device_dst);
        for (std::size_t done = 0, i = 0; done < count; done += chunk, ++i) {
            const std::size_t n = std::min(chunk, count - done);
            const int b = static_cast<int>(i & 1);
            ZCGVS_CUDA_CHECK(cudaEventSynchronize(copies.ready[b]));  // its previous copy has finished
            bytes(stage[b].data(), n);
            ZCGVS_CUDA_CHECK(cudaMemcpyAsync(dst + done, stage[b].data(), n, cudaMemcpyHostToDevice, copies.stream));
            ZCGVS_CUDA_CHECK(cudaEventRecord(copies.ready[b], copies.stream));
        }
        ZCGVS_CUDA_CHECK(cudaStreamSynchronize(copies.stream));
    }

private:
    // A copy stream and one event per staging chunk, synchronised and released on every exit
    // (a short file throws from bytes() with copies in flight).
    struct StreamGuard {
        cudaStream_t stream = nullptr;
        cudaEvent_t ready[2] = {nullptr, nullptr};
        StreamGuard() {
            ZCGVS_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
            for (auto& e : ready) {
                ZCGVS_CUDA_CHECK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
                ZCGVS_CUDA_CHECK(cudaEventRecord(e, stream));
            }
        }
        ~StreamGuard() {
            if (stream != nullptr) cudaStreamSynchronize(stream);
            for (auto e : ready) {
                if (e != nullptr) cudaEventDestroy(e);
            }
            if (stream != nullptr) cudaStreamDestroy(stream);
        }
        StreamGuard(const StreamGuard&) = delete;
        StreamGuard& operator=(const StreamGuard&) = delete;
    };

    std::ifstream in_;
    std::string path_;
};

// Stable per-term sort of the postings by document (scores unchanged: equal documents keep
// their order).
void sort_postings(const std::vector<std::int64_t>& offsets, std::vector<int>& docs, std::vector<float>& weights) {
    std::vector<std::size_t> order;
    std::vector<int> d2;
    std::vector<float> w2;
    for (std::size_t t = 0; t + 1 < offsets.size(); ++t) {
        const std::size_t begin = static_cast<std::size_t>(offsets[t]), end = static_cast<std::size_t>(offsets[t + 1]);
        if (std::is_sorted(docs.begin() + begin, docs.begin() + end)) continue;
        order.resize(end - begin);
        std::iota(order.begin(), order.end(), begin);
        std::stable_sort(order.begin(), order.end(), [&](std::size_t a, std::size_t b) { return docs[a] < docs[b]; });
        d2.resize(order.size());
        w2.resize(order.size());
        for (std::size_t i = 0; i < order.size(); ++i) {
            d2[i] = docs[order[i]];
            w2[i] = weights[order[i]];
        }
        std::copy(d2.begin(), d2.end(), docs.begin() + begin);
        std::copy(w2.begin(), w2.end(), weights.begin() + begin);
    }
}

}  // namespace

// ------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------
namespace cuda {

void launchSimilarity(const void* d_corpus, ScalarType dtype, float scale, int doc_count, int dim,
                      const void* d_queries, int batch, const std::uint8_t* d_mask, Metric metric,
                      float* d_scores, cudaStream_t stream) {
    if (doc_count <= 0 || batch <= 0 || dim <= 0) return;
    similaritySharedBytes(dtype, dim, batch);  // the reference's dimension limit
    check(zcgvs_similarity(d_corpus, static_cast<int>(dtype), scale, nullptr, doc_count, dim, d_queries, batch,
                           d_mask, static_cast<int>(metric), d_scores, stream),
          "zcgvs_similarity");
}

int similarityQueryTile() { return kQueryTile; }

std::size_t similaritySharedBytes(ScalarType dtype, int dim, int batch) {
    if (batch <= 0 || dim <= 0) return 0;
    const std::size_t per_query =
        dtype == ScalarType::Binary ? binaryWords(dim) * sizeof(unsigned int) : static_cast<std::size_t>(dim) * 4;
    if (per_query > kQueryStageLimit) {
        throw std::invalid_argument("zcgvs similarity: embedding dim " + std::to_string(dim) +
                                    " needs more shared memory than a block can stage");
    }
    const int tile = std::max(1, std::min({kQueryTile, static_cast<int>(kQueryStageLimit / per_query), batch}));
    return static_cast<std::size_t>(tile) * per_query;
}

int topKTileSize() { return kTopKTile; }
int topKMergeTile() { return 4 * kTopKTile; }
int topKMaxK() { return ZCGVS_MAX_K; }
int topKBlockCount(int doc_count) { return doc_count <= 0 ? 0 : (doc_count + kTopKTile - 1) / kTopKTile; }
int topKScratchElements(int doc_count, int k) { return (doc_count <= 0 || k <= 0) ? 0 : topKBlockCount(doc_count) * k; }

void launchTopK(const float* d_scores, int doc_count, int k, int batch, int* d_out_indices, float* d_out_values,
                float*, int*, float*, int*, cudaStream_t stream) {
    if (k <= 0 || doc_count <= 0 || batch <= 0) return;
    check(zcgvs_topk(d_scores, doc_count, k, batch, d_out_indices, d_out_values, stream), "zcgvs_topk");
}

void launchConvertF32ToF16(const float* src, void* dst_half, std::size_t count, cudaStream_t stream) {
    check(zcgvs_convert_f16(src, dst_half, count, stream), "zcgvs_convert_f16");
}

void launchConvertF32ToI8(const float* src, void* dst_int8, std::size_t count, float scale, cudaStream_t stream) {
    check(zcgvs_convert_i8(src, dst_int8, count, scale, stream), "zcgvs_convert_i8");
}

void launchPackBinary(const float* src, void* dst_words, int rows, int dim, cudaStream_t stream) {
    check(zcgvs_pack_binary(src, dst_words, rows, dim, stream), "zcgvs_pack_binary");
}

void launchConvertF32ToI8Rows(const float* src, void* dst_int8, float* row_scales, std::int64_t rows, int dim,
                              cudaStream_t stream) {
    check(zcgvs_convert_i8_rows(src, dst_int8, row_scales, rows, dim, stream), "zcgvs_convert_i8_rows");
}

void launchBm25(const std::int64_t* d_offsets, const int* d_docs, const float* d_weights, const int* d_query_terms,
                int term_count, int doc_count, float* d_scores, cudaStream_t stream) {
    check(zcgvs_bm25(d_offsets, d_docs, d_weights, d_query_terms, term_count, doc_count, d_scores, stream),
          "zcgvs_bm25");
}

void launchMaxPositive(const float* d_values, int count, float* d_max, cudaStream_t stream) {
    check(zcgvs_max_positive(d_values, count, d_max, stream), "zcgvs_max_positive");
}

void launchFuseScores(float* d_dense, const float* d_lexical, const float* d_lexical_max, float weight, int count,
                      cudaStream_t stream) {
    check(zcgvs_fuse_scores(d_dense, d_lexical, d_lexical_max, weight, count, stream), "zcgvs_fuse_scores");
}

void launchGatherRescore(const void* d_corpus, ScalarType dtype, float scale, int doc_count, int dim,
                         const float* d_queries, int batch, const int* d_candidate_indices, int candidate_count,
                         Metric metric, float* d_values, cudaStream_t stream) {
    check(zcgvs_gather_rescore(d_corpus, static_cast<int>(dtype), scale, nullptr, doc_count, dim, d_queries, batch,
                               d_candidate_indices, candidate_count, static_cast<int>(metric), d_values, stream),
          "zcgvs_gather_rescore");
}

void launchRemapIndices(const int* d_candidate_indices, const int* d_local_indices, int candidate_count, int k,
                        int batch, int* d_out_indices, cudaStream_t stream) {
    check(zcgvs_remap_indices(d_candidate_indices, d_local_indices, candidate_count, k, batch, d_out_indices, stream),
          "zcgvs_remap_indices");
}

std::size_t rescoreSharedBytes(int dim) { return static_cast<std::size_t>(dim) * sizeof(float); }

}  // namespace cuda

// ------------------------------------------------------------------------------------------
// EmbeddingStore
// ------------------------------------------------------------------------------------------
void EmbeddingStore::convertInto(std::uint8_t* destination, float* row_scales, const float* device_float32,
                                 std::int64_t rows, cudaStream_t stream) {
    const std::size_t elements = static_cast<std::size_t>(rows) * static_cast<std::size_t>(dim_);
    switch (dtype_) {
        case ScalarType::Float16: cuda::launchConvertF32ToF16(device_float32, destination, elements, stream); break;
        case ScalarType::Int8: cuda::launchConvertF32ToI8(device_float32, destination, elements, scale_, stream); break;
        case ScalarType::Int8PerRow:
            cuda::launchConvertF32ToI8Rows(device_float32, destination, row_scales, rows, dim_, stream);
            break;
        case ScalarType::Binary: cuda::launchPackBinary(device_float32, destination, static_cast<int>(rows), dim_, stream); break;
        default: throw std::invalid_argument("zcgvs: unsupported storage dtype");
    }
}

EmbeddingStore EmbeddingStore::fromHostMatrix(const float* host_float32, std::int64_t doc_count, int dim,
                                              ScalarType dtype, float scale, bool normalized) {
    if (host_float32 == nullptr || doc_count <= 0 || dim <= 0) {
        throw std::invalid_argument("zcgvs: fromHostMatrix requires a non-empty matrix");
    }
    EmbeddingStore store;
    store.dim_ = dim;
    store.dtype_ = dtype;
    store.normalized_ = normalized;
    store.scale_ = (dtype == ScalarType::Int8 && scale > 0.0f) ? scale : 1.0f;
    store.doc_count_ = doc_count;
    store.capacity_ = doc_count;
    store.device_.allocate(static_cast<std::size_t>(doc_count) * store.rowStride());
    if (dtype == ScalarType::Int8PerRow) store.row_scales_.allocate(static_cast<std::size_t>(doc_count));
    const std::size_t elements = static_cast<std::size_t>(doc_count) * static_cast<std::size_t>(dim);
    if (dtype == ScalarType::Float32) {
        ZCGVS_CUDA_CHECK(cudaMemcpy(store.device_.data(), host_float32, elements * sizeof(float), cudaMemcpyHostToDevice));
        return store;
    }
    DeviceBuffer<float> staging(elements);
    ZCGVS_CUDA_CHECK(cudaMemcpy(staging.data(), host_float32, elements * sizeof(float), cudaMemcpyHostToDevice));
    store.convertInto(store.device_.data(), store.row_scales_.data(), staging.data(), doc_count, nullptr);
    ZCGVS_CUDA_CHECK(cudaDeviceSynchronize());
    return store;
}

EmbeddingStore EmbeddingStore::loadFromFile(const std::string& path) {
    Reader in(path);
    in.magic(kEmbeddingMagic);
    const auto version = in.scalar<std::uint32_t>();
    if (version == 0 || version > kEmbeddingVersionRowScales) {
        throw std::runtime_error("zcgvs: unsupported embedding file version " + std::to_string(version));
    }
    const auto flags = in.scalar<std::uint32_t>();
    const auto doc_count = in.scalar<std::int64_t>();
    const auto dim = in.scalar<std::int32_t>();
    const auto code = in.scalar<std::int32_t>();
    if (doc_count <= 0 || dim <= 0) throw std::runtime_error("zcgvs: embedding file reports an empty matrix");
    if (code < 0 || code > 4) throw std::runtime_error("zcgvs: unsupported embedding dtype code " + std::to_string(code));
    if (code == kDtypeInt8PerRow && version < kEmbeddingVersionRowScales) {
        throw std::runtime_error("zcgvs: per-row int8 embeddings require file version 3");
    }
    EmbeddingStore store;
    store.dim_ = dim;
    store.dtype_ = static_cast<ScalarType>(code);
    store.normalized_ = (flags & kFlagNormalized) != 0;
    std::size_t stride = store.rowStride();
    if (version >= 2) {
        store.scale_ = in.scalar<float>();
        const auto recorded = in.scalar<std::int32_t>();
        if (recorded <= 0 || static_cast<std::size_t>(recorded) != stride) {
            throw std::runtime_error("zcgvs: embedding row stride does not match dtype and dim");
        }
    } else if (isQuantized(store.dtype_)) {
        throw std::runtime_error("zcgvs: quantized embeddings require file version 2");
    }
    const std::size_t total = static_cast<std::size_t>(doc_count) * stride;
    store.device_.allocate(total);
    in.toDevice(store.device_.data(), total);
    if (store.dtype_ == ScalarType::Int8PerRow) {
        store.row_scales_.allocate(static_cast<std::size_t>(doc_count));
        in.toDevice(store.row_scales_.data(), static_cast<std::size_t>(doc_count) * sizeof(float));
    }
    store.doc_count_ = doc_count;
    store.capacity_ = doc_count;
    return store;
}

void EmbeddingStore::ensureCapacity(std::int64_t required_docs, cudaStream_t stream) {
    if (capacity_ >= required_docs) return;
    const std::int64_t grown = std::max(required_docs, capacity_ * 2);
    DeviceBuffer<std::uint8_t> resized(static_cast<std::size_t>(grown) * rowStride());
    DeviceBuffer<float> resized_scales(dtype_ == ScalarType::Int8PerRow ? static_cast<std::size_t>(grown) : 0);
    if (doc_count_ > 0) {
        ZCGVS_CUDA_CHECK(cudaMemcpyAsync(resized.data(), device_.data(), static_cast<std::size_t>(doc_count_) * rowStride(),
                                         cudaMemcpyDeviceToDevice, stream));
        if (resized_scales.size() > 0) {
            ZCGVS_CUDA_CHECK(cudaMemcpyAsync(resized_scales.data(), row_scales_.data(),
                                             static_cast<std::size_t>(doc_count_) * sizeof(float),
                                             cudaMemcpyDeviceToDevice, stream));
        }
    }
    ZCGVS_CUDA_CHECK(cudaStreamSynchronize(stream));
    device_ = std::move(resized);
    row_scales_ = std::move(resized_scales);
    capacity_ = grown;
}

void EmbeddingStore::append(const float* host_float32, std::int64_t add_count, cudaStream_t stream) {
    if (add_count <= 0) return;
    if (dim_ <= 0) throw std::runtime_error("zcgvs: append requires an initialized store");
    ensureCapacity(doc_count_ + add_count, stream);
    const std::size_t elements = static_cast<std::size_t>(add_count) * static_cast<std::size_t>(dim_);
    std::uint8_t* destination = device_.data() + static_cast<std::size_t>(doc_count_) * rowStride();
    if (dtype_ == ScalarType::Float32) {
        ZCGVS_CUDA_CHECK(cudaMemcpyAsync(destination, host_float32, elements * sizeof(float), cudaMemcpyHostToDevice, stream));
    } else {
        DeviceBuffer<float> staging(elements);
        ZCGVS_CUDA_CHECK(cudaMemcpyAsync(staging.data(), host_float32, elements * sizeof(float), cudaMemcpyHostToDevice, stream));
        float* scales = row_scales_.size() > 0 ? row_scales_.data() + doc_count_ : nullptr;
        convertInto(destination, scales, staging.data(), add_count, stream);
        ZCGVS_CUDA_CHECK(cudaStreamSynchronize(stream));
    }
    ZCGVS_CUDA_CHECK(cudaStreamSynchronize(stream));
    doc_count_ += add_count;
}

// ------------------------------------------------------------------------------------------
// LexicalIndex
// ------------------------------------------------------------------------------------------
LexicalIndex LexicalIndex::fromHostCsr(const std::int64_t* offsets, int vocab_size, const int* docs,
                                       const float* weights, std::int64_t doc_count, float k1, float b,
                                       float average_doc_length) {
    if (offsets == nullptr || vocab_size <= 0 || doc_count <= 0) throw std::invalid_argument("zcgvs: empty lexical index");
    std::vector<std::int64_t> off(offsets, offsets + vocab_size + 1);
    if (off.front() != 0 || !std::is_sorted(off.begin(), off.end())) {
        throw std::invalid_argument("zcgvs: lexical index CSR offsets are inconsistent");
    }
    const std::size_t nnz = static_cast<std::size_t>(off.back());
    std::vector<int> d(docs, docs + nnz);
    std::vector<float> w(weights, weights + nnz);
    sort_postings(off, d, w);
    LexicalIndex index;
    index.doc_count_ = doc_count;
    index.vocab_size_ = vocab_size;
    index.posting_count_ = static_cast<std::int64_t>(nnz);
    index.k1_ = k1;
    index.b_ = b;
    index.average_doc_length_ = average_doc_length;
    index.offsets_.allocate(off.size());
    ZCGVS_CUDA_CHECK(cudaMemcpy(index.offsets_.data(), off.data(), off.size() * sizeof(std::int64_t), cudaMemcpyHostToDevice));
    if (nnz > 0) {
        index.posting_docs_.allocate(nnz);
        index.posting_weights_.allocate(nnz);
        ZCGVS_CUDA_CHECK(cudaMemcpy(index.posting_docs_.data(), d.data(), nnz * sizeof(int), cudaMemcpyHostToDevice));
        ZCGVS_CUDA_CHECK(cudaMemcpy(index.posting_weights_.data(), w.data(), nnz * sizeof(float), cudaMemcpyHostToDevice));
    }
    return index;
}

LexicalIndex LexicalIndex::loadFromFile(const std::string& path) {
    Reader in(path);
    in.magic(kLexicalMagic);
    const auto version = in.scalar<std::uint32_t>();
    if (version != kLexicalVersion) throw std::runtime_error("zcgvs: unsupported lexical index version " + std::to_string(version));
    const auto doc_count = in.scalar<std::int64_t>();
    const auto vocab = in.scalar<std::int32_t>();
    const auto nnz = in.scalar<std::int64_t>();
    const float k1 = in.scalar<float>();
    const float b = in.scalar<float>();
    const float avgdl = in.scalar<float>();
    if (doc_count <= 0 || vocab <= 0 || nnz < 0) throw std::runtime_error("zcgvs: lexical index header describes an empty index");
    std::vector<std::int64_t> offsets(static_cast<std::size_t>(vocab) + 1);
    in.bytes(offsets.data(), offsets.size() * sizeof(std::int64_t));
    if (offsets.front() != 0 || offsets.back() != nnz) throw std::runtime_error("zcgvs: lexical index CSR offsets are inconsistent with nnz");
    std::vector<int> docs(static_cast<std::size_t>(nnz));
    std::vector<float> weights(static_cast<std::size_t>(nnz));
    if (nnz > 0) {
        in.bytes(docs.data(), docs.size() * sizeof(int));
        in.bytes(weights.data(), weights.size() * sizeof(float));
    }
    return fromHostCsr(offsets.data(), vocab, docs.data(), weights.data(), doc_count, k1, b, avgdl);
}

// ------------------------------------------------------------------------------------------
// Corpus: embeddings + ZCVM metadata
// ------------------------------------------------------------------------------------------
Corpus Corpus::load(const std::string& embeddings_path, const std::string& metadata_path) {
    Corpus corpus;
    corpus.embeddings_ = EmbeddingStore::loadFromFile(embeddings_path);
    Reader in(metadata_path);
    in.magic(kMetadataMagic);
    const auto version = in.scalar<std::uint32_t>();
    if (version != kMetadataVersion) throw std::runtime_error("zcgvs: unsupported metadata version " + std::to_string(version));
    const auto count = in.scalar<std::int64_t>();
    if (count != corpus.embeddings_.docCount()) {
        throw std::runtime_error("zcgvs: metadata lists " + std::to_string(count) + " documents, the embeddings " +
                                 std::to_string(corpus.embeddings_.docCount()));
    }
    corpus.doc_ids_.reserve(static_cast<std::size_t>(count));
    corpus.texts_.reserve(static_cast<std::size_t>(count));
    for (std::int64_t i = 0; i < count; ++i) {
        corpus.doc_ids_.push_back(in.text(in.scalar<std::uint32_t>()));
        corpus.texts_.push_back(in.text(in.scalar<std::uint32_t>()));
    }
    return corpus;
}

void Corpus::addDocuments(const std::vector<std::string>& ids, const std::vector<std::string>& texts,
                          const float* host_float32, std::int64_t add_count, cudaStream_t stream) {
    if (static_cast<std::int64_t>(ids.size()) != add_count || static_cast<std::int64_t>(texts.size()) != add_count) {
        throw std::runtime_error("zcgvs: addDocuments needs one id and one text per added row");
    }
    if (add_count <= 0) return;
    embeddings_.append(host_float32, add_count, stream);
    doc_ids_.insert(doc_ids_.end(), ids.begin(), ids.end());
    texts_.insert(texts_.end(), texts.begin(), texts.end());
}

// ------------------------------------------------------------------------------------------
// Device context
// ------------------------------------------------------------------------------------------
void setDevice(int device_id) { ZCGVS_CUDA_CHECK(cudaSetDevice(device_id)); }

int currentDevice() {
    int device = 0;
    ZCGVS_CUDA_CHECK(cudaGetDevice(&device));
    return device;
}

int deviceCount() {
    int count = 0;
    ZCGVS_CUDA_CHECK(cudaGetDeviceCount(&count));
    return count;
}

DeviceInfo queryDevice(int device_id) {
    cudaDeviceProp prop{};
    ZCGVS_CUDA_CHECK(cudaGetDeviceProperties(&prop, device_id));
    int memory_khz = 0;  // an attribute: the property field is gone from newer runtimes
    ZCGVS_CUDA_CHECK(cudaDeviceGetAttribute(&memory_khz, cudaDevAttrMemoryClockRate, device_id));
    DeviceInfo info;
    info.device_id = device_id;
    info.name = prop.name;
    info.total_memory = prop.totalGlobalMem;
    info.compute_major = prop.major;
    info.compute_minor = prop.minor;
    info.multiprocessor_count = prop.multiProcessorCount;
    info.memory_clock_khz = memory_khz;
    info.memory_bus_width_bits = prop.memoryBusWidth;
    return info;
}

// ------------------------------------------------------------------------------------------
// Searcher
// ------------------------------------------------------------------------------------------
namespace {

template <typename Buffer>
bool grow(Buffer& buffer, std::size_t required) {
    if (buffer.size() >= required) return false;
    buffer.allocate(required);
    return true;
}

}  // namespace

// The bit pattern of one launch argument, for the graph key.
std::uint64_t argBits(const void* p) { return static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(p)); }
std::uint64_t argBits(std::int64_t v) { return static_cast<std::uint64_t>(v); }
std::uint64_t argBits(int v) { return static_cast<std::uint64_t>(static_cast<std::uint32_t>(v)); }
std::uint64_t argBits(std::size_t v) { return static_cast<std::uint64_t>(v); }
std::uint64_t argBits(float v) {
    std::uint32_t bits = 0;
    std::memcpy(&bits, &v, sizeof(bits));
    return bits;
}

// Either launches fn(args..., stream) or, when `key` is given, appends the arguments' bits to it
// instead: the graph key of a captured search is the exact argument list of its launches.
template <typename Fn, typename... Args>
void launchOrKey(std::vector<std::uint64_t>* key, const char* name, Fn fn, cudaStream_t stream, Args... args) {
    if (key != nullptr) {
        key->push_back(argBits(reinterpret_cast<const void*>(fn)));
        (key->push_back(argBits(args)), ...);
        return;
    }
    check(fn(args..., stream), name);
}

Searcher::Searcher(const EmbeddingStore& store) : store_(store), dim_(store.dim()) {
    ZCGVS_CUDA_CHECK(cudaEventCreate(&ev_start_));
    ZCGVS_CUDA_CHECK(cudaEventCreate(&ev_end_));
}

Searcher::~Searcher() {
    destroyGraph();
    if (ev_start_ != nullptr) cudaEventDestroy(ev_start_);
    if (ev_end_ != nullptr) cudaEventDestroy(ev_end_);
}

void Searcher::destroyGraph() noexcept {
    if (graph_exec_ != nullptr) cudaGraphExecDestroy(graph_exec_);
    graph_exec_ = nullptr;
    graph_valid_ = false;
}

void Searcher::setRescoreStore(const EmbeddingStore* store) {
    if (store != nullptr) {
        if (store->dim() != dim_) throw std::invalid_argument("zcgvs: rescore store dim does not match the corpus");
        if (store->dtype() == ScalarType::Binary) throw std::invalid_argument("zcgvs: rescore store must not be binary");
    }
    rescore_store_ = store;
    destroyGraph();
}

void Searcher::setLexicalIndex(const LexicalIndex* index) {
    lexical_index_ = index;
    destroyGraph();
}

bool Searcher::lexicalEnabled(const SearchParams& params) const {
    return lexical_index_ != nullptr && params.lexical_stride > 0 && params.host_query_terms != nullptr;
}

bool Searcher::rescoreEnabled(const SearchParams& params) const {
    return rescore_store_ != nullptr && params.rescore_candidates > 0;
}

void Searcher::validate(int dim, int batch, const SearchParams& params, std::int64_t doc_count) const {
    if (dim != dim_) {
        throw std::invalid_argument("zcgvs: query dim " + std::to_string(dim) + " does not match corpus dim " +
                                    std::to_string(dim_));
    }
    if (batch <= 0) throw std::invalid_argument("zcgvs: batch must be positive");
    if (params.k <= 0) throw std::invalid_argument("zcgvs: k must be positive");
    if (doc_count > static_cast<std::int64_t>(INT32_MAX)) throw std::runtime_error("zcgvs: corpus exceeds the supported document count");
    if (params.k > doc_count) {
        throw std::invalid_argument("zcgvs: k=" + std::to_string(params.k) + " exceeds corpus size " + std::to_string(doc_count));
    }
    if (params.k > ZCGVS_MAX_K) {
        throw std::invalid_argument("zcgvs: k=" + std::to_string(params.k) + " exceeds kernel capacity " +
                                    std::to_string(ZCGVS_MAX_K));
    }
    if (rescoreEnabled(params)) {
        if (params.rescore_candidates < params.k) throw std::invalid_argument("zcgvs: rescore_candidates must be at least k");
        if (params.rescore_candidates > doc_count) throw std::invalid_argument("zcgvs: rescore_candidates exceeds corpus size");
        if (params.rescore_candidates > ZCGVS_MAX_K) {
            throw std::invalid_argument("zcgvs: rescore_candidates=" + std::to_string(params.rescore_candidates) +
                                        " exceeds kernel capacity " + std::to_string(ZCGVS_MAX_K));
        }
        if (rescore_store_->docCount() < doc_count) {
            throw std::invalid_argument("zcgvs: rescore store holds fewer documents than the corpus");
        }
    }
    if (lexicalEnabled(params) && lexical_index_->docCount() < doc_count) {
        throw std::invalid_argument("zcgvs: lexical index holds fewer documents than the corpus");
    }
}

void Searcher::ensureCapacity(std::int64_t doc_count, int batch, const SearchParams& params) {
    const int width = rescoreEnabled(params) ? params.rescore_candidates : params.k;
    const int dtype = static_cast<int>(store_.dtype());
    const std::size_t ws = lexicalEnabled(params)
                               ? zcgvs_hybrid_topk_workspace_bytes(dtype, doc_count, dim_, batch, width)
                               : zcgvs_scan_topk_workspace_bytes(dtype, doc_count, dim_, batch, width);
    const std::size_t queries = static_cast<std::size_t>(batch);
    bool reallocated = false;
    if (grow(d_workspace_, std::max<std::size_t>(ws, 256))) {
        d_workspace_.fillZero();  // the streaming scan's counters start at zero once
        reallocated = true;
    }
    reallocated |= grow(d_queries_, queries * static_cast<std::size_t>(dim_));
    reallocated |= grow(d_out_indices_, queries * static_cast<std::size_t>(params.k));
    reallocated |= grow(d_out_values_, queries * static_cast<std::size_t>(params.k));
    if (rescoreEnabled(params)) {
        reallocated |= grow(d_coarse_indices_, queries * static_cast<std::size_t>(width));
        reallocated |= grow(d_coarse_values_, queries * static_cast<std::size_t>(width));
    }
    if (lexicalEnabled(params)) {
        reallocated |= grow(d_query_terms_, queries * static_cast<std::size_t>(params.lexical_stride));
        grow(h_query_terms_, queries * static_cast<std::size_t>(params.lexical_stride));
    }
    grow(h_queries_, queries * static_cast<std::size_t>(dim_));
    grow(h_out_indices_, queries * static_cast<std::size_t>(params.k));
    grow(h_out_values_, queries * static_cast<std::size_t>(params.k));
    grow(h_status_, 1);
    if (reallocated) destroyGraph();
}

void Searcher::recordPipeline(std::int64_t doc_count, int batch, const SearchParams& params, cudaStream_t stream,
                              std::vector<std::uint64_t>* key) {
    const bool rescore = rescoreEnabled(params);
    const int width = rescore ? params.rescore_candidates : params.k;
    // The final results go to the pinned host buffers themselves when they are small (host_out_):
    // the last kernel writes them across the bus, so copyResultToHost has no copy to make.
    int* out_ids = host_out_ ? h_out_indices_.data() : d_out_indices_.data();
    float* out_scores = host_out_ ? h_out_values_.data() : d_out_values_.data();
    int* ids = rescore ? d_coarse_indices_.data() : out_ids;
    float* scores = rescore ? d_coarse_values_.data() : out_scores;
    const int dtype = static_cast<int>(store_.dtype());
    const int metric = static_cast<int>(params.metric);
    const std::int64_t n = doc_count;
    if (lexicalEnabled(params)) {
        launchOrKey(key, "zcgvs_hybrid_topk", zcgvs_hybrid_topk, stream, store_.deviceData(), dtype, store_.scale(),
                    store_.rowScales(), n, dim_, static_cast<const float*>(d_queries_.data()), batch, params.d_mask,
                    metric, lexical_index_->deviceOffsets(), lexical_index_->devicePostingDocs(),
                    lexical_index_->devicePostingWeights(), lexical_index_->vocabSize(),
                    static_cast<const int*>(d_query_terms_.data()), params.lexical_stride, params.dense_weight, width,
                    ids, scores, static_cast<void*>(d_workspace_.data()), d_workspace_.bytes());
    } else {
        launchOrKey(key, "zcgvs_scan_topk", zcgvs_scan_topk, stream, store_.deviceData(), dtype, store_.scale(),
                    store_.rowScales(), n, dim_, static_cast<const float*>(d_queries_.data()), batch, params.d_mask,
                    metric, width, 0, ids, scores, static_cast<void*>(d_workspace_.data()), d_workspace_.bytes());
    }
    if (rescore) {
        launchOrKey(key, "zcgvs_rescore_topk", zcgvs_rescore_topk, stream, rescore_store_->deviceData(),
                    static_cast<int>(rescore_store_->dtype()), rescore_store_->scale(), rescore_store_->rowScales(),
                    rescore_store_->docCount(), dim_, static_cast<const float*>(d_queries_.data()), batch,
                    static_cast<const int*>(d_coarse_indices_.data()), width, metric, params.k, out_ids, out_scores);
    }
}

void Searcher::search(const float* host_queries, int dim, int batch, const SearchParams& params, const CudaStream& stream) {
    const std::int64_t doc_count = store_.docCount();
    validate(dim, batch, params, doc_count);
    ensureCapacity(doc_count, batch, params);

    // Host queries (and terms) through pinned staging, asynchronously on the caller's stream.
    const std::size_t elements = static_cast<std::size_t>(batch) * static_cast<std::size_t>(dim_);
    std::memcpy(h_queries_.data(), host_queries, elements * sizeof(float));
    d_queries_.copyFromHost(h_queries_.data(), elements, stream.get());
    if (lexicalEnabled(params)) {
        const std::size_t terms = static_cast<std::size_t>(batch) * static_cast<std::size_t>(params.lexical_stride);
        std::memcpy(h_query_terms_.data(), params.host_query_terms, terms * sizeof(int));
        d_query_terms_.copyFromHost(h_query_terms_.data(), terms, stream.get());
    }

    host_out_ = static_cast<long long>(batch) * params.k <= kHostResultMax;
    const bool graph_path = params.use_graph;
    if (graph_path) {
        std::vector<std::uint64_t> key;
        recordPipeline(doc_count, batch, params, stream.get(), &key);
        if (!graph_valid_ || graph_key_ != key) {
            // Capture outside the timed region; the uploads above are drained first so the graph
            // holds the search and nothing else.
            stream.synchronize();
            cudaGraph_t graph = nullptr;
            ZCGVS_CUDA_CHECK(cudaStreamBeginCapture(stream.get(), cudaStreamCaptureModeThreadLocal));
            try {
                recordPipeline(doc_count, batch, params, stream.get());
            } catch (...) {
                cudaStreamEndCapture(stream.get(), &graph);
                if (graph != nullptr) cudaGraphDestroy(graph);
                throw;
            }
            ZCGVS_CUDA_CHECK(cudaStreamEndCapture(stream.get(), &graph));
            destroyGraph();
            const cudaError_t status = cudaGraphInstantiateWithFlags(&graph_exec_, graph, 0);
            cudaGraphDestroy(graph);
            ZCGVS_CUDA_CHECK(status);
            graph_valid_ = true;
            graph_key_ = std::move(key);
            ++graph_captures_;
        }
    }

    ZCGVS_CUDA_CHECK(cudaEventRecord(ev_start_, stream.get()));
    if (graph_path) {
        ZCGVS_CUDA_CHECK(cudaGraphLaunch(graph_exec_, stream.get()));
        ++graph_launches_;
    } else {
        recordPipeline(doc_count, batch, params, stream.get());
    }
    ZCGVS_CUDA_CHECK(cudaEventRecord(ev_end_, stream.get()));
    used_graph_ = graph_path;
    current_k_ = params.k;
    current_batch_ = batch;
}

HostTopK Searcher::copyResultToHost(const CudaStream& stream) {
    if (current_k_ == 0 || current_batch_ == 0) throw std::runtime_error("zcgvs: copyResultToHost called before search");
    const std::size_t elements = static_cast<std::size_t>(current_batch_) * static_cast<std::size_t>(current_k_);
    if (!host_out_) {
        d_out_indices_.copyToHost(h_out_indices_.data(), elements, stream.get());
        d_out_values_.copyToHost(h_out_values_.data(), elements, stream.get());
    }
    // The device status word (first 4 bytes of the workspace) travels with the result.
    ZCGVS_CUDA_CHECK(cudaMemcpyAsync(h_status_.data(), d_workspace_.data(), sizeof(std::uint32_t),
                                     cudaMemcpyDeviceToHost, stream.get()));
    stream.synchronize();
    if (const std::uint32_t word = h_status_.data()[0]; word != 0u) {
        ZCGVS_CUDA_CHECK(cudaMemsetAsync(d_workspace_.data(), 0, sizeof(std::uint32_t), stream.get()));
        stream.synchronize();
        throw std::runtime_error("zcgvs: search incomplete, " + describeDeviceStatus(word));
    }
    HostTopK result;
    result.batch = current_batch_;
    result.k = current_k_;
    result.indices.assign(h_out_indices_.data(), h_out_indices_.data() + elements);
    result.scores.assign(h_out_values_.data(), h_out_values_.data() + elements);
    float elapsed_ms = 0.0f;
    ZCGVS_CUDA_CHECK(cudaEventElapsedTime(&elapsed_ms, ev_start_, ev_end_));
    last_gpu_ms_ = static_cast<double>(elapsed_ms);
    return result;
}

// ------------------------------------------------------------------------------------------
// ShardedSearcher
// ------------------------------------------------------------------------------------------
std::vector<char> ShardedSearcher::uniqueId() {
    std::vector<char> id(zcgvs_nccl_id_bytes());
    check(zcgvs_nccl_unique_id(id.data()), "zcgvs_nccl_unique_id");
    return id;
}

void ShardedSearcher::shardBounds(std::int64_t total_rows, int world, int rank, std::int64_t* begin,
                                  std::int64_t* end) {
    check(zcgvs_shard_bounds(total_rows, world, rank, begin, end), "zcgvs_shard_bounds");
}

ShardedSearcher::ShardedSearcher(const std::vector<char>& nccl_id, int world, int rank, std::int64_t total_rows) {
    if (nccl_id.size() != zcgvs_nccl_id_bytes()) throw std::invalid_argument("zcgvs: the NCCL id has the wrong size");
    check(zcgvs_sharded_create(nccl_id.data(), world, rank, total_rows, &handle_), "zcgvs_sharded_create");
    shardBounds(total_rows, world, rank, &begin_, &end_);
}

ShardedSearcher::~ShardedSearcher() { zcgvs_sharded_destroy(handle_); }

void ShardedSearcher::setRescoreStore(const EmbeddingStore* shard_store) {
    if (shard_store != nullptr) {
        if (shard_store->dtype() == ScalarType::Binary) throw std::invalid_argument("zcgvs: rescore store must not be binary");
        if (shard_store->docCount() != end_ - begin_) {
            throw std::invalid_argument("zcgvs: the rescore store must hold this rank's shard rows");
        }
    }
    rescore_store_ = shard_store;
}

void ShardedSearcher::search(const EmbeddingStore& shard, const float* host_queries, int dim, int batch,
                             const SearchParams& params, const CudaStream& stream) {
    if (dim != shard.dim()) throw std::invalid_argument("zcgvs: query dim does not match the shard");
    if (batch <= 0 || params.k <= 0) throw std::invalid_argument("zcgvs: batch and k must be positive");
    const bool rescore = rescore_store_ != nullptr && params.rescore_candidates > 0;
    if (rescore && rescore_store_->dim() != dim) throw std::invalid_argument("zcgvs: rescore store dim differs");
    const std::size_t elements = static_cast<std::size_t>(batch) * static_cast<std::size_t>(dim);
    const std::size_t results = static_cast<std::size_t>(batch) * static_cast<std::size_t>(params.k);
    grow(d_queries_, elements);
    grow(h_queries_, elements);
    grow(d_out_indices_, results);
    grow(d_out_values_, results);
    grow(h_out_indices_, results);
    grow(h_out_values_, results);
    std::memcpy(h_queries_.data(), host_queries, elements * sizeof(float));
    d_queries_.copyFromHost(h_queries_.data(), elements, stream.get());
    const unsigned flags = params.use_graph ? ZCGVS_SHARDED_GRAPH : 0u;
    if (rescore) {
        check(zcgvs_sharded_rescore_search(handle_, shard.deviceData(), static_cast<int>(shard.dtype()), shard.scale(),
                                           shard.rowScales(), rescore_store_->deviceData(),
                                           static_cast<int>(rescore_store_->dtype()), rescore_store_->scale(),
                                           rescore_store_->rowScales(), shard.docCount(), dim, d_queries_.data(), batch,
                                           static_cast<int>(params.metric), params.rescore_candidates, params.k, flags,
                                           d_out_indices_.data(), d_out_values_.data(), stream.get()),
              "zcgvs_sharded_rescore_search");
    } else {
        check(zcgvs_sharded_search(handle_, shard.deviceData(), static_cast<int>(shard.dtype()), shard.scale(),
                                   shard.rowScales(), shard.docCount(), dim, d_queries_.data(), batch, params.d_mask,
                                   static_cast<int>(params.metric), params.k, flags, d_out_indices_.data(),
                                   d_out_values_.data(), stream.get()),
              "zcgvs_sharded_search");
    }
    current_k_ = params.k;
    current_batch_ = batch;
}

HostTopK ShardedSearcher::copyResultToHost(const CudaStream& stream) {
    if (current_k_ == 0) throw std::runtime_error("zcgvs: copyResultToHost called before search");
    const std::size_t elements = static_cast<std::size_t>(current_batch_) * static_cast<std::size_t>(current_k_);
    d_out_indices_.copyToHost(h_out_indices_.data(), elements, stream.get());
    d_out_values_.copyToHost(h_out_values_.data(), elements, stream.get());
    std::uint32_t word = 0;
    int comm_error = 0;
    check(zcgvs_sharded_status(handle_, &word, &comm_error, stream.get()), "zcgvs_sharded_status");
    if (comm_error != 0) throw std::runtime_error("zcgvs: NCCL reported asynchronous error " + std::to_string(comm_error));
    if (word != 0u) {
        check(zcgvs_sharded_clear_status(handle_, stream.get()), "zcgvs_sharded_clear_status");
        stream.synchronize();
        throw std::runtime_error("zcgvs: search incomplete, " + describeDeviceStatus(word));
    }
    HostTopK result;
    result.batch = current_batch_;
    result.k = current_k_;
    result.indices.assign(h_out_indices_.data(), h_out_indices_.data() + elements);
    result.scores.assign(h_out_values_.data(), h_out_values_.data() + elements);
    return result;
}

}  // namespace zcgvs
