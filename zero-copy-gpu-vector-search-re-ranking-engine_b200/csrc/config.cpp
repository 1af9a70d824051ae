// JSON engine configs (include/zcgvs/engine/config_loader.hpp): a small JSON reader and the field
// mapping of the reference's python/zcgvs_tools/config.py:54-96.
#include "zcgvs/engine/config_loader.hpp"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <climits>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <functional>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace zcgvs {

namespace {

// A parsed JSON value.
struct Json {
    enum class Kind { Null, Bool, Number, String, Array, Object } kind = Kind::Null;
    bool boolean = false;
    double number = 0.0;
    bool integral = false;  // written without fraction or exponent
    long long integer = 0;  // its value when integral and in range
    std::string text;
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> fields;  // in document order
};

class JsonReader {
public:
    explicit JsonReader(const std::string& text) : s_(text) {}

    Json document() {
        Json v = value(0);
        skip();
        if (at_ != s_.size()) error("trailing characters after the value");
        return v;
    }

private:
    [[noreturn]] void error(const std::string& what) const {
        throw std::invalid_argument("zcgvs config: invalid JSON (" + what + ") at offset " + std::to_string(at_));
    }

    void skip() {
        while (at_ < s_.size() && (s_[at_] == ' ' || s_[at_] == '\t' || s_[at_] == '\n' || s_[at_] == '\r')) ++at_;
    }

    char peek() {
        skip();
        if (at_ >= s_.size()) error("unexpected end");
        return s_[at_];
    }

    void expect(const char* word) {
        const std::size_t n = std::char_traits<char>::length(word);
        if (s_.compare(at_, n, word) != 0) error(std::string("expected '") + word + "'");
        at_ += n;
    }

    Json value(int depth) {
        if (depth > 64) error("nesting too deep");
        Json v;
        const char c = peek();
        if (c == '{') {
            v.kind = Json::Kind::Object;
            ++at_;
            if (peek() == '}') {
                ++at_;
                return v;
            }
            for (;;) {
                if (peek() != '"') error("expected a member name");
                std::string key = string();
                if (peek() != ':') error("expected ':'");
                ++at_;
                v.fields.emplace_back(std::move(key), value(depth + 1));
                const char d = peek();
                ++at_;
                if (d == '}') return v;
                if (d != ',') error("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::Kind::Array;
            ++at_;
            if (peek() == ']') {
                ++at_;
                return v;
            }
            for (;;) {
                v.items.push_back(value(depth + 1));
                const char d = peek();
                ++at_;
                if (d == ']') return v;
                if (d != ',') error("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::Kind::String;
            v.text = string();
            return v;
        }
        if (c == 't' || c == 'f') {
            v.kind = Json::Kind::Bool;
            v.boolean = c == 't';
            expect(v.boolean ? "true" : "false");
            return v;
        }
        if (c == 'n') {
            expect("null");
            return v;
        }
        return number();
    }

    Json number() {
        const std::size_t start = at_;
        if (s_[at_] == '-') ++at_;
        auto digits = [&] {
            const std::size_t from = at_;
            while (at_ < s_.size() && std::isdigit(static_cast<unsigned char>(s_[at_]))) ++at_;
            return at_ - from;
        };
        if (at_ >= s_.size() || !std::isdigit(static_cast<unsigned char>(s_[at_]))) error("expected a value");
        if (s_[at_] == '0') {
            ++at_;
        } else {
            digits();
        }
        bool integral = true;
        if (at_ < s_.size() && s_[at_] == '.') {
            ++at_;
            if (digits() == 0) error("expected digits after '.'");
            integral = false;
        }
        if (at_ < s_.size() && (s_[at_] == 'e' || s_[at_] == 'E')) {
            ++at_;
            if (at_ < s_.size() && (s_[at_] == '+' || s_[at_] == '-')) ++at_;
            if (digits() == 0) error("expected exponent digits");
            integral = false;
        }
        const std::string literal = s_.substr(start, at_ - start);
        Json v;
        v.kind = Json::Kind::Number;
        v.number = std::strtod(literal.c_str(), nullptr);
        if (integral) {
            errno = 0;
            const long long i = std::strtoll(literal.c_str(), nullptr, 10);
            v.integral = errno != ERANGE;
            v.integer = i;
        }
        return v;
    }

    unsigned hex4() {
        if (at_ + 4 > s_.size()) error("short \\u escape");
        unsigned code = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = s_[at_++];
            code <<= 4;
            if (h >= '0' && h <= '9') {
                code |= static_cast<unsigned>(h - '0');
            } else if (h >= 'a' && h <= 'f') {
                code |= static_cast<unsigned>(h - 'a' + 10);
            } else if (h >= 'A' && h <= 'F') {
                code |= static_cast<unsigned>(h - 'A' + 10);
            } else {
                error("bad \\u escape");
            }
        }
        return code;
    }

    static void utf8(std::string& out, unsigned cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }

    std::string string() {
        ++at_;  // opening quote
        std::string out;
        for (;;) {
            if (at_ >= s_.size()) error("unterminated string");
            const char c = s_[at_++];
            if (c == '"') return out;
            if (static_cast<unsigned char>(c) < 0x20) error("control character in a string");
            if (c != '\\') {
                out += c;
                continue;
            }
            if (at_ >= s_.size()) error("unterminated escape");
            const char e = s_[at_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    unsigned cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && s_.compare(at_, 2, "\\u") == 0) {
                        at_ += 2;
                        const unsigned low = hex4();
                        if (low < 0xDC00 || low >= 0xE000) error("unpaired surrogate");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (low - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: error("unknown escape");
            }
        }
    }

    const std::string& s_;
    std::size_t at_ = 0;
};

std::string lower(std::string text) {
    std::transform(text.begin(), text.end(), text.begin(), [](unsigned char c) { return static_cast<char>(std::tolower(c)); });
    return text;
}

[[noreturn]] void wrong_type(const std::string& field, const char* want) {
    throw std::invalid_argument("zcgvs config: field '" + field + "' needs " + want);
}

std::string as_string(const std::string& field, const Json& v) {
    if (v.kind != Json::Kind::String) wrong_type(field, "a string");
    return v.text;
}

int as_int(const std::string& field, const Json& v) {
    if (v.kind != Json::Kind::Number || !v.integral || v.integer < INT_MIN || v.integer > INT_MAX) {
        wrong_type(field, "an integer");
    }
    return static_cast<int>(v.integer);
}

float as_float(const std::string& field, const Json& v) {
    if (v.kind != Json::Kind::Number) wrong_type(field, "a number");
    return static_cast<float>(v.number);
}

bool as_bool(const std::string& field, const Json& v) {
    if (v.kind != Json::Kind::Bool) wrong_type(field, "true or false");
    return v.boolean;
}

// An artifact path as written, or resolved against the first search root that holds it.
std::string resolve_path(const std::string& value, const std::vector<std::string>& roots) {
    namespace fs = std::filesystem;
    std::error_code ec;
    const fs::path candidate(value);
    if (candidate.is_absolute() || fs::exists(candidate, ec)) return value;
    for (const std::string& root : roots) {
        const fs::path resolved = fs::path(root) / candidate;
        if (fs::exists(resolved, ec)) return resolved.string();
    }
    return value;
}

using Setter = std::function<void(EngineConfig&, const std::string&, const Json&)>;

const std::map<std::string, Setter>& setters() {
    static const std::map<std::string, Setter> table = [] {
        std::map<std::string, Setter> t;
        auto text = [&](const char* name, std::string EngineConfig::*member) {
            t[name] = [member](EngineConfig& c, const std::string& f, const Json& v) { c.*member = as_string(f, v); };
        };
        auto integer = [&](const char* name, int EngineConfig::*member) {
            t[name] = [member](EngineConfig& c, const std::string& f, const Json& v) { c.*member = as_int(f, v); };
        };
        auto flag = [&](const char* name, bool EngineConfig::*member) {
            t[name] = [member](EngineConfig& c, const std::string& f, const Json& v) { c.*member = as_bool(f, v); };
        };
        text("embeddings_path", &EngineConfig::embeddings_path);
        text("metadata_path", &EngineConfig::metadata_path);
        text("vocab_path", &EngineConfig::vocab_path);
        text("rescore_embeddings_path", &EngineConfig::rescore_embeddings_path);
        text("lexical_index_path", &EngineConfig::lexical_index_path);
        text("encoder_model_path", &EngineConfig::encoder_model_path);
        text("encoder_output_name", &EngineConfig::encoder_output_name);
        integer("encoder_max_seq_len", &EngineConfig::encoder_max_seq_len);
        text("reranker_model_path", &EngineConfig::reranker_model_path);
        text("reranker_output_name", &EngineConfig::reranker_output_name);
        integer("reranker_max_seq_len", &EngineConfig::reranker_max_seq_len);
        integer("reranker_batch_size", &EngineConfig::reranker_batch_size);
        integer("device_id", &EngineConfig::device_id);
        flag("lowercase", &EngineConfig::lowercase);
        integer("default_top_k", &EngineConfig::default_top_k);
        integer("default_candidates", &EngineConfig::default_candidates);
        integer("rescore_candidates", &EngineConfig::rescore_candidates);
        flag("hybrid", &EngineConfig::hybrid);
        integer("max_query_terms", &EngineConfig::max_query_terms);
        flag("use_cuda_graphs", &EngineConfig::use_cuda_graphs);
        t["dense_weight"] = [](EngineConfig& c, const std::string& f, const Json& v) { c.dense_weight = as_float(f, v); };
        t["metric"] = [](EngineConfig& c, const std::string& f, const Json& v) {
            c.metric = configMetricFromName(as_string(f, v));
        };
        t["similarity_backend"] = [](EngineConfig& c, const std::string& f, const Json& v) {
            c.similarity_backend = similarityBackendFromName(as_string(f, v));
        };
        t["reranker_backend"] = [](EngineConfig& c, const std::string& f, const Json& v) {
            if (lower(as_string(f, v)) != "onnx") throw std::invalid_argument("zcgvs config: unknown reranker backend");
            c.reranker_backend = RerankerBackend::Onnx;
        };
        return t;
    }();
    return table;
}

bool is_path_field(const std::string& key) {
    static const char* const kPaths[] = {"embeddings_path",         "metadata_path",      "vocab_path",
                                         "rescore_embeddings_path", "lexical_index_path", "encoder_model_path",
                                         "reranker_model_path"};
    return std::find(std::begin(kPaths), std::end(kPaths), key) != std::end(kPaths);
}

}  // namespace

Metric configMetricFromName(const std::string& name) {
    const std::string n = lower(name);
    if (n == "cosine") return Metric::Cosine;
    if (n == "dot" || n == "dotproduct" || n == "ip") return Metric::DotProduct;
    if (n == "l2" || n == "euclidean") return Metric::L2;
    throw std::invalid_argument("unknown metric '" + name + "'");
}

SimilarityBackend similarityBackendFromName(const std::string& name) {
    const std::string n = lower(name);
    if (n == "custom") return SimilarityBackend::Custom;
    if (n == "cublas") return SimilarityBackend::Cublas;
    throw std::invalid_argument("unknown similarity backend '" + name + "'");
}

EngineConfig configFromJsonText(const std::string& json, const std::vector<std::string>& search_roots) {
    const Json doc = JsonReader(json).document();
    if (doc.kind != Json::Kind::Object) throw std::invalid_argument("zcgvs config: the document must be a JSON object");
    EngineConfig config;
    const auto& table = setters();
    for (const auto& [key, value] : doc.fields) {
        const auto it = table.find(key);
        if (it == table.end()) throw std::invalid_argument("unknown config field: " + key);
        if (is_path_field(key) && !search_roots.empty() && value.kind == Json::Kind::String && !value.text.empty()) {
            Json resolved = value;
            resolved.text = resolve_path(value.text, search_roots);
            it->second(config, key, resolved);
        } else {
            it->second(config, key, value);
        }
    }
    return config;
}

EngineConfig configFromJsonFile(const std::string& path) {
    namespace fs = std::filesystem;
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("zcgvs config: cannot read '" + path + "'");
    std::ostringstream text;
    text << in.rdbuf();
    std::error_code ec;
    const fs::path file = fs::absolute(fs::path(path), ec);
    const fs::path dir = file.parent_path();
    return configFromJsonText(text.str(), {dir.string(), dir.parent_path().string()});
}

VectorEngineConfig toVectorEngineConfig(const EngineConfig& config) {
    VectorEngineConfig v;
    v.metric = config.metric;
    v.similarity_backend = config.similarity_backend;
    v.default_top_k = config.default_top_k;
    v.default_candidates = config.default_candidates;
    v.rescore_candidates = config.rescore_candidates;
    v.hybrid = config.hybrid;
    v.dense_weight = config.dense_weight;
    v.max_query_terms = config.max_query_terms;
    v.use_cuda_graphs = config.use_cuda_graphs;
    v.device_id = config.device_id;
    return v;
}

}  // namespace zcgvs
