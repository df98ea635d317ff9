// GGUF v2/v3 reader and Llama shape validation for the engine's loader.
//
// Follows the reference's parser semantics (core/include/tvara/gguf.hpp:45-207
// and gguf_model.hpp:43-107): the same bounds, count limits, alignment and
// overlap checks and the same error texts, so a file the reference rejects is
// rejected here with the message the Python side already expects.  The file
// is memory-mapped read-only; tensor payloads are views into the mapping.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <span>
#include <string>
#include <variant>
#include <vector>

namespace tvara::gguf {

class Error : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

struct Value {
    using Array = std::vector<Value>;
    std::variant<std::uint64_t, std::int64_t, double, bool, std::string, Array> data;
};

struct TensorInfo {
    std::string name;
    std::vector<std::uint64_t> dims;  // innermost first
    std::uint32_t type = 0;
    std::uint64_t offset = 0;
};

struct Document {
    std::uint32_t version = 0;
    std::map<std::string, Value> metadata;
    std::map<std::string, TensorInfo> tensors;
    std::size_t alignment = 32;
    std::size_t data_offset = 0;
};

// gguf.hpp:152-170: payload bytes of a tensor, rejecting unknown types and
// rows that are not a whole number of blocks.
std::size_t tensor_bytes(const TensorInfo& t);
Document parse(std::span<const std::byte> bytes);

class MappedFile {
public:
    explicit MappedFile(const std::string& path);
    ~MappedFile();
    MappedFile(const MappedFile&) = delete;
    MappedFile& operator=(const MappedFile&) = delete;
    std::span<const std::byte> bytes() const { return {data_, size_}; }

private:
    const std::byte* data_ = nullptr;
    std::size_t size_ = 0;
    int fd_ = -1;
};

class File {
public:
    explicit File(const std::string& path);
    const Document& doc() const { return doc_; }
    bool has(const std::string& name) const { return doc_.tensors.count(name) != 0; }
    const TensorInfo& info(const std::string& name) const;
    std::span<const std::byte> payload(const std::string& name) const;
    // JSON object of all metadata, serialised like c_api.cpp:19-41.
    std::string metadata_json() const;

private:
    std::shared_ptr<MappedFile> map_;
    Document doc_;
};

// gguf_model.hpp:68-107 + model.hpp:9-21,149-153.
struct LlamaConfig {
    std::size_t vocab = 0, hidden = 0, ffn = 0, layers = 0, heads = 0, kv_heads = 0, context = 0;
    float eps = 1e-6f, theta = 10000.f;
    bool interleaved = true;
    std::size_t head_dim() const { return hidden / heads; }
    std::size_t kv_width() const { return head_dim() * kv_heads; }
};
LlamaConfig llama_config(const Document& doc);
// gguf_model.hpp:43-66: every Llama tensor present with its expected dims.
void validate_llama_tensors(const Document& doc, const LlamaConfig& c);

}  // namespace tvara::gguf
