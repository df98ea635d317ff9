// GGUF reader for the engine's loader; semantics follow the reference parser
// (core/include/tvara/gguf.hpp:45-207, gguf_model.hpp:43-107, mapped_file.hpp).
#include "gguf.hpp"

#include <cmath>
#include <cstring>
#include <fcntl.h>
#include <iomanip>
#include <limits>
#include <sstream>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace tvara::gguf {
namespace {

class Cursor {
public:
    explicit Cursor(std::span<const std::byte> b) : b_(b) {}
    std::size_t pos() const { return pos_; }
    std::size_t left() const { return b_.size() - pos_; }
    std::span<const std::byte> take(std::size_t n) {
        if (n > left()) throw Error("truncated GGUF data");
        auto s = b_.subspan(pos_, n);
        pos_ += n;
        return s;
    }
    std::uint64_t le(std::size_t width) {
        auto s = take(width);
        std::uint64_t v = 0;
        for (std::size_t i = 0; i < width; ++i) v |= std::uint64_t(std::to_integer<unsigned char>(s[i])) << (8 * i);
        return v;
    }
    float f32() {
        const auto bits = static_cast<std::uint32_t>(le(4));
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }
    double f64() {
        const auto bits = le(8);
        double d;
        std::memcpy(&d, &bits, 8);
        return d;
    }

private:
    std::span<const std::byte> b_;
    std::size_t pos_ = 0;
};

std::string read_string(Cursor& c) {
    const auto n = c.le(8);
    if (n > 16u * 1024 * 1024 || n > c.left()) throw Error("GGUF string length exceeds limits");
    auto s = c.take(static_cast<std::size_t>(n));
    return {reinterpret_cast<const char*>(s.data()), s.size()};
}

Value read_value(Cursor& c, std::uint32_t type) {
    switch (type) {
        case 0: return {c.le(1)};
        case 1: return {std::int64_t(static_cast<std::int8_t>(c.le(1)))};
        case 2: return {c.le(2)};
        case 3: return {std::int64_t(static_cast<std::int16_t>(c.le(2)))};
        case 4: return {c.le(4)};
        case 5: return {std::int64_t(static_cast<std::int32_t>(c.le(4)))};
        case 6: return {double(c.f32())};
        case 7: {
            const auto b = c.le(1);
            if (b > 1) throw Error("invalid boolean metadata");
            return {b != 0};
        }
        case 8: return {read_string(c)};
        case 9: {
            const auto inner = static_cast<std::uint32_t>(c.le(4));
            const auto count = c.le(8);
            if (inner == 9 || inner > 12 || count > 1000000 || count > c.left())
                throw Error("invalid or oversized metadata array");
            Value::Array a;
            a.reserve(static_cast<std::size_t>(count));
            for (std::uint64_t i = 0; i < count; ++i) a.push_back(read_value(c, inner));
            return {std::move(a)};
        }
        case 10: return {c.le(8)};
        case 11: return {static_cast<std::int64_t>(c.le(8))};
        case 12: return {c.f64()};
        default: throw Error("unsupported scalar metadata type");
    }
}

std::size_t align_up(std::size_t p, std::size_t a) {
    if (a == 0 || a > 65536 || (a & (a - 1))) throw Error("GGUF alignment must be a bounded power of two");
    if (p > std::numeric_limits<std::size_t>::max() - (a - 1)) throw Error("GGUF alignment overflow");
    return (p + a - 1) & ~(a - 1);
}

std::string quoted(const std::string& text) {
    std::ostringstream out;
    out << '"';
    for (unsigned char ch : text) {
        if (ch == '"' || ch == '\\') out << '\\' << static_cast<char>(ch);
        else if (ch < 32) out << "\\u" << std::hex << std::setw(4) << std::setfill('0') << unsigned(ch) << std::dec;
        else out << static_cast<char>(ch);
    }
    out << '"';
    return out.str();
}

std::string json(const Value& v) {
    return std::visit(
        [](const auto& x) -> std::string {
            using T = std::decay_t<decltype(x)>;
            if constexpr (std::is_same_v<T, std::string>) return quoted(x);
            else if constexpr (std::is_same_v<T, bool>) return x ? "true" : "false";
            else if constexpr (std::is_integral_v<T>) return std::to_string(x);
            else if constexpr (std::is_floating_point_v<T>) {
                if (!std::isfinite(x)) throw std::runtime_error("nonfinite metadata");
                std::ostringstream out;
                out << std::setprecision(17) << x;
                return out.str();
            } else {
                std::string out = "[";
                bool first = true;
                for (const auto& e : x) {
                    if (!first) out += ",";
                    first = false;
                    out += json(e);
                }
                return out + "]";
            }
        },
        v.data);
}

}  // namespace

std::size_t tensor_bytes(const TensorInfo& t) {
    std::size_t block = 1, width = 0;
    switch (t.type) {
        case 0: width = 4; break;
        case 1: width = 2; break;
        case 2: block = 32; width = 18; break;
        case 8: block = 32; width = 34; break;
        case 12: block = 256; width = 144; break;
        default: throw Error("unsupported GGUF tensor storage type");
    }
    if (t.dims.empty() || t.dims[0] % block) throw Error("invalid quantized row width");
    std::size_t n = 1;
    for (auto d : t.dims) {
        if (!d || d > std::numeric_limits<std::size_t>::max() / n) throw Error("tensor shape overflow");
        n *= static_cast<std::size_t>(d);
    }
    if (n / block > std::numeric_limits<std::size_t>::max() / width) throw Error("tensor size overflow");
    return n / block * width;
}

Document parse(std::span<const std::byte> bytes) {
    Cursor c(bytes);
    Document doc;
    if (c.le(4) != 0x46554747) throw Error("invalid GGUF magic or unsupported byte order");
    doc.version = static_cast<std::uint32_t>(c.le(4));
    if (doc.version != 2 && doc.version != 3) throw Error("unsupported GGUF version");
    const auto n_tensors = c.le(8), n_meta = c.le(8);
    if (n_tensors > 1000000 || n_meta > 1000000) throw Error("GGUF count limit exceeded");
    if (n_tensors > c.left() / 24 || n_meta > c.left() / 13) throw Error("GGUF counts exceed available bytes");
    for (std::uint64_t i = 0; i < n_meta; ++i) {
        auto key = read_string(c);
        auto val = read_value(c, static_cast<std::uint32_t>(c.le(4)));
        if (key.empty() || !doc.metadata.emplace(std::move(key), std::move(val)).second)
            throw Error("empty or duplicate GGUF metadata key");
    }
    for (std::uint64_t i = 0; i < n_tensors; ++i) {
        TensorInfo t;
        t.name = read_string(c);
        const auto rank = c.le(4);
        if (t.name.empty() || rank == 0 || rank > 4) throw Error("invalid GGUF tensor name or rank");
        for (std::uint64_t r = 0; r < rank; ++r) {
            const auto d = c.le(8);
            if (!d) throw Error("zero GGUF tensor dimension");
            t.dims.push_back(d);
        }
        t.type = static_cast<std::uint32_t>(c.le(4));
        t.offset = c.le(8);
        auto name = t.name;
        if (!doc.tensors.emplace(std::move(name), std::move(t)).second) throw Error("duplicate GGUF tensor name");
    }
    if (auto it = doc.metadata.find("general.alignment"); it != doc.metadata.end()) {
        auto v = std::get_if<std::uint64_t>(&it->second.data);
        if (!v || *v > 65536) throw Error("invalid general.alignment metadata");
        doc.alignment = static_cast<std::size_t>(*v);
    }
    doc.data_offset = align_up(c.pos(), doc.alignment);
    if (doc.data_offset > bytes.size()) throw Error("truncated GGUF alignment padding");
    for (const auto& [name, t] : doc.tensors)
        if (t.offset % doc.alignment) throw Error("unaligned GGUF tensor offset");
    std::map<std::uint64_t, std::uint64_t> regions;
    for (const auto& [name, t] : doc.tensors) {
        const auto n = tensor_bytes(t);
        if (t.offset > bytes.size() - doc.data_offset || n > bytes.size() - doc.data_offset - t.offset)
            throw Error("tensor payload exceeds GGUF file");
        const auto end = t.offset + n;
        auto next = regions.lower_bound(t.offset);
        if ((next != regions.end() && next->first < end) ||
            (next != regions.begin() && std::prev(next)->second > t.offset))
            throw Error("overlapping GGUF tensor payloads");
        regions.emplace(t.offset, end);
    }
    return doc;
}

MappedFile::MappedFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw Error("cannot open model file");
    struct stat st {};
    if (fstat(fd_, &st) != 0 || st.st_size <= 0) {
        ::close(fd_);
        throw Error("invalid model file size");
    }
    size_ = static_cast<std::size_t>(st.st_size);
    void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (p == MAP_FAILED) {
        ::close(fd_);
        throw Error("cannot map model file");
    }
    data_ = static_cast<const std::byte*>(p);
}

MappedFile::~MappedFile() {
    if (data_) munmap(const_cast<std::byte*>(data_), size_);
    if (fd_ >= 0) ::close(fd_);
}

File::File(const std::string& path) : map_(std::make_shared<MappedFile>(path)), doc_(parse(map_->bytes())) {}

const TensorInfo& File::info(const std::string& name) const {
    auto it = doc_.tensors.find(name);
    if (it == doc_.tensors.end()) throw Error("missing GGUF tensor: " + name);
    return it->second;
}

std::span<const std::byte> File::payload(const std::string& name) const {
    const auto& t = info(name);
    return map_->bytes().subspan(doc_.data_offset + static_cast<std::size_t>(t.offset), tensor_bytes(t));
}

std::string File::metadata_json() const {
    std::string out = "{";
    bool first = true;
    for (const auto& [k, v] : doc_.metadata) {
        if (!first) out += ",";
        first = false;
        out += quoted(k) + ":" + json(v);
    }
    return out + "}";
}

LlamaConfig llama_config(const Document& doc) {
    auto text = [&](const std::string& key) -> const std::string& {
        auto it = doc.metadata.find(key);
        if (it == doc.metadata.end()) throw Error("missing metadata: " + key);
        auto v = std::get_if<std::string>(&it->second.data);
        if (!v) throw Error("metadata must be a string: " + key);
        return *v;
    };
    auto number = [&](const std::string& key) -> std::uint64_t {
        auto it = doc.metadata.find(key);
        if (it == doc.metadata.end()) throw Error("missing metadata: " + key);
        auto v = std::get_if<std::uint64_t>(&it->second.data);
        if (!v || !*v || *v > 1000000) throw Error("invalid model dimension: " + key);
        return *v;
    };
    auto real = [&](const std::string& key, double fallback) {
        auto it = doc.metadata.find(key);
        if (it == doc.metadata.end()) return fallback;
        auto v = std::get_if<double>(&it->second.data);
        if (!v || !std::isfinite(*v) || *v <= 0) throw Error("invalid floating metadata: " + key);
        return *v;
    };
    if (text("general.architecture") != "llama") throw Error("unsupported model architecture");
    auto vit = doc.metadata.find("tokenizer.ggml.tokens");
    if (vit == doc.metadata.end()) throw Error("missing tokenizer vocabulary");
    auto vocab = std::get_if<Value::Array>(&vit->second.data);
    if (!vocab || vocab->empty()) throw Error("invalid tokenizer vocabulary");
    LlamaConfig c;
    c.vocab = vocab->size();
    c.hidden = number("llama.embedding_length");
    c.ffn = number("llama.feed_forward_length");
    c.layers = number("llama.block_count");
    c.heads = number("llama.attention.head_count");
    c.kv_heads = number("llama.attention.head_count_kv");
    c.context = number("llama.context_length");
    const double eps = real("llama.attention.layer_norm_rms_epsilon", 1e-6);
    const double theta = real("llama.rope.freq_base", 10000);
    if (c.hidden % c.heads || c.heads % c.kv_heads || (c.hidden / c.heads) % 2)
        throw Error("invalid Llama head layout");
    if (auto it = doc.metadata.find("llama.rope.scaling.type"); it != doc.metadata.end()) {
        auto v = std::get_if<std::string>(&it->second.data);
        if (!v || *v != "none") throw Error("scaled RoPE requires a separate implementation");
    }
    c.eps = static_cast<float>(eps);
    c.theta = static_cast<float>(theta);
    if (auto it = doc.metadata.find("tvara.rope.layout"); it != doc.metadata.end()) {
        auto v = std::get_if<std::string>(&it->second.data);
        if (!v || (*v != "split" && *v != "interleaved")) throw std::invalid_argument("invalid RoPE layout");
        c.interleaved = *v == "interleaved";
    }
    if (!std::isfinite(c.eps) || c.eps <= 0 || !std::isfinite(c.theta) || c.theta <= 0)
        throw std::invalid_argument("invalid native model configuration");
    return c;
}

void validate_llama_tensors(const Document& doc, const LlamaConfig& c) {
    const std::uint64_t kv = c.hidden / c.heads * c.kv_heads;
    auto require = [&](const std::string& name, std::vector<std::uint64_t> dims) {
        auto it = doc.tensors.find(name);
        if (it == doc.tensors.end() || it->second.dims != dims) throw Error("missing or malformed Llama tensor: " + name);
    };
    require("token_embd.weight", {c.hidden, c.vocab});
    require("output_norm.weight", {c.hidden});
    if (doc.tensors.count("output.weight")) require("output.weight", {c.hidden, c.vocab});
    for (std::size_t i = 0; i < c.layers; ++i) {
        const auto p = "blk." + std::to_string(i) + ".";
        require(p + "attn_norm.weight", {c.hidden});
        require(p + "ffn_norm.weight", {c.hidden});
        require(p + "attn_q.weight", {c.hidden, c.hidden});
        require(p + "attn_k.weight", {c.hidden, kv});
        require(p + "attn_v.weight", {c.hidden, kv});
        require(p + "attn_output.weight", {c.hidden, c.hidden});
        require(p + "ffn_gate.weight", {c.hidden, c.ffn});
        require(p + "ffn_up.weight", {c.hidden, c.ffn});
        require(p + "ffn_down.weight", {c.ffn, c.hidden});
    }
}

}  // namespace tvara::gguf
