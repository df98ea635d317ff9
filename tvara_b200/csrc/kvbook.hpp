// Host-side accounting of the device KV pool: block handles with generation
// tags, reference counts, the LIFO free list, per-sequence block tables,
// copy-on-write of shared partial tails, and the radix prefix cache.
//
// The accounting is the reference's, step for step, so block ids,
// generations, reference counts and free-list order match it exactly for the
// same operation sequence:
//   CacheGeometry / kv_offset        core/include/tvara/kv.hpp:12-33
//   BlockPool                        kv.hpp:36-75
//   PagedCache                       kv.hpp:78-165
//   RadixCache                       core/include/tvara/radix.hpp:17-130
// What differs is where the payload lives: block contents are in HBM, owned
// by the engine.  Operations that touch payload (copy-on-write) are reported
// to the caller as device copies to enqueue; allocation does not clear the
// block on the device because no kernel reads a slot at or past a sequence's
// length (tests poison those slots with NaN).
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <map>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace tvara {

struct CacheGeometry {
    std::size_t layers = 1, kv_heads = 1, head_dim = 4, tokens_per_block = 16, max_blocks = 64;
    std::size_t kv_width() const {
        if (!kv_heads || !head_dim || kv_heads > std::numeric_limits<std::size_t>::max() / head_dim)
            throw std::invalid_argument("KV width overflow");
        return kv_heads * head_dim;
    }
    std::size_t elements_per_block() const {
        std::size_t n = kv_width();
        for (auto d : {layers, tokens_per_block, std::size_t(2)}) {
            if (!d || n > std::numeric_limits<std::size_t>::max() / d) throw std::invalid_argument("KV block overflow");
            n *= d;
        }
        return n;
    }
    void validate() const {
        const auto e = elements_per_block();
        if (!max_blocks || max_blocks > 1000000 || e > std::numeric_limits<std::size_t>::max() / sizeof(float) / max_blocks ||
            tokens_per_block > std::numeric_limits<std::size_t>::max() / max_blocks)
            throw std::invalid_argument("KV capacity overflow");
    }
};

class CacheExhausted : public std::runtime_error {
public:
    CacheExhausted() : std::runtime_error("KV cache exhausted") {}
};

struct BlockHandle {
    std::size_t id = 0;
    std::uint64_t generation = 0;
};
struct BlockTable {
    std::vector<BlockHandle> blocks;
    std::size_t length = 0;
};

// Device work implied by accounting operations, drained by the engine.
struct BlockCopy {
    std::size_t from = 0, to = 0;
};

class BlockPool {
public:
    explicit BlockPool(CacheGeometry g) : geometry_(g) {
        g.validate();
        refs_.assign(g.max_blocks, 0);
        gens_.assign(g.max_blocks, 0);
        free_.reserve(g.max_blocks);
        for (std::size_t i = g.max_blocks; i > 0; --i) free_.push_back(i - 1);
    }
    BlockHandle allocate() {
        if (free_.empty()) throw CacheExhausted();
        const auto id = free_.back();
        if (gens_[id] == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("KV generation exhausted");
        free_.pop_back();
        refs_[id] = 1;
        ++gens_[id];
        return {id, gens_[id]};
    }
    void retain(BlockHandle h) {
        check(h);
        if (refs_[h.id] == std::numeric_limits<std::size_t>::max()) throw std::runtime_error("KV reference overflow");
        ++refs_[h.id];
    }
    void release(BlockHandle h) {
        check(h);
        if (--refs_[h.id] == 0) free_.push_back(h.id);
    }
    std::size_t references(BlockHandle h) const {
        check(h);
        return refs_[h.id];
    }
    std::size_t references_by_id(std::size_t id) const { return refs_.at(id); }
    std::uint64_t generation_by_id(std::size_t id) const { return gens_.at(id); }
    std::size_t available() const { return free_.size(); }
    const CacheGeometry& geometry() const { return geometry_; }
    const std::vector<std::size_t>& free_list() const { return free_; }
    void check(BlockHandle h) const {
        if (h.id >= refs_.size() || !refs_[h.id] || gens_[h.id] != h.generation)
            throw std::invalid_argument("stale or invalid KV handle");
    }
    void audit() const {
        std::vector<bool> seen(refs_.size());
        for (auto id : free_) {
            if (id >= refs_.size() || seen[id] || refs_[id]) throw std::logic_error("KV free-list invariant");
            seen[id] = true;
        }
        for (std::size_t i = 0; i < refs_.size(); ++i)
            if (seen[i] != (refs_[i] == 0)) throw std::logic_error("KV allocation invariant");
    }

private:
    CacheGeometry geometry_;
    std::vector<std::size_t> refs_;
    std::vector<std::uint64_t> gens_;
    std::vector<std::size_t> free_;
};

class PagedBook {
public:
    explicit PagedBook(CacheGeometry g) : pool_(g) {}
    const CacheGeometry& geometry() const { return pool_.geometry(); }
    BlockPool& pool() { return pool_; }
    const BlockPool& pool() const { return pool_; }

    std::uint64_t create_sequence() {
        if (next_ == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("sequence ID exhausted");
        const auto id = ++next_;
        tables_.emplace(id, BlockTable{});
        return id;
    }
    const BlockTable& sequence(std::uint64_t id) const {
        auto it = tables_.find(id);
        if (it == tables_.end()) throw std::invalid_argument("unknown KV sequence");
        return it->second;
    }
    bool contains(std::uint64_t id) const { return tables_.count(id) != 0; }
    BlockHandle physical_block(std::uint64_t id, std::size_t position) const {
        const auto& t = sequence(id);
        if (position >= t.length) throw std::invalid_argument("KV position beyond sequence");
        return t.blocks.at(position / geometry().tokens_per_block);
    }

    // kv.hpp:91-108, accounting half: a fresh block at slot 0; a shared
    // partial tail is replaced by a private copy (reported in *copy).
    void append(std::uint64_t id, BlockCopy* copy = nullptr) {
        auto& t = mutable_sequence(id);
        const auto& g = geometry();
        if (t.length >= g.max_blocks * g.tokens_per_block) throw std::invalid_argument("invalid paged KV append dimensions");
        const auto slot = t.length % g.tokens_per_block;
        if (slot == 0) {
            auto b = pool_.allocate();
            try {
                t.blocks.push_back(b);
            } catch (...) {
                pool_.release(b);
                throw;
            }
        }
        if (slot != 0 && pool_.references(t.blocks.back()) > 1) {
            const auto original = t.blocks.back();
            const auto replacement = pool_.allocate();
            if (copy) *copy = {original.id, replacement.id};
            t.blocks.back() = replacement;
            pool_.release(original);
        }
        ++t.length;
    }
    void drop(std::uint64_t id) {
        auto& t = mutable_sequence(id);
        for (auto b : t.blocks) pool_.release(b);
        tables_.erase(id);
    }
    std::uint64_t fork(std::uint64_t id) {
        const auto copy = sequence(id);
        std::size_t retained = 0;
        try {
            for (auto b : copy.blocks) {
                pool_.retain(b);
                ++retained;
            }
            if (next_ == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("sequence ID exhausted");
            const auto r = ++next_;
            tables_.emplace(r, copy);
            return r;
        } catch (...) {
            for (std::size_t i = 0; i < retained; ++i) pool_.release(copy.blocks[i]);
            throw;
        }
    }
    void truncate(std::uint64_t id, std::size_t length) {
        auto& t = mutable_sequence(id);
        if (length > t.length) throw std::invalid_argument("cannot extend KV by truncating");
        const auto tpb = geometry().tokens_per_block;
        const auto keep = length / tpb + (length % tpb ? 1 : 0);
        for (std::size_t i = keep; i < t.blocks.size(); ++i) pool_.release(t.blocks[i]);
        t.blocks.resize(keep);
        t.length = length;
    }
    std::uint64_t import_sequence(const BlockTable& source, std::size_t length) {
        if (length > source.length) throw std::invalid_argument("prefix exceeds snapshot");
        const auto tpb = geometry().tokens_per_block;
        const auto count = length / tpb + (length % tpb ? 1 : 0);
        if (source.blocks.size() < count) throw std::invalid_argument("invalid prefix snapshot");
        BlockTable t;
        t.length = length;
        t.blocks.assign(source.blocks.begin(), source.blocks.begin() + static_cast<std::ptrdiff_t>(count));
        std::size_t retained = 0;
        try {
            for (auto h : t.blocks) {
                pool_.retain(h);
                ++retained;
            }
            if (next_ == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("sequence ID exhausted");
            const auto id = ++next_;
            tables_.emplace(id, std::move(t));
            return id;
        } catch (...) {
            for (std::size_t i = 0; i < retained; ++i) pool_.release(source.blocks[i]);
            throw;
        }
    }
    void audit(std::span<const std::size_t> external = {}) const {
        pool_.audit();
        std::vector<std::size_t> counts(geometry().max_blocks);
        if (!external.empty() && external.size() != counts.size())
            throw std::invalid_argument("external reference counts mismatch");
        const auto tpb = geometry().tokens_per_block;
        for (const auto& [id, t] : tables_) {
            const auto expected = t.length / tpb + (t.length % tpb ? 1 : 0);
            if (t.blocks.size() != expected) throw std::logic_error("KV block table length invariant");
            for (auto b : t.blocks) {
                pool_.check(b);
                ++counts.at(b.id);
            }
        }
        for (std::size_t i = 0; i < counts.size(); ++i)
            if (counts[i] + (external.empty() ? 0 : external[i]) != pool_.references_by_id(i))
                throw std::logic_error("KV reference invariant");
    }
    std::size_t sequences() const { return tables_.size(); }

private:
    BlockTable& mutable_sequence(std::uint64_t id) {
        auto it = tables_.find(id);
        if (it == tables_.end()) throw std::invalid_argument("unknown KV sequence");
        return it->second;
    }
    BlockPool pool_;
    std::map<std::uint64_t, BlockTable> tables_;
    std::uint64_t next_ = 0;
};

// Token-path trie over cached prefixes (radix.hpp:17-130): compressed edges,
// per-node snapshots of a sequence's block table holding one reference per
// block, pins along the path, LRU eviction of unpinned leaves.
struct RadixNode {
    std::uint64_t id = 0, parent = 0;
    std::vector<std::int32_t> edge;
    std::map<std::int32_t, std::uint64_t> children;
    std::optional<BlockTable> kv;
    std::size_t pins = 0;
    std::uint64_t accessed = 0;
};

class RadixBook {
public:
    RadixBook(PagedBook& cache, std::string isolation) : cache_(cache), isolation_(std::move(isolation)) {
        if (isolation_.empty()) throw std::invalid_argument("prefix isolation key is required");
        nodes_.emplace(0, RadixNode{});
    }
    RadixBook(const RadixBook&) = delete;
    RadixBook& operator=(const RadixBook&) = delete;
    ~RadixBook() {
        for (auto& [id, n] : nodes_)
            if (n.kv)
                for (auto b : n.kv->blocks) cache_.pool().release(b);
    }
    const RadixNode& node(std::uint64_t id) const { return nodes_.at(id); }
    std::size_t size() const { return nodes_.size() - 1; }

    std::pair<std::uint64_t, std::size_t> lookup(std::span<const std::int32_t> tokens) const {
        std::uint64_t cur = 0;
        std::size_t off = 0;
        std::pair<std::uint64_t, std::size_t> r{0, 0};
        while (off < tokens.size()) {
            const auto& parent = nodes_.at(cur);
            auto it = parent.children.find(tokens[off]);
            if (it == parent.children.end()) break;
            const auto& child = nodes_.at(it->second);
            std::size_t common = 0;
            while (common < child.edge.size() && off + common < tokens.size() && child.edge[common] == tokens[off + common])
                ++common;
            off += common;
            r = {child.id, off};
            if (common != child.edge.size()) break;
            cur = child.id;
        }
        return r;
    }

    std::uint64_t insert(std::span<const std::int32_t> tokens) {
        if (tokens.empty()) throw std::invalid_argument("cannot cache empty prefix");
        std::uint64_t cur = 0;
        std::size_t off = 0;
        while (off < tokens.size()) {
            auto& parent = nodes_.at(cur);
            auto found = parent.children.find(tokens[off]);
            if (found == parent.children.end()) {
                if (next_ == std::numeric_limits<std::uint64_t>::max()) throw std::overflow_error("radix ID exhausted");
                const auto id = ++next_;
                RadixNode child;
                child.id = id;
                child.parent = cur;
                child.edge.assign(tokens.begin() + static_cast<std::ptrdiff_t>(off), tokens.end());
                nodes_.emplace(id, std::move(child));
                nodes_.at(cur).children.emplace(tokens[off], id);
                return id;
            }
            auto& child = nodes_.at(found->second);
            std::size_t common = 0;
            while (common < child.edge.size() && off + common < tokens.size() && child.edge[common] == tokens[off + common])
                ++common;
            if (common != child.edge.size()) {
                if (next_ == std::numeric_limits<std::uint64_t>::max()) throw std::overflow_error("radix ID exhausted");
                const auto split = ++next_;
                RadixNode middle;
                middle.id = split;
                middle.parent = cur;
                middle.pins = child.pins;
                middle.edge.assign(child.edge.begin(), child.edge.begin() + static_cast<std::ptrdiff_t>(common));
                child.edge.erase(child.edge.begin(), child.edge.begin() + static_cast<std::ptrdiff_t>(common));
                middle.children.emplace(child.edge.front(), child.id);
                child.parent = split;
                nodes_.at(cur).children[tokens[off]] = split;
                nodes_.emplace(split, std::move(middle));
                cur = split;
                off += common;
                continue;
            }
            cur = child.id;
            off += common;
        }
        return cur;
    }

    void attach(std::uint64_t id, std::uint64_t sequence) {
        auto& entry = nodes_.at(id);
        auto source = cache_.sequence(sequence);
        std::size_t depth = 0;
        for (auto c = id; c; c = nodes_.at(c).parent) depth += nodes_.at(c).edge.size();
        if (source.length != depth) throw std::invalid_argument("token and KV prefix lengths differ");
        std::size_t retained = 0;
        try {
            for (auto b : source.blocks) {
                cache_.pool().retain(b);
                ++retained;
            }
        } catch (...) {
            for (std::size_t i = 0; i < retained; ++i) cache_.pool().release(source.blocks[i]);
            throw;
        }
        if (entry.kv)
            for (auto b : entry.kv->blocks) cache_.pool().release(b);
        entry.kv = std::move(source);
    }

    std::vector<std::size_t> external_references() const {
        std::vector<std::size_t> counts(cache_.geometry().max_blocks);
        for (const auto& [id, n] : nodes_)
            if (n.kv)
                for (auto b : n.kv->blocks) ++counts.at(b.id);
        return counts;
    }

    std::pair<std::uint64_t, std::size_t> reuse(std::span<const std::int32_t> tokens, bool partial = false) {
        auto m = lookup(tokens);
        if (!m.first || !nodes_.at(m.first).kv) return {cache_.create_sequence(), 0};
        std::size_t length = m.second;
        if (!partial) length -= length % cache_.geometry().tokens_per_block;
        return {cache_.import_sequence(*nodes_.at(m.first).kv, length), length};
    }

    void pin(std::uint64_t id) {
        for (auto c = id; c; c = nodes_.at(c).parent)
            if (nodes_.at(c).pins == std::numeric_limits<std::size_t>::max()) throw std::overflow_error("prefix pin overflow");
        for (auto c = id; c; c = nodes_.at(c).parent) ++nodes_.at(c).pins;
    }
    void unpin(std::uint64_t id) {
        for (auto c = id; c; c = nodes_.at(c).parent)
            if (!nodes_.at(c).pins) throw std::invalid_argument("prefix pin underflow");
        for (auto c = id; c; c = nodes_.at(c).parent) --nodes_.at(c).pins;
    }
    void touch(std::uint64_t id) {
        auto& e = nodes_.at(id);
        if (clock_ == std::numeric_limits<std::uint64_t>::max()) throw std::overflow_error("prefix access clock exhausted");
        e.accessed = ++clock_;
    }
    std::optional<std::uint64_t> eviction_candidate() const {
        std::optional<std::uint64_t> r;
        for (const auto& [id, e] : nodes_)
            if (id && e.children.empty() && !e.pins && (!r || e.accessed < nodes_.at(*r).accessed)) r = id;
        return r;
    }
    bool evict_one() {
        auto cand = eviction_candidate();
        if (!cand) return false;
        auto& e = nodes_.at(*cand);
        if (e.kv)
            for (auto b : e.kv->blocks) cache_.pool().release(b);
        nodes_.at(e.parent).children.erase(e.edge.front());
        nodes_.erase(*cand);
        return true;
    }
    void reset() {
        for (const auto& [id, e] : nodes_)
            if (id && e.pins) throw std::logic_error("cannot reset pinned prefix nodes");
        for (auto& [id, e] : nodes_)
            if (e.kv)
                for (auto b : e.kv->blocks) cache_.pool().release(b);
        nodes_.clear();
        nodes_.emplace(0, RadixNode{});
        clock_ = 0;
    }

private:
    PagedBook& cache_;
    std::string isolation_;
    std::map<std::uint64_t, RadixNode> nodes_;
    std::uint64_t next_ = 0, clock_ = 0;
};

}  // namespace tvara
