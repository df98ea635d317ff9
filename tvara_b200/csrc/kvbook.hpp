// Host-side bookkeeping of the device KV pool.
//
// Three pieces, each holding only integers (the K/V payload lives in HBM and
// is owned by the engine):
//
//   BlockLedger   per-block reference count and generation in two parallel
//                 arrays, with the free blocks threaded through a third array
//                 as an intrusive LIFO chain (no separate free-list vector).
//   SequenceBook  one block table per sequence in a hash map; appends,
//                 copy-on-write of a shared partial tail, forks, truncation,
//                 prefix imports and the consistency audit.
//   PrefixTrie    a compressed token trie whose nodes live in an arena
//                 (vector + vacant-slot stack) addressed through a map from
//                 public node id to slot; children are a sorted flat vector,
//                 edges are matched with std::mismatch.
//
// The observable results are fixed by the reference so that an engine and the
// reference given the same operations hand out the same block ids,
// generations, sequence ids and prefix-node ids and end with the same
// reference counts and free-block order:
//   geometry checks and texts           core/include/tvara/kv.hpp:12-29
//   pool (LIFO reuse, generations)      kv.hpp:36-75
//   paged cache (append/CoW/fork/...)   kv.hpp:78-165
//   prefix cache (ids, splits, LRU)     core/include/tvara/radix.hpp:17-130
// Those contracts are replayed operation by operation against the reference
// compiled from its own sources (tests/test_host.py).
//
// Block allocation does not clear the device block: no kernel reads a slot at
// or past a sequence's length.  Copy-on-write is reported to the caller as a
// (source, destination) block pair to copy on the device.
#pragma once
#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace tvara {

struct CacheGeometry {
    std::size_t layers = 1, kv_heads = 1, head_dim = 4, tokens_per_block = 16, max_blocks = 64;

    // Width of one token's K (or V) row in elements; overflow-checked.
    std::size_t kv_width() const {
        if (kv_heads == 0 || head_dim == 0) throw std::invalid_argument("KV width overflow");
        std::size_t w = 0;
        if (__builtin_mul_overflow(kv_heads, head_dim, &w)) throw std::invalid_argument("KV width overflow");
        return w;
    }
    // Elements of one block: layers x {K, V} x slots x width.
    std::size_t elements_per_block() const {
        std::size_t e = kv_width();
        const std::size_t factors[] = {layers, tokens_per_block, 2};
        for (std::size_t f : factors)
            if (f == 0 || __builtin_mul_overflow(e, f, &e)) throw std::invalid_argument("KV block overflow");
        return e;
    }
    void validate() const {
        const std::size_t e = elements_per_block();
        const std::size_t top = std::numeric_limits<std::size_t>::max();
        const bool bad = max_blocks == 0 || max_blocks > 1000000 || e > top / sizeof(float) / max_blocks ||
                         tokens_per_block > top / max_blocks;
        if (bad) throw std::invalid_argument("KV capacity overflow");
    }
    std::size_t blocks_for(std::size_t tokens) const { return (tokens + tokens_per_block - 1) / tokens_per_block; }
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
// A device block copy implied by copy-on-write, drained by the engine.
struct BlockCopy {
    std::size_t from = 0, to = 0;
};

class BlockLedger {
    static constexpr std::size_t kEnd = std::numeric_limits<std::size_t>::max();

public:
    explicit BlockLedger(CacheGeometry g) : geometry_(g) {
        g.validate();
        const std::size_t n = g.max_blocks;
        refs_.assign(n, 0);
        generation_.assign(n, 0);
        chain_.resize(n);
        // Initially every block is free and block 0 is handed out first.
        for (std::size_t i = 0; i < n; ++i) chain_[i] = i + 1 < n ? i + 1 : kEnd;
        head_ = 0;
        free_count_ = n;
    }

    BlockHandle take() {
        if (head_ == kEnd) throw CacheExhausted();
        const std::size_t id = head_;
        if (generation_[id] == std::numeric_limits<std::uint64_t>::max())
            throw std::runtime_error("KV generation exhausted");
        head_ = chain_[id];
        chain_[id] = kEnd;
        --free_count_;
        refs_[id] = 1;
        return {id, ++generation_[id]};
    }
    void share(BlockHandle h) {
        std::uint64_t& r = refs_[checked(h)];
        if (r == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("KV reference overflow");
        ++r;
    }
    void unshare(BlockHandle h) {
        const std::size_t id = checked(h);
        if (--refs_[id] == 0) {
            chain_[id] = head_;
            head_ = id;
            ++free_count_;
        }
    }
    bool shared(BlockHandle h) const { return refs_[checked(h)] > 1; }
    std::size_t references(BlockHandle h) const { return refs_[checked(h)]; }
    std::size_t references_by_id(std::size_t id) const {
        if (id >= refs_.size()) throw std::out_of_range("KV block id out of range");
        return refs_[id];
    }
    std::size_t available() const { return free_count_; }
    const CacheGeometry& geometry() const { return geometry_; }
    std::size_t checked(BlockHandle h) const {
        if (h.id >= refs_.size() || refs_[h.id] == 0 || generation_[h.id] != h.generation)
            throw std::invalid_argument("stale or invalid KV handle");
        return h.id;
    }
    // Free chain well-formed (in range, acyclic, only unreferenced blocks),
    // and every unreferenced block on it.
    void audit() const {
        std::vector<char> on_chain(refs_.size(), 0);
        std::size_t walked = 0;
        for (std::size_t id = head_; id != kEnd; id = chain_[id]) {
            if (id >= refs_.size() || on_chain[id] || refs_[id] != 0) throw std::logic_error("KV free-list invariant");
            on_chain[id] = 1;
            ++walked;
        }
        if (walked != free_count_) throw std::logic_error("KV free-list invariant");
        for (std::size_t i = 0; i < refs_.size(); ++i)
            if (bool(on_chain[i]) != (refs_[i] == 0)) throw std::logic_error("KV allocation invariant");
    }

private:
    CacheGeometry geometry_;
    std::vector<std::uint64_t> refs_, generation_;
    std::vector<std::size_t> chain_;  // next free block after this one
    std::size_t head_ = kEnd, free_count_ = 0;
};

class SequenceBook {
public:
    explicit SequenceBook(CacheGeometry g) : ledger_(g) {}
    const CacheGeometry& geometry() const { return ledger_.geometry(); }
    BlockLedger& ledger() { return ledger_; }
    const BlockLedger& ledger() const { return ledger_; }

    std::uint64_t create_sequence() { return add(BlockTable{}); }
    const BlockTable& sequence(std::uint64_t id) const {
        const auto it = tables_.find(id);
        if (it == tables_.end()) throw std::invalid_argument("unknown KV sequence");
        return it->second;
    }
    bool contains(std::uint64_t id) const { return tables_.find(id) != tables_.end(); }
    std::size_t sequences() const { return tables_.size(); }

    // One more position.  A position opening a block takes a fresh block; a
    // position landing in a partial tail that another table also holds moves
    // the tail to a private block first (the pair is reported in *copy).
    void append(std::uint64_t id, BlockCopy* copy = nullptr) {
        BlockTable& t = table(id);
        const CacheGeometry& g = geometry();
        if (t.length >= g.max_blocks * g.tokens_per_block) throw std::invalid_argument("invalid paged KV append dimensions");
        if (t.length % g.tokens_per_block == 0) {
            t.blocks.reserve(t.blocks.size() + 1);  // so the push below cannot throw after take()
            t.blocks.push_back(ledger_.take());
        } else if (ledger_.shared(t.blocks.back())) {
            const BlockHandle mine = ledger_.take();
            const BlockHandle theirs = std::exchange(t.blocks.back(), mine);
            if (copy) *copy = {theirs.id, mine.id};
            ledger_.unshare(theirs);
        }
        ++t.length;
    }
    void drop(std::uint64_t id) {
        const auto it = tables_.find(id);
        if (it == tables_.end()) throw std::invalid_argument("unknown KV sequence");
        for (const BlockHandle& b : it->second.blocks) ledger_.unshare(b);
        tables_.erase(it);
    }
    std::uint64_t fork(std::uint64_t id) {
        const BlockTable& src = sequence(id);
        return add_sharing(src, src.length);
    }
    void truncate(std::uint64_t id, std::size_t length) {
        BlockTable& t = table(id);
        if (length > t.length) throw std::invalid_argument("cannot extend KV by truncating");
        const std::size_t keep = geometry().blocks_for(length);
        for (std::size_t i = keep; i < t.blocks.size(); ++i) ledger_.unshare(t.blocks[i]);
        t.blocks.erase(t.blocks.begin() + std::ptrdiff_t(keep), t.blocks.end());
        t.length = length;
    }
    // A new sequence holding the first `length` positions of `snapshot`.
    std::uint64_t import_sequence(const BlockTable& snapshot, std::size_t length) {
        if (length > snapshot.length) throw std::invalid_argument("prefix exceeds snapshot");
        if (snapshot.blocks.size() < geometry().blocks_for(length)) throw std::invalid_argument("invalid prefix snapshot");
        return add_sharing(snapshot, length);
    }
    // Ledger consistent, every table's block count matches its length, and
    // each block's reference count equals the tables holding it plus
    // `external` (references held elsewhere, e.g. by the prefix trie).
    void audit(std::span<const std::size_t> external = {}) const {
        ledger_.audit();
        const std::size_t n = geometry().max_blocks;
        if (!external.empty() && external.size() != n) throw std::invalid_argument("external reference counts mismatch");
        std::vector<std::size_t> held(n, 0);
        if (!external.empty()) std::copy(external.begin(), external.end(), held.begin());
        for (const auto& entry : tables_) {
            const BlockTable& t = entry.second;
            if (t.blocks.size() != geometry().blocks_for(t.length)) throw std::logic_error("KV block table length invariant");
            for (const BlockHandle& b : t.blocks) ++held[ledger_.checked(b)];
        }
        for (std::size_t i = 0; i < n; ++i)
            if (held[i] != ledger_.references_by_id(i)) throw std::logic_error("KV reference invariant");
    }

private:
    BlockTable& table(std::uint64_t id) {
        const auto it = tables_.find(id);
        if (it == tables_.end()) throw std::invalid_argument("unknown KV sequence");
        return it->second;
    }
    std::uint64_t next_id() {
        if (last_id_ == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("sequence ID exhausted");
        return ++last_id_;
    }
    std::uint64_t add(BlockTable t) {
        const std::uint64_t id = next_id();
        tables_.emplace(id, std::move(t));
        return id;
    }
    // New table over the leading blocks of `src` covering `length` positions,
    // each block's count raised; on any failure the counts already raised are
    // lowered again and nothing else changes.
    std::uint64_t add_sharing(const BlockTable& src, std::size_t length) {
        BlockTable t;
        t.length = length;
        t.blocks.assign(src.blocks.begin(), src.blocks.begin() + std::ptrdiff_t(geometry().blocks_for(length)));
        if (last_id_ == std::numeric_limits<std::uint64_t>::max()) throw std::runtime_error("sequence ID exhausted");
        std::size_t raised = 0;
        try {
            for (; raised < t.blocks.size(); ++raised) ledger_.share(t.blocks[raised]);
            return add(std::move(t));
        } catch (...) {
            while (raised) ledger_.unshare(src.blocks[--raised]);
            throw;
        }
    }

    BlockLedger ledger_;
    std::unordered_map<std::uint64_t, BlockTable> tables_;
    std::uint64_t last_id_ = 0;
};

class PrefixTrie {
    static constexpr std::uint32_t kNone = std::numeric_limits<std::uint32_t>::max();
    struct Node {
        std::uint64_t id = 0;
        std::uint32_t up = kNone;  // parent slot
        std::vector<std::int32_t> edge;
        std::vector<std::pair<std::int32_t, std::uint32_t>> kids;  // (first edge token, slot), sorted
        std::optional<BlockTable> snapshot;
        std::size_t pins = 0;
        std::uint64_t stamp = 0;
    };

public:
    PrefixTrie(SequenceBook& book, std::string isolation) : book_(book), isolation_(std::move(isolation)) {
        if (isolation_.empty()) throw std::invalid_argument("prefix isolation key is required");
        clear_arena();
    }
    PrefixTrie(const PrefixTrie&) = delete;
    PrefixTrie& operator=(const PrefixTrie&) = delete;
    ~PrefixTrie() {
        for (std::uint32_t s : slots_by_id()) release_snapshot(arena_[s]);
    }
    std::size_t size() const { return slot_of_.size() - 1; }

    // Deepest node reached by `tokens` and how many tokens matched; the last
    // node may be matched only part way along its edge.
    std::pair<std::uint64_t, std::size_t> lookup(std::span<const std::int32_t> tokens) const {
        std::pair<std::uint64_t, std::size_t> hit{0, 0};
        std::uint32_t at = 0;
        std::size_t done = 0;
        while (done < tokens.size()) {
            const std::uint32_t kid = child(at, tokens[done]);
            if (kid == kNone) break;
            const std::size_t same = matched(arena_[kid].edge, tokens.subspan(done));
            done += same;
            hit = {arena_[kid].id, done};
            if (same < arena_[kid].edge.size()) break;
            at = kid;
        }
        return hit;
    }

    // Node for exactly `tokens`, creating a leaf and splitting an edge where
    // the path leaves the trie part way along one.
    std::uint64_t insert(std::span<const std::int32_t> tokens) {
        if (tokens.empty()) throw std::invalid_argument("cannot cache empty prefix");
        std::uint32_t at = 0;
        std::size_t done = 0;
        while (done < tokens.size()) {
            const std::uint32_t kid = child(at, tokens[done]);
            if (kid == kNone) {
                const std::uint32_t leaf = make_node(at, {tokens.begin() + std::ptrdiff_t(done), tokens.end()});
                link(at, leaf);
                return arena_[leaf].id;
            }
            const std::size_t same = matched(arena_[kid].edge, tokens.subspan(done));
            if (same < arena_[kid].edge.size()) {
                std::vector<std::int32_t>& tail = arena_[kid].edge;
                const std::uint32_t mid = make_node(at, {tail.begin(), tail.begin() + std::ptrdiff_t(same)});
                Node& m = arena_[mid];
                Node& k = arena_[kid];  // arena_ may have grown: take references afresh
                m.pins = k.pins;
                k.edge.erase(k.edge.begin(), k.edge.begin() + std::ptrdiff_t(same));
                k.up = mid;
                m.kids.push_back({k.edge.front(), kid});
                replace_child(at, tokens[done], mid);
                at = mid;
            } else {
                at = kid;
            }
            done += same;
        }
        return arena_[at].id;
    }

    // Node `id` keeps its own reference to every block of `sequence`, whose
    // length must equal the node's depth in tokens; a previous snapshot is
    // released.
    void attach(std::uint64_t id, std::uint64_t sequence) {
        const std::uint32_t s = slot(id);
        BlockTable copy = book_.sequence(sequence);
        std::size_t depth = 0;
        for (std::uint32_t c = s; c != 0; c = arena_[c].up) depth += arena_[c].edge.size();
        if (copy.length != depth) throw std::invalid_argument("token and KV prefix lengths differ");
        std::size_t raised = 0;
        try {
            for (; raised < copy.blocks.size(); ++raised) book_.ledger().share(copy.blocks[raised]);
        } catch (...) {
            while (raised) book_.ledger().unshare(copy.blocks[--raised]);
            throw;
        }
        release_snapshot(arena_[s]);
        arena_[s].snapshot = std::move(copy);
    }

    std::vector<std::size_t> external_references() const {
        std::vector<std::size_t> held(book_.geometry().max_blocks, 0);
        for (const auto& [id, s] : slot_of_)
            if (arena_[s].snapshot)
                for (const BlockHandle& b : arena_[s].snapshot->blocks) ++held.at(b.id);
        return held;
    }

    // A new sequence sharing the longest cached prefix of `tokens` (whole
    // blocks only unless `partial`), or an empty one; returns (sequence,
    // positions shared).
    std::pair<std::uint64_t, std::size_t> reuse(std::span<const std::int32_t> tokens, bool partial = false) {
        const auto [node, count] = lookup(tokens);
        if (node == 0) return {book_.create_sequence(), 0};
        const Node& n = arena_[slot(node)];
        if (!n.snapshot) return {book_.create_sequence(), 0};
        const std::size_t tpb = book_.geometry().tokens_per_block;
        const std::size_t length = partial ? count : count / tpb * tpb;
        return {book_.import_sequence(*n.snapshot, length), length};
    }

    void pin(std::uint64_t id) {
        const std::uint32_t s = slot(id);
        for (std::uint32_t c = s; c != 0; c = arena_[c].up)
            if (arena_[c].pins == std::numeric_limits<std::size_t>::max()) throw std::overflow_error("prefix pin overflow");
        for (std::uint32_t c = s; c != 0; c = arena_[c].up) ++arena_[c].pins;
    }
    void unpin(std::uint64_t id) {
        const std::uint32_t s = slot(id);
        for (std::uint32_t c = s; c != 0; c = arena_[c].up)
            if (arena_[c].pins == 0) throw std::invalid_argument("prefix pin underflow");
        for (std::uint32_t c = s; c != 0; c = arena_[c].up) --arena_[c].pins;
    }
    void touch(std::uint64_t id) {
        Node& n = arena_[slot(id)];
        if (clock_ == std::numeric_limits<std::uint64_t>::max()) throw std::overflow_error("prefix access clock exhausted");
        n.stamp = ++clock_;
    }
    // Least recently touched unpinned leaf; ties go to the lowest node id.
    std::optional<std::uint64_t> eviction_candidate() const {
        std::optional<std::pair<std::uint64_t, std::uint64_t>> best;  // (stamp, id)
        for (const auto& [id, s] : slot_of_) {
            const Node& n = arena_[s];
            if (id == 0 || !n.kids.empty() || n.pins) continue;
            const std::pair<std::uint64_t, std::uint64_t> key{n.stamp, id};
            if (!best || key < *best) best = key;
        }
        if (!best) return std::nullopt;
        return best->second;
    }
    bool evict_one() {
        const auto victim = eviction_candidate();
        if (!victim) return false;
        const std::uint32_t s = slot(*victim);
        release_snapshot(arena_[s]);
        unlink(arena_[s].up, arena_[s].edge.front());
        free_node(s);
        return true;
    }
    // Drops every node (ids keep counting up); refused while any is pinned.
    void reset() {
        for (const auto& [id, s] : slot_of_)
            if (id != 0 && arena_[s].pins) throw std::logic_error("cannot reset pinned prefix nodes");
        for (std::uint32_t s : slots_by_id()) release_snapshot(arena_[s]);
        clear_arena();
        clock_ = 0;
    }

private:
    static std::size_t matched(const std::vector<std::int32_t>& edge, std::span<const std::int32_t> rest) {
        const std::size_t n = std::min(edge.size(), rest.size());
        return std::size_t(std::mismatch(edge.begin(), edge.begin() + std::ptrdiff_t(n), rest.begin()).first - edge.begin());
    }
    std::uint32_t slot(std::uint64_t id) const {
        const auto it = slot_of_.find(id);
        if (it == slot_of_.end()) throw std::invalid_argument("unknown prefix node");
        return it->second;
    }
    std::uint32_t child(std::uint32_t at, std::int32_t token) const {
        const auto& k = arena_[at].kids;
        const auto it = std::lower_bound(k.begin(), k.end(), token, [](const auto& e, std::int32_t t) { return e.first < t; });
        return it != k.end() && it->first == token ? it->second : kNone;
    }
    void link(std::uint32_t at, std::uint32_t kid) {
        auto& k = arena_[at].kids;
        const std::int32_t token = arena_[kid].edge.front();
        const auto it = std::lower_bound(k.begin(), k.end(), token, [](const auto& e, std::int32_t t) { return e.first < t; });
        k.insert(it, {token, kid});
    }
    void replace_child(std::uint32_t at, std::int32_t token, std::uint32_t kid) {
        for (auto& e : arena_[at].kids)
            if (e.first == token) e.second = kid;
    }
    void unlink(std::uint32_t at, std::int32_t token) {
        auto& k = arena_[at].kids;
        k.erase(std::remove_if(k.begin(), k.end(), [&](const auto& e) { return e.first == token; }), k.end());
    }
    std::uint32_t make_node(std::uint32_t up, std::vector<std::int32_t> edge) {
        if (last_id_ == std::numeric_limits<std::uint64_t>::max()) throw std::overflow_error("radix ID exhausted");
        std::uint32_t s;
        if (!vacant_.empty()) {
            s = vacant_.back();
            vacant_.pop_back();
            arena_[s] = Node{};
        } else {
            s = std::uint32_t(arena_.size());
            arena_.emplace_back();
        }
        Node& n = arena_[s];
        n.id = ++last_id_;
        n.up = up;
        n.edge = std::move(edge);
        slot_of_.emplace(n.id, s);
        return s;
    }
    void free_node(std::uint32_t s) {
        slot_of_.erase(arena_[s].id);
        arena_[s] = Node{};
        vacant_.push_back(s);
    }
    void release_snapshot(Node& n) {
        if (!n.snapshot) return;
        for (const BlockHandle& b : n.snapshot->blocks) book_.ledger().unshare(b);
        n.snapshot.reset();
    }
    // Live slots in ascending node id, the order releases reach the free chain.
    std::vector<std::uint32_t> slots_by_id() const {
        std::vector<std::pair<std::uint64_t, std::uint32_t>> v(slot_of_.begin(), slot_of_.end());
        std::sort(v.begin(), v.end());
        std::vector<std::uint32_t> out;
        out.reserve(v.size());
        for (const auto& e : v) out.push_back(e.second);
        return out;
    }
    void clear_arena() {
        arena_.assign(1, Node{});
        vacant_.clear();
        slot_of_.clear();
        slot_of_.emplace(0, 0);
    }

    SequenceBook& book_;
    std::string isolation_;
    std::vector<Node> arena_;
    std::vector<std::uint32_t> vacant_;
    std::unordered_map<std::uint64_t, std::uint32_t> slot_of_;
    std::uint64_t last_id_ = 0, clock_ = 0;
};

}  // namespace tvara
